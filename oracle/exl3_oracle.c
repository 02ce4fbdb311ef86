/*
 * TEST INFRASTRUCTURE ONLY -- the CPU checker for the B200 kernels, never the product path.
 *
 * Plain-C restatement of the reference's routed-expert MoE FFN over EXL3 mul1 K=3 weights.
 * Each function cites the reference lines it restates (paths inside the reference project).
 * Parity of this restatement is pinned against the reference's own ft_core.h, compiled
 * unchanged into oracle/_ref/ by oracle/Makefile (see tests/test_oracle_golden.py).
 */
#include "exl3_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------------------------------
 * half <-> float, IEEE binary16, round to nearest even (the reference uses F16C:
 * kernels/cpu_avx2/ft_core.h:34-36)
 * ------------------------------------------------------------------------------------- */
float orc_h2f(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        const float v = ldexpf((float)m, -24);
        return sign ? -v : v;
    }
    if (e == 31) bits = sign | 0x7f800000u | (m << 13);
    else bits = sign | ((e + 112u) << 23) | (m << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f2h(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) return sign | (a > 0x7f800000u ? 0x7e00u : 0x7c00u);
    if (a >= 0x477ff000u) return sign | 0x7c00u;              /* rounds to +-inf */
    if (a < 0x38800000u) {                                     /* half subnormal range */
        const float v = fabsf(f) * 16777216.0f;                /* exact: power-of-two scale */
        return sign | (uint16_t)nearbyintf(v);                 /* default mode = RNE */
    }
    const uint32_t r = a + 0x0fffu + ((a >> 13) & 1u);          /* RNE on the 13 dropped bits */
    return sign | (uint16_t)((r >> 13) - (112u << 10));
}

static inline float r16(float f) { return orc_h2f(orc_f2h(f)); }

/* ---------------------------------------------------------------------------------------
 * Format: ft_core.h:28-31 (MUL1, HAD, K=3, 96-byte tiles), :38-40 (KINV, KBIAS),
 * :48-61 (PERM), :63-73 (state_scalar), :75-83 (bytesum, w_gpu)
 * ------------------------------------------------------------------------------------- */
#define ORC_MUL1 0x83DCD12Du
#define ORC_HAD 0.088388347648f

/* Bits per weight K (3 in the reference's build, ft_core.h:30). The tile format is generic in K
 * (ft_core.h:63-73 state_scalar is written for any BITS): a 16x16 tile is 16*K int16 words, a
 * circular 256*K-bit stream. Set once before use (the layer oracle's threads only read it). */
static int g_bits = 3;
void orc_set_bits(int bits) { g_bits = (bits == 2 || bits == 4) ? bits : 3; }
int orc_get_bits(void) { return g_bits; }
#define ORC_TILE_WORDS16 (16 * g_bits)

int orc_perm(int i)
{
    /* symbol i of a tile belongs to fragment lane t = i/8, element q = i%8; a lane holds rows
     * {2(t%4), +1, +8, +9} of columns t/4 and t/4+8 (tensor-core B-fragment order) */
    const int t = i >> 3, q = i & 7;
    const int r0 = (t % 4) * 2, c0 = t / 4;
    static const int dr[4] = {0, 1, 8, 9};
    const int r = r0 + dr[q & 3];
    const int c = c0 + ((q >> 2) ? 8 : 0);
    return r * 16 + c;
}

static inline uint32_t word32(const uint16_t* tile, int w)
{
    /* 32-bit little-endian word w (0..8K-1) of the 32K-byte tile */
    return (uint32_t)tile[2 * w] | ((uint32_t)tile[2 * w + 1] << 16);
}

uint16_t orc_state(const uint16_t* tile, int t)
{
    /* The tile is a circular 256K-bit stream read MSB-first through its 8K words; the state of
     * symbol t is the 16-bit window ending at stream bit K*t+K-1, i.e. starting at K*t+K-16
     * (K = 3: 768 bits, 24 words, start 3t-13). */
    const int K = g_bits, nbits = 256 * K, nwords = 8 * K;
    const int start = (K * t + K - 16 + nbits) % nbits;
    const int a = start >> 5, o = start & 31;
    const uint64_t win = ((uint64_t)word32(tile, a) << 32) | word32(tile, (a + 1) % nwords);
    return (uint16_t)((win >> (48 - o)) & 0xffffu);
}

int orc_bytesum(uint16_t state)
{
    const uint32_t x = (uint32_t)state * ORC_MUL1;
    return (int)((x & 0xffu) + ((x >> 8) & 0xffu) + ((x >> 16) & 0xffu) + (x >> 24));
}

uint16_t orc_weight_bits(uint16_t state)
{
    /* one fp16 rounding of fma(1024 + s, KINV, KBIAS); the fp32 fma is exact here
     * (ft_core.h:40, :81-82) */
    const float kinv = orc_h2f(0x1eee), kbias = orc_h2f(0xc931);
    return orc_f2h(fmaf((float)(1024 + orc_bytesum(state)), kinv, kbias));
}

void orc_decode_matrix(const uint16_t* trellis, int k, int n, uint16_t* W)
{
    /* dense_weights (ft_core.h:977-992): tile (tk, tn) at [k/16][n/16][16K] */
    const int tn_count = n / 16;
    for (int tk = 0; tk < k / 16; ++tk)
        for (int tn = 0; tn < tn_count; ++tn) {
            const uint16_t* tile = trellis + ((size_t)tk * tn_count + tn) * ORC_TILE_WORDS16;
            for (int i = 0; i < 256; ++i) {
                const int rc = orc_perm(i);
                W[(size_t)(tk * 16 + rc / 16) * n + tn * 16 + rc % 16] = orc_weight_bits(orc_state(tile, i));
            }
        }
}

/* ---------------------------------------------------------------------------------------
 * Transforms: ft_core.h:89-110 (had128, prep_block, out_block); act: :123-133
 * ------------------------------------------------------------------------------------- */
void orc_had128(float* v)
{
    for (int w = 1; w < 128; w <<= 1)
        for (int b = 0; b < 128; b += 2 * w)
            for (int i = b; i < b + w; ++i) {
                const float p = v[i], q = v[i + w];
                v[i] = p + q;
                v[i + w] = p - q;
            }
}

void orc_prep_block(const float* x, const uint16_t* suh, float* xt)
{
    for (int i = 0; i < 128; ++i) xt[i] = x[i] * orc_h2f(suh[i]);
    orc_had128(xt);
    for (int i = 0; i < 128; ++i) xt[i] = r16(xt[i] * ORC_HAD);
}

void orc_out_block(float* y, const uint16_t* svh)
{
    for (int i = 0; i < 128; ++i) y[i] = r16(y[i]);
    orc_had128(y);
    for (int i = 0; i < 128; ++i) y[i] = r16(y[i] * ORC_HAD * orc_h2f(svh[i]));
}

float orc_act(float g, float u, float limit)
{
    float s = g / (1.0f + expf(-g));
    if (limit != 0.0f) {
        u = fminf(fmaxf(u, -limit), limit);
        s = fminf(s, limit);
    }
    return s * u;
}

/* ---------------------------------------------------------------------------------------
 * Reference linear / expert: ft_core.h:994-1011 (double accumulation, same rounding points),
 * generalised to m tokens and any I (the reference's ref_expert fixes I = 2048)
 * ------------------------------------------------------------------------------------- */
void orc_linear(const uint16_t* trellis, const uint16_t* suh, const uint16_t* svh, int k, int n,
                int m, const float* x, float* y)
{
    float* xt = (float*)malloc(sizeof(float) * (size_t)m * k);
    double* acc = (double*)calloc((size_t)m * n, sizeof(double));
    for (int j = 0; j < m; ++j)
        for (int b = 0; b < k / 128; ++b)
            orc_prep_block(x + (size_t)j * k + b * 128, suh + b * 128, xt + (size_t)j * k + b * 128);
    const int tn_count = n / 16;
    float w[256];
    for (int tk = 0; tk < k / 16; ++tk)
        for (int tn = 0; tn < tn_count; ++tn) {
            const uint16_t* tile = trellis + ((size_t)tk * tn_count + tn) * ORC_TILE_WORDS16;
            for (int i = 0; i < 256; ++i) w[orc_perm(i)] = orc_h2f(orc_weight_bits(orc_state(tile, i)));
            for (int j = 0; j < m; ++j) {
                const float* xr = xt + (size_t)j * k + tk * 16;
                double* ar = acc + (size_t)j * n + tn * 16;
                for (int r = 0; r < 16; ++r) {
                    const double xv = xr[r];
                    for (int c = 0; c < 16; ++c) ar[c] += xv * w[r * 16 + c];
                }
            }
        }
    for (int j = 0; j < m; ++j) {
        for (int c = 0; c < n; ++c) y[(size_t)j * n + c] = (float)acc[(size_t)j * n + c];
        for (int b = 0; b < n / 128; ++b) orc_out_block(y + (size_t)j * n + b * 128, svh + b * 128);
    }
    free(xt);
    free(acc);
}

void orc_expert(const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                const uint16_t* suh_g, const uint16_t* svh_g, const uint16_t* suh_u,
                const uint16_t* svh_u, const uint16_t* suh_d, const uint16_t* svh_d,
                int H, int I, int m, const float* x, float limit, float* y)
{
    float* g = (float*)malloc(sizeof(float) * (size_t)m * I);
    float* u = (float*)malloc(sizeof(float) * (size_t)m * I);
    orc_linear(gate, suh_g, svh_g, H, I, m, x, g);
    orc_linear(up, suh_u, svh_u, H, I, m, x, u);
    for (size_t i = 0; i < (size_t)m * I; ++i) g[i] = r16(orc_act(g[i], u[i], limit));
    orc_linear(down, suh_d, svh_d, I, H, m, g, y);
    free(g);
    free(u);
}

/* ---------------------------------------------------------------------------------------
 * Routing permutation: the routing prep of apply_exl3_fused_moe
 * (patches/vllm-exl3-host-dma.patch:204-226, :300-312): flat_token = arange(T) repeated topk
 * times, local ids with the n_exp sentinel for invalid routes, expert_count[E+1], and the
 * expert-sorted order (stable: ties keep flat order).
 * ------------------------------------------------------------------------------------- */
static inline int local_id(int64_t id, int E, const int32_t* map, int map_len)
{
    if (map) {
        if (id < 0 || id >= map_len) return E;
        const int l = map[id];
        return (l < 0 || l >= E) ? E : l;
    }
    return (id < 0 || id >= E) ? E : (int)id;
}

int orc_permute(const int64_t* ids, const float* weights, int T, int topk, int E,
                const int32_t* expert_map, int map_len, int64_t* counts, int64_t* offsets,
                int32_t* token_sorted, float* weight_sorted, int32_t* route_sorted,
                int32_t* route_pos)
{
    const int n = T * topk;
    memset(counts, 0, sizeof(int64_t) * (size_t)(E + 1));
    for (int i = 0; i < n; ++i) counts[local_id(ids[i], E, expert_map, map_len)]++;
    int64_t run = 0;
    for (int e = 0; e <= E; ++e) {
        offsets[e] = run;
        run += counts[e];
    }
    int64_t* cur = (int64_t*)malloc(sizeof(int64_t) * (size_t)(E + 1));
    memcpy(cur, offsets, sizeof(int64_t) * (size_t)(E + 1));
    for (int i = 0; i < n; ++i) {
        const int l = local_id(ids[i], E, expert_map, map_len);
        const int64_t p = cur[l]++;
        token_sorted[p] = i / topk;
        weight_sorted[p] = weights ? weights[i] : 0.0f;
        route_sorted[p] = i;
        route_pos[i] = (l == E) ? -1 : (int32_t)p;
    }
    free(cur);
    return 0;
}

/* ---------------------------------------------------------------------------------------
 * MoE layer: per-expert jobs over the routed tokens, then the weighted accumulate in fp32
 * (ft_core.h:686-696 / :911-931; tier_forward ft_tier_ext.cpp:177-191)
 * ------------------------------------------------------------------------------------- */
typedef struct {
    const float* x;
    int T, H, I, topk, E;
    const int64_t* ids;
    const int32_t* map;
    int map_len;
    const uint16_t *const *gate, *const *up, *const *down;
    const uint16_t *w13_suh, *w13_svh, *w2_suh, *w2_svh;
    float limit;
    float* yroutes;
    const int64_t* counts;
    const int64_t* offsets;
    const int32_t* route_sorted;
    volatile int next;
} routes_job;

static void* routes_worker(void* arg)
{
    routes_job* J = (routes_job*)arg;
    const size_t H = (size_t)J->H, I = (size_t)J->I;
    for (;;) {
        const int e = __sync_fetch_and_add(&J->next, 1);
        if (e >= J->E) break;
        const int m = (int)J->counts[e];
        if (!m) continue;
        float* xm = (float*)malloc(sizeof(float) * (size_t)m * H);
        float* ym = (float*)malloc(sizeof(float) * (size_t)m * H);
        for (int j = 0; j < m; ++j) {
            const int r = J->route_sorted[J->offsets[e] + j];
            memcpy(xm + (size_t)j * H, J->x + (size_t)(r / J->topk) * H, sizeof(float) * H);
        }
        orc_expert(J->gate[e], J->up[e], J->down[e], J->w13_suh + (size_t)e * 2 * H,
                   J->w13_svh + (size_t)e * 2 * I, J->w13_suh + (size_t)e * 2 * H + H,
                   J->w13_svh + (size_t)e * 2 * I + I, J->w2_suh + (size_t)e * I,
                   J->w2_svh + (size_t)e * H, (int)H, (int)I, m, xm, J->limit, ym);
        for (int j = 0; j < m; ++j) {
            const int r = J->route_sorted[J->offsets[e] + j];
            memcpy(J->yroutes + (size_t)r * H, ym + (size_t)j * H, sizeof(float) * H);
        }
        free(xm);
        free(ym);
    }
    return NULL;
}

void orc_moe_routes(const float* x, int T, int H, int I, const int64_t* ids, int topk, int E,
                    const int32_t* expert_map, int map_len, const uint16_t* const* gate,
                    const uint16_t* const* up, const uint16_t* const* down,
                    const uint16_t* w13_suh, const uint16_t* w13_svh, const uint16_t* w2_suh,
                    const uint16_t* w2_svh, float limit, int nthreads, float* yroutes)
{
    const int n = T * topk;
    int64_t* counts = (int64_t*)malloc(sizeof(int64_t) * (size_t)(E + 1));
    int64_t* offsets = (int64_t*)malloc(sizeof(int64_t) * (size_t)(E + 1));
    int32_t* ts = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n + 1));
    float* ws = (float*)malloc(sizeof(float) * (size_t)(n + 1));
    int32_t* rs = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n + 1));
    int32_t* rp = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n + 1));
    orc_permute(ids, NULL, T, topk, E, expert_map, map_len, counts, offsets, ts, ws, rs, rp);
    memset(yroutes, 0, sizeof(float) * (size_t)n * H);
    routes_job J = {x, T, H, I, topk, E, ids, expert_map, map_len, gate, up, down,
                    w13_suh, w13_svh, w2_suh, w2_svh, limit, yroutes, counts, offsets, rs, 0};
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    for (int i = 1; i < nthreads; ++i) pthread_create(&th[i], NULL, routes_worker, &J);
    routes_worker(&J);
    for (int i = 1; i < nthreads; ++i) pthread_join(th[i], NULL);
    free(counts);
    free(offsets);
    free(ts);
    free(ws);
    free(rs);
    free(rp);
}

void orc_moe_layer(const float* x, int T, int H, int I, const int64_t* ids, const float* weights,
                   int topk, int E, const int32_t* expert_map, int map_len,
                   const uint16_t* const* gate, const uint16_t* const* up,
                   const uint16_t* const* down, const uint16_t* w13_suh,
                   const uint16_t* w13_svh, const uint16_t* w2_suh, const uint16_t* w2_svh,
                   float limit, int nthreads, float* out)
{
    const size_t n = (size_t)T * topk;
    float* y = (float*)malloc(sizeof(float) * n * H);
    orc_moe_routes(x, T, H, I, ids, topk, E, expert_map, map_len, gate, up, down, w13_suh, w13_svh,
                   w2_suh, w2_svh, limit, nthreads, y);
    for (int t = 0; t < T; ++t) {
        float* o = out + (size_t)t * H;
        memset(o, 0, sizeof(float) * H);
        for (int j = 0; j < topk; ++j) {
            const size_t r = (size_t)t * topk + j;
            if (local_id(ids[r], E, expert_map, map_len) == E) continue;
            const float wt = weights[r];
            const float* yr = y + r * H;
            for (int c = 0; c < H; ++c) o[c] += wt * yr[c];
        }
    }
    free(y);
}
