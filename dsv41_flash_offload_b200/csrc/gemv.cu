// Fused decode-GEMV for experts with few rows (decode steps; the GEMV share of prefill).
//
// Replaces the grouped per-expert decode/GEMV of exllamav3_ext.exl3_moe as launched by
// apply_exl3_fused_moe (patches/vllm-exl3-host-dma.patch:315-449), restating the math of the
// reference CPU tier (kernels/cpu_avx2/ft_core.h:587-727 moe_forward phases, :994-1011 ref_*):
//   pass 0 (gate/up): y_g, y_u = xt_{g,u} . W_{g,u}; out_block each 128 block; a = fp16(act);
//                     xt_d = prep_block(a, suh_d)              -> xt_d [rows][I] fp16
//   pass 1 (down):    y = out_block(xt_d . W_d)                -> y    [rows][H] fp16
//
// Work unit = (row group of <= 16 rows of one expert, column block, K split). A persistent grid
// of 2 CTAs per SM walks the units. Per CTA: 8 consumer warps + 1 producer warp.
//   producer: one 1-D bulk async copy (cp.async.bulk, into this CTA only) per 8/16-tile trellis
//             k-row segment and per 256-byte activation row into a 2-stage mbarrier ring of 16
//             k-rows per stage; trellis reads carry an L2 evict-first hint (each expert byte is
//             read once).
//   consumer warp w: owns two adjacent 16-column n-tiles that share one ldmatrix'd fragment of the
//             group's tokens; per k-tile and n-tile it loads the window words of its lane from the
//             staged tile, decodes its 8 weights in registers and issues mma.m16n8k16 with the
//             decoded tile as the A operand (16 features x 16 k) and the tokens as the B operand
//             (k16 x n8): one MMA per tile for groups of up to 8 rows, two for 9-16. The lane's 8
//             symbols are the mma fragment's (k, n) pairs in either operand role (the format is laid
//             out for it), only the register order differs. Decoded weights never leave registers.
//   affine form (DSV41_GEMV_AFFINE, default): the A fragments carry the weights' affine codes
//             1024 + bytesum (decode_tile_codes), one more MMA per k-row against an all-ones A
//             gives the token sums, and the epilogue forms KINV * sum(code x) + KBIAS * sum(x) in
//             fp32 -- the reference CPU tier's AFFINE mode (kernels/cpu_avx2/ft_core.h:293, chosen
//             by its auto mode at decode sizes, :936). It differs from the exact form (fp16-rounded
//             weights, DSV41_GEMV_AFFINE=0) by the weights' fp16 rounding only.
// Split-K partials (small batches) are reduced in a fixed order by the last-arriving CTA, so
// results are deterministic.
#include "common.cuh"
#include "internal.h"

namespace dsv41 {

// launch-shape parameters (compile-time; the defaults are the tuned values)
#ifndef DSV41_GEMV_MIN_BLOCKS
#define DSV41_GEMV_MIN_BLOCKS 2       // resident CTAs per SM (register budget follows)
#endif
#ifndef DSV41_GEMV_STAGE_ROWS
#define DSV41_GEMV_STAGE_ROWS 16      // k-tile rows per pipeline stage
#endif
#ifndef DSV41_GEMV_STAGES
#define DSV41_GEMV_STAGES 2
#endif
// Measured on B200 (gate/up GEMV of the decode T=64 step, 285 experts): tokens as the A operand
// (two MMAs per tile) with exact weights 1.217 ms; the same with affine codes 1.177; weights as the A
// operand, exact 1.122, affine 1.102 (kept). Not kept: byte sums on the tensor pipe (two int8 MMAs per
// tile instead of 8 DP4A) 1.279; one tile per warp (16 consumer warps) 1.277; 3 CTAs/SM with 8-row
// stages 1.147; 8-row stages x 4 1.176; an L2 prefetch of the trellis rows 4 or 8 stages ahead of the
// ring 1.185 (and T=1 0.046 -> 0.061 ms). Earlier: 16-row stages x 2 beat 8 x 4 and 1 or 3 CTAs/SM.
// The one-CTA form (KS = 2, 4 stages) takes T=1 from 0.0473 to 0.0463 ms: small calls are bound by the
// same per-SM decode rate (128 units = 8 experts x 16 column blocks on 128 SMs).

#ifndef DSV41_GEMV_AFFINE
#define DSV41_GEMV_AFFINE 1
#endif
#ifndef DSV41_GEMV_IMAD_PACKS
#define DSV41_GEMV_IMAD_PACKS 3       // of the 4 half2 code packs per lane and tile, how many on IMAD (measured 2: 1.577, 3: 1.556, 4: 1.576 ms GEMV at T=64)
#endif

#ifndef DSV41_GEMV_PAIRED
#define DSV41_GEMV_PAIRED 1           // decode a warp's two tiles with their states interleaved (K = 3)
#endif

#ifndef DSV41_GEMV_ROW_UNROLL
#define DSV41_GEMV_ROW_UNROLL 16      // k-rows of a stage unrolled in the consumer loop
#endif
constexpr int kRowUnroll = DSV41_GEMV_ROW_UNROLL;

#ifndef DSV41_GEMV_TILES_PER_WARP
#define DSV41_GEMV_TILES_PER_WARP 2   // adjacent n-tiles per consumer warp (they share the A fragment)
#endif

constexpr int kTilesPerWarp = DSV41_GEMV_TILES_PER_WARP;
// KS = 1: 8 consumer warps cover the 16 n-tiles of each staged k-row, 2 CTAs per SM (the default).
// KS = 2 (calls with fewer units than SMs, e.g. one-token decode): 16 consumer warps in one CTA per SM,
// warp w decodes the tiles of warp w % 8 on the k-rows of parity w / 8, and the two partial sums are
// added in shared memory in a fixed order -- twice the warps per unit without global partials.
template <int KS>
__host__ __device__ constexpr int consumer_warps() { return KS * 16 / kTilesPerWarp; }
template <int KS>
__host__ __device__ constexpr int gemv_threads() { return (consumer_warps<KS>() + 1) * 32; }
constexpr int kStageRows = DSV41_GEMV_STAGE_ROWS;
// ring stages: the 2-CTA form (KS = 1) fits two 16-row stages per CTA; the one-CTA form (KS = 2) four
template <int KS>
__host__ __device__ constexpr int gemv_stages() { return KS == 1 ? DSV41_GEMV_STAGES : 2 * DSV41_GEMV_STAGES; }

template <int K>
__host__ __device__ constexpr int row_bytes() { return 16 * TileFmt<K>::bytes; }   // 16 tiles of one k-row (1536 B at K = 3)
constexpr int kXRowStride = kStageRows * 32 + 16;  // stage's k-tiles x 16 halves, + 16 B pad (ldmatrix banks)
constexpr int kXMatBytes = 16 * kXRowStride;
constexpr int kEpFloats = 4096;

template <int K, int ST>
struct GemvSmem {
    static constexpr int kStages = ST;
    uint8_t tr[kStages][kStageRows * row_bytes<K>()];
    uint8_t x[kStages][2][kXMatBytes];
    float ep[kEpFloats];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    int stage_unit[kStages];   // ticket of the unit a stage belongs to (-1: no more work)
    int next_unit;             // consumers' shared decision of the next unit
    int abort_flag;
    int last_flag;
};

size_t gemv_smem_bytes(int bits)
{
    return bits == 2 ? sizeof(GemvSmem<2, 2>) : bits == 4 ? sizeof(GemvSmem<4, 2>) : sizeof(GemvSmem<3, 2>);
}
int gemv_stage_rows() { return kStageRows; }

__device__ __forceinline__ void out_block4(float (&y)[4], const __half* svh, int lane)
{
#pragma unroll
    for (int q = 0; q < 4; ++q) y[q] = r16(y[q]);
    had128_warp(y, lane);
    const uint2 u = *reinterpret_cast<const uint2*>(svh);
    const __half2 a = u32_as_half2(u.x), b = u32_as_half2(u.y);
    const float s[4] = {__low2float(a), __high2float(a), __low2float(b), __high2float(b)};
#pragma unroll
    for (int q = 0; q < 4; ++q) y[q] = r16(__fmul_rn(__fmul_rn(y[q], kHad), s[q]));
}

__device__ __forceinline__ void ldmatrix_x2(uint32_t (&a)[4], uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(a[0]), "=r"(a[1]) : "r"(addr));
}

// One staged k-row block: for each k-row, the tokens' B fragments (TWO: tokens 8-15 as a second n8
// block), then per tile the decoded A fragment {b0, b2, b1, b3} (decode_tile returns the lane's
// weights in B-fragment register order: (k 2q.., n g), (k 2q+8.., n g), (k 2q.., n g+8), (k 2q+8..,
// n g+8)) and one MMA per n8 block. The affine form adds the token sums from an all-ones A.
template <int K, bool TWO, int KS>
__device__ __forceinline__ void gemv_stage(const uint32_t* trow, uint32_t xaddr, const LaneDec<K>& lw,
                                                   uint32_t k16, float (&acc)[kTilesPerWarp][2][4],
                                                   float (&rs)[2][4], int par)
{
    constexpr int kTW = TileFmt<K>::words, kRowWords = row_bytes<K>() / 4;
#pragma unroll kRowUnroll
    for (int r0 = 0; r0 < kStageRows; r0 += KS) {
        const int r = r0 + par;
        uint32_t bx[4];
        if (TWO)
            ldmatrix_x4(bx, xaddr + r * 32);
        else
            ldmatrix_x2(bx, xaddr + r * 32);
#if DSV41_GEMV_AFFINE
        const uint32_t ones[4] = {0x3c003c00u, 0x3c003c00u, 0x3c003c00u, 0x3c003c00u};
        mma_16816(rs[0], ones, bx[0], bx[1]);
        if (TWO) mma_16816(rs[1], ones, bx[2], bx[3]);
#endif
#if DSV41_GEMV_AFFINE && DSV41_GEMV_PAIRED && DSV41_CODES_WIN2
        if constexpr (K == 3 && kTilesPerWarp == 2) {
            uint32_t b[2][4];
            decode_tiles_codes3<2, DSV41_GEMV_IMAD_PACKS>(trow + r * kRowWords, lw, k16, b);
            const uint32_t a0[4] = {b[0][0], b[0][2], b[0][1], b[0][3]}, a1[4] = {b[1][0], b[1][2], b[1][1], b[1][3]};
            mma_16816(acc[0][0], a0, bx[0], bx[1]);
            mma_16816(acc[1][0], a1, bx[0], bx[1]);
            if (TWO) {
                mma_16816(acc[0][1], a0, bx[2], bx[3]);
                mma_16816(acc[1][1], a1, bx[2], bx[3]);
            }
            continue;
        }
#endif
#pragma unroll
        for (int t = 0; t < kTilesPerWarp; ++t) {
            const uint32_t* tw = trow + r * kRowWords + t * kTW;
            uint32_t b[4];
#if DSV41_GEMV_AFFINE
            decode_tile_codes<K, DSV41_GEMV_IMAD_PACKS>(tw, lw, k16, b);
#else
            decode_tile<K>(tw, lw, k16, b);
#endif
            const uint32_t a[4] = {b[0], b[2], b[1], b[3]};
            mma_16816(acc[t][0], a, bx[0], bx[1]);
            if (TWO) mma_16816(acc[t][1], a, bx[2], bx[3]);
        }
    }
}

// One decode-GEMV launch: pass 0 (gate/up) and/or pass 1 (down) of the same row groups. Units of pass
// m: n_groups x (N_m / cols_m) x split_m. The producer warp of each CTA takes units from a global ticket
// counter, in order, and hands each to its consumer warps through the ring (the unit's ticket rides in
// the stage slot), so the units handed out are always being processed by running CTAs: a launch that
// runs both passes takes every gate/up unit first, and the producer of a down unit of group g waits
// (bounded) until all gate/up units of g have stored their rows (ready[g]) -- no dependence on which
// CTAs are resident, and the down units fill the gate/up pass's last wave.
struct GemvWork {
    GemvParams p[2];
    int first, last;   // passes run: first..last
    int* tickets;      // [1] next unit (zero before the launch)
    int* ready;        // [groups] finished gate/up units per group (zero; used when both passes run)
};

template <int MODE>
__device__ __forceinline__ int gemv_pass_units(const GemvParams& p, int ng)
{
    return ng * (p.N / (MODE == 0 ? 128 : 256)) * p.split;
}

// bounded wait until *cnt >= need (acquire, gpu scope); false (status 1) on expiry or abort
__device__ __forceinline__ bool wait_count(const int* cnt, int need, volatile int* abort_flag, int* status)
{
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        int v;
        asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
        if (v >= need) return true;
        if ((it & 15u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                *abort_flag = 1;
                if (status) atomicExch(status, kStatusWaitTimeout);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// producer side of one unit (ticket v): its stages' bulk copies into the ring
template <int MODE, int K, int ST>
__device__ __forceinline__ bool gemv_produce(const GemvParams& p, GemvSmem<K, ST>& S, int u, int v, uint32_t& it,
                                             int lane, uint64_t pol_w, uint64_t pol_x, const int* ready,
                                             int ready_need)
{
    constexpr int kTB = TileFmt<K>::bytes, kRowBytes = row_bytes<K>();
    constexpr int nmat = MODE == 0 ? 2 : 1;
    constexpr int cols = MODE == 0 ? 128 : 256;
    const int n_cb = p.N / cols;
    const int k_per_split = p.K / 16 / p.split;
    const int stages_per_unit = k_per_split / kStageRows;
    const int ntile_row = p.N / 16;
    const int s = u % p.split, ucb = u / p.split, cb = ucb % n_cb, g = ucb / n_cb;
    const int4 G = p.groups[g];
    const int e = G.x, row0 = G.y, rows = G.z;
    if (ready) {   // this down unit reads the group's gate/up outputs
        int ok = 1;
        if (lane == 0) ok = wait_count(ready + g, ready_need, &S.abort_flag, p.status) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) return false;
        fence_proxy_async_global();   // the rows were written through the generic proxy
    }
    const uint8_t* ta = reinterpret_cast<const uint8_t*>(p.tab_a[e]);
    const uint8_t* tb = MODE == 0 ? reinterpret_cast<const uint8_t*>(p.tab_b[e]) : nullptr;
    for (int st = 0; st < stages_per_unit; ++st, ++it) {
        const int stage = it % ST;
        const uint32_t round = it / ST;
        if (!mbar_wait_bounded(&S.empty[stage], (round & 1) ^ 1, &S.abort_flag, p.status)) return false;
        const int kt0 = s * k_per_split + st * kStageRows;
        if (lane == 0) {
            S.stage_unit[stage] = v;
            mbar_arrive_expect_tx(&S.full[stage], kStageRows * kRowBytes + nmat * rows * kStageRows * 32);
        }
        __syncwarp();
        if (MODE == 0) {
            if (lane < 2 * kStageRows) {
                const int r = lane >> 1, which = lane & 1;
                const uint8_t* src = (which ? tb : ta) + ((size_t)(kt0 + r) * ntile_row + cb * 8) * kTB;
                bulk_g2s(S.tr[stage] + r * kRowBytes + which * 8 * kTB, src, 8 * kTB, &S.full[stage], pol_w);
            }
        } else {
            if (lane < kStageRows) {
                const uint8_t* src = ta + ((size_t)(kt0 + lane) * ntile_row + cb * 16) * kTB;
                bulk_g2s(S.tr[stage] + lane * kRowBytes, src, kRowBytes, &S.full[stage], pol_w);
            }
        }
        for (int c = lane; c < nmat * rows; c += 32) {
            const int m = c / rows, j = c % rows;
            const __half* src = (m ? p.xb : p.xa) + (size_t)(row0 + j) * p.K + kt0 * 16;
            bulk_g2s(S.x[stage][m] + j * kXRowStride, src, kStageRows * 32, &S.full[stage], pol_x);
        }
    }
    return true;
}

// consumer side of one unit: decode + MMAs over its stages, the ordered partial-sum merge, split-K
// reduction and the epilogue; with `ready`, a gate/up unit counts itself done for its group
template <int MODE, int K, int KS, int ST>
__device__ __forceinline__ void gemv_consume(const GemvParams& p, GemvSmem<K, ST>& S, int u, uint32_t& it, int warp,
                                             int lane, const LaneDec<K>& lw, int* ready)
{
    constexpr int kConsumerWarps = consumer_warps<KS>();
    constexpr int kTW = TileFmt<K>::words;
    constexpr int cols = MODE == 0 ? 128 : 256;
    const int n_cb = p.N / cols;
    const int stages_per_unit = p.K / 16 / p.split / kStageRows;
    const uint32_t k16 = p.k16;
    const int par = warp / 8;                              // k-row parity of this warp (KS = 2)
    const int tile0 = (warp % 8) * kTilesPerWarp;          // first of this warp's adjacent n-tiles (0..15)
    const int mat = MODE == 0 ? (tile0 >> 3) : 0;          // gate/up pass: tiles 0-7 gate, 8-15 up
    // B fragments: matrices (tokens 0-7, k 0-7), (0-7, 8-15), (8-15, 0-7), (8-15, 8-15)
    const uint32_t x_lane = ((lane & 7) + ((lane >> 4) & 1) * 8) * kXRowStride + ((lane >> 3) & 1) * 16;
    const int ucb = u / p.split, cb = ucb % n_cb, g = ucb / n_cb;
    const int4 G = p.groups[g];
    const int e = G.x, row0 = G.y, rows = G.z;
    float acc[kTilesPerWarp][2][4];
#pragma unroll
    for (int t = 0; t < kTilesPerWarp; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[t][h][q] = 0.f;
    float rs[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};   // token sums (affine form)
    const bool two = rows > 8;
    for (int st = 0; st < stages_per_unit; ++st, ++it) {
        const int stage = it % ST;
        const uint32_t round = it / ST;
        // a wait that runs out (or a CTA that already gave up) skips the stage's compute: the staged
        // bytes may never have arrived. The warp still takes every barrier step below.
        if (mbar_wait_bounded(&S.full[stage], round & 1, &S.abort_flag, p.status)) {
            // this warp's tiles sit at byte offset tile * 32K of each staged 16-tile k-row
            const uint32_t* trow = reinterpret_cast<const uint32_t*>(S.tr[stage]) + tile0 * kTW;
            const uint32_t xaddr = smem_addr(S.x[stage][mat]) + x_lane;
            if (two)
                gemv_stage<K, true, KS>(trow, xaddr, lw, k16, acc, rs, par);
            else
                gemv_stage<K, false, KS>(trow, xaddr, lw, k16, acc, rs, par);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[stage]);
    }

#if DSV41_GEMV_AFFINE
    // sum_k w x = KINV * sum_k code x + KBIAS * sum_k x (per split: the partial sums add up the same)
#pragma unroll
    for (int t = 0; t < kTilesPerWarp; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[t][h][q] = fmaf(kKinv, acc[t][h][q], kKbias * rs[h][q]);
#endif
    // accumulators (feature g / g + 8 of the tile, tokens 8h + 2q, + 1) -> shared [mat][row][cols];
    // with KS = 2 the odd-row warps add their partial sums to the even-row warps' (fixed order)
#pragma unroll
    for (int phase = 0; phase < KS; ++phase) {
        if (par == phase) {
#pragma unroll
            for (int t = 0; t < kTilesPerWarp; ++t) {
                const int tile = tile0 + t;
                const int fcol = (MODE == 0 ? (tile & 7) : tile) * 16 + (lane >> 2);
                float* ep = S.ep + (MODE == 0 ? mat * 16 * cols : 0);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    if (h == 1 && !two) break;
                    const int tok = 8 * h + (lane & 3) * 2;
                    float* e0 = ep + tok * cols + fcol;
                    float* e1 = e0 + cols;
                    if (phase == 0) {
                        e0[0] = acc[t][h][0];
                        e1[0] = acc[t][h][1];
                        e0[8] = acc[t][h][2];
                        e1[8] = acc[t][h][3];
                    } else {
                        e0[0] += acc[t][h][0];
                        e1[0] += acc[t][h][1];
                        e0[8] += acc[t][h][2];
                        e1[8] += acc[t][h][3];
                    }
                }
            }
        }
        named_bar_sync(1, kConsumerWarps * 32);
    }

    if (p.split > 1) {
        float* slot = p.partials + (size_t)u * kEpFloats;
        for (int i = threadIdx.x * 4; i < kEpFloats; i += kConsumerWarps * 32 * 4)
            __stcg(reinterpret_cast<float4*>(slot + i), *reinterpret_cast<const float4*>(S.ep + i));
        __threadfence();
        named_bar_sync(1, kConsumerWarps * 32);
        if (threadIdx.x == 0) {
            const int old = atomicAdd(p.counters + ucb, 1);
            S.last_flag = (old == p.split - 1);
        }
        named_bar_sync(1, kConsumerWarps * 32);
        if (!S.last_flag) return;
        __threadfence();
        for (int i = threadIdx.x * 4; i < kEpFloats; i += kConsumerWarps * 32 * 4) {
            float4 v = __ldcg(reinterpret_cast<const float4*>(p.partials + (size_t)ucb * p.split * kEpFloats + i));
            for (int s2 = 1; s2 < p.split; ++s2) {
                const float4 w = __ldcg(reinterpret_cast<const float4*>(
                    p.partials + ((size_t)ucb * p.split + s2) * kEpFloats + i));
                v.x += w.x; v.y += w.y; v.z += w.z; v.w += w.w;
            }
            *reinterpret_cast<float4*>(S.ep + i) = v;
        }
        if (threadIdx.x == 0) p.counters[ucb] = 0;
        named_bar_sync(1, kConsumerWarps * 32);
    }

    // epilogue: warp w transforms rows w, w + kConsumerWarps, ... of the group. Once this CTA has given
    // up on a wait, its remaining rows are written as zeros (the status word says why).
    const bool aborted = *reinterpret_cast<volatile int*>(&S.abort_flag) != 0;
    for (int j = warp; j < rows; j += kConsumerWarps) {
        __half* orow = out_row(p.out, p.push, row0 + j, p.N);
        if (aborted) {
            for (int c = lane * 4; c < cols; c += 128)
                *reinterpret_cast<uint2*>(orow + cb * cols + c) = make_uint2(0u, 0u);
            continue;
        }
        if (MODE == 0) {
            float gv[4], uv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                gv[q] = S.ep[j * 128 + lane * 4 + q];
                uv[q] = S.ep[(16 + j) * 128 + lane * 4 + q];
            }
            const size_t sv = (size_t)e * 2 * p.N + cb * 128 + lane * 4;
            out_block4(gv, p.svh_a + sv, lane);
            out_block4(uv, p.svh_a + sv + p.N, lane);
            const uint2 su = *reinterpret_cast<const uint2*>(p.suh_d + (size_t)e * p.N + cb * 128 + lane * 4);
            const __half2 s01 = u32_as_half2(su.x), s23 = u32_as_half2(su.y);
            const float sd[4] = {__low2float(s01), __high2float(s01), __low2float(s23), __high2float(s23)};
            float v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) v[q] = __fmul_rn(r16(act_gu(gv[q], uv[q], p.limit)), sd[q]);
            had128_warp(v, lane);
            uint2 o;
            o.x = half2_as_u32(__floats2half2_rn(__fmul_rn(v[0], kHad), __fmul_rn(v[1], kHad)));
            o.y = half2_as_u32(__floats2half2_rn(__fmul_rn(v[2], kHad), __fmul_rn(v[3], kHad)));
            *reinterpret_cast<uint2*>(orow + cb * 128 + lane * 4) = o;
        } else {
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
                float y[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) y[q] = S.ep[j * 256 + blk * 128 + lane * 4 + q];
                const size_t c = (size_t)cb * 256 + blk * 128 + lane * 4;
                out_block4(y, p.svh_a + (size_t)e * p.N + c, lane);
                uint2 o;
                o.x = half2_as_u32(__floats2half2_rn(y[0], y[1]));
                o.y = half2_as_u32(__floats2half2_rn(y[2], y[3]));
                *reinterpret_cast<uint2*>(orow + c) = o;
            }
        }
    }
    named_bar_sync(1, kConsumerWarps * 32);
    if (MODE == 0 && ready && threadIdx.x == 0) {
        // the group's rows of this column block are stored (every consumer warp passed the barrier):
        // publish them to the down units' producers (bulk copies, the async proxy)
        fence_proxy_async_global();
        __threadfence();
        atomicAdd(ready + g, 1);
    }
}

template <int K, int KS>
__global__ void __launch_bounds__(gemv_threads<KS>(), KS == 1 ? DSV41_GEMV_MIN_BLOCKS : 1)
    exl3_gemv_kernel(const __grid_constant__ GemvWork w)
{
    griddep_enter();
    constexpr int kConsumerWarps = consumer_warps<KS>();
    constexpr int kStages = gemv_stages<KS>();
    using Smem = GemvSmem<K, kStages>;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem& S = *reinterpret_cast<Smem*>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ng = *w.p[w.first].n_groups;
    const int u0 = w.first == 0 ? gemv_pass_units<0>(w.p[0], ng) : gemv_pass_units<1>(w.p[1], ng);
    const int total = u0 + (w.last > w.first ? gemv_pass_units<1>(w.p[1], ng) : 0);
    const bool fused = w.last > w.first;
    // ticket v -> pass and unit within the pass
    auto which = [&](int v, int& mode, int& u) {
        if (v < u0) {
            mode = w.first;
            u = v;
        } else {
            mode = 1;
            u = v - u0;
        }
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], kConsumerWarps);
        }
        S.abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ------------------------------ producer warp ------------------------------
        const uint64_t pol_w = l2_policy_evict_first();
        const uint64_t pol_x = l2_policy_evict_last();
        uint32_t it = 0;
        bool ok = true;
        while (ok) {
            int v = 0;
            if (lane == 0) v = atomicAdd(w.tickets, 1);
            v = __shfl_sync(0xffffffffu, v, 0);
            if (v >= total) {
                // end of the work: the next ring stage carries ticket -1
                const int stage = it % kStages;
                ok = mbar_wait_bounded(&S.empty[stage], ((it / kStages) & 1) ^ 1, &S.abort_flag, w.p[w.first].status);
                if (ok && lane == 0) {
                    S.stage_unit[stage] = -1;
                    mbar_arrive(&S.full[stage]);
                }
                break;
            }
            int mode, u;
            which(v, mode, u);
            if (mode == 0)
                ok = gemv_produce<0, K, kStages>(w.p[0], S, u, v, it, lane, pol_w, pol_x, nullptr, 0);
            else
                ok = gemv_produce<1, K, kStages>(w.p[1], S, u, v, it, lane, pol_w, pol_x, fused ? w.ready : nullptr,
                                                 w.p[0].N / 128 * w.p[0].split);
        }
        if (!ok && lane == 0) {
            // drain: do not leave the CTA while copies into its shared memory are in flight
            const uint32_t n_back = it < (uint32_t)kStages ? it : (uint32_t)kStages;
            for (uint32_t q = 1; q <= n_back; ++q) {
                const uint32_t j = it - q;
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(&S.full[j % kStages], (j / kStages) & 1) && globaltimer_ns() - t0 < kWaitLimitNs) {}
            }
        }
        return;
    }

    // ------------------------------ consumer warps ------------------------------
    const LaneDec<K> lw = lane_dec_setup<K>(lane);
    uint32_t it = 0;
    for (;;) {
        // the unit of the next stage, decided once for all consumer warps: thread 0 reads it (or -1 once
        // the CTA has given up, including on a wait of the producer) between two consumer barriers
        const int stage = it % kStages;
        mbar_wait_bounded(&S.full[stage], (it / kStages) & 1, &S.abort_flag, w.p[w.first].status);
        named_bar_sync(1, kConsumerWarps * 32);
        if (threadIdx.x == 0) S.next_unit = *reinterpret_cast<volatile int*>(&S.abort_flag) ? -1 : S.stage_unit[stage];
        named_bar_sync(1, kConsumerWarps * 32);
        const int v = S.next_unit;
        if (v < 0) break;
        int mode, u;
        which(v, mode, u);
        if (mode == 0)
            gemv_consume<0, K, KS, kStages>(w.p[0], S, u, it, warp, lane, lw, fused ? w.ready : nullptr);
        else
            gemv_consume<1, K, KS, kStages>(w.p[1], S, u, it, warp, lane, lw, nullptr);
    }
    // output rows stored into peers' memory are made visible at system scope before the kernel ends (the
    // exchange's release stamp follows on the stream)
    if (w.p[1].push.route) __threadfence_system();
}

int gemv_units_bound(int groups_bound, int K, int N, int mode, int split)
{
    const int cols = mode == 0 ? 128 : 256;
    return groups_bound * (N / cols) * split;
}

// buffer sizing over both passes (gate/up: I/128 column blocks, down: H/256)
int gemv_units_alloc(int groups_bound, int H, int I, int split)
{
    const int cb = (I / 128 > H / 256) ? I / 128 : H / 256;
    return groups_bound * cb * split;
}

template <int K, int KS>
static cudaError_t launch_work_k(const GemvWork& w, int units_bound, cudaStream_t st)
{
    const size_t smem = sizeof(GemvSmem<K, gemv_stages<KS>()>);
    cudaError_t err =
        cudaFuncSetAttribute((const void*)exl3_gemv_kernel<K, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    int grid = (KS == 1 ? DSV41_GEMV_MIN_BLOCKS : 1) * num_sms();
    if (units_bound < grid) grid = units_bound;
    if (grid < 1) grid = 1;
    return launch_k(exl3_gemv_kernel<K, KS>, grid, gemv_threads<KS>(), smem, st, w);
}

// calls whose passes each fit in one CTA per SM run the 16-warp form (twice the warps per unit)
template <int K>
static cudaError_t launch_work(const GemvWork& w, int pass_bound, int units_bound, cudaStream_t st)
{
    if (pass_bound <= num_sms()) return launch_work_k<K, 2>(w, units_bound, st);
    return launch_work_k<K, 1>(w, units_bound, st);
}

int gemv_sched_ints(int groups_bound) { return groups_bound + 2; }

cudaError_t launch_gemv_passes(const GemvParams& gateup, const GemvParams& down, int first, int last, int* sched,
                               int groups_bound, bool clear, cudaStream_t st)
{
    if (clear) {
        const cudaError_t err = cudaMemsetAsync(sched, 0, (size_t)gemv_sched_ints(groups_bound) * 4, st);
        if (err != cudaSuccess) return err;
    }
    GemvWork w{};
    w.p[0] = gateup;
    w.p[1] = down;
    w.first = first;
    w.last = last;
    w.tickets = sched + first;   // one ticket counter per pass launch
    w.ready = sched + 2;
    const int b0 = gemv_units_bound(groups_bound, gateup.K, gateup.N, 0, gateup.split);
    const int b1 = gemv_units_bound(groups_bound, down.K, down.N, 1, down.split);
    const int pass_bound = first == 0 && last == 0 ? b0 : first == 1 ? b1 : (b0 > b1 ? b0 : b1);
    const int units_bound = (first == 0 ? b0 : 0) + (last == 1 ? b1 : 0);
    const int bits = first == 0 ? gateup.bits : down.bits;
    if (bits == 2) return launch_work<2>(w, pass_bound, units_bound, st);
    if (bits == 4) return launch_work<4>(w, pass_bound, units_bound, st);
    return launch_work<3>(w, pass_bound, units_bound, st);
}

}  // namespace dsv41
