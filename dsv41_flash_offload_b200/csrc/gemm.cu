// Busy-expert ("fat") path: decode-to-shared-memory + tcgen05/TMEM grouped GEMM.
//
// Replaces apply_exl3_batched_fat (patches/vllm-exl3-host-dma.patch:182-201: reconstruct fp16 W,
// then a 128x128 FP16 GEMM per busy expert; runtime/dma_gemm.py:5-26) with one persistent kernel
// per pass in which the weights are decoded straight into the tensor-core operand layout:
//   pass 0 (gate/up): D_g, D_u [rows x 128 features] = xt_{g,u} . W_{g,u}; epilogue per row:
//                     out_block, SwiGLU clamp, fp16, down-input transform -> xt_d
//   pass 1 (down):    D [rows x 128 features] = xt_d . W_d; epilogue: out_block -> y (fp16)
// Work unit = (busy expert, row pass of 256 (gate/up) or 512 (down) rows, 128-feature block).
// One CTA per SM, 12 warps, two mbarrier rings (activations + decoded weights advance together under
// one full/empty pair; trellis words run ahead in their own ring):
//   warp 0     activation producer: TMA (cp.async.bulk.tensor, SWIZZLE_128B, into this CTA only) of
//              128-row x 64-k tiles; a stage is reused once the MMAs that read it have committed
//   warps 1, 3 TMEM allocator (warp 1, 512 columns) and two single-thread tcgen05.mma issuers
//              (kind::f16, M=128, N=128, K=16, fp32 accumulators in TMEM); tcgen05.commit releases
//              the activation and weight stages and signals the finished accumulators
//   warp 2     trellis producer: 1-D bulk copies of the compressed k-rows into a 4-8 stage ring
//              that the decoders release, so the words stream ahead of the MMAs
//   warps 4-11 decoders: each lane decodes its 8 weights of a 16x16 tile in registers (the same
//              exact decode as the GEMV) and stores them as K-major 128B-swizzled fp16 B-operand
//              rows; after the last k chunk they are the epilogue (tcgen05.ld, one row per thread,
//              128-point Hadamard in registers, intermediate results parked in TMEM, the unit's scale
//              rows prefetched into L1 while the last MMAs run, 32-byte row stores)
// Experts with more rows than one pass reuse each decoded weight for 256/512 rows.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemm.h"
#include "internal.h"

namespace dsv41 {

// warp roles
// (warp w issues on SM sub-partition w % 4 and may only touch TMEM lanes 32*(w%4)..+31: the two
// producers and two MMA issuers take one sub-partition each, so every sub-partition runs one of
// them plus two decoders, and the decoders cover each TMEM lane quarter twice)
constexpr int kWarpA = 0;        // TMA producer of the activation tiles
constexpr int kWarpMma = 1;      // TMEM allocator + single-thread tcgen05.mma issuer
constexpr int kWarpT = 2;        // bulk-copy producer of the trellis k-rows
constexpr int kWarpMma2 = 3;     // second MMA issuer (merged ring)
constexpr int kWarpDec0 = 4;     // warps 4..11: decoders, then epilogue
constexpr int kDecWarps = 8;
constexpr int kGemmThreads = (kWarpDec0 + kDecWarps) * 32;   // 384
#ifndef DSV41_GEMM_DEC_UNROLL
#define DSV41_GEMM_DEC_UNROLL 4
#endif
constexpr int kDecUnroll = DSV41_GEMM_DEC_UNROLL;   // tiles of the decode loop in flight per warp
#ifndef DSV41_GEMM_PAIRED
#define DSV41_GEMM_PAIRED 1   // decode a warp's tiles 2 (1 or 2), 4 or 8 at a time, states interleaved (K = 3)
#endif
#ifndef DSV41_GEMM_IMAD_PACKS
#define DSV41_GEMM_IMAD_PACKS 4   // of the 4 half2 code packs per lane and tile, how many on IMAD
#endif
#ifndef DSV41_GEMM_MERGED_RING
#define DSV41_GEMM_MERGED_RING 1
#endif
// 1: the activation and decoded-weight stages advance together under one full barrier (TMA bytes +
// one arrival per decoder warp) and one empty barrier, so the MMA thread waits once and commits once
// per chunk (each wait and commit of the issuing thread costs the tensor pipe a few hundred cycles)
constexpr bool kMergedRing = DSV41_GEMM_MERGED_RING != 0;
// Two threads issue the MMAs, each for its own accumulators ((M tile, matrix) pairs alternate): every
// wait -> MMAs -> commit cycle of one issuing thread leaves the tensor pipe idle for ~500 cycles
// (measured on B200, independent of the group size), and the other thread's MMAs fill that gap
// (probe: 16-MMA groups at 97 cycles per MMA with one issuer, 64 with two; ideal 64).
constexpr int kIssuers = kMergedRing ? 2 : 1;
constexpr int kBM = 128;        // rows per M tile (TMEM lanes)
constexpr int kBN = 128;        // features per unit (TMEM columns per accumulator)
#ifndef DSV41_GEMM_BK
#define DSV41_GEMM_BK 64
#endif
// k per chunk: 64 (one 128-byte SWIZZLE_128B row of fp16 per operand row) or 32 (SWIZZLE_64B, twice
// the ring stages in the same shared memory). Measured on B200, 16k-token prefill: gate/up GEMM
// 7.36 ms with 64, 8.68 ms with 32 (twice the barrier hand-offs per FLOP; the decoders, not the
// ring depth, bound the main loop).
constexpr int kBK = DSV41_GEMM_BK;
static_assert(kBK == 32 || kBK == 64, "chunk must be 32 or 64");
constexpr int kKT = kBK / 16;           // k-tiles (16 k) per chunk
constexpr int kRowB = kBK * 2;          // bytes of one operand row in a stage (= swizzle span)
constexpr int kAtom = 8 * kRowB;        // bytes of one 8-row swizzle atom
constexpr int kTileA = kBM * kRowB;     // one 128-row activation tile
constexpr int kTileB = kBN * kRowB;     // one 128-feature decoded weight tile
template <int K>
__host__ __device__ constexpr int tr_row() { return 8 * TileFmt<K>::bytes; }   // 8 n-tiles of one k-tile row (768 B at K = 3)

// Rings per CTA (each with full/empty mbarriers):
//   A (activations, TMA)   released by tcgen05.commit after the chunk's MMAs
//   B (decoded weights)    written by the decoders, released by tcgen05.commit (with the merged ring,
//                          A and B stages share one full barrier: TMA bytes + one arrival per decoder)
//   T (trellis k-rows)     filled by the trellis producer, released by the decoders, so the
//                          compressed words stream ahead of the MMAs by several chunks
template <int MODE, int K>
struct GemmCfg {
    static constexpr int nmat = MODE == 0 ? 2 : 1;
    static constexpr int mtiles = MODE == 0 ? 2 : 4;      // M tiles per pass
    static constexpr int rows_per_pass = mtiles * kBM;
    static constexpr int a_bytes = nmat * mtiles * kTileA;
    static constexpr int b_bytes = nmat * kTileB;
    static constexpr int t_bytes = nmat * kKT * tr_row<K>();
    static constexpr int a_stages = 2 * (64 / kBK);
    static constexpr int b_stages = kMergedRing ? a_stages : (MODE == 0 ? 2 : 3) * (64 / kBK);
    static constexpr int t_stages = (MODE == 0 ? 4 : 8) * (64 / kBK);
    static constexpr int a_off = 0;
    static constexpr int b_off = a_off + a_stages * a_bytes;
    static constexpr int t_off = b_off + b_stages * b_bytes;
    static constexpr int bar_off = t_off + t_stages * t_bytes;   // multiple of 1024
    static constexpr int n_bars = 2 * (a_stages + b_stages + t_stages) + 1;
    static constexpr int smem_bytes = bar_off + 1024 /* align */ + n_bars * 8 + 16;
    static_assert(smem_bytes <= 232448, "shared memory over the 227 KB per-block limit");
};

struct GemmParams {
    CUtensorMap tm_a;       // xt_g (gate/up) or xt_d (down): [rows][K] fp16
    CUtensorMap tm_b;       // xt_u (gate/up)
    const int4* passes;     // {expert, row_begin, rows, 0}
    const int* n_passes;
    const int64_t* tab_a;   // gate / down trellis addresses
    const int64_t* tab_b;   // up
    const __half* svh_a;    // gate/up: w13_svh [E][2][N]; down: w2_svh [E][N]
    const __half* suh_d;    // gate/up: w2_suh [E][N]
    __half* out;            // gate/up: xt_d [rows][N]; down: y [rows][N]
    RowPush push;           // down under expert-parallel push: where each row goes instead of out
    const float* rs;        // activation sums per sorted row: gate/up [2 rows] (gate, up); down [rows][K/128]
    float* xs_out;          // gate/up: block sums of the stored down inputs [rows][N/128]
    int* status;
    int K, N;
    float limit;
    uint32_t k16;
};

// ---------------------------------------------------------------------------------------------
// tcgen05 / TMA primitives
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t sw_desc(uint32_t saddr)
{
    // K-major swizzled canonical layout: 8-row atoms of kRowB-byte rows, atoms kAtom bytes apart;
    // layout type 2 = SWIZZLE_128B, 4 = SWIZZLE_64B (tcgen05 shared memory descriptor, version 1)
    constexpr uint64_t layout = kBK == 64 ? 2 : 4;
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(kAtom >> 4) << 32) |
           ((uint64_t)1 << 46) | (layout << 61);
}

// kind::f16, fp16 A/B, fp32 D, K-major A and B, N = 128, M = 128
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32])
{
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
        "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
        "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int c0, int c1, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
        : "memory");
}

// one 32-byte store (256-bit st.global on sm_100; `p` 32-byte aligned), not allocated in L1
__device__ __forceinline__ void st_global_32B(void* p, const uint32_t (&o)[8])
{
    asm volatile("st.global.L1::no_allocate.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(o[0]),
                 "r"(o[1]), "r"(o[2]), "r"(o[3]), "r"(o[4]), "r"(o[5]), "r"(o[6]), "r"(o[7])
                 : "memory");
}

__device__ __forceinline__ void stmatrix_x4(uint32_t addr, const uint32_t (&r)[4])
{
    asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3])
                 : "memory");
}

__device__ __forceinline__ void load_half8(const __half* p, float* dst)
{
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const __half2 h = u32_as_half2(w[q]);
        dst[2 * q] = __low2float(h);
        dst[2 * q + 1] = __high2float(h);
    }
}

// y = r16(H128(r16(y)) * HAD * svh), svh = 128 fp16 scales
__device__ __forceinline__ void out_block128(float (&v)[128], const __half* svh)
{
#pragma unroll
    for (int i = 0; i < 128; i += 2) r16x2(v[i], v[i + 1]);
    had128_thread(v);
#pragma unroll
    for (int c = 0; c < 16; ++c) {
        float s[8];
        load_half8(svh + c * 8, s);
#pragma unroll
        for (int q = 0; q < 8; ++q) v[c * 8 + q] = __fmul_rn(__fmul_rn(v[c * 8 + q], kHad), s[q]);
#pragma unroll
        for (int q = 0; q < 8; q += 2) r16x2(v[c * 8 + q], v[c * 8 + q + 1]);
    }
}

// gate/up epilogue of one row and one 128-feature block (accumulators at TMEM columns tg / tu of this
// thread's lane, sums of the affine weight codes times the inputs): g = KINV * acc_g + KBIAS * rsum[0]
// (the row's gate input sum; NULL for rows past the pass), likewise u; v = H128(fp16(act(out_block(g),
// out_block(u))) * suh_d) *
// HAD, the down-input row before its fp16 rounding. Intermediate blocks are parked in TMEM, 32 columns
// at a time, so no more than 128 + 64 values are live in registers.
__device__ __forceinline__ void gateup_epilogue(float (&v)[128], uint32_t tg, uint32_t tu, const __half* svg,
                                                const __half* svu, const __half* sd, float limit, const float* rsum)
{
#pragma unroll 1
    for (int m = 0; m < 2; ++m) {
        const uint32_t col = m ? tu : tg;
        const float bias = rsum ? kKbias * rsum[m] : 0.0f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float t[32];
            tmem_ld32(col + q * 32, t);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[q * 32 + i] = fmaf(kKinv, t[i], bias);
        }
        out_block128(v, m ? svu : svg);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float t[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] = v[q * 32 + i];
            tmem_st32(col + q * 32, t);
        }
    }
    // SwiGLU and the down-input scale, 32 columns at a time (into the gate columns)
#pragma unroll 1
    for (int q = 0; q < 4; ++q) {
        float g[32], uu[32];
        tmem_ld32(tg + q * 32, g);
        tmem_ld32(tu + q * 32, uu);
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
            float s8[8];
            load_half8(sd + q * 32 + c8 * 8, s8);
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                float a0 = act_gu(g[c8 * 8 + i], uu[c8 * 8 + i], limit);
                float a1 = act_gu(g[c8 * 8 + i + 1], uu[c8 * 8 + i + 1], limit);
                r16x2(a0, a1);
                g[c8 * 8 + i] = __fmul_rn(a0, s8[i]);
                g[c8 * 8 + i + 1] = __fmul_rn(a1, s8[i + 1]);
            }
        }
        tmem_st32(tg + q * 32, g);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        float t[32];
        tmem_ld32(tg + q * 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[q * 32 + i] = t[i];
    }
    had128_thread(v);
#pragma unroll
    for (int i = 0; i < 128; ++i) v[i] = __fmul_rn(v[i], kHad);
}

// the 128 accumulator columns of one block of this thread's lane
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float (&v)[128])
{
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        float t[32];
        tmem_ld32(taddr + q * 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[q * 32 + i] = t[i];
    }
}

// ---------------------------------------------------------------------------------------------
// kernel
// ---------------------------------------------------------------------------------------------
template <int MODE, int K>
__global__ void __launch_bounds__(kGemmThreads, 1) exl3_gemm_kernel(const __grid_constant__ GemmParams p)
{
    griddep_enter();
    using Cfg = GemmCfg<MODE, K>;
    constexpr int kTrRow = tr_row<K>();
    constexpr int AS = Cfg::a_stages, BS = Cfg::b_stages, TS = Cfg::t_stages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    uint8_t* smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::bar_off);
    uint64_t* a_full = bars;
    uint64_t* a_empty = a_full + AS;
    uint64_t* b_full = a_empty + AS;
    uint64_t* b_empty = b_full + BS;
    uint64_t* t_full = b_empty + BS;
    uint64_t* t_empty = t_full + TS;
    uint64_t* acc_full = t_empty + TS;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + Cfg::n_bars);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::n_bars) + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_fb = p.N / kBN;
    const int n_chunks = p.K / kBK;
    const int n_units = (*p.n_passes) * n_fb;
    const int ntile_row = p.N / 16;
    // no busy expert in this call (the usual decode case): leave before allocating TMEM
    if (n_units <= (int)blockIdx.x) return;

    if (threadIdx.x == 0) {
        for (int s = 0; s < AS; ++s) {
            mbar_init(&a_full[s], kMergedRing ? 1 + kDecWarps : 1);
            mbar_init(&a_empty[s], kIssuers);
        }
        for (int s = 0; s < BS; ++s) {
            mbar_init(&b_full[s], kDecWarps);
            mbar_init(&b_empty[s], 1);
        }
        for (int s = 0; s < TS; ++s) {
            mbar_init(&t_full[s], 1);
            mbar_init(&t_empty[s], kDecWarps);
        }
        mbar_init(acc_full, kIssuers);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kWarpMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto stage_a = [&](int s, int mat, int mt) { return smem + Cfg::a_off + s * Cfg::a_bytes + (mat * Cfg::mtiles + mt) * kTileA; };
    auto stage_b = [&](int s, int mat) { return smem + Cfg::b_off + s * Cfg::b_bytes + mat * kTileB; };
    auto stage_t = [&](int s, int mat, int kt) { return smem + Cfg::t_off + s * Cfg::t_bytes + (mat * kKT + kt) * kTrRow; };

    if (warp == kWarpA) {
        // ------------------------------ activation producer ------------------------------
        uint32_t it = 0;
        bool ok = true;
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tm_a)) : "memory");
            if (MODE == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tm_b)) : "memory");
            for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
                const int4 P = p.passes[u / n_fb];
                const int row0 = P.y, act_mt = (P.z + kBM - 1) / kBM;
                for (int c = 0; c < n_chunks; ++c, ++it) {
                    const int s = it % AS;
                    if (!mbar_wait_bounded(&a_empty[s], ((it / AS) & 1) ^ 1, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&a_full[s], Cfg::nmat * act_mt * kTileA);
                    for (int mat = 0; mat < Cfg::nmat; ++mat)
                        for (int mt = 0; mt < act_mt; ++mt)
                            tma_load_2d(stage_a(s, mat, mt), mat ? &p.tm_b : &p.tm_a, c * kBK, row0 + mt * kBM, &a_full[s]);
                }
            }
            // on abort, let the copies already issued land before the CTA exits
            for (uint32_t q = 1; !ok && q <= (it < (uint32_t)AS ? it : (uint32_t)AS); ++q) {
                const uint32_t j = it - q;
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(&a_full[j % AS], (j / AS) & 1) && globaltimer_ns() - t0 < kWaitLimitNs) {}
            }
        }
        __syncwarp();
    } else if (warp == kWarpT) {
        // ------------------------------ trellis producer ------------------------------
        uint32_t it = 0;
        bool ok = true;
        const uint64_t pol = l2_policy_evict_first();
        // lane l < nmat*kKT streams k-tile row l % kKT of matrix l / kKT. The words of a unit start at
        // unit_base(u); the per-chunk loop only adds offsets (the table lookups are dependent global loads
        // of several hundred ns each and would otherwise pace the whole ring).
        const bool lact = lane < Cfg::nmat * kKT;
        const int lmat = lane / kKT, lkt = lane % kKT;
        auto unit_base = [&](int u) -> const uint8_t* {
            if (!lact || u >= n_units) return nullptr;
            const int e = p.passes[u / n_fb].x, fb = u % n_fb;
            const int64_t base = lmat ? p.tab_b[e] : p.tab_a[e];
            return reinterpret_cast<const uint8_t*>(base) + (size_t)(fb * 8) * TileFmt<K>::bytes;
        };
        const size_t chunk_stride = (size_t)kKT * ntile_row * TileFmt<K>::bytes;
        const size_t lane_off = (size_t)lkt * ntile_row * TileFmt<K>::bytes;
        // L2 prefetch runs kTrPrefetch chunks ahead of the copies (into the next unit near the end),
        // so the ring's copies see L2 latency rather than HBM latency
        constexpr int kTrPrefetch = 16 * (64 / kBK);
        const uint8_t* cur = unit_base(blockIdx.x);
        const uint8_t* nxt = unit_base(blockIdx.x + gridDim.x);
        for (int c = 0; c < kTrPrefetch && c < n_chunks; ++c)
            if (cur) l2_prefetch_bulk(cur + c * chunk_stride + lane_off, kTrRow);
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
            for (int c = 0; c < n_chunks; ++c, ++it) {
                const int s = it % TS;
                {
                    const int cp = c + kTrPrefetch;
                    const uint8_t* q = cp < n_chunks ? cur : nxt;
                    const int cq = cp < n_chunks ? cp : cp - n_chunks;
                    if (q && cq < n_chunks) l2_prefetch_bulk(q + cq * chunk_stride + lane_off, kTrRow);
                }
                if (!mbar_wait_bounded(&t_empty[s], ((it / TS) & 1) ^ 1, abort_flag, p.status)) {
                    ok = false;
                    break;
                }
                if (lane == 0) mbar_arrive_expect_tx(&t_full[s], Cfg::t_bytes);
                __syncwarp();
                if (lact) bulk_g2s(stage_t(s, lmat, lkt), cur + c * chunk_stride + lane_off, kTrRow, &t_full[s], pol);
            }
            cur = nxt;
            nxt = unit_base(u + 2 * gridDim.x);
        }
        if (!ok && lane == 0) {
            for (uint32_t q = 1; q <= (it < (uint32_t)TS ? it : (uint32_t)TS); ++q) {
                const uint32_t j = it - q;
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(&t_full[j % TS], (j / TS) & 1) && globaltimer_ns() - t0 < kWaitLimitNs) {}
            }
        }
        __syncwarp();
    } else if (warp == kWarpMma || (kIssuers == 2 && warp == kWarpMma2)) {
        // ---------------------------------- MMA issuers ----------------------------------
        const int me = warp == kWarpMma ? 0 : 1;
        if (lane == 0) {
            uint32_t ia = 0, ib = 0;
            bool ok = true;
            // A single thread issues each accumulator's MMAs, so its per-MMA instruction count
            // matters: the descriptors of stage 0 are built once, and a stage / tile / k step only
            // adds its byte offset / 16 to the 14-bit start-address field (shared memory stays
            // below 256 KB, so the field never carries).
            const uint64_t adesc0 = sw_desc(smem_addr(smem + Cfg::a_off));
            const uint64_t bdesc0 = sw_desc(smem_addr(smem + Cfg::b_off));
            for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
                const int act_mt = (p.passes[u / n_fb].z + kBM - 1) / kBM;
                for (int c = 0; c < n_chunks; ++c, ++ia, ++ib) {
                    const int sa = ia % AS, sb = ib % BS;
                    if ((!kMergedRing && !mbar_wait_bounded(&b_full[sb], (ib / BS) & 1, abort_flag, p.status)) ||
                        !mbar_wait_bounded(&a_full[sa], (ia / AS) & 1, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad_s = adesc0 + (uint64_t)((sa * Cfg::a_bytes) >> 4);
                    const uint64_t bd_s = bdesc0 + (uint64_t)((sb * Cfg::b_bytes) >> 4);
                    const uint32_t acc0 = c > 0 ? 1u : 0u;
                    int issued = 0;
#pragma unroll
                    for (int mt = 0; mt < Cfg::mtiles; ++mt) {
                        if (mt >= act_mt) break;
#pragma unroll
                        for (int mat = 0; mat < Cfg::nmat; ++mat) {
                            if ((mt * Cfg::nmat + mat) % kIssuers != me) continue;
                            ++issued;
                            const uint32_t d = tmem + (uint32_t)((mt * Cfg::nmat + mat) * kBN);
                            const uint64_t ad = ad_s + (uint64_t)(((mat * Cfg::mtiles + mt) * kTileA) >> 4);
                            const uint64_t bd = bd_s + (uint64_t)((mat * kTileB) >> 4);
#pragma unroll
                            for (int kk = 0; kk < kBK / 16; ++kk)
                                umma_f16(d, ad + 2 * kk, bd + 2 * kk, kk ? 1u : acc0);
                        }
                    }
                    if (issued)
                        umma_commit(&a_empty[sa]);
                    else
                        mbar_arrive(&a_empty[sa]);   // nothing of this stage read by this issuer
                    if (!kMergedRing) umma_commit(&b_empty[sb]);
                }
                if (ok) umma_commit(acc_full);
            }
            // the last MMAs must finish before TMEM is released
            if (ib > 0) {
                const uint32_t j = ib - 1;
                const uint64_t t0 = globaltimer_ns();
                uint64_t* last = kMergedRing ? &a_empty[j % AS] : &b_empty[j % BS];
                while (!mbar_try_wait(last, (j / BS) & 1) && globaltimer_ns() - t0 < kWaitLimitNs) {}
            }
        }
        __syncwarp();
    } else if (warp >= kWarpDec0) {
        // ------------------------------- decoders + epilogue -------------------------------
        const int d = warp - kWarpDec0;               // 0..7
        const LaneDec<K> lw = lane_dec_setup<K>(lane);
        const uint32_t k16 = p.k16;
        // decode assignment: the chunk's nmat * kKT (matrix, k-tile) rows of 8 n-tiles are split
        // evenly over the 8 decoder warps (wpg warps per row, ntn adjacent n-tiles each)
        constexpr int wpg = kDecWarps / (Cfg::nmat * kKT);
        constexpr int ntn = 8 / wpg;
        const int grp = d / wpg;
        const int dmat = grp / kKT, dkt = grp % kKT;
        const int nt0 = (d % wpg) * ntn;
        // One stmatrix.x4 per tile stores the lane's four fragment registers: matrix q holds features
        // n = 8 (q >> 1) + 0..7 and k = 8 (q & 1) + 0..7 of the tile (register q of every lane, rows as
        // the mma fragment), and lane i gives the address of row i % 8 of matrix i / 8. In the swizzled
        // K-major operand, element (n, k) sits at (n/8)*kAtom + (n%8)*kRowB + ((k/8) ^ sw(n%8))*16 +
        // (k%8)*2, sw(r) = r for the 128-byte swizzle and r/2 for the 64-byte one, so each matrix row
        // is one 16-byte chunk.
        uint32_t soff;
        {
            const int q = lane >> 3, n = (lane & 7) + ((q >> 1) << 3);
            const int kc = dkt * 2 + (q & 1);   // 16-byte chunk index of the row within the stage
            const int sw = kBK == 64 ? (n & 7) : ((n & 7) >> 1);
            soff = (uint32_t)((n >> 3) * kAtom + (n & 7) * kRowB + ((kc ^ sw) * 16));
        }
        const int quarter = warp & 3;                 // TMEM lanes this warp may access
        uint32_t it = 0, ib = 0, units_done = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++units_done) {
            const int pass = u / n_fb, fb = u % n_fb;
            const int4 P = p.passes[pass];
            const int e = P.x, row0 = P.y, rows = P.z;
            for (int c = 0; c < n_chunks; ++c, ++it, ++ib) {
                const int st = it % TS, sb = ib % BS;
                if (!mbar_wait_bounded(&t_full[st], (it / TS) & 1, abort_flag, p.status) ||
                    !mbar_wait_bounded(kMergedRing ? &a_empty[sb] : &b_empty[sb], ((ib / BS) & 1) ^ 1, abort_flag,
                                       p.status)) {
                    ok = false;
                    break;
                }
                const uint32_t* trw = reinterpret_cast<const uint32_t*>(stage_t(st, dmat, dkt));
                const uint32_t bt = smem_addr(stage_b(sb, dmat) + nt0 * 2 * kAtom) + soff;
#if DSV41_GEMM_PAIRED && DSV41_CODES_WIN2
                if constexpr (K == 3 && ntn % DSV41_GEMM_PAIRED == 0) {
                    constexpr int NP = DSV41_GEMM_PAIRED == 1 ? 2 : DSV41_GEMM_PAIRED;   // tiles interleaved
#pragma unroll
                    for (int j = 0; j < ntn; j += NP) {
                        const uint32_t* tw = trw + (nt0 + j) * TileFmt<K>::words;
                        uint32_t b[NP][4];
                        decode_tiles_codes3<NP, DSV41_GEMM_IMAD_PACKS>(tw, lw, k16, b);
#pragma unroll
                        for (int n = 0; n < NP; ++n) stmatrix_x4(bt + (j + n) * 2 * kAtom, b[n]);
                    }
                } else
#endif
                {
#pragma unroll kDecUnroll
                for (int j = 0; j < ntn; ++j) {
                    const uint32_t* tw = trw + (nt0 + j) * TileFmt<K>::words;
                    uint32_t b[4];
                    decode_tile_codes<K, DSV41_GEMM_IMAD_PACKS>(tw, lw, k16, b);   // affine codes: the epilogue applies KINV, KBIAS
                    stmatrix_x4(bt + j * 2 * kAtom, b);
                }
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(kMergedRing ? &a_full[sb] : &b_full[sb]);
                    mbar_arrive(&t_empty[st]);
                }
            }
            if (!ok) break;
            // ------------------------------- epilogue -------------------------------
            // the unit's scale rows (128 fp16 each) into L1 while the last MMAs finish
            if (lane < 2 * (MODE == 0 ? 3 : 1)) {
                const int which = lane >> 1;
                const __half* sv = MODE == 0 ? (which == 2 ? p.suh_d + (size_t)e * p.N : p.svh_a + ((size_t)e * 2 + which) * p.N)
                                             : p.svh_a + (size_t)e * p.N;
                asm volatile("prefetch.global.L1 [%0];" ::"l"(sv + fb * kBN + (lane & 1) * 64));
            }
            if (!mbar_wait_bounded(acc_full, units_done & 1, abort_flag, p.status)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int ept = MODE == 0 ? 1 : 2;  // M tiles per warp
            for (int ei = 0; ei < ept; ++ei) {
                const int mt = MODE == 0 ? d / 4 : d / 4 + 2 * ei;
                const int row = mt * kBM + quarter * 32 + lane;
                const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
                if (mt * kBM >= rows) continue;  // whole M tile empty (warp-uniform)
                float v[128];
                // the row's input sum(s) of the affine form (rows past the pass are never stored)
                const bool live = row < rows;
                const size_t grow = (size_t)(row0 + row);
                __half* dst = nullptr;   // the row's 128 outputs (resolved while few registers are live)
                if (MODE == 0) {
                    const uint32_t colg = (uint32_t)((mt * 2 + 0) * kBN), colu = (uint32_t)((mt * 2 + 1) * kBN);
                    const __half* svg = p.svh_a + (size_t)e * 2 * p.N + fb * kBN;
                    gateup_epilogue(v, lane_addr + colg, lane_addr + colu, svg, svg + p.N,
                                    p.suh_d + (size_t)e * p.N + fb * kBN, p.limit, live ? p.rs + 2 * grow : nullptr);
                    dst = p.out + grow * p.N + fb * kBN;
                } else {
                    float xs = 0.0f;
                    if (live) {
                        for (int b = 0; b < p.K / 128; ++b) xs += p.rs[grow * (p.K / 128) + b];
                        dst = out_row(p.out, p.push, row0 + row, p.N) + fb * kBN;
                    }
                    tmem_ld128(lane_addr + (uint32_t)(mt * kBN), v);
#pragma unroll
                    for (int i = 0; i < 128; ++i) v[i] = fmaf(kKinv, v[i], kKbias * xs);
                    out_block128(v, p.svh_a + (size_t)e * p.N + fb * kBN);
                }
                if (live) {
                    // 256 B of the row as eight 32-byte stores (rows are 4-8 KB, blocks 256 B: 32-byte aligned)
                    float bs = 0.0f;   // gate/up: block sum of the stored down inputs (the down pass's affine form)
#pragma unroll
                    for (int c16 = 0; c16 < 8; ++c16) {
                        uint32_t o[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const __half2 h = __floats2half2_rn(v[c16 * 16 + 2 * j], v[c16 * 16 + 2 * j + 1]);
                            if (MODE == 0) bs += __low2float(h) + __high2float(h);
                            o[j] = half2_as_u32(h);
                        }
                        if (MODE == 1 && p.push.route) {
                            // a peer's receive slot: 16-byte stores over NVLink
                            *reinterpret_cast<uint4*>(dst + c16 * 16) = make_uint4(o[0], o[1], o[2], o[3]);
                            *reinterpret_cast<uint4*>(dst + c16 * 16 + 8) = make_uint4(o[4], o[5], o[6], o[7]);
                        } else {
                            st_global_32B(dst + c16 * 16, o);
                        }
                    }
                    if (MODE == 0) p.xs_out[grow * (p.N / kBN) + fb] = bs;
                }
            }
            tc_fence_before();
        }
    }
    // output rows stored into peers' memory are visible at system scope before the kernel ends
    if (MODE == 1 && p.push.route) __threadfence_system();
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// ---------------------------------------------------------------------------------------------
// plan: row passes of the busy experts (gate/up 256 rows, down 512 rows)
// ---------------------------------------------------------------------------------------------
__global__ void gemm_plan_kernel(const int* fat_experts, const int* n_fat, const int* counts, const int* offsets,
                                 int rp0, int rp1, int4* passes0, int* n0, int4* passes1, int* n1)
{
    griddep_enter();
    if (threadIdx.x != 0) return;
    const int nf = *n_fat;
    int a = 0, b = 0;
    for (int i = 0; i < nf; ++i) {
        const int e = fat_experts[i], R = counts[e], r0 = offsets[e];
        for (int r = 0; r < R; r += rp0) passes0[a++] = make_int4(e, r0 + r, min(rp0, R - r), 0);
        for (int r = 0; r < R; r += rp1) passes1[b++] = make_int4(e, r0 + r, min(rp1, R - r), 0);
    }
    *n0 = a;
    *n1 = b;
}

// passes = sum over busy experts of ceil(rows / rp) <= N / rp + (number of experts, <= min(N, kMaxExperts))
static int max_passes(int N, int /*E*/, int rp) { return N / rp + (N < kMaxExperts ? N : kMaxExperts) + 1; }

static size_t pass_list_bytes(int N, int E)
{
    return (size_t)(max_passes(N, E, GemmCfg<0, 3>::rows_per_pass) + max_passes(N, E, GemmCfg<1, 3>::rows_per_pass)) * 16;
}

size_t gemm_scratch_bytes(int N, int E, int H, int I)
{
    const size_t n = (size_t)(N > 0 ? N : 1);
    return 256 + pass_list_bytes(N, E) + (2 * n + n * (size_t)(I / 128)) * 4;
}

float* gemm_row_sums(uint8_t* scratch, int N, int E)
{
    return reinterpret_cast<float*>(scratch + 256 + pass_list_bytes(N, E));
}

float* gemm_down_sums(uint8_t* scratch, int N, int E)
{
    return gemm_row_sums(scratch, N, E) + 2 * (size_t)(N > 0 ? N : 1);
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// [rows][K] fp16 rows, box kBK (k) x 128 (rows), swizzle matching the descriptors, zero fill out of bounds
static cudaError_t make_map(CUtensorMap* m, const void* base, int rows, int K)
{
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)(rows > 0 ? rows : 1)};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
    const CUtensorMapSwizzle swz = kBK == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int MODE, int K>
static cudaError_t launch_mode(const GemmArgs& a, cudaStream_t st)
{
    using Cfg = GemmCfg<MODE, K>;
    const int H = a.layer->hidden, I = a.layer->intermediate, E = a.layer->num_experts;
    const int N = a.rows_bound;
    int4* passes0 = reinterpret_cast<int4*>(a.scratch + 256);
    int4* passes1 = passes0 + max_passes(N, E, GemmCfg<0, 3>::rows_per_pass);
    int* counters = reinterpret_cast<int*>(a.scratch);
    cudaError_t err;
    if (MODE == 0) {
        const int rp0 = GemmCfg<0, K>::rows_per_pass, rp1 = GemmCfg<1, K>::rows_per_pass;
        if ((err = launch_k(gemm_plan_kernel, 1, 32, 0, st, a.fat_experts, a.n_fat, a.counts, a.offsets, rp0, rp1,
                            passes0, counters, passes1, counters + 1)) != cudaSuccess)
            return err;
    }
    GemmParams p{};
    if (MODE == 0) {
        if ((err = make_map(&p.tm_a, a.xt_g, N, H)) != cudaSuccess) return err;
        if ((err = make_map(&p.tm_b, a.xt_u, N, H)) != cudaSuccess) return err;
        p.passes = passes0;
        p.n_passes = counters;
        p.tab_a = a.layer->gate_ptrs;
        p.tab_b = a.layer->up_ptrs;
        p.svh_a = static_cast<const __half*>(a.layer->w13_svh);
        p.suh_d = static_cast<const __half*>(a.layer->w2_suh);
        p.out = a.xt_d;
        p.rs = gemm_row_sums(a.scratch, N, E);
        p.xs_out = gemm_down_sums(a.scratch, N, E);
        p.K = H;
        p.N = I;
    } else {
        if ((err = make_map(&p.tm_a, a.xt_d, N, I)) != cudaSuccess) return err;
        p.tm_b = p.tm_a;
        p.passes = passes1;
        p.n_passes = counters + 1;
        p.tab_a = a.layer->down_ptrs;
        p.tab_b = nullptr;
        p.svh_a = static_cast<const __half*>(a.layer->w2_svh);
        p.suh_d = nullptr;
        p.out = a.y;
        p.push = a.push;
        p.rs = gemm_down_sums(a.scratch, N, E);
        p.xs_out = nullptr;
        p.K = I;
        p.N = H;
    }
    p.status = a.status;
    p.limit = a.limit;
    p.k16 = 65536u;
    const size_t smem = Cfg::smem_bytes;
    if ((err = cudaFuncSetAttribute((const void*)exl3_gemm_kernel<MODE, K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem)) != cudaSuccess)
        return err;
    const int units_bound = max_passes(N, E, Cfg::rows_per_pass) * (p.N / kBN);
    int grid = num_sms();
    if (units_bound < grid) grid = units_bound;
    if (grid < 1) grid = 1;
    return launch_k(exl3_gemm_kernel<MODE, K>, grid, kGemmThreads, smem, st, p);
}

static int args_bits(const GemmArgs& a) { return a.layer->bits ? a.layer->bits : 3; }

cudaError_t launch_gemm_gateup(const GemmArgs& a, cudaStream_t st)
{
    const int b = args_bits(a);
    return b == 2 ? launch_mode<0, 2>(a, st) : b == 4 ? launch_mode<0, 4>(a, st) : launch_mode<0, 3>(a, st);
}
cudaError_t launch_gemm_down(const GemmArgs& a, cudaStream_t st)
{
    const int b = args_bits(a);
    return b == 2 ? launch_mode<1, 2>(a, st) : b == 4 ? launch_mode<1, 4>(a, st) : launch_mode<1, 3>(a, st);
}

}  // namespace dsv41
