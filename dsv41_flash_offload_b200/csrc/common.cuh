// Shared device helpers for the EXL3 mul1 K=3 MoE kernels (sm_100a).
//
// Format (restated from the reference's kernels/cpu_avx2/ft_core.h:28-83, which mirrors
// exllamav3's GPU decode): a 16x16 weight tile is a circular 768-bit stream (96 bytes = 24
// little-endian 32-bit words, read MSB-first). Symbol i's 16-bit state is the stream window
// ending at bit 3i+2; its weight is fp16(fma(1024 + bytesum(state * 0x83DCD12D), KINV, KBIAS)).
// Symbols 8t..8t+7 belong to tensor-core fragment lane t, laid out exactly as the B operand of
// mma.m16n8k16 (rows k = 2(t%4)+{0,1,8,9}, cols n = t/4 and t/4+8), so each lane decodes its own
// B fragments in registers and the decoded weights never touch memory.
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dsv41 {

constexpr uint32_t kMul1 = 0x83DCD12Du;
constexpr float kHad = 0.088388347648f;  // 2^-3.5
constexpr int kTileBytes = 96;
constexpr int kTileWords = 24;
constexpr uint16_t kKinvBits = 0x1eee;
constexpr uint16_t kKbiasBits = 0xc931;

// status word codes written by kernels (never a trap)
enum : int { kStatusOk = 0, kStatusWaitTimeout = 1, kStatusBadShape = 2, kStatusRouteCapacity = 3 };

// ------------------------------------------------------------------------------------------
// decode
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ __half2 u32_as_half2(uint32_t v)
{
    __half2 h;
    *reinterpret_cast<uint32_t*>(&h) = v;
    return h;
}
__device__ __forceinline__ uint32_t half2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// one state -> 0x6400 + bytesum(state * MUL1) = the fp16 bit pattern of (1024 + s) (s <= 1020)
__device__ __forceinline__ uint32_t state_code(uint32_t st)
{
    return __dp4a(st * kMul1, 0x01010101u, 0x6400u);
}

// ------------------------------------------------------------------------------------------
// Pipe-balanced decode (used by the GEMV kernels). Lane t's 8 states all lie in the 64 stream bits
// that start at stream byte 3t-4 (mod 96): with that window in (hi, lo), state j is bits
// [29-3j, 45-3j) for every lane, so all shifts are immediates. The window is assembled from three
// words with two funnel shifts by 8*(byte offset % 4).
//
// Measured on B200 (sm_100a, one SM, independent chains): IMAD, DP4A and HFMA2 share one pipe at
// half rate (16 lanes/clk per SM sub-partition); SHF, LOP3 and PRMT share another at half rate;
// the two co-issue; mul.hi and bfe run at quarter rate. Per lane and tile the decode below issues
// IMAD x8 + DP4A x8 + HFMA2 x4 + IMAD x1 (one half2 pack) on the first pipe and funnel/shift x9 +
// LOP3 x7 + PRMT x4 (state 7 is byte aligned: one PRMT extracts it; three half2 packs) on the
// second, about 21 each. `k16` must be the run-time value 65536 so the pack stays an IMAD.
// ------------------------------------------------------------------------------------------
struct LaneWindow {
    int q0, q1, q2;  // word indices of the window
    uint32_t r8;     // left funnel shift (0, 8, 16, 24)
};

__device__ __forceinline__ LaneWindow lane_window_setup(int t)
{
    const int b0 = (3 * t - 4 + 96) % 96;
    LaneWindow w;
    w.q0 = b0 >> 2;
    w.q1 = (w.q0 + 1) % kTileWords;
    w.q2 = (w.q0 + 2) % kTileWords;
    w.r8 = 8u * (uint32_t)(b0 & 3);
    return w;
}

__device__ __forceinline__ void decode_lane_u(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t r8, uint32_t k16,
                                              uint32_t (&b)[4])
{
    const uint32_t hi = __funnelshift_l(w1, w0, r8);
    const uint32_t lo = __funnelshift_l(w2, w1, r8);
    uint32_t s[8];
#pragma unroll
    for (int j = 0; j < 5; ++j) s[j] = __funnelshift_r(lo, hi, 29 - 3 * j) & 0xffffu;
    s[5] = (lo >> 14) & 0xffffu;
    s[6] = (lo >> 11) & 0xffffu;
    s[7] = __byte_perm(lo, 0u, 0x4421);  // bits [8, 24): bytes 1, 2 of lo, zero above
    const __half2 kinv = u32_as_half2((uint32_t)kKinvBits * 0x10001u);
    const __half2 kbias = u32_as_half2((uint32_t)kKbiasBits * 0x10001u);
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
        const uint32_t c0 = state_code(s[j]), c1 = state_code(s[j + 1]);
        const uint32_t c = (j == 0) ? c1 * k16 + c0 : __byte_perm(c0, c1, 0x5410);
        b[j >> 1] = half2_as_u32(__hfma2(u32_as_half2(c), kinv, kbias));
    }
}

// ------------------------------------------------------------------------------------------
// Bits per weight K = 2, 3, 4. A tile is 16*K int16 words = 32*K bytes, a circular 256*K-bit stream
// whose symbol i state is the 16-bit window ending at stream bit K*i+K-1 (the reference's
// BITS-generic state_scalar, ft_core.h:63-73). K = 3 uses the lane-uniform window above; for
// K = 4 and 2 lane t's 8 states lie in two consecutive 32-bit words (a, b):
//   K = 4: a = t-1, b = t (mod 32); state j = bits [28-4j, 44-4j) of (word a : word b)
//   K = 2: a = t/2-1, b = t/2 (mod 16); state j = bits [s0-2j, s0-2j+16), s0 = 30 (even t) or
//          14 (odd t)
// so every state is one funnel shift (by less than 32) and a 16-bit mask.
// ------------------------------------------------------------------------------------------
template <int K>
struct TileFmt {
    static_assert(K == 2 || K == 3 || K == 4, "2, 3 or 4 bits per weight");
    static constexpr int bytes = 32 * K;
    static constexpr int words = 8 * K;
};

template <int K>
struct LaneDec {
    int q0, q1, q2;
    uint32_t r;   // K = 3: left funnel shift of the window; K = 2, 4: shift of state 0
    int c0, c1;   // K = 3, affine codes: the two words that hold the lane's 37 stream bits
    uint32_t cs;  //                      and the right shift that puts them at bits [0, 37)
};

template <int K>
__device__ __forceinline__ LaneDec<K> lane_dec_setup(int t)
{
    LaneDec<K> d;
    if constexpr (K == 3) {
        const LaneWindow w = lane_window_setup(t);
        d.q0 = w.q0;
        d.q1 = w.q1;
        d.q2 = w.q2;
        d.r = w.r8;
        // lane t's 8 states cover stream bits [24t - 13, 24t + 24) (mod 768): 37 bits starting at bit
        // p = (24t - 13) mod 32 of word a, and p is 3, 11, 19 or 27, so they always lie in words a, a + 1
        const int sb = (24 * t - 13 + 768) % 768;
        d.c0 = sb >> 5;
        d.c1 = (d.c0 + 1) % kTileWords;
        d.cs = 27u - (uint32_t)(sb & 31);
    } else if constexpr (K == 4) {
        d.q0 = (t + 31) & 31;
        d.q1 = t;
        d.q2 = 0;
        d.r = 28;
    } else {
        d.q0 = ((t >> 1) + 15) & 15;
        d.q1 = t >> 1;
        d.q2 = 0;
        d.r = (t & 1) ? 14u : 30u;
    }
    return d;
}

// this lane's 8 weights of the tile at `tw` as 4 half2 mma B-fragment registers (bit-exact)
template <int K>
__device__ __forceinline__ void decode_tile(const uint32_t* tw, const LaneDec<K>& d, uint32_t k16, uint32_t (&b)[4])
{
    if constexpr (K == 3) {
        decode_lane_u(tw[d.q0], tw[d.q1], tw[d.q2], d.r, k16, b);
    } else {
        const uint32_t hi = tw[d.q0], lo = tw[d.q1];
        const __half2 kinv = u32_as_half2((uint32_t)kKinvBits * 0x10001u);
        const __half2 kbias = u32_as_half2((uint32_t)kKbiasBits * 0x10001u);
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
            const uint32_t s0 = __funnelshift_r(lo, hi, d.r - K * j) & 0xffffu;
            const uint32_t s1 = __funnelshift_r(lo, hi, d.r - K * (j + 1)) & 0xffffu;
            const uint32_t c0 = state_code(s0), c1 = state_code(s1);
            const uint32_t c = (j == 0) ? c1 * k16 + c0 : __byte_perm(c0, c1, 0x5410);
            b[j >> 1] = half2_as_u32(__hfma2(u32_as_half2(c), kinv, kbias));
        }
    }
}

// ------------------------------------------------------------------------------------------
// Affine form of the same decode (the reference CPU tier's AFFINE mode, ft_core.h:293 and its
// mode choice :936): w = KINV * code + KBIAS with code = 1024 + bytesum, so for any activations x
//   sum_k w_k x_k = KINV * sum_k code_k x_k + KBIAS * sum_k x_k   (exact in real arithmetic).
// The fragments then carry the codes themselves (fp16 1024..2044, exact) and the per-weight
// HFMA2 is gone; the caller applies KINV / KBIAS to the fp32 sums. It skips only the fp16 rounding
// of each weight (a half-ulp, 2^-11 relative). `kImadPacks` of the 4 half2 packs per lane go to the
// IMAD pipe (c1 * 65536 + c0), the rest to PRMT, to balance the two integer pipes.
// ------------------------------------------------------------------------------------------
#ifndef DSV41_CODES_WIN2
#define DSV41_CODES_WIN2 1   // K = 3 codes: the lane's states from two staged words (1: two loads, 0: three)
#endif
constexpr float kKinv = 0.00676727294921875f;   // fp16 0x1eee = 1774 * 2^-18 (exact)
constexpr float kKbias = -10.3828125f;          // fp16 0xc931 = -1329 * 2^-7 (exact)

template <int K, int kImadPacks = 2>
__device__ __forceinline__ void decode_tile_codes(const uint32_t* tw, const LaneDec<K>& d, uint32_t k16,
                                                  uint32_t (&b)[4])
{
    uint32_t s[8];
    if constexpr (K == 3) {
#if DSV41_CODES_WIN2
        // two words (MSB-first: word c0 is the high half), shifted right by cs: the lane's 37 bits at
        // [0, 37) of (hi:lo), state j at bits [21 - 3j, 37 - 3j) for every lane
        const uint32_t w0 = tw[d.c0], w1 = tw[d.c1];
        const uint32_t hi = w0 >> d.cs;
        const uint32_t lo = __funnelshift_r(w1, w0, d.cs);
        s[0] = __funnelshift_r(lo, hi, 21) & 0xffffu;
        s[1] = __funnelshift_r(lo, hi, 18) & 0xffffu;
#pragma unroll
        for (int j = 2; j < 7; ++j) s[j] = (lo >> (21 - 3 * j)) & 0xffffu;
        s[7] = lo & 0xffffu;
#else
        const uint32_t hi = __funnelshift_l(tw[d.q1], tw[d.q0], d.r);
        const uint32_t lo = __funnelshift_l(tw[d.q2], tw[d.q1], d.r);
#pragma unroll
        for (int j = 0; j < 5; ++j) s[j] = __funnelshift_r(lo, hi, 29 - 3 * j) & 0xffffu;
        s[5] = (lo >> 14) & 0xffffu;
        s[6] = (lo >> 11) & 0xffffu;
        s[7] = __byte_perm(lo, 0u, 0x4421);
#endif
    } else {
        const uint32_t hi = tw[d.q0], lo = tw[d.q1];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j] = __funnelshift_r(lo, hi, d.r - K * j) & 0xffffu;
    }
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
        const uint32_t c0 = state_code(s[j]), c1 = state_code(s[j + 1]);
        b[j >> 1] = (j / 2 < kImadPacks) ? c1 * k16 + c0 : __byte_perm(c0, c1, 0x5410);
    }
}

// Several tiles' codes with the extraction of one state and the codes of the previous state interleaved
// across the tiles at the source level (K = 3, two-word window): the shift/mask pipe and the IMAD/DP4A pipe
// get work from every tile in turn. Measured on B200: two tiles per call, decode T=64 GEMV 1.540 -> 1.523 ms,
// busy-expert gate/up GEMM ~2% faster; four or eight tiles per call in the GEMM, or two k-rows' tiles in the
// GEMV, slower (register pressure).
// N consecutive n-tiles of one k-row (96 bytes apart)
template <int N, int kImadPacks>
__device__ __forceinline__ void decode_tiles_codes3(const uint32_t* tw, const LaneDec<3>& d, uint32_t k16,
                                                    uint32_t (&b)[N][4])
{
    uint32_t hi[N], lo[N], c[N][8];
#pragma unroll
    for (int n = 0; n < N; ++n) {
        const uint32_t w0 = tw[n * kTileWords + d.c0], w1 = tw[n * kTileWords + d.c1];
        hi[n] = w0 >> d.cs;
        lo[n] = __funnelshift_r(w1, w0, d.cs);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int n = 0; n < N; ++n) {
            uint32_t st;
            if (j < 2)
                st = __funnelshift_r(lo[n], hi[n], 21 - 3 * j) & 0xffffu;
            else if (j < 7)
                st = (lo[n] >> (21 - 3 * j)) & 0xffffu;
            else
                st = lo[n] & 0xffffu;
            c[n][j] = state_code(st);
        }
#pragma unroll
    for (int n = 0; n < N; ++n)
#pragma unroll
        for (int j = 0; j < 8; j += 2)
            b[n][j >> 1] = (j / 2 < kImadPacks) ? c[n][j + 1] * k16 + c[n][j] : __byte_perm(c[n][j], c[n][j + 1], 0x5410);
}

// ------------------------------------------------------------------------------------------
// fp16 rounding helper and the 128-point Walsh-Hadamard transform over a warp
// (lane holds elements lane*4 + q, q = 0..3; stage order w = 1, 2, 4, ..., 64 as the reference's
// had128, ft_core.h:89-94, so every fp32 intermediate is the same)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ float r16(float f) { return __half2float(__float2half_rn(f)); }
// the same rounding of two values through one packed f32x2 -> f16x2 conversion
__device__ __forceinline__ void r16x2(float& a, float& b)
{
    const float2 f = __half22float2(__floats2half2_rn(a, b));
    a = f.x;
    b = f.y;
}

__device__ __forceinline__ void had128_warp(float (&v)[4], int lane)
{
    float a = v[0], b = v[1];
    v[0] = a + b; v[1] = a - b;
    a = v[2]; b = v[3];
    v[2] = a + b; v[3] = a - b;
    a = v[0]; b = v[2];
    v[0] = a + b; v[2] = a - b;
    a = v[1]; b = v[3];
    v[1] = a + b; v[3] = a - b;
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const bool upper = (lane & m) != 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float p = __shfl_xor_sync(0xffffffffu, v[q], m);
            v[q] = upper ? (p - v[q]) : (v[q] + p);
        }
    }
}

// 128-point Hadamard of one row held by one thread, stage order w = 1..64 (ft_core.h:89-94)
__device__ __forceinline__ void had128_thread(float (&v)[128])
{
#pragma unroll
    for (int w = 1; w < 128; w <<= 1)
#pragma unroll
        for (int b = 0; b < 128; b += 2 * w)
#pragma unroll
            for (int i = b; i < b + w; ++i) {
                const float p = v[i], q = v[i + w];
                v[i] = p + q;
                v[i + w] = p - q;
            }
}

// 1: silu's exp and division use the hardware exp2 / reciprocal approximations (a few fp32 ulp from
// the libm expf and IEEE division of the reference's CPU tier, before the result is rounded to fp16;
// the layer tolerance is 2e-2 max-abs / cosine 0.9999). Measured on B200: the busy-expert epilogue's
// SwiGLU step drops from ~18k to ~7.4k cycles per 128-feature block. 0: the exact library forms.
#ifndef DSV41_FAST_ACT
#define DSV41_FAST_ACT 1
#endif
// silu(g) with the reference's clamp (u to [-L, L], silu from above; L = 0 disables),
// ft_core.h:123-133
__device__ __forceinline__ float act_gu(float g, float u, float limit)
{
#if DSV41_FAST_ACT
    float s = __fdividef(g, 1.0f + __expf(-g));
#else
    float s = g / (1.0f + expf(-g));
#endif
    if (limit != 0.0f) {
        u = fminf(fmaxf(u, -limit), limit);
        s = fminf(s, limit);
    }
    return __fmul_rn(s, u);
}

// 4-element row loads/stores (fp16 storage; inputs of any of the three ABI dtypes rounded to fp16)
__device__ __forceinline__ void load4_as_half(const void* x, int dtype, size_t idx, float (&v)[4])
{
    if (dtype == 0) {
        const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __half*>(x) + idx);
        const __half2 a = u32_as_half2(u.x), b = u32_as_half2(u.y);
        v[0] = __low2float(a); v[1] = __high2float(a); v[2] = __low2float(b); v[3] = __high2float(b);
    } else if (dtype == 1) {
        const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(x) + idx);
        v[0] = __uint_as_float(u.x << 16); v[1] = __uint_as_float(u.x & 0xffff0000u);
        v[2] = __uint_as_float(u.y << 16); v[3] = __uint_as_float(u.y & 0xffff0000u);
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = r16(v[q]);
    } else {
        const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + idx);
        v[0] = r16(f.x); v[1] = r16(f.y); v[2] = r16(f.z); v[3] = r16(f.w);
    }
}

__device__ __forceinline__ void load4_half(const __half* p, float (&v)[4])
{
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __half2 a = u32_as_half2(u.x), b = u32_as_half2(u.y);
    v[0] = __low2float(a); v[1] = __high2float(a); v[2] = __low2float(b); v[3] = __high2float(b);
}

__device__ __forceinline__ void store4_half(__half* p, const float (&v)[4])
{
    uint2 u;
    u.x = half2_as_u32(__floats2half2_rn(v[0], v[1]));
    u.y = half2_as_u32(__floats2half2_rn(v[2], v[3]));
    *reinterpret_cast<uint2*>(p) = u;
}

// ------------------------------------------------------------------------------------------
// async copy / mbarrier primitives (bounded waits: a wait that runs out records a status code
// and returns false; it never traps)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// The same test, but a thread whose phase is not complete may be suspended in hardware until the
// phase completes or about `hint_ns` have passed. A suspended warp issues nothing, so a waiting
// producer / MMA / consumer warp leaves the sub-partition's issue slots to the warps that decode
// (measured: the plain try_wait polling loop cost ~0.7 try_waits per decoded tile in the GEMV and
// ~4 in the GEMM, with their branches and yields around them).
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s, as the reference's combine wait

// programmatic dependent launch (see launch_k in internal.h): wait for the preceding grid on the stream
// (a no-op for a kernel launched without the attribute), then let the next grid be scheduled
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void griddep_enter()
{
    griddep_wait();
    griddep_launch_dependents();
}
#ifndef DSV41_WAIT_HINT_NS
#define DSV41_WAIT_HINT_NS 20000   // suspend hint of one try_wait (0: poll without suspending)
#endif

// Wait for phase `parity` of `bar`. Returns false (and records kStatusWaitTimeout) if it has
// not completed within `limit_ns` (default kWaitLimitNs) or if `abort_flag` is already set.
// Each retry may sleep up to DSV41_WAIT_HINT_NS in hardware, so the limit and the abort flag are
// checked after every retry; a wait therefore ends at most one hint after its limit.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                                  uint64_t limit_ns = kWaitLimitNs)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
#if DSV41_WAIT_HINT_NS > 0
        if (mbar_try_wait_hint(bar, parity, DSV41_WAIT_HINT_NS)) return true;
        {
#else
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0) {
#endif
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > limit_ns) {
                *abort_flag = 1;
                if (status) atomicExch(status, kStatusWaitTimeout);
                return false;
            }
        }
    }
}

// 1-D bulk async copy global -> this CTA's shared memory, completing on an mbarrier
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}
// bring `bytes` (multiple of 16, 16-byte aligned) of global memory into L2, no completion tracking
__device__ __forceinline__ void l2_prefetch_bulk(const void* src, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&a)[4], uint32_t addr)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
                 : "r"(addr));
}

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace dsv41
