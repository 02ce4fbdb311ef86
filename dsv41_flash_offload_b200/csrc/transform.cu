// Row transforms and the weighted combine.
//
// prep:    xt = fp16(H128(fp16(x) * suh) * 2^-3.5) per 128-block, for gate and up of the row's
//          expert (kernels/cpu_avx2/ft_core.h:96-102 prep_block; the fp16 cast of the hidden
//          states is apply_exl3_fused_moe's x2d.half(), patches/vllm-exl3-host-dma.patch:224).
// combine: out[t] = sum_j w[t, j] * y[route(t, j)] in fp32, routes in topk order
//          (ft_core.h:686-696 / :929-930, the weighted accumulate; ct/ft_tier_cu_v.cu:103-127).
// decode:  dense fp16 W from trellis, one warp per tile (ft_core.h:977-992 dense_weights).
#include "common.cuh"
#include "internal.h"

namespace dsv41 {

// 8 consecutive columns of row `idx` (any of the three ABI dtypes) rounded to fp16, as floats
__device__ __forceinline__ void load8_as_half(const void* x, int dtype, size_t idx, float (&v)[8])
{
    if (dtype == 2) {
        const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + idx);
        const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + idx + 4);
        v[0] = r16(a.x); v[1] = r16(a.y); v[2] = r16(a.z); v[3] = r16(a.w);
        v[4] = r16(b.x); v[5] = r16(b.y); v[6] = r16(b.z); v[7] = r16(b.w);
        return;
    }
    const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + idx);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        if (dtype == 0) {
            const __half2 h = u32_as_half2(w[q]);
            v[2 * q] = __low2float(h);
            v[2 * q + 1] = __high2float(h);
        } else {
            v[2 * q] = r16(__uint_as_float(w[q] << 16));
            v[2 * q + 1] = r16(__uint_as_float(w[q] & 0xffff0000u));
        }
    }
}

__device__ __forceinline__ void load8_half(const __half* p, float (&v)[8])
{
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const __half2 h = u32_as_half2(w[q]);
        v[2 * q] = __low2float(h);
        v[2 * q + 1] = __high2float(h);
    }
}

__device__ __forceinline__ void store8_half(__half* p, const float (&v)[8])
{
    uint4 u;
    u.x = half2_as_u32(__floats2half2_rn(v[0], v[1]));
    u.y = half2_as_u32(__floats2half2_rn(v[2], v[3]));
    u.z = half2_as_u32(__floats2half2_rn(v[4], v[5]));
    u.w = half2_as_u32(__floats2half2_rn(v[6], v[7]));
    *reinterpret_cast<uint4*>(p) = u;
}

// 128-point Hadamard of one block held by L lanes x 128/L consecutive values (element (128/L)*hl + q):
// stages w = 1 .. 64/L inside the thread, then w = 128/L .. 64 across lanes hl ^ 1, hl ^ 2, ... -- the
// same pairs and order as the reference's had128 (ft_core.h:89-94), log2(L) of the 7 stages on the
// shuffle unit
template <int L>
__device__ __forceinline__ void had128_lanes(float (&v)[128 / L], int hl)
{
    constexpr int V = 128 / L;
#pragma unroll
    for (int w = 1; w < V; w <<= 1)
#pragma unroll
        for (int b = 0; b < V; b += 2 * w)
#pragma unroll
            for (int i = b; i < b + w; ++i) {
                const float a = v[i], c = v[i + w];
                v[i] = a + c;
                v[i + w] = a - c;
            }
#pragma unroll
    for (int m = 1; m < L; m <<= 1) {
        // lower element: v + partner; upper: partner - v -- one FFMA with +-1 rounds exactly as the add
        const float sg = (hl & m) ? -1.0f : 1.0f;
#pragma unroll
        for (int q = 0; q < V; ++q) {
            const float pv = __shfl_xor_sync(0xffffffffu, v[q], m);
            v[q] = fmaf(sg, v[q], pv);
        }
    }
}

// one warp per sorted row p (rows p < *nrows; rows whose expert_sorted entry is negative are skipped):
// lanes L*g .. L*g+L-1 transform 128-block (32/L)*j + g of the row for gate and up,
//   xt_{g,u}[p] = fp16(H128(fp16(x[token]) * suh_{g,u}) * 2^-3.5)
// with 16-byte loads and stores; the row's indices are read once. With rsum, it also writes the sums of
// the stored (fp16) values of the row, rsum[2p] (gate) and rsum[2p + 1] (up), in fp32 in a fixed order:
// the activation sums of the busy-expert GEMM's affine weight codes.
#ifndef DSV41_PREP_LANES
#define DSV41_PREP_LANES 8        // lanes per 128-block (4: 32 values per lane; 8: 16 values, fewer registers)
#endif
#ifndef DSV41_PREP_MIN_BLOCKS
#define DSV41_PREP_MIN_BLOCKS 4   // resident blocks per SM (measured on the 16k prefill: 4 lanes x 2 blocks 1.07 ms, 8 x 3 0.93, 8 x 4 0.87)
#endif
constexpr int kPrepLanes = DSV41_PREP_LANES;
// CTA_ROW: one CTA per sorted row, its 8 warps splitting the row's 128-blocks (calls with few rows: decode
// batches; measured at T=64 22.7 -> 11.6 us, T=1 18.7 -> 8.3 us); otherwise one warp per row (the prefill:
// 0.89 ms at 16k tokens against 1.02 ms for the CTA form)
template <bool CTA_ROW>
__global__ void __launch_bounds__(256, DSV41_PREP_MIN_BLOCKS)
    prep_kernel(const __grid_constant__ XRows x, int x_dtype, const int* token_sorted, const int* expert_sorted,
                const int* nrows, const __half* w13_suh, int H, __half* xt_g, __half* xt_u, float* rsum)
{
    griddep_enter();
    constexpr int L = kPrepLanes, V = 128 / L, BPW = 32 / L;   // lanes per block, values per lane, blocks per warp
    const int lane = threadIdx.x & 31, hl = lane % L, g = lane / L;
    const int nvalid = *nrows;
    const int nb = H / 128;
    // CTA_ROW: warp w transforms blocks BPW * (w + 8 j) + g of the CTA's row, and the row sums of the 8
    // warps are added in warp order through shared memory
    __shared__ float wsum[8][2];
    const int warp = threadIdx.x >> 5;
    const int nit = CTA_ROW ? (nb + 8 * BPW - 1) / (8 * BPW) : (nb + BPW - 1) / BPW;
    const int p0 = CTA_ROW ? (int)blockIdx.x : (int)(blockIdx.x * (blockDim.x >> 5) + warp);
    const int pstride = CTA_ROW ? (int)gridDim.x : (int)(gridDim.x * (blockDim.x >> 5));
    for (int p = p0; p < nvalid; p += pstride) {
        const int e = expert_sorted[p];
        if (e < 0) continue;   // uniform over the CTA in the CTA_ROW form
        const int t = token_sorted[p];
        // token t's row: the caller's rows, or (expert parallel) row t % per of rank t / per
        const void* xb = x.base[0];
        size_t row = (size_t)t;
        if (x.n > 1) {
            xb = x.base[t / x.per];
            row = (size_t)(t % x.per);
        }
        const __half* sg = w13_suh + (size_t)e * 2 * H;
        float sum[2] = {0.0f, 0.0f};
        for (int j = 0; j < nit; ++j) {
            const int blk = CTA_ROW ? BPW * (warp + 8 * j) + g : BPW * j + g;
            const bool act = blk < nb;   // lanes past the last block transform a copy of block 0, unstored
            const int c = (act ? blk : 0) * 128 + hl * V;
            float xv[V];
#pragma unroll
            for (int k = 0; k < V / 8; ++k) {
                float x8[8];
                load8_as_half(xb, x_dtype, row * H + c + 8 * k, x8);
#pragma unroll
                for (int q = 0; q < 8; ++q) xv[8 * k + q] = x8[q];
            }
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                float v[V];
#pragma unroll
                for (int k = 0; k < V / 8; ++k) {
                    float sv[8];
                    load8_half(sg + (size_t)m * H + c + 8 * k, sv);
#pragma unroll
                    for (int q = 0; q < 8; ++q) v[8 * k + q] = __fmul_rn(xv[8 * k + q], sv[q]);
                }
                had128_lanes<L>(v, hl);
                __half* o = (m ? xt_u : xt_g) + (size_t)p * H + c;
#pragma unroll
                for (int k = 0; k < V / 8; ++k) {
                    float w8[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) w8[q] = __fmul_rn(v[8 * k + q], kHad);
                    if (act) {
                        store8_half(o + 8 * k, w8);
#pragma unroll
                        for (int q = 0; q < 8; ++q) sum[m] += r16(w8[q]);
                    }
                }
            }
        }
        if (rsum) {
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) sum[m] += __shfl_xor_sync(0xffffffffu, sum[m], o);
            if (CTA_ROW) {
                if (lane == 0) {
                    wsum[warp][0] = sum[0];
                    wsum[warp][1] = sum[1];
                }
                __syncthreads();
                if (threadIdx.x == 0) {
                    float a = 0.0f, b = 0.0f;
                    for (int w = 0; w < 8; ++w) {
                        a += wsum[w][0];
                        b += wsum[w][1];
                    }
                    *reinterpret_cast<float2*>(rsum + 2 * (size_t)p) = make_float2(a, b);
                }
                __syncthreads();
            } else if (lane == 0) {
                *reinterpret_cast<float2*>(rsum + 2 * (size_t)p) = make_float2(sum[0], sum[1]);
            }
        }
    }
}

cudaError_t launch_prep(const void* x, int x_dtype, const int* token_sorted, const int* expert_sorted,
                        const int* nrows, int N, const __half* w13_suh, int H, __half* xt_g, __half* xt_u,
                        float* rsum, cudaStream_t st)
{
    XRows xr{};
    xr.base[0] = x;
    xr.per = 1;
    xr.n = 1;
    return launch_prep_rows(xr, x_dtype, token_sorted, expert_sorted, nrows, N, w13_suh, H, xt_g, xt_u, rsum, st);
}

cudaError_t launch_prep_rows(const XRows& x, int x_dtype, const int* token_sorted, const int* expert_sorted,
                             const int* nrows, int N, const __half* w13_suh, int H, __half* xt_g, __half* xt_u,
                             float* rsum, cudaStream_t st)
{
    // rows of the call's bound: few rows (up to 32 per SM: decode batches, also expert-parallel ones whose
    // bound counts every rank's routes) take one CTA each, more take one warp each
    const bool cta_row = (long long)N <= (long long)num_sms() * 32;
    long long blocks = cta_row ? (long long)N : ((long long)N + 7) / 8;
    const long long cap = (long long)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return launch_k(cta_row ? prep_kernel<true> : prep_kernel<false>, (int)blocks, 256, 0, st, x, x_dtype, token_sorted,
                    expert_sorted, nrows, w13_suh, H, xt_g, xt_u, rsum);
}

// thread = (token t, 8 consecutive columns)
__global__ void __launch_bounds__(256) combine_kernel(const __half* y, const int* route_pos, const float* w, int T,
                                                      int topk, int H, int accumulate, float* out)
{
    griddep_enter();
    const int chunks = H / 8;
    const long long n = (long long)T * chunks;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / chunks), c = (int)(i % chunks) * 8;
        float acc[8];
        float* o = out + (size_t)t * H + c;
        if (accumulate) {
            const float4 a = *reinterpret_cast<const float4*>(o), b = *reinterpret_cast<const float4*>(o + 4);
            acc[0] = a.x; acc[1] = a.y; acc[2] = a.z; acc[3] = a.w; acc[4] = b.x; acc[5] = b.y; acc[6] = b.z; acc[7] = b.w;
        } else {
#pragma unroll
            for (int q = 0; q < 8; ++q) acc[q] = 0.0f;
        }
        // routes in groups of 8: every route position, weight and output row of the group is loaded before
        // the first of them is added (three dependent memory round trips per group instead of two per route);
        // the sum still runs over the routes in order
        for (int j0 = 0; j0 < topk; j0 += 8) {
            int pos[8];
            float wt[8];
            uint4 u[8];
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) pos[jj] = j0 + jj < topk ? route_pos[t * topk + j0 + jj] : -1;
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                wt[jj] = pos[jj] >= 0 ? w[t * topk + j0 + jj] : 0.0f;
                u[jj] = pos[jj] >= 0 ? *reinterpret_cast<const uint4*>(y + (size_t)pos[jj] * H + c) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                if (pos[jj] < 0) continue;
                const uint32_t v[4] = {u[jj].x, u[jj].y, u[jj].z, u[jj].w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const __half2 h = u32_as_half2(v[q]);
                    acc[2 * q] = __fmaf_rn(wt[jj], __low2float(h), acc[2 * q]);
                    acc[2 * q + 1] = __fmaf_rn(wt[jj], __high2float(h), acc[2 * q + 1]);
                }
            }
        }
        *reinterpret_cast<float4*>(o) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4*>(o + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
}

cudaError_t launch_combine(const __half* y, const int* route_pos, const float* w, int T, int topk, int H,
                           int accumulate, float* out, cudaStream_t st)
{
    const long long n = (long long)T * (H / 8);
    long long blocks = (n + 255) / 256;
    const long long cap = (long long)num_sms() * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return launch_k(combine_kernel, (int)blocks, 256, 0, st, y, route_pos, w, T, topk, H, accumulate, out);
}

// Busy-expert rows accumulated into out with fp32 atomics (the reference fat path accumulates
// into its out buffer the same way): for each listed expert, each of its rows adds w * y.
__global__ void __launch_bounds__(256) scatter_add_kernel(const __half* y, const int* expert_list, int nl,
                                                          const int* counts, const int* offsets,
                                                          const int* token_sorted, const float* weight_sorted,
                                                          int H, float* out)
{
    const int chunks = H / 8;
    for (int li = blockIdx.y; li < nl; li += gridDim.y) {
        const int e = expert_list[li];
        const int c = counts[e], r0 = offsets[e];
        const long long n = (long long)c * chunks;
        for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
            const int r = r0 + (int)(i / chunks), col = (int)(i % chunks) * 8;
            const float wt = weight_sorted[r];
            const uint4 u = *reinterpret_cast<const uint4*>(y + (size_t)r * H + col);
            const uint32_t v[4] = {u.x, u.y, u.z, u.w};
            float* o = out + (size_t)token_sorted[r] * H + col;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const __half2 h = u32_as_half2(v[q]);
                atomicAdd(o + 2 * q, wt * __low2float(h));
                atomicAdd(o + 2 * q + 1, wt * __high2float(h));
            }
        }
    }
}

cudaError_t launch_scatter_add(const __half* y, const int* expert_list, int n_list, const int* counts,
                               const int* offsets, const int* token_sorted, const float* weight_sorted, int H,
                               int rows_bound, float* out, cudaStream_t st)
{
    dim3 grid(32, 64);
    scatter_add_kernel<<<grid, 256, 0, st>>>(y, expert_list, n_list, counts, offsets, token_sorted, weight_sorted, H,
                                              out);
    return cudaGetLastError();
}

// one warp per 16x16 tile
template <int K>
__global__ void __launch_bounds__(256) decode_dense_kernel(const uint32_t* trellis, int k, int n, __half* w)
{
    const int lane = threadIdx.x & 31;
    const int tn_count = n / 16;
    const long long tiles = (long long)(k / 16) * tn_count;
    const LaneDec<K> ld = lane_dec_setup<K>(lane);
    const int r0 = (lane % 4) * 2, c0 = lane / 4;
    for (long long tile = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); tile < tiles;
         tile += (long long)gridDim.x * (blockDim.x >> 5)) {
        const uint32_t* tw = trellis + tile * TileFmt<K>::words;
        uint32_t b[4];
        decode_tile<K>(tw, ld, 65536u, b);
        const int tk = (int)(tile / tn_count), tn = (int)(tile % tn_count);
        __half* base = w + (size_t)(tk * 16) * n + tn * 16;
        const int rows[4] = {r0, r0 + 8, r0, r0 + 8};
        const int cols[4] = {c0, c0, c0 + 8, c0 + 8};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const __half2 h = u32_as_half2(b[q]);
            base[(size_t)rows[q] * n + cols[q]] = __low2half(h);
            base[(size_t)(rows[q] + 1) * n + cols[q]] = __high2half(h);
        }
    }
}

cudaError_t launch_decode_dense(const void* trellis, int k, int n, int bits, __half* w, cudaStream_t st)
{
    const long long tiles = (long long)(k / 16) * (n / 16);
    long long blocks = (tiles + 7) / 8;
    const long long cap = (long long)num_sms() * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    const uint32_t* t = static_cast<const uint32_t*>(trellis);
    if (bits == 2) decode_dense_kernel<2><<<(int)blocks, 256, 0, st>>>(t, k, n, w);
    else if (bits == 4) decode_dense_kernel<4><<<(int)blocks, 256, 0, st>>>(t, k, n, w);
    else decode_dense_kernel<3><<<(int)blocks, 256, 0, st>>>(t, k, n, w);
    return cudaGetLastError();
}

// Failure-detection self test: one warp waits on an mbarrier that nothing ever arrives on, with
// the same bounded wait the GEMV/GEMM pipelines use. The wait must give up after `limit_ns`,
// record kStatusWaitTimeout in `status` and return, leaving the context usable.
__global__ void __launch_bounds__(32) wait_selftest_kernel(int* status, uint64_t limit_ns)
{
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncwarp();
    mbar_wait_bounded(&bar, 0, &abort_flag, status, limit_ns);
}

cudaError_t launch_wait_selftest(int* status, uint64_t limit_ns, cudaStream_t st)
{
    wait_selftest_kernel<<<1, 32, 0, st>>>(status, limit_ns);
    return cudaGetLastError();
}

}  // namespace dsv41
