// Expert parallelism over NVLink peer memory: the dispatch and combine exchanges are folded into
// the layer's own kernels instead of running as collectives.
//
// Every rank owns one device allocation shared with its peers through CUDA IPC (identical layout
// on all ranks; host side in capi.cu). Per step, with parity p = step & 1:
//   publish   this rank's tokens (fp16 rows, the reference's x2d.half()), global expert ids and
//             routing weights into its own buffers [p], then stamp in_flag[rank] on every peer
//   gather    wait (bounded) for every peer's in_flag stamp, read each peer's id/weight table with
//             peer loads and keep the routes that land on this rank's experts (local ids, -1 else)
//   prep      (transform.cu) pulls the token row of each local route straight from the owning
//             rank's published rows -- the dispatch exchange happens inside the row transform
//   experts   the unchanged decode-GEMV / tcgen05 GEMM passes write fp16 expert outputs into this
//             rank's workspace [p], which peers can read
//   signal    stamp out_flag[rank] on every peer
//   combine   wait (bounded) for every peer's out_flag stamp, then for each own token pull the
//             expert output rows of its routes from their owners (position from the owner's
//             route_pos table) and accumulate w * y in fp32 in route order -- the combine
//             exchange happens inside the weighted sum
// Buffers alternate by step parity; a rank only publishes step s after it has seen every peer's
// step s-1 stamp, which each peer writes only after finishing its step s-2 reads, so no buffer is
// overwritten while a peer may still read it. Stamps are step + 1 (0 = nothing published).
// All waits are bounded by %globaltimer (the group's wait_limit_us, 2 s by default): on expiry the
// kernel records status 1 in the control block, writes an empty result and returns (no trap). Plain
// peer loads and stores only.
#include "common.cuh"
#include "internal.h"

namespace dsv41 {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// thread 0 of the block waits until every peer's stamp in flags[0..world) reached `stamp`, at most
// limit_ns in all; returns false for the whole block on timeout (and records kStatusWaitTimeout)
__device__ bool block_wait_stamps(const uint32_t* flags, int world, uint32_t stamp, int* status, uint64_t limit_ns)
{
    __shared__ int ok;
    if (threadIdx.x == 0) {
        ok = 1;
        const uint64_t t0 = globaltimer_ns();
        for (int d = 0; d < world && ok; ++d) {
            uint32_t it = 0;
            while ((int)(ld_acquire_sys(flags + d) - stamp) < 0) {
                if ((++it & 63u) == 0 && globaltimer_ns() - t0 > limit_ns) {
                    atomicExch(status, kStatusWaitTimeout);
                    ok = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    return ok != 0;
}

__global__ void __launch_bounds__(256) ep_publish_kernel(const void* x, int x_dtype, const int64_t* ids,
                                                         const float* w, int T, int tcap, int k, int E, int H,
                                                         __half* X, int* IDS, float* W)
{
    const long long stride = (long long)gridDim.x * blockDim.x;
    const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long nx = (long long)T * H / 4;
    for (long long i = tid; i < nx; i += stride) {
        float v[4];
        load4_as_half(x, x_dtype, (size_t)i * 4, v);
        store4_half(X + (size_t)i * 4, v);
    }
    const long long nr = (long long)tcap * k;
    for (long long i = tid; i < nr; i += stride) {
        int e = -1;
        float wt = 0.0f;
        if (i < (long long)T * k) {
            const int64_t g = ids[i];
            e = (g >= 0 && g < E) ? (int)g : -1;
            wt = w[i];
        }
        IDS[i] = e;
        W[i] = wt;
    }
}

__global__ void ep_signal_kernel(PeerTable peers, int world, int rank, size_t flag_off, uint32_t stamp)
{
    const int d = threadIdx.x;
    if (d >= world) return;
    __threadfence_system();
    uint32_t* f = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(peers.base[d]) + flag_off) + rank;
    st_release_sys(f, stamp);
}

__global__ void __launch_bounds__(256) ep_gather_kernel(PeerTable peers, int world, int rank, int tcap, int k, int lo,
                                                        int hi, uint32_t stamp, size_t in_flags_off, size_t ids_off,
                                                        size_t w_off, int64_t* ids_loc, float* w_loc, int* status,
                                                        uint64_t limit_ns)
{
    const uint32_t* flags =
        reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(peers.base[rank]) + in_flags_off);
    const bool ok = block_wait_stamps(flags, world, stamp, status, limit_ns);
    const long long per = (long long)tcap * k, n = per * world;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        int64_t le = -1;
        float wt = 0.0f;
        if (ok) {
            const int d = (int)(i / per);
            const long long r = i % per;
            const uint8_t* b = static_cast<const uint8_t*>(peers.base[d]);
            const int e = __ldcg(reinterpret_cast<const int*>(b + ids_off) + r);
            if (e >= lo && e < hi) {
                le = e - lo;
                wt = __ldcg(reinterpret_cast<const float*>(b + w_off) + r);
            }
        }
        ids_loc[i] = le;
        w_loc[i] = wt;
    }
}

// block = own token t (grid-stride). Threads j < k first resolve route j of the token: the owner's sorted
// position (one peer load each, all routes at once) and the weight, into shared memory; then every thread
// takes 8-column chunks of the row and issues the loads of all routes' 16-byte pieces before it adds
// them up in route order (fp32, the same order for every chunk), so the pull costs two dependent NVLink
// round trips per token rather than two per route.
constexpr int kCombineRoutes = 32;   // routes resolved per shared-memory batch
__global__ void __launch_bounds__(256) ep_combine_kernel(PeerTable peers, int world, int rank, int tcap, int k,
                                                         int e_loc, uint32_t stamp, size_t out_flags_off,
                                                         const int* ids, const float* w, int T, int H,
                                                         size_t route_pos_off, size_t y_off, float* out, int* status,
                                                         uint64_t limit_ns)
{
    __shared__ const __half* src[kCombineRoutes];
    __shared__ float wts[kCombineRoutes];
    const uint32_t* flags =
        reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(peers.base[rank]) + out_flags_off);
    const bool ok = block_wait_stamps(flags, world, stamp, status, limit_ns);
    const int chunks = H / 8;
    for (int t = blockIdx.x; t < T; t += gridDim.x) {
        // this thread's chunks of the row: c = threadIdx.x + 256 * i (at most 4 for H <= 8192)
        float acc[4][8];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int q = 0; q < 8; ++q) acc[i][q] = 0.0f;
        for (int j0 = 0; ok && j0 < k; j0 += kCombineRoutes) {
            const int nj = min(kCombineRoutes, k - j0);
            if ((int)threadIdx.x < nj) {
                const int j = j0 + threadIdx.x;
                const int e = ids[t * k + j];
                const __half* sp = nullptr;
                float wt = 0.0f;
                if (e >= 0 && e / e_loc < world) {
                    const uint8_t* b = static_cast<const uint8_t*>(peers.base[e / e_loc]);
                    const int pos = __ldcg(reinterpret_cast<const int*>(b + route_pos_off) + ((size_t)rank * tcap + t) * k + j);
                    if (pos >= 0) {
                        sp = reinterpret_cast<const __half*>(b + y_off) + (size_t)pos * H;
                        wt = w[t * k + j];
                    }
                }
                src[threadIdx.x] = sp;
                wts[threadIdx.x] = wt;
            }
            __syncthreads();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int c = (int)threadIdx.x + 256 * i;
                if (c >= chunks) break;
                for (int jb = 0; jb < nj; jb += 8) {
                    uint4 u[8];
#pragma unroll
                    for (int r = 0; r < 8; ++r)
                        if (jb + r < nj && src[jb + r]) u[r] = *reinterpret_cast<const uint4*>(src[jb + r] + (size_t)c * 8);
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        if (jb + r >= nj || !src[jb + r]) continue;
                        const float wt = wts[jb + r];
                        const uint32_t v[4] = {u[r].x, u[r].y, u[r].z, u[r].w};
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const __half2 h = u32_as_half2(v[q]);
                            acc[i][2 * q] = __fmaf_rn(wt, __low2float(h), acc[i][2 * q]);
                            acc[i][2 * q + 1] = __fmaf_rn(wt, __high2float(h), acc[i][2 * q + 1]);
                        }
                    }
                }
            }
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int c = (int)threadIdx.x + 256 * i;
            if (c >= chunks) break;
            float* o = out + (size_t)t * H + (size_t)c * 8;
            *reinterpret_cast<float4*>(o) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
            *reinterpret_cast<float4*>(o + 4) = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
        }
    }
}

static int grid_for(long long work, int per_block, int cap_per_sm)
{
    long long b = (work + per_block - 1) / per_block;
    const long long cap = (long long)num_sms() * cap_per_sm;
    if (b > cap) b = cap;
    return (int)(b < 1 ? 1 : b);
}

cudaError_t launch_ep_publish(const void* x, int x_dtype, const int64_t* ids, const float* w, int T, int tcap, int k,
                              int E, int H, __half* X, int* IDS, float* W, cudaStream_t st)
{
    const long long work = (long long)T * H / 4 > (long long)tcap * k ? (long long)T * H / 4 : (long long)tcap * k;
    ep_publish_kernel<<<grid_for(work, 256, 8), 256, 0, st>>>(x, x_dtype, ids, w, T, tcap, k, E, H, X, IDS, W);
    return cudaGetLastError();
}

cudaError_t launch_ep_signal(const PeerTable& peers, int world, int rank, size_t flag_off, uint32_t stamp,
                             cudaStream_t st)
{
    ep_signal_kernel<<<1, 32, 0, st>>>(peers, world, rank, flag_off, stamp);
    return cudaGetLastError();
}

cudaError_t launch_ep_gather(const PeerTable& peers, int world, int rank, int tcap, int k, int lo, int hi,
                             uint32_t stamp, size_t in_flags_off, size_t ids_off, size_t w_off, int64_t* ids_loc,
                             float* w_loc, int* status, uint64_t limit_ns, cudaStream_t st)
{
    ep_gather_kernel<<<grid_for((long long)world * tcap * k, 256, 4), 256, 0, st>>>(
        peers, world, rank, tcap, k, lo, hi, stamp, in_flags_off, ids_off, w_off, ids_loc, w_loc, status, limit_ns);
    return cudaGetLastError();
}

cudaError_t launch_ep_combine(const PeerTable& peers, int world, int rank, int tcap, int k, int e_loc, uint32_t stamp,
                              size_t out_flags_off, const int* ids, const float* w, int T, int H, size_t route_pos_off,
                              size_t y_off, float* out, int* status, uint64_t limit_ns, cudaStream_t st)
{
    if (H > 8 * 256 * 4) return cudaErrorInvalidValue;   // the combine's 4 chunks of 8 columns per thread
    ep_combine_kernel<<<grid_for(T, 1, 8), 256, 0, st>>>(
        peers, world, rank, tcap, k, e_loc, stamp, out_flags_off, ids, w, T, H, route_pos_off, y_off, out, status,
        limit_ns);
    return cudaGetLastError();
}

}  // namespace dsv41
