// Expert parallelism over NVLink peer memory: the dispatch and combine exchanges are folded into
// the layer's own kernels instead of running as collectives.
//
// Every rank owns one device allocation shared with its peers through CUDA IPC (identical layout
// on all ranks; host side in capi.cu). Per step, with parity p = step & 1:
//   publish   this rank's tokens (fp16 rows, the reference's x2d.half()), global expert ids and
//             routing weights into its own buffers [p]; the last block of the same launch stamps
//             in_flag[rank] on every peer
//   gather    wait (bounded) for every peer's in_flag stamp, read each peer's id/weight table with
//             peer loads and keep the routes that land on this rank's experts (local ids, -1 else)
//   prep      (transform.cu) pulls the token row of each local route straight from the owning
//             rank's published rows -- the dispatch exchange happens inside the row transform
//   experts   the unchanged decode-GEMV / tcgen05 GEMM passes; the down pass's epilogue stores each
//             output row straight into the receive slot of the route's token owner (recv [p], slot
//             t * k + j) -- the combine exchange happens inside the expert kernels, tile by tile
//   signal    drop flag (this rank served none of its routes this step: route-capacity overflow) and
//             out_flag[rank] stamp on every peer
//   combine   wait (bounded) for every peer's out_flag stamp, then for each own token accumulate
//             w * y over its routes in route order in fp32 from the local receive slots (routes of a
//             rank that dropped its work contribute nothing)
// Buffers alternate by step parity; a rank only publishes step s after it has seen every peer's
// step s-1 stamp, which each peer writes only after finishing its step s-2 reads, so no buffer is
// overwritten while a peer may still read it; a rank stores into a peer's receive slots of step s
// only after it saw that peer's step s in-stamp, which the peer writes after its step s-1 combine.
// Stamps are step + 1 (0 = nothing published). All waits are bounded by %globaltimer (the group's
// wait_limit_us, 2 s by default): on expiry the kernel records status 1 in the control block, writes
// an empty result and returns (no trap). Plain peer loads and stores only.
#include "ep_device.cuh"

namespace dsv41 {

__global__ void __launch_bounds__(256) ep_publish_kernel(const void* x, int x_dtype, const int64_t* ids,
                                                         const float* w, int T, int tcap, int k, int E, int H,
                                                         __half* X, int* IDS, float* W, PeerTable peers, int world,
                                                         int rank, size_t flag_off, uint32_t stamp, int* done)
{
    griddep_enter();
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
    // the block's stores, then its arrival; the last block to arrive stamps every peer (the counter is
    // reset for the next step, which stream order puts after this launch)
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(done, 1) == (int)gridDim.x - 1;
        if (last) *done = 0;
    }
    __syncthreads();
    if (last && (int)threadIdx.x < world) {
        __threadfence_system();
        uint32_t* f = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(peers.base[threadIdx.x]) + flag_off) + rank;
        st_release_sys(f, stamp);
    }
}

// out-stamp: with `nrows`, first this rank's drop flag on every peer (stamp when its expert passes did no
// work this step, i.e. the routes were dropped on a route-capacity overflow), then the release of the stamp
__global__ void ep_signal_kernel(PeerTable peers, int world, int rank, size_t flag_off, uint32_t stamp,
                                 const int* nrows, size_t drop_off)
{
    griddep_enter();
    const int d = threadIdx.x;
    if (d >= world) return;
    uint8_t* b = static_cast<uint8_t*>(peers.base[d]);
    if (nrows) reinterpret_cast<uint32_t*>(b + drop_off)[rank] = (*nrows == 0) ? stamp : 0u;
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(b + flag_off) + rank, stamp);
}

__global__ void __launch_bounds__(256) ep_gather_kernel(const EpGather g)
{
    griddep_enter();
    const bool ok = block_wait_stamps(g.in_flags, g.world, g.stamp, g.status, g.limit_ns);
    ep_gather_routes(g, ok, (long long)blockIdx.x * blockDim.x + threadIdx.x, (long long)gridDim.x * blockDim.x);
}

// block = own token t (grid-stride). Threads j < k first resolve route j of the token -- its weight, or 0
// when the route is invalid or its serving rank dropped its work -- into shared memory; then every thread
// takes 8-column chunks of the row, issues the loads of all live routes' 16-byte pieces from the local
// receive slots and adds them up in route order (fp32, the same order for every chunk: deterministic for a
// given routing, and the order of the single-GPU combine).
constexpr int kCombineRoutes = 32;   // routes resolved per shared-memory batch
__global__ void __launch_bounds__(256) ep_combine_kernel(const uint32_t* flags, const uint32_t* drops, int world,
                                                         int e_loc, uint32_t stamp, const int* ids, const float* w,
                                                         int T, int k, int H, const __half* recv, float* out,
                                                         int* status, uint64_t limit_ns)
{
    griddep_enter();
    __shared__ float wts[kCombineRoutes];
    __shared__ int live[kCombineRoutes];
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
                const bool on = e >= 0 && e / e_loc < world && __ldcg(drops + e / e_loc) != stamp;
                live[threadIdx.x] = on;
                wts[threadIdx.x] = on ? w[t * k + j] : 0.0f;
            }
            __syncthreads();
            const __half* rows = recv + ((size_t)t * k + j0) * H;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int c = (int)threadIdx.x + 256 * i;
                if (c >= chunks) break;
                for (int jb = 0; jb < nj; jb += 8) {
                    uint4 u[8];
#pragma unroll
                    for (int r = 0; r < 8; ++r)
                        if (jb + r < nj && live[jb + r])
                            u[r] = __ldcg(reinterpret_cast<const uint4*>(rows + (size_t)(jb + r) * H + (size_t)c * 8));
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        if (jb + r >= nj || !live[jb + r]) continue;
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
                              int E, int H, __half* X, int* IDS, float* W, const PeerTable& peers, int world, int rank,
                              size_t flag_off, uint32_t stamp, int* done, cudaStream_t st)
{
    const long long work = (long long)T * H / 4 > (long long)tcap * k ? (long long)T * H / 4 : (long long)tcap * k;
    return launch_k(ep_publish_kernel, grid_for(work, 256, 8), 256, 0, st, x, x_dtype, ids, w, T, tcap, k, E, H, X, IDS,
                    W, peers, world, rank, flag_off, stamp, done);
}

cudaError_t launch_ep_signal(const PeerTable& peers, int world, int rank, size_t flag_off, uint32_t stamp,
                             const int* nrows, size_t drop_off, cudaStream_t st)
{
    return launch_k(ep_signal_kernel, 1, 32, 0, st, peers, world, rank, flag_off, stamp, nrows, drop_off);
}

cudaError_t launch_ep_gather(const EpGather& g, cudaStream_t st)
{
    return launch_k(ep_gather_kernel, grid_for((long long)g.world * g.per, 4 * 256, 4), 256, 0, st, g);
}

cudaError_t launch_ep_combine(const uint32_t* out_flags, const uint32_t* drops, int world, int e_loc, uint32_t stamp,
                              const int* ids, const float* w, int T, int k, int H, const __half* recv, float* out,
                              int* status, uint64_t limit_ns, cudaStream_t st)
{
    if (H > 8 * 256 * 4) return cudaErrorInvalidValue;   // the combine's 4 chunks of 8 columns per thread
    return launch_k(ep_combine_kernel, grid_for(T, 1, 8), 256, 0, st, out_flags, drops, world, e_loc, stamp, ids, w, T,
                    k, H, recv, out, status, limit_ns);
}

}  // namespace dsv41
