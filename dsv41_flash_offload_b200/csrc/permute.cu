// Routing permutation: the routing prep of apply_exl3_fused_moe
// (patches/vllm-exl3-host-dma.patch:204-226, :300-312 -- local ids with the n_exp sentinel,
// expert_count[E+1], expert-sorted order) and the histogram/compaction of ft_split
// (ct/ft_tier_cu_v.cu:16-101), as warp-segment histograms + scan + stable scatter.
//
// Order: stable by (local expert, flat route index), bit-exact with a stable argsort. Each warp
// owns a contiguous segment of flat routes; __match_any_sync groups equal experts inside a
// 32-route window, so ranks inside a segment follow flat order, and segments are prefixed in
// order. No atomics decide positions, so the output is deterministic.
//
// The same pass builds the work lists of the expert kernels: row groups of <= 16 rows for
// experts on the decode-GEMV path, and the list of experts over fat_threshold rows (GEMM path).
#include "common.cuh"
#include "ep_device.cuh"
#include "internal.h"

namespace dsv41 {

__device__ __forceinline__ int local_id(int64_t id, int E, const int32_t* map, int map_len)
{
    if (map) {
        if (id < 0 || id >= map_len) return E;
        const int l = map[id];
        return (l < 0 || l >= E) ? E : l;
    }
    return (id < 0 || id >= E) ? E : (int)id;
}

// In-place exclusive scan of n ints in shared memory by the whole block; returns the total.
// `scratch` holds >= 33 ints.
__device__ int block_exclusive_scan(int* data, int n, int* scratch)
{
    const int nt = blockDim.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int per = (n + nt - 1) / nt;
    const int b = min(n, t * per), e = min(n, b + per);
    int s = 0;
    for (int i = b; i < e; ++i) s += data[i];
    int inc = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane == 31) scratch[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int nw = (nt + 31) >> 5;
        int v = lane < nw ? scratch[lane] : 0;
        int vi = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, vi, o);
            if (lane >= o) vi += u;
        }
        if (lane < nw) scratch[lane] = vi - v;
        if (lane == 31) scratch[32] = vi;
    }
    __syncthreads();
    int run = scratch[warp] + inc - s;
    for (int i = b; i < e; ++i) {
        const int v = data[i];
        data[i] = run;
        run += v;
    }
    const int total = scratch[32];
    __syncthreads();
    return total;
}

struct PermArgs {
    const int64_t* ids;
    const float* w;
    int N, topk, E;
    const int32_t* map;
    int map_len;
    int fat;
    PermBuffers pb;
    int gather;   // single-CTA path: first gather ids/w from the expert-parallel peers (g)
    EpGather g;
};

// tot[e] (e <= E) holds the per-expert totals in shared memory; writes counts/offsets and the
// GEMV group list / fat list. `tmp` is a shared array of >= E+1 ints.
__device__ void finish_lists(const PermArgs& a, int* tot, int* tmp, int* scratch)
{
    const int E = a.E;
    const int t = threadIdx.x, nt = blockDim.x;
    for (int e = t; e <= E; e += nt) {
        a.pb.counts[e] = tot[e];
        if (a.pb.counts64) a.pb.counts64[e] = tot[e];
    }
    __syncthreads();
    block_exclusive_scan(tot, E + 1, scratch);  // tot -> offsets
    for (int e = t; e <= E; e += nt) {
        a.pb.offsets[e] = tot[e];
        if (a.pb.offsets64) a.pb.offsets64[e] = tot[e];
    }
    // more valid routes than the row buffers hold: no expert work at all (status 3, zero output)
    const bool over = tot[E] > a.pb.rows_cap;
    // row groups of GEMV experts
    for (int e = t; e <= E; e += nt) {
        const int c = (e < E && !over) ? a.pb.counts[e] : 0;
        const bool fat = a.fat >= 0 && c > a.fat;
        tmp[e] = (c == 0 || fat) ? 0 : (c + kRowsPerGroup - 1) / kRowsPerGroup;
    }
    __syncthreads();
    const int ng = block_exclusive_scan(tmp, E + 1, scratch);
    for (int e = t; e < E; e += nt) {
        const int c = over ? 0 : a.pb.counts[e];
        const bool fat = a.fat >= 0 && c > a.fat;
        if (c == 0 || fat) continue;
        const int g0 = tmp[e], row0 = tot[e];
        for (int r = 0; r < c; r += kRowsPerGroup)
            a.pb.groups[g0 + r / kRowsPerGroup] = make_int4(e, row0 + r, min(kRowsPerGroup, c - r), 0);
    }
    __syncthreads();
    for (int e = t; e <= E; e += nt) {
        const int c = (e < E && !over) ? a.pb.counts[e] : 0;
        tmp[e] = (a.fat >= 0 && c > a.fat) ? 1 : 0;
    }
    __syncthreads();
    const int nf = block_exclusive_scan(tmp, E + 1, scratch);
    for (int e = t; e < E; e += nt) {
        const int c = over ? 0 : a.pb.counts[e];
        if (a.fat >= 0 && c > a.fat) a.pb.fat_experts[tmp[e]] = e;
    }
    if (t == 0) {
        *a.pb.n_groups = ng;
        *a.pb.n_fat = nf;
        if (a.pb.nrows) *a.pb.nrows = over ? 0 : tot[E];
        if (over && a.pb.status) atomicExch(a.pb.status, kStatusRouteCapacity);
    }
}

// Walk this warp's segment [b, e) in order; `row` is the warp's per-expert counter row in
// shared memory. Histogram mode adds counts; scatter mode assigns positions base + rank.
template <bool SCATTER>
__device__ void walk_segment(const PermArgs& a, int b, int e, int* row, const int* off, bool drop = false)
{
    const int lane = threadIdx.x & 31;
    for (int i0 = b; i0 < e; i0 += 32) {
        const int i = i0 + lane;
        const bool valid = i < e;
        const int l = valid ? local_id(a.ids[i], a.E, a.map, a.map_len) : -1 - lane;
        const unsigned peers = __match_any_sync(0xffffffffu, l);
        const int leader = __ffs(peers) - 1;
        const int rank = __popc(peers & ((1u << lane) - 1u));
        if (!SCATTER) {
            if (valid && lane == leader) row[l] += __popc(peers);
        } else {
            int base = 0;
            if (valid && lane == leader) base = off[l] + row[l];
            base = __shfl_sync(0xffffffffu, base, leader);
            __syncwarp();
            if (valid) {
                const int pos = base + rank;
                a.pb.token_sorted[pos] = i / a.topk;
                a.pb.weight_sorted[pos] = a.w ? a.w[i] : 0.0f;
                a.pb.route_sorted[pos] = i;
                a.pb.expert_sorted[pos] = l;
                a.pb.route_pos[i] = (l == a.E || drop) ? -1 : pos;
                if (lane == leader) row[l] += __popc(peers);
            }
        }
        __syncwarp();
    }
}

// Single CTA (N <= kPermSmallMax): 32 warp segments, all phases in shared memory.
__global__ void __launch_bounds__(1024) permute_small_kernel(const PermArgs a)
{
    griddep_enter();
    extern __shared__ int sm[];
    const int E1 = a.E + 1;
    int* seg = sm;                    // [32][E1]
    int* tot = seg + 32 * E1;         // [E1]
    int* tmp = tot + E1;              // [E1]
    int* scratch = tmp + E1;          // [33]
    if (a.gather) {
        // expert parallel: the routes of this rank's experts from every peer's tables, into a.ids / a.w
        const bool ok = block_wait_stamps(a.g.in_flags, a.g.world, a.g.stamp, a.g.status, a.g.limit_ns);
        ep_gather_routes(a.g, ok, threadIdx.x, blockDim.x);
        __syncthreads();
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = (a.N + 31) / 32;
    const int b = min(a.N, warp * S), e = min(a.N, b + S);
    int* row = seg + warp * E1;
    for (int x = lane; x < E1; x += 32) row[x] = 0;
    __syncwarp();
    walk_segment<false>(a, b, e, row, nullptr);
    __syncthreads();
    for (int x = threadIdx.x; x < E1; x += blockDim.x) {
        int run = 0;
        for (int w = 0; w < 32; ++w) {
            const int c = seg[w * E1 + x];
            seg[w * E1 + x] = run;
            run += c;
        }
        tot[x] = run;
    }
    __syncthreads();
    finish_lists(a, tot, tmp, scratch);  // tot becomes offsets
    __syncthreads();
    walk_segment<true>(a, b, e, row, tot, tot[a.E] > a.pb.rows_cap);
}

// Multi-CTA path: (1) per-segment histograms, (2) one CTA scans, (3) stable scatter.
constexpr int kPermWarps = 8;

__global__ void __launch_bounds__(kPermWarps * 32) permute_hist_kernel(const PermArgs a)
{
    griddep_enter();
    extern __shared__ int sm[];
    const int E1 = a.E + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sg = blockIdx.x * kPermWarps + warp;
    int* row = sm + warp * E1;
    for (int x = lane; x < E1; x += 32) row[x] = 0;
    __syncwarp();
    const int b = min(a.N, sg * kPermSegment), e = min(a.N, b + kPermSegment);
    walk_segment<false>(a, b, e, row, nullptr);
    __syncwarp();
    const int nseg = (a.N + kPermSegment - 1) / kPermSegment;
    if (sg < nseg)
        for (int x = lane; x < E1; x += 32) a.pb.seg_hist[(size_t)sg * E1 + x] = row[x];
}

__global__ void __launch_bounds__(1024) permute_scan_kernel(const PermArgs a)
{
    griddep_enter();
    extern __shared__ int sm[];
    const int E1 = a.E + 1;
    int* tot = sm;
    int* tmp = tot + E1;
    int* scratch = tmp + E1;
    const int nseg = (a.N + kPermSegment - 1) / kPermSegment;
    for (int x = threadIdx.x; x < E1; x += blockDim.x) {
        int run = 0;
        for (int s = 0; s < nseg; ++s) {
            int* p = a.pb.seg_hist + (size_t)s * E1 + x;
            const int c = *p;
            *p = run;
            run += c;
        }
        tot[x] = run;
    }
    __syncthreads();
    finish_lists(a, tot, tmp, scratch);
}

__global__ void __launch_bounds__(kPermWarps * 32) permute_scatter_kernel(const PermArgs a)
{
    griddep_enter();
    extern __shared__ int sm[];
    const int E1 = a.E + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sg = blockIdx.x * kPermWarps + warp;
    const int nseg = (a.N + kPermSegment - 1) / kPermSegment;
    int* row = sm + warp * E1;
    int* off = sm + kPermWarps * E1;
    for (int x = threadIdx.x; x < E1; x += blockDim.x) off[x] = a.pb.offsets[x];
    if (sg < nseg)
        for (int x = lane; x < E1; x += 32) row[x] = a.pb.seg_hist[(size_t)sg * E1 + x];
    __syncthreads();
    const int b = min(a.N, sg * kPermSegment), e = min(a.N, b + kPermSegment);
    walk_segment<true>(a, b, e, row, off, off[a.E] > a.pb.rows_cap);
}

// Work lists for a caller-given expert list over caller-permuted rows (run_batch semantics).
__global__ void __launch_bounds__(1024) list_setup_kernel(const int32_t* experts, int n_experts, const int64_t* counts64,
                                                          const int64_t* offsets64, int E, int total_rows, int fat,
                                                          PermBuffers pb, int* nrows)
{
    extern __shared__ int sm[];
    int* tmp = sm;                     // [n_experts + 1]
    int* scratch = tmp + n_experts + 1;
    const int t = threadIdx.x, nt = blockDim.x;
    for (int e = t; e <= E; e += nt) {
        pb.counts[e] = (int)counts64[e];
        pb.offsets[e] = (int)offsets64[e];
    }
    for (int p = t; p < total_rows; p += nt) pb.expert_sorted[p] = -1;
    __syncthreads();
    for (int i = t; i <= n_experts; i += nt) {
        int ng = 0;
        if (i < n_experts) {
            const int e = experts[i];
            const int c = (e >= 0 && e < E) ? (int)counts64[e] : 0;
            ng = (c == 0 || (fat >= 0 && c > fat)) ? 0 : (c + kRowsPerGroup - 1) / kRowsPerGroup;
        }
        tmp[i] = ng;
    }
    __syncthreads();
    const int ng = block_exclusive_scan(tmp, n_experts + 1, scratch);
    for (int i = 0; i < n_experts; ++i) {  // rows of listed experts (block-strided inside)
        const int e = experts[i];
        if (e < 0 || e >= E) continue;
        const int c = (int)counts64[e], r0 = (int)offsets64[e];
        for (int r = t; r < c; r += nt)
            if (r0 + r < total_rows) pb.expert_sorted[r0 + r] = e;
        const bool is_fat = fat >= 0 && c > fat;
        if (!is_fat)
            for (int r = t * kRowsPerGroup; r < c; r += nt * kRowsPerGroup)
                pb.groups[tmp[i] + r / kRowsPerGroup] = make_int4(e, r0 + r, min(kRowsPerGroup, c - r), 0);
    }
    __syncthreads();
    for (int i = t; i <= n_experts; i += nt) {
        int f = 0;
        if (i < n_experts) {
            const int e = experts[i];
            const int c = (e >= 0 && e < E) ? (int)counts64[e] : 0;
            f = (fat >= 0 && c > fat) ? 1 : 0;
        }
        tmp[i] = f;
    }
    __syncthreads();
    const int nf = block_exclusive_scan(tmp, n_experts + 1, scratch);
    for (int i = t; i < n_experts; i += nt) {
        const int e = experts[i];
        const int c = (e >= 0 && e < E) ? (int)counts64[e] : 0;
        if (fat >= 0 && c > fat) pb.fat_experts[tmp[i]] = e;
    }
    if (t == 0) {
        *pb.n_groups = ng;
        *pb.n_fat = nf;
        *nrows = total_rows;
    }
}

cudaError_t launch_list_setup(const int32_t* experts, int n_experts, const int64_t* counts64, const int64_t* offsets64,
                              int E, int total_rows, int fat, const PermBuffers& pb, int* nrows, cudaStream_t st)
{
    const size_t smem = ((size_t)n_experts + 1 + 33) * sizeof(int);
    if (smem > 48 * 1024) {
        cudaError_t err = cudaFuncSetAttribute((const void*)list_setup_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (err != cudaSuccess) return err;
    }
    list_setup_kernel<<<1, 1024, smem, st>>>(experts, n_experts, counts64, offsets64, E, total_rows, fat, pb, nrows);
    return cudaGetLastError();
}

size_t perm_seg_hist_ints(int N, int E)
{
    const size_t nseg = (size_t)(N + kPermSegment - 1) / kPermSegment;
    return perm_uses_small(N, E) ? 0 : nseg * (size_t)(E + 1);
}

// the single-CTA path keeps 32 warp rows + 2 arrays of E+1 ints in shared memory
bool perm_uses_small(int N, int E) { return N <= kPermSmallMax && (size_t)(34 * (E + 1) + 33) * 4 <= 200 * 1024; }

int max_groups(int N, int E) { return N / kRowsPerGroup + (N < E ? N : E) + 1; }

static cudaError_t set_smem(const void* fn, size_t bytes)
{
    if (bytes <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

cudaError_t launch_permute(const int64_t* ids, const float* weights, int N, int topk, int E,
                           const int32_t* expert_map, int map_len, int fat_threshold,
                           const PermBuffers& pb, cudaStream_t st)
{
    PermArgs a{ids, weights, N, topk, E, expert_map, map_len, fat_threshold, pb};
    const size_t E1 = (size_t)E + 1;
    cudaError_t err;
    if (perm_uses_small(N, E)) {
        const size_t smem = (32 * E1 + 2 * E1 + 33) * sizeof(int);
        if ((err = set_smem((const void*)permute_small_kernel, smem)) != cudaSuccess) return err;
        return launch_k(permute_small_kernel, 1, 1024, smem, st, a);
    }
    const int nseg = (N + kPermSegment - 1) / kPermSegment;
    const int blocks = (nseg + kPermWarps - 1) / kPermWarps;
    const size_t smem_h = kPermWarps * E1 * sizeof(int);
    const size_t smem_s = (2 * E1 + 33) * sizeof(int);
    const size_t smem_x = (kPermWarps + 1) * E1 * sizeof(int);
    if ((err = set_smem((const void*)permute_hist_kernel, smem_h)) != cudaSuccess) return err;
    if ((err = set_smem((const void*)permute_scan_kernel, smem_s)) != cudaSuccess) return err;
    if ((err = set_smem((const void*)permute_scatter_kernel, smem_x)) != cudaSuccess) return err;
    if ((err = launch_k(permute_hist_kernel, blocks, kPermWarps * 32, smem_h, st, a)) != cudaSuccess) return err;
    if ((err = launch_k(permute_scan_kernel, 1, 1024, smem_s, st, a)) != cudaSuccess) return err;
    return launch_k(permute_scatter_kernel, blocks, kPermWarps * 32, smem_x, st, a);
}

cudaError_t launch_permute_gathered(const EpGather& g, int topk, int E, int fat_threshold, const PermBuffers& pb,
                                    cudaStream_t st)
{
    const int N = g.world * g.per;
    if (perm_uses_small(N, E)) {
        PermArgs a{g.ids_out, g.w_out, N, topk, E, nullptr, 0, fat_threshold, pb};
        a.gather = 1;
        a.g = g;
        const size_t E1 = (size_t)E + 1;
        const size_t smem = (32 * E1 + 2 * E1 + 33) * sizeof(int);
        cudaError_t err;
        if ((err = set_smem((const void*)permute_small_kernel, smem)) != cudaSuccess) return err;
        return launch_k(permute_small_kernel, 1, 1024, smem, st, a);
    }
    const cudaError_t err = launch_ep_gather(g, st);
    if (err != cudaSuccess) return err;
    return launch_permute(g.ids_out, g.w_out, N, topk, E, nullptr, 0, fat_threshold, pb, st);
}

}  // namespace dsv41
