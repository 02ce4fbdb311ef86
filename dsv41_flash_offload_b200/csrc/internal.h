// Internal launch interface shared by the kernel files and the C ABI (capi.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace dsv41 {

constexpr int kRowsPerGroup = 16;     // decode-GEMV row group (one mma M tile)
constexpr int kPermSmallMax = 8192;   // routes handled by the single-CTA permutation
constexpr int kPermSegment = 256;     // routes per warp segment in the multi-CTA permutation
constexpr int kMaxExperts = 4096;
constexpr int kMaxPeers = 8;     // expert-parallel ranks reachable by peer loads

// device base pointers of every rank's shared buffer (index = rank), passed by value to kernels
struct PeerTable {
    void* base[kMaxPeers];
};
// where the row transform reads token t: n == 1: base[0] + t rows; else base[t / per] + (t % per) rows
struct XRows {
    const void* base[kMaxPeers];
    int per, n;
};
// Where an expert pass stores its output rows. route == nullptr: the pass's own output array, row r at
// out + r * N. Otherwise (expert-parallel push): sorted row r serves flat route i = route[r] of rank
// d = i / per, and its output row goes straight into that rank's receive slots, base[d] + (i % per) rows --
// a peer store over NVLink issued by the epilogue, so the combine exchange overlaps the expert math.
struct RowPush {
    void* base[kMaxPeers];
    const int* route;
    int per;
};
#ifdef __CUDACC__
__device__ __forceinline__ __half* out_row(__half* out, const RowPush& push, int row, int N)
{
    if (!push.route) return out + (size_t)row * N;
    const int i = push.route[row];
    const int d = i / push.per;
    return static_cast<__half*>(push.base[d]) + (size_t)(i - d * push.per) * N;
}
#endif

// Expert-parallel gather: after a bounded wait for every peer's in-stamp, the routes of experts [lo, hi)
// from every peer's published id/weight tables (per entries each, at ids_off / w_off of its buffer), as
// local ids (-1 for other ranks' experts) and weights in ids_out / w_out [world * per]
struct EpGather {
    PeerTable peers;
    const uint32_t* in_flags;   // this rank's in_flag[world]
    size_t ids_off, w_off;
    int64_t* ids_out;
    float* w_out;
    int world, per, lo, hi;
    uint32_t stamp;
    int* status;
    uint64_t limit_ns;
};

// Routing permutation results (device pointers; int32 internally)
struct PermBuffers {
    int* counts;         // [E+1]
    int* offsets;        // [E+1] exclusive
    int* token_sorted;   // [N]
    float* weight_sorted;// [N]
    int* route_sorted;   // [N] flat route index of each sorted row
    int* expert_sorted;  // [N] local expert of each sorted row (E for invalid)
    int* route_pos;      // [N] sorted position of each flat route (-1 invalid)
    int4* groups;        // [max_groups] {expert, row_begin, rows, 0} for GEMV experts
    int* n_groups;       // [1]
    int* fat_experts;    // [E] experts routed to the GEMM path
    int* n_fat;          // [1]
    int* seg_hist;       // [nseg][E+1] (multi-CTA path)
    int64_t* counts64;   // optional [E+1] (reference contract, int64)
    int64_t* offsets64;  // optional [E+1]
    int* nrows;          // [1] sorted rows the expert passes process (valid routes, 0 on overflow)
    int* status;         // optional status word (route-capacity overflow)
    int rows_cap;        // capacity of the row buffers (valid routes beyond it: overflow)
};

size_t perm_seg_hist_ints(int N, int E);
bool perm_uses_small(int N, int E);
int max_groups(int N, int E);

cudaError_t launch_permute(const int64_t* ids, const float* weights, int N, int topk, int E,
                           const int32_t* expert_map, int map_len, int fat_threshold,
                           const PermBuffers& pb, cudaStream_t st);
// the expert-parallel gather followed by the permutation of the gathered routes (N = world * per); when
// the single-CTA permutation applies, the gather runs inside it (one launch)
cudaError_t launch_permute_gathered(const EpGather& g, int topk, int E, int fat_threshold, const PermBuffers& pb,
                                    cudaStream_t st);

// rsum (optional, [2 * N] fp32): per sorted row, the sums of the row's stored xt_g / xt_u values
cudaError_t launch_prep(const void* x, int x_dtype, const int* token_sorted, const int* expert_sorted,
                        const int* nrows, int N, const __half* w13_suh, int H, __half* xt_g, __half* xt_u,
                        float* rsum, cudaStream_t st);
cudaError_t launch_router_topk(const void* logits, int logits_dtype, int T, int E, int k, int scoring,
                               int renormalize, int n_group, int topk_group, const float* bias, float scale,
                               int64_t* ids, float* w, cudaStream_t st);
cudaError_t launch_prep_rows(const XRows& x, int x_dtype, const int* token_sorted, const int* expert_sorted,
                             const int* nrows, int N, const __half* w13_suh, int H, __half* xt_g, __half* xt_u,
                             float* rsum, cudaStream_t st);
// publish this rank's tokens, ids and weights, then (last block) stamp in_flag[rank] on every peer;
// `done` is a zeroed int of this rank's control block (reset by the launch)
cudaError_t launch_ep_publish(const void* x, int x_dtype, const int64_t* ids, const float* w, int T, int tcap, int k,
                              int E, int H, __half* X, int* IDS, float* W, const PeerTable& peers, int world, int rank,
                              size_t flag_off, uint32_t stamp, int* done, cudaStream_t st);
// stamp flag_off[rank] on every peer; with nrows, first the drop flag drop_off[rank] (stamp if *nrows == 0)
cudaError_t launch_ep_signal(const PeerTable& peers, int world, int rank, size_t flag_off, uint32_t stamp,
                             const int* nrows, size_t drop_off, cudaStream_t st);
cudaError_t launch_ep_gather(const EpGather& g, cudaStream_t st);
// wait for every rank's out stamp, then out[t] = sum_j w[t, j] * recv[t * k + j] over live routes
cudaError_t launch_ep_combine(const uint32_t* out_flags, const uint32_t* drops, int world, int e_loc, uint32_t stamp,
                              const int* ids, const float* w, int T, int k, int H, const __half* recv, float* out,
                              int* status, uint64_t limit_ns, cudaStream_t st);

// Work lists for an explicit expert list over caller-permuted rows (run_batch semantics):
// int32 counts/offsets copies, expert_sorted (-1 for rows of unlisted experts), GEMV groups of the
// listed experts with <= fat rows (all when fat < 0) and the fat list; *nrows = total_rows.
cudaError_t launch_list_setup(const int32_t* experts, int n_experts, const int64_t* counts64,
                              const int64_t* offsets64, int E, int total_rows, int fat, const PermBuffers& pb,
                              int* nrows, cudaStream_t st);

struct GemvParams {
    int bits;              // bits per weight K of the trellis (2, 3, 4)
    const int4* groups;
    const int* n_groups;
    const int64_t* tab_a;  // gate (gate/up pass) or down trellis addresses [E]
    const int64_t* tab_b;  // up
    const __half* xa;      // gate/up pass: xt_g [rows][K]; down pass: xt_d [rows][K]
    const __half* xb;      // gate/up pass: xt_u
    const __half* svh_a;   // gate/up pass: w13_svh [E][2][N]; down pass: w2_svh [E][N]
    const __half* suh_d;   // gate/up pass: w2_suh [E][N]
    __half* out;           // gate/up pass: xt_d [rows][N]; down pass: y [rows][N]
    RowPush push;          // down pass under expert-parallel push: where each row goes instead of out
    float* partials;       // split-K partials [units][4096]
    int* counters;         // split-K arrival counters [units / split]
    int* status;
    int K, N, split;
    float limit;
    uint32_t k16;          // 65536, passed at run time (keeps the decode multiplies on the FMA pipe)
};

int gemv_units_bound(int groups_bound, int K, int N, int mode, int split);
int gemv_units_alloc(int groups_bound, int H, int I, int split);
size_t gemv_smem_bytes(int bits);
int gemv_stage_rows();   // k-tile rows per pipeline stage: a K split must be a multiple of it
// Decode-GEMV passes first..last (0 = gate/up, 1 = down) of the same row groups in one launch; both
// passes run together only with split 1 (the down units wait for their group's gate/up units).
// sched: gemv_sched_ints(groups_bound) ints of workspace (ticket counters, per-group ready counters),
// zeroed by the launch when `clear`.
int gemv_sched_ints(int groups_bound);
cudaError_t launch_gemv_passes(const GemvParams& gateup, const GemvParams& down, int first, int last, int* sched,
                               int groups_bound, bool clear, cudaStream_t st);

cudaError_t launch_combine(const __half* y, const int* route_pos, const float* w, int T, int topk,
                           int H, int accumulate, float* out, cudaStream_t st);
cudaError_t launch_scatter_add(const __half* y, const int* expert_list, int n_list,
                               const int* counts, const int* offsets, const int* token_sorted,
                               const float* weight_sorted, int H, int rows_bound, float* out,
                               cudaStream_t st);

cudaError_t launch_decode_dense(const void* trellis, int k, int n, int bits, __half* w, cudaStream_t st);
cudaError_t launch_wait_selftest(int* status, uint64_t limit_ns, cudaStream_t st);

int num_sms();

// Programmatic dependent launch for the kernels of one single-GPU layer forward (dsv41_moe_forward):
// while a PdlScope is alive on this thread, launch_k gives each launch the programmatic stream
// serialization attribute, so a kernel can be scheduled while the one before it on the stream finishes
// (its launch and prologue overlap the predecessor's tail). Every kernel launched this way begins with
// griddep_wait() (common.cuh), which returns once the preceding grid has completed and its memory is
// visible, and only then touches data another kernel wrote; launched without the attribute the wait
// returns at once.
#ifndef DSV41_PDL
#define DSV41_PDL 1   // 0: plain launches everywhere
#endif
inline thread_local int g_pdl_scopes = 0;
struct PdlScope {
    PdlScope() { ++g_pdl_scopes; }
    ~PdlScope() { --g_pdl_scopes; }
};
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args... args)
{
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (DSV41_PDL && g_pdl_scopes > 0) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// record a message for dsv41_last_error() and return `code`
int set_error(int code, const char* fmt, ...);

}  // namespace dsv41

struct dsv41_moe_layer;
struct dsv41_moe_options;

namespace dsv41 {

// every argument check of dsv41_moe_forward except the workspace ones (size, NULL, alignment):
// DSV41_OK or the error code, with the message recorded for dsv41_last_error()
int validate_forward(const dsv41_moe_layer* layer, const void* x, int x_dtype, int T, const int64_t* ids,
                     const float* weights, int topk, const dsv41_moe_options* opt, const float* out);

}  // namespace dsv41
