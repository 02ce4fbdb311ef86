// C ABI of the B200 routed-expert MoE path (declared in include/dsv41_b200.h).
//
// dsv41_moe_forward replaces apply_exl3_fused_moe (patches/vllm-exl3-host-dma.patch:203-449,
// wrapped in the reference by ct/ct_vllm.py:181-225): permute -> row transforms -> decode-GEMV
// gate/up (+act, down-input transform) -> decode-GEMV down -> busy-expert GEMM -> combine,
// all on the caller's stream, nothing allocated, no host synchronisation (CUDA-graph safe).
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/dsv41_b200.h"
#include "common.cuh"
#include "gemm.h"
#include "internal.h"

namespace dsv41 {

static thread_local std::string g_last_error;

static int fail(int code, const char* fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int set_error(int code, const char* fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

static int cuda_fail(cudaError_t e, const char* what)
{
    return fail(DSV41_E_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int num_sms()
{
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ------------------------------------------------------------------------------------------
// workspace layout
// ------------------------------------------------------------------------------------------
struct Layout {
    size_t status, counts, offsets, token_sorted, weight_sorted, route_sorted, expert_sorted, route_pos, groups,
        nlists, fat_experts, seg_hist, xt_g, xt_u, xt_d, y, partials, counters, gemm, r_ids, r_w, total;
    int N, E, H, I, split, groups_bound, units_bound, rows;
};

static int auto_split(int N, int E, int H, int I, int requested)
{
    const int r = gemv_stage_rows();
    auto fits = [&](int s) { return s >= 1 && (H / 16) % (s * r) == 0 && (I / 16) % (s * r) == 0; };
    if (requested > 0) return fits(requested) ? requested : 1;
    // split K only while the gate/up units cannot occupy half the SMs: the partial sums and the fixed-order
    // reduction cost more than they gain beyond that (measured on B200, T=1 top-8, 128 units: 108.8 us
    // unsplit, 110.7 split 2, 120.0 split 4, 151 split 8; a lone expert group still splits 8 ways)
    const int groups = N < E ? (N > 0 ? N : 1) : E;
    const long long units = (long long)groups * (I / 128);
    const long long target = num_sms() / 2;
    int s = 1;
    while (units * s < target && s < 8 && fits(s * 2)) s *= 2;
    return s;
}

static Layout make_layout(int T, int topk, int E, int H, int I, int split_req, int fat, int max_routes = 0)
{
    Layout L{};
    L.N = T * topk;
    L.E = E;
    L.H = H;
    L.I = I;
    // row buffers hold the valid (locally routed) rows only; max_routes bounds them when the caller knows
    L.rows = (max_routes > 0 && max_routes < L.N) ? max_routes : L.N;
    L.split = auto_split(L.rows, E, H, I, split_req);
    L.groups_bound = max_groups(L.rows, E);
    L.units_bound = gemv_units_alloc(L.groups_bound, H, I, L.split);
    const size_t N = (size_t)(L.N > 0 ? L.N : 1), E1 = (size_t)E + 1;
    const size_t R = (size_t)(L.rows > 0 ? L.rows : 1);
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = align_up(o + bytes, 256);
        return at;
    };
    L.status = take(256);
    L.counts = take(E1 * 4);
    L.offsets = take(E1 * 4);
    L.token_sorted = take(N * 4);
    L.weight_sorted = take(N * 4);
    L.route_sorted = take(N * 4);
    L.expert_sorted = take(N * 4);
    L.route_pos = take(N * 4);
    L.groups = take((size_t)L.groups_bound * 16);
    L.nlists = take(16);
    L.fat_experts = take(E1 * 4);
    L.seg_hist = take(perm_seg_hist_ints(L.N, E) * 4 + 4);
    L.xt_g = take(R * H * 2);
    L.xt_u = take(R * H * 2);
    L.xt_d = take(R * I * 2);
    L.y = take(R * H * 2);
    L.partials = take(L.split > 1 ? (size_t)L.units_bound * 4096 * 4 : 16);
    L.counters = take((size_t)(L.units_bound / L.split + 1 + gemv_sched_ints(L.groups_bound)) * 4);
    L.gemm = take(fat >= 0 ? gemm_scratch_bytes(L.rows, E, H, I) : 16);
    L.r_ids = take(N * 8);   // router output of dsv41_moe_forward_logits
    L.r_w = take(N * 4);
    L.total = o;
    return L;
}

template <typename T>
static T* at(void* ws, size_t off)
{
    return reinterpret_cast<T*>(static_cast<uint8_t*>(ws) + off);
}

// where the row transform leaves the rows' input sums for the busy-expert GEMM (its affine weight codes),
// or NULL when no expert of the call can take the GEMM path
static float* gemm_sums(void* ws, const Layout& L, int fat)
{
    return (fat >= 0 && L.rows > fat) ? gemm_row_sums(at<uint8_t>(ws, L.gemm), L.rows, L.E) : nullptr;
}

static PermBuffers perm_buffers(void* ws, const Layout& L)
{
    PermBuffers pb{};
    pb.counts = at<int>(ws, L.counts);
    pb.offsets = at<int>(ws, L.offsets);
    pb.token_sorted = at<int>(ws, L.token_sorted);
    pb.weight_sorted = at<float>(ws, L.weight_sorted);
    pb.route_sorted = at<int>(ws, L.route_sorted);
    pb.expert_sorted = at<int>(ws, L.expert_sorted);
    pb.route_pos = at<int>(ws, L.route_pos);
    pb.groups = at<int4>(ws, L.groups);
    pb.n_groups = at<int>(ws, L.nlists);
    pb.n_fat = at<int>(ws, L.nlists) + 1;
    pb.fat_experts = at<int>(ws, L.fat_experts);
    pb.seg_hist = at<int>(ws, L.seg_hist);
    pb.nrows = at<int>(ws, L.nlists) + 2;
    pb.status = at<int>(ws, L.status);
    pb.rows_cap = L.rows;
    return pb;
}

// ------------------------------------------------------------------------------------------
// expert parallelism over peer memory: layout of each rank's shared buffer (same on all ranks)
// ------------------------------------------------------------------------------------------
constexpr size_t kCtrlInFlags = 0;     // uint32 in_flag[kMaxPeers]: step stamps written by peers
constexpr size_t kCtrlOutFlags = 64;   // uint32 out_flag[kMaxPeers]
constexpr size_t kCtrlStatus = 128;    // int status of the exchange waits
constexpr size_t kCtrlOutDrop = 160;   // uint32 out_drop[kMaxPeers]: stamp of a step whose routes a peer dropped
constexpr size_t kCtrlPubDone = 224;   // int: blocks of this rank's publish launch that finished

struct PeerLayout {
    size_t ctrl, x[2], ids[2], w[2], ids_loc[2], w_loc[2], recv[2], ws, total;
    Layout L;  // the local forward over world * tokens_cap tokens
};

static PeerLayout make_peer_layout(int world, int tcap, int k, int e_loc, int H, int I, int fat)
{
    PeerLayout P{};
    P.L = make_layout(world * tcap, k, e_loc, H, I, 0, fat);
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = align_up(o + bytes, 256);
        return at;
    };
    const size_t n = (size_t)tcap * k, nl = (size_t)world * tcap * k;
    P.ctrl = take(256);
    for (int p = 0; p < 2; ++p) {
        P.x[p] = take((size_t)tcap * H * 2);
        P.ids[p] = take(n * 4);
        P.w[p] = take(n * 4);
        P.ids_loc[p] = take(nl * 8);
        P.w_loc[p] = take(nl * 4);
        P.recv[p] = take(n * H * 2);   // expert output rows of this rank's routes, slot t * k + j
    }
    // the local forward's workspace: only this rank's own kernels touch it, in stream order, so one copy
    // serves both parities (peers read x / ids / w and write recv, never the workspace)
    P.ws = take(P.L.total);
    P.total = o;
    return P;
}

static int check_group(const dsv41_ep_peer_group* g)
{
    if (!g) return fail(DSV41_E_INVALID, "group is NULL");
    if (g->world < 1 || g->world > kMaxPeers || g->rank < 0 || g->rank >= g->world)
        return fail(DSV41_E_INVALID, "rank %d / world %d out of range (world 1..%d)", g->rank, g->world, kMaxPeers);
    if (g->num_global_experts <= 0 || g->num_global_experts % g->world)
        return fail(DSV41_E_INVALID, "%d experts do not shard over %d ranks", g->num_global_experts, g->world);
    if (g->tokens_cap <= 0) return fail(DSV41_E_INVALID, "tokens_cap %d", g->tokens_cap);
    for (int d = 0; d < g->world; ++d)
        if (!g->bases[d]) return fail(DSV41_E_INVALID, "base of rank %d is NULL", d);
    if (g->wait_limit_us < 0 || g->wait_limit_us > 2000000)
        return fail(DSV41_E_INVALID, "wait_limit_us %d out of range (0 = default, 1..2000000)", g->wait_limit_us);
    return DSV41_OK;
}

// limit of each wait for the peers' step stamps
static uint64_t peer_wait_limit_ns(const dsv41_ep_peer_group* g)
{
    return g->wait_limit_us > 0 ? (uint64_t)g->wait_limit_us * 1000ull : kWaitLimitNs;
}

// run_batch semantics: listed experts with more rows than this use the tcgen05 GEMM, the rest the
// decode GEMV (the reference's FAT_EXPERT_THRESHOLD as deployed, docker/entrypoint.sh:69)
constexpr int kExpertGemmFat = 32;

static int layer_bits(const dsv41_moe_layer* layer) { return layer->bits ? layer->bits : 3; }

// the kernels move rows with 16- and 32-byte vector accesses and carve the workspace at 256-byte offsets
static bool aligned_to(const void* p, size_t a) { return reinterpret_cast<uintptr_t>(p) % a == 0; }
static int check_alignment(const void* x, const void* out, const void* workspace)
{
    if (x && !aligned_to(x, 16)) return fail(DSV41_E_INVALID, "activations must be 16-byte aligned");
    if (out && !aligned_to(out, 16)) return fail(DSV41_E_INVALID, "out must be 16-byte aligned");
    if (workspace && !aligned_to(workspace, 256)) return fail(DSV41_E_INVALID, "workspace must be 256-byte aligned");
    return DSV41_OK;
}

static int check_layer(const dsv41_moe_layer* layer)
{
    if (!layer) return fail(DSV41_E_INVALID, "layer is NULL");
    const int E = layer->num_experts, H = layer->hidden, I = layer->intermediate;
    if (E <= 0 || E > kMaxExperts) return fail(DSV41_E_INVALID, "num_experts %d out of range (1..%d)", E, kMaxExperts);
    if (H <= 0 || I <= 0 || H % 256 || I % 256)
        return fail(DSV41_E_INVALID, "hidden %d / intermediate %d must be positive multiples of 256", H, I);
    if (!layer->gate_ptrs || !layer->up_ptrs || !layer->down_ptrs || !layer->w13_suh || !layer->w13_svh ||
        !layer->w2_suh || !layer->w2_svh)
        return fail(DSV41_E_INVALID, "layer has a NULL tensor pointer");
    if (layer->bits != 0 && (layer->bits < 2 || layer->bits > 4))
        return fail(DSV41_E_INVALID, "bits %d per weight (2, 3 or 4)", layer->bits);
    return DSV41_OK;
}

int validate_forward(const dsv41_moe_layer* layer, const void* x, int x_dtype, int T, const int64_t* ids,
                     const float* weights, int topk, const dsv41_moe_options* opt, const float* out)
{
    int rc = check_layer(layer);
    if (rc) return rc;
    if (T < 0 || topk <= 0) return fail(DSV41_E_INVALID, "bad T=%d topk=%d", T, topk);
    if (x_dtype < DSV41_DTYPE_F16 || x_dtype > DSV41_DTYPE_F32) return fail(DSV41_E_INVALID, "bad x_dtype %d", x_dtype);
    if (T > 0 && (!x || !ids || !weights || !out)) return fail(DSV41_E_INVALID, "NULL input/output pointer");
    if ((rc = check_alignment(x, out, nullptr))) return rc;
    if (opt && opt->expert_map && opt->map_len <= 0)
        return fail(DSV41_E_INVALID, "expert_map given with map_len %d", opt->map_len);
    if (opt && opt->max_routes < 0) return fail(DSV41_E_INVALID, "max_routes %d < 0", opt->max_routes);
    return DSV41_OK;
}

// ------------------------------------------------------------------------------------------
// optional stage timing (profiling): CUDA events at the forward's stage boundaries
// ------------------------------------------------------------------------------------------
struct StageTimer {
    bool enabled = false;
    int device = -1;
    int calls = 0;      // recorded calls
    bool active = false;  // current call records
    cudaEvent_t ev[DSV41_TIMING_MAX_CALLS][DSV41_N_STAGES + 1];
};
static StageTimer g_timer;

static void timer_begin(cudaStream_t st)
{
    g_timer.active = false;
    if (!g_timer.enabled || g_timer.calls >= DSV41_TIMING_MAX_CALLS) return;
    cudaStreamCaptureStatus cs;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != g_timer.device) return;
    g_timer.active = true;
    cudaEventRecord(g_timer.ev[g_timer.calls][0], st);
}

static void timer_mark(cudaStream_t st, int boundary)
{
    if (g_timer.active) cudaEventRecord(g_timer.ev[g_timer.calls][boundary], st);
}

static void timer_end(cudaStream_t st)
{
    if (!g_timer.active) return;
    cudaEventRecord(g_timer.ev[g_timer.calls][DSV41_N_STAGES], st);
    g_timer.calls++;
    g_timer.active = false;
}

// the decode-GEMV's ticket and ready counters within the workspace's counter block (after the split-K
// arrival counters)
static int* gemv_sched(int* counters, int groups_bound, int H, int I, int split)
{
    return counters + gemv_units_alloc(groups_bound, H, I, split) / split + 1;
}

// gate/up pass (GEMV groups, then GEMM for fat experts) and down pass over prepared rows; with
// sched_cleared the caller has zeroed the decode-GEMV counters (and the split-K ones) already
static cudaError_t run_expert_passes(const dsv41_moe_layer* layer, const PermBuffers& pb, __half* xt_g, __half* xt_u,
                                     __half* xt_d, __half* y, float* partials, int* counters, int* status, int split,
                                     int groups_bound, int rows_bound, float limit, int fat, uint8_t* gemm_scratch,
                                     cudaStream_t st, const RowPush& push = RowPush{}, bool sched_cleared = false)
{
    const int H = layer->hidden, I = layer->intermediate;
    // an expert takes the GEMM path with more than `fat` rows; no expert has more rows than the call's
    // row bound, so small calls (e.g. decode with T * topk <= fat) launch no GEMM kernels at all
    const bool gemm_on = fat >= 0 && rows_bound > fat;
    cudaError_t err;
    // the split-K arrival counters, then the GEMV launches' ticket and ready counters
    const int n_split_counters = gemv_units_alloc(groups_bound, H, I, split) / split + 1;
    int* sched = gemv_sched(counters, groups_bound, H, I, split);
    if (split > 1 && !sched_cleared) {
        const size_t n = (size_t)(n_split_counters + gemv_sched_ints(groups_bound)) * 4;
        if ((err = cudaMemsetAsync(counters, 0, n, st)) != cudaSuccess) return err;
    }
    GemmArgs ga{};
    ga.layer = layer;
    ga.fat_experts = pb.fat_experts;
    ga.n_fat = pb.n_fat;
    ga.counts = pb.counts;
    ga.offsets = pb.offsets;
    ga.xt_g = xt_g;
    ga.xt_u = xt_u;
    ga.xt_d = xt_d;
    ga.y = y;
    ga.push = push;
    ga.rows_bound = rows_bound;
    ga.limit = limit;
    ga.scratch = gemm_scratch;
    ga.status = status;
    GemvParams gp{};
    gp.bits = layer_bits(layer);
    gp.groups = pb.groups;
    gp.n_groups = pb.n_groups;
    gp.partials = partials;
    gp.counters = counters;
    gp.status = status;
    gp.split = split;
    gp.limit = limit;
    gp.k16 = 65536u;
    gp.tab_a = layer->gate_ptrs;
    gp.tab_b = layer->up_ptrs;
    gp.xa = xt_g;
    gp.xb = xt_u;
    gp.svh_a = static_cast<const __half*>(layer->w13_svh);
    gp.suh_d = static_cast<const __half*>(layer->w2_suh);
    gp.out = xt_d;
    gp.K = H;
    gp.N = I;
    GemvParams gd = gp;
    gd.tab_a = layer->down_ptrs;
    gd.tab_b = nullptr;
    gd.xa = xt_d;
    gd.xb = nullptr;
    gd.svh_a = static_cast<const __half*>(layer->w2_svh);
    gd.suh_d = nullptr;
    gd.out = y;
    gd.push = push;
    gd.K = I;
    gd.N = H;
    if (split == 1) {
        // both decode-GEMV passes in one launch (stage "gemv_gateup"; "gemv_down" stays empty)
        if ((err = launch_gemv_passes(gp, gd, 0, 1, sched, groups_bound, !sched_cleared, st)) != cudaSuccess)
            return err;
        timer_mark(st, 3);
        if (gemm_on && (err = launch_gemm_gateup(ga, st)) != cudaSuccess) return err;
        timer_mark(st, 4);
        timer_mark(st, 5);
    } else {
        if ((err = launch_gemv_passes(gp, gd, 0, 0, sched, groups_bound, false, st)) != cudaSuccess) return err;
        timer_mark(st, 3);
        if (gemm_on && (err = launch_gemm_gateup(ga, st)) != cudaSuccess) return err;
        timer_mark(st, 4);
        if ((err = launch_gemv_passes(gp, gd, 1, 1, sched, groups_bound, false, st)) != cudaSuccess) return err;
        timer_mark(st, 5);
    }
    if (gemm_on && (err = launch_gemm_down(ga, st)) != cudaSuccess) return err;
    timer_mark(st, 6);
    return cudaSuccess;
}

}  // namespace dsv41

using namespace dsv41;

extern "C" {

const char* dsv41_last_error(void) { return g_last_error.c_str(); }

int dsv41_abi_version(void) { return DSV41_ABI_VERSION; }

const char* dsv41_build_info(void)
{
    return "dsv41_b200: sm_100a; EXL3 mul1 K=3; decode-GEMV mma.m16n8k16 (register-decoded B), "
           "tcgen05 grouped GEMM; nvcc " DSV41_NVCC_VERSION;
}

int dsv41_moe_workspace_size(int32_t T, int32_t topk, int32_t num_experts, int32_t hidden, int32_t intermediate,
                             const dsv41_moe_options* opt, size_t* bytes)
{
    if (!bytes) return fail(DSV41_E_INVALID, "bytes is NULL");
    if (T < 0 || topk <= 0 || num_experts <= 0 || num_experts > kMaxExperts || hidden <= 0 || intermediate <= 0 ||
        hidden % 256 || intermediate % 256)
        return fail(DSV41_E_INVALID, "bad sizes T=%d topk=%d E=%d H=%d I=%d", T, topk, num_experts, hidden,
                    intermediate);
    const int split = opt ? opt->split_k : 0;
    // busy experts are only possible with more tokens than the threshold (the reference's
    // fat_possible = tokens > FAT_EXPERT_THRESHOLD, patch:245); otherwise everything is GEMV
    const int fat = (opt && opt->fat_threshold >= 0 && T > opt->fat_threshold) ? opt->fat_threshold : -1;
    const int max_routes = opt ? opt->max_routes : 0;
    if (max_routes < 0) return fail(DSV41_E_INVALID, "max_routes %d < 0", max_routes);
    *bytes = make_layout(T, topk, num_experts, hidden, intermediate, split, fat, max_routes).total;
    return DSV41_OK;
}

int dsv41_moe_forward(const dsv41_moe_layer* layer, const void* x, int32_t x_dtype, int32_t T, const int64_t* ids,
                      const float* weights, int32_t topk, const dsv41_moe_options* opt, float* out, void* workspace,
                      size_t workspace_bytes, void* stream)
{
    int rc = validate_forward(layer, x, x_dtype, T, ids, weights, topk, opt, out);
    if (rc) return rc;
    if (!workspace) return fail(DSV41_E_INVALID, "workspace is NULL");
    if ((rc = check_alignment(nullptr, nullptr, workspace))) return rc;
    const int E = layer->num_experts, H = layer->hidden, I = layer->intermediate;
    const dsv41_moe_options dflt{-1, 0.0f, nullptr, 0, 0, 0};
    const dsv41_moe_options& o = opt ? *opt : dflt;
    const int fat = (o.fat_threshold >= 0 && T > o.fat_threshold) ? o.fat_threshold : -1;  // fat_possible
    const Layout L = make_layout(T, topk, E, H, I, o.split_k, fat, o.max_routes);
    if (workspace_bytes < L.total)
        return fail(DSV41_E_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes, L.total);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (T == 0) return DSV41_OK;
    cudaError_t err;
    const PermBuffers pb = perm_buffers(workspace, L);
    int* status = at<int>(workspace, L.status);
    // the decode-GEMV's counters (split-K arrivals, tickets, ready counts) are cleared before the first
    // kernel, so the chain of kernels below has no memset node between two kernels and every launch of it
    // can be programmatic
    int* counters = at<int>(workspace, L.counters);
    {
        int* from = L.split == 1 ? gemv_sched(counters, L.groups_bound, H, I, 1) : counters;
        int* to = gemv_sched(counters, L.groups_bound, H, I, L.split) + gemv_sched_ints(L.groups_bound);
        if ((err = cudaMemsetAsync(from, 0, (size_t)(to - from) * 4, st)) != cudaSuccess)
            return cuda_fail(err, "clear the decode-GEMV counters");
    }
    const PdlScope pdl;
    timer_begin(st);
    if ((err = launch_permute(ids, weights, L.N, topk, E, o.expert_map, o.map_len, fat, pb, st)) !=
        cudaSuccess)
        return cuda_fail(err, "permute");
    timer_mark(st, 1);
    __half* xt_g = at<__half>(workspace, L.xt_g);
    __half* xt_u = at<__half>(workspace, L.xt_u);
    __half* xt_d = at<__half>(workspace, L.xt_d);
    __half* y = at<__half>(workspace, L.y);
    if ((err = launch_prep(x, x_dtype, pb.token_sorted, pb.expert_sorted, pb.nrows, L.rows,
                           static_cast<const __half*>(layer->w13_suh), H, xt_g, xt_u,
                           gemm_sums(workspace, L, fat), st)) != cudaSuccess)
        return cuda_fail(err, "prep");
    timer_mark(st, 2);
    if ((err = run_expert_passes(layer, pb, xt_g, xt_u, xt_d, y, at<float>(workspace, L.partials), counters, status,
                                 L.split, L.groups_bound, L.rows, o.limit, fat, at<uint8_t>(workspace, L.gemm), st,
                                 RowPush{}, /*sched_cleared=*/true)) != cudaSuccess)
        return cuda_fail(err, "expert passes");
    if ((err = launch_combine(y, pb.route_pos, weights, T, topk, H, 0, out, st)) != cudaSuccess)
        return cuda_fail(err, "combine");
    timer_end(st);
    return DSV41_OK;
}

int dsv41_ep_peer_buffer_size(const dsv41_ep_peer_group* g, const dsv41_moe_layer* local_layer, int32_t topk,
                               int32_t fat_threshold, size_t* bytes)
{
    int rc = check_group(g);
    if (rc) return rc;
    if ((rc = check_layer(local_layer))) return rc;
    if (!bytes || topk <= 0) return fail(DSV41_E_INVALID, "bad topk %d or NULL bytes", topk);
    if (local_layer->num_experts != g->num_global_experts / g->world)
        return fail(DSV41_E_INVALID, "local layer has %d experts, expected %d", local_layer->num_experts,
                    g->num_global_experts / g->world);
    const int tl = g->world * g->tokens_cap;
    const int fat = (fat_threshold >= 0 && tl > fat_threshold) ? fat_threshold : -1;
    *bytes = make_peer_layout(g->world, g->tokens_cap, topk, local_layer->num_experts, local_layer->hidden,
                              local_layer->intermediate, fat).total;
    return DSV41_OK;
}

int dsv41_ep_peer_alloc(size_t bytes, void** base, void* ipc_handle)
{
    if (!base || !ipc_handle || bytes == 0) return fail(DSV41_E_INVALID, "bad arguments");
    *base = nullptr;
    cudaError_t err = cudaMalloc(base, bytes);
    if (err != cudaSuccess) return cuda_fail(err, "peer buffer cudaMalloc");
    if ((err = cudaMemset(*base, 0, bytes)) != cudaSuccess) {
        cudaFree(*base);
        *base = nullptr;
        return cuda_fail(err, "peer buffer clear");
    }
    cudaIpcMemHandle_t h;
    if ((err = cudaIpcGetMemHandle(&h, *base)) != cudaSuccess) {
        cudaFree(*base);
        *base = nullptr;
        return cuda_fail(err, "cudaIpcGetMemHandle");
    }
    static_assert(sizeof(h) == DSV41_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(ipc_handle, &h, sizeof(h));
    return DSV41_OK;
}

int dsv41_ep_peer_open(const void* ipc_handle, void** peer_base)
{
    if (!ipc_handle || !peer_base) return fail(DSV41_E_INVALID, "NULL pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    cudaError_t err = cudaIpcOpenMemHandle(peer_base, h, cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) return cuda_fail(err, "cudaIpcOpenMemHandle");
    return DSV41_OK;
}

int dsv41_ep_peer_close(void* peer_base)
{
    if (!peer_base) return DSV41_OK;
    cudaError_t err = cudaIpcCloseMemHandle(peer_base);
    if (err != cudaSuccess) return cuda_fail(err, "cudaIpcCloseMemHandle");
    return DSV41_OK;
}

int dsv41_ep_peer_free(void* base)
{
    if (!base) return DSV41_OK;
    cudaError_t err = cudaFree(base);
    if (err != cudaSuccess) return cuda_fail(err, "peer buffer cudaFree");
    return DSV41_OK;
}

int dsv41_ep_peer_forward(const dsv41_moe_layer* local_layer, const dsv41_ep_peer_group* g, uint32_t step,
                          const void* x, int32_t x_dtype, int32_t T, const int64_t* ids, const float* weights,
                          int32_t topk, float limit, int32_t fat_threshold, float* out, void* stream)
{
    int rc = check_group(g);
    if (rc) return rc;
    if ((rc = check_layer(local_layer))) return rc;
    const int world = g->world, rank = g->rank, tcap = g->tokens_cap, k = topk;
    const int E = g->num_global_experts, e_loc = E / world, H = local_layer->hidden, I = local_layer->intermediate;
    if (local_layer->num_experts != e_loc)
        return fail(DSV41_E_INVALID, "local layer has %d experts, expected %d", local_layer->num_experts, e_loc);
    if (T < 0 || T > tcap || k <= 0) return fail(DSV41_E_INVALID, "T=%d (tokens_cap %d), topk=%d", T, tcap, k);
    if (H > 8192) return fail(DSV41_E_INVALID, "expert-parallel peer path supports hidden <= 8192, got %d", H);
    if (x_dtype < DSV41_DTYPE_F16 || x_dtype > DSV41_DTYPE_F32) return fail(DSV41_E_INVALID, "bad x_dtype %d", x_dtype);
    if (T > 0 && (!x || !ids || !weights || !out)) return fail(DSV41_E_INVALID, "NULL input/output pointer");
    if ((rc = check_alignment(x, out, nullptr))) return rc;
    const int tl = world * tcap;
    const int fat = (fat_threshold >= 0 && tl > fat_threshold) ? fat_threshold : -1;
    const PeerLayout P = make_peer_layout(world, tcap, k, e_loc, H, I, fat);
    const Layout& L = P.L;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int p = (int)(step & 1u);
    const uint32_t stamp = step + 1u;
    PeerTable peers{};
    for (int d = 0; d < world; ++d) peers.base[d] = g->bases[d];
    uint8_t* own = static_cast<uint8_t*>(g->bases[rank]);
    int* xstatus = reinterpret_cast<int*>(own + P.ctrl + kCtrlStatus);
    void* ws = own + P.ws;
    cudaError_t err;
    // the decode-GEMV's counters cleared before the first kernel (no memset node inside the kernel chain,
    // whose launches are programmatic as in dsv41_moe_forward)
    {
        int* counters = at<int>(ws, L.counters);
        int* from = L.split == 1 ? gemv_sched(counters, L.groups_bound, H, I, 1) : counters;
        int* to = gemv_sched(counters, L.groups_bound, H, I, L.split) + gemv_sched_ints(L.groups_bound);
        if ((err = cudaMemsetAsync(from, 0, (size_t)(to - from) * 4, st)) != cudaSuccess)
            return cuda_fail(err, "clear the decode-GEMV counters");
    }
    const PdlScope pdl;
    timer_begin(st);  // stages as dsv41_moe_forward; permute includes publish + gather, combine the wait + sum
    // 1. publish this rank's tokens; the launch's last block stamps in_flag[rank] on every peer
    if ((err = launch_ep_publish(x, x_dtype, ids, weights, T, tcap, k, E, H, reinterpret_cast<__half*>(own + P.x[p]),
                                 reinterpret_cast<int*>(own + P.ids[p]), reinterpret_cast<float*>(own + P.w[p]), peers,
                                 world, rank, P.ctrl + kCtrlInFlags, stamp,
                                 reinterpret_cast<int*>(own + P.ctrl + kCtrlPubDone), st)) != cudaSuccess)
        return cuda_fail(err, "ep publish");
    // 2. every peer's routes that land on this rank's experts (after a bounded wait for the in-stamps),
    // 3. permuted: one launch when the single-CTA permutation applies
    EpGather eg{};
    eg.peers = peers;
    eg.in_flags = reinterpret_cast<const uint32_t*>(own + P.ctrl + kCtrlInFlags);
    eg.ids_off = P.ids[p];
    eg.w_off = P.w[p];
    eg.ids_out = reinterpret_cast<int64_t*>(own + P.ids_loc[p]);
    eg.w_out = reinterpret_cast<float*>(own + P.w_loc[p]);
    eg.world = world;
    eg.per = tcap * k;
    eg.lo = rank * e_loc;
    eg.hi = (rank + 1) * e_loc;
    eg.stamp = stamp;
    eg.status = xstatus;
    eg.limit_ns = peer_wait_limit_ns(g);
    const PermBuffers pb = perm_buffers(ws, L);
    if ((err = launch_permute_gathered(eg, k, e_loc, fat, pb, st)) != cudaSuccess)
        return cuda_fail(err, "ep gather + permute");
    timer_mark(st, 1);
    XRows xr{};
    for (int d = 0; d < world; ++d) xr.base[d] = static_cast<const uint8_t*>(g->bases[d]) + P.x[p];
    xr.per = tcap;
    xr.n = world;
    if ((err = launch_prep_rows(xr, DSV41_DTYPE_F16, pb.token_sorted, pb.expert_sorted, pb.nrows, L.rows,
                                static_cast<const __half*>(local_layer->w13_suh), H, at<__half>(ws, L.xt_g),
                                at<__half>(ws, L.xt_u), gemm_sums(ws, L, fat), st)) != cudaSuccess)
        return cuda_fail(err, "prep");
    timer_mark(st, 2);
    // 4. the expert passes; the down pass stores each output row into its token owner's receive slot
    RowPush push{};
    for (int d = 0; d < world; ++d) push.base[d] = static_cast<uint8_t*>(g->bases[d]) + P.recv[p];
    push.route = pb.route_sorted;
    push.per = tcap * k;
    if ((err = run_expert_passes(local_layer, pb, at<__half>(ws, L.xt_g), at<__half>(ws, L.xt_u),
                                 at<__half>(ws, L.xt_d), at<__half>(ws, L.y), at<float>(ws, L.partials),
                                 at<int>(ws, L.counters), at<int>(ws, L.status), L.split, L.groups_bound, L.rows, limit,
                                 fat, at<uint8_t>(ws, L.gemm), st, push, /*sched_cleared=*/true)) != cudaSuccess)
        return cuda_fail(err, "expert passes");
    // 5. outputs delivered: drop flag + out stamp on every peer; 6. sum this rank's routes from its slots
    if ((err = launch_ep_signal(peers, world, rank, P.ctrl + kCtrlOutFlags, stamp, pb.nrows, P.ctrl + kCtrlOutDrop,
                                st)) != cudaSuccess)
        return cuda_fail(err, "ep signal out");
    if (T > 0 &&
        (err = launch_ep_combine(reinterpret_cast<const uint32_t*>(own + P.ctrl + kCtrlOutFlags),
                                 reinterpret_cast<const uint32_t*>(own + P.ctrl + kCtrlOutDrop), world, e_loc, stamp,
                                 reinterpret_cast<const int*>(own + P.ids[p]), reinterpret_cast<const float*>(own + P.w[p]),
                                 T, k, H, reinterpret_cast<const __half*>(own + P.recv[p]), out, xstatus,
                                 peer_wait_limit_ns(g), st)) != cudaSuccess)
        return cuda_fail(err, "ep combine");
    timer_end(st);
    return DSV41_OK;
}

int dsv41_ep_peer_read_status(const dsv41_ep_peer_group* g, const dsv41_moe_layer* local_layer, int32_t topk,
                              int32_t fat_threshold, void* stream, int32_t* status)
{
    int rc = check_group(g);
    if (rc) return rc;
    if ((rc = check_layer(local_layer))) return rc;
    if (!status) return fail(DSV41_E_INVALID, "status is NULL");
    const int tl = g->world * g->tokens_cap;
    const int fat = (fat_threshold >= 0 && tl > fat_threshold) ? fat_threshold : -1;
    const PeerLayout P = make_peer_layout(g->world, g->tokens_cap, topk, local_layer->num_experts, local_layer->hidden,
                                          local_layer->intermediate, fat);
    uint8_t* own = static_cast<uint8_t*>(g->bases[g->rank]);
    int worst = 0;
    const size_t words[2] = {P.ctrl + kCtrlStatus, P.ws + P.L.status};
    for (size_t off : words) {
        int32_t v = 0;
        if ((rc = dsv41_read_status(own + off, stream, &v))) return rc;
        if (v > worst) worst = v;
    }
    *status = worst;
    return DSV41_OK;
}

static int check_router(const dsv41_router_options* r, int E, int k)
{
    if (!r) return fail(DSV41_E_INVALID, "router options are NULL");
    if (E <= 0 || E > 1024) return fail(DSV41_E_INVALID, "router supports 1..1024 experts, got %d", E);
    if (k <= 0 || k > 32 || k > E) return fail(DSV41_E_INVALID, "router topk %d out of range (1..min(32, E))", k);
    if (r->scoring != DSV41_ROUTER_SOFTMAX && r->scoring != DSV41_ROUTER_SIGMOID)
        return fail(DSV41_E_INVALID, "bad scoring %d", r->scoring);
    const int ng = r->num_expert_group;
    if (ng > 1) {
        if (ng > 32 || E % ng) return fail(DSV41_E_INVALID, "num_expert_group %d must divide E=%d and be <= 32", ng, E);
        if (r->topk_group < 1 || r->topk_group > ng)
            return fail(DSV41_E_INVALID, "topk_group %d out of range 1..%d", r->topk_group, ng);
        if (k > r->topk_group * (E / ng)) return fail(DSV41_E_INVALID, "topk %d exceeds the competing experts", k);
    }
    return DSV41_OK;
}

int dsv41_router_topk(const void* logits, int32_t logits_dtype, int32_t T, int32_t num_experts, int32_t topk,
                      const dsv41_router_options* r, int64_t* ids, float* weights, void* stream)
{
    int rc = check_router(r, num_experts, topk);
    if (rc) return rc;
    if (T < 0 || logits_dtype < DSV41_DTYPE_F16 || logits_dtype > DSV41_DTYPE_F32)
        return fail(DSV41_E_INVALID, "bad T=%d or logits dtype %d", T, logits_dtype);
    if (T > 0 && (!logits || !ids || !weights)) return fail(DSV41_E_INVALID, "NULL pointer");
    cudaError_t err = launch_router_topk(logits, logits_dtype, T, num_experts, topk, r->scoring, r->renormalize,
                                         r->num_expert_group > 1 ? r->num_expert_group : 1, r->topk_group,
                                         r->correction_bias, r->routed_scaling_factor, ids, weights,
                                         static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "router top-k");
    return DSV41_OK;
}

int dsv41_moe_forward_logits(const dsv41_moe_layer* layer, const void* x, int32_t x_dtype, int32_t T,
                             const void* logits, int32_t logits_dtype, const dsv41_router_options* r, int32_t topk,
                             const dsv41_moe_options* opt, float* out, int64_t* ids_out, float* weights_out,
                             void* workspace, size_t workspace_bytes, void* stream)
{
    int rc = check_layer(layer);
    if (rc) return rc;
    if ((rc = check_router(r, layer->num_experts, topk))) return rc;
    if (!workspace) return fail(DSV41_E_INVALID, "workspace is NULL");
    if ((rc = check_alignment(x, out, workspace))) return rc;
    const dsv41_moe_options dflt{-1, 0.0f, nullptr, 0, 0, 0};
    const dsv41_moe_options& o = opt ? *opt : dflt;
    const int fat = (o.fat_threshold >= 0 && T > o.fat_threshold) ? o.fat_threshold : -1;
    const Layout L = make_layout(T, topk, layer->num_experts, layer->hidden, layer->intermediate, o.split_k, fat,
                                 o.max_routes);
    if (workspace_bytes < L.total)
        return fail(DSV41_E_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes, L.total);
    if (T == 0) return DSV41_OK;
    int64_t* ids = ids_out ? ids_out : at<int64_t>(workspace, L.r_ids);
    float* w = weights_out ? weights_out : at<float>(workspace, L.r_w);
    if ((rc = dsv41_router_topk(logits, logits_dtype, T, layer->num_experts, topk, r, ids, w, stream))) return rc;
    return dsv41_moe_forward(layer, x, x_dtype, T, ids, w, topk, opt, out, workspace, workspace_bytes, stream);
}

size_t dsv41_permute_workspace_size(int32_t T, int32_t topk, int32_t num_experts)
{
    const int N = T * topk;
    const size_t E1 = (size_t)num_experts + 1, n = (size_t)(N > 0 ? N : 1);
    // counts, offsets, token/weight/route/expert sorted, route_pos, groups, lists, fat, seg_hist
    return align_up(E1 * 4, 256) * 3 + align_up(n * 4, 256) * 5 + align_up((size_t)max_groups(N, num_experts) * 16, 256) +
           256 + align_up(perm_seg_hist_ints(N, num_experts) * 4 + 4, 256) + 4096;
}

int dsv41_permute(const int64_t* ids, const float* weights, int32_t T, int32_t topk, int32_t num_experts,
                  const int32_t* expert_map, int32_t map_len, int64_t* counts, int64_t* offsets, int32_t* token_sorted,
                  float* weight_sorted, int32_t* route_sorted, int32_t* route_pos, void* workspace,
                  size_t workspace_bytes, void* stream)
{
    if (T < 0 || topk <= 0 || num_experts <= 0 || num_experts > kMaxExperts)
        return fail(DSV41_E_INVALID, "bad sizes T=%d topk=%d E=%d", T, topk, num_experts);
    if (T > 0 && !ids) return fail(DSV41_E_INVALID, "ids is NULL");
    if (expert_map && map_len <= 0) return fail(DSV41_E_INVALID, "expert_map given with map_len %d", map_len);
    if (!workspace || workspace_bytes < dsv41_permute_workspace_size(T, topk, num_experts))
        return fail(DSV41_E_WORKSPACE, "permute workspace too small");
    if (int rc = check_alignment(nullptr, nullptr, workspace)) return rc;
    const int N = T * topk;
    const size_t E1 = (size_t)num_experts + 1, n = (size_t)(N > 0 ? N : 1);
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t a = o;
        o = align_up(o + bytes, 256);
        return a;
    };
    PermBuffers pb{};
    pb.counts = at<int>(workspace, take(E1 * 4));
    pb.offsets = at<int>(workspace, take(E1 * 4));
    pb.fat_experts = at<int>(workspace, take(E1 * 4));
    pb.token_sorted = token_sorted ? token_sorted : at<int>(workspace, take(n * 4));
    pb.weight_sorted = weight_sorted ? weight_sorted : at<float>(workspace, take(n * 4));
    pb.route_sorted = route_sorted ? route_sorted : at<int>(workspace, take(n * 4));
    pb.expert_sorted = at<int>(workspace, take(n * 4));
    pb.route_pos = route_pos ? route_pos : at<int>(workspace, take(n * 4));
    pb.groups = at<int4>(workspace, take((size_t)max_groups(N, num_experts) * 16));
    pb.n_groups = at<int>(workspace, take(16));
    pb.n_fat = pb.n_groups + 1;
    pb.seg_hist = at<int>(workspace, take(perm_seg_hist_ints(N, num_experts) * 4 + 4));
    pb.counts64 = counts;
    pb.offsets64 = offsets;
    pb.nrows = pb.n_groups + 2;
    pb.status = nullptr;
    pb.rows_cap = N;
    cudaError_t err = launch_permute(ids, weights, N, topk, num_experts, expert_map, map_len, -1, pb,
                                     static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "permute");
    return DSV41_OK;
}

int dsv41_combine(const void* y, const int32_t* route_pos, const float* weights, int32_t T, int32_t topk,
                  int32_t hidden, int32_t accumulate, float* out, void* stream)
{
    if (T < 0 || topk <= 0 || hidden <= 0 || hidden % 8) return fail(DSV41_E_INVALID, "bad sizes");
    if (T == 0) return DSV41_OK;
    if (!y || !route_pos || !weights || !out) return fail(DSV41_E_INVALID, "NULL pointer");
    if (int rc = check_alignment(y, out, nullptr)) return rc;
    cudaError_t err = launch_combine(static_cast<const __half*>(y), route_pos, weights, T, topk, hidden, accumulate, out,
                                     static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "combine");
    return DSV41_OK;
}

int dsv41_decode_dense_bits(const void* trellis, int32_t k, int32_t n, int32_t bits, void* w_out, void* stream)
{
    if (k <= 0 || n <= 0 || k % 16 || n % 16) return fail(DSV41_E_INVALID, "k=%d n=%d must be multiples of 16", k, n);
    if (bits < 2 || bits > 4) return fail(DSV41_E_INVALID, "bits %d (2, 3 or 4)", bits);
    if (!trellis || !w_out) return fail(DSV41_E_INVALID, "NULL pointer");
    if (reinterpret_cast<uintptr_t>(trellis) % 4) return fail(DSV41_E_INVALID, "trellis must be 4-byte aligned");
    cudaError_t err =
        launch_decode_dense(trellis, k, n, bits, static_cast<__half*>(w_out), static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "decode_dense");
    return DSV41_OK;
}

int dsv41_decode_dense(const void* trellis, int32_t k, int32_t n, void* w_out, void* stream)
{
    return dsv41_decode_dense_bits(trellis, k, n, 3, w_out, stream);
}

static size_t expert_gemm_layout(int R, int n_experts, int H, int I, size_t* offs)
{
    const size_t E1 = (size_t)kMaxExperts + 1, n = (size_t)(R > 0 ? R : 1);
    const int split = auto_split(R, n_experts > 0 ? n_experts : 1, H, I, 0);
    const int gb = max_groups(R, n_experts > 0 ? n_experts : 1);
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t a = o;
        o = align_up(o + bytes, 256);
        return a;
    };
    offs[0] = take(256);                      // status
    offs[1] = take(E1 * 4);                   // counts32
    offs[2] = take(E1 * 4);                   // offsets32
    offs[3] = take(E1 * 4);                   // fat list
    offs[4] = take(n * 4);                    // expert_sorted
    offs[5] = take((size_t)gb * 16);          // groups
    offs[6] = take(16);                       // n_groups, n_fat, nrows
    offs[7] = take(n * H * 2);                // xt_g
    offs[8] = take(n * H * 2);                // xt_u
    offs[9] = take(n * I * 2);                // xt_d
    offs[10] = take(n * H * 2);               // y
    offs[11] = take(split > 1 ? (size_t)gemv_units_alloc(gb, H, I, split) * 4096 * 4 : 16);
    offs[12] = take((size_t)(gemv_units_alloc(gb, H, I, split) / split + 1 + gemv_sched_ints(gb)) * 4);
    offs[13] = take(gemm_scratch_bytes(R, n_experts, H, I));
    offs[14] = (size_t)split;
    offs[15] = (size_t)gb;
    return o;
}

int dsv41_expert_gemm_workspace_size(int32_t total_rows, int32_t n_experts, int32_t hidden, int32_t intermediate,
                                     size_t* bytes)
{
    if (!bytes || total_rows < 0 || n_experts < 0 || n_experts > kMaxExperts || hidden <= 0 || intermediate <= 0 ||
        hidden % 256 || intermediate % 256)
        return fail(DSV41_E_INVALID, "bad sizes rows=%d n=%d H=%d I=%d", total_rows, n_experts, hidden, intermediate);
    size_t offs[16];
    *bytes = expert_gemm_layout(total_rows, n_experts, hidden, intermediate, offs);
    return DSV41_OK;
}

int dsv41_expert_gemm(const dsv41_moe_layer* layer, const void* x, int32_t x_dtype, int32_t T, const int32_t* experts,
                      int32_t n_experts, const int64_t* counts, const int64_t* offsets, const int32_t* token_sorted,
                      const float* weight_sorted, int32_t total_rows, float limit, float* out, void* workspace,
                      size_t workspace_bytes, void* stream)
{
    int rc = check_layer(layer);
    if (rc) return rc;
    if (x_dtype < DSV41_DTYPE_F16 || x_dtype > DSV41_DTYPE_F32) return fail(DSV41_E_INVALID, "bad x_dtype %d", x_dtype);
    if (n_experts < 0 || n_experts > layer->num_experts || total_rows < 0 || T < 0)
        return fail(DSV41_E_INVALID, "bad sizes n_experts=%d total_rows=%d T=%d", n_experts, total_rows, T);
    if (n_experts == 0 || total_rows == 0) return DSV41_OK;
    if (!x || !experts || !counts || !offsets || !token_sorted || !weight_sorted || !out || !workspace)
        return fail(DSV41_E_INVALID, "NULL pointer");
    if ((rc = check_alignment(x, out, workspace))) return rc;
    const int H = layer->hidden, I = layer->intermediate, E = layer->num_experts;
    size_t offs[16];
    const size_t need = expert_gemm_layout(total_rows, n_experts, H, I, offs);
    if (workspace_bytes < need) return fail(DSV41_E_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes, need);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int split = (int)offs[14], gb = (int)offs[15];
    const int fat = kExpertGemmFat;
    PermBuffers pb{};
    pb.counts = at<int>(workspace, offs[1]);
    pb.offsets = at<int>(workspace, offs[2]);
    pb.fat_experts = at<int>(workspace, offs[3]);
    pb.expert_sorted = at<int>(workspace, offs[4]);
    pb.groups = at<int4>(workspace, offs[5]);
    pb.n_groups = at<int>(workspace, offs[6]);
    pb.n_fat = pb.n_groups + 1;
    int* nrows = pb.n_groups + 2;
    pb.nrows = nrows;
    pb.rows_cap = total_rows;
    pb.token_sorted = const_cast<int*>(token_sorted);
    pb.weight_sorted = const_cast<float*>(weight_sorted);
    cudaError_t err;
    if ((err = launch_list_setup(experts, n_experts, counts, offsets, E, total_rows, fat, pb, nrows, st)) != cudaSuccess)
        return cuda_fail(err, "list setup");
    __half* xt_g = at<__half>(workspace, offs[7]);
    __half* xt_u = at<__half>(workspace, offs[8]);
    __half* xt_d = at<__half>(workspace, offs[9]);
    __half* y = at<__half>(workspace, offs[10]);
    float* rsum = total_rows > fat ? gemm_row_sums(at<uint8_t>(workspace, offs[13]), total_rows, n_experts) : nullptr;
    if ((err = launch_prep(x, x_dtype, token_sorted, pb.expert_sorted, nrows, total_rows,
                           static_cast<const __half*>(layer->w13_suh), H, xt_g, xt_u, rsum, st)) != cudaSuccess)
        return cuda_fail(err, "prep");
    if ((err = run_expert_passes(layer, pb, xt_g, xt_u, xt_d, y, at<float>(workspace, offs[11]),
                                 at<int>(workspace, offs[12]), at<int>(workspace, offs[0]), split, gb, total_rows, limit,
                                 fat, at<uint8_t>(workspace, offs[13]), st)) != cudaSuccess)
        return cuda_fail(err, "expert passes");
    if ((err = launch_scatter_add(y, experts, n_experts, pb.counts, pb.offsets, token_sorted, weight_sorted, H, total_rows,
                                  out, st)) != cudaSuccess)
        return cuda_fail(err, "scatter add");
    return DSV41_OK;
}

int dsv41_set_stage_timing(int32_t enable)
{
    cudaError_t err;
    int dev = 0;
    if ((err = cudaGetDevice(&dev)) != cudaSuccess) return cuda_fail(err, "get device");
    if (enable && !g_timer.enabled) {
        if (g_timer.device >= 0 && g_timer.device != dev) {
            // events belong to the device they were created on
            int cur = dev;
            cudaSetDevice(g_timer.device);
            for (auto& row : g_timer.ev)
                for (auto& e : row) cudaEventDestroy(e);
            cudaSetDevice(cur);
            g_timer.device = -1;
        }
        if (g_timer.device < 0) {
            for (auto& row : g_timer.ev)
                for (auto& e : row)
                    if ((err = cudaEventCreate(&e)) != cudaSuccess) return cuda_fail(err, "event create");
            g_timer.device = dev;
        }
    }
    g_timer.enabled = enable != 0;
    g_timer.calls = 0;
    g_timer.active = false;
    return DSV41_OK;
}

int dsv41_read_stage_times(float* ms, int32_t max_calls, int32_t* n_calls)
{
    if (!n_calls || (max_calls > 0 && !ms)) return fail(DSV41_E_INVALID, "NULL pointer");
    const int n = g_timer.calls < max_calls ? g_timer.calls : max_calls;
    cudaError_t err;
    if (g_timer.calls > 0 && (err = cudaEventSynchronize(g_timer.ev[g_timer.calls - 1][DSV41_N_STAGES])) != cudaSuccess)
        return cuda_fail(err, "event synchronize");
    for (int c = 0; c < n; ++c)
        for (int s = 0; s < DSV41_N_STAGES; ++s) {
            float v = 0.0f;
            if ((err = cudaEventElapsedTime(&v, g_timer.ev[c][s], g_timer.ev[c][s + 1])) != cudaSuccess)
                return cuda_fail(err, "event elapsed");
            ms[c * DSV41_N_STAGES + s] = v;
        }
    *n_calls = n;
    g_timer.calls = 0;
    return DSV41_OK;
}

int dsv41_read_status(const void* workspace, void* stream, int32_t* status)
{
    if (!workspace || !status) return fail(DSV41_E_INVALID, "NULL pointer");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t err = cudaStreamSynchronize(st);
    if (err != cudaSuccess) return cuda_fail(err, "synchronize");
    int v = 0;
    if ((err = cudaMemcpy(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(err, "read status");
    if (v && (err = cudaMemset(const_cast<void*>(workspace), 0, sizeof(int))) != cudaSuccess)
        return cuda_fail(err, "clear status");
    *status = v;
    return DSV41_OK;
}

int dsv41_wait_selftest(void* workspace, uint32_t limit_us, void* stream)
{
    if (!workspace) return fail(DSV41_E_INVALID, "NULL workspace");
    if (limit_us < 1 || limit_us > 2000000u) return fail(DSV41_E_INVALID, "limit_us must be in [1, 2000000]");
    cudaError_t err = launch_wait_selftest(static_cast<int*>(workspace), (uint64_t)limit_us * 1000ull,
                                           static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "wait self test launch");
    return DSV41_OK;
}

}  // extern "C"
