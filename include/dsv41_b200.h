/*
 * dsv41_b200 -- C ABI of the B200 (sm_100a) routed-expert MoE FFN over EXL3 mul1 K=3 weights.
 *
 * Plain pointers and sizes only (no torch types). Every compute entry point is asynchronous on
 * the caller's CUDA stream (`stream` is a cudaStream_t passed as void*; NULL = legacy default
 * stream), allocates nothing, returns 0 on success or a negative DSV41_E* code, and leaves a
 * message for dsv41_last_error(). Kernels never trap: a device-side wait that runs out writes a
 * nonzero status word into the workspace, read back with dsv41_read_status().
 *
 * Reference interfaces replaced (paths inside the reference project 0xSero/dsv41-flash-offload):
 *   dsv41_moe_forward       apply_exl3_fused_moe(x2d, ids, weights, layer, inners, expert_map,
 *                           limit) -> out fp32 [T, H]: the routing prep
 *                           (patches/vllm-exl3-host-dma.patch:203-312) plus the
 *                           exllamav3_ext.exl3_moe launch contract (patch:315-449), and the
 *                           busy-expert path apply_exl3_batched_fat (patch:182-201) for experts
 *                           over fat_threshold rows; wrapped in the reference by
 *                           ct/ct_vllm.py:181-225 (_fused)
 *   dsv41_permute           the routing prep alone (patch:204-226, :300-312) and the split
 *                           kernel's histogram/compaction (ct/ft_tier_cu_v.cu:16-101, ft_split)
 *   dsv41_combine           the weighted accumulate of routed expert outputs into the fp32
 *                           layer output (ct/ft_tier_cu_v.cu:103-127 ft_combine;
 *                           kernels/cpu_avx2/ft_core.h:911-931)
 *   dsv41_decode_dense      the reconstruct step of the fat path / LinearEXL3.get_weight_tensor
 *                           (patch:182-201, pack/prepare_pack.py:64-65), restated from
 *                           kernels/cpu_avx2/ft_core.h:977-992 (dense_weights)
 *   dsv41_expert_gemm       runtime/dma_gemm.py:5-26 run_batch -> apply_exl3_batched_fat:
 *                           busy experts' reconstruct + GEMM, accumulated into out
 */
#ifndef DSV41_B200_H
#define DSV41_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSV41_ABI_VERSION 2

enum {
    DSV41_OK = 0,
    DSV41_E_INVALID = -1,  /* bad argument / shape */
    DSV41_E_CUDA = -2,     /* CUDA runtime error (launch or attribute) */
    DSV41_E_WORKSPACE = -3 /* workspace too small */
};

enum { DSV41_DTYPE_F16 = 0, DSV41_DTYPE_BF16 = 1, DSV41_DTYPE_F32 = 2 };

/* One MoE layer's expert weights, all device pointers (vllm_exl3 Exl3MoEMethod layout,
 * patches/vllm-exl3-host-dma.patch:633-684 and its per-expert pointer tables, patch:66-69):
 *   gate_ptrs/up_ptrs [E]  int64 addresses of int16 trellis [H/16][I/16][16*bits] (48 at 3 bits)
 *   down_ptrs [E]          int64 addresses of int16 trellis [I/16][H/16][16*bits]
 *   w13_suh [E][2][H], w13_svh [E][2][I], w2_suh [E][I], w2_svh [E][H]  fp16
 * Every trellis address must be 16-byte aligned. H and I are multiples of 256. */
typedef struct dsv41_moe_layer {
    int32_t num_experts;
    int32_t hidden;
    int32_t intermediate;
    int32_t bits;       /* bits per weight K of every trellis tile: 2, 3 or 4 (0 = 3, the reference's build) */
    const int64_t* gate_ptrs;
    const int64_t* up_ptrs;
    const int64_t* down_ptrs;
    const void* w13_suh;
    const void* w13_svh;
    const void* w2_suh;
    const void* w2_svh;
} dsv41_moe_layer;

/* Options of one forward call.
 *   fat_threshold: experts with more than this many rows use the tensor-core grouped GEMM
 *                  (VLLM_EXL3_FAT_THRESHOLD, patch:146; 32 deployed); < 0 routes everything
 *                  through the decode GEMV.
 *   limit:         SwiGLU clamp (SWIGLU_LIMIT_DEFAULT 10.0, patch:5); 0 disables it.
 *   expert_map:    optional device int32 [map_len] global -> local expert id (-1 = not local),
 *                  as vLLM's expert_map; NULL = identity. */
typedef struct dsv41_moe_options {
    int32_t fat_threshold;
    float limit;
    const int32_t* expert_map;
    int32_t map_len;
    int32_t split_k;    /* 0 = automatic */
    int32_t max_routes; /* upper bound on routes with a valid local expert; row buffers are sized by it
                           (0 = T*topk). A call with more valid routes drops them all, writes zeros and
                           sets status 3 (see dsv41_read_status). Used by expert-parallel callers whose
                           rows carry mostly non-local route slots. */
} dsv41_moe_options;

/* Last error message of the calling thread ("" if none). */
const char* dsv41_last_error(void);
/* ABI version (DSV41_ABI_VERSION) and a build string. */
int dsv41_abi_version(void);
const char* dsv41_build_info(void);

/* Workspace bytes that dsv41_moe_forward needs for T tokens x topk routes. */
int dsv41_moe_workspace_size(int32_t T, int32_t topk, int32_t num_experts, int32_t hidden,
                             int32_t intermediate, const dsv41_moe_options* opt, size_t* bytes);

/* out[T][H] (fp32, overwritten) = sum over valid routes (t, j) of weights[t][j] * expert(x[t]).
 *   x [T][H] of x_dtype (cast to fp16 first, as the reference does), ids [T][topk] int64
 *   (negative or >= E = skipped), weights [T][topk] fp32. x and out must be 16-byte aligned and
 *   the workspace 256-byte aligned (DSV41_E_INVALID otherwise; device allocations are). */
int dsv41_moe_forward(const dsv41_moe_layer* layer, const void* x, int32_t x_dtype, int32_t T,
                      const int64_t* ids, const float* weights, int32_t topk,
                      const dsv41_moe_options* opt, float* out, void* workspace,
                      size_t workspace_bytes, void* stream);

/* dsv41_moe_forward for callers that cannot allocate device memory (no counterpart in the
 * reference). Same arguments and results as dsv41_moe_forward, minus the workspace: the scratch
 * is a fixed 32 MiB device array inside this library, held by every GPU that uses it until the
 * process exits. Requests needing more scratch than that fail with DSV41_E_WORKSPACE and a
 * message (at E=384 H=4096 I=2048 top-8 it covers decode batches up to 64 tokens). The first
 * call on a device looks the array up (make it before any stream capture); calls share the array,
 * so calls that overlap on the GPU race. Every argument is checked before anything is queued.
 * Allocates nothing. The status word of these calls lives in the array: read it with
 * dsv41_moe_noalloc_read_status, not dsv41_read_status. */
int dsv41_moe_forward_noalloc(const dsv41_moe_layer* layer, const void* x, int32_t x_dtype, int32_t T,
                              const int64_t* ids, const float* weights, int32_t topk,
                              const dsv41_moe_options* opt, float* out, void* stream);
/* dsv41_read_status for dsv41_moe_forward_noalloc on the current device (no counterpart in the
 * reference): synchronise `stream`, return the status word of the library's static scratch (0 = ok,
 * 1 = a bounded device wait ran out, 3 = more valid routes than options.max_routes) and clear it.
 * The next dsv41_moe_forward_noalloc call also clears it, so read it after each call you check. */
int dsv41_moe_noalloc_read_status(void* stream, int32_t* status);

/* Routing permutation (bit-exact, stable by (local expert, flat route index)):
 *   counts/offsets [E+1] int64 (index E = invalid-route sentinel), token_sorted/route_sorted
 *   [T*topk] int32, weight_sorted [T*topk] fp32, route_pos [T*topk] int32 (sorted position of
 *   each flat route, -1 when skipped). Any output pointer may be NULL. */
size_t dsv41_permute_workspace_size(int32_t T, int32_t topk, int32_t num_experts);
int dsv41_permute(const int64_t* ids, const float* weights, int32_t T, int32_t topk,
                  int32_t num_experts, const int32_t* expert_map, int32_t map_len,
                  int64_t* counts, int64_t* offsets, int32_t* token_sorted, float* weight_sorted,
                  int32_t* route_sorted, int32_t* route_pos, void* workspace,
                  size_t workspace_bytes, void* stream);

/* out[T][H] fp32 = sum_j weights[t][j] * y[route_pos[t*topk+j]][:] over route_pos >= 0;
 * y [rows][H] fp16. accumulate != 0 adds into out instead of overwriting it. */
int dsv41_combine(const void* y, const int32_t* route_pos, const float* weights, int32_t T,
                  int32_t topk, int32_t hidden, int32_t accumulate, float* out, void* stream);

/* Decode one trellis matrix [k/16][n/16][48] int16 into dense fp16 W [k][n] (bit-exact). */
int dsv41_decode_dense(const void* trellis, int32_t k, int32_t n, void* w_out, void* stream);
/* Same for K = bits per weight (2, 3 or 4): trellis [k/16][n/16][16*bits] int16 (the 2-bit packs
 * and 4-bit layers the reference's checkpoints also carry, patch:519-528, pack/prepare_pack.py:47). */
int dsv41_decode_dense_bits(const void* trellis, int32_t k, int32_t n, int32_t bits, void* w_out, void* stream);

/* Busy-expert GEMM path on pre-permuted rows (run_batch semantics): for each listed expert e
 * with counts[e] rows starting at offsets[e] of token_sorted/weight_sorted, out[token] +=
 * weight * expert_e(x[token]). experts [n_experts] int32 (device). */
int dsv41_expert_gemm(const dsv41_moe_layer* layer, const void* x, int32_t x_dtype, int32_t T,
                      const int32_t* experts, int32_t n_experts, const int64_t* counts,
                      const int64_t* offsets, const int32_t* token_sorted,
                      const float* weight_sorted, int32_t total_rows, float limit, float* out,
                      void* workspace, size_t workspace_bytes, void* stream);
int dsv41_expert_gemm_workspace_size(int32_t total_rows, int32_t n_experts, int32_t hidden,
                                     int32_t intermediate, size_t* bytes);

/* Synchronise `stream` and return the device status word of a workspace (0 = ok,
 * 1 = a bounded device wait ran out, 3 = more valid routes than options.max_routes), then clear it. */
int dsv41_read_status(const void* workspace, void* stream, int32_t* status);

/* Failure-detection self test (no counterpart entry in the reference; its combine kernel
 * ct/ft_tier_cu_v.cu:103-127 bounds its device spin the same way, by %globaltimer, and counts a
 * timeout in a stats word instead of trapping): launches one warp that waits
 * on a device barrier nothing ever completes, through the bounded wait every pipeline kernel uses;
 * after limit_us (1..2,000,000) it writes status 1 into the workspace's status word and returns.
 * Read it with dsv41_read_status; the stream and context stay usable. */
int dsv41_wait_selftest(void* workspace, uint32_t limit_us, void* stream);

/* Router top-k (no counterpart in the reference: vLLM's FusedMoE router produces topk_ids/weights before
 * apply_exl3_experts, patches/vllm-exl3-host-dma.patch:496-505). vLLM's two published rules:
 * scores = softmax(logits) over all experts, or sigmoid(logits); selection = scores (+ correction_bias
 * when given); with num_expert_group > 1 only the topk_group best groups compete (group score: sum
 * of its two best selection values with a bias, else its best); ids = top-k selection (ties: lower
 * id); weights = scores at ids, renormalised to sum 1 if `renormalize`, times routed_scaling_factor.
 * E <= 1024, topk <= 32. dsv41_moe_forward_logits = router + dsv41_moe_forward in one call (ids and
 * weights stay in the workspace unless ids_out/weights_out are given). */
enum { DSV41_ROUTER_SOFTMAX = 0, DSV41_ROUTER_SIGMOID = 1 };
typedef struct dsv41_router_options {
    int32_t scoring;                /* DSV41_ROUTER_SOFTMAX or DSV41_ROUTER_SIGMOID */
    int32_t renormalize;            /* nonzero: weights / sum(weights) over the k chosen */
    int32_t num_expert_group;       /* 0 or 1 = no grouping */
    int32_t topk_group;
    const float* correction_bias;   /* device [E] fp32 or NULL */
    float routed_scaling_factor;    /* 1.0 = none */
} dsv41_router_options;

int dsv41_router_topk(const void* logits, int32_t logits_dtype, int32_t T, int32_t num_experts, int32_t topk,
                      const dsv41_router_options* router, int64_t* ids, float* weights, void* stream);
int dsv41_moe_forward_logits(const dsv41_moe_layer* layer, const void* x, int32_t x_dtype, int32_t T,
                             const void* logits, int32_t logits_dtype, const dsv41_router_options* router, int32_t topk,
                             const dsv41_moe_options* opt, float* out, int64_t* ids_out, float* weights_out,
                             void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------
 * Expert parallelism over NVLink peer memory (no counterpart in the reference, which runs one GPU
 * with experts in host RAM, docker/entrypoint.sh:135-140). Experts are sharded: global expert e
 * lives on rank e / (num_global_experts / world). Each rank allocates one shared buffer
 * (dsv41_ep_peer_alloc: cudaMalloc + cudaIpcGetMemHandle), exchanges the 64-byte handles with its
 * peers over the host, opens theirs (dsv41_ep_peer_open) and fills bases[] (own buffer at
 * bases[rank]). dsv41_ep_peer_forward then runs one step of the layer for this rank's T <=
 * tokens_cap tokens with no collective library: the row transform reads each routed token row
 * from its rank (plain peer loads) and the down pass stores each expert output row into the
 * receive slot of its token's rank (plain peer stores), whose combine then sums its own slots;
 * step stamps in the shared buffers order the ranks (bounded waits, status 1 on expiry ->
 * dsv41_ep_peer_read_status). Every rank must call it once per step with the same
 * `step` sequence (0, 1, 2, ...), topk and tokens_cap. The buffers alternate by step parity, so a
 * CUDA graph of one step replays only for steps of the same parity. Hidden size up to 8192.
 * ------------------------------------------------------------------------------------------ */
#define DSV41_MAX_PEERS 8
#define DSV41_IPC_HANDLE_BYTES 64
typedef struct dsv41_ep_peer_group {
    int32_t rank, world;            /* world <= DSV41_MAX_PEERS */
    int32_t num_global_experts;     /* divisible by world */
    int32_t tokens_cap;             /* max tokens per rank and step (same on every rank) */
    void* bases[DSV41_MAX_PEERS];   /* device address of each rank's shared buffer in this process */
    int32_t wait_limit_us;          /* limit of each wait for the peers' step stamps, 1..2,000,000 us
                                       (0 = 2 s, the reference combine wait's bound); on expiry the
                                       step's exchange gives up with status 1 */
} dsv41_ep_peer_group;

int dsv41_ep_peer_buffer_size(const dsv41_ep_peer_group* group, const dsv41_moe_layer* local_layer, int32_t topk,
                              int32_t fat_threshold, size_t* bytes);
int dsv41_ep_peer_alloc(size_t bytes, void** base, void* ipc_handle);
int dsv41_ep_peer_open(const void* ipc_handle, void** peer_base);
int dsv41_ep_peer_close(void* peer_base);
int dsv41_ep_peer_free(void* base);
int dsv41_ep_peer_forward(const dsv41_moe_layer* local_layer, const dsv41_ep_peer_group* group, uint32_t step,
                          const void* x, int32_t x_dtype, int32_t T, const int64_t* ids, const float* weights,
                          int32_t topk, float limit, int32_t fat_threshold, float* out, void* stream);
int dsv41_ep_peer_read_status(const dsv41_ep_peer_group* group, const dsv41_moe_layer* local_layer, int32_t topk,
                              int32_t fat_threshold, void* stream, int32_t* status);

/* Profiling (no counterpart in the reference; used by bench.py to time each kernel on the stream
 * it runs on). While enabled, dsv41_moe_forward records CUDA events at its stage boundaries for up
 * to DSV41_TIMING_MAX_CALLS calls (not under stream capture). dsv41_read_stage_times synchronises
 * them and writes DSV41_N_STAGES times in ms per recorded call, in the order permute, row prep,
 * decode-GEMV (both passes, one launch, when split_k is 1), gate/up GEMM, down decode-GEMV (its own
 * launch when split_k > 1, else empty), down GEMM, combine; then it forgets them. */
#define DSV41_N_STAGES 7
#define DSV41_TIMING_MAX_CALLS 256
int dsv41_set_stage_timing(int32_t enable);
int dsv41_read_stage_times(float* ms, int32_t max_calls, int32_t* n_calls);

#ifdef __cplusplus
}
#endif
#endif /* DSV41_B200_H */
