// Router top-k: gating logits -> top-k expert ids and routing weights, feeding the permute kernel
// in the same call (dsv41_moe_forward_logits) so ids never round-trip through a separate op.
//
// The reference receives topk_ids/topk_weights from vLLM's FusedMoE router (vLLM is not vendored;
// the ids arrive at apply_exl3_experts, patches/vllm-exl3-host-dma.patch:496-505, and are cast at
// :204-215). This kernel implements vLLM's two published routing rules (vLLM 0.22,
// model_executor/layers/fused_moe/router/{fused_topk_router,grouped_topk_router}.py):
//   scores      = softmax(logits) over all experts, or sigmoid(logits)
//   selection   = scores + correction bias when a bias is given, else scores
//   groups      (n_group > 1): group score = sum of the top-2 selection values of the group with a
//               bias, else the group maximum; only the best topk_group groups compete
//   ids         = top-k of the selection values in the competing groups (ties: lower expert id)
//   weights     = scores at ids (never the biased values); renormalised to sum 1 if asked;
//               times routed_scaling_factor
// One warp per token; lane l holds experts l, l+32, ... (E <= 1024).
#include "common.cuh"
#include "internal.h"

namespace dsv41 {

constexpr int kRouterMaxPerLane = 32;  // E <= 1024

__device__ __forceinline__ void warp_argmax(float& v, int& i)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (ov > v || (ov == v && oi < i)) {
            v = ov;
            i = oi;
        }
    }
}

__global__ void __launch_bounds__(256) router_topk_kernel(const void* logits, int logits_dtype, int T, int E, int k,
                                                          int scoring, int renormalize, int n_group, int topk_group,
                                                          const float* bias, float scale, int64_t* ids, float* w)
{
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    const int per = (E + 31) / 32;
    float score[kRouterMaxPerLane], sel[kRouterMaxPerLane];
    // load logits (fp32 math)
    float mx = -INFINITY;
#pragma unroll
    for (int q = 0; q < kRouterMaxPerLane; ++q) {
        if (q >= per) break;
        const int e = lane + 32 * q;
        float l = -INFINITY;
        if (e < E) {
            const size_t idx = (size_t)t * E + e;
            l = logits_dtype == 2 ? static_cast<const float*>(logits)[idx]
                : logits_dtype == 1 ? __bfloat162float(static_cast<const __nv_bfloat16*>(logits)[idx])
                                    : __half2float(static_cast<const __half*>(logits)[idx]);
        }
        score[q] = l;
        mx = fmaxf(mx, l);
    }
    if (scoring == 0) {   // softmax over all experts
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.0f;
#pragma unroll
        for (int q = 0; q < kRouterMaxPerLane; ++q) {
            if (q >= per) break;
            const int e = lane + 32 * q;
            score[q] = e < E ? expf(score[q] - mx) : 0.0f;
            sum += score[q];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float inv = 1.0f / sum;
#pragma unroll
        for (int q = 0; q < kRouterMaxPerLane; ++q)
            if (q < per) score[q] *= inv;
    } else {              // sigmoid
#pragma unroll
        for (int q = 0; q < kRouterMaxPerLane; ++q)
            if (q < per) score[q] = 1.0f / (1.0f + expf(-score[q]));
    }
#pragma unroll
    for (int q = 0; q < kRouterMaxPerLane; ++q) {
        if (q >= per) break;
        const int e = lane + 32 * q;
        sel[q] = e < E ? (bias ? score[q] + bias[e] : score[q]) : -INFINITY;
    }
    // group restriction: competing groups keep their selection values, the rest drop to -inf
    if (n_group > 1) {
        const int gsize = E / n_group;
        float gscore = -INFINITY;   // lane g < n_group holds group g's score
        for (int g = 0; g < n_group; ++g) {
            float a = -INFINITY, b = -INFINITY;   // this lane's top-2 within group g
#pragma unroll
            for (int q = 0; q < kRouterMaxPerLane; ++q) {
                if (q >= per) break;
                const int e = lane + 32 * q;
                if (e / gsize != g || e >= E) continue;
                const float v = sel[q];
                if (v > a) {
                    b = a;
                    a = v;
                } else if (v > b) {
                    b = v;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {   // merge top-2 across lanes
                const float oa = __shfl_xor_sync(0xffffffffu, a, o), ob = __shfl_xor_sync(0xffffffffu, b, o);
                const float hi = fmaxf(a, oa), lo = fmaxf(fminf(a, oa), fmaxf(b, ob));
                a = hi;
                b = lo;
            }
            const float gs = bias ? a + b : a;
            if (lane == g) gscore = gs;
        }
        unsigned keep = 0;   // bit g set: group g competes
        for (int r = 0; r < topk_group; ++r) {
            float v = lane < n_group && !((keep >> lane) & 1u) ? gscore : -INFINITY;
            int i = lane < n_group && !((keep >> lane) & 1u) ? lane : 0x7fffffff;
            warp_argmax(v, i);
            if (i < n_group) keep |= 1u << i;
        }
#pragma unroll
        for (int q = 0; q < kRouterMaxPerLane; ++q) {
            if (q >= per) break;
            const int e = lane + 32 * q;
            if (e < E && !((keep >> (e / gsize)) & 1u)) sel[q] = -INFINITY;
        }
    }
    // top-k by repeated warp arg-max (lower id wins ties)
    float wsum = 0.0f, wk = 0.0f;
    int myid = -1;
    for (int r = 0; r < k; ++r) {
        float v = -INFINITY;
        int i = 0x7fffffff;
#pragma unroll
        for (int q = 0; q < kRouterMaxPerLane; ++q) {
            if (q >= per) break;
            const int e = lane + 32 * q;
            if (e < E && (sel[q] > v || (sel[q] == v && e < i))) {
                v = sel[q];
                i = e;
            }
        }
        warp_argmax(v, i);
        float sw = 0.0f;
#pragma unroll
        for (int q = 0; q < kRouterMaxPerLane; ++q) {
            if (q >= per) break;
            if (lane + 32 * q == i) {
                sw = score[q];
                sel[q] = -INFINITY;   // taken
            }
        }
        sw = __shfl_sync(0xffffffffu, sw, i & 31);
        if (i == 0x7fffffff) sw = 0.0f;   // fewer competing experts than k
        wsum += sw;
        if (lane == r) {
            myid = i == 0x7fffffff ? -1 : i;
            wk = sw;
        }
    }
    if (lane < k) {
        float wt = wk;
        if (renormalize) wt = wsum > 0.0f ? wt / wsum : 0.0f;
        ids[(size_t)t * k + lane] = myid;
        w[(size_t)t * k + lane] = wt * scale;
    }
}

cudaError_t launch_router_topk(const void* logits, int logits_dtype, int T, int E, int k, int scoring,
                               int renormalize, int n_group, int topk_group, const float* bias, float scale,
                               int64_t* ids, float* w, cudaStream_t st)
{
    if (T <= 0) return cudaSuccess;
    const int warps = 8;
    router_topk_kernel<<<(T + warps - 1) / warps, warps * 32, 0, st>>>(logits, logits_dtype, T, E, k, scoring,
                                                                        renormalize, n_group, topk_group, bias, scale,
                                                                        ids, w);
    return cudaGetLastError();
}

}  // namespace dsv41
