/*
 * TEST INFRASTRUCTURE ONLY -- not part of the product path.
 *
 * CPU restatement (plain C) of the reference's routed-expert MoE FFN over EXL3 mul1 K=3
 * trellis-coded weights. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
 * may load this library, and only as the checker.
 *
 * Reference files (paths inside the reference project):
 *   kernels/cpu_avx2/ft_core.h        decode spec, transforms, act, reference expert
 *   patches/vllm-exl3-host-dma.patch  routing prep of apply_exl3_fused_moe (count/argsort)
 *   kernels/cpu_avx2/ft_tier_ext.cpp  tier_forward route lists / weighted accumulate
 *
 * Parity is pinned against the reference itself: oracle/Makefile compiles the reference's
 * ft_core.h unchanged through oracle/ref_shim.cpp into oracle/_ref/, and
 * tests/golden/make_golden.py writes the golden vectors from that build.
 */
#ifndef DSV41_EXL3_ORACLE_H
#define DSV41_EXL3_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* IEEE half <-> float (round to nearest even). */
float orc_h2f(uint16_t h);
uint16_t orc_f2h(float f);

/* stream index (0..255) -> r*16 + c inside a 16x16 tile (r = input row k, c = output col n) */
int orc_perm(int i);
/* 16-bit trellis state of stream index t of one 96-byte tile (48 uint16 words) */
uint16_t orc_state(const uint16_t* tile, int t);
/* byte sum of state * 0x83DCD12D (0..1020) */
int orc_bytesum(uint16_t state);
/* bits per weight K of the trellis tiles (2, 3 or 4; default 3 = the reference's build) */
void orc_set_bits(int bits);
int orc_get_bits(void);
/* fp16 bits of the decoded weight for one state */
uint16_t orc_weight_bits(uint16_t state);
/* whole matrix: trellis [k/16][n/16][16K] int16 -> W [k][n] fp16 bits */
void orc_decode_matrix(const uint16_t* trellis, int k, int n, uint16_t* W);

/* transforms on one 128-block (fp32 math, fp16 rounding points) */
void orc_had128(float* v);
void orc_prep_block(const float* x, const uint16_t* suh, float* xt);
void orc_out_block(float* y, const uint16_t* svh);
float orc_act(float g, float u, float limit);

/* y[m][n] = out_block(sum_k prep(x)[k] W[k][n]) with double accumulation; x [m][k] fp16-valued */
void orc_linear(const uint16_t* trellis, const uint16_t* suh, const uint16_t* svh, int k, int n,
                int m, const float* x, float* y);
/* one expert on m tokens: gate/up -> act -> down, x [m][H] fp16-valued -> y [m][H] */
void orc_expert(const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                const uint16_t* suh_g, const uint16_t* svh_g, const uint16_t* suh_u,
                const uint16_t* svh_u, const uint16_t* suh_d, const uint16_t* svh_d,
                int H, int I, int m, const float* x, float limit, float* y);

/* Routing permutation: local = map(ids) with invalid -> E sentinel; counts[E+1];
 * offsets[E+1] exclusive; stable order by (local, flat index). Outputs have T*topk entries;
 * route_pos[flat] = sorted position of each flat route. Returns 0. */
int orc_permute(const int64_t* ids, const float* weights, int T, int topk, int E,
                const int32_t* expert_map, int map_len, int64_t* counts, int64_t* offsets,
                int32_t* token_sorted, float* weight_sorted, int32_t* route_sorted,
                int32_t* route_pos);

/* Full MoE layer: out[T][H] (fp32) = sum over valid routes of w * expert_e(x_t).
 * x [T][H] fp16-valued floats; gate/up/down per-expert trellis pointers; scales stacked as
 * vllm_exl3 lays them out: w13_suh [E][2][H], w13_svh [E][2][I], w2_suh [E][I], w2_svh [E][H].
 * nthreads > 1 decodes experts in parallel (pthreads). */
void orc_moe_layer(const float* x, int T, int H, int I, const int64_t* ids, const float* weights,
                   int topk, int E, const int32_t* expert_map, int map_len,
                   const uint16_t* const* gate, const uint16_t* const* up,
                   const uint16_t* const* down, const uint16_t* w13_suh,
                   const uint16_t* w13_svh, const uint16_t* w2_suh, const uint16_t* w2_svh,
                   float limit, int nthreads, float* out);

/* per-route expert outputs y [T*topk][H] (zeros for invalid routes), same arguments */
void orc_moe_routes(const float* x, int T, int H, int I, const int64_t* ids, int topk, int E,
                    const int32_t* expert_map, int map_len, const uint16_t* const* gate,
                    const uint16_t* const* up, const uint16_t* const* down,
                    const uint16_t* w13_suh, const uint16_t* w13_svh, const uint16_t* w2_suh,
                    const uint16_t* w2_svh, float limit, int nthreads, float* yroutes);

#ifdef __cplusplus
}
#endif
#endif
