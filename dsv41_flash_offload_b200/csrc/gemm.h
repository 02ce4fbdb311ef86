// Busy-expert ("fat") path: decode-to-shared-memory + tcgen05/TMEM grouped GEMM for experts with
// more than fat_threshold rows (the reference's apply_exl3_batched_fat, reconstruct + FP16 GEMM:
// patches/vllm-exl3-host-dma.patch:182-201; runtime/dma_gemm.py:5-26).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/dsv41_b200.h"
#include "internal.h"

namespace dsv41 {

struct GemmArgs {
    const dsv41_moe_layer* layer;
    const int* fat_experts;  // [n_fat] experts on this path (device list)
    const int* n_fat;        // device count
    const int* counts;       // [E+1] rows per expert
    const int* offsets;      // [E+1] first sorted row per expert
    const __half* xt_g;      // [rows][H] transformed gate inputs (sorted rows)
    const __half* xt_u;      // [rows][H]
    __half* xt_d;            // [rows][I] down inputs (written by gate/up, read by down)
    __half* y;               // [rows][H] expert outputs (written by down)
    RowPush push;            // expert-parallel push: the down rows go to their token owners instead of y
    int rows_bound;          // upper bound of the total sorted rows
    float limit;
    uint8_t* scratch;
    int* status;
};

// GEMM scratch (N = row bound, E = experts): pass counters and lists, then the per-row activation sums
// of the affine weight codes -- gemm_row_sums [2 N] (gate, up; written by the row transform) and
// gemm_down_sums [N][I / 128] (block sums of the down inputs; written by the gate/up epilogue)
size_t gemm_scratch_bytes(int N, int E, int H, int I);
float* gemm_row_sums(uint8_t* scratch, int N, int E);
float* gemm_down_sums(uint8_t* scratch, int N, int E);
cudaError_t launch_gemm_gateup(const GemmArgs& a, cudaStream_t st);
cudaError_t launch_gemm_down(const GemmArgs& a, cudaStream_t st);

}  // namespace dsv41
