// Mixture-of-experts kernels: routing, grouping rows by expert, and the weighted combine.
//
// The contract is the reference's (crates/furiosa-opt-models/src/modules/feedforward/moe.rs:1-7,
// 41-47, 352-400): a row's router logits are BF16; probabilities are an FP32 softmax over the
// experts; a row selects its K largest logits, best first, equal logits (-0 and +0 alike) in
// ascending expert order; optionally the K probabilities are divided by their FP32 sum; expert
// outputs are BF16 rows; the combine sums weight x row in FP32 in choice order and rounds once.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace foa {

// Routing of `rows` rows of BF16 logits [rows, experts] (row stride ld): ids [rows, k] (int32) and
// weights [rows, k] (FP32), best first. experts <= 512, k <= experts.
int moe_route(const __nv_bfloat16* logits, long ld, int rows, int experts, int k, bool normalize,
              int32_t* ids, float* weights, cudaStream_t stream);

// Groups the rows x k selections by expert for a grouped GEMM with `tile`-row token tiles. Only
// experts [first, first + count) are grouped (an expert-parallel rank's); others are skipped.
// Sorted positions start each expert at a multiple of `tile`, selections of one expert keep their
// (row, choice) order. Outputs:
//   pos[rows * k]       sorted position of each selection, or -1 (not a local expert)
//   src[capacity]       source row of each sorted position, -1 for padding
//   tile_expert[..]     local expert (0-based) of each token tile
//   tiles[1]            token tiles in use
// capacity must be at least rows * k + count * (tile - 1) rounded up to `tile`.
int moe_align(const int32_t* ids, int rows, int k, int experts, int first, int count, int tile,
              int capacity, int32_t* pos, int32_t* src, int32_t* tile_expert, int32_t* tiles,
              cudaStream_t stream);

// Every expert-parallel rank's grouping at once: rank c (one CTA each) groups the experts
// [first + c * count, first + (c + 1) * count) into pos + c * rows * k; `src`, `tile_expert` and
// `tiles` are the grouping of rank `local`.
int moe_align_ranks(const int32_t* ids, int rows, int k, int experts, int first, int count, int ranks,
                    int local, int tile, int capacity, int32_t* pos, int32_t* src, int32_t* tile_expert,
                    int32_t* tiles, cudaStream_t stream);

// out[p] = x[src[p]] for the sorted rows in use (zeros for padding), BF16 rows of `cols`.
int moe_gather(const __nv_bfloat16* x, long ldx, const int32_t* src, const int32_t* tiles, int tile,
               int capacity, int cols, __nv_bfloat16* out, cudaStream_t stream);

// residual[r] = bf16(residual[r] + bf16(sum_j w[r, j] * y[pos[r, j]])) in choice order (FP32),
// where y holds BF16 expert rows [capacity, cols]. Selections with pos < 0 contribute nothing.
int moe_combine(const __nv_bfloat16* y, long ldy, const int32_t* pos, const float* weights, int rows,
                int k, int cols, __nv_bfloat16* residual, long ldr, cudaStream_t stream);

// The combine followed by the next RMSNorm: residual = bf16(residual + bf16(sum_j w_j * y_j)),
// out = bf16(RMSNorm(residual) * norm). cols <= 8192.
int moe_combine_norm(const __nv_bfloat16* y, long ldy, const int32_t* pos, const float* weights, int rows,
                     int k, int cols, __nv_bfloat16* residual, long ldr, const __nv_bfloat16* norm, float eps,
                     __nv_bfloat16* out, long ldo, cudaStream_t stream);

}  // namespace foa
