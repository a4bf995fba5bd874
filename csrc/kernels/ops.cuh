// Host-visible interface of the engine's non-GEMM kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gemm.cuh"

namespace foa {

// h = x (+ residual), FP32 sum rounded once to BF16 into residual_out (when given);
// out = BF16(h * weight / sqrt(mean(h^2) + eps)) with FP32 statistics and one rounding.
// `residual` and `residual_out` may be null; `residual_out` may alias `residual` or `x`.
int rmsnorm(const __nv_bfloat16* x, long ldx, const __nv_bfloat16* residual, long ldr,
            const __nv_bfloat16* weight, __nv_bfloat16* out, long ldo,
            __nv_bfloat16* residual_out, long ldro, int rows, int cols, float eps,
            cudaStream_t stream);

// x = BF16(sum of the GEMM's K splits in split order (FP32) + x), in place, then
// out = BF16(x * weight / sqrt(mean(x^2) + eps)): the residual projection's split reduction, its
// residual add and the norm after it in one kernel (`splits` from gemm_bf16_splits).
int rmsnorm_splits(const GemmSplits& splits, __nv_bfloat16* x, long ldx, const __nv_bfloat16* weight,
                   __nv_bfloat16* out, long ldo, int rows, int cols, float eps, cudaStream_t stream);

// out[r, :] = table[ids[r], :] for r < rows, BF16 rows of `cols` elements. Rows of the table
// outside [row_begin, row_end) (a vocabulary shard) give zeros, and ids are shifted by row_begin.
int embedding(const int32_t* ids, const __nv_bfloat16* table, long ldt, int row_begin,
              int row_end, __nv_bfloat16* out, long ldo, int rows, int cols, cudaStream_t stream);

// For each of `rows` FP32 rows of `cols` logits: the first index of the maximum (NaN never wins)
// and its value. Padded vocabulary columns >= `valid_cols` never win. `index_base` is added to
// every index (a vocabulary shard's offset).
int argmax_rows(const float* logits, long ld, int rows, int cols, int valid_cols, int index_base,
                int32_t* out_index, float* out_value, cudaStream_t stream);

// Merges per-rank (value, index) argmax candidates [ranks, rows] into tokens: the largest value,
// the lowest index among equal values.
int argmax_merge(const float* values, const int32_t* indices, int ranks, int rows,
                 int32_t* out_tokens, cudaStream_t stream);

// Rotary embedding parameters: inverse frequencies for the `head_dim/2` rotated pairs, and the
// attention factor YaRN scales cos/sin by.
struct RopeTable {
  const float* inv_freq;  // [head_dim / 2]
  float attention_factor;
};

// Attention front of one call: splits the packed q/k/v projection rows, applies the per-head
// RMSNorm to q and k (when q_norm/k_norm are given), rotates q and k by position (half-split
// pairs j, j + d/2), writes rotated q to `q_out` [rows, q_heads, head_dim] and k/v into the paged
// cache slot of each row.
//
// Cache layout per layer: block b is `page_bytes` bytes holding K[kv_heads][16][head_dim] then
// V[kv_heads][16][head_dim] in BF16. slot_mapping[r] = block * 16 + offset, or -1 to skip. With
// `cache_slots` > 0 (blocks * 16) a slot at or past it writes nothing and records kBadIndex in
// `status`.
int qk_norm_rope_cache(const __nv_bfloat16* qkv, long ld_qkv, int rows, int q_heads, int kv_heads,
                       int head_dim, const __nv_bfloat16* q_norm, const __nv_bfloat16* k_norm,
                       float eps, const int32_t* positions, RopeTable rope,
                       __nv_bfloat16* q_out, __nv_bfloat16* cache, const int32_t* slot_mapping,
                       cudaStream_t stream, long cache_slots = 0, int* status = nullptr,
                       const GemmSplits* splits = nullptr);

// With `splits` (from gemm_bf16_splits of the q/k/v GEMM, more than one split) the projection is
// read as the sum of its K splits' FP32 partials in split order, rounded once to BF16 (what the
// GEMM would have stored), and `qkv` is not read.

// LoRA: zeroes z[r, 0:cols) (row stride ldz) of every row r whose row_slot[r] is not `slot`.
int lora_mask(__nv_bfloat16* z, long ldz, int rows, int cols, int slot, const int32_t* row_slot,
              cudaStream_t stream);

// Fills `n` BF16 values with N(0, std) from a counter-based hash of (seed, index): the same
// values on every device and every run.
int init_normal_bf16(__nv_bfloat16* dst, long n, float std, uint64_t seed, cudaStream_t stream);

// Fills a [rows, cols] BF16 shard of a larger logical matrix with N(0, std): shard row r is
// logical row full_row[r] of the matrix tagged tag[r], columns start at col_offset of full_cols.
// The values depend on (seed, tag, logical index) only, so every tensor-parallel split of one
// model holds the same logical weights.
int init_normal_rows(__nv_bfloat16* dst, int rows, int cols, const int32_t* full_row,
                     const uint32_t* tag, long full_cols, long col_offset, float std, uint64_t seed,
                     cudaStream_t stream);

// Fills `n` BF16 values with a constant.
int fill_bf16(__nv_bfloat16* dst, long n, float value, cudaStream_t stream);

// Token gather: `sources` holds `count` records (address low, address high, length, first row) of
// I32 device arrays; copies each into `out` at its first row.
int gather_tokens(const int32_t* sources, int count, int32_t* out, cudaStream_t stream);

// out[i, :] = in[rows[i], :] for i < n, BF16 rows of `cols` elements.
int gather_rows(const __nv_bfloat16* in, long ldi, const int32_t* rows, int n, __nv_bfloat16* out,
                long ldo, int cols, cudaStream_t stream);

}  // namespace foa
