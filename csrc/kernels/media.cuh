// Row kernels of the media encoders (the Gemma-4 unified patch and audio embedders): LayerNorm,
// the vision embedder's tail after its patch projection, and the unit-gain RMS norm.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace foa {

// out = bf16((x - mean) * rsqrt(var + eps) * w + b) per row, FP32 statistics (torch.nn.LayerNorm
// over BF16 rows). cols a multiple of 8, at most 12288.
int media_layernorm(const __nv_bfloat16* x, long ldx, const __nv_bfloat16* w, const __nv_bfloat16* b,
                    float eps, __nv_bfloat16* out, long ldo, int rows, int cols, cudaStream_t stream);

// The vision embedder after its patch projection, per patch row (each step rounded to BF16 as the
// BF16 forward of the reference model rounds it):
//   v = bf16(acc + bias); a = LayerNorm(v; ln); s = bf16(a + bf16(table[2x] + table[2y + 1]));
//   n = LayerNorm(s; pos_norm); out = bf16(n * rsqrt(mean(n^2) + unit_eps))
// `acc` holds the projection's FP32 sums, `table` the factorized positions [positions][2][cols]
// and `positions` each row's (x, y).
int media_vision_tail(const float* acc, long lda, const float* bias, const __nv_bfloat16* ln_w,
                      const __nv_bfloat16* ln_b, const __nv_bfloat16* table, const int32_t* positions,
                      const __nv_bfloat16* pn_w, const __nv_bfloat16* pn_b, float ln_eps, float unit_eps,
                      __nv_bfloat16* out, long ldo, int rows, int cols, cudaStream_t stream);

// out = bf16(x * rsqrt(mean(x^2) + eps)) per row (RMS norm without a gain).
int media_unit_rmsnorm(const __nv_bfloat16* x, long ldx, float eps, __nv_bfloat16* out, long ldo,
                       int rows, int cols, cudaStream_t stream);

}  // namespace foa
