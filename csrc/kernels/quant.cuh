// Weight and activation quantizers of the FP8 and NVFP4 formats.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace foa {

// Block-scaled FP8: W [rows, cols] BF16 -> E4M3 codes [rows, cols] and FP32 scales
// [ceil(rows/128), ceil(cols/128)] with one scale per 128x128 block:
// scale = max(amax(block), 1e-10) * fl(1/448), code = e4m3_rne(w / scale) saturated to +-448.
int quantize_fp8_block(const __nv_bfloat16* w, int rows, int cols, uint8_t* codes, float* scales,
                       cudaStream_t stream);

// FP8 at load (the reference's per-channel / per-tensor granularity): E4M3 codes [rows, cols] and
// one FP32 scale per row, scale = amax / 448 over the row, or `tensor_amax` / 448 for every row
// when tensor_amax >= 0 (a tensor scale covering the weights fused with it); code =
// e4m3_sat(w * (1 / scale)), zero codes for a zero scale.
int quantize_fp8_rows(const __nv_bfloat16* w, int rows, int cols, float tensor_amax, uint8_t* codes,
                      float* scales, cudaStream_t stream);

// NVFP4 (E2M1 codes, E4M3 scale per 16 elements along cols, FP32 tensor scale):
// global = 448 * 6 / amax(W) (the tensor's "weight_scale_2" is 1 / global);
// block scale s = e4m3(amax(block) / 6 * global); code = e2m1_rne(w / (s * (1 / global))).
// Codes pack two per byte, the lower column in the low nibble. `amax` is a device FP32 holding
// amax(W) (absmax_bf16 computes it); `tensor_scale`, when not null, receives 1 / global.
int quantize_nvfp4(const __nv_bfloat16* w, int rows, int cols, uint8_t* codes, uint8_t* scales,
                   const float* amax, float* tensor_scale, cudaStream_t stream);

// The W8A8 GEMM's weight-scale layout: each of n FP32 block scales four times (16 bytes apiece), so
// that the GEMM stages one block's scale with a 16-byte bulk copy.
int fp8_scales_pad4(const float* scales, long n, float* padded, cudaStream_t stream);

// FP8 activations per (row, 128-input group), the W8A8 input form of the block-scaled FP8 GEMM:
// scale = max(amax, 1e-10) * fl(1/448), codes [rows, K] E4M3 (row stride ldc bytes), scales FP32
// [K/128][rows_pad] (rows_pad >= rows; entries past `rows` are not written).
int quantize_fp8_act(const __nv_bfloat16* x, long ldx, int rows, int K, uint8_t* codes, long ldc,
                     float* scales, int rows_pad, cudaStream_t stream);

// NVFP4 activations under a fixed tensor scale `global` (1 / the checkpoint's input_scale), the
// W4A4 input form of the block-scaled GEMM: codes [rows, K/2] (row stride ldc bytes) and scales as
// 128-row-blocked atoms [ceil(rows/128)][K/64][512] (padded rows zero).
int quantize_nvfp4_act(const __nv_bfloat16* x, long ldx, int rows, int K, float global,
                       uint8_t* codes, long ldc, uint8_t* sf_atoms, cudaStream_t stream);

// Row-major E4M3 scales [rows][K/16] (row stride lds) -> the 128-row-blocked atoms the
// block-scaled GEMM reads.
int nvfp4_scale_atoms(const uint8_t* scales, long lds, int rows, int K, uint8_t* sf_atoms,
                      cudaStream_t stream);

// amax over n BF16 values into *out (out must start at 0).
int absmax_bf16(const __nv_bfloat16* x, long n, float* out, cudaStream_t stream);

}  // namespace foa
