// Quantizers of the FP8 block-scaled and NVFP4 weight formats (the reference's forms:
// crates/furiosa-opt-models/src/tensor/form/{fp8,nvfp4}.rs; NVFP4 rounding as vLLM's reference
// quantizer rounds).
#include <cuda_fp8.h>

#include <algorithm>

#include "launch.cuh"
#include "quant.cuh"
#include "sm100.cuh"

namespace foa {
namespace {

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  return m;
}

// One CTA of 256 threads per 128x128 block.
__global__ void __launch_bounds__(256) fp8_block_kernel(const __nv_bfloat16* w, int rows, int cols,
                                                        uint8_t* codes, float* scales) {
  pdl_wait();  // no early trigger: a dependent GEMM reads these codes before its own wait
  __shared__ float red[8];
  const int br = blockIdx.y, bc = blockIdx.x;
  const int r0 = br * 128, c0 = bc * 128;
  float m = 0.f;
  for (int i = threadIdx.x; i < 128 * 128; i += 256) {
    const int r = r0 + i / 128, c = c0 + i % 128;
    if (r < rows && c < cols) m = fmaxf(m, fabsf(__bfloat162float(w[(long)r * cols + c])));
  }
  const float amax = block_max(m, red);
  const float scale = fmaxf(amax, 1e-10f) * (1.f / 448.f);
  if (threadIdx.x == 0) scales[(long)br * gridDim.x + bc] = scale;
  for (int i = threadIdx.x; i < 128 * 128; i += 256) {
    const int r = r0 + i / 128, c = c0 + i % 128;
    if (r < rows && c < cols)
      codes[(long)r * cols + c] =
          __nv_cvt_float_to_fp8(__bfloat162float(w[(long)r * cols + c]) / scale, __NV_SATFINITE, __NV_E4M3);
  }
}

// FP8 activations per (row, 128-input group), one warp per group: scale = max(amax, 1e-10) *
// fl(1/448), code = e4m3_sat(x / scale). Scales land transposed, [K/128][rows_pad], so that the
// scales of one k-block are contiguous over rows.
__global__ void fp8_act_kernel(const __nv_bfloat16* x, long ldx, int rows, int K, uint8_t* codes,
                               long ldc, float* scales, int rows_pad) {
  pdl_wait();
  pdl_trigger();
  const int groups = K / 128;
  const long wid = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (long)rows * groups) return;
  const long r = wid / groups;
  const int g = (int)(wid % groups);
  const uint2 q = *reinterpret_cast<const uint2*>(x + r * ldx + g * 128 + lane * 4);
  float v[4] = {__uint_as_float(q.x << 16), __uint_as_float(q.x & 0xFFFF0000u),
                __uint_as_float(q.y << 16), __uint_as_float(q.y & 0xFFFF0000u)};
  float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float scale = fmaxf(m, 1e-10f) * (1.f / 448.f);
  if (lane == 0) scales[(long)g * rows_pad + r] = scale;
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    packed |= (uint32_t)__nv_cvt_float_to_fp8(v[i] / scale, __NV_SATFINITE, __NV_E4M3) << (8 * i);
  *reinterpret_cast<uint32_t*>(codes + r * ldc + g * 128 + lane * 4) = packed;
}

__global__ void absmax_kernel(const __nv_bfloat16* x, long n, float* out) {
  pdl_wait();  // no early trigger: a dependent GEMM reads these codes before its own wait
  float m = 0.f;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(__bfloat162float(x[i])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  // Non-negative floats order as their bit patterns.
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<int*>(out), __float_as_int(m));
}

// E2M1 code of |x| (x >= 0) rounded to nearest, ties to the even code.
__device__ __forceinline__ uint32_t e2m1_magnitude(float m) {
  return m <= 0.25f ? 0u : m < 0.75f ? 1u : m <= 1.25f ? 2u : m < 1.75f ? 3u
       : m <= 2.5f ? 4u : m < 3.5f ? 5u : m <= 5.f ? 6u : 7u;
}

// The factor a group's values take before E2M1 rounding: 1 / (s * (1 / global)), 0 when the
// block scale s is 0 (the order of vLLM's reference NVFP4 quantizer).
__device__ __forceinline__ float code_factor(__nv_fp8_storage_t s8, float global) {
  const __half_raw hr = __nv_cvt_fp8_to_halfraw(s8, __NV_E4M3);
  const float s = __half2float(__half(hr));
  const float restore = s * (1.f / global);
  return restore != 0.f ? 1.f / restore : 0.f;
}

// 16 values -> 8 bytes of E2M1 codes (lower index in the low nibble).
__device__ __forceinline__ uint2 e2m1_pack16(const float (&v)[16], float k) {
  uint32_t packed[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float x = v[i] * k;
    const uint32_t code = e2m1_magnitude(fabsf(x)) | (x < 0.f ? 8u : 0u);
    packed[i / 8] |= code << (4 * (i % 8));
  }
  return make_uint2(packed[0], packed[1]);
}

// Byte offset of the scale of (row, 16-group g) in 128-row-blocked atoms of a K-column matrix.
__device__ __forceinline__ long sf_atom_offset(long row, int g, int K) {
  const long rb = row >> 7;
  const int rr = (int)(row & 127);
  return (rb * (K / 64) + g / 4) * 512 + (rr & 31) * 16 + (rr >> 5) * 4 + (g & 3);
}

// One thread per 16-element group.
__global__ void nvfp4_kernel(const __nv_bfloat16* w, int rows, int cols, uint8_t* codes,
                             uint8_t* scales, const float* amax_p, float* tensor_scale) {
  pdl_wait();  // no early trigger: a dependent GEMM reads these codes before its own wait
  const int groups = cols / 16;
  const long g = blockIdx.x * (long)blockDim.x + threadIdx.x;
  const float amax = *amax_p;
  const float global = amax > 0.f ? 448.f * 6.f / amax : 1.f;
  if (g == 0 && tensor_scale != nullptr) *tensor_scale = 1.f / global;
  if (g >= (long)rows * groups) return;
  const long r = g / groups, c0 = (g % groups) * 16;
  float v[16], m = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    v[i] = __bfloat162float(w[r * cols + c0 + i]);
    m = fmaxf(m, fabsf(v[i]));
  }
  const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(m / 6.f * global, __NV_SATFINITE, __NV_E4M3);
  scales[r * groups + c0 / 16] = s8;
  const float k = code_factor(s8, global);
  *reinterpret_cast<uint2*>(codes + r * (cols / 2) + c0 / 2) = e2m1_pack16(v, k);
}

// Activations under a fixed tensor scale (W4A4 inputs): one thread per 16-group of the padded
// rows; rows past `rows` get zero codes and zero scales.
__global__ void nvfp4_act_kernel(const __nv_bfloat16* x, long ldx, int rows, int rows_pad, int K,
                                 float global, uint8_t* codes, long ldc, uint8_t* sf) {
  pdl_wait();
  pdl_trigger();
  const int groups = K / 16;
  const long g = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (g >= (long)rows_pad * groups) return;
  const long r = g / groups;
  const int gi = (int)(g % groups);
  if (r >= rows) {
    sf[sf_atom_offset(r, gi, K)] = 0;
    return;
  }
  float v[16], m = 0.f;
  const uint4* src = reinterpret_cast<const uint4*>(x + r * ldx + gi * 16);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint4 q = src[h];
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[h * 8 + 2 * i] = __uint_as_float(w[i] << 16);
      v[h * 8 + 2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[i]));
  const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(m / 6.f * global, __NV_SATFINITE, __NV_E4M3);
  sf[sf_atom_offset(r, gi, K)] = s8;
  *reinterpret_cast<uint2*>(codes + r * ldc + gi * 8) = e2m1_pack16(v, code_factor(s8, global));
}

// Row-major scales [rows][K/16] -> 128-row-blocked atoms (zero for the padded rows).
__global__ void sf_atoms_kernel(const uint8_t* src, long lds, int rows, int rows_pad, int K, uint8_t* dst) {
  pdl_wait();  // weight producer: no early trigger
  const int groups = K / 16;
  const long g = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (g >= (long)rows_pad * groups) return;
  const long r = g / groups;
  const int gi = (int)(g % groups);
  dst[sf_atom_offset(r, gi, K)] = r < rows ? src[r * lds + gi] : 0;
}

}  // namespace

int quantize_fp8_block(const __nv_bfloat16* w, int rows, int cols, uint8_t* codes, float* scales,
                       cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return 0;
  dim3 grid((cols + 127) / 128, (rows + 127) / 128);
  return launch_pdl(fp8_block_kernel, grid, dim3(256), 0, stream, w, rows, cols, codes, scales) ==
                 cudaSuccess
             ? 0
             : -5;
}

__global__ void pad4_kernel(const float* src, long n, float4* dst) {
  pdl_wait();  // weight producer: no early trigger
  const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
  if (i < n) {
    const float v = src[i];
    dst[i] = make_float4(v, v, v, v);
  }
}

int fp8_scales_pad4(const float* scales, long n, float* padded, cudaStream_t stream) {
  if (n <= 0) return 0;
  return launch_pdl(pad4_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, stream, scales, n,
                    reinterpret_cast<float4*>(padded)) == cudaSuccess
             ? 0
             : -5;
}

// One warp per row: scale = amax / 448 (the row's, or `tensor_amax` when >= 0), code =
// e4m3_sat(w * (1 / scale)); a zero scale gives zero codes.
__global__ void fp8_rows_kernel(const __nv_bfloat16* w, int rows, int cols, float tensor_amax, uint8_t* codes,
                                float* scales) {
  pdl_wait();  // weight producer: no early trigger
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const __nv_bfloat16* src = w + (long)r * cols;
  float m = 0.f;
  if (tensor_amax >= 0.f) {
    m = tensor_amax;
  } else {
    for (int c = lane; c < cols; c += 32) m = fmaxf(m, fabsf(__bfloat162float(src[c])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  }
  const float scale = m / 448.f;
  const float rcp = scale == 0.f ? 0.f : 1.f / scale;
  if (lane == 0) scales[r] = scale;
  for (int c = lane; c < cols; c += 32)
    codes[(long)r * cols + c] = __nv_cvt_float_to_fp8(__bfloat162float(src[c]) * rcp, __NV_SATFINITE, __NV_E4M3);
}

int quantize_fp8_rows(const __nv_bfloat16* w, int rows, int cols, float tensor_amax, uint8_t* codes,
                      float* scales, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return 0;
  return launch_pdl(fp8_rows_kernel, dim3((unsigned)((rows * 32L + 255) / 256)), dim3(256), 0, stream, w, rows,
                    cols, tensor_amax, codes, scales) == cudaSuccess
             ? 0
             : -5;
}

int quantize_fp8_act(const __nv_bfloat16* x, long ldx, int rows, int K, uint8_t* codes, long ldc,
                     float* scales, int rows_pad, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (K % 128 != 0 || ldx % 4 != 0 || (reinterpret_cast<uintptr_t>(x) & 7) || ldc % 4 != 0 ||
      rows_pad < rows)
    return -2;
  const long warps = (long)rows * (K / 128);
  return launch_pdl(fp8_act_kernel, dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, stream,
                    x, ldx, rows, K, codes, ldc, scales, rows_pad) == cudaSuccess
             ? 0
             : -5;
}

int quantize_nvfp4_act(const __nv_bfloat16* x, long ldx, int rows, int K, float global,
                       uint8_t* codes, long ldc, uint8_t* sf_atoms, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (K % 64 != 0 || ldx % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || ldc % 8 != 0) return -2;
  const int rows_pad = (rows + 127) / 128 * 128;
  const long groups = (long)rows_pad * (K / 16);
  return launch_pdl(nvfp4_act_kernel, dim3((unsigned)((groups + 255) / 256)), dim3(256), 0, stream, x,
                    ldx, rows, rows_pad, K, global, codes, ldc, sf_atoms) == cudaSuccess
             ? 0
             : -5;
}

int nvfp4_scale_atoms(const uint8_t* scales, long lds, int rows, int K, uint8_t* sf_atoms,
                      cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (K % 64 != 0) return -2;
  const int rows_pad = (rows + 127) / 128 * 128;
  const long groups = (long)rows_pad * (K / 16);
  return launch_pdl(sf_atoms_kernel, dim3((unsigned)((groups + 255) / 256)), dim3(256), 0, stream,
                    scales, lds, rows, rows_pad, K, sf_atoms) == cudaSuccess
             ? 0
             : -5;
}

int absmax_bf16(const __nv_bfloat16* x, long n, float* out, cudaStream_t stream) {
  if (n <= 0) return 0;
  const int grid = (int)std::min<long>((n + 255) / 256, 148L * 8);
  return launch_pdl(absmax_kernel, dim3(grid), dim3(256), 0, stream, x, n, out) == cudaSuccess ? 0 : -5;
}

int quantize_nvfp4(const __nv_bfloat16* w, int rows, int cols, uint8_t* codes, uint8_t* scales,
                   const float* amax, float* tensor_scale, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return 0;
  if (cols % 16 != 0) return -2;
  const long groups = (long)rows * (cols / 16);
  return launch_pdl(nvfp4_kernel, dim3((unsigned)((groups + 255) / 256)), dim3(256), 0, stream, w,
                    rows, cols, codes, scales, amax, tensor_scale) == cudaSuccess
             ? 0
             : -5;
}

}  // namespace foa
