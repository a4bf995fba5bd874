// Row kernels of the media encoders: one CTA of 256 threads per row, the row staged in shared
// memory as FP32, statistics reduced in FP32 over the block.
//
// Reference: the Gemma-4 unified embedders (crates/furiosa-opt-models/src/models/vision_language/
// gemma4_unified.rs:1-13, :83-95): the patch path normalizes, projects, normalizes, adds one row
// of a factorized position table per coordinate and normalizes again, every sum rounded to BF16;
// `embed_vision` / `embed_audio` apply a unit-gain RMS norm before their projection.

#include "launch.cuh"
#include "media.cuh"
#include "sm100.cuh"

namespace foa {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Sum over the CTA (every thread gets the total); `red` holds 8 floats.
__device__ __forceinline__ float cta_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();  // `red` free from a previous use
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) t += red[w];
  return t;
}

// LayerNorm of the row staged in `xs` (FP32 values of BF16 numbers), results rounded into `xs`.
__device__ __forceinline__ void layernorm_row(float* xs, int cols, const __nv_bfloat16* w,
                                              const __nv_bfloat16* b, float eps, float* red) {
  float s = 0.f;
  for (int c = threadIdx.x; c < cols; c += kThreads) s += xs[c];
  const float mean = cta_sum(s, red) / (float)cols;
  float q = 0.f;
  for (int c = threadIdx.x; c < cols; c += kThreads) {
    const float d = xs[c] - mean;
    q += d * d;
  }
  const float rstd = rsqrtf(cta_sum(q, red) / (float)cols + eps);
  for (int c = threadIdx.x; c < cols; c += kThreads)
    xs[c] = bf16r((xs[c] - mean) * rstd * __bfloat162float(w[c]) + __bfloat162float(b[c]));
  __syncthreads();
}

__global__ void __launch_bounds__(kThreads) media_layernorm_kernel(
    const __nv_bfloat16* __restrict__ x, long ldx, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ b, float eps, __nv_bfloat16* __restrict__ out, long ldo, int cols) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float xs[];
  __shared__ float red[kThreads / 32];
  const long row = blockIdx.x;
  for (int c = threadIdx.x; c < cols; c += kThreads) xs[c] = __bfloat162float(x[row * ldx + c]);
  __syncthreads();
  layernorm_row(xs, cols, w, b, eps, red);
  for (int c = threadIdx.x; c < cols; c += kThreads) out[row * ldo + c] = __float2bfloat16_rn(xs[c]);
}

__global__ void __launch_bounds__(kThreads) media_vision_tail_kernel(
    const float* __restrict__ acc, long lda, const float* __restrict__ bias,
    const __nv_bfloat16* __restrict__ ln_w, const __nv_bfloat16* __restrict__ ln_b,
    const __nv_bfloat16* __restrict__ table, const int32_t* __restrict__ positions,
    const __nv_bfloat16* __restrict__ pn_w, const __nv_bfloat16* __restrict__ pn_b, float ln_eps,
    float unit_eps, __nv_bfloat16* __restrict__ out, long ldo, int cols) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float xs[];
  __shared__ float red[kThreads / 32];
  const long row = blockIdx.x;
  // The projection with its bias, rounded once.
  for (int c = threadIdx.x; c < cols; c += kThreads) xs[c] = bf16r(acc[row * lda + c] + bias[c]);
  __syncthreads();
  layernorm_row(xs, cols, ln_w, ln_b, ln_eps, red);
  // The factorized position row: x's row of coordinate 0 plus y's of coordinate 1, rounded once,
  // then added to the patch row.
  const __nv_bfloat16* px = table + (long)(2 * positions[2 * row]) * cols;
  const __nv_bfloat16* py = table + (long)(2 * positions[2 * row + 1] + 1) * cols;
  for (int c = threadIdx.x; c < cols; c += kThreads)
    xs[c] = bf16r(xs[c] + bf16r(__bfloat162float(px[c]) + __bfloat162float(py[c])));
  __syncthreads();
  layernorm_row(xs, cols, pn_w, pn_b, ln_eps, red);
  float q = 0.f;
  for (int c = threadIdx.x; c < cols; c += kThreads) q += xs[c] * xs[c];
  const float inv = rsqrtf(cta_sum(q, red) / (float)cols + unit_eps);
  for (int c = threadIdx.x; c < cols; c += kThreads) out[row * ldo + c] = __float2bfloat16_rn(xs[c] * inv);
}

__global__ void __launch_bounds__(kThreads) media_unit_rmsnorm_kernel(
    const __nv_bfloat16* __restrict__ x, long ldx, float eps, __nv_bfloat16* __restrict__ out, long ldo, int cols) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[kThreads / 32];
  const long row = blockIdx.x;
  float q = 0.f;
  for (int c = threadIdx.x; c < cols; c += kThreads) {
    const float v = __bfloat162float(x[row * ldx + c]);
    q += v * v;
  }
  const float inv = rsqrtf(cta_sum(q, red) / (float)cols + eps);
  for (int c = threadIdx.x; c < cols; c += kThreads)
    out[row * ldo + c] = __float2bfloat16_rn(__bfloat162float(x[row * ldx + c]) * inv);
}

int row_smem(int cols) { return cols * (int)sizeof(float); }

template <typename K>
bool allow_smem(K kernel, int bytes) {
  if (bytes <= 48 * 1024) return true;
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess;
}

}  // namespace

int media_layernorm(const __nv_bfloat16* x, long ldx, const __nv_bfloat16* w, const __nv_bfloat16* b,
                    float eps, __nv_bfloat16* out, long ldo, int rows, int cols, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (cols <= 0 || cols > 12288) return -2;
  if (!allow_smem(media_layernorm_kernel, row_smem(cols))) return -5;
  return launch_pdl(media_layernorm_kernel, dim3(rows), dim3(kThreads), row_smem(cols), stream, x, ldx, w, b,
                    eps, out, ldo, cols) == cudaSuccess
             ? 0
             : -5;
}

int media_vision_tail(const float* acc, long lda, const float* bias, const __nv_bfloat16* ln_w,
                      const __nv_bfloat16* ln_b, const __nv_bfloat16* table, const int32_t* positions,
                      const __nv_bfloat16* pn_w, const __nv_bfloat16* pn_b, float ln_eps, float unit_eps,
                      __nv_bfloat16* out, long ldo, int rows, int cols, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (cols <= 0 || cols > 12288) return -2;
  if (!allow_smem(media_vision_tail_kernel, row_smem(cols))) return -5;
  return launch_pdl(media_vision_tail_kernel, dim3(rows), dim3(kThreads), row_smem(cols), stream, acc, lda,
                    bias, ln_w, ln_b, table, positions, pn_w, pn_b, ln_eps, unit_eps, out, ldo, cols) ==
                 cudaSuccess
             ? 0
             : -5;
}

int media_unit_rmsnorm(const __nv_bfloat16* x, long ldx, float eps, __nv_bfloat16* out, long ldo,
                       int rows, int cols, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (cols <= 0) return -2;
  return launch_pdl(media_unit_rmsnorm_kernel, dim3(rows), dim3(kThreads), 0, stream, x, ldx, eps, out, ldo,
                    cols) == cudaSuccess
             ? 0
             : -5;
}

}  // namespace foa
