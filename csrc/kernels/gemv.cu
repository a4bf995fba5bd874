// Decode projections of one row: C = epilogue(A . W^T) as a weight stream.
//
// With few rows a projection reads every weight once and does M multiply-adds a weight: it is
// bound by HBM, and the tensor-core GEMM's per-launch cost (a full shared-memory ring, TMEM, the
// pipeline fill, split-K reduction) dominates its few microseconds. This kernel keeps no shared
// memory: every warp streams two weight rows with 16-byte non-allocating loads (four in flight a
// row), multiplies them against the rows of A read through L2, and reduces across the warp. Its
// small CTAs fit beside the previous kernel's, and each issues its first weight loads before the
// programmatic-dependent-launch wait, so the stream starts while the producer of A finishes.
//
// Numerics: FP32 accumulation and one rounding, the epilogues of the tensor-core GEMM (residual
// add before the rounding; SwiGLU rounded as the reference rounds it). The sum runs in another
// order than the tensor-core GEMM, so batch-invariant loads keep that GEMM for every row count.

#include <cuda_bf16.h>

#include "gemm.cuh"
#include "launch.cuh"
#include "sm100.cuh"

namespace foa {
namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvUnroll = 4;  // 16-byte weight loads in flight a row

struct GemvArgs {
  const __nv_bfloat16* a;
  long lda;
  const __nv_bfloat16* w;
  long ldw;
  int M, N, K;
  void* c;
  long ldc;
  const __nv_bfloat16* res;
  long ldr;
  int epilogue;
};

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void fma8(float& acc, const uint4& w, const uint4& x) {
  acc = fmaf(bf16_lo(w.x), bf16_lo(x.x), acc);
  acc = fmaf(bf16_hi(w.x), bf16_hi(x.x), acc);
  acc = fmaf(bf16_lo(w.y), bf16_lo(x.y), acc);
  acc = fmaf(bf16_hi(w.y), bf16_hi(x.y), acc);
  acc = fmaf(bf16_lo(w.z), bf16_lo(x.z), acc);
  acc = fmaf(bf16_hi(w.z), bf16_hi(x.z), acc);
  acc = fmaf(bf16_lo(w.w), bf16_lo(x.w), acc);
  acc = fmaf(bf16_hi(w.w), bf16_hi(x.w), acc);
}

__device__ __forceinline__ float silu_times(float g_acc, float u_acc) {
  const float g = __bfloat162float(__float2bfloat16_rn(g_acc));
  const float u = __bfloat162float(__float2bfloat16_rn(u_acc));
  const float s = __bfloat162float(__float2bfloat16_rn(g / (1.0f + __expf(-g))));
  return s * u;
}

template <int MB>
__global__ void __launch_bounds__(32 * kGemvWarps) gemv_kernel(const GemvArgs p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int unit = blockIdx.x * kGemvWarps + warp;  // a pair of weight rows
  const bool swiglu = p.epilogue == kEpiSwiGLU;
  // SwiGLU: output column j reads gate row (j / 128) * 256 + j % 128 and the up row 128 below.
  const int r0 = swiglu ? (unit / 128) * 256 + unit % 128 : 2 * unit;
  const int r1 = swiglu ? r0 + 128 : r0 + 1;
  const bool ok0 = r0 < p.N, ok1 = r1 < p.N;
  const __nv_bfloat16* w0 = p.w + (long)(ok0 ? r0 : 0) * p.ldw;
  const __nv_bfloat16* w1 = p.w + (long)(ok1 ? r1 : 0) * p.ldw;
  const int steps = (p.K + 255) / 256;  // 256 columns a step (8 a lane)
  float acc[2][MB];
#pragma unroll
  for (int m = 0; m < MB; ++m) acc[0][m] = acc[1][m] = 0.f;

  // The first weights do not depend on the previous kernel: load them before waiting for it.
  uint4 wa[kGemvUnroll], wb[kGemvUnroll];
  auto load = [&](int s0) {
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u) {
      const int k = (s0 + u) * 256 + lane * 8;
      const bool in = k < p.K;
      wa[u] = in && ok0 ? ld_stream(w0 + k) : make_uint4(0, 0, 0, 0);
      wb[u] = in && ok1 ? ld_stream(w1 + k) : make_uint4(0, 0, 0, 0);
    }
  };
  load(0);
  pdl_trigger();
  pdl_wait();
  for (int s0 = 0; s0 < steps; s0 += kGemvUnroll) {
    uint4 ca[kGemvUnroll], cb[kGemvUnroll];
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u) {
      ca[u] = wa[u];
      cb[u] = wb[u];
    }
    if (s0 + kGemvUnroll < steps) load(s0 + kGemvUnroll);  // the next weights while this step multiplies
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u) {
      const int k = (s0 + u) * 256 + lane * 8;
      if (k >= p.K) break;
#pragma unroll
      for (int m = 0; m < MB; ++m) {
        if (m >= p.M) break;
        const uint4 x = __ldcg(reinterpret_cast<const uint4*>(p.a + (long)m * p.lda + k));
        fma8(acc[0][m], ca[u], x);
        fma8(acc[1][m], cb[u], x);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MB; ++m) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc[0][m] += __shfl_xor_sync(0xffffffffu, acc[0][m], o);
      acc[1][m] += __shfl_xor_sync(0xffffffffu, acc[1][m], o);
    }
  }
  // Lane m writes row m's outputs of this pair.
#pragma unroll
  for (int m = 0; m < MB; ++m) {
    if (lane != m || m >= p.M) continue;
    if (swiglu) {
      if (unit < p.N / 2)
        static_cast<__nv_bfloat16*>(p.c)[(long)m * p.ldc + unit] =
            __float2bfloat16_rn(silu_times(acc[0][m], acc[1][m]));
    } else if (p.epilogue == kEpiF32) {
      float* c = static_cast<float*>(p.c);
      if (ok0) c[(long)m * p.ldc + r0] = acc[0][m];
      if (ok1) c[(long)m * p.ldc + r1] = acc[1][m];
    } else {
      __nv_bfloat16* c = static_cast<__nv_bfloat16*>(p.c);
      float v0 = acc[0][m], v1 = acc[1][m];
      if (p.res != nullptr) {
        if (ok0) v0 += __bfloat162float(p.res[(long)m * p.ldr + r0]);
        if (ok1) v1 += __bfloat162float(p.res[(long)m * p.ldr + r1]);
      }
      if (ok0) c[(long)m * p.ldc + r0] = __float2bfloat16_rn(v0);
      if (ok1) c[(long)m * p.ldc + r1] = __float2bfloat16_rn(v1);
    }
  }
}

}  // namespace

bool gemv_applies(const GemmArgs& a) {
  const bool aligned = (reinterpret_cast<uintptr_t>(a.a) | reinterpret_cast<uintptr_t>(a.w)) % 16 == 0 &&
                       a.lda % 8 == 0 && a.ldw % 8 == 0;
  const bool epi = a.epilogue == kEpiBf16 || a.epilogue == kEpiF32 ||
                   (a.epilogue == kEpiSwiGLU && a.N % 256 == 0);
  // The weight stream beats the tensor-core GEMM at one row, K up to 4096 and N up to 16384 (B200,
  // the Qwen3-1.7B projections: o 4.8 against 6.0 us, gate/up 13.5 against 14.3 us); with two rows,
  // a longer K or a vocabulary-wide N the tensor-core GEMM is faster.
  return a.M == 1 && a.K <= 4096 && a.N <= 16384 && a.mode == kModeAuto && a.splits == 0 && a.w_format == 0 && a.K % 8 == 0 &&
         aligned && epi && a.seg[0].K == 0 && a.group_tiles == nullptr && a.trace == nullptr &&
         a.cta_trace == nullptr && a.debug == 0 && a.reduction == 0 && (a.epilogue != kEpiSwiGLU || a.residual == nullptr);
}

int gemv_bf16(const GemmArgs& a, cudaStream_t stream) {
  GemvArgs p;
  p.a = static_cast<const __nv_bfloat16*>(a.a);
  p.lda = a.lda;
  p.w = static_cast<const __nv_bfloat16*>(a.w);
  p.ldw = a.ldw;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.c = a.c;
  p.ldc = a.ldc;
  p.res = static_cast<const __nv_bfloat16*>(a.residual);
  p.ldr = a.ldr;
  p.epilogue = a.epilogue;
  const int units = a.epilogue == kEpiSwiGLU ? a.N / 2 : (a.N + 1) / 2;
  const dim3 grid((units + kGemvWarps - 1) / kGemvWarps), block(32 * kGemvWarps);
  cudaError_t e;
  if (a.M <= 1) e = launch_pdl(gemv_kernel<1>, grid, block, 0, stream, p);
  else if (a.M <= 2) e = launch_pdl(gemv_kernel<2>, grid, block, 0, stream, p);
  else if (a.M <= 4) e = launch_pdl(gemv_kernel<4>, grid, block, 0, stream, p);
  else e = launch_pdl(gemv_kernel<8>, grid, block, 0, stream, p);
  return e == cudaSuccess ? 0 : -5;
}

}  // namespace foa
