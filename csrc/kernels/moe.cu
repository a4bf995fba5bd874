// Mixture-of-experts routing, grouping and combine (contract in moe.cuh).
#include <cuda_bf16.h>

#include "launch.cuh"
#include "moe.cuh"

namespace foa {
namespace {

constexpr int kMaxExperts = 512;

// One warp per row: softmax over the experts, then k rounds of a warp-wide (largest logit, lowest
// expert) selection.
__global__ void route_kernel(const __nv_bfloat16* logits, long ld, int rows, int experts, int k,
                             int normalize, int32_t* ids, float* weights) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const __nv_bfloat16* row = logits + (long)warp * ld;
  float v[kMaxExperts / 32];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxExperts / 32; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < experts ? __bfloat162float(row[e]) : -INFINITY;
    m = fmaxf(m, v[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxExperts / 32; ++i)
    if (lane + 32 * i < experts) sum += expf(v[i] - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  uint32_t taken = 0;
  float total = 0.f;
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int be = 0x7fffffff;  // none yet
#pragma unroll
    for (int i = 0; i < kMaxExperts / 32; ++i) {
      const int e = lane + 32 * i;
      if (e < experts && !(taken >> i & 1u) && (be == 0x7fffffff || v[i] > best)) {
        best = v[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      const bool take = oe != 0x7fffffff &&
                        (be == 0x7fffffff || ob > best || (ob == best && oe < be));
      if (take) {
        best = ob;
        be = oe;
      }
    }
    if ((be & 31) == lane) taken |= 1u << (be >> 5);
    const float pr = expf(best - m) / sum;
    total += pr;  // choice order
    if (lane == 0) {
      ids[(long)warp * k + j] = be;
      weights[(long)warp * k + j] = pr;
    }
  }
  if (lane == 0 && normalize)
    for (int j = 0; j < k; ++j) weights[(long)warp * k + j] /= total;
}

constexpr int kAlignThreads = 512;
constexpr int kAlignWarps = kAlignThreads / 32;

// CTA c groups the experts [first + c * count, first + (c + 1) * count) and writes its positions
// to pos + c * rows * k; only CTA `local` writes the sorted rows' sources and tiles.
__global__ void __launch_bounds__(kAlignThreads) align_kernel(const int32_t* ids, int rows, int k,
                                                             int first0, int count, int tile,
                                                             int capacity, int local, int32_t* pos_all,
                                                             int32_t* src, int32_t* tile_expert,
                                                             int32_t* tiles) {
  pdl_wait();
  pdl_trigger();
  const int first = first0 + (int)blockIdx.x * count;
  const bool mine = (int)blockIdx.x == local;
  int32_t* pos = pos_all + (long)blockIdx.x * rows * k;
  __shared__ int cnt[kMaxExperts], off[kMaxExperts], running[kMaxExperts], add[kMaxExperts];
  __shared__ int wcount[kAlignWarps][kMaxExperts];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = rows * k;
  for (int e = tid; e < count; e += kAlignThreads) {
    cnt[e] = 0;
    running[e] = 0;
    add[e] = 0;
    for (int w = 0; w < kAlignWarps; ++w) wcount[w][e] = 0;
  }
  if (mine)
    for (int p = tid; p < capacity; p += kAlignThreads) src[p] = -1;
  __syncthreads();
  for (int i = tid; i < n; i += kAlignThreads) {
    const int e = ids[i] - first;
    if (e >= 0 && e < count) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int o = 0;
    for (int e = 0; e < count; ++e) {
      off[e] = o;
      o += (cnt[e] + tile - 1) / tile * tile;
    }
    if (mine) *tiles = o / tile;
  }
  __syncthreads();
  for (int e = tid; e < count && mine; e += kAlignThreads) {
    const int t0 = off[e] / tile, nt = (cnt[e] + tile - 1) / tile;
    for (int t = 0; t < nt; ++t) tile_expert[t0 + t] = e;
  }
  // Stable positions: chunk by chunk, a selection's rank among the earlier selections of its
  // expert (earlier chunks, earlier warps of this chunk, earlier lanes of its warp).
  const unsigned lt = (1u << lane) - 1u;
  for (int c = 0; c < n; c += kAlignThreads) {
    const int i = c + tid;
    int e = -1;
    if (i < n) {
      e = ids[i] - first;
      if (e < 0 || e >= count) e = -1;
    }
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int before_lane = __popc(same & lt);
    if (e >= 0 && before_lane == 0) wcount[warp][e] = __popc(same);
    __syncthreads();
    if (e >= 0) {
      int before = 0;
      for (int w = 0; w < warp; ++w) before += wcount[w][e];
      const int p = off[e] + running[e] + before + before_lane;
      pos[i] = p;
      if (mine) src[p] = i / k;
    } else if (i < n) {
      pos[i] = -1;
    }
    __syncthreads();
    if (e >= 0 && before_lane == 0) {
      atomicAdd(&add[e], __popc(same));
      wcount[warp][e] = 0;
    }
    __syncthreads();
    for (int x = tid; x < count; x += kAlignThreads) {
      running[x] += add[x];
      add[x] = 0;
    }
    __syncthreads();
  }
}

__global__ void gather_kernel(const __nv_bfloat16* x, long ldx, const int32_t* src, const int32_t* tiles,
                              int tile, int cols, __nv_bfloat16* out) {
  pdl_wait();
  pdl_trigger();
  const int p = blockIdx.x;
  if (p >= *tiles * tile) return;
  const int r = src[p];
  uint4* dst = reinterpret_cast<uint4*>(out + (long)p * cols);
  const uint4* s = reinterpret_cast<const uint4*>(x + (long)r * ldx);
  for (int c = threadIdx.x; c < cols / 8; c += blockDim.x) dst[c] = r >= 0 ? s[c] : make_uint4(0, 0, 0, 0);
}

__global__ void combine_kernel(const __nv_bfloat16* y, long ldy, const int32_t* pos, const float* weights,
                               int k, int cols, __nv_bfloat16* residual, long ldr) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  for (int c = threadIdx.x * 8; c < cols; c += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int p = pos[(long)r * k + j];
      if (p < 0) continue;
      const float w = weights[(long)r * k + j];
      const uint4 q = *reinterpret_cast<const uint4*>(y + (long)p * ldy + c);
      const uint32_t v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        // A product, then a sum, each rounded (no contraction into one FMA).
        acc[2 * t] = __fadd_rn(acc[2 * t], __fmul_rn(w, __uint_as_float(v[t] << 16)));
        acc[2 * t + 1] = __fadd_rn(acc[2 * t + 1], __fmul_rn(w, __uint_as_float(v[t] & 0xFFFF0000u)));
      }
    }
    __nv_bfloat16* xr = residual + (long)r * ldr + c;
    uint4 q = *reinterpret_cast<const uint4*>(xr);
    uint32_t v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float m0 = __bfloat162float(__float2bfloat16_rn(acc[2 * t]));
      const float m1 = __bfloat162float(__float2bfloat16_rn(acc[2 * t + 1]));
      const __nv_bfloat162 o = __floats2bfloat162_rn(__uint_as_float(v[t] << 16) + m0,
                                                     __uint_as_float(v[t] & 0xFFFF0000u) + m1);
      v[t] = *reinterpret_cast<const uint32_t*>(&o);
    }
    *reinterpret_cast<uint4*>(xr) = make_uint4(v[0], v[1], v[2], v[3]);
  }
}

// One CTA of 256 threads per row: x = bf16(x + bf16(sum_j w_j * y_j)), then RMSNorm(x) * weight.
template <int kVec>
__global__ void __launch_bounds__(256) combine_norm_kernel(const __nv_bfloat16* y, long ldy, const int32_t* pos,
                                                          const float* weights, int k, int cols,
                                                          __nv_bfloat16* residual, long ldr,
                                                          const __nv_bfloat16* norm, float eps,
                                                          __nv_bfloat16* out, long ldo) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8];
  const int r = blockIdx.x;
  float xs[kVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c >= cols) continue;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int p = pos[(long)r * k + j];
      if (p < 0) continue;
      const float w = weights[(long)r * k + j];
      const uint4 q = *reinterpret_cast<const uint4*>(y + (long)p * ldy + c);
      const uint32_t v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        acc[2 * t] = __fadd_rn(acc[2 * t], __fmul_rn(w, __uint_as_float(v[t] << 16)));
        acc[2 * t + 1] = __fadd_rn(acc[2 * t + 1], __fmul_rn(w, __uint_as_float(v[t] & 0xFFFF0000u)));
      }
    }
    __nv_bfloat16* xr = residual + (long)r * ldr + c;
    const uint4 q = *reinterpret_cast<const uint4*>(xr);
    const uint32_t v[4] = {q.x, q.y, q.z, q.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float m0 = __bfloat162float(__float2bfloat16_rn(acc[2 * t]));
      const float m1 = __bfloat162float(__float2bfloat16_rn(acc[2 * t + 1]));
      const __nv_bfloat162 b = __floats2bfloat162_rn(__uint_as_float(v[t] << 16) + m0,
                                                     __uint_as_float(v[t] & 0xFFFF0000u) + m1);
      o[t] = *reinterpret_cast<const uint32_t*>(&b);
      xs[i][2 * t] = __low2float(b);
      xs[i][2 * t + 1] = __high2float(b);
      ss += xs[i][2 * t] * xs[i][2 * t] + xs[i][2 * t + 1] * xs[i][2 * t + 1];
    }
    *reinterpret_cast<uint4*>(xr) = make_uint4(o[0], o[1], o[2], o[3]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.f;
  for (int w = 0; w < 8; ++w) total += red[w];
  const float inv = rsqrtf(total / (float)cols + eps);
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c >= cols) continue;
    const uint4 wq = *reinterpret_cast<const uint4*>(norm + c);
    const uint32_t wv[4] = {wq.x, wq.y, wq.z, wq.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(xs[i][2 * t] * inv * __uint_as_float(wv[t] << 16),
                                                     xs[i][2 * t + 1] * inv * __uint_as_float(wv[t] & 0xFFFF0000u));
      o[t] = *reinterpret_cast<const uint32_t*>(&b);
    }
    *reinterpret_cast<uint4*>(out + (long)r * ldo + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace

int moe_combine_norm(const __nv_bfloat16* y, long ldy, const int32_t* pos, const float* weights, int rows,
                     int k, int cols, __nv_bfloat16* residual, long ldr, const __nv_bfloat16* norm, float eps,
                     __nv_bfloat16* out, long ldo, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (cols % 8 != 0 || ldy % 8 != 0 || ldr % 8 != 0 || ldo % 8 != 0 || cols > 8 * 256 * 4) return -2;
  const int vec = (cols / 8 + 255) / 256;
  auto kernel = vec <= 1 ? combine_norm_kernel<1> : vec <= 2 ? combine_norm_kernel<2> : combine_norm_kernel<4>;
  return launch_pdl(kernel, dim3(rows), dim3(256), 0, stream, y, ldy, pos, weights, k, cols, residual, ldr,
                    norm, eps, out, ldo) == cudaSuccess
             ? 0
             : -5;
}

int moe_route(const __nv_bfloat16* logits, long ld, int rows, int experts, int k, bool normalize,
              int32_t* ids, float* weights, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (experts <= 0 || experts > kMaxExperts || k <= 0 || k > experts || k > 32) return -2;
  const int warps = rows, per_block = 8;
  return launch_pdl(route_kernel, dim3((warps + per_block - 1) / per_block), dim3(32 * per_block), 0,
                    stream, logits, ld, rows, experts, k, normalize ? 1 : 0, ids, weights) == cudaSuccess
             ? 0
             : -5;
}

int moe_align(const int32_t* ids, int rows, int k, int experts, int first, int count, int tile,
              int capacity, int32_t* pos, int32_t* src, int32_t* tile_expert, int32_t* tiles,
              cudaStream_t stream) {
  return moe_align_ranks(ids, rows, k, experts, first, count, 1, 0, tile, capacity, pos, src,
                         tile_expert, tiles, stream);
}

int moe_align_ranks(const int32_t* ids, int rows, int k, int experts, int first, int count, int ranks,
                    int local, int tile, int capacity, int32_t* pos, int32_t* src, int32_t* tile_expert,
                    int32_t* tiles, cudaStream_t stream) {
  if (count <= 0 || count > kMaxExperts || first < 0 || first + ranks * count > experts || tile <= 0 ||
      ranks <= 0 || local < 0 || local >= ranks)
    return -2;
  const long need = ((long)rows * k + (long)count * (tile - 1) + tile - 1) / tile * tile;
  if (capacity < need) return -3;
  return launch_pdl(align_kernel, dim3(ranks), dim3(kAlignThreads), 0, stream, ids, rows, k, first, count,
                    tile, capacity, local, pos, src, tile_expert, tiles) == cudaSuccess
             ? 0
             : -5;
}

int moe_gather(const __nv_bfloat16* x, long ldx, const int32_t* src, const int32_t* tiles, int tile,
               int capacity, int cols, __nv_bfloat16* out, cudaStream_t stream) {
  if (capacity <= 0) return 0;
  if (cols % 8 != 0 || ldx % 8 != 0) return -2;
  return launch_pdl(gather_kernel, dim3(capacity), dim3(128), 0, stream, x, ldx, src, tiles, tile, cols,
                    out) == cudaSuccess
             ? 0
             : -5;
}

int moe_combine(const __nv_bfloat16* y, long ldy, const int32_t* pos, const float* weights, int rows,
                int k, int cols, __nv_bfloat16* residual, long ldr, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (cols % 8 != 0 || ldy % 8 != 0 || ldr % 8 != 0) return -2;
  return launch_pdl(combine_kernel, dim3(rows), dim3(128), 0, stream, y, ldy, pos, weights, k, cols,
                    residual, ldr) == cudaSuccess
             ? 0
             : -5;
}

}  // namespace foa
