// Memory-bound kernels of the decoder step: RMSNorm with the residual add, the embedding gather,
// the attention front (QK-norm, RoPE, paged KV write) and the greedy readout.
//
// Reference contracts: RMSNorm `ops/normalization/rms_norm.rs:15-20` (FP32 statistics, one
// rounding), residual add `ops/pointwise/add.rs:1` (FP32 sum rounded once), QK-norm
// `ops/attention/full/head.rs:41`, RoPE `ops/rotary.rs:55-57` (half-split pairs), KV store
// `ops/index/scatter.rs:30`, greedy head `ops/reduction.rs:73-77` (first maximum wins).

#include <cfloat>
#include <climits>
#include <algorithm>

#include <cooperative_groups.h>

#include "ops.cuh"
#include "launch.cuh"
#include "sm100.cuh"

namespace foa {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------------------------ RMSNorm
// One CTA of 128 threads per row; each thread keeps up to kVec 8-element vectors in registers.
template <int kVec>
__global__ void __launch_bounds__(128) rmsnorm_kernel(
    const __nv_bfloat16* __restrict__ x, long ldx, const __nv_bfloat16* __restrict__ residual,
    long ldr, const __nv_bfloat16* __restrict__ weight, __nv_bfloat16* __restrict__ out, long ldo,
    __nv_bfloat16* residual_out, long ldro, int cols, float eps) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  const int nvec = cols / 8;
  float h[kVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int v = threadIdx.x + i * 128;
    if (v < nvec) {
      const uint4 xv = *reinterpret_cast<const uint4*>(x + (long)row * ldx + v * 8);
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        h[i][2 * t] = bf16_lo(xw[t]);
        h[i][2 * t + 1] = bf16_hi(xw[t]);
      }
      if (residual != nullptr) {
        const uint4 rv = *reinterpret_cast<const uint4*>(residual + (long)row * ldr + v * 8);
        const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          h[i][2 * t] += bf16_lo(rw[t]);
          h[i][2 * t + 1] += bf16_hi(rw[t]);
        }
      }
      // The residual stream is BF16: the norm reads the rounded sum.
      uint32_t packed[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        packed[t] = pack_bf16x2(h[i][2 * t], h[i][2 * t + 1]);
        h[i][2 * t] = bf16_lo(packed[t]);
        h[i][2 * t + 1] = bf16_hi(packed[t]);
        ss += h[i][2 * t] * h[i][2 * t] + h[i][2 * t + 1] * h[i][2 * t + 1];
      }
      if (residual_out != nullptr)
        *reinterpret_cast<uint4*>(residual_out + (long)row * ldro + v * 8) =
            make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
  }
  __shared__ float red[4];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float total = red[0] + red[1] + red[2] + red[3];
  const float inv = rsqrtf(total / (float)cols + eps);
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int v = threadIdx.x + i * 128;
    if (v < nvec) {
      const uint4 wv = *reinterpret_cast<const uint4*>(weight + v * 8);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int t = 0; t < 4; ++t)
        o[t] = pack_bf16x2(h[i][2 * t] * inv * bf16_lo(ww[t]), h[i][2 * t + 1] * inv * bf16_hi(ww[t]));
      *reinterpret_cast<uint4*>(out + (long)row * ldo + v * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// ------------------------------------------------------------------------------------ embedding
__global__ void embedding_kernel(const int32_t* __restrict__ ids,
                                 const __nv_bfloat16* __restrict__ table, long ldt,
                                 int row_begin, int row_end, __nv_bfloat16* __restrict__ out,
                                 long ldo, int cols) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  const int id = ids[row];
  const bool local = id >= row_begin && id < row_end;
  const int nvec = cols / 8;
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    uint4 val = make_uint4(0, 0, 0, 0);
    if (local) val = *reinterpret_cast<const uint4*>(table + (long)(id - row_begin) * ldt + v * 8);
    *reinterpret_cast<uint4*>(out + (long)row * ldo + v * 8) = val;
  }
}

// ------------------------------------------------------------------------------------ argmax
__device__ __forceinline__ void better(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

// One row's argmax split over a cluster of kArgmaxCtas CTAs: CTA c scans its slice of the row
// (slices start on 4-float boundaries), the CTAs' (value, index) pairs meet in CTA 0's shared
// memory through the cluster, and CTA 0 keeps the first maximum. A one-CTA scan of a 152K-entry
// vocabulary row is bound by one SM's load rate; the split reads the row on eight SMs.
constexpr int kArgmaxCtas = 8;

__global__ void __launch_bounds__(512) argmax_kernel(const float* __restrict__ logits, long ld,
                                                     int cols, int valid, int base,
                                                     int32_t* out_index, float* out_value) {
  pdl_wait();
  pdl_trigger();
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int part = static_cast<int>(cluster.block_rank());
  const int row = blockIdx.y;
  const float* src = logits + (long)row * ld;
  float bv = -INFINITY;
  int bi = INT_MAX;
  const int n = min(cols, valid);
  const int per = ((n + kArgmaxCtas - 1) / kArgmaxCtas + 3) & ~3;
  const int lo = min(n, part * per), hi = min(n, lo + per);
  const bool vec = ld % 4 == 0;
  const int hi4 = vec ? lo + ((hi - lo) & ~3) : lo;
  for (int i = lo + 4 * threadIdx.x; i < hi4; i += 4 * blockDim.x) {
    const float4 x = __ldg(reinterpret_cast<const float4*>(src + i));
    better(bv, bi, x.x, i);
    better(bv, bi, x.y, i + 1);
    better(bv, bi, x.z, i + 2);
    better(bv, bi, x.w, i + 3);
  }
  for (int i = hi4 + threadIdx.x; i < hi; i += blockDim.x) better(bv, bi, src[i], i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  __shared__ float sv[16];
  __shared__ int si[16];
  __shared__ float cta_v;
  __shared__ int cta_i;
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) better(bv, bi, sv[w], si[w]);
    cta_v = bv;
    cta_i = bi;
  }
  cluster.sync();  // every CTA's pair is in its shared memory
  if (part == 0 && threadIdx.x == 0) {
    for (int c = 1; c < kArgmaxCtas; ++c)
      better(bv, bi, *cluster.map_shared_rank(&cta_v, c), *cluster.map_shared_rank(&cta_i, c));
    if (bi == INT_MAX) bi = 0;
    out_index[row] = bi + base;
    if (out_value != nullptr) out_value[row] = bv;
  }
  cluster.sync();  // no CTA leaves while CTA 0 still reads its shared memory
}

__global__ void argmax_merge_kernel(const float* values, const int32_t* indices, int ranks,
                                    int rows, int32_t* out) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  float bv = -INFINITY;
  int bi = INT_MAX;
  for (int r = 0; r < ranks; ++r) better(bv, bi, values[(long)r * rows + row], indices[(long)r * rows + row]);
  out[row] = bi == INT_MAX ? 0 : bi;
}

// ------------------------------------------------------------------------------------ attention front
// One warp per (row, head) of the packed projection. A lane holds elements
// [lane*E, lane*E+E) of the first half of the head and the same offsets of the second half, so
// each rotated pair (j, j + d/2) stays in one lane.
template <int kHD>
__global__ void __launch_bounds__(128) qk_norm_rope_cache_kernel(
    const __nv_bfloat16* __restrict__ qkv, long ld_qkv, int rows, int q_heads, int kv_heads,
    const __nv_bfloat16* __restrict__ q_norm, const __nv_bfloat16* __restrict__ k_norm, float eps,
    const int32_t* __restrict__ positions, const float* __restrict__ inv_freq, float attn_factor,
    __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ cache,
    const int32_t* __restrict__ slots, long cache_slots, int* status) {
  pdl_wait();
  pdl_trigger();
  constexpr int E = kHD / 64;  // elements per lane in each half
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = q_heads + 2 * kv_heads;
  const int task = blockIdx.x * 4 + warp;
  if (task >= rows * heads) return;
  const int row = task / heads, head = task % heads;
  const __nv_bfloat16* src = qkv + (long)row * ld_qkv + (long)head * kHD;
  float a[E], b[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    a[e] = __bfloat162float(src[lane * E + e]);
    b[e] = __bfloat162float(src[kHD / 2 + lane * E + e]);
  }
  const bool is_q = head < q_heads;
  const bool is_k = !is_q && head < q_heads + kv_heads;
  if (is_q || is_k) {
    const __nv_bfloat16* nw = is_q ? q_norm : k_norm;
    if (nw != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) ss += a[e] * a[e] + b[e] * b[e];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / (float)kHD + eps);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        a[e] = __bfloat162float(__float2bfloat16_rn(a[e] * inv * __bfloat162float(nw[lane * E + e])));
        b[e] = __bfloat162float(
            __float2bfloat16_rn(b[e] * inv * __bfloat162float(nw[kHD / 2 + lane * E + e])));
      }
    }
    const float pos = (float)positions[row];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float s, c;
      sincosf(pos * inv_freq[lane * E + e], &s, &c);
      c *= attn_factor;
      s *= attn_factor;
      const float x1 = a[e], x2 = b[e];
      a[e] = x1 * c - x2 * s;
      b[e] = x2 * c + x1 * s;
    }
  }
  if (is_q) {
    __nv_bfloat16* dst = q_out + ((long)row * q_heads + head) * kHD;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      dst[lane * E + e] = __float2bfloat16_rn(a[e]);
      dst[kHD / 2 + lane * E + e] = __float2bfloat16_rn(b[e]);
    }
    return;
  }
  const int slot = slots[row];
  if (slot < 0) return;
  if (cache_slots > 0 && slot >= cache_slots) {  // a slot past the cache: nothing is written
    if (lane == 0) record_status(status, kBadIndex);
    return;
  }
  const int kvh = is_k ? head - q_heads : head - q_heads - kv_heads;
  const long page = 2L * kv_heads * 16 * kHD;
  __nv_bfloat16* dst = cache + (long)(slot / 16) * page + (is_k ? 0 : (long)kv_heads * 16 * kHD) +
                       ((long)kvh * 16 + slot % 16) * kHD;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    dst[lane * E + e] = __float2bfloat16_rn(a[e]);
    dst[kHD / 2 + lane * E + e] = __float2bfloat16_rn(b[e]);
  }
}

// Row-per-CTA form of the same operation for 16-byte aligned operands (a CTA: one row, a group of
// its heads): the row's rotation (cos, sin) pairs are computed once into shared memory and shared
// by the group's heads; a head is kHD / 8 lanes of 8 consecutive elements (16-byte loads and
// stores), so a warp handles 256 / kHD heads at once; the partner of element j (j + d/2) sits
// kHD / 16 lanes away.
template <int kHD, int kPasses, bool kSplits>
__global__ void __launch_bounds__(128) qk_norm_rope_cache_rows_kernel(
    const __nv_bfloat16* __restrict__ qkv, long ld_qkv, int rows, int q_heads, int kv_heads,
    const __nv_bfloat16* __restrict__ q_norm, const __nv_bfloat16* __restrict__ k_norm, float eps,
    const int32_t* __restrict__ positions, const float* __restrict__ inv_freq, float attn_factor,
    __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ cache,
    const int32_t* __restrict__ slots, long cache_slots, int* status, const GemmSplits sp) {
  constexpr int kLanes = kHD / 8;        // lanes of one head
  constexpr int kPerWarp = 32 / kLanes;  // heads of one warp pass
  constexpr int kHalf = kLanes / 2;      // lane distance of the rotation partner
  __shared__ float cs[kHD / 2], sn[kHD / 2];
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  if (row >= rows) return;
  const float pos = (float)positions[row];
  for (int j = threadIdx.x; j < kHD / 2; j += blockDim.x) {
    float sv, cv;
    sincosf(pos * inv_freq[j], &sv, &cv);
    cs[j] = cv * attn_factor;
    sn[j] = sv * attn_factor;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / kLanes, hl = lane % kLanes;
  const bool second = hl >= kHalf;
  const int j0 = (hl % kHalf) * 8;  // frequency index of this lane's first element
  const int heads = q_heads + 2 * kv_heads;
  const int slot = slots[row];
  const bool bad_slot = slot >= 0 && cache_slots > 0 && slot >= cache_slots;
  if (bad_slot && threadIdx.x == 0 && blockIdx.y == 0) record_status(status, kBadIndex);  // nothing of the row is cached
  // blockIdx.y picks the row's group of kGroup heads; a warp takes kPasses passes of kPerWarp
  // heads, with every pass's load issued before the first is processed.
  constexpr int kGroup = 4 * kPerWarp * kPasses;
  uint4 raws[kPasses];
#pragma unroll
  for (int ps = 0; ps < kPasses; ++ps) {
    const int head = blockIdx.y * kGroup + (ps * 4 + warp) * kPerWarp + sub;
    if (head >= heads) {
      raws[ps] = make_uint4(0, 0, 0, 0);
    } else if constexpr (kSplits) {
      // The projection's K splits, added in split order and rounded once.
      float4 p0[GemmSplits::kMax], p1[GemmSplits::kMax];
#pragma unroll
      for (int s2 = 0; s2 < GemmSplits::kMax; ++s2)
        if (s2 < sp.splits) {
          const float4* src = reinterpret_cast<const float4*>(sp.ws + sp.at(s2, row, (long)head * kHD + hl * 8));
          p0[s2] = __ldcg(src);
          p1[s2] = __ldcg(src + 1);
        }
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s2 = 0; s2 < GemmSplits::kMax; ++s2)
        if (s2 < sp.splits) {
          acc[0] += p0[s2].x; acc[1] += p0[s2].y; acc[2] += p0[s2].z; acc[3] += p0[s2].w;
          acc[4] += p1[s2].x; acc[5] += p1[s2].y; acc[6] += p1[s2].z; acc[7] += p1[s2].w;
        }
      raws[ps] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                            pack_bf16x2(acc[6], acc[7]));
    } else {
      raws[ps] = __ldcs(reinterpret_cast<const uint4*>(qkv + (long)row * ld_qkv + (long)head * kHD) + hl);
    }
  }
#pragma unroll
  for (int ps = 0; ps < kPasses; ++ps) {
    const int head = blockIdx.y * kGroup + (ps * 4 + warp) * kPerWarp + sub;
    const bool valid = head < heads;
    const uint4 raw = raws[ps];
    const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
    float x[8];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      x[2 * t] = __uint_as_float(rw[t] << 16);
      x[2 * t + 1] = __uint_as_float(rw[t] & 0xFFFF0000u);
    }
    const bool is_q = head < q_heads;
    const bool is_k = !is_q && head < q_heads + kv_heads;
    const bool roped = valid && (is_q || is_k);
    const __nv_bfloat16* nw = is_q ? q_norm : k_norm;
    // Every lane takes part in the shuffles; only a roped head's lanes use them.
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += x[e] * x[e];
#pragma unroll
    for (int o = kHalf; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (roped && nw != nullptr) {
      const float inv = rsqrtf(ss / (float)kHD + eps);
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(nw) + hl);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        x[2 * t] = __bfloat162float(__float2bfloat16_rn(x[2 * t] * inv * __uint_as_float(ww[t] << 16)));
        x[2 * t + 1] =
            __bfloat162float(__float2bfloat16_rn(x[2 * t + 1] * inv * __uint_as_float(ww[t] & 0xFFFF0000u)));
      }
    }
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float partner = __shfl_xor_sync(0xffffffffu, x[e], kHalf);
      const float c = cs[j0 + e], sv = sn[j0 + e];
      // First half: x1 c - x2 s; second half: x2 c + x1 s.
      y[e] = roped ? (second ? x[e] * c + partner * sv : x[e] * c - partner * sv) : x[e];
    }
    if (!valid) continue;
    const uint4 out = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                                 pack_bf16x2(y[6], y[7]));
    if (is_q) {
      reinterpret_cast<uint4*>(q_out + ((long)row * q_heads + head) * kHD)[hl] = out;
      continue;
    }
    if (slot < 0 || bad_slot) continue;
    const int kvh = is_k ? head - q_heads : head - q_heads - kv_heads;
    const long page = 2L * kv_heads * 16 * kHD;
    __nv_bfloat16* dst = cache + (long)(slot / 16) * page + (is_k ? 0 : (long)kv_heads * 16 * kHD) +
                         ((long)kvh * 16 + slot % 16) * kHD;
    reinterpret_cast<uint4*>(dst)[hl] = out;
  }
}

// ------------------------------------------------------------------------------------ init / gather
// SplitMix64-style mixing of (seed, index) into 64 random bits.
__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__global__ void init_normal_kernel(__nv_bfloat16* dst, long n, float std, uint64_t seed) {
  pdl_wait();  // weight producers: no early trigger, since GEMMs load weights before waiting
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const uint64_t r = mix64(seed * 0x100000001B3ull + (uint64_t)i);
    // Box-Muller on two 24-bit uniforms in (0, 1].
    const float u1 = ((float)(r & 0xFFFFFF) + 1.0f) * (1.0f / 16777216.0f);
    const float u2 = (float)((r >> 24) & 0xFFFFFF) * (1.0f / 16777216.0f);
    const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    dst[i] = __float2bfloat16_rn(z * std);
  }
}

__global__ void init_normal_rows_kernel(__nv_bfloat16* dst, int rows, int cols,
                                        const int32_t* full_row, const uint32_t* tag,
                                        long full_cols, long col_offset, float std, uint64_t seed) {
  pdl_wait();  // weight producers: no early trigger, since GEMMs load weights before waiting
  const long n = (long)rows * cols;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    const uint64_t logical = (uint64_t)full_row[r] * (uint64_t)full_cols + (uint64_t)(col_offset + c);
    const uint64_t x = mix64((seed * 0x100000001B3ull) ^ ((uint64_t)tag[r] << 40) ^ logical);
    const float u1 = ((float)(x & 0xFFFFFF) + 1.0f) * (1.0f / 16777216.0f);
    const float u2 = (float)((x >> 24) & 0xFFFFFF) * (1.0f / 16777216.0f);
    dst[i] = __float2bfloat16_rn(sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2) * std);
  }
}

__global__ void fill_bf16_kernel(__nv_bfloat16* dst, long n, float v) {
  pdl_wait();  // weight producers: no early trigger, since GEMMs load weights before waiting
  const __nv_bfloat16 b = __float2bfloat16_rn(v);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    dst[i] = b;
}

// Zeroes the `cols` columns of z rows whose slot is not `slot` (LoRA: a row runs one adapter).
__global__ void lora_mask_kernel(__nv_bfloat16* z, long ldz, int rows, int cols, int slot, const int32_t* row_slot) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  if (r >= rows || row_slot[r] == slot) return;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) z[(long)r * ldz + c] = __float2bfloat16_rn(0.f);
}

__global__ void gather_tokens_kernel(const int32_t* sources, int count, int32_t* out) {
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x;
  if (s >= count) return;
  const int32_t* rec = sources + 4 * s;
  const uint64_t addr = (uint64_t)(uint32_t)rec[0] | ((uint64_t)(uint32_t)rec[1] << 32);
  const int32_t* src = reinterpret_cast<const int32_t*>(addr);
  const int len = rec[2], first = rec[3];
  for (int i = threadIdx.x; i < len; i += blockDim.x) out[first + i] = src[i];
}

__global__ void gather_rows_kernel(const __nv_bfloat16* in, long ldi, const int32_t* rows,
                                   __nv_bfloat16* out, long ldo, int cols) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x;
  const int r = rows[i];
  for (int v = threadIdx.x; v < cols / 8; v += blockDim.x)
    reinterpret_cast<uint4*>(out + (long)i * ldo)[v] =
        reinterpret_cast<const uint4*>(in + (long)r * ldi)[v];
}

}  // namespace

int lora_mask(__nv_bfloat16* z, long ldz, int rows, int cols, int slot, const int32_t* row_slot,
              cudaStream_t stream) {
  if (rows <= 0) return 0;
  return launch_pdl(lora_mask_kernel, dim3(rows), dim3(128), 0, stream, z, ldz, rows, cols, slot, row_slot) ==
                 cudaSuccess
             ? 0
             : -5;
}

int init_normal_bf16(__nv_bfloat16* dst, long n, float std, uint64_t seed, cudaStream_t stream) {
  if (n <= 0) return 0;
  const int grid = (int)std::min<long>((n + 255) / 256, 148L * 16);
  launch_pdl(init_normal_kernel, dim3(grid), dim3(256), 0, stream, dst, n, std, seed);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int init_normal_rows(__nv_bfloat16* dst, int rows, int cols, const int32_t* full_row,
                     const uint32_t* tag, long full_cols, long col_offset, float std, uint64_t seed,
                     cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return 0;
  const long n = (long)rows * cols;
  const int grid = (int)std::min<long>((n + 255) / 256, 148L * 16);
  launch_pdl(init_normal_rows_kernel, dim3(grid), dim3(256), 0, stream, dst, rows, cols, full_row,
             tag, full_cols, col_offset, std, seed);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int fill_bf16(__nv_bfloat16* dst, long n, float value, cudaStream_t stream) {
  if (n <= 0) return 0;
  const int grid = (int)std::min<long>((n + 255) / 256, 148L * 16);
  launch_pdl(fill_bf16_kernel, dim3(grid), dim3(256), 0, stream, dst, n, value);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int gather_tokens(const int32_t* sources, int count, int32_t* out, cudaStream_t stream) {
  if (count <= 0) return 0;
  launch_pdl(gather_tokens_kernel, dim3(count), dim3(128), 0, stream, sources, count, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int gather_rows(const __nv_bfloat16* in, long ldi, const int32_t* rows, int n, __nv_bfloat16* out,
                long ldo, int cols, cudaStream_t stream) {
  if (n <= 0) return 0;
  if (cols % 8 != 0) return -2;
  launch_pdl(gather_rows_kernel, dim3(n), dim3(128), 0, stream, in, ldi, rows, out, ldo, cols);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

// One CTA of 128 threads per row, as rmsnorm_kernel; each 8-column vector first adds the K
// splits' FP32 partials (two 16-byte loads a split) and the residual.
template <int kVec>
__global__ void __launch_bounds__(128) rmsnorm_splits_kernel(const GemmSplits sp, __nv_bfloat16* x, long ldx,
                                                             const __nv_bfloat16* __restrict__ weight,
                                                             __nv_bfloat16* __restrict__ out, long ldo, int cols,
                                                             float eps) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  const int nvec = cols / 8;
  float h[kVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int v = threadIdx.x + i * 128;
    if (v < nvec) {
      // Every split's two 16-byte loads go out before the sum (in split order) starts.
      float4 p0[GemmSplits::kMax], p1[GemmSplits::kMax];
#pragma unroll
      for (int s = 0; s < GemmSplits::kMax; ++s)
        if (s < sp.splits) {
          const float4* src = reinterpret_cast<const float4*>(sp.ws + sp.at(s, row, (long)v * 8));
          p0[s] = __ldcg(src);
          p1[s] = __ldcg(src + 1);
        }
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < GemmSplits::kMax; ++s)
        if (s < sp.splits) {
          acc[0] += p0[s].x; acc[1] += p0[s].y; acc[2] += p0[s].z; acc[3] += p0[s].w;
          acc[4] += p1[s].x; acc[5] += p1[s].y; acc[6] += p1[s].z; acc[7] += p1[s].w;
        }
      const uint4 rv = *reinterpret_cast<const uint4*>(x + (long)row * ldx + v * 8);
      const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
      uint32_t packed[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        packed[t] = pack_bf16x2(acc[2 * t] + bf16_lo(rw[t]), acc[2 * t + 1] + bf16_hi(rw[t]));
        h[i][2 * t] = bf16_lo(packed[t]);
        h[i][2 * t + 1] = bf16_hi(packed[t]);
        ss += h[i][2 * t] * h[i][2 * t] + h[i][2 * t + 1] * h[i][2 * t + 1];
      }
      *reinterpret_cast<uint4*>(x + (long)row * ldx + v * 8) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
  }
  __shared__ float red[4];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float total = red[0] + red[1] + red[2] + red[3];
  const float inv = rsqrtf(total / (float)cols + eps);
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int v = threadIdx.x + i * 128;
    if (v < nvec) {
      const uint4 wv = *reinterpret_cast<const uint4*>(weight + v * 8);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int t = 0; t < 4; ++t)
        o[t] = pack_bf16x2(h[i][2 * t] * inv * bf16_lo(ww[t]), h[i][2 * t + 1] * inv * bf16_hi(ww[t]));
      *reinterpret_cast<uint4*>(out + (long)row * ldo + v * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

int rmsnorm_splits(const GemmSplits& sp, __nv_bfloat16* x, long ldx, const __nv_bfloat16* weight,
                   __nv_bfloat16* out, long ldo, int rows, int cols, float eps, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (cols % 8 != 0 || cols > 16384 || sp.ws == nullptr || sp.splits < 1 || sp.splits > GemmSplits::kMax ||
      sp.kbn <= 0)
    return -2;
  const int vec = (cols / 8 + 127) / 128;
  cudaError_t e;
  switch (vec) {
    case 1: e = launch_pdl(rmsnorm_splits_kernel<1>, dim3(rows), dim3(128), 0, stream, sp, x, ldx, weight, out, ldo, cols, eps); break;
    case 2: e = launch_pdl(rmsnorm_splits_kernel<2>, dim3(rows), dim3(128), 0, stream, sp, x, ldx, weight, out, ldo, cols, eps); break;
    case 3: case 4: e = launch_pdl(rmsnorm_splits_kernel<4>, dim3(rows), dim3(128), 0, stream, sp, x, ldx, weight, out, ldo, cols, eps); break;
    case 5: case 6: case 7: case 8: e = launch_pdl(rmsnorm_splits_kernel<8>, dim3(rows), dim3(128), 0, stream, sp, x, ldx, weight, out, ldo, cols, eps); break;
    default: e = launch_pdl(rmsnorm_splits_kernel<16>, dim3(rows), dim3(128), 0, stream, sp, x, ldx, weight, out, ldo, cols, eps); break;
  }
  return e == cudaSuccess ? 0 : -5;
}

int rmsnorm(const __nv_bfloat16* x, long ldx, const __nv_bfloat16* residual, long ldr,
            const __nv_bfloat16* weight, __nv_bfloat16* out, long ldo,
            __nv_bfloat16* residual_out, long ldro, int rows, int cols, float eps,
            cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (cols % 8 != 0 || cols > 16384) return -2;
  const int vec = (cols / 8 + 127) / 128;
#define FOA_RMS(V)                                                                          \
  case V:                                                                                   \
    launch_pdl(rmsnorm_kernel<V>, dim3(rows), dim3(128), 0, stream, x, ldx, residual, ldr, weight, out, ldo,    \
                                                residual_out, ldro, cols, eps);             \
    break;
  switch (vec) {
    FOA_RMS(1)
    FOA_RMS(2)
    FOA_RMS(3)
    FOA_RMS(4)
    FOA_RMS(5)
    FOA_RMS(6)
    FOA_RMS(7)
    FOA_RMS(8)
    FOA_RMS(9)
    FOA_RMS(10)
    FOA_RMS(11)
    FOA_RMS(12)
    FOA_RMS(13)
    FOA_RMS(14)
    FOA_RMS(15)
    FOA_RMS(16)
    default:
      return -2;
  }
#undef FOA_RMS
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int embedding(const int32_t* ids, const __nv_bfloat16* table, long ldt, int row_begin,
              int row_end, __nv_bfloat16* out, long ldo, int rows, int cols,
              cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (cols % 8 != 0) return -2;
  launch_pdl(embedding_kernel, dim3(rows), dim3(128), 0, stream, ids, table, ldt, row_begin, row_end, out, ldo, cols);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int argmax_rows(const float* logits, long ld, int rows, int cols, int valid_cols, int index_base,
                int32_t* out_index, float* out_value, cudaStream_t stream) {
  if (rows <= 0) return 0;
  if (rows > 65535) return -2;
  launch_pdl_cluster(argmax_kernel, dim3(kArgmaxCtas, rows), dim3(512), kArgmaxCtas, 0, stream, logits, ld, cols,
                     valid_cols, index_base, out_index, out_value);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int argmax_merge(const float* values, const int32_t* indices, int ranks, int rows,
                 int32_t* out_tokens, cudaStream_t stream) {
  if (rows <= 0) return 0;
  launch_pdl(argmax_merge_kernel, dim3((rows + 127) / 128), dim3(128), 0, stream, values, indices, ranks, rows,
                                                              out_tokens);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int qk_norm_rope_cache(const __nv_bfloat16* qkv, long ld_qkv, int rows, int q_heads, int kv_heads,
                       int head_dim, const __nv_bfloat16* q_norm, const __nv_bfloat16* k_norm,
                       float eps, const int32_t* positions, RopeTable rope,
                       __nv_bfloat16* q_out, __nv_bfloat16* cache, const int32_t* slots,
                       cudaStream_t stream, long cache_slots, int* status, const GemmSplits* splits) {
  if (rows <= 0) return 0;
  GemmSplits sp;
  if (splits != nullptr && splits->splits > 1) {
    sp = *splits;
    if (sp.ws == nullptr || (reinterpret_cast<uintptr_t>(sp.ws) & 15) || head_dim % 8 != 0 ||
        sp.splits > GemmSplits::kMax)
      return -2;
  } else {
    sp.splits = 0;
  }
  const bool aligned = ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(q_out) |
                         reinterpret_cast<uintptr_t>(cache) | reinterpret_cast<uintptr_t>(q_norm) |
                         reinterpret_cast<uintptr_t>(k_norm)) & 15) == 0 && ld_qkv % 8 == 0;
  if (aligned && (head_dim == 64 || head_dim == 128 || head_dim == 256)) {
    // Row-per-CTA kernel: shared rotation table, 16-byte accesses.
    // Many rows: four passes a warp (more loads in flight); few rows (decode): one pass, more CTAs.
    // Only the one-pass form reads GEMM splits (the split partials exist for decode rows only).
    const bool many = rows >= 148 && sp.splits <= 1;
    const bool split = sp.splits > 1;
    const auto kernel =
        head_dim == 64    ? (many ? qk_norm_rope_cache_rows_kernel<64, 4, false>
                                  : split ? qk_norm_rope_cache_rows_kernel<64, 1, true> : qk_norm_rope_cache_rows_kernel<64, 1, false>)
        : head_dim == 128 ? (many ? qk_norm_rope_cache_rows_kernel<128, 4, false>
                                  : split ? qk_norm_rope_cache_rows_kernel<128, 1, true> : qk_norm_rope_cache_rows_kernel<128, 1, false>)
                          : (many ? qk_norm_rope_cache_rows_kernel<256, 4, false>
                                  : split ? qk_norm_rope_cache_rows_kernel<256, 1, true> : qk_norm_rope_cache_rows_kernel<256, 1, false>);
    const int group = (many ? 16 : 4) * (256 / head_dim);  // heads of one CTA: 4 warps x passes
    const int groups = (q_heads + 2 * kv_heads + group - 1) / group;
    return launch_pdl(kernel, dim3(rows, groups), dim3(128), 0, stream, qkv, ld_qkv, rows, q_heads, kv_heads, q_norm,
                      k_norm, eps, positions, rope.inv_freq, rope.attention_factor, q_out, cache, slots,
                      cache_slots, status, sp) == cudaSuccess ? 0 : -5;
  }
  if (sp.splits > 1) return -2;  // split partials are read by the row kernel only
  const long tasks = (long)rows * (q_heads + 2 * kv_heads);
  const int grid = (int)((tasks + 3) / 4);
  switch (head_dim) {
    case 64:
      launch_pdl(qk_norm_rope_cache_kernel<64>, dim3(grid), dim3(128), 0, stream, 
          qkv, ld_qkv, rows, q_heads, kv_heads, q_norm, k_norm, eps, positions, rope.inv_freq,
          rope.attention_factor, q_out, cache, slots, cache_slots, status);
      break;
    case 128:
      launch_pdl(qk_norm_rope_cache_kernel<128>, dim3(grid), dim3(128), 0, stream, 
          qkv, ld_qkv, rows, q_heads, kv_heads, q_norm, k_norm, eps, positions, rope.inv_freq,
          rope.attention_factor, q_out, cache, slots, cache_slots, status);
      break;
    case 256:
      launch_pdl(qk_norm_rope_cache_kernel<256>, dim3(grid), dim3(128), 0, stream, 
          qkv, ld_qkv, rows, q_heads, kv_heads, q_norm, k_norm, eps, positions, rope.inv_freq,
          rope.attention_factor, q_out, cache, slots, cache_slots, status);
      break;
    default:
      return -2;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

}  // namespace foa
