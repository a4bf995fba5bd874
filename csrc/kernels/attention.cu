// Paged GQA attention over the block-table KV cache: flash-decoding for one-row requests and a
// causal chunked-prefill kernel for prompt chunks.
//
// Reference behaviour: decode work items with split histories merged by log-sum-exp
// (`ops/attention/full/paged/gqa/items/{mod,plan,attend}.rs`, `wide/merge.rs:1-7`); prompt chunks
// attending the committed history plus their own rows causally (`ops/attention/full/paged/append/*`).
//
// Design for Blackwell:
// - Query heads of one key/value head are packed into the MMA's M rows (16 per warp), so every
//   key/value byte read from HBM serves the whole GQA group.
// - Key/value pages (16 tokens x head_dim, contiguous per head) stream into swizzled shared
//   memory with cp.async and feed the tensor cores through ldmatrix; softmax runs online in FP32
//   with exp2.
// - Decode splits each history into chunks whose size depends on the model's geometry only (2048
//   keys, or 256 when a row has at most two KV heads, so that such small grids still fill 148
//   SMs): a row's tiling never depends on the rest of the batch (batch invariant). Two warps
//   (four with four KV heads) share a chunk, each streaming its pages in a two-stage cp.async
//   ring, and merge through shared memory; a second pass merges the chunks by log-sum-exp in
//   chunk order. Two-warp CTAs let four CTAs share an SM's load queue: on B200 (64 rows of 2048
//   keys, 8 KV heads of 128) this read 97 % of the measured HBM copy bandwidth under ncu, against
//   63 % of DRAM peak for four-warp CTAs. A TMA-fed variant (one producer warp, mbarrier ring)
//   measured slower and is not kept.
// - Decode is bound by HBM bandwidth (every key/value byte is read once per step). Prefill runs on
//   the tcgen05 kernel of attention_tc.cu where it applies; the mma.sync prefill kernel here is the
//   fallback for the geometries that kernel does not take.

#include <cfloat>
#include <cstdlib>

#include "attention.cuh"
#include "launch.cuh"
#include "sm100.cuh"

namespace foa {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// 16-byte async copy; `bytes` 0 fills the destination with zeros.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Byte offset of 16-byte chunk `c` of row `r` in a [rows][D] BF16 tile with XOR swizzling, so
// eight rows' chunks of one ldmatrix land in eight different bank groups.
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * (D * 2) + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ float warp_max4(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}
__device__ __forceinline__ float warp_sum4(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

// Online-softmax state of a warp's 16 query rows: this thread's rows g and g + 8.
template <int D>
struct Flash {
  float o[D / 8][4];
  float m[2], l[2];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int j = 0; j < D / 8; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) o[j][i] = 0.f;
    m[0] = m[1] = -INFINITY;
    l[0] = l[1] = 0.f;
  }
  // Folds a block of NT*8 keys whose scores (already scaled to log2 units, masked with -inf)
  // are s[NT][4]; the values are rows of the swizzled [keys][D] tile at `vtile`, starting at
  // key row `vrow0`.
  template <int NT>
  __device__ __forceinline__ void fold(float (&s)[NT][4], uint32_t vtile, int vrow0, int lane) {
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
      mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
    }
    mx0 = warp_max4(mx0);
    mx1 = warp_max4(mx1);
    const float n0 = fmaxf(m[0], mx0), n1 = fmaxf(m[1], mx1);
    // A row with no finite score yet keeps a zero state (n == -inf).
    const float c0 = n0 == -INFINITY ? 1.f : exp2f(m[0] - n0);
    const float c1 = n1 == -INFINITY ? 1.f : exp2f(m[1] - n1);
    const float b0 = n0 == -INFINITY ? 0.f : n0, b1 = n1 == -INFINITY ? 0.f : n1;
    m[0] = n0;
    m[1] = n1;
    float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      s[n][0] = exp2f(s[n][0] - b0);
      s[n][1] = exp2f(s[n][1] - b0);
      s[n][2] = exp2f(s[n][2] - b1);
      s[n][3] = exp2f(s[n][3] - b1);
      sum0 += s[n][0] + s[n][1];
      sum1 += s[n][2] + s[n][3];
    }
    l[0] = l[0] * c0 + sum0;
    l[1] = l[1] * c1 + sum1;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      o[j][0] *= c0;
      o[j][1] *= c0;
      o[j][2] *= c1;
      o[j][3] *= c1;
    }
    // O += P V, 16 keys per k-step.
#pragma unroll
    for (int ks = 0; ks < NT / 2; ++ks) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * ks][0], s[2 * ks][1]);
      pa[1] = pack_bf16x2(s[2 * ks][2], s[2 * ks][3]);
      pa[2] = pack_bf16x2(s[2 * ks + 1][0], s[2 * ks + 1][1]);
      pa[3] = pack_bf16x2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
      // ldmatrix.trans: lanes 0-7 keys 0-7 chunk j, 8-15 keys 8-15 chunk j, 16-23 keys 0-7
      // chunk j+1, 24-31 keys 8-15 chunk j+1.
      const int krow = vrow0 + ks * 16 + (lane & 15);
      const int cadd = lane >> 4;
#pragma unroll
      for (int j = 0; j < D / 8; j += 2) {
        uint32_t r[4];
        ldsm_x4_t(r, vtile + swz<D>(krow, j + cadd));
        mma16816(o[j], pa, r[0], r[1]);
        mma16816(o[j + 1], pa, r[2], r[3]);
      }
    }
  }
};

// S[NT][4] = Q K^T for NT*8 keys of the swizzled [keys][D] tile at `ktile` from key row `krow0`.
template <int D, int NT>
__device__ __forceinline__ void qk(float (&s)[NT][4], const uint32_t (&qa)[D / 16][4],
                                   uint32_t ktile, int krow0, int lane) {
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) s[n][i] = 0.f;
  // ldmatrix (no trans): lanes 0-7 keys 0-7 chunk 2kk, 8-15 keys 0-7 chunk 2kk+1,
  // 16-23 keys 8-15 chunk 2kk, 24-31 keys 8-15 chunk 2kk+1.
  const int rsel = (lane & 7) + ((lane >> 4) << 3);
  const int csel = (lane >> 3) & 1;
#pragma unroll
  for (int n = 0; n < NT; n += 2) {
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t r[4];
      ldsm_x4(r, ktile + swz<D>(krow0 + n * 8 + rsel, 2 * kk + csel));
      mma16816(s[n], qa[kk], r[0], r[1]);
      mma16816(s[n + 1], qa[kk], r[2], r[3]);
    }
  }
}

// Loads the A fragments of 16 query rows; `row_ptr(m)` gives row m's address or null (zeros).
template <int D, class RowPtr>
__device__ __forceinline__ void load_q(uint32_t (&qa)[D / 16][4], RowPtr row_ptr, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const __nv_bfloat16* r0 = row_ptr(g);
  const __nv_bfloat16* r1 = row_ptr(g + 8);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int c = kk * 16 + 2 * t;
    qa[kk][0] = r0 ? *reinterpret_cast<const uint32_t*>(r0 + c) : 0u;
    qa[kk][1] = r1 ? *reinterpret_cast<const uint32_t*>(r1 + c) : 0u;
    qa[kk][2] = r0 ? *reinterpret_cast<const uint32_t*>(r0 + c + 8) : 0u;
    qa[kk][3] = r1 ? *reinterpret_cast<const uint32_t*>(r1 + c + 8) : 0u;
  }
}

// ------------------------------------------------------------------------------------ decode
// One CTA per (segment, key/value head, 2048-key split); kWarps warps take the split's 16-key
// blocks in turn, each keeping kStages blocks in a cp.async ring. Small CTAs (2 warps, 32 KiB)
// let 6 of them share an SM, so a decode batch's CTAs fit the GPU in one wave.
// CTAs of a decode configuration an SM holds: by shared memory, and at most 12 warps (the
// registers of 168 a thread).
constexpr int decode_ctas_per_sm(int d, int warps, int stages) {
  const int by_smem = (220 * 1024) / (warps * stages * 2 * 16 * d * 2);
  const int by_regs = 12 / warps;
  return by_smem < by_regs ? by_smem : by_regs;
}

template <int D, int kWarps, int kStages>
__global__ void __launch_bounds__(32 * kWarps, decode_ctas_per_sm(D, kWarps, kStages))
    paged_decode_kernel(const PagedAttention p, int max_splits) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t smem[];
  const int G = p.q_heads / p.kv_heads;
  const int seg_index = blockIdx.x / p.kv_heads, kvh = blockIdx.x % p.kv_heads;
  const int split = blockIdx.y;
  const Segment seg = p.segments[seg_index];
  const int keys = seg.cached + seg.len;
  const int nsplit = (keys + p.keys_per_split - 1) / p.keys_per_split;
  if (nsplit > max_splits) {
    // A history longer than the launch's max_keys has more splits than its partial slots: the
    // row's heads are written as zeros and the status word (when given) records the bad argument.
    if (split == 0) {
      const int row = seg.row_start + seg.len - 1;
      const int G = p.q_heads / p.kv_heads;
      for (int i = threadIdx.x; i < G * D; i += blockDim.x)
        p.o[((long)row * p.q_heads + kvh * G + i / D) * D + i % D] = __float2bfloat16_rn(0.f);
      if (threadIdx.x == 0) record_status(p.status, kBadArgument);
    }
    return;
  }
  if (split >= nsplit) return;
  const int k0 = split * p.keys_per_split;
  const int k1 = min(keys, k0 + p.keys_per_split);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = seg.row_start + seg.len - 1;
  const float scale = p.scale * kLog2e;

  uint32_t qa[D / 16][4];
  load_q<D>(qa, [&](int m) -> const __nv_bfloat16* {
    return m < G ? p.q + ((long)row * p.q_heads + kvh * G + m) * D : nullptr;
  }, lane);

  Flash<D> f;
  f.init();
  constexpr int kTile = 16 * D * 2;  // bytes of one 16-key K (or V) block
  const uint32_t wbase = smem_u32(smem) + warp * kStages * 2 * kTile;  // [stage][K, V]
  const long page = 2L * p.kv_heads * 16 * D;
  const int b_first = k0 / 16, b_last = (k1 - 1) / 16;

  auto issue = [&](int b, int stage) {
    int id = p.table[seg.table_start + b];
    // A block ID past the cache (when its size is known) reads zeros and records the bad index.
    const bool valid = p.cache_blocks <= 0 || (id >= 0 && id < p.cache_blocks);
    if (!valid) {
      if (lane == 0) record_status(p.status, kBadIndex);
      id = 0;
    }
    const __nv_bfloat16* kp = p.cache + (long)id * page + (long)kvh * 16 * D;
    const __nv_bfloat16* vp = kp + (long)p.kv_heads * 16 * D;
    const uint32_t kt = wbase + stage * 2 * kTile, vt = kt + kTile;
#pragma unroll
    for (int i = 0; i < (16 * D / 8) / 32; ++i) {
      const int chunk = lane + i * 32;
      const int r = chunk / (D / 8), c = chunk % (D / 8);
      cp_async16(kt + swz<D>(r, c), kp + r * D + c * 8, valid ? 16 : 0);
      cp_async16(vt + swz<D>(r, c), vp + r * D + c * 8, valid ? 16 : 0);
    }
    cp_async_commit();
  };

  // kStages - 1 blocks in flight ahead of the one being folded (empty groups past the end keep
  // the group count uniform).
  int b = b_first + warp;
#pragma unroll
  for (int i = 0; i < kStages - 1; ++i) {
    if (b + i * kWarps <= b_last)
      issue(b + i * kWarps, i);
    else
      cp_async_commit();
  }
  for (int stage = 0; b <= b_last; b += kWarps, stage = stage + 1 == kStages ? 0 : stage + 1) {
    const int ahead = b + (kStages - 1) * kWarps;
    if (ahead <= b_last)
      issue(ahead, stage == 0 ? kStages - 1 : stage - 1);
    else
      cp_async_commit();
    cp_async_wait<kStages - 1>();
    __syncwarp();
    const uint32_t kt = wbase + stage * 2 * kTile, vt = kt + kTile;
    float s[2][4];
    qk<D, 2>(s, qa, kt, 0, lane);
    const int t = lane & 3;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int key = b * 16 + n * 8 + 2 * t + (i & 1);
        s[n][i] = key < k1 ? s[n][i] * scale : -INFINITY;
      }
    f.template fold<2>(s, vt, 0, lane);
    __syncwarp();
  }

  // Merge the warps: row statistics, then the rescaled outputs, through shared memory.
  f.l[0] = warp_sum4(f.l[0]);
  f.l[1] = warp_sum4(f.l[1]);
  __syncthreads();  // every warp is done with its K/V buffers
  float* sm_m = reinterpret_cast<float*>(smem);  // [kWarps][16]
  float* sm_l = sm_m + 16 * kWarps;              // [kWarps][16]
  float* sm_o = sm_l + 16 * kWarps;              // [16][D]
  const int g = lane >> 2, t = lane & 3;
  if (t == 0) {
    sm_m[warp * 16 + g] = f.m[0];
    sm_m[warp * 16 + g + 8] = f.m[1];
    sm_l[warp * 16 + g] = f.l[0];
    sm_l[warp * 16 + g + 8] = f.l[1];
  }
  for (int i = threadIdx.x; i < 16 * D; i += 32 * kWarps) sm_o[i] = 0.f;
  __syncthreads();
  float M[2], L[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = g + 8 * h;
    float mm = -INFINITY;
    for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, sm_m[w * 16 + r]);
    float ll = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float mw = sm_m[w * 16 + r];
      ll += mw == -INFINITY ? 0.f : sm_l[w * 16 + r] * exp2f(mw - mm);
    }
    M[h] = mm;
    L[h] = ll;
  }
  const float w0 = f.m[0] == -INFINITY ? 0.f : exp2f(f.m[0] - M[0]);
  const float w1 = f.m[1] == -INFINITY ? 0.f : exp2f(f.m[1] - M[1]);
  for (int w = 0; w < kWarps; ++w) {
    if (warp == w) {
#pragma unroll
      for (int j = 0; j < D / 8; ++j) {
        const int c = j * 8 + 2 * t;
        sm_o[g * D + c] += f.o[j][0] * w0;
        sm_o[g * D + c + 1] += f.o[j][1] * w0;
        sm_o[(g + 8) * D + c] += f.o[j][2] * w1;
        sm_o[(g + 8) * D + c + 1] += f.o[j][3] * w1;
      }
    }
    __syncthreads();
  }
  // Rows 0..G-1 hold the group's heads.
  for (int i = threadIdx.x; i < G * D; i += 32 * kWarps) {
    const int r = i / D, c = i % D;
    float mm = -INFINITY, ll = 0.f;
    for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, sm_m[w * 16 + r]);
    for (int w = 0; w < kWarps; ++w) {
      const float mw = sm_m[w * 16 + r];
      ll += mw == -INFINITY ? 0.f : sm_l[w * 16 + r] * exp2f(mw - mm);
    }
    const float v = sm_o[r * D + c] / ll;
    const int head = kvh * G + r;
    if (nsplit == 1) {
      p.o[((long)row * p.q_heads + head) * D + c] = __float2bfloat16_rn(v);
    } else {
      const long idx = ((long)seg_index * p.q_heads + head) * max_splits + split;
      p.partial_o[idx * D + c] = v;
      if (c == 0) p.partial_lse[idx] = mm + log2f(ll);
    }
  }
  if (nsplit == 1 || p.merge_counters == nullptr) return;
  // The last split of this (segment, key/value head) to finish merges the group's heads, in split
  // order as the separate merge kernel does (the same bits), and leaves its counter at zero.
  __shared__ int last_s;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* counter = p.merge_counters + seg_index * p.kv_heads + kvh;
    last_s = atomicAdd(counter, 1) == nsplit - 1;
    if (last_s) *counter = 0;
  }
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  for (int i = threadIdx.x; i < G * D; i += 32 * kWarps) {
    const int r = i / D, c = i % D;
    const long base = ((long)seg_index * p.q_heads + kvh * G + r) * max_splits;
    float mx = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) mx = fmaxf(mx, __ldcg(p.partial_lse + base + sp));
    float num = 0.f, den = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float w = exp2f(__ldcg(p.partial_lse + base + sp) - mx);
      num += w * __ldcg(p.partial_o + (base + sp) * D + c);
      den += w;
    }
    p.o[((long)row * p.q_heads + kvh * G + r) * D + c] = __float2bfloat16_rn(num / den);
  }
}

// Merges the 2048-key splits of each (segment, head) by log-sum-exp, in split order.
template <int D>
__global__ void decode_merge_kernel(const PagedAttention p, int max_splits) {
  pdl_wait();
  pdl_trigger();
  const int seg_index = blockIdx.x, head = blockIdx.y;
  const Segment seg = p.segments[seg_index];
  const int keys = seg.cached + seg.len;
  const int nsplit = (keys + p.keys_per_split - 1) / p.keys_per_split;
  if (nsplit == 1 || nsplit > max_splits) return;  // one split: written in place; too many: zeros
  const long base = ((long)seg_index * p.q_heads + head) * max_splits;
  float mx = -INFINITY;
  for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, p.partial_lse[base + s]);
  const int row = seg.row_start + seg.len - 1;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float num = 0.f, den = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float w = exp2f(p.partial_lse[base + s] - mx);
      num += w * p.partial_o[(base + s) * D + c];
      den += w;
    }
    p.o[((long)row * p.q_heads + head) * D + c] = __float2bfloat16_rn(num / den);
  }
}

// ------------------------------------------------------------------------------------ prefill
// The mma.sync path, for geometries the tensor-core kernel (attention_tc.cu) does not take: two
// CTAs per (work item = segment and 128-row query tile, key/value head), 64 rows each. Rows of the
// tile are (token, head) pairs of the group; 64-key tiles of K and V are double-buffered in shared
// memory and shared by the four warps.
template <int D>
__global__ void __launch_bounds__(128) paged_prefill_kernel(const PagedAttention p,
                                                            const int32_t* work) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t smem[];
  const int G = p.q_heads / p.kv_heads;
  // Two CTAs per 128-row work item, 64 rows each.
  const int seg_index = work[2 * (blockIdx.x >> 1)], tile = work[2 * (blockIdx.x >> 1) + 1];
  const int kvh = blockIdx.y;
  const Segment seg = p.segments[seg_index];
  const int total = seg.len * G;
  const int m0 = tile * kPrefillTile + (blockIdx.x & 1) * 64;
  if (m0 >= total) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const float scale = p.scale * kLog2e;

  uint32_t qa[D / 16][4];
  const int wm = m0 + warp * 16;
  load_q<D>(qa, [&](int m) -> const __nv_bfloat16* {
    const int pair = wm + m;
    if (pair >= total) return nullptr;
    const int tok = pair / G, h = pair % G;
    return p.q + ((long)(seg.row_start + tok) * p.q_heads + kvh * G + h) * D;
  }, lane);
  // Key limits (inclusive) of this thread's two rows, and of the warp and CTA.
  const int pr0 = wm + g, pr1 = wm + g + 8;
  const int all = seg.cached + seg.len - 1;  // bidirectional: every row attends every key
  const int lim0 = pr0 < total ? (p.bidirectional ? all : seg.cached + pr0 / G) : -1;
  const int lim1 = pr1 < total ? (p.bidirectional ? all : seg.cached + pr1 / G) : -1;
  const int last_pair = min(m0 + 63, total - 1);
  const int keys_end = p.bidirectional ? all + 1 : seg.cached + last_pair / G + 1;
  const int warp_last = min(wm + 15, total - 1);
  const int warp_end = wm < total ? (p.bidirectional ? all + 1 : seg.cached + warp_last / G + 1) : 0;

  Flash<D> f;
  f.init();
  constexpr int kTile = 64 * D * 2;
  const uint32_t sbase = smem_u32(smem);  // [stage][K, V]
  const long page = 2L * p.kv_heads * 16 * D;
  const int ntiles = (keys_end + 63) / 64;

  auto issue = [&](int kt, int stage) {
    const uint32_t ktile = sbase + stage * 2 * kTile, vtile = ktile + kTile;
    constexpr int kChunks = 64 * D / 8;
#pragma unroll
    for (int i = 0; i < kChunks / 128; ++i) {
      const int chunk = threadIdx.x + i * 128;
      const int r = chunk / (D / 8), c = chunk % (D / 8);
      const int blk = kt * 4 + r / 16;
      bool ok = blk < seg.nblocks;
      int id = ok ? p.table[seg.table_start + blk] : 0;
      if (ok && p.cache_blocks > 0 && (id < 0 || id >= p.cache_blocks)) {
        record_status(p.status, kBadIndex);  // read as zeros
        ok = false;
        id = 0;
      }
      const __nv_bfloat16* kp = p.cache + (long)id * page + (long)kvh * 16 * D + (r % 16) * D + c * 8;
      const __nv_bfloat16* vp = kp + (long)p.kv_heads * 16 * D;
      cp_async16(ktile + swz<D>(r, c), kp, ok ? 16 : 0);
      cp_async16(vtile + swz<D>(r, c), vp, ok ? 16 : 0);
    }
    cp_async_commit();
  };

  issue(0, 0);
  for (int kt = 0, stage = 0; kt < ntiles; ++kt, stage ^= 1) {
    if (kt + 1 < ntiles) {
      issue(kt + 1, stage ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kt * 64 < warp_end) {
      const uint32_t ktile = sbase + stage * 2 * kTile, vtile = ktile + kTile;
      float s[8][4];
      qk<D, 8>(s, qa, ktile, 0, lane);
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int key = kt * 64 + n * 8 + 2 * t + (i & 1);
          const int lim = i < 2 ? lim0 : lim1;
          s[n][i] = key <= lim ? s[n][i] * scale : -INFINITY;
        }
      f.template fold<8>(s, vtile, 0, lane);
    }
    __syncthreads();
  }
  f.l[0] = warp_sum4(f.l[0]);
  f.l[1] = warp_sum4(f.l[1]);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int pair = wm + g + 8 * h;
    if (pair >= total) continue;
    const int tok = pair / G, hd = pair % G;
    __nv_bfloat16* dst = p.o + ((long)(seg.row_start + tok) * p.q_heads + kvh * G + hd) * D;
    const float inv = 1.f / f.l[h];
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const int c = j * 8 + 2 * t;
      *reinterpret_cast<uint32_t*>(dst + c) =
          pack_bf16x2(f.o[j][2 * h] * inv, f.o[j][2 * h + 1] * inv);
    }
  }
}

// Warps of a decode CTA and blocks each keeps in its cp.async ring (see paged_decode_kernel).
constexpr int kDecodeWarps = 2;
constexpr int kDecodeStages = 2;

template <int D>
int decode_launch(const PagedAttention& p, cudaStream_t stream) {
  const int max_splits = (p.max_keys + p.keys_per_split - 1) / p.keys_per_split;
  if (max_splits > 1) {
    const size_t need = (size_t)p.num_segments * p.q_heads * max_splits;
    if (p.partial_o == nullptr || p.partial_lse == nullptr || need > p.partial_capacity) return -3;
  }
  const int warps = p.decode_warps >= 2 && p.decode_warps <= 4 ? p.decode_warps : kDecodeWarps;
  const int stages = p.decode_stages == 2 || p.decode_stages == 3 ? p.decode_stages : kDecodeStages;
  const int smem = warps * stages * 2 * 16 * D * 2;
  auto kernel = stages == 2 ? (warps == 2 ? paged_decode_kernel<D, 2, 2>
                               : warps == 3 ? paged_decode_kernel<D, 3, 2>
                                            : paged_decode_kernel<D, 4, 2>)
                            : (warps == 2 ? paged_decode_kernel<D, 2, 3>
                               : warps == 3 ? paged_decode_kernel<D, 3, 3>
                                            : paged_decode_kernel<D, 4, 3>);
  static bool configured[3][2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[warps - 2][stages - 2][dev & 63]) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured[warps - 2][stages - 2][dev & 63] = true;
  }
  dim3 grid(p.num_segments * p.kv_heads, max_splits);
  launch_pdl(kernel, dim3(grid), dim3(32 * warps), smem, stream, p, max_splits);
  if (max_splits > 1 && p.merge_counters == nullptr)
    launch_pdl(decode_merge_kernel<D>, dim3(p.num_segments, p.q_heads), dim3(D), 0, stream, p, max_splits);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

template <int D>
int prefill_launch(const PagedAttention& p, const int32_t* work, int num_work, cudaStream_t stream) {
  const int smem = 2 * 2 * 64 * D * 2;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaFuncSetAttribute(paged_prefill_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    configured[dev & 63] = true;
  }
  launch_pdl(paged_prefill_kernel<D>, dim3(2 * num_work, p.kv_heads), dim3(128), smem, stream, p, work);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

}  // namespace

int paged_decode(const PagedAttention& p, cudaStream_t stream) {
  if (p.num_segments <= 0) return 0;
  if (p.kv_heads <= 0 || p.q_heads % p.kv_heads != 0 || p.q_heads / p.kv_heads > 16) return -2;
  if (p.keys_per_split % 64 != 0 || p.max_keys <= 0) return -2;
  switch (p.head_dim) {
    case 64: return decode_launch<64>(p, stream);
    case 128: return decode_launch<128>(p, stream);
    default: return -2;
  }
}

int paged_prefill(const PagedAttention& p, const int32_t* work, int num_work, cudaStream_t stream) {
  if (num_work <= 0) return 0;
  if (p.kv_heads <= 0 || p.q_heads % p.kv_heads != 0) return -2;
  if (prefill_tc_supported(p)) return paged_prefill_tc(p, work, num_work, stream);
  switch (p.head_dim) {
    case 64: return prefill_launch<64>(p, work, num_work, stream);
    case 128: return prefill_launch<128>(p, work, num_work, stream);
    default: return -2;
  }
}

}  // namespace foa
