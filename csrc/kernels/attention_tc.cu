// Paged causal prefill attention on the tcgen05 tensor cores (flash attention over the block-table
// KV cache).
//
// Reference behaviour: prompt chunks attend the committed history plus their own rows causally
// (`ops/attention/full/paged/append/*`), softmax in FP32 over the scaled scores.
//
// Design for Blackwell (one CTA per 128-row query tile of one key/value head):
// - Rows are (token, head) pairs of the GQA group, so every key/value byte serves the whole group.
//   The query tile arrives by one 3-D TMA box per 64 columns ([tokens][heads][64]), 128-byte
//   swizzled: the K-major A operand of S = Q K^T.
// - Key/value tiles of 128 keys are eight 16-token pages, each a 16 x 64 TMA box per 64 columns
//   from its block of the cache (keys past the history read the box's zero fill). K is the K-major
//   B operand of S; V, stored [key][dim], is the MN-major B operand of O += P V, so neither needs a
//   transpose. Two K/V stages ring through shared memory.
// - S (two buffers) and O live in TMEM. One thread issues the MMAs: S_{j+1} while the softmax warps
//   work on S_j, then O += P_j V_j once P_j is in shared memory.
// - Eight softmax warps, two threads a row (TMEM lane = row, half the columns each): they read S_j,
//   mask causally (only tiles that cross the diagonal), keep a running maximum that moves only when
//   it grows by more than 2^8 (the O rescale by tcgen05.ld/st is then rare), write
//   P_j = exp2(S * scale - m) (one FMA and one ex2.approx an element) as BF16 into the swizzled
//   A-operand layout, and in the end divide O by the row sums and store the rows.
// - Every wait is bounded (mbarrier waits give up after 2 s, record a status and abort).

#include "attention.cuh"
#include "launch.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace foa {
namespace {

constexpr float kLog2eTc = 1.4426950408889634f;
constexpr int kRowsTc = 128;  // (token, head) rows of a query tile
constexpr int kKeysTc = 128;  // keys of a K/V tile (eight pages)

template <int D>
struct TcCfg {
  static constexpr int kHalfRows = 128 * 128;          // bytes of one 64-column half of a 128-row tile
  static constexpr int kQBytes = kRowsTc * D * 2;
  static constexpr int kKVBytes = kKeysTc * D * 2;
  static constexpr int kPBytes = kRowsTc * kKeysTc * 2;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQBytes;
  static constexpr int kOffV = kOffK + 2 * kKVBytes;
  static constexpr int kOffP = kOffV + 2 * kKVBytes;
  static constexpr int kOffBar = kOffP + kPBytes;
  static constexpr int kOffRed = kOffBar + 256;  // row maxima [2 tiles][2 halves][128], sums [2][128]
  // Barriers, reductions, then 1 KiB alignment slack; head_dim 64 pads to keep one CTA per SM (its
  // 512 TMEM columns are the whole SM's).
  static constexpr int kRaw = kOffRed + 6 * 128 * 4 + 1024;
  static constexpr int kSmem = kRaw < 120 * 1024 ? 120 * 1024 : kRaw;
  static constexpr int kColO = 2 * kKeysTc;  // TMEM: S0, S1 (128 columns each), then O
};

// Shared-memory descriptor of an MN-major operand stored as TMA writes [K rows][64 MN elements]
// with 128-byte swizzling: eight-row atoms along K `sbo` bytes apart, 64-element groups along MN
// `lbo` bytes apart.
__device__ __forceinline__ uint64_t sdesc_mnmajor_sw128(const void* smem, uint32_t lbo, uint32_t sbo) {
  const uint64_t addr = smem_u32(smem);
  uint64_t desc = 0;
  desc |= (addr >> 4) & 0x3FFFull;               // start address
  desc |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;  // leading byte offset: next 64 MN elements
  desc |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;  // stride byte offset: next 8 rows of K
  desc |= (uint64_t)1 << 46;                     // descriptor version of sm_100
  desc |= (uint64_t)2 << 61;                     // layout: 128-byte swizzle
  return desc;
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32"
      " [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

struct TcMaps {
  CUtensorMap q;      // [rows][q_heads][D] BF16, boxes of [128 / G tokens][G heads][64]
  CUtensorMap cache;  // [blocks * 2 * kv_heads * 16][D] BF16, boxes of [16 rows][64]
};

// 2^x by the hardware's approximate exponential (relative error about 2^-22; ex2(-inf) = 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
__global__ void __launch_bounds__(320, 1)
    paged_prefill_tc_kernel(const __grid_constant__ TcMaps maps, const PagedAttention p,
                            const int32_t* work, int cache_rows) {
  using C = TcCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem + C::kOffQ;
  uint8_t* sk = smem + C::kOffK;
  uint8_t* sv = smem + C::kOffV;
  uint8_t* sp = smem + C::kOffP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;     // [2]
  uint64_t* v_full = bars + 3;     // [2]
  uint64_t* kv_empty = bars + 5;   // [2]
  uint64_t* s_full = bars + 7;     // [2]
  uint64_t* s_empty = bars + 9;    // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* pv_done = bars + 12;
  uint64_t* mma_idle = bars + 13;  // every MMA issued has completed (before TMEM is freed)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  uint64_t* xbar = bars + 15;      // [2] the two threads of each row exchanged their tile maxima
  uint64_t* lbar = bars + 17;      // ... and their row sums
  uint64_t* k_empty = bars + 18;   // [2] S of the stage's tile completed (its K may be replaced)
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.q_heads / p.kv_heads;
  const int seg_index = work[2 * blockIdx.x], tile = work[2 * blockIdx.x + 1];
  const int kvh = blockIdx.y;
  const Segment seg = p.segments[seg_index];
  const int tok_per_tile = kRowsTc / G;
  const int tok0 = tile * tok_per_tile;                   // first token of the tile in the segment
  const int last_tok = min(seg.len, tok0 + tok_per_tile) - 1;
  // Keys any row of the tile attends (every key of the segment when bidirectional).
  const int keys_end = p.bidirectional ? seg.cached + seg.len : seg.cached + last_tok + 1;
  const int ntiles = (keys_end + kKeysTc - 1) / kKeysTc;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(kv_empty + s, 1);
      mbar_init(s_full + s, 1);
      mbar_init(s_empty + s, 256);
    }
    mbar_init(p_full, 256);
    mbar_init(pv_done, 1);
    mbar_init(mma_idle, 1);
    mbar_init(xbar, 256);
    mbar_init(xbar + 1, 256);
    mbar_init(lbar, 256);
    mbar_init(k_empty, 1);
    mbar_init(k_empty + 1, 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.q);
    tma_prefetch_desc(&maps.cache);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // the queries and the cache pages are the kernels' before
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (elect_one()) {
      mbar_arrive_expect_tx(q_full, C::kQBytes);
      for (int h = 0; h < D / 64; ++h)
        tma_load_3d(sq + h * C::kHalfRows, &maps.q, q_full, h * 64, kvh * G, seg.row_start + tok0);
      // Page rows of tile j in the cache (pages past the history read as the box's zero fill);
      // tile j + 1's block IDs are read while tile j's stage is awaited.
      auto page_rows = [&](int j, int (&kr)[8], int (&vr)[8]) {
#pragma unroll
        for (int pg = 0; pg < 8; ++pg) {
          const int b = j * 8 + pg;
          bool in = j < ntiles && b * 16 < keys_end && b < seg.nblocks;
          const long id = in ? p.table[seg.table_start + b] : 0;
          if (in && (id < 0 || id >= p.cache_blocks)) {
            record_status(p.status, kBadIndex);  // the page reads as the box's zero fill
            in = false;
          }
          kr[pg] = in ? (int)((id * 2 * p.kv_heads + kvh) * 16) : cache_rows;
          vr[pg] = in ? (int)((id * 2 * p.kv_heads + p.kv_heads + kvh) * 16) : cache_rows;
        }
      };
      int kr[8], vr[8];
      page_rows(0, kr, vr);
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int s = j & 1;
        // K of tile j - 2 is free once S_{j-2} completed; V once P_{j-2} V_{j-2} completed.
        if (j >= 2 && !mbar_wait(k_empty + s, ((j >> 1) + 1) & 1, p.status, kTimeoutSmemEmpty, abort)) break;
        mbar_arrive_expect_tx(k_full + s, C::kKVBytes);
#pragma unroll
        for (int pg = 0; pg < 8; ++pg)
#pragma unroll
          for (int h = 0; h < D / 64; ++h)
            tma_load_2d(sk + s * C::kKVBytes + h * C::kHalfRows + pg * 2048, &maps.cache, k_full + s, h * 64, kr[pg]);
        ++issued_k;
        if (j >= 2 && !mbar_wait(kv_empty + s, ((j >> 1) + 1) & 1, p.status, kTimeoutSmemEmpty, abort)) break;
        mbar_arrive_expect_tx(v_full + s, C::kKVBytes);
#pragma unroll
        for (int pg = 0; pg < 8; ++pg)
#pragma unroll
          for (int h = 0; h < D / 64; ++h)
            tma_load_2d(sv + s * C::kKVBytes + h * C::kHalfRows + pg * 2048, &maps.cache, v_full + s, h * 64, vr[pg]);
        ++issued_v;
        page_rows(j + 1, kr, vr);
      }
      // Let the loads in flight land before the CTA may exit (an abort stops the loop early).
      mbar_wait(q_full, 0, p.status, kTimeoutDrain, nullptr);
      for (int j = issued_k > 2 ? issued_k - 2 : 0; j < issued_k; ++j)
        mbar_wait(k_full + (j & 1), (j >> 1) & 1, p.status, kTimeoutDrain, nullptr);
      for (int j = issued_v > 2 ? issued_v - 2 : 0; j < issued_v; ++j)
        mbar_wait(v_full + (j & 1), (j >> 1) & 1, p.status, kTimeoutDrain, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(kRowsTc, kKeysTc);
      constexpr uint32_t idesc_o = idesc_bf16_f32(kRowsTc, D) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(q_full, 0, p.status, kTimeoutTmaFull, abort);
      auto issue_pv = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(p_full, j & 1, p.status, kTimeoutTmemFull, abort) ||
            !mbar_wait(v_full + s, (j >> 1) & 1, p.status, kTimeoutTmaFull, abort))
          return false;
        tc_fence_after();
        const uint8_t* vt = sv + s * C::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < kKeysTc / 16; ++kk) {
          const uint64_t a = sdesc_kmajor_sw128(sp + (kk >> 2) * C::kHalfRows + (kk & 3) * 32);
          const uint64_t b = sdesc_mnmajor_sw128(vt + kk * 2048, C::kHalfRows, 1024);
          mma_bf16(tmem + C::kColO, a, b, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(pv_done);
        mma_commit(kv_empty + s);
        return true;
      };
      for (int j = 0; ok && j < ntiles; ++j) {
        const int s = j & 1;
        if (!mbar_wait(k_full + s, (j >> 1) & 1, p.status, kTimeoutTmaFull, abort)) break;
        if (j >= 2 && !mbar_wait(s_empty + s, ((j >> 1) + 1) & 1, p.status, kTimeoutTmemEmpty, abort)) break;
        tc_fence_after();
        const uint8_t* kt = sk + s * C::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t a = sdesc_kmajor_sw128(sq + (kk >> 2) * C::kHalfRows + (kk & 3) * 32);
          const uint64_t b = sdesc_kmajor_sw128(kt + (kk >> 2) * C::kHalfRows + (kk & 3) * 32);
          mma_bf16(tmem + s * kKeysTc, a, b, idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(s_full + s);
        mma_commit(k_empty + s);
        if (j >= 1 && !issue_pv(j - 1)) ok = false;
      }
      if (ok && ntiles > 0) issue_pv(ntiles - 1);
      // No MMA may still write TMEM when it is freed (an abort can leave some in flight).
      mma_commit(mma_idle);
      mbar_wait(mma_idle, 0, p.status, kTimeoutDrain, nullptr);
    }
  } else {
    // ------------------------------------------------------------------ softmax (8 warps)
    // Warps 2-9: warp w reads TMEM lane quadrant w % 4 (its rows) and column half (w - 2) / 4 of
    // each S tile and of O; the two threads of a row meet through shared memory for the row
    // maximum (once a tile) and the row sum (at the end).
    const int q = warp & 3;
    const int ch = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const int tok = tok0 + row / G, head = row % G;
    const bool valid = tok < seg.len;
    // The last key this row attends, and the keys every row of the tile attends (tiles below
    // need no mask).
    const int qpos = !valid ? -1 : p.bidirectional ? seg.cached + seg.len - 1 : seg.cached + tok;
    const int unmasked_end = p.bidirectional ? seg.cached + seg.len : seg.cached + tok0 + 1;
    const float scale = p.scale * kLog2eTc;
    float m_use = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles && ok; ++j) {
      const int s = j & 1;
      int got = 1;
      if (lane == 0) got = mbar_wait(s_full + s, (j >> 1) & 1, p.status, kTimeoutTmemFull, abort);
      if (!__shfl_sync(0xffffffffu, got, 0)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float x[64];
#pragma unroll
      for (int c0 = 0; c0 < 64; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(lane_base + s * kKeysTc + ch * 64 + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 32; ++t) x[c0 + t] = __uint_as_float(r[t]);
      }
      tc_fence_before();
      mbar_arrive(s_empty + s);
      // Causal mask (tiles that reach past some row's position only), then the row maximum.
      const int k0 = j * kKeysTc + ch * 64;
      if (k0 + 63 >= unmasked_end) {
        const int lim = qpos - k0;  // columns above it are masked
#pragma unroll
        for (int c = 0; c < 64; ++c) x[c] = c > lim ? -INFINITY : x[c];
      }
      float mx = x[0];
#pragma unroll
      for (int c = 1; c < 64; ++c) mx = fmaxf(mx, x[c]);
      float* red = reinterpret_cast<float*>(smem + C::kOffRed) + (s * 2) * kRowsTc;  // [tile parity][half][row]
      red[ch * kRowsTc + row] = mx;
      mbar_arrive(xbar + s);  // bounded exchange (a named barrier could not give up)
      if (!mbar_wait(xbar + s, (j >> 1) & 1, p.status, kTimeoutTmemFull, abort)) {
        ok = false;
        break;
      }
      mx = fmaxf(red[row], red[kRowsTc + row]) * scale;
      // The reference maximum moves only when the tile's maximum exceeds it by 2^8 (or on the
      // first finite maximum): exp2 of the difference then stays within BF16 and FP32 range.
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_use + 8.f) {
        alpha = m_use == -INFINITY ? 0.f : ex2_approx(m_use - mx);
        rescale = m_use != -INFINITY;
        m_use = mx;
      }
      l *= alpha;
      // O may be rescaled and P overwritten once the previous tile's P V has completed.
      if (j >= 1) {
        int done = 1;
        if (lane == 0) done = mbar_wait(pv_done, (j - 1) & 1, p.status, kTimeoutTmemFull, abort);
        if (!__shfl_sync(0xffffffffu, done, 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int c0 = 0; c0 < D / 2; c0 += 32) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(lane_base + C::kColO + ch * (D / 2) + c0, r);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < 32; ++t) r[t] = __float_as_uint(__uint_as_float(r[t]) * alpha);
            tmem_st_32x32b_x32(lane_base + C::kColO + ch * (D / 2) + c0, r);
          }
          tmem_st_wait();
        }
      }
      // P = exp2(S * scale - m) as BF16 into half `ch` of the swizzled K-major layout
      // ([2 halves][128 rows][128 bytes]); a row never seen unmasked keeps exp2(-inf) = 0.
      const float neg = m_use == -INFINITY ? 0.f : -m_use;
      const uint32_t prow = smem_u32(sp) + ch * C::kHalfRows + row * 128;
#pragma unroll
      for (int c16 = 0; c16 < 8; ++c16) {
        uint32_t w[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float e0 = ex2_approx(fmaf(x[c16 * 8 + 2 * t], scale, neg));
          const float e1 = ex2_approx(fmaf(x[c16 * 8 + 2 * t + 1], scale, neg));
          l += e0 + e1;
          w[t] = pack_bf16x2(e0, e1);
        }
        st_shared_v4(prow + ((c16 ^ (row & 7)) << 4), w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // Epilogue: O / l for the tile's valid rows, each thread its half of the columns.
    int done = ok ? 1 : 0;
    if (ok && ntiles > 0 && lane == 0) done = mbar_wait(pv_done, (ntiles - 1) & 1, p.status, kTimeoutTmemFull, abort);
    done = __shfl_sync(0xffffffffu, done, 0);
    float* lred = reinterpret_cast<float*>(smem + C::kOffRed) + 4 * kRowsTc;  // [half][row]
    lred[ch * kRowsTc + row] = l;
    mbar_arrive(lbar);
    if (done && !mbar_wait(lbar, 0, p.status, kTimeoutTmemFull, abort)) done = 0;
    done = __all_sync(0xffffffffu, done);
    if (done && ntiles > 0) {
      tc_fence_after();
      const float lt = lred[row] + lred[kRowsTc + row];
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      __nv_bfloat16* dst = p.o + ((long)(seg.row_start + tok) * p.q_heads + kvh * G + head) * D + ch * (D / 2);
#pragma unroll
      for (int c0 = 0; c0 < D / 2; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(lane_base + C::kColO + ch * (D / 2) + c0, r);
        tmem_ld_wait();
        if (valid) {
#pragma unroll
          for (int t = 0; t < 32; t += 8) {
            const uint4 v4 = make_uint4(pack_bf16x2(__uint_as_float(r[t]) * inv, __uint_as_float(r[t + 1]) * inv),
                                        pack_bf16x2(__uint_as_float(r[t + 2]) * inv, __uint_as_float(r[t + 3]) * inv),
                                        pack_bf16x2(__uint_as_float(r[t + 4]) * inv, __uint_as_float(r[t + 5]) * inv),
                                        pack_bf16x2(__uint_as_float(r[t + 6]) * inv, __uint_as_float(r[t + 7]) * inv));
            *reinterpret_cast<uint4*>(dst + c0 + t) = v4;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// 3-D tensor map of the queries [rows][q_heads][D]: boxes of [tokens][G heads][64 columns].
bool encode_q_map(CUtensorMap* map, const void* q, int rows, int q_heads, int d, int group) {
  auto fn = tmap_encoder();
  if (fn == nullptr || (reinterpret_cast<uintptr_t>(q) & 15) != 0) return false;
  cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)q_heads, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)d * 2, (cuuint64_t)q_heads * d * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)group, (cuuint32_t)(kRowsTc / group)};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D>
int prefill_tc_launch(const PagedAttention& p, const int32_t* work, int num_work, cudaStream_t stream) {
  using C = TcCfg<D>;
  const int G = p.q_heads / p.kv_heads;
  const long rows64 = (long)p.cache_blocks * 2 * p.kv_heads * 16;
  if (rows64 <= 0 || rows64 >= (1L << 31) - 16) return -2;
  TcMaps maps;
  if (!encode_q_map(&maps.q, p.q, p.rows, p.q_heads, D, G)) return -4;
  if (!encode_tmap_2d(&maps.cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.cache, rows64, D, D, 16, 64,
                      CU_TENSOR_MAP_SWIZZLE_128B))
    return -4;
  auto kernel = paged_prefill_tc_kernel<D>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    configured[dev & 63] = true;
  }
  return launch_pdl(kernel, dim3(num_work, p.kv_heads), dim3(320), C::kSmem, stream, maps, p, work,
                    (int)rows64) == cudaSuccess
             ? 0
             : -5;
}

}  // namespace

bool prefill_tc_supported(const PagedAttention& p) {
  const int G = p.kv_heads > 0 ? p.q_heads / p.kv_heads : 0;
  return (p.head_dim == 64 || p.head_dim == 128) && G >= 1 && G <= 16 && kRowsTc % G == 0 &&
         p.rows > 0 && p.cache_blocks > 0;
}

int paged_prefill_tc(const PagedAttention& p, const int32_t* work, int num_work, cudaStream_t stream) {
  if (num_work <= 0) return 0;
  if (!prefill_tc_supported(p)) return -2;
  return p.head_dim == 64 ? prefill_tc_launch<64>(p, work, num_work, stream)
                          : prefill_tc_launch<128>(p, work, num_work, stream);
}

}  // namespace foa
