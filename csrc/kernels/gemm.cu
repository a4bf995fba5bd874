// BF16 GEMM on the sm_100a tensor cores: C = epilogue(A . W^T).
//
// One persistent kernel family serves every dense projection of the decoders (the packed
// q/k/v projection, the output projection, gate/up with its SwiGLU, down, and the vocabulary
// head). It replaces the reference's Tensor-Unit contractions
// (crates/furiosa-opt-models/src/ops/linear/{mod,kernel,rows}.rs, ops/swiglu/mod.rs:1-8) with a
// design for Blackwell:
//
// - Warp roles, 192 threads: warp 0 issues TMA loads (one elected thread), warp 1 allocates TMEM
//   and issues tcgen05.mma (one elected thread), warps 2-5 drain the FP32 accumulators from TMEM
//   with tcgen05.ld and apply the epilogue in registers.
// - Operands are staged by TMA with 128-byte swizzling into a ring of shared-memory stages
//   guarded by full/empty mbarriers; MMAs read them through K-major shared-memory descriptors.
// - Accumulators live in TMEM, double-buffered where they fit, so the epilogue of one tile
//   overlaps the MMAs of the next.
// - Two operand mappings: "rows" (activations on the MMA's M side, 128 x 256 tiles) for prefill
//   and "swap" (weight rows on M, the few activation rows on N) for decode, where a 64-row batch
//   would waste half of a 128-row MMA.
// - Split-K for launches with fewer tiles than SMs: each split writes FP32 partials to scratch and
//   the last split of a tile (an arrival counter) adds them in split order, so the result does not
//   depend on which split finishes first.
//
// Numerics: FP32 accumulation, one rounding to BF16 (after the residual add where there is one),
// as the reference's contractions round once (ops/pointwise/add.rs:1).

#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "gemm.cuh"
#include "launch.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace foa {
namespace {

constexpr int kBlockK = 64;  // 64 BF16 = 128 bytes: one swizzled row

struct KParams {
  int Mp, Nq;                 // rows of the M-side and N-side operands
  int tiles_p, tiles_q;       // tile counts along M and N
  int splits, kblocks, kb_per_split;
  int units;                  // tiles * splits
  int swap;                   // 1: C[j, i] (N-side rows are output rows)
  int tma_store;              // rows mapping, BF16 output through shared memory and TMA stores
  int external;               // split partials stay in ws for the next kernel (GemmSplits layout)
  void* c;
  long ldc;
  const __nv_bfloat16* res;
  long ldr;
  float* ws;
  int* counters;
  int* status;
  int out_rows, out_cols;     // logical output shape
  unsigned long long* trace;  // milestone timestamps of CTA 0, or null
  unsigned long long* cta_trace;  // per-CTA timestamps (8 a CTA; see GemmArgs), or null
  int debug;                  // measurement switches (GemmArgs::debug): 1 no stores, 2 no TMEM loads
  // Quantized weights (kWF != 0): block scales and the factor the FP32 sums take.
  const void* wscale;         // FP8: FP32 [ceil(N/128)][ceil(K/128)]; NVFP4: E4M3 [N][K/16]
  long wscale_ld;             // scale elements per scale row
  int wscale_row_shift;       // FP8 converter: scale row = weight row >> shift (7: 128-row blocks, 0: rows)
  int wscale_k_shift;         // FP8 converter: scale column = k-block >> shift (1: 128 columns, 31: one)
  float acc_scale;            // NVFP4 tensor scale (1 otherwise), applied to the reduced sum
  // Block-scaled operands (kWF == kWNvfp4A4): scale atoms of the M-side and N-side operands,
  // [row block of 128][K/64][512 bytes], and the bytes between two row blocks.
  const uint8_t* sf_p;
  const uint8_t* sf_q;
  long sf_stride_p, sf_stride_q;
  int sf_blocks_q;            // 128-row blocks of the N side's atoms
  // FP8 W8A8 (kWF == kWFp8A8): activation scales [K/128][ascale_ld] (transposed per k-block).
  const float* ascale;
  long ascale_ld;
  // Grouped (mixture-of-experts) swap GEMM: the N-side token tiles and the group (expert) whose
  // weights each tile multiplies come from the device; weights of group g start at row
  // g * group_rows.
  // Extra K segments (BF16): k-blocks [seg_kb[0], seg_kb[1]) read aux p1/q1 and [seg_kb[1],
  // kblocks) read aux p2/q2, each from its own column 0. seg_kb[0] == kblocks: one segment.
  int seg_kb[2];
  const int* group_tiles;  // number of token tiles (device), or null
  const int* tile_group;   // group of each token tile (device)
  long group_rows;
};

// Weight formats a GEMM reads: BF16; FP8 block-scaled or NVFP4 codes dequantized to BF16 in
// shared memory (BF16 activations); NVFP4 codes of both operands on the block-scaled MMA.
// FP8 codes of both operands on the FP8 MMA, each 128-input block's sum scaled by the
// epilogue warps before the blocks add (W8A8).
enum : int { kWBf16 = 0, kWFp8Block = 1, kWNvfp4 = 2, kWNvfp4A4 = 3, kWFp8A8 = 4 };

// Eight E4M3 codes times their block scale, rounded to BF16.
__device__ __forceinline__ uint4 dequant_fp8x8(uint2 v, float scale) {
  uint32_t w[4];
  const uint32_t in[2] = {v.x, v.y};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_fp8x2_storage_t pair = static_cast<__nv_fp8x2_storage_t>(in[i >> 1] >> (16 * (i & 1)));
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3);
    const float2 f = __half22float2(__half2(h));
    w[i] = pack_bf16x2(f.x * scale, f.y * scale);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// An E4M3 scale as two BF16 copies (exact: E4M3 values are BF16 values).
__device__ __forceinline__ uint32_t e4m3_bf16x2(uint8_t scale_byte) {
  const __half_raw hs = __nv_cvt_fp8_to_halfraw(scale_byte, __NV_E4M3);
  const uint32_t b = __bfloat16_as_ushort(__float2bfloat16_rn(__half2float(__half(hs))));
  return b | (b << 16);
}

// Eight E2M1 codes (low nibble first) times their scale (`scale2`, two BF16 copies), by byte
// permutes: each 3-bit magnitude indexes the high and the low BF16 bytes of {0, 0.5, 1, 1.5, 2, 3,
// 4, 6} (high {00 3F 3F 3F 40 40 40 40}, low {00 00 80 C0 00 40 80 C0}), the sign bits move into the
// high bytes, and the bytes interleave into BF16 pairs. The products are exact in BF16.
__device__ __forceinline__ uint4 dequant_e2m1x8_permute(uint32_t v, uint32_t scale2) {
  const uint32_t m = v & 0x77777777u;
  const uint32_t hi_a = prmt(0x3F3F3F00u, 0x40404040u, m);
  const uint32_t lo_a = prmt(0xC0800000u, 0xC0804000u, m);
  const uint32_t hi_b = prmt(0x3F3F3F00u, 0x40404040u, m >> 16);
  const uint32_t lo_b = prmt(0xC0800000u, 0xC0804000u, m >> 16);
  // Byte i of `even` / `odd` holds the sign of code 2i / 2i + 1 in its top bit.
  const uint32_t even = (v << 4) & 0x80808080u, odd = v & 0x80808080u;
  const uint32_t h0 = hi_a | prmt(even, odd, 0x5140u);
  const uint32_t h1 = hi_b | prmt(even, odd, 0x7362u);
  return make_uint4(mul_bf16x2(prmt(lo_a, h0, 0x5140u), scale2), mul_bf16x2(prmt(lo_a, h0, 0x7362u), scale2),
                    mul_bf16x2(prmt(lo_b, h1, 0x5140u), scale2), mul_bf16x2(prmt(lo_b, h1, 0x7362u), scale2));
}

__device__ __forceinline__ void mark(const KParams& p, int i) {
  if (p.trace != nullptr && blockIdx.x == 0) p.trace[i] = global_ns();
  // Milestones 0, 5, 6 of every CTA (its end is written after the last barrier).
  if (p.cta_trace != nullptr && (i == 0 || i == 5 || i == 6)) p.cta_trace[8 * blockIdx.x + (i == 0 ? 0 : i - 4)] = global_ns();
}

template <int kMB, int kBN, int kStages, int kAcc, int kWF = kWBf16>
struct Cfg {
  static constexpr int kPRows = 128 * kMB;
  static constexpr int kPBytes = kPRows * 128;
  static constexpr int kQBytes = kBN * 128;
  static constexpr int kStageBytes = kPBytes + kQBytes;
  // Quantized weights land raw in a side ring first (rows of one k-block: 64 FP8 bytes or 32
  // packed NVFP4 bytes), sized for the larger of the two operand tiles.
  static constexpr int kWRows = kPRows > kBN ? kPRows : kBN;
  static constexpr int kRawRow = kWF == kWFp8Block ? 64 : kWF == kWNvfp4 ? 32 : 0;
  static constexpr int kRawBytes = kWRows * kRawRow;
  // Block-scaled operands: per stage one 2 KiB group of scale atoms (4 MMAs x 512 bytes) for each
  // 128 rows of either side, copied into TMEM columns after the accumulators. An MMA reads the
  // scales of its 32-row slices from consecutive columns, four bytes (four K groups) a column.
  static constexpr int kQGroups = (kBN + 127) / 128;
  static constexpr int kSfBytes = kWF == kWNvfp4A4 ? (kMB + kQGroups) * 2048 : 0;
  static constexpr int kSfCols = kWF == kWNvfp4A4 ? 16 * (kMB + kQGroups) : 0;
  static constexpr int kBoxX = (kWF == kWNvfp4A4 || kWF == kWFp8A8) ? 128 : 64;  // TMA x of a k-block
  // W8A8: the FP32 activation scales of one k-block for the tile's tokens, then the weight scale
  // of each M block (16 bytes apiece, as stored).
  static constexpr int kAscOnly = 4 * (kBN > 128 ? kBN : 128);
  static constexpr int kAscBytes = kWF == kWFp8A8 ? kAscOnly + 16 * kMB : 0;
  static constexpr int kAccCols = kMB * kBN;
  static constexpr int kSfCol0 = kAcc * kAccCols;
  static constexpr int kColsRaw = kAcc * kAccCols + kSfCols;
  static constexpr int kTmemCols = kColsRaw <= 32    ? 32
                                   : kColsRaw <= 64  ? 64
                                   : kColsRaw <= 128 ? 128
                                   : kColsRaw <= 256 ? 256
                                                     : 512;
  static constexpr int kBarrierBytes = 512;
  // BF16 rows-mapping output staging: one 32 x 64 box (4 KiB) for each epilogue warp.
  static constexpr int kOutStage = (kWF == kWBf16 && kMB == 1) ? 4 * 4096 : 0;
  static constexpr int kSmemBytes =
      kStages * (kStageBytes + kRawBytes + kSfBytes + kAscBytes) + kOutStage + kBarrierBytes + 1024;
  // Converter warps (kWF 1, 2: warps 6-13) or a second stream of scaling warps (kWF 4: warps 6-9).
  static constexpr int kConvWarps = (kWF == kWFp8Block || kWF == kWNvfp4) ? 8 : 0;
  static constexpr int kThreadsCta = kConvWarps ? 192 + 32 * kConvWarps : kWF == kWFp8A8 ? 320 : 192;
  // Items of 8 codes a converter thread expands a stage (weight rows x 8 column groups).
  static constexpr int kConvItems = kConvWarps ? (kWRows * 8) / (32 * kConvWarps) : 1;
  static_assert(kColsRaw <= 512, "accumulators exceed TMEM");
  static_assert(kSmemBytes <= 232448, "stages exceed shared memory");
  static_assert(kBN % 16 == 0 && kBN >= 16 && kBN <= 256, "invalid MMA N");
};

__device__ __forceinline__ void epi_barrier() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

__device__ __forceinline__ float silu_bf16_times(float g_acc, float u_acc) {
  // Rounded as the reference's SwiGLU rounds: each projection to BF16, SiLU(gate) to BF16, then
  // the product to BF16 by the caller.
  const float g = __bfloat162float(__float2bfloat16_rn(g_acc));
  const float u = __bfloat162float(__float2bfloat16_rn(u_acc));
  const float s = __bfloat162float(__float2bfloat16_rn(g / (1.0f + __expf(-g))));
  return s * u;
}

// Stores 16 consecutive output values of one output row (rows mapping) or one output column
// (swap mapping), applying the residual add and the output type of the epilogue.
template <int kEpi>
__device__ __forceinline__ void store16(const KParams& p, int row, int col, const float (&v)[16],
                                        bool along_row) {
  // along_row: the 16 values are C[row, col + t]; otherwise C[row + t, col].
  if (p.debug & 1) return;
  if (kEpi == kEpiF32) {
    float* c = static_cast<float*>(p.c);
    if (along_row) {
      if (row >= p.out_rows) return;
      float* dst = c + (long)row * p.ldc + col;
      if (col + 16 <= p.out_cols) {
#pragma unroll
        for (int t = 0; t < 16; t += 4)
          *reinterpret_cast<float4*>(dst + t) = make_float4(v[t], v[t + 1], v[t + 2], v[t + 3]);
      } else {
        for (int t = 0; t < 16 && col + t < p.out_cols; ++t) dst[t] = v[t];
      }
    } else {
      if (col >= p.out_cols) return;
#pragma unroll
      for (int t = 0; t < 16; ++t)
        if (row + t < p.out_rows) c[(long)(row + t) * p.ldc + col] = v[t];
    }
    return;
  }
  __nv_bfloat16* c = static_cast<__nv_bfloat16*>(p.c);
  if (along_row) {
    if (row >= p.out_rows) return;
    float w[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) w[t] = v[t];
    if (p.res != nullptr) {
      const __nv_bfloat16* r = p.res + (long)row * p.ldr + col;
#pragma unroll
      for (int t = 0; t < 16; ++t)
        if (col + t < p.out_cols) w[t] += __bfloat162float(r[t]);
    }
    __nv_bfloat16* dst = c + (long)row * p.ldc + col;
    if (col + 16 <= p.out_cols) {
      uint4 lo = make_uint4(pack_bf16x2(w[0], w[1]), pack_bf16x2(w[2], w[3]),
                            pack_bf16x2(w[4], w[5]), pack_bf16x2(w[6], w[7]));
      uint4 hi = make_uint4(pack_bf16x2(w[8], w[9]), pack_bf16x2(w[10], w[11]),
                            pack_bf16x2(w[12], w[13]), pack_bf16x2(w[14], w[15]));
      reinterpret_cast<uint4*>(dst)[0] = lo;
      reinterpret_cast<uint4*>(dst)[1] = hi;
    } else {
      for (int t = 0; t < 16 && col + t < p.out_cols; ++t) dst[t] = __float2bfloat16_rn(w[t]);
    }
  } else {
    if (col >= p.out_cols) return;
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      const int r = row + t;
      if (r < p.out_rows) {
        float x = v[t];
        if (p.res != nullptr) x += __bfloat162float(p.res[(long)r * p.ldr + col]);
        c[(long)r * p.ldc + col] = __float2bfloat16_rn(x);
      }
    }
  }
}

// kRed: how K splits meet. kRedNone: one split. kRedGlobal: FP32 partials in global scratch, the
// last split of a tile (arrival counter) adds them in split order. kRedCluster: the splits of a tile
// form one thread-block cluster; each stages its partial in its own shared memory and every CTA
// reduces a slice of the tile's rows over distributed shared memory, in split order.
enum : int { kRedNone = 0, kRedGlobal = 1, kRedCluster = 2 };

template <int kEpi>
__device__ __forceinline__ void store_one(const KParams& p, int row, int col, float v) {
  if (row >= p.out_rows || col >= p.out_cols) return;
  if (kEpi == kEpiF32) {
    static_cast<float*>(p.c)[(long)row * p.ldc + col] = v;
    return;
  }
  if (p.res != nullptr) v += __bfloat162float(p.res[(long)row * p.ldr + col]);
  static_cast<__nv_bfloat16*>(p.c)[(long)row * p.ldc + col] = __float2bfloat16_rn(v);
}

// Stores 8 consecutive output values C[row, col .. col + 7] (col a multiple of 8), applying the
// residual add and the output type of the epilogue; the cluster split-K reduction's store.
template <int kEpi>
__device__ __forceinline__ void store8(const KParams& p, int row, int col, const float (&v)[8]) {
  if (row >= p.out_rows || col >= p.out_cols) return;
  const bool whole = col + 8 <= p.out_cols;
  if (kEpi == kEpiF32) {
    float* dst = static_cast<float*>(p.c) + (long)row * p.ldc + col;
    if (whole) {
      reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t)
        if (col + t < p.out_cols) dst[t] = v[t];
    }
    return;
  }
  float w[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) w[t] = v[t];
  __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.c) + (long)row * p.ldc + col;
  if (whole) {
    if (p.res != nullptr) {
      const uint4 rv = *reinterpret_cast<const uint4*>(p.res + (long)row * p.ldr + col);
      const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        w[2 * t] += bf16_lo(rw[t]);
        w[2 * t + 1] += bf16_hi(rw[t]);
      }
    }
    *reinterpret_cast<uint4*>(dst) = make_uint4(pack_bf16x2(w[0], w[1]), pack_bf16x2(w[2], w[3]),
                                                pack_bf16x2(w[4], w[5]), pack_bf16x2(w[6], w[7]));
  } else {
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      if (col + t >= p.out_cols) continue;
      float x = w[t];
      if (p.res != nullptr) x += __bfloat162float(p.res[(long)row * p.ldr + col + t]);
      dst[t] = __float2bfloat16_rn(x);
    }
  }
}

// Rows of the tile one CTA of a split-K cluster reduces: an equal share rounded up to 8, so each
// thread of the reduction adds and stores 8 consecutive outputs at a time.
__device__ __forceinline__ int slice_rows(int rows, int splits) {
  return (((rows + splits - 1) / splits) + 7) & ~7;
}

// Tensor maps beyond the two operands: the raw quantized weights a converter reads, and the
// operand pairs of up to two extra K segments (BF16 only: LoRA updates [X | Z1 | Z2] x
// [W | B1 | B2]^T, one rounding for the whole sum).
struct AuxMaps {
  CUtensorMap w;
  CUtensorMap p1, q1, p2, q2;
  CUtensorMap c;  // BF16 output [rows, cols], boxes of 32 rows x 64 columns (TMA stores)
};

template <int kMB, int kBN, int kStages, int kAcc, int kEpi, int kRed, int kWF = kWBf16>
__global__ void __launch_bounds__((Cfg<kMB, kBN, kStages, kAcc, kWF>::kThreadsCta), 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmP,
                     const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ AuxMaps aux, const KParams p) {
  const CUtensorMap& tmW = aux.w;
  using C = Cfg<kMB, kBN, kStages, kAcc, kWF>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* raw = smem + kStages * C::kStageBytes;  // quantized weight ring (kWF 1, 2)
  uint8_t* sfr = raw + kStages * C::kRawBytes;      // scale-atom ring (kWF 3)
  uint8_t* asr = sfr + kStages * C::kSfBytes;       // activation-scale ring (kWF 4)
  uint8_t* outst = asr + kStages * C::kAscBytes;  // output staging (kOutStage bytes, 1 KiB aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(outst + C::kOutStage);
  uint64_t* empty = full + kStages;
  uint64_t* rawfull = empty + kStages;
  uint64_t* tfull = rawfull + kStages;
  uint64_t* tempty = tfull + kAcc;
  uint64_t* xfer = tempty + kAcc;  // W8A8: odd-block stream's sum ready / taken (two barriers)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xfer + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  // The next kernel may launch at once; its own grid-dependency wait orders it after this one.
  pdl_trigger();
  if (threadIdx.x == 0) mark(p, 0);
  // A grouped launch learns its token tiles from the routing kernel before it.
  int units = p.units;
  if (p.group_tiles != nullptr) {
    pdl_wait();
    units = p.tiles_p * min(*reinterpret_cast<const volatile int*>(p.group_tiles), p.tiles_q) * p.splits;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      // A stage is full when its TMA bytes land and, for quantized weights, every converter warp
      // has written its share of the weight tile.
      mbar_init(full + s, 1 + C::kConvWarps);
      // W8A8: a stage is free once its MMAs completed and the eight scaling warps read its scales.
      mbar_init(empty + s, kWF == kWFp8A8 ? 9 : 1);
      mbar_init(rawfull + s, 1);
    }
    for (int b = 0; b < kAcc; ++b) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, kWF == kWFp8A8 ? 256 : 128);  // W8A8: both scaling streams
    }
    mbar_init(xfer, 128);
    mbar_init(xfer + 1, 128);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmP);
    tma_prefetch_desc(&tmQ);
    if (kWF == kWFp8Block || kWF == kWNvfp4) tma_prefetch_desc(&tmW);
    if (kWF == kWBf16 && p.seg_kb[0] < p.kblocks) {
      tma_prefetch_desc(&aux.p1);
      tma_prefetch_desc(&aux.q1);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) mark(p, 1);

  if (warp == 0) {
    // ----------------------------------------------------------------- TMA producer
    if (elect_one()) {
      uint32_t it = 0;
      bool ok = true;
      // Weight tile of stage s: straight into the stage (BF16), or raw into the side ring for the
      // converter warps (quantized formats).
      // Scale atoms of stage s: the M side's 128-row blocks first, then the N side's block.
      auto load_sf = [&](int s, int kb, int tp, int tq, bool p_side) {
        uint8_t* dst = sfr + s * C::kSfBytes;
        if (p_side) {
          for (int mb = 0; mb < kMB; ++mb)
            bulk_load(dst + mb * 2048, p.sf_p + (long)(tp * kMB + mb) * p.sf_stride_p + (long)kb * 2048,
                      2048, full + s);
        } else {
          // A 256-row tile past the last block re-reads that block: its rows have zero codes.
          for (int g = 0; g < C::kQGroups; ++g)
            bulk_load(dst + (kMB + g) * 2048,
                      p.sf_q + (long)min(((tq * kBN) >> 7) + g, p.sf_blocks_q - 1) * p.sf_stride_q +
                          (long)kb * 2048,
                      2048, full + s);
        }
      };
      // The K segment of k-block kb: its maps and its first column.
      auto seg_maps = [&](int kb, const CUtensorMap*& mp, const CUtensorMap*& mq, int& x) {
        mp = &tmP;
        mq = &tmQ;
        x = kb * C::kBoxX;
        if constexpr (kWF == kWBf16) {
          if (kb >= p.seg_kb[1]) {
            mp = &aux.p2;
            mq = &aux.q2;
            x = (kb - p.seg_kb[1]) * C::kBoxX;
          } else if (kb >= p.seg_kb[0]) {
            mp = &aux.p1;
            mq = &aux.q1;
            x = (kb - p.seg_kb[0]) * C::kBoxX;
          }
        }
      };
      auto load_w = [&](int s, int kb, int tp, int tq) {
        uint8_t* st = smem + s * C::kStageBytes;
        if constexpr (kWF == kWBf16 || kWF == kWNvfp4A4 || kWF == kWFp8A8) {
          const CUtensorMap *mp, *mq;
          int x;
          seg_maps(kb, mp, mq, x);
          if (p.swap) {
            const long g0 = p.tile_group != nullptr ? (long)p.tile_group[tq] * p.group_rows : 0;
            tma_load_2d(st, mp, full + s, x, (int)(g0 + tp * C::kPRows));
          } else {
            tma_load_2d(st + C::kPBytes, mq, full + s, x, tq * kBN);
          }
          if constexpr (kWF == kWNvfp4A4) load_sf(s, kb, tp, tq, p.swap != 0);
        } else {
          const int rows = p.swap ? C::kPRows : kBN;
          mbar_arrive_expect_tx(rawfull + s, rows * C::kRawRow);
          tma_load_2d(raw + s * C::kRawBytes, &tmW, rawfull + s, kb * C::kRawRow,
                      p.swap ? tp * C::kPRows : tq * kBN);
        }
      };
      auto load_a = [&](int s, int kb, int tp, int tq) {
        uint8_t* st = smem + s * C::kStageBytes;
        const CUtensorMap *mp, *mq;
        int x;
        seg_maps(kb, mp, mq, x);
        if (p.swap)
          tma_load_2d(st + C::kPBytes, mq, full + s, x, tq * kBN);
        else
          tma_load_2d(st, mp, full + s, x, tp * C::kPRows);
        if constexpr (kWF == kWNvfp4A4) load_sf(s, kb, tp, tq, p.swap == 0);
        if constexpr (kWF == kWFp8A8) {
          if (p.swap)
            bulk_load(asr + s * C::kAscBytes, p.ascale + (long)kb * p.ascale_ld + tq * kBN, kBN * 4, full + s);
          else
            bulk_load(asr + s * C::kAscBytes, p.ascale + (long)kb * p.ascale_ld + tp * 128, 512, full + s);
          // Weight scales [row block][K/128][4 copies]: one 16-byte entry per M block.
          const float* wsc = static_cast<const float*>(p.wscale);
          for (int mb = 0; mb < (p.swap ? kMB : 1); ++mb)
            bulk_load(asr + s * C::kAscBytes + C::kAscOnly + 16 * mb,
                      wsc + ((long)(p.swap ? tp * kMB + mb : tq) * p.wscale_ld + kb) * 4, 16, full + s);
        }
      };
      const uint32_t full_bytes = kWF == kWBf16      ? C::kStageBytes
                                  : kWF == kWNvfp4A4 ? C::kStageBytes + C::kSfBytes
                                  : kWF == kWFp8A8   ? C::kStageBytes + (p.swap ? kBN * 4 + 16 * kMB : 512 + 16)
                                                     : (p.swap ? C::kQBytes : C::kPBytes);
      // The first stages' weight tiles do not depend on earlier kernels: issue them before
      // waiting for the previous kernel (PDL), then their activation tiles after it.
      int pre = 0;
      if (blockIdx.x < units) {
        const int split = blockIdx.x % p.splits, tile = blockIdx.x / p.splits;
        const int tp = tile % p.tiles_p, tq = tile / p.tiles_p;
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.kblocks);
        pre = min(kStages, kb1 - kb0);
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(full + i, full_bytes);
          load_w(i, kb0 + i, tp, tq);
        }
        pdl_wait();
        mark(p, 2);
        for (int i = 0; i < pre; ++i) load_a(i, kb0 + i, tp, tq);
      } else {
        pdl_wait();
      }
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int tile = u / p.splits, split = u % p.splits;
        const int tp = tile % p.tiles_p, tq = tile / p.tiles_p;
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.kblocks);
        for (int kb = kb0 + (u == (int)blockIdx.x ? pre : 0); kb < kb1; ++kb) {
          const uint32_t i2 = it + (u == (int)blockIdx.x ? pre : 0);
          const int s = i2 % kStages;
          const uint32_t ph = (i2 / kStages) & 1;
          if (!mbar_wait(empty + s, ph ^ 1, p.status, kTimeoutSmemEmpty, abort)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full + s, full_bytes);
          load_w(s, kb, tp, tq);
          load_a(s, kb, tp, tq);
          ++it;
        }
        if (u == (int)blockIdx.x) it += pre;
      }
      if (!ok) {
        // Drain: let every load issued into the ring land before the CTA exits.
        const uint32_t first = it > (uint32_t)kStages ? it - kStages : 0;
        for (uint32_t j = first; j < it; ++j)
          mbar_wait(full + (j % kStages), (j / kStages) & 1, p.status, kTimeoutDrain, nullptr);
      }
    }
  } else if (kWF == kWFp8A8 && warp == 1) {
    // ----------------------------------------------------------------- MMA issuer (W8A8)
    // One 128-input block at a time into alternating TMEM buffers: the epilogue warps scale each
    // block's sum before the blocks add.
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_e4m3_f32(128, kBN);
      uint32_t it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int split = u % p.splits;
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.kblocks);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          const int b = it % kAcc;
          const uint32_t bph = (it / kAcc) & 1;
          if (!mbar_wait(tempty + b, bph ^ 1, p.status, kTimeoutTmemEmpty, abort) ||
              !mbar_wait(full + s, ph, p.status, kTimeoutTmaFull, abort)) {
            ok = false;
            break;
          }
          if (it == 0) mark(p, 3);
          tc_fence_after();
          const uint8_t* st = smem + s * C::kStageBytes;
          const uint32_t d0 = tmem_base + b * C::kAccCols;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bdesc = sdesc_kmajor_sw128(st + C::kPBytes + kk * 32);
#pragma unroll
            for (int mb = 0; mb < kMB; ++mb)
              mma_e4m3(d0 + mb * kBN, sdesc_kmajor_sw128(st + mb * 16384 + kk * 32), bdesc, idesc,
                       kk > 0 ? 1u : 0u);
          }
          mma_commit(empty + s);
          mma_commit(tfull + b);
        }
        if (u == (int)blockIdx.x) mark(p, 4);
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc =
          kWF == kWNvfp4A4 ? idesc_nvf4_f32(128, kBN) : idesc_bf16_f32(128, kBN);
      const uint32_t sfa_t = tmem_base + C::kSfCol0;
      const uint32_t sfb_t = sfa_t + 16 * kMB;
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++tc) {
        const int split = u % p.splits;
        // A 64-row N tile reads the second half of its 128-row scale atoms when it is odd.
        const uint32_t sfb_shift = (kBN == 64 && ((u / p.splits) / p.tiles_p) % 2 == 1) ? 2u : 0u;
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.kblocks);
        const int b = tc % kAcc;
        const uint32_t aph = (tc / kAcc) & 1;
        if (!mbar_wait(tempty + b, aph ^ 1, p.status, kTimeoutTmemEmpty, abort)) break;
        tc_fence_after();
        const uint32_t d0 = tmem_base + b * C::kAccCols;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!mbar_wait(full + s, ph, p.status, kTimeoutTmaFull, abort)) {
            ok = false;
            break;
          }
          if (it == 0) mark(p, 3);
          tc_fence_after();
          const uint8_t* st = smem + s * C::kStageBytes;
          if constexpr (kWF == kWNvfp4A4) {
            // Scales into TMEM, then four K=64 block-scaled MMAs (32 bytes of each row apiece);
            // the copies and MMAs of this thread execute in issue order.
            // TMEM: A scales [mb][kk][4 columns]; B scales [kk][group][4 columns].
            const uint8_t* sf = sfr + s * C::kSfBytes;
#pragma unroll
            for (int mb = 0; mb < kMB; ++mb)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                tmem_cp_sf_atom(sfa_t + mb * 16 + kk * 4, sdesc_sf_atom(sf + mb * 2048 + kk * 512));
#pragma unroll
            for (int g = 0; g < C::kQGroups; ++g)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                tmem_cp_sf_atom(sfb_t + kk * 4 * C::kQGroups + g * 4,
                                sdesc_sf_atom(sf + (kMB + g) * 2048 + kk * 512));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t bdesc = sdesc_kmajor_sw128(st + C::kPBytes + kk * 32);
#pragma unroll
              for (int mb = 0; mb < kMB; ++mb) {
                const uint64_t adesc = sdesc_kmajor_sw128(st + mb * 16384 + kk * 32);
                mma_nvf4(d0 + mb * kBN, adesc, bdesc, idesc, sfa_t + mb * 16 + kk * 4,
                         sfb_t + kk * 4 * C::kQGroups + sfb_shift, (kb > kb0 || kk > 0) ? 1u : 0u);
              }
            }
          } else {
#pragma unroll
            for (int kk = 0; kk < kBlockK / 16; ++kk) {
              const uint64_t bdesc = sdesc_kmajor_sw128(st + C::kPBytes + kk * 32);
#pragma unroll
              for (int mb = 0; mb < kMB; ++mb) {
                const uint64_t adesc = sdesc_kmajor_sw128(st + mb * 16384 + kk * 32);
                mma_bf16(d0 + mb * kBN, adesc, bdesc, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
              }
            }
          }
          mma_commit(empty + s);
        }
        if (ok) mma_commit(tfull + b);
        if (tc == 0) mark(p, 4);
      }
    }
  } else if ((kWF == kWFp8Block || kWF == kWNvfp4) && warp >= 6) {
    // ----------------------------------------------------------------- weight converters (8 warps)
    // Expand each raw weight tile into the BF16 128-byte-swizzled layout the MMA reads: FP8 codes
    // times their 128x128 block scale (rounded once to BF16), or E2M1 codes times their E4M3
    // 16-element scale (exact in BF16; the tensor scale multiplies the FP32 sums later). A thread
    // converts items of 8 codes (rows r = its row + 32 j, column group c); each k-block's scales
    // are fetched from global memory four k-blocks ahead.
    constexpr int kConvThreads = 32 * (C::kConvWarps ? C::kConvWarps : 1);
    constexpr int kItems = C::kConvItems;  // most items a thread converts a stage
    const int ct = threadIdx.x - 192;
    const int c = ct & 7, r0 = ct >> 3;
    const int wrows_total = p.swap ? p.Mp : p.Nq;
    uint32_t it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const int tile = u / p.splits, split = u % p.splits;
      const int tp = tile % p.tiles_p, tq = tile / p.tiles_p;
      const int kb0 = split * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.kblocks);
      const int rows = p.swap ? C::kPRows : kBN;
      const int wrow0 = p.swap ? tp * C::kPRows : tq * kBN;
      // Scales of one k-block for this thread's items (FP8: float bits; NVFP4: BF16 pairs).
      auto fetch = [&](int kb, uint32_t (&sv)[C::kConvItems]) {
#pragma unroll
        for (int j = 0; j < kItems; ++j) {
          const int r = r0 + j * (kConvThreads / 8), grow = wrow0 + r;
          sv[j] = 0;
          if (r < rows && grow < wrows_total) {
            if constexpr (kWF == kWFp8Block)
              sv[j] = __float_as_uint(__ldg(static_cast<const float*>(p.wscale) +
                                            (long)(grow >> p.wscale_row_shift) * p.wscale_ld +
                                            (kb >> p.wscale_k_shift)));
            else
              sv[j] = __ldg(static_cast<const uint8_t*>(p.wscale) + (long)grow * p.wscale_ld + kb * 4 + (c >> 1));
          }
        }
      };
      // A ring of kAhead k-blocks' scales: the loads for k-block kb + kAhead go out when kb's
      // scales are used, so their latency hides behind kAhead conversions.
      constexpr int kAhead = 4;
      uint32_t sv[kAhead][kItems];
#pragma unroll
      for (int d = 0; d < kAhead; ++d)
        if (kb0 + d < kb1) fetch(kb0 + d, sv[d]);
      for (int kbb = kb0; kbb < kb1 && ok; kbb += kAhead) {
#pragma unroll
        for (int d = 0; d < kAhead; ++d) {
          const int kb = kbb + d;
          if (kb >= kb1) break;
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          int got = 1;
          if (lane == 0) got = mbar_wait(rawfull + s, ph, p.status, kTimeoutTmaFull, abort);
          got = __shfl_sync(0xffffffffu, got, 0);
          if (!got) {
            ok = false;
            break;
          }
          const uint8_t* src = raw + s * C::kRawBytes;
          uint8_t* dst = smem + s * C::kStageBytes + (p.swap ? 0 : C::kPBytes);
#pragma unroll
          for (int j = 0; j < kItems; ++j) {
            const int r = r0 + j * (kConvThreads / 8);
            if (r >= rows) break;
            uint4 out = make_uint4(0, 0, 0, 0);
            if (wrow0 + r < wrows_total) {
              if constexpr (kWF == kWFp8Block) {
                const uint2 v = *reinterpret_cast<const uint2*>(src + r * 64 + c * 8);
                out = dequant_fp8x8(v, __uint_as_float(sv[d][j]));
              } else {
                const uint32_t v = *reinterpret_cast<const uint32_t*>(src + r * 32 + c * 4);
                out = dequant_e2m1x8_permute(v, e4m3_bf16x2(static_cast<uint8_t>(sv[d][j])));
              }
            }
            *reinterpret_cast<uint4*>(dst + r * 128 + ((c ^ (r & 7)) << 4)) = out;
          }
          fence_proxy_async();  // the tile is read by the tensor cores (async proxy)
          __syncwarp();
          if (lane == 0) mbar_arrive(full + s);
          ++it;
          if (kb + kAhead < kb1) fetch(kb + kAhead, sv[d]);
        }
      }
    }
  } else {
    // ----------------------------------------------------------------- epilogue (4 warps)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int lrow = q * 32 + lane;
    pdl_wait();  // the residual and the output may be earlier kernels' memory
    uint32_t tc = 0;
    uint32_t kit = 0;  // W8A8: k-blocks consumed (stage and buffer sequence of the MMA warp)
    uint32_t xfer_count = 0;  // W8A8: hand-overs between the two scaling streams
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++tc) {
      const int tile = u / p.splits, split = u % p.splits;
      const int tp = tile % p.tiles_p, tq = tile / p.tiles_p;
      int b = tc % kAcc;
      if constexpr (kWF == kWFp8A8) {
        // Each 128-input block's FP32 sum times its combined activation and weight scale, added in
        // block order in registers by two streams of four warps that split the tile: warps 2-5
        // take the first half of the columns (or the first M block), warps 6-9 the rest. The odd
        // stream stores its half of the total into the last block's buffer and hands over; the
        // even stream then runs the epilogue below over the whole tile.
        const int stream = warp >= 6 ? 1 : 0;
        constexpr int kCnt = kMB == 2 ? kBN : kBN / 2;  // values a thread sums
        const int mb_s = kMB == 2 ? stream : 0;
        const int c_s = kMB == 2 ? 0 : stream * kCnt;
        const uint32_t col_s = mb_s * kBN + c_s;        // first TMEM column of this stream
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.kblocks);
        float acc[kCnt];
#pragma unroll
        for (int c = 0; c < kCnt; ++c) acc[c] = 0.f;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++kit) {
          const int s = kit % kStages;
          const uint32_t ph = (kit / kStages) & 1;
          b = kit % kAcc;
          const uint32_t bph = (kit / kAcc) & 1;
          int got = 1;
          if (lane == 0)
            got = mbar_wait(tfull + b, bph, p.status, kTimeoutTmemFull, abort) &&
                  mbar_wait(full + s, ph, p.status, kTimeoutTmaFull, abort);
          if (!__shfl_sync(0xffffffffu, got, 0)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // TMEM loads go out in batches with one wait each: the round trips bound this loop.
          const float* asc = reinterpret_cast<const float*>(asr + s * C::kAscBytes);
          const float sw = *reinterpret_cast<const float*>(asr + s * C::kAscBytes + C::kAscOnly +
                                                           16 * (p.swap ? mb_s : 0));
          const float srow = p.swap ? 0.f : asc[lrow] * sw;
          const uint32_t tb = tmem_base + (uint32_t(q * 32) << 16) + b * C::kAccCols + col_s;
          constexpr int kBatch = kCnt >= 32 ? 32 : kCnt;
#pragma unroll
          for (int c0 = 0; c0 < kCnt; c0 += kBatch) {
            uint32_t r[kBatch];
            if constexpr (kBatch == 32)
              tmem_ld_32x32b_x32(tb + c0, *reinterpret_cast<uint32_t(*)[32]>(r));
            else
              tmem_ld_32x32b_x16(tb + c0, *reinterpret_cast<uint32_t(*)[16]>(r));
            float sc[kBatch];
            if (p.swap) {
#pragma unroll
              for (int t = 0; t < kBatch; t += 4) {
                const float4 a4 = *reinterpret_cast<const float4*>(asc + c_s + c0 + t);
                sc[t] = a4.x * sw;
                sc[t + 1] = a4.y * sw;
                sc[t + 2] = a4.z * sw;
                sc[t + 3] = a4.w * sw;
              }
            } else {
#pragma unroll
              for (int t = 0; t < kBatch; ++t) sc[t] = srow;
            }
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < kBatch; ++t) acc[c0 + t] = fmaf(__uint_as_float(r[t]), sc[t], acc[c0 + t]);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(empty + s);
          if (kb + 1 < kb1) {
            tc_fence_before();
            mbar_arrive(tempty + b);
          }
        }
        if (!ok) break;
#pragma unroll
        for (int c0 = 0; c0 < kCnt; c0 += 16) {
          uint32_t r[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) r[t] = __float_as_uint(acc[c0 + t]);
          tmem_st_32x32b_x16(tmem_base + (uint32_t(q * 32) << 16) + b * C::kAccCols + col_s + c0, r);
        }
        tmem_st_wait();
        tc_fence_before();
        const uint32_t xph = xfer_count & 1;
        ++xfer_count;
        if (stream == 1) {
          // Hand over, release the buffer (the even stream releases it too), and wait until the
          // hand-over was taken so that the two barriers never run a phase ahead.
          mbar_arrive(xfer);
          mbar_arrive(tempty + b);
          int taken = 1;
          if (lane == 0) taken = mbar_wait(xfer + 1, xph, p.status, kTimeoutTmemFull, abort);
          if (!__shfl_sync(0xffffffffu, taken, 0)) break;
          continue;
        }
        int ready = 1;
        if (lane == 0) ready = mbar_wait(xfer, xph, p.status, kTimeoutTmemFull, abort);
        if (!__shfl_sync(0xffffffffu, ready, 0)) break;
        mbar_arrive(xfer + 1);
      } else {
        const uint32_t aph = (tc / kAcc) & 1;
        if (!mbar_wait(tfull + b, aph, p.status, kTimeoutTmemFull, abort)) break;
      }
      if (tc == 0 && lrow == 0) mark(p, 5);
      tc_fence_after();
      const uint32_t tbase = tmem_base + (uint32_t(q * 32) << 16) + b * C::kAccCols;

      auto tmem16 = [&](int mb, int c0, float (&v)[16]) {
        uint32_t r[16];
        if (p.debug & 2) {
#pragma unroll
          for (int t = 0; t < 16; ++t) r[t] = 0;
        } else {
          tmem_ld_32x32b_x16(tbase + mb * kBN + c0, r);
          tmem_ld_wait();
        }
#pragma unroll
        for (int t = 0; t < 16; ++t)
          v[t] = (kWF == kWNvfp4 || kWF == kWNvfp4A4) ? __uint_as_float(r[t]) * p.acc_scale
                                                       : __uint_as_float(r[t]);
      };
      // Partials are stored column-major ([col][row]) so a warp's 32 rows are 128 contiguous bytes.
      const long tile_elems = (long)C::kPRows * kBN;
      auto ws_at = [&](int s, int mb, int c) {
        return p.ws + ((long)tile * p.splits + s) * tile_elems + (long)c * C::kPRows + mb * 128 + lrow;
      };
      if (kRed == kRedCluster) continue;  // pushed after the cluster barrier below
      bool from_ws = false;
      if (kRed == kRedGlobal && p.splits > 1 && p.external) {
        // The next kernel adds the splits: store this split's partial and take the next unit.
#pragma unroll 1
        for (int mb = 0; mb < kMB; ++mb)
          for (int c0 = 0; c0 < kBN; c0 += 16) {
            float v[16];
            tmem16(mb, c0, v);
#pragma unroll
            for (int t = 0; t < 16; ++t) __stcg(ws_at(split, mb, c0 + t), v[t]);
          }
        tc_fence_before();
        mbar_arrive(tempty + b);
        continue;
      }
      if (kRed == kRedGlobal && p.splits > 1) {
        for (int mb = 0; mb < kMB; ++mb)
          for (int c0 = 0; c0 < kBN; c0 += 16) {
            float v[16];
            tmem16(mb, c0, v);
#pragma unroll
            for (int t = 0; t < 16; ++t) __stcg(ws_at(split, mb, c0 + t), v[t]);
          }
        tc_fence_before();
        mbar_arrive(tempty + b);
        __threadfence();
        epi_barrier();
        if (lrow == 0) {
          const int old = atomicAdd(p.counters + tile, 1);
          const int last = (old == p.splits - 1);
          if (last) p.counters[tile] = 0;
          *last_flag = last;
        }
        epi_barrier();
        if (!*last_flag) continue;
        __threadfence();
        from_ws = true;
      }
      auto get16 = [&](int mb, int c0, float (&v)[16]) {
        if (!from_ws) {
          tmem16(mb, c0, v);
          return;
        }
#pragma unroll
        for (int t = 0; t < 16; ++t) v[t] = 0.f;
        for (int s = 0; s < p.splits; ++s) {
          float x[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) x[t] = __ldcg(ws_at(s, mb, c0 + t));
#pragma unroll
          for (int t = 0; t < 16; ++t) v[t] += x[t];
        }
      };

      // Rows mapping, output through this warp's staging box (32 rows of 128 bytes: 64 BF16 or 32
      // FP32 values) and a TMA store: the thread of row r writes its values as 16-byte chunks into
      // the 128-byte-swizzled box; `flush` stores the box at output column x, and `reuse` waits
      // until the previous box has been read before the box is written again.
      uint8_t* box = outst + (size_t)q * 4096;
      auto reuse = [&]() {
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
      };
      auto stage16 = [&](int c1, const uint32_t (&w)[8]) {
        const int ch = c1 / 8;
        *reinterpret_cast<uint4*>(box + lane * 128 + (((ch) ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(box + lane * 128 + (((ch + 1) ^ (lane & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
      };
      auto flush = [&](int x) {
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&aux.c, box, x, tp * C::kPRows + q * 32);
          bulk_commit();
        }
      };
      const bool staged = C::kOutStage > 0 && p.tma_store && !p.swap && !(p.debug & 1);
      if (kEpi == kEpiSwiGLU && staged) {
        // Rows mapping: the tile's first kBN/2 columns are gate rows, the rest up rows.
        for (int c0 = 0; c0 < kBN / 2; c0 += 64) {
          reuse();
#pragma unroll
          for (int c1 = 0; c1 < 64; c1 += 16) {
            float g[16], v[16];
            get16(0, c0 + c1, g);
            get16(0, c0 + c1 + kBN / 2, v);
            uint32_t w[8];
#pragma unroll
            for (int t = 0; t < 8; ++t)
              w[t] = pack_bf16x2(silu_bf16_times(g[2 * t], v[2 * t]), silu_bf16_times(g[2 * t + 1], v[2 * t + 1]));
            stage16(c1, w);
          }
          flush(tq * (kBN / 2) + c0);
        }
      } else if (kEpi == kEpiF32 && staged && kMB == 1 && kBN % 32 == 0) {
        // Rows mapping, FP32 output (a tensor-parallel partial): 32 x 32 boxes of 128-byte rows.
        for (int c0 = 0; c0 < kBN; c0 += 32) {
          reuse();
#pragma unroll
          for (int c1 = 0; c1 < 32; c1 += 16) {
            float v[16];
            get16(0, c0 + c1, v);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const int ch = c1 / 4 + t;
              *reinterpret_cast<float4*>(box + lane * 128 + ((ch ^ (lane & 7)) << 4)) =
                  make_float4(v[4 * t], v[4 * t + 1], v[4 * t + 2], v[4 * t + 3]);
            }
          }
          flush(tq * kBN + c0);
        }
      } else if (kEpi == kEpiBf16 && staged && kMB == 1 && kBN % 64 == 0 &&
                 (p.res == nullptr ||
                  ((tq + 1) * kBN <= p.out_cols && (reinterpret_cast<uintptr_t>(p.res) & 15) == 0 && (p.ldr & 7) == 0))) {
        // Rows mapping, BF16 output (o_proj and down_proj at one chip add the residual: 64 of its
        // columns load with eight 16-byte loads in flight before the accumulator columns are read).
        const int i = tp * C::kPRows + lrow;
        const bool in = i < p.out_rows;
        for (int c0 = 0; c0 < kBN; c0 += 64) {
          const int j0 = tq * kBN + c0;
          uint4 rr[8];
          if (p.res != nullptr) {
            const uint4* rsrc = reinterpret_cast<const uint4*>(p.res + (long)i * p.ldr + j0);
#pragma unroll
            for (int qq = 0; qq < 8; ++qq) rr[qq] = in ? __ldcs(rsrc + qq) : make_uint4(0, 0, 0, 0);
          } else {
#pragma unroll
            for (int qq = 0; qq < 8; ++qq) rr[qq] = make_uint4(0, 0, 0, 0);
          }
          reuse();
#pragma unroll
          for (int c1 = 0; c1 < 64; c1 += 16) {
            float v[16];
            get16(0, c0 + c1, v);
            const uint32_t rw[8] = {rr[c1 / 8].x, rr[c1 / 8].y, rr[c1 / 8].z, rr[c1 / 8].w,
                                    rr[c1 / 8 + 1].x, rr[c1 / 8 + 1].y, rr[c1 / 8 + 1].z, rr[c1 / 8 + 1].w};
            uint32_t w[8];
#pragma unroll
            for (int t = 0; t < 8; ++t)
              w[t] = pack_bf16x2(v[2 * t] + __uint_as_float(rw[t] << 16), v[2 * t + 1] + __uint_as_float(rw[t] & 0xFFFF0000u));
            stage16(c1, w);
          }
          flush(j0);
        }
      } else if (kEpi == kEpiSwiGLU) {
        if (!p.swap) {
          // Rows mapping: the tile's first kBN/2 columns are gate rows, the rest up rows.
          const int row = tp * C::kPRows + lrow;
          for (int c0 = 0; c0 < kBN / 2; c0 += 16) {
            float g[16], v[16];
            get16(0, c0, g);
            get16(0, c0 + kBN / 2, v);
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = silu_bf16_times(g[t], v[t]);
            store16<kEpiBf16>(p, row, tq * (kBN / 2) + c0, v, true);
          }
        } else {
          // Swap mapping: M block 0 holds gate rows, block 1 the up rows of the same features.
          const int feature = tp * 128 + lrow;
          for (int c0 = 0; c0 < kBN; c0 += 16) {
            float g[16], v[16];
            get16(0, c0, g);
            get16(1, c0, v);
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = silu_bf16_times(g[t], v[t]);
            store16<kEpiBf16>(p, tq * kBN + c0, feature, v, false);
          }
        }
      } else if (kEpi == kEpiBf16 && kMB == 1 && kBN % 64 == 0 && !p.swap && p.res != nullptr &&
                 (tq + 1) * kBN <= p.out_cols &&
                 ((reinterpret_cast<uintptr_t>(p.res) | reinterpret_cast<uintptr_t>(p.c)) & 15) == 0 &&
                 ((p.ldr | p.ldc) & 7) == 0) {
        // Rows mapping with a residual (o_proj, down_proj at one chip): each thread owns one output
        // row; the residual of 64 columns is loaded with eight 16-byte loads in flight before the
        // accumulator columns are read, so the tile pays the load latency once per 64 columns.
        const int i = tp * C::kPRows + lrow;
        const bool in = i < p.out_rows;
        for (int c0 = 0; c0 < kBN; c0 += 64) {
          const int j0 = tq * kBN + c0;
          uint4 rr[8];
          const uint4* rsrc = reinterpret_cast<const uint4*>(p.res + (long)i * p.ldr + j0);
#pragma unroll
          for (int q = 0; q < 8; ++q) rr[q] = in ? __ldcs(rsrc + q) : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int c1 = 0; c1 < 64; c1 += 16) {
            float v[16];
            get16(0, c0 + c1, v);
            const uint32_t rw[8] = {rr[c1 / 8].x, rr[c1 / 8].y, rr[c1 / 8].z, rr[c1 / 8].w,
                                    rr[c1 / 8 + 1].x, rr[c1 / 8 + 1].y, rr[c1 / 8 + 1].z, rr[c1 / 8 + 1].w};
            uint32_t out[8];
#pragma unroll
            for (int t = 0; t < 8; ++t)
              out[t] = pack_bf16x2(v[2 * t] + __uint_as_float(rw[t] << 16), v[2 * t + 1] + __uint_as_float(rw[t] & 0xFFFF0000u));
            if (in && !(p.debug & 1)) {
              uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.c) + (long)i * p.ldc + j0 + c1);
              dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
              dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
            }
          }
        }
      } else {
        for (int mb = 0; mb < kMB; ++mb) {
          const int i = tp * C::kPRows + mb * 128 + lrow;
          for (int c0 = 0; c0 < kBN; c0 += 16) {
            float v[16];
            get16(mb, c0, v);
            const int j = tq * kBN + c0;
            if (!p.swap)
              store16<kEpi>(p, i, j, v, true);
            else
              store16<kEpi>(p, j, i, v, false);
          }
        }
      }
      if (!from_ws) {
        tc_fence_before();
        mbar_arrive(tempty + b);
      }
    }
    if (lane == 0) bulk_wait_all();  // the output boxes stored by TMA have landed
    if (lrow == 0) mark(p, 6);
  }

  if (kRed == kRedCluster) {
    // 1. Every CTA of the cluster has drained its MMAs (its epilogue saw the accumulator
    //    complete), so every operand ring is idle and may receive partials.
    cluster_sync();
    if (p.cta_trace != nullptr && threadIdx.x == 64) p.cta_trace[8 * blockIdx.x + 3] = global_ns();
    // 2. Push this split's partial into the shared memory of the CTA that reduces each row;
    //    DSMEM stores do not stall. Receive layout per CTA: [split][half][col][row of slice].
    if (warp >= 2 && warp < 6 && !*abort) {
      const int q = warp & 3;
      const int lrow = q * 32 + lane;
      const int S = p.splits;
      const int split = blockIdx.x % S;
      // One unit per CTA here: its accumulator is buffer 0, or (W8A8) its last k-block's buffer.
      int bsel = 0;
      if constexpr (kWF == kWFp8A8) {
        const int kb0 = split * p.kb_per_split;
        bsel = (min(kb0 + p.kb_per_split, p.kblocks) - kb0 - 1) % kAcc;
      }
      const uint32_t tbase = tmem_base + (uint32_t(q * 32) << 16) + bsel * C::kAccCols;
      const uint32_t red = smem_u32(smem);
      for (int mb = 0; mb < kMB; ++mb) {
        int owner, rl, rs, half;
        if (kEpi == kEpiSwiGLU) {
          rs = slice_rows(128, S);
          owner = lrow / rs;
          rl = lrow % rs;
          half = mb;
        } else {
          rs = slice_rows(C::kPRows, S);
          const int r = mb * 128 + lrow;
          owner = r / rs;
          rl = r % rs;
          half = 0;
        }
        const int halves = kEpi == kEpiSwiGLU ? 2 : 1;
        const uint32_t base =
            dsmem_addr(red, owner) + 4u * (uint32_t)(((split * halves + half) * kBN) * rs + rl);
        for (int c0 = 0; c0 < kBN; c0 += 16) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(tbase + mb * kBN + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 16; ++t)
            dsmem_st_f32(base + 4u * (uint32_t)((c0 + t) * rs),
                         (kWF == kWNvfp4 || kWF == kWNvfp4A4) ? __uint_as_float(r[t]) * p.acc_scale
                                                              : __uint_as_float(r[t]));
        }
      }
      tc_fence_before();
    }
    if (p.cta_trace != nullptr && threadIdx.x == 64) p.cta_trace[8 * blockIdx.x + 4] = global_ns();
    // 3. Every partial has landed; each CTA adds its slice in split order.
    cluster_sync();
    if (p.cta_trace != nullptr && threadIdx.x == 64) p.cta_trace[8 * blockIdx.x + 5] = global_ns();
    if (warp >= 2 && warp < 6) {
      const int tid = threadIdx.x - 64;
      const int S = p.splits;
      const int rank = (int)cluster_rank();
      const int tile = blockIdx.x / S;
      const int tp = tile % p.tiles_p, tq = tile / p.tiles_p;
      const float* red = reinterpret_cast<const float*>(smem);
      // Each thread adds 8 consecutive rows of the slice (output features) of one column (token)
      // over the splits in split order; consecutive threads take consecutive groups of 8.
      const int rows_here = kEpi == kEpiSwiGLU ? 128 : C::kPRows;
      const int rs = slice_rows(rows_here, S);
      const int r0 = rank * rs;
      const int groups = max(0, min(rs, rows_here - r0)) / 8;
        for (int e = tid; e < groups * kBN; e += 128) {
        const int g = e % groups, c = e / groups;
        if (kEpi == kEpiSwiGLU) {
          float gs[8], us[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) gs[t] = us[t] = 0.f;
          for (int sp = 0; sp < S; ++sp) {
            const float4* gq = reinterpret_cast<const float4*>(red + ((sp * 2 + 0) * kBN + c) * rs + g * 8);
            const float4* uq = reinterpret_cast<const float4*>(red + ((sp * 2 + 1) * kBN + c) * rs + g * 8);
            const float4 g0 = gq[0], g1 = gq[1], u0 = uq[0], u1 = uq[1];
            gs[0] += g0.x; gs[1] += g0.y; gs[2] += g0.z; gs[3] += g0.w;
            gs[4] += g1.x; gs[5] += g1.y; gs[6] += g1.z; gs[7] += g1.w;
            us[0] += u0.x; us[1] += u0.y; us[2] += u0.z; us[3] += u0.w;
            us[4] += u1.x; us[5] += u1.y; us[6] += u1.z; us[7] += u1.w;
          }
          float o[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) o[t] = silu_bf16_times(gs[t], us[t]);
          store8<kEpiBf16>(p, tq * kBN + c, tp * 128 + r0 + g * 8, o);
        } else {
          float v[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) v[t] = 0.f;
          for (int sp = 0; sp < S; ++sp) {
            const float4* q4 = reinterpret_cast<const float4*>(red + (sp * kBN + c) * rs + g * 8);
            const float4 x0 = q4[0], x1 = q4[1];
            v[0] += x0.x; v[1] += x0.y; v[2] += x0.z; v[3] += x0.w;
            v[4] += x1.x; v[5] += x1.y; v[6] += x1.z; v[7] += x1.w;
          }
          store8<kEpi>(p, tq * kBN + c, tp * C::kPRows + r0 + g * 8, v);
        }
      }
    }
    if (p.cta_trace != nullptr && threadIdx.x == 64) p.cta_trace[8 * blockIdx.x + 6] = global_ns();
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
    if (lane == 0) mark(p, 7);
  }
  if (p.cta_trace != nullptr) {
    __syncthreads();
    if (threadIdx.x == 0) p.cta_trace[8 * blockIdx.x + 7] = global_ns();
  }
}

// ------------------------------------------------------------------------------------ host side

int g_num_sms[64] = {0};

int device_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (g_num_sms[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_num_sms[dev] = n > 0 ? n : 148;
  }
  return g_num_sms[dev];
}

struct Plan {
  int swap, kbn, mb, red;
  int tiles_p, tiles_q, splits, kb_per_split, kblocks, units, grid;
};

int pick_swap_bn(int m) {
  if (m <= 16) return 16;
  if (m <= 32) return 32;
  if (m <= 64) return 64;
  if (m <= 128) return 128;
  return 256;
}

// Shared-memory bytes of the operand ring of a swap-mapping configuration (see launch_swap).
// Pipeline shape of a (tile, weight format): as many stages as fit 220 KiB of shared memory (at
// most 8), and double-buffered accumulators when two fit in TMEM.
template <int kMB, int kBN, int kWF>
struct Shape {
  static constexpr int kStage = 128 * kMB * 128 + kBN * 128;
  static constexpr int kRaw = (kMB * 128 > kBN ? kMB * 128 : kBN) * (kWF == 1 ? 64 : kWF == 2 ? 32 : 0);
  static constexpr int kSfGroups = kWF == 3 ? kMB + (kBN + 127) / 128 : 0;
  static constexpr int kAsc = kWF == 4 ? 4 * (kBN > 128 ? kBN : 128) + 16 * kMB : 0;
  static constexpr int kOut = (kWF == 0 && kMB == 1) ? 4 * 4096 : 0;  // output staging (Cfg::kOutStage)
  static constexpr int kFit = (220 * 1024 - 2048 - kOut) / (kStage + kRaw + kSfGroups * 2048 + kAsc);
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  // W8A8 keeps up to eight per-block partial sums in flight so the MMAs run ahead of the scaling.
  static constexpr int kAccW8 = 512 / (kMB * kBN) > 8 ? 8 : 512 / (kMB * kBN);
  static constexpr int kAcc = kWF == 4 ? kAccW8 : kMB * kBN * 2 + 16 * kSfGroups <= 512 ? 2 : 1;
};

// Bytes of the operand ring of a swap-mapping configuration (the cluster reduction reuses it).
int swap_ring_bytes(int mb, int kbn, int wf) {
  const int stage = 128 * mb * 128 + kbn * 128;
  const int raw = (mb * 128 > kbn ? mb * 128 : kbn) * (wf == 1 ? 64 : wf == 2 ? 32 : 0);
  const int sf = wf == 3 ? (mb + (kbn + 127) / 128) * 2048 : wf == 4 ? 4 * std::max(kbn, 128) + 16 * mb : 0;
  const int out = (wf == 0 && mb == 1) ? 4 * 4096 : 0;
  int stages = (220 * 1024 - 2048 - out) / (stage + raw + sf);
  if (stages > 8) stages = 8;
  return stage * stages;
}

using ClusterLimit = int (*)(int mb, int kbn, int epilogue, int size);
int cluster_limit_of(int mb, int kbn, int epi, int size);

Plan make_plan(const GemmArgs& a, int num_sms, size_t ws_bytes, int counters_len,
               ClusterLimit cluster_limit = cluster_limit_of) {
  Plan pl{};
  // W8A8 SwiGLU runs on the swap mapping at every row count (its rows tiles hold 128 columns).
  const bool swap = a.mode == kModeSwap || (a.mode == kModeAuto && a.M <= 256) ||
                    (a.w_format == kWFp8A8 && a.epilogue == kEpiSwiGLU) || a.group_tiles != nullptr;
  pl.swap = swap;
  const int kelems = a.w_format == kWNvfp4A4 ? 256 : a.w_format == kWFp8A8 ? 128 : kBlockK;
  pl.kblocks = (a.K + kelems - 1) / kelems + a.seg[0].K / kBlockK + a.seg[1].K / kBlockK;
  if (!swap) {
    pl.mb = 1;
    pl.kbn = a.w_format == kWFp8A8 ? 128 : 256;  // W8A8 sums a tile row in registers
    // (128-column BF16 tiles against wave quantization measured slower: down_proj of 8192 rows
    // 183 -> 214 us.)

    pl.tiles_p = (a.M + 127) / 128;
    pl.tiles_q = (a.N + pl.kbn - 1) / pl.kbn;
  } else {
    pl.mb = a.epilogue == kEpiSwiGLU ? 2 : 1;
    pl.kbn = pick_swap_bn(a.M);
    if (a.w_format == kWNvfp4A4) {
      // Block-scaled N tiles read whole 64-row halves of a scale atom; two M blocks and their
      // scales leave TMEM room for N <= 128.
      pl.kbn = std::max(pl.kbn, 64);
      if (pl.mb == 2) pl.kbn = std::min(pl.kbn, 128);
    }
    if (a.w_format == kWFp8A8) pl.kbn = std::max(32, std::min(pl.kbn, pl.mb == 2 ? 64 : 128));
    if (a.group_tiles != nullptr) {
      pl.kbn = a.group_tile;
      pl.tiles_q = (a.M + pl.kbn - 1) / pl.kbn;
    }
    pl.tiles_p = (a.N + 128 * pl.mb - 1) / (128 * pl.mb);
    pl.tiles_q = (a.M + pl.kbn - 1) / pl.kbn;
  }
  const int tiles = pl.tiles_p * pl.tiles_q;
  int splits = a.group_tiles != nullptr ? 1 : a.splits;
  if (splits <= 0) {
    splits = 1;
    if (tiles * 2 <= num_sms) splits = std::min(8, num_sms / tiles);
    splits = std::min(splits, std::max(1, pl.kblocks / 2));
  }
  splits = std::max(1, std::min(splits, pl.kblocks));
  const size_t red_bytes = (size_t)128 * pl.mb * pl.kbn * sizeof(float);
  // The cluster reduction receives every split's slice rows (slice_rows on the device).
  const int slice = ((128 + splits - 1) / splits + 7) & ~7;
  const size_t recv_bytes = (size_t)splits * slice * pl.mb * pl.kbn * sizeof(float);
  const bool cluster_fits =
      pl.swap && splits <= 8 && (int)recv_bytes <= swap_ring_bytes(pl.mb, pl.kbn, a.w_format);
  pl.red = splits == 1 ? 0 : cluster_fits ? 2 : 1;
  // A measurement may ask how the splits meet (1 global scratch, 2 cluster).
  if (a.reduction == 1 && splits > 1) pl.red = 1;
  if (a.reduction == 2 && splits > 1 && cluster_fits) pl.red = 2;
  if (pl.red == 1) {
    // Global scratch bounds the split count.
    while (splits > 1 && ((size_t)tiles * splits * red_bytes > ws_bytes || tiles > counters_len))
      --splits;
    if (splits == 1) pl.red = 0;
  }
  pl.kb_per_split = (pl.kblocks + splits - 1) / splits;
  pl.splits = (pl.kblocks + pl.kb_per_split - 1) / pl.kb_per_split;
  if (pl.splits == 1) pl.red = 0;
  if (pl.red == 2 && cluster_limit != nullptr) {
    // All clusters must be resident in one wave: shrink the split count until they are.
    while (pl.splits > 1 && tiles > cluster_limit(pl.mb, pl.kbn, a.epilogue, pl.splits)) {
      const int want = pl.splits - 1;
      pl.kb_per_split = (pl.kblocks + want - 1) / want;
      pl.splits = (pl.kblocks + pl.kb_per_split - 1) / pl.kb_per_split;
    }
    if (pl.splits == 1) pl.red = 0;
  }
  pl.units = tiles * pl.splits;
  pl.grid = pl.red == 2 ? pl.units : std::min(pl.units, num_sms);
  return pl;
}

template <int kMB, int kBN, int kEpi, int kRed, int kWF>
int launch(const CUtensorMap& tp, const CUtensorMap& tq, const AuxMaps& tw, const KParams& kp,
           const Plan& pl, cudaStream_t stream) {
  using S = Shape<kMB, kBN, kWF>;
  using C = Cfg<kMB, kBN, S::kStages, S::kAcc, kWF>;
  auto kernel = gemm_bf16_kernel<kMB, kBN, S::kStages, S::kAcc, kEpi, kRed, kWF>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    configured[dev & 63] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(C::kThreadsCta);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (kRed == kRedCluster) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = pl.splits;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, tp, tq, tw, kp);
  return err == cudaSuccess ? 0 : -5;
}

// Clusters of `size` CTAs of this configuration that the device holds at once (cached).
template <int kMB, int kBN, int kEpi, int kWF>
int max_active_clusters(int size) {
  using S = Shape<kMB, kBN, kWF>;
  using C = Cfg<kMB, kBN, S::kStages, S::kAcc, kWF>;
  static int cache[64][9] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  int& slot = cache[dev & 63][size];
  if (slot == 0) {
    auto kernel = gemm_bf16_kernel<kMB, kBN, S::kStages, S::kAcc, kEpi, kRedCluster, kWF>;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(size * 64);
    cfg.blockDim = dim3(C::kThreadsCta);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148 / size;
    }
    slot = n;
  }
  return slot;
}

template <int kMB, int kBN, int kEpi, int kWF>
int launch_red(const CUtensorMap& tp, const CUtensorMap& tq, const AuxMaps& tw,
               const KParams& kp, const Plan& pl, cudaStream_t stream) {
  switch (pl.red) {
    case kRedNone:
      return launch<kMB, kBN, kEpi, kRedNone, kWF>(tp, tq, tw, kp, pl, stream);
    case kRedGlobal:
      return launch<kMB, kBN, kEpi, kRedGlobal, kWF>(tp, tq, tw, kp, pl, stream);
    default:
      if constexpr (kMB * kBN * 128 * 4 <= 232448 - 2048)
        return launch<kMB, kBN, kEpi, kRedCluster, kWF>(tp, tq, tw, kp, pl, stream);
      return -2;
  }
}

template <int kMB, int kBN, int kWF>
int launch_plain_epi(int epi, const CUtensorMap& tp, const CUtensorMap& tq, const AuxMaps& tw,
                     const KParams& kp, const Plan& pl, cudaStream_t stream) {
  if (epi == kEpiBf16) return launch_red<kMB, kBN, kEpiBf16, kWF>(tp, tq, tw, kp, pl, stream);
  if (epi == kEpiF32) return launch_red<kMB, kBN, kEpiF32, kWF>(tp, tq, tw, kp, pl, stream);
  return -2;
}

template <int kWF>
int launch_swap(int epi, const CUtensorMap& tp, const CUtensorMap& tq, const AuxMaps& tw,
                const KParams& kp, const Plan& pl, cudaStream_t stream) {
  if (pl.mb == 2) {
    if (epi != kEpiSwiGLU) return -2;
    switch (pl.kbn) {
      case 16: return launch_red<2, 16, kEpiSwiGLU, kWF>(tp, tq, tw, kp, pl, stream);
      case 32: return launch_red<2, 32, kEpiSwiGLU, kWF>(tp, tq, tw, kp, pl, stream);
      case 64: return launch_red<2, 64, kEpiSwiGLU, kWF>(tp, tq, tw, kp, pl, stream);
      case 128: return launch_red<2, 128, kEpiSwiGLU, kWF>(tp, tq, tw, kp, pl, stream);
      default: return launch_red<2, 256, kEpiSwiGLU, kWF>(tp, tq, tw, kp, pl, stream);
    }
  }
  switch (pl.kbn) {
    case 16: return launch_plain_epi<1, 16, kWF>(epi, tp, tq, tw, kp, pl, stream);
    case 32: return launch_plain_epi<1, 32, kWF>(epi, tp, tq, tw, kp, pl, stream);
    case 64: return launch_plain_epi<1, 64, kWF>(epi, tp, tq, tw, kp, pl, stream);
    case 128: return launch_plain_epi<1, 128, kWF>(epi, tp, tq, tw, kp, pl, stream);
    default: return launch_plain_epi<1, 256, kWF>(epi, tp, tq, tw, kp, pl, stream);
  }
}

// Block-scaled NVFP4 configurations: swap N tiles of 64/128/256 (two M blocks: 64/128).
int launch_swap_nvf4(int epi, const CUtensorMap& tp, const CUtensorMap& tq, const AuxMaps& tw,
                     const KParams& kp, const Plan& pl, cudaStream_t stream) {
  constexpr int W = kWNvfp4A4;
  if (pl.mb == 2) {
    if (epi != kEpiSwiGLU) return -2;
    return pl.kbn == 64 ? launch_red<2, 64, kEpiSwiGLU, W>(tp, tq, tw, kp, pl, stream)
                        : launch_red<2, 128, kEpiSwiGLU, W>(tp, tq, tw, kp, pl, stream);
  }
  switch (pl.kbn) {
    case 64: return launch_plain_epi<1, 64, W>(epi, tp, tq, tw, kp, pl, stream);
    case 128: return launch_plain_epi<1, 128, W>(epi, tp, tq, tw, kp, pl, stream);
    default: return launch_plain_epi<1, 256, W>(epi, tp, tq, tw, kp, pl, stream);
  }
}

// W8A8 configurations: swap N tiles of 32..128 (two M blocks: up to 64), rows 128 x 128.
int launch_swap_fp8(int epi, const CUtensorMap& tp, const CUtensorMap& tq, const AuxMaps& tw,
                    const KParams& kp, const Plan& pl, cudaStream_t stream) {
  constexpr int W = kWFp8A8;
  if (pl.mb == 2) {
    if (epi != kEpiSwiGLU) return -2;
    switch (pl.kbn) {
      case 32: return launch_red<2, 32, kEpiSwiGLU, W>(tp, tq, tw, kp, pl, stream);
      default: return launch_red<2, 64, kEpiSwiGLU, W>(tp, tq, tw, kp, pl, stream);
    }
  }
  switch (pl.kbn) {
    case 32: return launch_plain_epi<1, 32, W>(epi, tp, tq, tw, kp, pl, stream);
    case 64: return launch_plain_epi<1, 64, W>(epi, tp, tq, tw, kp, pl, stream);
    default: return launch_plain_epi<1, 128, W>(epi, tp, tq, tw, kp, pl, stream);
  }
}

int cluster_limit_fp8(int mb, int kbn, int epi, int size) {
  constexpr int W = kWFp8A8;
  if (mb == 2) {
    switch (kbn) {
      case 32: return max_active_clusters<2, 32, kEpiSwiGLU, W>(size);
      default: return max_active_clusters<2, 64, kEpiSwiGLU, W>(size);
    }
  }
  const bool f32 = epi == kEpiF32;
  switch (kbn) {
    case 32: return f32 ? max_active_clusters<1, 32, kEpiF32, W>(size) : max_active_clusters<1, 32, kEpiBf16, W>(size);
    case 64: return f32 ? max_active_clusters<1, 64, kEpiF32, W>(size) : max_active_clusters<1, 64, kEpiBf16, W>(size);
    default: return f32 ? max_active_clusters<1, 128, kEpiF32, W>(size) : max_active_clusters<1, 128, kEpiBf16, W>(size);
  }
}

int cluster_limit_nvf4(int mb, int kbn, int epi, int size) {
  constexpr int W = kWNvfp4A4;
  if (mb == 2)
    return kbn == 64 ? max_active_clusters<2, 64, kEpiSwiGLU, W>(size)
                     : max_active_clusters<2, 128, kEpiSwiGLU, W>(size);
  const bool f32 = epi == kEpiF32;
  switch (kbn) {
    case 64: return f32 ? max_active_clusters<1, 64, kEpiF32, W>(size) : max_active_clusters<1, 64, kEpiBf16, W>(size);
    case 128: return f32 ? max_active_clusters<1, 128, kEpiF32, W>(size) : max_active_clusters<1, 128, kEpiBf16, W>(size);
    default: return f32 ? max_active_clusters<1, 256, kEpiF32, W>(size) : max_active_clusters<1, 256, kEpiBf16, W>(size);
  }
}

template <int kWF>
int launch_rows(int epi, const CUtensorMap& tp, const CUtensorMap& tq, const AuxMaps& tw,
                const KParams& kp, const Plan& pl, cudaStream_t stream) {
  switch (epi) {
    case kEpiBf16: return launch_red<1, 256, kEpiBf16, kWF>(tp, tq, tw, kp, pl, stream);
    case kEpiF32: return launch_red<1, 256, kEpiF32, kWF>(tp, tq, tw, kp, pl, stream);
    case kEpiSwiGLU: return launch_red<1, 256, kEpiSwiGLU, kWF>(tp, tq, tw, kp, pl, stream);
  }
  return -2;
}

template <int kWF>
int cluster_limit_wf(int mb, int kbn, int epi, int size) {
  if (mb == 2) {
    switch (kbn) {
      case 16: return max_active_clusters<2, 16, kEpiSwiGLU, kWF>(size);
      case 32: return max_active_clusters<2, 32, kEpiSwiGLU, kWF>(size);
      case 64: return max_active_clusters<2, 64, kEpiSwiGLU, kWF>(size);
      default: return max_active_clusters<2, 128, kEpiSwiGLU, kWF>(size);
    }
  }
  const bool f32 = epi == kEpiF32;
  switch (kbn) {
    case 16: return f32 ? max_active_clusters<1, 16, kEpiF32, kWF>(size) : max_active_clusters<1, 16, kEpiBf16, kWF>(size);
    case 32: return f32 ? max_active_clusters<1, 32, kEpiF32, kWF>(size) : max_active_clusters<1, 32, kEpiBf16, kWF>(size);
    case 64: return f32 ? max_active_clusters<1, 64, kEpiF32, kWF>(size) : max_active_clusters<1, 64, kEpiBf16, kWF>(size);
    case 128: return f32 ? max_active_clusters<1, 128, kEpiF32, kWF>(size) : max_active_clusters<1, 128, kEpiBf16, kWF>(size);
    default: return f32 ? max_active_clusters<1, 256, kEpiF32, kWF>(size) : max_active_clusters<1, 256, kEpiBf16, kWF>(size);
  }
}

int g_cluster_wf = 0;  // weight format of the plan being made (read by cluster_limit_of)

int cluster_limit_of(int mb, int kbn, int epi, int size) {
  switch (g_cluster_wf) {
    case kWFp8Block: return cluster_limit_wf<kWFp8Block>(mb, kbn, epi, size);
    case kWNvfp4: return cluster_limit_wf<kWNvfp4>(mb, kbn, epi, size);
    case kWNvfp4A4: return cluster_limit_nvf4(mb, kbn, epi, size);
    case kWFp8A8: return cluster_limit_fp8(mb, kbn, epi, size);
    default: return cluster_limit_wf<kWBf16>(mb, kbn, epi, size);
  }
}

}  // namespace

void gemm_bf16_scratch(const GemmArgs& args, size_t* workspace_bytes, int* counters) {
  const int sms = args.num_sms > 0 ? args.num_sms : device_sms();
  Plan pl = make_plan(args, sms, ~size_t(0) >> 1, 1 << 30, nullptr);
  const bool global = pl.red == 1;
  *workspace_bytes =
      global ? (size_t)pl.tiles_p * pl.tiles_q * pl.splits * 128 * pl.mb * pl.kbn * 4 : 0;
  *counters = global ? pl.tiles_p * pl.tiles_q : 0;
}

namespace {
// The plan of an external-splits GEMM: the split count the plan picks for the shape (before any
// cluster-residency shrink), every split's partial kept in global scratch.
bool external_plan(const GemmArgs& a, int sms, Plan* out) {
  if (a.w_format != kWBf16 || a.epilogue == kEpiSwiGLU || a.group_tiles != nullptr || gemv_applies(a)) return false;
  Plan pl = make_plan(a, sms, ~size_t(0) >> 1, 1 << 30, nullptr);
  if (!pl.swap || pl.mb != 1 || pl.splits <= 1) return false;
  pl.red = 1;
  pl.grid = std::min(pl.units, sms);
  *out = pl;
  return true;
}
}  // namespace

GemmSplits gemm_bf16_splits(const GemmArgs& a) {
  GemmSplits l;
  l.ws = a.workspace;
  Plan pl{};
  if (a.M > 0 && a.N > 0 && a.K > 0 && external_plan(a, a.num_sms > 0 ? a.num_sms : device_sms(), &pl)) {
    l.splits = pl.splits;
    l.kbn = pl.kbn;
    l.tiles_p = pl.tiles_p;
  }
  return l;
}

int gemm_bf16(const GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return -2;
  if (a.K % 8 != 0 || a.lda % 8 != 0 || a.ldw % 8 != 0) return -1;
  if ((reinterpret_cast<uintptr_t>(a.a) & 15) || (reinterpret_cast<uintptr_t>(a.w) & 15)) return -1;
  // One row of BF16 weights: a weight stream without the tensor-core pipeline (gemv.cu).
  if (gemv_applies(a)) return gemv_bf16(a, stream);
  if (a.epilogue == kEpiSwiGLU && (a.N % 256 != 0 || a.residual != nullptr)) return -2;
  if (a.epilogue != kEpiF32 && (a.ldc % 8 != 0 || (reinterpret_cast<uintptr_t>(a.c) & 15))) return -1;
  if (a.epilogue == kEpiF32 && (a.ldc % 4 != 0 || (reinterpret_cast<uintptr_t>(a.c) & 15))) return -1;
  if (a.residual != nullptr && a.epilogue != kEpiBf16) return -2;
  if (a.w_format != kWBf16 && a.w_scale == nullptr) return -2;
  if (a.w_format == kWNvfp4 && a.K % 64 != 0) return -2;
  const bool nvf4 = a.w_format == kWNvfp4A4;
  const bool fp8 = a.w_format == kWFp8A8;
  const bool grouped = a.group_tiles != nullptr;
  const int nseg = (a.seg[0].K > 0) + (a.seg[1].K > 0);
  if (nseg > 0) {
    if (a.w_format != kWBf16 || grouped || (a.seg[0].K <= 0 && a.seg[1].K > 0)) return -2;
    for (int i = 0; i < nseg; ++i)
      if (a.seg[i].K % kBlockK != 0 || a.seg[i].lda % 8 != 0 || a.seg[i].ldw % 8 != 0 ||
          (reinterpret_cast<uintptr_t>(a.seg[i].a) & 15) || (reinterpret_cast<uintptr_t>(a.seg[i].w) & 15))
        return -1;
  }
  if (grouped) {
    const int t = a.group_tile;
    if (a.w_format != kWBf16 || a.tile_group == nullptr || a.groups <= 0 || a.N % 128 != 0 ||
        !(t == 16 || t == 32 || t == 64 || t == 128 || t == 256) || a.residual != nullptr)
      return -2;
    if (a.epilogue == kEpiSwiGLU && t > 128) return -2;
  }
  if (fp8) {
    // E4M3 codes of both operands (one a byte), FP32 activation scales [K/128][a_scale_ld].
    if (a.K % 128 != 0 || a.lda % 16 != 0 || a.ldw % 16 != 0 || a.a_scale == nullptr) return -2;
    if (a.a_scale_ld < ((a.M + 127) / 128) * 128 || (reinterpret_cast<uintptr_t>(a.a_scale) & 15) ||
        (reinterpret_cast<uintptr_t>(a.w_scale) & 15))
      return -1;
  }
  if (nvf4) {
    // Both operands are packed E2M1 codes (two a byte) with 128-row-blocked scale atoms.
    if (a.K % 256 != 0 || a.lda % 32 != 0 || a.ldw % 32 != 0 || a.a_scale == nullptr) return -2;
    if ((reinterpret_cast<uintptr_t>(a.a_scale) & 15) || (reinterpret_cast<uintptr_t>(a.w_scale) & 15))
      return -1;
  }

  const int sms = a.num_sms > 0 ? a.num_sms : device_sms();
  g_cluster_wf = a.w_format;
  Plan pl{};
  if (a.external_splits) {
    // The next kernel adds the splits: they stay in the workspace in the GemmSplits layout.
    if (!external_plan(a, sms, &pl) || a.workspace == nullptr) return -2;
    if ((size_t)pl.tiles_p * pl.tiles_q * pl.splits * 128 * pl.kbn * 4 > a.workspace_bytes) return -3;
  } else {
    pl = make_plan(a, sms, a.workspace ? a.workspace_bytes : 0, a.counters ? a.counters_len : 0);
  }

  KParams kp{};
  kp.tiles_p = pl.tiles_p;
  kp.tiles_q = pl.tiles_q;
  kp.splits = pl.splits;
  kp.kblocks = pl.kblocks;
  kp.kb_per_split = pl.kb_per_split;
  kp.units = pl.units;
  kp.swap = pl.swap;
  kp.c = a.c;
  kp.ldc = a.ldc;
  kp.res = static_cast<const __nv_bfloat16*>(a.residual);
  kp.ldr = a.ldr;
  kp.ws = a.workspace;
  kp.counters = a.counters;
  kp.status = a.status;
  kp.trace = a.trace;
  kp.cta_trace = a.cta_trace;
  kp.debug = a.debug;
  kp.external = a.external_splits ? 1 : 0;
  kp.out_rows = a.M;
  kp.out_cols = a.epilogue == kEpiSwiGLU ? a.N / 2 : a.N;
  kp.wscale = a.w_scale;
  kp.wscale_ld = a.w_scale_ld;
  {
    const int main_kb = pl.kblocks - a.seg[0].K / kBlockK - a.seg[1].K / kBlockK;
    kp.seg_kb[0] = nseg > 0 ? main_kb : pl.kblocks;
    kp.seg_kb[1] = nseg > 1 ? main_kb + a.seg[0].K / kBlockK : pl.kblocks;
  }
  kp.wscale_row_shift = a.w_scale_rows == 1 ? 0 : 7;
  kp.wscale_k_shift = a.w_scale_rows == 1 ? 31 : 1;
  if (grouped) {
    kp.group_tiles = a.group_tiles;
    kp.tile_group = a.tile_group;
    kp.group_rows = a.N;
  }
  kp.acc_scale = (a.w_format == kWNvfp4 || nvf4) ? a.w_tensor_scale : 1.0f;
  if (nvf4) {
    const long atoms = (long)(a.K / 64) * 512;  // bytes of one 128-row block of scale atoms
    const uint8_t* sw = static_cast<const uint8_t*>(a.w_scale);
    const uint8_t* sa = static_cast<const uint8_t*>(a.a_scale);
    kp.sf_p = pl.swap ? sw : sa;
    kp.sf_q = pl.swap ? sa : sw;
    kp.sf_stride_p = kp.sf_stride_q = atoms;
    kp.sf_blocks_q = ((pl.swap ? a.M : a.N) + 127) / 128;
  }
  if (fp8) {
    kp.ascale = static_cast<const float*>(a.a_scale);
    kp.ascale_ld = a.a_scale_ld;
  }
  if (pl.red == 1 && (a.workspace == nullptr || (a.counters == nullptr && !a.external_splits))) return -3;

  CUtensorMap tp, tq;
  AuxMaps tw;
  std::memset(&tw, 0, sizeof(tw));
  const int prow_box = 128 * pl.mb;
  const int wrows_box = pl.swap ? prow_box : pl.kbn;
  const bool converted = a.w_format == kWFp8Block || a.w_format == kWNvfp4;
  if (converted) {
    // Raw quantized rows: K bytes (FP8) or K/2 bytes (NVFP4) a row, one k-block per box.
    const long row_bytes = a.w_format == kWFp8Block ? a.K : a.K / 2;
    const long ld_bytes = a.w_format == kWFp8Block ? a.ldw : a.ldw / 2;
    const int box_bytes = a.w_format == kWFp8Block ? 64 : 32;
    if (!encode_tmap_2d(&tw.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.w, a.N, row_bytes, ld_bytes,
                        wrows_box, box_bytes, CU_TENSOR_MAP_SWIZZLE_NONE))
      return -4;
  }
  // Rows mapping with BF16 weights: BF16 outputs leave through shared memory as TMA stores of
  // 32 x 64 boxes (whole 128-byte row segments instead of one 16-byte store a row and a thread).
  kp.tma_store = 0;
  if (!pl.swap && a.w_format == kWBf16 && a.debug == 0 && (reinterpret_cast<uintptr_t>(a.c) & 15) == 0) {
    if ((a.epilogue == kEpiBf16 || a.epilogue == kEpiSwiGLU) && a.ldc % 8 == 0) {
      const long out_cols = a.epilogue == kEpiSwiGLU ? a.N / 2 : a.N;
      if (encode_tmap_bf16_kmajor(&tw.c, a.c, a.M, out_cols, a.ldc, 32)) kp.tma_store = 1;
    } else if (a.epilogue == kEpiF32 && a.ldc % 4 == 0) {
      // FP32 rows of 32 elements (128 bytes) a box, 32 rows.
      if (encode_tmap_2d(&tw.c, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.c, a.M, a.N, a.ldc, 32, 32,
                         CU_TENSOR_MAP_SWIZZLE_128B))
        kp.tma_store = 1;
    }
  }
  // Operand maps: BF16 rows of 64 elements, or packed E2M1 rows of 128 bytes (256 elements).
  auto operand = [&](CUtensorMap* m, const void* base, long rows, long ld, int box) {
    if (nvf4) return encode_tmap_u8_kmajor(m, base, rows, a.K / 2, ld / 2, box);
    if (fp8) return encode_tmap_u8_kmajor(m, base, rows, a.K, ld, box);
    return encode_tmap_bf16_kmajor(m, base, rows, a.K, ld, box);
  };
  // Extra K segments: P is the weight side in the swap mapping, the activation side otherwise.
  for (int i = 0; i < nseg; ++i) {
    CUtensorMap* mp = i == 0 ? &tw.p1 : &tw.p2;
    CUtensorMap* mq = i == 0 ? &tw.q1 : &tw.q2;
    const GemmSegment& sg = a.seg[i];
    const bool ok = pl.swap ? (encode_tmap_bf16_kmajor(mp, sg.w, a.N, sg.K, sg.ldw, prow_box) &&
                               encode_tmap_bf16_kmajor(mq, sg.a, a.M, sg.K, sg.lda, pl.kbn))
                            : (encode_tmap_bf16_kmajor(mp, sg.a, a.M, sg.K, sg.lda, prow_box) &&
                               encode_tmap_bf16_kmajor(mq, sg.w, a.N, sg.K, sg.ldw, pl.kbn));
    if (!ok) return -4;
  }
  if (!pl.swap) {
    kp.Mp = a.M;
    kp.Nq = a.N;
    if (!operand(&tp, a.a, a.M, a.lda, prow_box)) return -4;
    if (converted) tq = tw.w;  // unused by the converting producer
    else if (!operand(&tq, a.w, a.N, a.ldw, pl.kbn)) return -4;
    if (pl.red == 2) return -2;
    switch (a.w_format) {
      case kWFp8Block: return launch_rows<kWFp8Block>(a.epilogue, tp, tq, tw, kp, pl, stream);
      case kWNvfp4: return launch_rows<kWNvfp4>(a.epilogue, tp, tq, tw, kp, pl, stream);
      case kWNvfp4A4: return launch_rows<kWNvfp4A4>(a.epilogue, tp, tq, tw, kp, pl, stream);
      case kWFp8A8:
        if (a.epilogue == kEpiSwiGLU) return -2;
        return a.epilogue == kEpiF32
                   ? launch_red<1, 128, kEpiF32, kWFp8A8>(tp, tq, tw, kp, pl, stream)
                   : launch_red<1, 128, kEpiBf16, kWFp8A8>(tp, tq, tw, kp, pl, stream);
      default: return launch_rows<kWBf16>(a.epilogue, tp, tq, tw, kp, pl, stream);
    }
  }
  kp.Mp = a.N;
  kp.Nq = a.M;
  if (converted) tp = tw.w;
  else if (!operand(&tp, a.w, (long)a.N * (grouped ? a.groups : 1), a.ldw, prow_box)) return -4;
  if (!operand(&tq, a.a, a.M, a.lda, pl.kbn)) return -4;
  switch (a.w_format) {
    case kWFp8Block: return launch_swap<kWFp8Block>(a.epilogue, tp, tq, tw, kp, pl, stream);
    case kWNvfp4: return launch_swap<kWNvfp4>(a.epilogue, tp, tq, tw, kp, pl, stream);
    case kWNvfp4A4: return launch_swap_nvf4(a.epilogue, tp, tq, tw, kp, pl, stream);
    case kWFp8A8: return launch_swap_fp8(a.epilogue, tp, tq, tw, kp, pl, stream);
    default: return launch_swap<kWBf16>(a.epilogue, tp, tq, tw, kp, pl, stream);
  }
}

}  // namespace foa
