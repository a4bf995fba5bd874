// Host-visible interface of the BF16 tcgen05 GEMM family.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace foa {

// What the epilogue does with each FP32 accumulator value.
enum GemmEpilogue : int {
  kEpiBf16 = 0,        // C = bf16(acc)                  (+ residual: C = bf16(acc + res))
  kEpiF32 = 1,         // C = acc as FP32
  kEpiSwiGLU = 2,      // weights interleave gate/up in 128-row blocks; C = bf16(bf16(silu(bf16 g)) * bf16 u)
};

// Which operand feeds the MMA's M side.
enum GemmMode : int {
  kModeAuto = 0,
  kModeRows = 1,   // activations on M (large row counts: prefill)
  kModeSwap = 2,   // weights on M, activations on N (few rows: decode)
};

// An extra K segment of a BF16 GEMM: activations [M, K] (row stride lda) times weights [N, K]
// (row stride ldw), added into the same FP32 sums before the epilogue (K a multiple of 64).
struct GemmSegment {
  const void* a = nullptr;
  long lda = 0;
  const void* w = nullptr;
  long ldw = 0;
  int K = 0;
};

struct GemmArgs {
  const void* a = nullptr;  // activations [M, K] BF16, row stride lda elements
  long lda = 0;
  const void* w = nullptr;  // weights [N, K] BF16, row stride ldw elements
  long ldw = 0;
  int M = 0, N = 0, K = 0;
  void* c = nullptr;  // output [M, N'] (N' = N, or N/2 for SwiGLU), row stride ldc elements
  long ldc = 0;
  const void* residual = nullptr;  // optional BF16 [M, N] added before rounding (kEpiBf16 only)
  long ldr = 0;
  int epilogue = kEpiBf16;
  int mode = kModeAuto;
  int splits = 0;  // K splits; 0 chooses
  // Swap mapping, splits > 1, BF16 weights: the K splits' FP32 partials stay in `workspace` for the
  // next kernel to add (GemmSplits describes where); the GEMM neither reduces nor writes `c`.
  int external_splits = 0;
  // Scratch for split-K partial sums: FP32 partials and one arrival counter per output tile.
  // The counters must be zero before the first launch; every launch leaves them zero.
  float* workspace = nullptr;
  size_t workspace_bytes = 0;
  int* counters = nullptr;
  int counters_len = 0;
  int* status = nullptr;  // device status word (see sm100.cuh)
  // Optional: CTA 0 writes %globaltimer at 8 milestones here (kernel entry, setup done, first
  // loads issued, first stage landed, last MMA issued, accumulator seen, epilogue done, exit).
  unsigned long long* trace = nullptr;
  // Optional: every CTA writes %globaltimer into cta_trace[8 * blockIdx.x + i]: 0 entry, 1 its first
  // accumulator seen by the epilogue, 2 its epilogue done; cluster split-K: 3 first cluster barrier
  // passed, 4 partials pushed, 5 second barrier passed, 6 slice reduced and stored; 7 exit.
  unsigned long long* cta_trace = nullptr;
  int num_sms = 0;        // 0: query the device
  // Quantized weights (W8A16 / W4A16): `w` then holds raw codes and the kernel dequantizes each
  // k-block into BF16 in shared memory before the MMAs read it.
  //   kWeightFp8Block: E4M3 codes [N, K] (ldw bytes a row), w_scale FP32 [ceil(N/128), w_scale_ld]
  //                    with one scale per 128x128 block (K % 64 == 0).
  //   kWeightNvfp4:    E2M1 codes [N, K/2 bytes] (ldw counts elements, two a byte, lower column in
  //                    the low nibble), w_scale E4M3 [N, w_scale_ld] one per 16 columns,
  //                    w_tensor_scale the FP32 factor of the whole tensor ("weight_scale_2")
  //                    that multiplies the FP32 sums (K % 64 == 0).
  //   kWeightNvfp4A4:  block-scaled NVFP4 on both operands (W4A4): `a` and `w` hold packed E2M1
  //                    codes (lda/ldw count elements), `a_scale` and `w_scale` their UE4M3 scales
  //                    as 128-row-blocked atoms [ceil(rows/128)][K/64][512 bytes] (in each atom the
  //                    scale of row r, group k sits at byte (r % 32) * 16 + (r / 32) * 4 + k), and
  //                    w_tensor_scale the product of both tensor scales (K % 256 == 0).
  int w_format = 0;
  const void* w_scale = nullptr;
  long w_scale_ld = 0;
  // kWeightFp8Block only: 128 (one scale per 128x128 block) or 1 (one scale per weight row, as
  // FP8 quantized at load per channel or per tensor; w_scale FP32 [N], w_scale_ld unused).
  int w_scale_rows = 128;
  float w_tensor_scale = 1.0f;
  //   kWeightFp8A8:    block-scaled FP8 on both operands (W8A8): `a` and `w` hold E4M3 codes,
  //                    w_scale FP32 [ceil(N/128), w_scale_ld, 4] per 128x128 block (each scale four
  //                    times, one 16-byte entry; see fp8_scales_pad4), a_scale FP32
  //                    [K/128, a_scale_ld] per (128-input group, row) with a_scale_ld >= M rounded
  //                    up to 128 (K % 128 == 0).
  const void* a_scale = nullptr;
  long a_scale_ld = 0;
  // Grouped GEMM (mixture-of-experts experts, BF16 weights, swap mapping, no split-K): `w` holds
  // `groups` weight matrices [N, K] one after another; `a` holds M token rows sorted by group with
  // each group's rows padded to `group_tile` (16, 32, 64, 128 or 256); `group_tiles` (device) is the
  // number of token tiles in use and `tile_group` (device) the group of each tile.
  const int* group_tiles = nullptr;
  const int* tile_group = nullptr;
  int group_tile = 0;
  int groups = 0;
  // Up to two extra K segments (BF16 weights, not grouped): C = epilogue(A.W^T + A1.W1^T + A2.W2^T).
  GemmSegment seg[2];
  // Measurement only (kernel_bench): how split-K partials meet (0 the plan's choice, 1 global
  // scratch, 2 cluster shared memory) and work left out (bit 0 no output stores, bit 1 no TMEM loads).
  int reduction = 0;
  int debug = 0;
};

enum GemmWeightFormat : int {
  kWeightBf16 = 0,
  kWeightFp8Block = 1,
  kWeightNvfp4 = 2,
  kWeightNvfp4A4 = 3,
  kWeightFp8A8 = 4,
};

// Plans and launches one GEMM on `stream`. Returns 0, or a negative code for a rejected argument
// (no launch happens then): -1 misaligned pointer/stride, -2 bad shape, -3 scratch too small,
// -4 tensor-map encoding failed, -5 launch failed.
int gemm_bf16(const GemmArgs& args, cudaStream_t stream);

// Projections of one row (K <= 4096, N <= 16384) of BF16 weights (mode and splits left to the plan, no extra K
// segment, no group, an unquantized weight): `gemm_bf16` runs them as a weight stream on the CUDA
// cores (gemv.cu), whose FP32 sums run in another order than the tensor-core GEMM's.
bool gemv_applies(const GemmArgs& args);
int gemv_bf16(const GemmArgs& args, cudaStream_t stream);

// Where a GEMM with external_splits leaves its K splits' FP32 partials: the partial of split s,
// token t (an A row) and feature f (a W row) sits at
//   ws[((f / 128 + (t / kbn) * tiles_p) * splits + s) * 128 * kbn + (t % kbn) * 128 + f % 128],
// so a token's 128 features of one split are contiguous.
struct GemmSplits {
  static constexpr int kMax = 8;  // the plan splits K at most 8 ways
  const float* ws = nullptr;
  int splits = 1, kbn = 0, tiles_p = 0;
  __host__ __device__ long at(int s, long t, long f) const {
    return ((f / 128 + (t / kbn) * (long)tiles_p) * splits + s) * 128L * kbn + (t % kbn) * 128 + f % 128;
  }
};

// The split layout the plan of `args` (mode and splits as given) would use: splits > 1 only when
// it runs on the swap mapping with a split K and no weight stream; otherwise splits == 1.
GemmSplits gemm_bf16_splits(const GemmArgs& args);

// Scratch the launch of `args` needs: FP32 workspace bytes and counter entries.
void gemm_bf16_scratch(const GemmArgs& args, size_t* workspace_bytes, int* counters);

}  // namespace foa
