// Host-visible interface of the paged attention kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace foa {

// One sequence's rows in a call: rows [row_start, row_start + len) of the call append positions
// cached .. cached + len - 1; the sequence's block IDs are table[table_start .. table_start +
// nblocks). The same five fields the reference's compact history encodes per segment.
struct Segment {
  int32_t row_start;
  int32_t len;
  int32_t cached;
  int32_t table_start;
  int32_t nblocks;
};

struct PagedAttention {
  const __nv_bfloat16* q = nullptr;  // [rows, q_heads, head_dim]
  __nv_bfloat16* o = nullptr;        // [rows, q_heads, head_dim]
  const __nv_bfloat16* cache = nullptr;  // layer pages: K[kv_heads][16][d] then V[kv_heads][16][d]
  const int32_t* table = nullptr;        // block IDs
  const Segment* segments = nullptr;
  int num_segments = 0;
  int q_heads = 0, kv_heads = 0, head_dim = 128;
  float scale = 0.f;  // softmax scale (1/sqrt(head_dim) by default)
  // Decode split scratch: FP32 partial outputs and log-sum-exps of every (row, head, split).
  float* partial_o = nullptr;
  float* partial_lse = nullptr;
  size_t partial_capacity = 0;  // elements of partial_lse (partial_o holds head_dim times more)
  int max_keys = 0;             // longest history of any segment (bounds the split count)
  int keys_per_split = 2048;    // fixed split width: each row's tiling depends on its own length
  int* status = nullptr;
  // Prefill on the tensor cores (TMA tensor maps): rows of q and o, and pages in the layer's cache.
  int rows = 0;
  long cache_blocks = 0;
  // Decode: warps a CTA (2, 3 or 4; 0 takes the default of 2) and 16-key blocks each warp keeps
  // in flight (2 or 3; 0 takes the default of 2).
  int decode_warps = 0;
  int decode_stages = 0;
  // Decode: one zeroed counter per (segment, key/value head) (num_segments * kv_heads of them);
  // given, the last split of each merges the splits in the decode kernel (no merge launch), and
  // the counters are zero again afterwards. Null: a separate merge kernel.
  int* merge_counters = nullptr;
  // Prefill: 0 causal (row i of a segment attends keys 0 .. cached + i); 1 bidirectional (every
  // row attends all cached + len keys of its segment: encoders, dense attention over visible keys).
  int bidirectional = 0;
};

// Decode: every segment appends one row (len == 1) and attends its whole history. A segment whose
// history (cached + 1) exceeds `max_keys` gets zeros in its output rows and records kBadArgument
// in `status`: `max_keys` sizes the split scratch, so it must bound every segment.
int paged_decode(const PagedAttention& args, cudaStream_t stream);

// Prefill / chunks: segments of any length attend their history plus their own rows causally.
// `work` lists (segment, query tile) pairs, `num_work` of them; a tile is 128 (token, head) rows
// of one key/value head. Runs on the tcgen05 tensor cores when `prefill_tc_supported` (head_dim
// 64 or 128, a GQA group dividing 128, `rows` and `cache_blocks` set), else on mma.sync.
int paged_prefill(const PagedAttention& args, const int32_t* work, int num_work,
                  cudaStream_t stream);
bool prefill_tc_supported(const PagedAttention& args);
int paged_prefill_tc(const PagedAttention& args, const int32_t* work, int num_work,
                     cudaStream_t stream);

// Rows of a prefill query tile, and the query tiles of a segment of `len` rows with `group`
// query heads per key/value head.
constexpr int kPrefillTile = 128;
inline int prefill_tiles(int len, int group) { return (len * group + kPrefillTile - 1) / kPrefillTile; }

}  // namespace foa
