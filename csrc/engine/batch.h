// One call of a decoder: its requests validated and planned on the host, then its operands
// staged on the device in one copy.
//
// Rules and messages follow the reference planner (crates/furiosa-opt-engine/src/decoder/batch/
// mod.rs:100-246): the planner is the only place a request is validated, it reads no token ID,
// and one-row (decode) requests take the call's first rows, then the others in request order
// (`layout`, mod.rs:267-277). The compact history of each request is the reference's five-field
// segment (compact.rs:40-83); per-row positions and cache slots are the reference's launch
// operands (operands.rs:52-133); every array lands in one device buffer of 256-byte aligned
// arrays through one host-to-device copy (staging.rs:13-26, :114).
#pragma once

#include <cstdint>
#include <optional>
#include <string>
#include <vector>

#include "runtime.h"

namespace foa::engine {

// ------------------------------------------------------------------------------------ cache spec
enum class KindTag { Paged, State, Cross };
struct Kind {
  KindTag tag = KindTag::Paged;
  int64_t length = 0;  // Cross only
  bool operator==(const Kind& o) const { return tag == o.tag && length == o.length; }
};

struct Pool {
  int64_t block = 16;  // tokens one block holds
  int64_t bytes = 0;   // bytes one block of one layer spans (per chip)
  bool operator==(const Pool& o) const { return block == o.block && bytes == o.bytes; }
};

struct Group {
  int64_t pool = 0;
  int64_t layers_begin = 0, layers_end = 0;
  Kind kind;
  std::optional<int64_t> window;
  bool operator==(const Group& o) const {
    return pool == o.pool && layers_begin == o.layers_begin && layers_end == o.layers_end &&
           kind == o.kind && window == o.window;
  }
};

struct CacheSpec {
  std::vector<Pool> pools;
  std::vector<Group> groups;
  bool operator==(const CacheSpec& o) const { return pools == o.pools && groups == o.groups; }
  // Bytes of each layer's storage of `blocks` blocks, group by group (refusals as the
  // reference's `CacheSpec::sizes`, cache.rs:69-90).
  std::vector<size_t> sizes(int64_t blocks) const;
};

// The storage of a spec: `blocks` pages of every layer, one zeroed allocation per layer.
class Cache {
 public:
  Cache(const Device& device, const CacheSpec& spec, int64_t blocks);
  int64_t blocks() const { return blocks_; }
  const CacheSpec& spec() const { return spec_; }
  const std::vector<HbmBuffer>& layers() const { return layers_; }
  // One call at a time borrows the cache (the reference lends its views under a mutex).
  void lend();
  void give_back();

 private:
  std::vector<HbmBuffer> layers_;
  int64_t blocks_;
  CacheSpec spec_;
  std::mutex mu_;
  bool lent_ = false;
};

// ------------------------------------------------------------------------------------ requests
enum class KeepKind { None, Last, All, Range };
struct Keep {
  KeepKind kind = KeepKind::Last;
  int64_t from = 0, to = 0;
};

struct Request {
  std::vector<std::vector<int64_t>> rows;  // block IDs per cache group
  int64_t cached = 0;
  HbmBuffer tokens;     // I32 IDs on the device
  int64_t length = 0;   // number of tokens
  Keep keep;
  std::optional<int64_t> adapter;
  bool positions = false, mask = false, overrides = false;
};

struct Limits {
  int64_t window = 0;
  int64_t rows = 0;
  CacheSpec cache;
  int64_t adapters = 0;
};

// The 256-byte alignment of every staged array.
constexpr size_t kStageAlign = 256;

// Staged operands of one call (byte offsets into the staging buffer).
struct Staged {
  size_t tokens = 0;      // I32 [rows_padded]
  size_t positions = 0;   // I32 [rows_padded]
  size_t slots = 0;       // I32 [rows_padded]: block * 16 + offset, or -1
  size_t segments = 0;    // I32 [segments_padded][5]: decode segments first
  size_t work = 0;        // I32 [work][2]: (prefill segment, query tile)
  size_t kept = 0;        // I32 [kept_padded]: call rows returned, in order
  size_t sources = 0;     // I32 [requests][4]: token arrays (address lo, hi, length, first row)
  size_t adapters = 0;    // I32 [rows_padded]: adapter slot of each row, -1 for none
  size_t table = 0;       // I32 block IDs
  size_t bytes = 0;       // bytes to copy
};

// The plan of one call.
struct Plan {
  int64_t rows = 0, rows_padded = 0;
  int64_t decode = 0;        // one-row segments (the call's first rows)
  int64_t prefill = 0;       // other segments
  int64_t segments_padded = 0;
  int64_t work = 0;          // prefill query tiles
  int64_t kept = 0, kept_padded = 0;
  int64_t requests = 0;
  int64_t max_keys = 0;      // longest decode history, keys
  int64_t max_len = 0;       // longest appended run
  bool adapted = false;
  Staged staged;
  std::vector<int64_t> kept_rows;  // host copy
};

// Validates `requests` against `limits` and `cache` and writes the call's operands into `host`
// (grown as needed). `group` is the query heads per key/value head (for the prefill tiles);
// `pad_decode` pads an all-decode call to `pad_rows` rows (CUDA-graph buckets, 0: no padding).
// Throws ValueError (invalid input) or Unsupported with the reference's messages.
Plan plan_call(const std::vector<Request>& requests, const Limits& limits, const CacheSpec& spec,
               int64_t blocks, int64_t adapters_given,
               const std::vector<bool>& adapter_slots_filled, int group, int64_t pad_rows,
               std::vector<uint8_t>& host);

// The call rows of requests of the given lengths: one-row requests first, then the others, each
// in request order. Returns [start, end) per request.
std::vector<std::pair<int64_t, int64_t>> layout(const std::vector<int64_t>& lengths);

}  // namespace foa::engine
