#include "batch.h"
#include "trace.h"

#include "kernels/attention.cuh"

#include <algorithm>
#include <cstring>
#include <unordered_set>

namespace foa::engine {

namespace {
// Rotary positions are FP32 values, exact below this.
constexpr int64_t kPositions = int64_t(1) << 24;

size_t align_up(size_t v) { return (v + kStageAlign - 1) / kStageAlign * kStageAlign; }
int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
}  // namespace

// ------------------------------------------------------------------------------------ cache
std::vector<size_t> CacheSpec::sizes(int64_t blocks) const {
  if (blocks <= 0) throw ValueError("cache blocks must be positive");
  std::vector<size_t> out;
  for (const Group& g : groups) {
    if (g.pool < 0 || g.pool >= static_cast<int64_t>(pools.size()))
      throw ValueError("cache group names no pool");
    const Pool& p = pools[g.pool];
    if (p.block <= 0 || p.bytes <= 0) throw ValueError("cache pool has empty blocks");
    // A page's byte offset within its layer stays an I32, as the reference's device tables hold.
    if (blocks > (int64_t(1) << 31) / p.bytes) throw ValueError("cache blocks pass I32 byte offsets");
    for (int64_t l = g.layers_begin; l < g.layers_end; ++l)
      out.push_back(static_cast<size_t>(blocks * p.bytes));
  }
  return out;
}

Cache::Cache(const Device& device, const CacheSpec& spec, int64_t blocks)
    : blocks_(blocks), spec_(spec) {
  const auto sizes = spec.sizes(blocks);
  auto st = device.state();
  for (size_t s : sizes) {
    HbmBuffer b(device, s);
    // Zeroed: a key/value slot a row has not written reads as zeros, never as NaN bits.
    st->check_cuda(cudaMemsetAsync(b.data(), 0, s, st->stream), "cache zero");
    layers_.push_back(std::move(b));
  }
  st->check_cuda(cudaStreamSynchronize(st->stream), "cache zero");
  size_t bytes = 0;
  for (size_t b : sizes) bytes += b;
  log_event(LogLevel::Info, "KV cache: " + std::to_string(blocks) + " blocks, " + std::to_string(bytes >> 20) + " MiB on GPU " +
                          std::to_string(st->ordinal));
}

void Cache::lend() {
  std::lock_guard<std::mutex> g(mu_);
  if (lent_) throw ValueError("cache is already borrowed");
  lent_ = true;
}

void Cache::give_back() {
  std::lock_guard<std::mutex> g(mu_);
  lent_ = false;
}

// ------------------------------------------------------------------------------------ layout
std::vector<std::pair<int64_t, int64_t>> layout(const std::vector<int64_t>& lengths) {
  std::vector<std::pair<int64_t, int64_t>> spans(lengths.size());
  int64_t start = 0;
  for (int pass = 0; pass < 2; ++pass)
    for (size_t i = 0; i < lengths.size(); ++i) {
      const bool one = lengths[i] == 1;
      if ((pass == 0) != one) continue;
      spans[i] = {start, start + lengths[i]};
      start += lengths[i];
    }
  return spans;
}

// ------------------------------------------------------------------------------------ planning
Plan plan_call(const std::vector<Request>& requests, const Limits& limits, const CacheSpec& spec,
               int64_t cache_blocks, int64_t adapters_given, const std::vector<bool>& filled,
               int group, int64_t pad_rows, std::vector<uint8_t>& host) {
  if (!(spec == limits.cache)) throw ValueError("cache was allocated for another model");
  std::vector<int64_t> blocks;
  for (const Group& g : limits.cache.groups) {
    if (g.kind.tag != KindTag::Paged) throw Unsupported("a call plans paged cache groups");
    blocks.push_back(limits.cache.pools[g.pool].block);
  }
  if (blocks.empty()) throw Unsupported("a call plans paged cache groups");
  if (requests.empty()) throw ValueError("call has no requests");
  bool adapted = adapters_given > 0;
  for (const auto& r : requests) adapted = adapted || r.adapter.has_value();
  if (adapted && limits.adapters == 0) throw Unsupported("adapters are not served");
  if (adapters_given > limits.adapters) throw ValueError("call holds more adapters than compiled");

  for (const auto& r : requests) {
    if (r.adapter && (*r.adapter < 0 || *r.adapter >= static_cast<int64_t>(filled.size()) ||
                      !filled[*r.adapter]))
      throw ValueError("request names a slot that holds no adapter");
    if (r.positions) throw Unsupported("explicit positions are not served");
    if (r.mask) throw Unsupported("visibility masks are not served");
    if (r.overrides) throw Unsupported("row overrides are not served");
    const int64_t len = r.length;
    const int64_t end = r.cached + len;
    if (r.rows.size() != blocks.size())
      throw ValueError("request holds a block list for each cache group");
    if (len == 0) throw ValueError("request has no tokens");
    if (end > limits.window) throw ValueError("request extends past the context window");
    if (end > kPositions) throw ValueError("position is not below 2^24");
    for (size_t g = 0; g < blocks.size(); ++g) {
      const int64_t used = ceil_div(end, blocks[g]);
      if (used > static_cast<int64_t>(r.rows[g].size()))
        throw ValueError("request has fewer blocks than its positions need");
      for (int64_t i = 0; i < used; ++i) {
        const int64_t id = r.rows[g][i];
        if (id < 0 || id >= cache_blocks) throw ValueError("block ID is outside the cache");
      }
    }
    if (r.keep.kind == KeepKind::Range && (r.keep.from > r.keep.to || r.keep.to > len))
      throw ValueError("kept rows lie outside the appended rows");
  }
  std::vector<int64_t> lengths;
  for (const auto& r : requests) lengths.push_back(r.length);
  const auto spans = layout(lengths);
  int64_t count = 0;
  for (const auto& s : spans) count = std::max(count, s.second);
  if (count > limits.rows) throw ValueError("call has more rows than compiled");
  for (size_t g = 0; g < blocks.size(); ++g) {
    std::unordered_set<int64_t> written;
    written.reserve(static_cast<size_t>(count) * 2);
    for (const auto& r : requests)
      for (int64_t p = r.cached; p < r.cached + r.length; ++p)
        if (!written.insert(r.rows[g][p / blocks[g]] * blocks[g] + p % blocks[g]).second)
          throw ValueError("two appended positions share a cache slot");
  }

  // ---------------------------------------------------------------- plan
  Plan plan;
  plan.rows = count;
  plan.requests = static_cast<int64_t>(requests.size());
  plan.adapted = adapted;
  for (size_t i = 0; i < requests.size(); ++i) {
    const auto& r = requests[i];
    const auto& s = spans[i];
    switch (r.keep.kind) {
      case KeepKind::None: break;
      case KeepKind::Last: plan.kept_rows.push_back(s.second - 1); break;
      case KeepKind::All:
        for (int64_t x = s.first; x < s.second; ++x) plan.kept_rows.push_back(x);
        break;
      case KeepKind::Range:
        for (int64_t x = s.first + r.keep.from; x < s.first + r.keep.to; ++x) plan.kept_rows.push_back(x);
        break;
    }
  }
  plan.kept = static_cast<int64_t>(plan.kept_rows.size());
  // Requests in call-row order: decode segments first.
  std::vector<size_t> order(requests.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = i;
  std::sort(order.begin(), order.end(),
            [&](size_t a, size_t b) { return spans[a].first < spans[b].first; });
  for (size_t i : order) {
    if (requests[i].length == 1) {
      ++plan.decode;
      plan.max_keys = std::max(plan.max_keys, requests[i].cached + 1);
    } else {
      ++plan.prefill;
    }
    plan.max_len = std::max(plan.max_len, requests[i].length);
  }
  const bool all_decode = plan.prefill == 0;
  plan.rows_padded = plan.rows;
  plan.segments_padded = plan.decode + plan.prefill;
  plan.kept_padded = plan.kept;
  if (all_decode && pad_rows > plan.rows) {
    plan.rows_padded = pad_rows;
    plan.segments_padded = pad_rows;
    plan.kept_padded = pad_rows;
  }
  int64_t work = 0;
  for (size_t i : order)
    if (requests[i].length != 1) work += ceil_div(requests[i].length * group, foa::kPrefillTile);
  plan.work = work;
  int64_t table_len = 1;  // one entry for padded segments
  for (const auto& r : requests) table_len += ceil_div(r.cached + r.length, blocks[0]);

  Staged& st = plan.staged;
  size_t off = 0;
  st.tokens = off;
  off = align_up(off + 4 * plan.rows_padded);
  st.positions = off;
  off = align_up(off + 4 * plan.rows_padded);
  st.slots = off;
  off = align_up(off + 4 * plan.rows_padded);
  st.segments = off;
  off = align_up(off + 4 * 5 * plan.segments_padded);
  st.work = off;
  off = align_up(off + 4 * 2 * std::max<int64_t>(work, 1));
  st.kept = off;
  off = align_up(off + 4 * std::max<int64_t>(plan.kept_padded, 1));
  st.sources = off;
  off = align_up(off + 4 * 4 * std::max(plan.requests, plan.rows_padded));
  st.adapters = off;
  off = align_up(off + 4 * plan.rows_padded);
  st.table = off;
  off = align_up(off + 4 * table_len);
  st.bytes = off;
  if (host.size() < off) host.resize(off * 2);
  std::memset(host.data(), 0, off);
  auto arr = [&](size_t o) { return reinterpret_cast<int32_t*>(host.data() + o); };
  int32_t* positions = arr(st.positions);
  int32_t* slots = arr(st.slots);
  int32_t* segments = arr(st.segments);
  int32_t* work_arr = arr(st.work);
  int32_t* kept = arr(st.kept);
  int32_t* sources = arr(st.sources);
  int32_t* adapter_rows = arr(st.adapters);
  int32_t* table = arr(st.table);
  const int64_t bsz = blocks[0];
  int64_t t = 0, seg = 0;
  for (size_t i : order) {
    const auto& r = requests[i];
    const auto& s = spans[i];
    const int64_t nb = ceil_div(r.cached + r.length, bsz);
    for (int64_t b = 0; b < nb; ++b) table[t + b] = static_cast<int32_t>(r.rows[0][b]);
    for (int64_t x = 0; x < r.length; ++x) {
      const int64_t p = r.cached + x;
      positions[s.first + x] = static_cast<int32_t>(p);
      slots[s.first + x] = static_cast<int32_t>(r.rows[0][p / bsz] * bsz + p % bsz);
      adapter_rows[s.first + x] = r.adapter ? static_cast<int32_t>(*r.adapter) : -1;
    }
    int32_t* sg = segments + 5 * seg;
    sg[0] = static_cast<int32_t>(s.first);
    sg[1] = static_cast<int32_t>(r.length);
    sg[2] = static_cast<int32_t>(r.cached);
    sg[3] = static_cast<int32_t>(t);
    sg[4] = static_cast<int32_t>(nb);
    t += nb;
    ++seg;
  }
  // Padded rows attend one key of a valid block and write no cache slot.
  table[t] = table[0];
  for (int64_t row = plan.rows; row < plan.rows_padded; ++row) {
    slots[row] = -1;
    adapter_rows[row] = -1;
    int32_t* sg = segments + 5 * row;
    sg[0] = static_cast<int32_t>(row);
    sg[1] = 1;
    sg[2] = 0;
    sg[3] = static_cast<int32_t>(t);
    sg[4] = 1;
  }
  int64_t w = 0;
  for (int64_t k = plan.decode; k < plan.decode + plan.prefill; ++k) {
    const int64_t len = segments[5 * k + 1];
    for (int64_t tile = 0; tile < ceil_div(len * group, foa::kPrefillTile); ++tile) {
      work_arr[2 * w] = static_cast<int32_t>(k);
      work_arr[2 * w + 1] = static_cast<int32_t>(tile);
      ++w;
    }
  }
  for (int64_t k = 0; k < plan.kept_padded; ++k)
    kept[k] = k < plan.kept ? static_cast<int32_t>(plan.kept_rows[k]) : 0;
  for (size_t i = 0; i < requests.size(); ++i) {
    const auto addr = reinterpret_cast<uint64_t>(requests[i].tokens.data());
    sources[4 * i] = static_cast<int32_t>(addr & 0xffffffffu);
    sources[4 * i + 1] = static_cast<int32_t>(addr >> 32);
    sources[4 * i + 2] = static_cast<int32_t>(requests[i].length);
    sources[4 * i + 3] = static_cast<int32_t>(spans[i].first);
  }
  return plan;
}

}  // namespace foa::engine
