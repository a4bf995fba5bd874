#include "model.h"

#include "trace.h"

#include <algorithm>
#include <cmath>
#include <cstring>

#include "kernels/attention.cuh"
#include "kernels/gemm.cuh"
#include "kernels/quant.cuh"
#include "kernels/moe.cuh"
#include "kernels/ops.cuh"
#include "lora.h"
#include "modules.h"

namespace foa::engine {

namespace {
constexpr size_t kAlign = 256;
size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }
int64_t next_pow2(int64_t v) {
  int64_t p = 1;
  while (p < v) p <<= 1;
  return p;
}
__nv_bfloat16* bf(const HbmBuffer& b) { return static_cast<__nv_bfloat16*>(b.data()); }
uint8_t* u8(const HbmBuffer& b) { return static_cast<uint8_t*>(b.data()); }
int32_t* i32(const HbmBuffer& b, size_t off = 0) {
  return reinterpret_cast<int32_t*>(static_cast<char*>(b.data()) + off);
}
}  // namespace

// ------------------------------------------------------------------------------------ RoPE
std::vector<float> rope_inv_freq(const RopeSpec& r, int d, float* attention_factor) {
  const int half = d / 2;
  std::vector<double> base(half);
  for (int j = 0; j < half; ++j) base[j] = 1.0 / std::pow(r.theta, (2.0 * j) / d);
  std::vector<double> out = base;
  double attn = 1.0;
  if (r.type == "linear") {
    for (auto& f : out) f /= r.factor;
  } else if (r.type == "llama3") {
    const double old = r.original_max_positions;
    const double low_wl = old / r.low_freq_factor, high_wl = old / r.high_freq_factor;
    for (int j = 0; j < half; ++j) {
      const double f = base[j], wl = 2.0 * M_PI / f;
      if (wl < high_wl) {
        out[j] = f;
      } else if (wl > low_wl) {
        out[j] = f / r.factor;
      } else {
        const double smooth = (old / wl - r.low_freq_factor) / (r.high_freq_factor - r.low_freq_factor);
        out[j] = (1.0 - smooth) * f / r.factor + smooth * f;
      }
    }
  } else if (r.type == "yarn") {
    const double old = r.original_max_positions;
    auto corr_dim = [&](double rot) {
      return (d * std::log(old / (rot * 2.0 * M_PI))) / (2.0 * std::log(r.theta));
    };
    double low = corr_dim(r.beta_fast), high = corr_dim(r.beta_slow);
    if (r.truncate) {
      low = std::floor(low);
      high = std::ceil(high);
    }
    low = std::max(low, 0.0);
    high = std::min(high, double(d - 1));
    if (low == high) high += 0.001;
    for (int j = 0; j < half; ++j) {
      const double ramp = std::clamp((j - low) / (high - low), 0.0, 1.0);
      const double extrap = 1.0 - ramp;
      out[j] = (base[j] / r.factor) * (1.0 - extrap) + base[j] * extrap;
    }
    auto mscale = [](double s, double m) { return s <= 1.0 ? 1.0 : 0.1 * m * std::log(s) + 1.0; };
    if (r.attention_factor > 0)
      attn = r.attention_factor;
    else if (r.mscale_all_dim > 0)
      attn = mscale(r.factor, r.mscale) / mscale(r.factor, r.mscale_all_dim);
    else
      attn = mscale(r.factor, 1.0);
  }
  if (attention_factor) *attention_factor = static_cast<float>(attn);
  return std::vector<float>(out.begin(), out.end());
}

// ------------------------------------------------------------------------------------ model
DecoderModel::DecoderModel(const Device& device, ModelConfig cfg, int tp, int rank)
    : device_(device), cfg_(std::move(cfg)), tp_(tp), rank_(rank) {
  if (cfg_.q_heads % tp_ != 0) throw Unsupported("query heads do not split evenly over the chips");
  qh_l_ = cfg_.q_heads / tp_;
  qh_first_ = rank_ * qh_l_;
  if (cfg_.kv_heads >= tp_) {
    if (cfg_.kv_heads % tp_ != 0) throw Unsupported("key/value heads do not split evenly over the chips");
    kvh_l_ = cfg_.kv_heads / tp_;
    kvh_first_ = rank_ * kvh_l_;
  } else {
    // Fewer key/value heads than chips: each chip holds a replica of the head its queries read.
    if (tp_ % cfg_.kv_heads != 0) throw Unsupported("key/value heads do not split evenly over the chips");
    kvh_l_ = 1;
    kvh_first_ = rank_ * cfg_.kv_heads / tp_;
  }
  // Decode attention splits every history into fixed chunks of keys, with two or four warps a CTA.
  // With few key/value heads on a chip (tensor parallelism) a decode batch gives the GPU few CTAs:
  // four heads take four warps a CTA, one or two heads 256-key chunks (measured on B200, 64 rows of
  // 1100 keys: 41.6 against 44.2 us at four heads; 29.7 against 36.6 us at two; 21.9 against
  // 33.6 us at one). Both depend on the geometry only: a row's result does not depend on its batch.
  keys_per_split_ = kvh_l_ <= 2 ? 256 : 2048;
  decode_warps_ = kvh_l_ == 4 ? 4 : 2;
  const int inter = cfg_.experts > 0 ? 0 : cfg_.intermediate;
  if (inter % tp_ != 0 || (inter / tp_) % 128 != 0)
    throw Unsupported("the intermediate width does not split into 128-row blocks over the chips");
  inter_l_ = inter / tp_;
  if (cfg_.experts > 0) {
    // Experts split evenly over the ranks (expert parallelism = tensor parallelism here).
    if (cfg_.experts % tp_ != 0) throw Unsupported("the experts do not split evenly over the chips");
    if (cfg_.expert_intermediate % 128 != 0) throw Unsupported("the expert width is not a multiple of 128");
    if (cfg_.top_k <= 0 || cfg_.top_k > 32 || cfg_.experts > 512) throw Unsupported("the routing is outside 32 of 512 experts");
    experts_l_ = cfg_.experts / tp_;
    expert_first_ = rank_ * experts_l_;
  }
  vocab_l_ = (cfg_.vocab + tp_ - 1) / tp_;
  vocab_l_ = (vocab_l_ + 7) / 8 * 8;
  vocab_begin_ = rank_ * vocab_l_;
  vocab_end_ = std::min(cfg_.vocab, vocab_begin_ + vocab_l_);
  inv_freq_host_ = rope_inv_freq(cfg_.rope, cfg_.head_dim, &attention_factor_);
  allocate_weights();
  auto st = device_.state();
  inv_freq_ = HbmBuffer(device_, inv_freq_host_.size() * sizeof(float));
  st->check_cuda(cudaMemcpy(inv_freq_.data(), inv_freq_host_.data(), inv_freq_.size(),
                            cudaMemcpyHostToDevice),
                 "rope table");
  for (auto& e : stage_done_) st->check_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
}

DecoderModel::~DecoderModel() {
  device_.state()->activate();
  cudaStreamSynchronize(device_.state()->stream);
  clear_graphs();
  for (auto& e : stage_done_)
    if (e) cudaEventDestroy(e);
}

int DecoderModel::moe_tile(int64_t rows) const {
  // Token tiles near the rows an expert receives on average (16 to 128).
  const int64_t per = rows * std::max(cfg_.top_k, 1) / std::max(cfg_.experts, 1);
  return per <= 16 ? 16 : per <= 32 ? 32 : per <= 64 ? 64 : 128;
}

int64_t DecoderModel::moe_capacity(int64_t rows) const {
  // Every selection plus a partial tile per local expert, for the largest tile.
  return (rows * cfg_.top_k + static_cast<int64_t>(experts_l_) * 127 + 127) / 128 * 128;
}

void DecoderModel::clear_graphs() {
  for (auto& g : graphs_)
    if (g.second.exec) cudaGraphExecDestroy(g.second.exec);
  graphs_.clear();
}

Limits DecoderModel::limits() const {
  Limits l;
  l.window = cfg_.window;
  l.rows = cfg_.rows;
  Pool pool;
  pool.block = 16;
  pool.bytes = 2LL * kvh_l_ * 16 * cfg_.head_dim * 2;
  l.cache.pools.push_back(pool);
  Group g;
  g.pool = 0;
  g.layers_begin = 0;
  g.layers_end = cfg_.layers;
  l.cache.groups.push_back(g);
  l.adapters = adapter_slots_;
  return l;
}

void DecoderModel::allocate_weights() {
  const int H = cfg_.hidden, D = cfg_.head_dim;
  std::vector<std::pair<std::string, std::vector<int64_t>>> plan;
  // The embedding is whole on every chip, padded to the chips' head shards; the head is the
  // chip's vocabulary shard (a view into the embedding when they are tied).
  plan.push_back({"embed", {static_cast<int64_t>(vocab_l_) * tp_, H}});
  // Only a decoder that returns tokens reads a vocabulary head.
  if (!cfg_.tied && cfg_.output == Output::Tokens) plan.push_back({"lm_head", {vocab_l_, H}});
  plan.push_back({"final_norm", {H}});
  if (cfg_.output == Output::Scores) plan.push_back({"score", {cfg_.labels, H}});
  for (int l = 0; l < cfg_.layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    plan.push_back({p + "in_norm", {H}});
    plan.push_back({p + "qkv", {(qh_l_ + 2 * kvh_l_) * D, H}});
    if (cfg_.qk_norm) {
      plan.push_back({p + "q_norm", {D}});
      plan.push_back({p + "k_norm", {D}});
    }
    plan.push_back({p + "o", {H, qh_l_ * D}});
    plan.push_back({p + "post_norm", {H}});
    if (cfg_.experts == 0) {
      plan.push_back({p + "gate_up", {2 * inter_l_, H}});
      plan.push_back({p + "down", {H, inter_l_}});
    } else {
      // Router (every expert, on every rank) and this rank's experts, one after another.
      const int64_t I = cfg_.expert_intermediate;
      plan.push_back({p + "router", {cfg_.experts, H}});
      plan.push_back({p + "experts_gate_up", {static_cast<int64_t>(experts_l_) * 2 * I, H}});
      plan.push_back({p + "experts_down", {static_cast<int64_t>(experts_l_) * H, I}});
    }
  }
  const std::string& wf = cfg_.weight_format;
  // FP8 codes with one FP32 scale per weight row: quantized at load per channel or per tensor,
  // or read from a static per-tensor FP8 checkpoint (each projection's scale on its rows).
  const bool per_row = wf == "fp8_channel" || wf == "fp8_tensor" || wf == "fp8_static";
  const int format = wf == "fp8_block" ? foa::kWeightFp8A8
                     : per_row          ? foa::kWeightFp8Block
                     : wf == "nvfp4"   ? foa::kWeightNvfp4
                     : wf == "nvfp4_a4" ? foa::kWeightNvfp4A4
                                        : foa::kWeightBf16;
  if (format == foa::kWeightBf16 && wf != "bf16") throw ValueError("unknown weight format " + wf);
  auto projection = [](const std::string& name) {
    const auto dot = name.rfind('.');
    const std::string leaf = dot == std::string::npos ? name : name.substr(dot + 1);
    return leaf == "qkv" || leaf == "o" || leaf == "gate_up" || leaf == "down";
  };
  // Byte sizes of a slot: [BF16 or codes, scales].
  auto sizes = [&](const std::string& name, const std::vector<int64_t>& shape) -> std::pair<size_t, size_t> {
    size_t n = 1;
    for (auto s : shape) n *= static_cast<size_t>(s);
    if (format == foa::kWeightBf16 || !projection(name)) return {n * 2, 0};
    const int64_t rows = shape[0], cols = shape[1];
    const int64_t rb = (rows + 127) / 128;
    if (per_row) {
      if (cols % 64 != 0) throw Unsupported(name + ": FP8 inputs here come in multiples of 64");
      return {n, static_cast<size_t>(rows * 4)};
    }
    if (format == foa::kWeightFp8A8) {
      if (cols % 128 != 0) throw Unsupported(name + ": FP8 block inputs come in multiples of 128");
      return {n, static_cast<size_t>(rb * (cols / 128) * 16)};  // each scale four times
    }
    if (cols % (format == foa::kWeightNvfp4A4 ? 256 : 64) != 0)
      throw Unsupported(name + ": NVFP4 inputs here come in multiples of " +
                        std::to_string(format == foa::kWeightNvfp4A4 ? 256 : 64));
    if (format == foa::kWeightNvfp4) return {n / 2, static_cast<size_t>(rows * (cols / 16))};
    return {n / 2, static_cast<size_t>(rb * (cols / 64) * 512)};
  };
  size_t total = 0;
  std::vector<std::pair<size_t, size_t>> offs;
  for (auto& e : plan) {
    const auto [a, b] = sizes(e.first, e.second);
    const size_t o0 = total;
    total = align_up(total + a);
    const size_t o1 = total;
    total = align_up(total + b);
    offs.push_back({o0, b ? o1 : 0});
  }
  arena_ = HbmBuffer(device_, std::max<size_t>(total, 256));
  arena_bytes_ = total;
  for (size_t i = 0; i < plan.size(); ++i) {
    WeightSlot w;
    char* base = static_cast<char*>(arena_.data());
    w.shape = plan[i].second;
    if (format != foa::kWeightBf16 && projection(plan[i].first)) {
      w.format = format;
      w.codes = reinterpret_cast<uint8_t*>(base + offs[i].first);
      w.scales = base + offs[i].second;
      const int64_t cols = w.shape[1];
      w.scale_ld = format == foa::kWeightFp8A8 ? cols / 128 : format == foa::kWeightNvfp4 ? cols / 16 : cols / 64 * 512;
      if (per_row) {
        w.scale_rows = 1;
        w.scale_ld = 1;
      }
    } else {
      w.ptr = reinterpret_cast<__nv_bfloat16*>(base + offs[i].first);
    }
    weights_[plan[i].first] = w;
  }
  if (cfg_.tied && cfg_.output == Output::Tokens) {
    WeightSlot head = weights_["embed"];
    head.ptr += static_cast<size_t>(vocab_begin_) * H;
    head.shape = {vocab_l_, H};
    weights_["lm_head"] = head;
  }
}

namespace {
uint32_t name_tag(const std::string& s) {
  uint32_t h = 2166136261u;  // FNV-1a
  for (unsigned char c : s) h = (h ^ c) * 16777619u;
  return h & 0xFFFFFu;
}
}  // namespace

void DecoderModel::quantize_slot(WeightSlot& w, const __nv_bfloat16* src, float stdv, float amax) {
  auto st = device_.state();
  const int rows = static_cast<int>(w.shape[0]), cols = static_cast<int>(w.shape[1]);
  if (w.format == foa::kWeightFp8Block && w.scale_rows == 1) {
    // Per channel: each row's magnitude; per tensor: a magnitude bound the whole tensor shares
    // (the checkpoint's fused amax at load, 8 standard deviations for synthetic weights).
    float bound = -1.f;
    if (cfg_.weight_format == "fp8_tensor") bound = amax >= 0.f ? amax : 8.f * stdv;
    if (foa::quantize_fp8_rows(src, rows, cols, bound, w.codes, static_cast<float*>(w.scales), st->stream) != 0)
      st->fail("weight quantization launch failed");
    st->check_cuda(cudaStreamSynchronize(st->stream), "weight quantization");
    return;
  }
  if (w.format == foa::kWeightFp8A8) {
    const long n = static_cast<long>((rows + 127) / 128) * (cols / 128);
    HbmBuffer plain(device_, n * 4);
    if (foa::quantize_fp8_block(src, rows, cols, w.codes, static_cast<float*>(plain.data()), st->stream) != 0 ||
        foa::fp8_scales_pad4(static_cast<const float*>(plain.data()), n, static_cast<float*>(w.scales), st->stream) != 0)
      st->fail("weight quantization launch failed");
    st->check_cuda(cudaStreamSynchronize(st->stream), "weight quantization");
    return;
  }
  // NVFP4: one tensor scale from a fixed magnitude bound (8 standard deviations), the same on
  // every tensor-parallel shard of the weight; synthetic inputs quantize under a bound of 8.
  const float bound[2] = {8.f * stdv, 0.f};
  HbmBuffer amax_buf(device_, 16);
  st->check_cuda(cudaMemcpyAsync(amax_buf.data(), bound, 8, cudaMemcpyHostToDevice, st->stream), "amax");
  HbmBuffer rowmajor;
  uint8_t* sc = static_cast<uint8_t*>(w.scales);
  if (w.format == foa::kWeightNvfp4A4) {
    rowmajor = HbmBuffer(device_, static_cast<size_t>(rows) * (cols / 16));
    sc = static_cast<uint8_t*>(rowmajor.data());
  }
  float* amax_p = static_cast<float*>(amax_buf.data());
  if (foa::quantize_nvfp4(src, rows, cols, w.codes, sc, amax_p, amax_p + 1, st->stream) != 0)
    st->fail("weight quantization launch failed");
  if (w.format == foa::kWeightNvfp4A4 &&
      foa::nvfp4_scale_atoms(sc, cols / 16, rows, cols, static_cast<uint8_t*>(w.scales), st->stream) != 0)
    st->fail("weight quantization launch failed");
  float ts = 1.f;
  st->check_cuda(cudaMemcpyAsync(&ts, amax_p + 1, 4, cudaMemcpyDeviceToHost, st->stream), "tensor scale");
  st->check_cuda(cudaStreamSynchronize(st->stream), "weight quantization");
  w.tensor_scale = ts;
  w.input_scale = 8.f / (6.f * 448.f);
}

void DecoderModel::init_random(uint64_t seed, float stdv) {
  auto st = device_.state();
  st->activate();
  const int H = cfg_.hidden, D = cfg_.head_dim;
  HbmBuffer map_rows, map_tags, init_tmp;
  for (auto& [name, w] : weights_) {
    if (name == "lm_head" && cfg_.tied) continue;
    if (w.format != foa::kWeightBf16 && w.codes == nullptr) continue;
    long n = 1;
    for (auto s : w.shape) n *= s;
    if (name.find("norm") != std::string::npos) {
      if (foa::fill_bf16(w.ptr, n, 1.0f, st->stream) != 0) st->fail("weight initialisation launch failed");
      continue;
    }
    // The logical row, tag and column window of every shard row, so each tensor-parallel split
    // of one model holds the same logical weights.
    const int rows = static_cast<int>(w.shape[0]), cols = static_cast<int>(w.shape[1]);
    std::vector<int32_t> full(rows);
    std::vector<uint32_t> tags(rows);
    long full_cols = cols, col_offset = 0;
    const auto dot = name.rfind('.');
    const std::string prefix = dot == std::string::npos ? "" : name.substr(0, dot + 1);
    const std::string leaf = dot == std::string::npos ? name : name.substr(dot + 1);
    for (int r = 0; r < rows; ++r) {
      full[r] = r;
      tags[r] = name_tag(name);
    }
    if (leaf == "lm_head") {
      for (int r = 0; r < rows; ++r) full[r] = vocab_begin_ + r;
    } else if (leaf == "qkv") {
      for (int r = 0; r < rows; ++r) {
        if (r < qh_l_ * D) {
          full[r] = qh_first_ * D + r;
          tags[r] = name_tag(prefix + "q");
        } else if (r < (qh_l_ + kvh_l_) * D) {
          full[r] = kvh_first_ * D + (r - qh_l_ * D);
          tags[r] = name_tag(prefix + "k");
        } else {
          full[r] = kvh_first_ * D + (r - (qh_l_ + kvh_l_) * D);
          tags[r] = name_tag(prefix + "v");
        }
      }
    } else if (leaf == "o") {
      full_cols = static_cast<long>(cfg_.q_heads) * D;
      col_offset = static_cast<long>(qh_first_) * D;
    } else if (leaf == "gate_up") {
      for (int r = 0; r < rows; ++r) {
        const int block = r / 128;
        full[r] = rank_ * inter_l_ + (block / 2) * 128 + r % 128;
        tags[r] = name_tag(prefix + (block % 2 == 0 ? "gate" : "up"));
      }
    } else if (leaf == "down") {
      full_cols = cfg_.intermediate;
      col_offset = static_cast<long>(rank_) * inter_l_;
    } else if (leaf == "experts_gate_up") {
      const int I = cfg_.expert_intermediate;
      for (int r = 0; r < rows; ++r) {
        const int e = expert_first_ + r / (2 * I), rr = r % (2 * I), block = rr / 128;
        full[r] = (block / 2) * 128 + rr % 128;
        tags[r] = name_tag(prefix + "experts." + std::to_string(e) + (block % 2 == 0 ? ".gate" : ".up"));
      }
    } else if (leaf == "experts_down") {
      for (int r = 0; r < rows; ++r) {
        const int e = expert_first_ + r / H;
        full[r] = r % H;
        tags[r] = name_tag(prefix + "experts." + std::to_string(e) + ".down");
      }
    }
    (void)H;
    if (map_rows.size() < static_cast<size_t>(rows) * 4) {
      map_rows = HbmBuffer(device_, static_cast<size_t>(rows) * 4);
      map_tags = HbmBuffer(device_, static_cast<size_t>(rows) * 4);
    }
    st->check_cuda(cudaMemcpyAsync(map_rows.data(), full.data(), rows * 4, cudaMemcpyHostToDevice, st->stream), "init map");
    st->check_cuda(cudaMemcpyAsync(map_tags.data(), tags.data(), rows * 4, cudaMemcpyHostToDevice, st->stream), "init map");
    __nv_bfloat16* dst = w.ptr;
    if (w.format != foa::kWeightBf16) {
      if (init_tmp.size() < static_cast<size_t>(rows) * cols * 2) init_tmp = HbmBuffer(device_, static_cast<size_t>(rows) * cols * 2);
      dst = static_cast<__nv_bfloat16*>(init_tmp.data());
    }
    if (foa::init_normal_rows(dst, rows, cols, static_cast<const int32_t*>(map_rows.data()),
                              static_cast<const uint32_t*>(map_tags.data()), full_cols, col_offset,
                              stdv, seed, st->stream) != 0)
      st->fail("weight initialisation launch failed");
    if (w.format != foa::kWeightBf16) quantize_slot(w, dst, stdv);
    // The host maps must outlive their copies.
    st->check_cuda(cudaStreamSynchronize(st->stream), "weight initialisation");
  }
  st->check_cuda(cudaStreamSynchronize(st->stream), "weight initialisation");
}

void DecoderModel::ensure_workspace(int64_t rows, int64_t kept, int64_t splits, int64_t decode_rows) {
  const int H = cfg_.hidden, D = cfg_.head_dim;
  bool changed = false;
  if (rows > ws_rows_) {
    const int64_t R = std::max<int64_t>(256, next_pow2(rows));
    ws_x_ = HbmBuffer(device_, R * H * 2);
    ws_h_ = HbmBuffer(device_, R * H * 2);
    ws_qkv_ = HbmBuffer(device_, R * (qh_l_ + 2 * kvh_l_) * D * 2);
    ws_q_ = HbmBuffer(device_, R * qh_l_ * D * 2);
    ws_attn_ = HbmBuffer(device_, R * qh_l_ * D * 2);
    ws_act_ = HbmBuffer(device_, std::max<int64_t>(R * inter_l_ * 2, 256));
    if (cfg_.weight_format != "bf16") {
      // Quantized inputs of the widest projection input: FP8 codes (1 byte) or NVFP4 codes (half),
      // FP8 scales [K/128][R] or NVFP4 atoms [R/128][K/64][512] (R a multiple of 128).
      const int64_t kmax = std::max<int64_t>({H, static_cast<int64_t>(qh_l_) * D, inter_l_});
      ws_qa_ = HbmBuffer(device_, R * kmax);
      ws_qs_ = HbmBuffer(device_, std::max<int64_t>(kmax / 128 * R * 4, R * kmax / 16));
    }
    ws_rows_ = R;
    changed = true;
  }
  if (cfg_.experts > 0 && rows > ws_moe_rows_) {
    const int64_t R = std::max<int64_t>(256, next_pow2(rows));
    const int64_t E = cfg_.experts, K = cfg_.top_k, I = cfg_.expert_intermediate;
    const int64_t cap = moe_capacity(R);
    ws_logits_e_ = HbmBuffer(device_, R * E * 2);
    ws_ids_ = HbmBuffer(device_, R * K * 4);
    ws_rw_ = HbmBuffer(device_, R * K * 4);
    ws_pos_ = HbmBuffer(device_, static_cast<int64_t>(tp_) * R * K * 4);
    ws_src_ = HbmBuffer(device_, cap * 4);
    ws_tile_e_ = HbmBuffer(device_, (cap / 16 + 1) * 4);
    ws_tiles_ = HbmBuffer(device_, 256);
    ws_xs_ = HbmBuffer(device_, cap * H * 2);
    ws_eact_ = HbmBuffer(device_, cap * I * 2);
    ws_y_ = HbmBuffer(device_, cap * H * 2);
    ws_moe_rows_ = R;
    changed = true;
  }
  if (adapter_slots_ > 0 && (changed || !ws_lora_z_.valid())) {
    const int64_t R = std::max<int64_t>(256, next_pow2(std::max(rows, ws_rows_)));
    ws_lora_z_ = HbmBuffer(device_, R * 2 * 128 * 2);
  }
  if (kept > ws_kept_) {
    const int64_t K = std::max<int64_t>(64, next_pow2(kept));
    ws_hk_ = HbmBuffer(device_, K * H * 2);
    const int64_t cols = cfg_.output == Output::Scores ? cfg_.labels : vocab_l_;
    ws_logits_ = HbmBuffer(device_, K * std::max<int64_t>(cols, 8) * 4);
    ws_idx_ = HbmBuffer(device_, K * 4);
    ws_val_ = HbmBuffer(device_, K * 4);
    ws_tokens_ = HbmBuffer(device_, K * 4);
    ws_kept_ = K;
    changed = true;
  }
  if (splits > ws_splits_ || decode_rows > ws_decode_) {
    const int64_t S = std::max(splits, ws_splits_), Rd = std::max<int64_t>(std::max(decode_rows, ws_decode_), 64);
    ws_part_o_ = HbmBuffer(device_, Rd * qh_l_ * S * D * 4);
    ws_part_lse_ = HbmBuffer(device_, Rd * qh_l_ * S * 4);
    ws_splits_ = S;
    ws_decode_ = Rd;
    changed = true;
  }
  if (!ws_gemm_.valid()) {
    ws_gemm_ = HbmBuffer(device_, 64 << 20);
    ws_counters_ = HbmBuffer(device_, 65536 * 4);
    auto st = device_.state();
    st->check_cuda(cudaMemsetAsync(ws_counters_.data(), 0, ws_counters_.size(), st->stream), "zero");
    changed = true;
  }
  if (changed) clear_graphs();
}

int64_t DecoderModel::graph_bucket(int64_t rows) const {
  static const int64_t kBuckets[] = {1, 2, 4, 8, 16, 32, 48, 64, 96, 128, 192, 256, 384, 512};
  for (int64_t b : kBuckets)
    if (rows <= b) return b;
  return 0;
}

HbmTensor DecoderModel::forward(const std::vector<Request>& requests, Cache& cache,
                                const std::vector<std::shared_ptr<const LoraAdapter>>& adapters) {
  auto st = device_.state();
  st->check();
  st->activate();
  TraceScope call_span("forward", "call");
  const TraceLevel tracing = trace_level();
  cudaEvent_t device_begin = tracing >= TraceLevel::Info ? Tracer::get().record(st->ordinal, st->stream) : nullptr;
  const Limits lim = limits();
  std::vector<bool> filled;
  for (const auto& a : adapters) {
    if (a && a->owner() != this) throw ValueError("the adapter belongs to another model");
    filled.push_back(a != nullptr);
  }
  call_adapters_ = adapters;
  // Decode-only calls whose every request keeps its last row run as CUDA graphs of padded size
  // (calls with adapters run eagerly: their factors differ call to call).
  // (Per-kernel tracing runs eagerly: its events sit between the launches.)
  bool graphable = graphs_enabled_ && adapters.empty() && tracing < TraceLevel::Trace;
  int64_t rows = 0;
  for (const auto& r : requests) {
    rows += r.length;
    graphable = graphable && r.length == 1 && r.keep.kind == KeepKind::Last;
  }
  const int64_t bucket = graphable ? graph_bucket(rows) : 0;
  if (bucket == 0) graphable = false;

  cache.lend();
  struct GiveBack {
    Cache& c;
    ~GiveBack() { c.give_back(); }
  } give_back{cache};

  const int group = qh_l_ / kvh_l_;
  // Host staging ring: wait until the slot's previous copy has left the pinned buffer.
  const int slot = stage_slot_;
  stage_slot_ ^= 1;
  st->check_cuda(cudaEventSynchronize(stage_done_[slot]), "staging wait");
  TraceScope plan_span("plan", "host", TraceLevel::Debug);
  Plan plan = plan_call(requests, lim, cache.spec(), cache.blocks(), static_cast<int64_t>(adapters.size()), filled, group,
                        graphable ? bucket : 0, host_stage_);
  plan_span.end();
  TraceScope launch_span("stage and launch", "host", TraceLevel::Debug);
  if (pinned_stage_[slot].size() < plan.staged.bytes)
    pinned_stage_[slot] = HostBuffer(std::max<size_t>(plan.staged.bytes * 2, 1 << 16));
  std::memcpy(pinned_stage_[slot].data(), host_stage_.data(), plan.staged.bytes);

  const int64_t splits_needed = plan.decode > 0 ? (plan.max_keys + keys_per_split_ - 1) / keys_per_split_ : 1;
  const int64_t splits = next_pow2(splits_needed);
  ensure_workspace(plan.rows_padded, std::max<int64_t>(plan.kept_padded, 1), splits,
                   plan.segments_padded);
  if (!ws_stage_.valid() || ws_stage_.size() < plan.staged.bytes) {
    ws_stage_ = HbmBuffer(device_, std::max<size_t>(plan.staged.bytes * 2, 1 << 20));
    clear_graphs();
  }
  st->check_cuda(cudaMemcpyAsync(ws_stage_.data(), pinned_stage_[slot].data(), plan.staged.bytes,
                                 cudaMemcpyHostToDevice, st->stream),
                 "stage operands");
  st->check_cuda(cudaEventRecord(stage_done_[slot], st->stream), "staging event");
  plan.max_keys = splits * keys_per_split_;  // the decode grid covers the bucket's splits
  if (coll_) coll_->begin_call(st->stream);

  if (graphable) {
    const GraphKey key{bucket, splits};
    const void* cache_id = cache.layers().empty() ? nullptr : cache.layers()[0].data();
    auto it = graphs_.find(key);
    if (it != graphs_.end() && it->second.cache != cache_id) {
      // The graph reads another cache's layers: capture it again.
      if (it->second.exec) cudaGraphExecDestroy(it->second.exec);
      graphs_.erase(it);
      it = graphs_.end();
    }
    if (it != graphs_.end() && it->second.exec != nullptr) {
      st->check_cuda(cudaGraphLaunch(it->second.exec, st->stream), "graph launch");
      launches_ += it->second.kernels;
    } else if (it == graphs_.end()) {
      // First sight of the shape: run eagerly (configures every kernel), capture next time.
      launches_ += launch(plan, cache);
      GraphEntry e;
      e.cache = cache_id;
      graphs_[key] = e;
    } else {
      cudaGraph_t graph = nullptr;
      st->check_cuda(cudaStreamBeginCapture(st->stream, cudaStreamCaptureModeThreadLocal), "capture");
      const int kernels = launch(plan, cache);
      st->check_cuda(cudaStreamEndCapture(st->stream, &graph), "capture");
      cudaGraphExec_t exec = nullptr;
      st->check_cuda(cudaGraphInstantiate(&exec, graph, 0), "graph instantiate");
      cudaGraphDestroy(graph);
      it->second.exec = exec;
      it->second.kernels = kernels;
      log_event(LogLevel::Debug, "captured a decode graph: " + std::to_string(bucket) + " rows, " +
                                     std::to_string(kernels) + " kernels");
      st->check_cuda(cudaGraphLaunch(exec, st->stream), "graph launch");
      launches_ += kernels;
    }
  } else {
    launches_ += launch(plan, cache);
  }

  launch_span.end();
  // The kept rows' output in its own buffer, so later calls do not overwrite it.
  const int H = cfg_.hidden;
  HbmTensor result = [&]() {
    if (cfg_.output == Output::Tokens) {
      HbmBuffer out(device_, std::max<int64_t>(plan.kept * 4, 8));
      if (plan.kept)
        st->check_cuda(cudaMemcpyAsync(out.data(), ws_tokens_.data(), plan.kept * 4,
                                       cudaMemcpyDeviceToDevice, st->stream),
                       "output copy");
      return HbmTensor(out, {plan.kept}, DType::I32);
    }
    if (cfg_.output == Output::Hidden) {
      HbmBuffer out(device_, std::max<int64_t>(plan.kept * H * 2, 8));
      if (plan.kept)
        st->check_cuda(cudaMemcpyAsync(out.data(), ws_hk_.data(), plan.kept * H * 2,
                                       cudaMemcpyDeviceToDevice, st->stream),
                       "output copy");
      return HbmTensor(out, {plan.kept, H}, DType::BF16);
    }
    HbmBuffer out(device_, std::max<int64_t>(plan.kept * cfg_.labels * 4, 8));
    if (plan.kept)
      st->check_cuda(cudaMemcpyAsync(out.data(), ws_logits_.data(), plan.kept * cfg_.labels * 4,
                                     cudaMemcpyDeviceToDevice, st->stream),
                     "output copy");
    return HbmTensor(out, {plan.kept, cfg_.labels}, DType::F32);
  }();
  if (device_begin != nullptr) {
    cudaEvent_t device_end = Tracer::get().record(st->ordinal, st->stream);
    Tracer::get().device_span("forward.device", "GPU", st->ordinal, device_begin, device_end);
    call_span.args("{\"rows\": " + std::to_string(plan.rows) + ", \"decode\": " + std::to_string(plan.decode) +
                   ", \"prefill\": " + std::to_string(plan.prefill) + "}");
  }
  last_plan_ = std::move(plan);
  return result;
}

// ------------------------------------------------------------------------------------ launch
// One call's launch state: the plan and its staged operands, the stream, the activation buffers
// and the kernel accounting (count, per-kernel trace spans, host-side fault drills).
struct Launch {
  DecoderModel& m;
  const Plan& plan;
  const Cache& cache;
  DeviceState* st;
  cudaStream_t s;
  const ModelConfig& cfg;
  int H, D;
  int64_t T;
  const Staged& sg;
  const HbmBuffer& stage;
  int kernels = 0;
  bool per_kernel;
  cudaEvent_t prev = nullptr;
  __nv_bfloat16* x;  // residual stream [T, H]
  __nv_bfloat16* h;  // normed rows [T, H]
  foa::PagedAttention attn;
  foa::RopeTable rope;

  Launch(DecoderModel& model, const Plan& p, const Cache& c)
      : m(model), plan(p), cache(c), st(model.device_.state().get()), s(st->stream), cfg(model.cfg_),
        H(cfg.hidden), D(cfg.head_dim), T(p.rows_padded), sg(p.staged), stage(model.ws_stage_),
        per_kernel(trace_level() >= TraceLevel::Trace) {
    if (per_kernel) prev = Tracer::get().record(st->ordinal, s);
    // Tensor-parallel ranks keep the residual stream and the normed rows in the symmetric heap,
    // where the fused collectives write them.
    x = m.coll_ ? m.coll_->residual_buffer() : bf(m.ws_x_);
    h = m.coll_ ? m.coll_->hidden_buffer() : bf(m.ws_h_);
    attn.q = bf(m.ws_q_);
    attn.o = bf(m.ws_attn_);
    attn.table = op(sg.table);
    attn.segments = reinterpret_cast<const foa::Segment*>(op(sg.segments));
    attn.q_heads = m.qh_l_;
    attn.kv_heads = m.kvh_l_;
    attn.head_dim = D;
    attn.scale = 1.0f / std::sqrt(static_cast<float>(D));
    attn.partial_o = static_cast<float*>(m.ws_part_o_.data());
    attn.partial_lse = static_cast<float*>(m.ws_part_lse_.data());
    attn.partial_capacity = static_cast<size_t>(m.ws_decode_ * m.qh_l_ * m.ws_splits_);
    attn.max_keys = static_cast<int>(p.max_keys);
    attn.keys_per_split = m.keys_per_split_;
    attn.decode_warps = m.decode_warps_;
    attn.status = st->status;
    attn.rows = static_cast<int>(T);
    attn.cache_blocks = c.blocks();
    // The second half of the counters (the GEMMs use the first): the decode splits' merge.
    attn.merge_counters = i32(m.ws_counters_) + 32768;
    rope = foa::RopeTable{static_cast<const float*>(m.inv_freq_.data()), m.attention_factor_};
  }

  int32_t* op(size_t off) const { return i32(stage, off); }
  const WeightSlot& w(const std::string& n) const { return m.weights_.at(n); }
  __nv_bfloat16* wp(const std::string& n) const { return m.weights_.at(n).ptr; }
  bool tp() const { return m.tp_ > 1; }

  // Accounts for one enqueued kernel (`rc` its launcher's code): a rejected launch poisons the
  // device; at trace level the kernel gets its own device span.
  void done(int rc, const char* what) {
    if (rc == 0 && st->injected("launch")) rc = -5;
    if (rc != 0) st->fail(std::string(what) + " launch rejected (" + std::to_string(rc) + ")");
    ++kernels;
    if (per_kernel) {
      cudaEvent_t now = Tracer::get().record(st->ordinal, s);
      Tracer::get().device_span(what, "GPU", st->ordinal, prev, now);
      prev = now;
    }
  }

  // One projection C = epilogue(A W^T) in the weight's format, with this call's LoRA segments.
  // `external` (non-null): when the plan splits K (decode rows on the swap mapping), the splits'
  // FP32 partials stay in the GEMM workspace for the next kernel to add (*external describes them,
  // splits > 1) and `c` is not written; otherwise *external has one split and the GEMM stores `c`.
  void gemm(const char* gemm_name, const void* a, long lda, const WeightSlot& w, int M, int N, int K, void* c,
            long ldc, int epi, const void* res, int lora_layer = -1, int lora_module = 0,
            foa::GemmSplits* external = nullptr) {
    foa::GemmArgs g;
    // LoRA slots: Z_s = X A_s^T (its rows zeroed outside slot s), added as extra K segments
    // Z_s B_s^T into the projection's FP32 sums.
    int nseg = 0;
    if (lora_layer >= 0) {
      int kpad = 0;
      for (const auto& ad : m.call_adapters_)
        if (ad) kpad = std::max(kpad, ad->factor(lora_layer, lora_module).kpad);
      if (kpad > 0) {
        __nv_bfloat16* z = bf(m.ws_lora_z_);
        const int ldz = 2 * 128;
        for (size_t slot = 0; slot < m.call_adapters_.size(); ++slot) {
          const auto& ad = m.call_adapters_[slot];
          if (!ad) continue;
          const LoraFactor& f = ad->factor(lora_layer, lora_module);
          if (f.kpad == 0) continue;
          foa::GemmArgs sh;
          sh.a = a;
          sh.lda = lda;
          sh.w = f.a.data();
          sh.ldw = K;
          sh.M = M;
          sh.N = f.kpad;
          sh.K = K;
          sh.c = z + slot * 128;
          sh.ldc = ldz;
          sh.status = st->status;
          sh.workspace = static_cast<float*>(m.ws_gemm_.data());
          sh.workspace_bytes = m.ws_gemm_.size();
          sh.counters = i32(m.ws_counters_);
          sh.counters_len = 32768;
          if (m.batch_invariant_) {
            sh.mode = foa::kModeRows;
            sh.splits = 1;
          }
          done(foa::gemm_bf16(sh, s), "lora shrink");
          done(foa::lora_mask(z + slot * 128, ldz, M, f.kpad, static_cast<int>(slot),
                              op(sg.adapters), s),
               "lora mask");
          g.seg[nseg].a = z + slot * 128;
          g.seg[nseg].lda = ldz;
          g.seg[nseg].w = f.b.data();
          g.seg[nseg].ldw = f.kpad;
          g.seg[nseg].K = f.kpad;
          ++nseg;
        }
      }
    }
    g.a = a;
    g.lda = lda;
    g.w = w.format == foa::kWeightBf16 ? static_cast<const void*>(w.ptr) : w.codes;
    g.ldw = K;
    g.w_format = w.format;
    g.w_scale = w.scales;
    g.w_scale_ld = w.scale_ld;
    g.w_scale_rows = w.scale_rows;
    if (w.format == foa::kWeightNvfp4) g.w_tensor_scale = w.tensor_scale;
    if (w.format == foa::kWeightFp8A8) {
      // Inputs quantized per (row, 128-input group) ahead of the FP8 MMA.
      const int pad = (M + 127) / 128 * 128;
      done(foa::quantize_fp8_act(static_cast<const __nv_bfloat16*>(a), lda, M, K, u8(m.ws_qa_), K,
                                 static_cast<float*>(m.ws_qs_.data()), pad, s),
           "input quantization");
      g.a = m.ws_qa_.data();
      g.lda = K;
      g.a_scale = m.ws_qs_.data();
      g.a_scale_ld = pad;
    } else if (w.format == foa::kWeightNvfp4A4) {
      // Inputs quantized under the projection's input scale ahead of the block-scaled MMA.
      done(foa::quantize_nvfp4_act(static_cast<const __nv_bfloat16*>(a), lda, M, K, 1.f / w.input_scale,
                                   u8(m.ws_qa_), K / 2, u8(m.ws_qs_), s),
           "input quantization");
      g.a = m.ws_qa_.data();
      g.lda = K;
      g.a_scale = m.ws_qs_.data();
      g.w_tensor_scale = w.input_scale * w.tensor_scale;
    }
    g.M = M;
    g.N = N;
    g.K = K;
    g.c = c;
    g.ldc = ldc;
    g.residual = res;
    g.ldr = ldc;
    g.epilogue = epi;
    g.workspace = static_cast<float*>(m.ws_gemm_.data());
    g.workspace_bytes = m.ws_gemm_.size();
    g.counters = i32(m.ws_counters_);
    g.counters_len = 32768;  // the first half; the second serves the attention merge
    g.status = st->status;
    if (m.batch_invariant_) {
      // W8A8 SwiGLU tiles only on the swap mapping; its sums do not depend on the tile shape.
      g.mode = (w.format == foa::kWeightFp8A8 && epi == foa::kEpiSwiGLU) ? foa::kModeSwap : foa::kModeRows;
      g.splits = 1;
    }
    if (external != nullptr) {
      *external = foa::gemm_bf16_splits(g);
      g.external_splits = external->splits > 1 ? 1 : 0;
    }
    done(foa::gemm_bf16(g, s), gemm_name);
  }
};

namespace {

std::string layer_prefix(int l) { return "layers." + std::to_string(l) + "."; }
// The norm after layer l's last block: the next layer's input norm, or the final norm.
std::string next_norm(int l, int layers) { return l + 1 < layers ? layer_prefix(l + 1) + "in_norm" : "final_norm"; }

}  // namespace

// The leaf modules of the decoder families (friends of DecoderModel: they read its workspace).
struct DecoderBlocks {
// Token IDs gathered into the call's rows (padded rows read ID 0), then their embedding rows. The
// table is whole on every chip (the head is vocabulary-parallel).
class Embed final : public Module {
 public:
  void forward(Launch& e) const override {
    const int64_t count = std::max<int64_t>(e.plan.requests, e.plan.rows_padded);
    e.done(foa::gather_tokens(e.op(e.sg.sources), static_cast<int>(count), e.op(e.sg.tokens), e.s), "gather tokens");
    e.done(foa::embedding(e.op(e.sg.tokens), e.wp("embed"), e.H, 0, e.cfg.vocab, e.x, e.H, static_cast<int>(e.T),
                          e.H, e.s),
           "embedding");
  }
  std::string name() const override { return "Embed"; }
};

// h = RMSNorm(x) * weight.
class Norm final : public Module {
 public:
  explicit Norm(std::string weight) : weight_(std::move(weight)) {}
  void forward(Launch& e) const override {
    e.done(foa::rmsnorm(e.x, e.H, nullptr, 0, e.wp(weight_), e.h, e.H, nullptr, 0, static_cast<int>(e.T), e.H,
                        e.cfg.eps, e.s),
           "rmsnorm");
  }
  std::string name() const override { return "Norm " + weight_; }

 private:
  std::string weight_;
};

// Packed q/k/v projection of h, then QK-norm, RoPE and the paged K/V store of layer l.
class AttentionFront final : public Module {
 public:
  explicit AttentionFront(int l) : l_(l) {}
  void forward(Launch& e) const override {
    const std::string p = layer_prefix(l_);
    const int cols = (e.m.qh_l_ + 2 * e.m.kvh_l_) * e.D;
    // Decode rows: the GEMM's K splits are added by the next kernel as it reads them.
    foa::GemmSplits sp;
    e.gemm("gemm qkv", e.h, e.H, e.w(p + "qkv"), static_cast<int>(e.T), cols, e.H, e.m.ws_qkv_.data(), cols,
           foa::kEpiBf16, nullptr, l_, LoraAdapter::kQkv, &sp);
    __nv_bfloat16* layer_cache = static_cast<__nv_bfloat16*>(e.cache.layers()[l_].data());
    e.done(foa::qk_norm_rope_cache(bf(e.m.ws_qkv_), cols, static_cast<int>(e.T), e.m.qh_l_, e.m.kvh_l_, e.D,
                                   e.cfg.qk_norm ? e.wp(p + "q_norm") : nullptr,
                                   e.cfg.qk_norm ? e.wp(p + "k_norm") : nullptr, e.cfg.eps, e.op(e.sg.positions),
                                   e.rope, bf(e.m.ws_q_), layer_cache, e.op(e.sg.slots), e.s,
                                   e.cache.blocks() * 16, e.st->status, sp.splits > 1 ? &sp : nullptr),
           "attention front");
    e.attn.cache = layer_cache;
  }
  std::string name() const override { return "AttentionFront (q/k/v, QK-norm, RoPE, KV store)"; }

 private:
  int l_;
};

// Split-KV flash decoding of the call's one-row segments (they come first in the call).
class DecodeAttention final : public Module {
 public:
  void forward(Launch& e) const override {
    e.attn.num_segments = static_cast<int>(e.plan.prefill > 0 ? e.plan.decode : e.plan.segments_padded);
    // The splits merge in the decode kernel while the counters cover the call, else by a second
    // kernel (very large eager calls).
    const bool fused = static_cast<int64_t>(e.attn.num_segments) * e.m.kvh_l_ <= 32768;
    int* counters = e.attn.merge_counters;
    if (!fused) e.attn.merge_counters = nullptr;
    e.done(foa::paged_decode(e.attn, e.s), "decode attention");
    if (!fused && e.plan.max_keys > e.attn.keys_per_split) ++e.kernels;  // the split merge
    e.attn.merge_counters = counters;
  }
  std::string name() const override { return "DecodeAttention"; }
};

// Causal attention of the call's prompt chunks over their history and themselves.
class PrefillAttention final : public Module {
 public:
  void forward(Launch& e) const override {
    e.attn.num_segments = static_cast<int>(e.plan.decode + e.plan.prefill);
    e.done(foa::paged_prefill(e.attn, e.op(e.sg.work), static_cast<int>(e.plan.work), e.s), "prefill attention");
  }
  std::string name() const override { return "PrefillAttention"; }
};

// A row-parallel projection whose output is added to the residual stream and normalised:
// x += A W^T (one rounding), h = RMSNorm(x) * norm. One chip: the GEMM's residual epilogue and a
// norm. Tensor parallelism: the GEMM writes its FP32 partial and the fused collective adds every
// rank's partial in rank order with the residual and the norm.
class ResidualProjection final : public Module {
 public:
  ResidualProjection(const char* trace_name, int l, std::string weight, int lora_module, std::string norm,
                     bool input_is_attention)
      : trace_(trace_name), l_(l), weight_(std::move(weight)), lora_(lora_module), norm_(std::move(norm)),
        attention_(input_is_attention) {}
  void forward(Launch& e) const override {
    const void* a = attention_ ? e.m.ws_attn_.data() : e.m.ws_act_.data();
    const int K = attention_ ? e.m.qh_l_ * e.D : e.m.inter_l_;
    const int M = static_cast<int>(e.T);
    if (!e.tp()) {
      // Decode rows: the norm adds the GEMM's K splits and the residual as it reads them.
      foa::GemmSplits sp;
      e.gemm(trace_, a, K, e.w(weight_), M, e.H, K, e.x, e.H, foa::kEpiBf16, e.x, l_, lora_, &sp);
      if (sp.splits > 1)
        e.done(foa::rmsnorm_splits(sp, e.x, e.H, e.wp(norm_), e.h, e.H, M, e.H, e.cfg.eps, e.s), "rmsnorm");
      else
        e.done(foa::rmsnorm(e.x, e.H, nullptr, 0, e.wp(norm_), e.h, e.H, nullptr, 0, M, e.H, e.cfg.eps, e.s),
               "rmsnorm");
      return;
    }
    // Decode rows: the reducer adds the GEMM's K splits as it scatters them to the peers.
    foa::GemmSplits sp;
    const bool inline_scatter = e.m.coll_->inline_scatter(M);
    e.gemm(trace_, a, K, e.w(weight_), M, e.H, K, e.m.coll_->partial_buffer(), e.H, foa::kEpiF32, nullptr, l_,
           lora_, inline_scatter ? &sp : nullptr);
    if (e.m.coll_->add_norm(e.x, e.wp(norm_), e.cfg.eps, e.h, M, e.H, e.s, sp.splits > 1 ? &sp : nullptr) > 1)
      e.done(0, "tp scatter");
    e.done(0, "tp add_norm");
  }
  std::string name() const override {
    return std::string("ResidualProjection ") + weight_ + " + norm " + norm_ +
           " (under TP: local FP32 partial, scatter to the reducing ranks, rank-ordered sum)";
  }

 private:
  const char* trace_;
  int l_;
  std::string weight_;
  int lora_;
  std::string norm_;
  bool attention_;
};

// gate/up projection of h with the SwiGLU epilogue (act = silu(gate) * up, the intermediate rows).
class GateUp final : public Module {
 public:
  explicit GateUp(int l) : l_(l) {}
  void forward(Launch& e) const override {
    const int I = e.m.inter_l_;
    e.gemm("gemm gate_up", e.h, e.H, e.w(layer_prefix(l_) + "gate_up"), static_cast<int>(e.T), 2 * I, e.H,
           e.m.ws_act_.data(), I, foa::kEpiSwiGLU, nullptr, l_, LoraAdapter::kGateUp);
  }
  std::string name() const override { return "GateUp (SwiGLU epilogue)"; }

 private:
  int l_;
};

// Routed experts of layer l: router GEMM, top-k routing, grouping by expert, the grouped gate/up
// (SwiGLU) and down GEMMs of this rank's experts, then the combine in choice order fused with the
// residual add and the next norm (reading the peers' expert rows under expert parallelism).
class Experts final : public Module {
 public:
  Experts(int l, std::string norm) : l_(l), norm_(std::move(norm)) {}
  void forward(Launch& e) const override {
    DecoderModel& m = e.m;
    const std::string p = layer_prefix(l_);
    const int E = e.cfg.experts, Kc = e.cfg.top_k, I = e.cfg.expert_intermediate, H = e.H;
    const int T = static_cast<int>(e.T);
    const int tile = m.moe_tile(e.T);
    const int64_t cap = m.moe_capacity(e.T);
    e.gemm("gemm router", e.h, H, e.w(p + "router"), T, E, H, m.ws_logits_e_.data(), E, foa::kEpiBf16, nullptr);
    e.done(foa::moe_route(bf(m.ws_logits_e_), E, T, E, Kc, e.cfg.norm_topk, i32(m.ws_ids_),
                          static_cast<float*>(m.ws_rw_.data()), e.s),
           "moe route");
    e.done(foa::moe_align_ranks(i32(m.ws_ids_), T, Kc, E, 0, m.experts_l_, m.tp_, m.rank_, tile, static_cast<int>(cap),
                                i32(m.ws_pos_), i32(m.ws_src_), i32(m.ws_tile_e_), i32(m.ws_tiles_), e.s),
           "moe align");
    e.done(foa::moe_gather(e.h, H, i32(m.ws_src_), i32(m.ws_tiles_), tile, static_cast<int>(cap), H, bf(m.ws_xs_), e.s),
           "moe gather");
    __nv_bfloat16* y = e.tp() ? m.coll_->moe_rows(l_ & 1, static_cast<size_t>(cap)) : bf(m.ws_y_);
    auto grouped = [&](const char* what, const void* a, const WeightSlot& wt, int N, int Kd, void* c, int ldc,
                       int epi) {
      foa::GemmArgs g;
      g.a = a;
      g.lda = Kd;
      g.w = wt.ptr;
      g.ldw = Kd;
      g.M = static_cast<int>(cap);
      g.N = N;
      g.K = Kd;
      g.c = c;
      g.ldc = ldc;
      g.epilogue = epi;
      g.mode = foa::kModeSwap;
      g.status = e.st->status;
      g.group_tiles = i32(m.ws_tiles_);
      g.tile_group = i32(m.ws_tile_e_);
      g.group_tile = tile;
      g.groups = m.experts_l_;
      e.done(foa::gemm_bf16(g, e.s), what);
    };
    grouped("grouped gemm gate_up", m.ws_xs_.data(), e.w(p + "experts_gate_up"), 2 * I, H, m.ws_eact_.data(), I,
            foa::kEpiSwiGLU);
    grouped("grouped gemm down", m.ws_eact_.data(), e.w(p + "experts_down"), H, I, y, H, foa::kEpiBf16);
    if (!e.tp()) {
      e.done(foa::moe_combine_norm(y, H, i32(m.ws_pos_), static_cast<float*>(m.ws_rw_.data()), T, Kc, H, e.x, H,
                                   e.wp(norm_), e.cfg.eps, e.h, H, e.s),
             "moe combine");
    } else {
      m.coll_->moe_combine_norm(l_ & 1, i32(m.ws_pos_), i32(m.ws_ids_), static_cast<float*>(m.ws_rw_.data()),
                                m.experts_l_, e.wp(norm_), e.cfg.eps, T, Kc, H, e.s);
      e.done(0, "tp moe combine");
    }
  }
  std::string name() const override { return "Experts (route, group, grouped SwiGLU GEMMs, combine + norm " + norm_ + ")"; }

 private:
  int l_;
  std::string norm_;
};

// The kept rows' outputs: final-normed hidden rows, label scores, or the first-maximum token of
// the vocabulary-parallel head (candidates exchanged across ranks under tensor parallelism).
class Head final : public Module {
 public:
  explicit Head(Output output) : output_(output) {}
  void forward(Launch& e) const override {
    DecoderModel& m = e.m;
    const int K = static_cast<int>(std::max<int64_t>(e.plan.kept_padded, 0));
    if (K == 0) return;
    e.done(foa::gather_rows(e.h, e.H, e.op(e.sg.kept), K, bf(m.ws_hk_), e.H, e.H, e.s), "gather rows");
    if (output_ == Output::Hidden) return;
    if (output_ == Output::Scores) {
      e.gemm("gemm score", m.ws_hk_.data(), e.H, e.w("score"), K, e.cfg.labels, e.H, m.ws_logits_.data(),
             e.cfg.labels, foa::kEpiF32, nullptr);
      return;
    }
    e.gemm("gemm lm_head", m.ws_hk_.data(), e.H, e.w("lm_head"), K, m.vocab_l_, e.H, m.ws_logits_.data(), m.vocab_l_,
           foa::kEpiF32, nullptr);
    const int valid = m.vocab_end_ - m.vocab_begin_;
    if (!e.tp()) {
      e.done(foa::argmax_rows(static_cast<float*>(m.ws_logits_.data()), m.vocab_l_, K, m.vocab_l_, valid, 0,
                              i32(m.ws_tokens_), nullptr, e.s),
             "argmax");
      return;
    }
    e.done(foa::argmax_rows(static_cast<float*>(m.ws_logits_.data()), m.vocab_l_, K, m.vocab_l_, valid,
                            m.vocab_begin_, i32(m.ws_idx_), static_cast<float*>(m.ws_val_.data()), e.s),
           "argmax");
    m.coll_->argmax(static_cast<float*>(m.ws_val_.data()), i32(m.ws_idx_), K, i32(m.ws_tokens_), e.s);
    e.done(0, "tp argmax");
  }
  std::string name() const override {
    return output_ == Output::Hidden ? "Head (hidden rows)"
           : output_ == Output::Scores ? "Head (label scores)"
                                       : "Head (vocabulary-parallel greedy token)";
  }

 private:
  Output output_;
};

  static ModulePtr build(const ModelConfig& cfg);
};

// The decoder families' launch program: embedding, then per layer the attention block (front,
// decode and prefill attention as the call holds them, output projection + residual + norm) and
// the feed-forward block (SwiGLU MLP, or routed experts), then the head.
ModulePtr DecoderBlocks::build(const ModelConfig& cfg) {
  auto prog = std::make_unique<Sequential>(cfg.family + " decoder");
  prog->then(std::make_unique<Embed>());
  prog->then(std::make_unique<Norm>("layers.0.in_norm"));
  prog->then(std::make_unique<Layers>(cfg.layers, [&](int l) -> ModulePtr {
    const std::string p = layer_prefix(l), next = next_norm(l, cfg.layers);
    auto layer = std::make_unique<Sequential>("Layer");
    auto attention = std::make_unique<Sequential>("Attention");
    attention->then(std::make_unique<AttentionFront>(l));
    attention->then(std::make_unique<Choice>(
        "decode rows", [](const Launch& e) { return e.plan.decode > 0; }, std::make_unique<DecodeAttention>()));
    attention->then(std::make_unique<Choice>(
        "prompt chunks", [](const Launch& e) { return e.plan.prefill > 0; }, std::make_unique<PrefillAttention>()));
    attention->then(std::make_unique<ResidualProjection>("gemm o", l, p + "o", LoraAdapter::kO, p + "post_norm", true));
    layer->then(std::move(attention));
    if (cfg.experts > 0) {
      layer->then(std::make_unique<Experts>(l, next));
    } else {
      auto mlp = std::make_unique<Sequential>("MLP");
      mlp->then(std::make_unique<GateUp>(l));
      mlp->then(std::make_unique<ResidualProjection>("gemm down", l, p + "down", LoraAdapter::kDown, next, false));
      layer->then(std::move(mlp));
    }
    return layer;
  }));
  prog->then(std::make_unique<Head>(cfg.output));
  return prog;
}

int DecoderModel::launch(const Plan& plan, const Cache& cache) {
  if (!program_) program_ = DecoderBlocks::build(cfg_);
  Launch env(*this, plan, cache);
  program_->forward(env);
  return env.kernels;
}

std::string DecoderModel::describe() const {
  std::string out;
  if (program_) program_->describe(out, 0);
  else DecoderBlocks::build(cfg_)->describe(out, 0);
  return out;
}

}  // namespace foa::engine
