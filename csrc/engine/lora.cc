#include "lora.h"

#include <cmath>
#include <cstring>
#include <map>
#include <set>

namespace foa::engine {

namespace {

[[noreturn]] void invalid(const std::string& where, const std::string& why) { throw ValueError(where + ": " + why); }
[[noreturn]] void unsupported(const std::string& what, const std::string& why) { throw Unsupported(what + ": " + why); }

uint16_t to_bf16(float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  if ((b & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((b >> 16) | 0x40);
  b += 0x7fffu + ((b >> 16) & 1u);
  return static_cast<uint16_t>(b >> 16);
}

float value(const StoredTensor* t, int64_t i) {
  const uint8_t* p = t->data();
  switch (t->dtype) {
    case StDType::BF16: {
      uint16_t h;
      std::memcpy(&h, p + i * 2, 2);
      const uint32_t b = static_cast<uint32_t>(h) << 16;
      float f;
      std::memcpy(&f, &b, 4);
      return f;
    }
    case StDType::F32: {
      float f;
      std::memcpy(&f, p + i * 4, 4);
      return f;
    }
    case StDType::F16: {
      uint16_t h;
      std::memcpy(&h, p + i * 2, 2);
      const uint32_t s = (h & 0x8000u) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ff;
      if (e == 0) return (s ? -1.f : 1.f) * std::ldexp(static_cast<float>(m), -24);
      uint32_t b = e == 31 ? (s | 0x7f800000u | (m << 13)) : (s | ((e + 112) << 23) | (m << 13));
      float f;
      std::memcpy(&f, &b, 4);
      return f;
    }
    default:
      invalid(t->file, std::string("a LoRA factor of dtype ") + st_dtype_name(t->dtype) + " does not load");
  }
}

}  // namespace

LoraAdapter::LoraAdapter(const DecoderModel& model, const Checkpoint& ck) : owner_(&model) {
  const ModelConfig& cfg = model.config();
  if (model.limits().adapters == 0) unsupported("adapters", "the decoder was loaded without adapters");
  if (cfg.weight_format != "bf16" || cfg.experts > 0)
    unsupported("adapters", "adapters update dense BF16 projections");
  const Json& c = ck.config();
  const int64_t r = c["r"].is_number() ? static_cast<int64_t>(c["r"].as_double()) : 8;
  if (r <= 0) invalid("adapter_config.json:r", "not a positive rank");
  if (r > kRank) unsupported("r", std::to_string(r) + ", past the rank " + std::to_string(kRank) + " a term holds");
  if (c["use_dora"].is_bool() && c["use_dora"].as_bool()) unsupported("use_dora", "DoRA updates are not served");
  if (c["bias"].is_string() && c["bias"].as_string() != "none") unsupported("bias", "adapters without biases");
  for (const char* k : {"rank_pattern", "alpha_pattern"})
    if (c[k].is_object() && c[k].size() > 0) unsupported(k, "one rank and scale for every module");
  if (c["layers_to_transform"].is_array() || c["layers_to_transform"].is_number())
    unsupported("layers_to_transform", "adapters cover every layer they name tensors for");
  const double alpha = c["lora_alpha"].is_number() ? c["lora_alpha"].as_double() : static_cast<double>(r);
  const bool rslora = c["use_rslora"].is_bool() && c["use_rslora"].as_bool();
  const float scale = static_cast<float>(rslora ? alpha / std::sqrt(static_cast<double>(r)) : alpha / static_cast<double>(r));

  const int H = cfg.hidden, D = cfg.head_dim;
  const int qh = model.q_heads_local(), kvh = model.kv_heads_local();
  const int qh0 = model.q_head_first(), kvh0 = model.kv_head_first();
  const int inter = model.intermediate_local(), rank = model.rank();
  std::set<std::string> used;
  auto find = [&](int l, const std::string& path, const char* ab) -> const StoredTensor* {
    for (const std::string pre : {"base_model.model.model.layers.", "base_model.model.layers.", "model.layers."}) {
      const std::string n = pre + std::to_string(l) + "." + path + ".lora_" + ab + ".weight";
      if (const StoredTensor* t = ck.get(n)) {
        used.insert(n);
        return t;
      }
    }
    return nullptr;
  };
  // One part: lora_A [r, in_full], lora_B [out_full, r].
  struct Part {
    const StoredTensor *a = nullptr, *b = nullptr;
  };
  auto part = [&](int l, const std::string& path, int64_t in_full, int64_t out_full) {
    Part p{find(l, path, "A"), find(l, path, "B")};
    if ((p.a == nullptr) != (p.b == nullptr)) invalid(path, "lora_A and lora_B come in pairs");
    if (p.a && (p.a->shape != std::vector<int64_t>{r, in_full} || p.b->shape != std::vector<int64_t>{out_full, r}))
      invalid(path, "factors of another shape than r x in and out x r");
    return p;
  };
  auto st = model.device().state();
  auto upload = [&](HbmBuffer& dst, const std::vector<uint16_t>& host) {
    dst = HbmBuffer(model.device(), host.size() * 2);
    st->check_cuda(cudaMemcpy(dst.data(), host.data(), host.size() * 2, cudaMemcpyHostToDevice), "adapter upload");
  };
  // Builds one fused module from its parts: part i occupies A rows and B columns [32 i, 32 i + r).
  // a_cols: [col0, n) of the part's input columns this rank reads; out_rows[i]: (source row of
  // each local output row, or -1) for part i.
  auto build = [&](LoraFactor& f, const std::vector<Part>& parts, int64_t in_local, int64_t a_col0,
                   const std::vector<std::vector<int64_t>>& out_rows, int64_t out_local) {
    bool any = false;
    for (const Part& p : parts) any = any || p.a;
    if (!any) return;
    const int kpad = (static_cast<int>(parts.size()) * kRank + 63) / 64 * 64;
    std::vector<uint16_t> A(static_cast<size_t>(kpad) * in_local, 0), B(static_cast<size_t>(out_local) * kpad, 0);
    for (size_t i = 0; i < parts.size(); ++i) {
      const Part& p = parts[i];
      if (!p.a) continue;
      const int64_t in_full = p.a->shape[1];
      for (int64_t j = 0; j < r; ++j)
        for (int64_t c = 0; c < in_local; ++c)
          A[(i * kRank + j) * in_local + c] = to_bf16(value(p.a, j * in_full + a_col0 + c));
      for (int64_t o = 0; o < out_local; ++o) {
        const int64_t src = out_rows[i][o];
        if (src < 0) continue;
        for (int64_t j = 0; j < r; ++j)
          B[o * kpad + i * kRank + j] = to_bf16(value(p.b, src * r + j) * scale);
      }
    }
    f.kpad = kpad;
    f.in = static_cast<int>(in_local);
    f.out = static_cast<int>(out_local);
    upload(f.a, A);
    upload(f.b, B);
  };
  layers_.resize(cfg.layers);
  const int64_t qrows = static_cast<int64_t>(cfg.q_heads) * D, kvrows = static_cast<int64_t>(cfg.kv_heads) * D;
  const int64_t qkv_local = static_cast<int64_t>(qh + 2 * kvh) * D;
  for (int l = 0; l < cfg.layers; ++l) {
    // q/k/v: column-parallel; local rows: this rank's q heads, then its k and v heads.
    std::vector<std::vector<int64_t>> rows(3, std::vector<int64_t>(qkv_local, -1));
    for (int64_t o = 0; o < qkv_local; ++o) {
      if (o < qh * D) rows[0][o] = static_cast<int64_t>(qh0) * D + o;
      else if (o < (qh + kvh) * D) rows[1][o] = static_cast<int64_t>(kvh0) * D + (o - qh * D);
      else rows[2][o] = static_cast<int64_t>(kvh0) * D + (o - (qh + kvh) * D);
    }
    build(layers_[l][kQkv],
          {part(l, "self_attn.q_proj", H, qrows), part(l, "self_attn.k_proj", H, kvrows),
           part(l, "self_attn.v_proj", H, kvrows)},
          H, 0, rows, qkv_local);
    // o: row-parallel; this rank's input columns, every output row.
    std::vector<std::vector<int64_t>> all_h(1, std::vector<int64_t>(H));
    for (int64_t o = 0; o < H; ++o) all_h[0][o] = o;
    build(layers_[l][kO], {part(l, "self_attn.o_proj", qrows, H)}, static_cast<int64_t>(qh) * D,
          static_cast<int64_t>(qh0) * D, all_h, H);
    if (cfg.experts == 0) {
      // gate/up: column-parallel, rows alternate gate and up in 128-row blocks.
      const int64_t gu_local = 2L * inter;
      std::vector<std::vector<int64_t>> gu(2, std::vector<int64_t>(gu_local, -1));
      for (int64_t o = 0; o < gu_local; ++o) {
        const int64_t block = o / 256, within = o % 256;
        const int64_t src = static_cast<int64_t>(rank) * inter + block * 128 + within % 128;
        gu[within < 128 ? 0 : 1][o] = src;
      }
      build(layers_[l][kGateUp],
            {part(l, "mlp.gate_proj", H, cfg.intermediate), part(l, "mlp.up_proj", H, cfg.intermediate)}, H, 0, gu,
            gu_local);
      build(layers_[l][kDown], {part(l, "mlp.down_proj", cfg.intermediate, H)}, inter,
            static_cast<int64_t>(rank) * inter, all_h, H);
    }
  }
  for (const auto& n : ck.names())
    if (!used.count(n)) invalid("checkpoint", "the adapter holds a tensor no adapted module reads: " + n);
}

}  // namespace foa::engine
