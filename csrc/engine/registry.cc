#include "registry.h"

#include "encoder.h"

#include "kernels/gemm.cuh"
#include "kernels/quant.cuh"

#include <cmath>
#include <cstring>
#include <map>

namespace foa::engine {

void LoadRefusal::raise() const {
  const std::string msg = name + ": " + reason;
  if (unsupported) throw Unsupported(msg);
  throw ValueError(msg);
}

namespace {

[[noreturn]] void invalid(const std::string& name, const std::string& reason) {
  LoadRefusal{false, name, reason}.raise();
}
[[noreturn]] void unsupported(const std::string& name, const std::string& reason) {
  LoadRefusal{true, name, reason}.raise();
}

const std::vector<std::string> kNames = {
#include "architectures.inc"
};

// ------------------------------------------------------------------------------------ config
int64_t need_int(const Json& c, const char* key) {
  const Json& v = c[key];
  if (!v.is_number()) invalid(std::string("config.json:") + key, "missing or not a number");
  return v.as_int();
}

double get_num(const Json& c, const char* key, double def) {
  const Json& v = c[key];
  return v.is_number() ? v.as_double() : def;
}

bool get_bool(const Json& c, const char* key, bool def) {
  const Json& v = c[key];
  return v.is_bool() ? v.as_bool() : def;
}

RopeSpec rope_of(const Json& c, double default_theta) {
  RopeSpec r;
  r.theta = get_num(c, "rope_theta", default_theta);
  const Json* s = &c["rope_scaling"];
  if (s->is_null() && c["rope_parameters"].is_object()) s = &c["rope_parameters"];
  if (s->is_object()) {
    std::string type = (*s)["rope_type"].is_string() ? (*s)["rope_type"].as_string()
                       : (*s)["type"].is_string()    ? (*s)["type"].as_string()
                                                     : "default";
    if ((*s)["rope_theta"].is_number()) r.theta = (*s)["rope_theta"].as_double();
    if (type == "dynamic" || type == "longrope" || type == "mrope")
      unsupported("rope_scaling", type + " scaling is not served");
    if (type != "default" && type != "linear" && type != "llama3" && type != "yarn")
      unsupported("rope_scaling", "unknown rope type " + type);
    r.type = type;
    r.factor = get_num(*s, "factor", 1.0);
    r.low_freq_factor = get_num(*s, "low_freq_factor", 1.0);
    r.high_freq_factor = get_num(*s, "high_freq_factor", 4.0);
    r.original_max_positions =
        get_num(*s, "original_max_position_embeddings", get_num(c, "max_position_embeddings", 0));
    r.beta_fast = get_num(*s, "beta_fast", 32.0);
    r.beta_slow = get_num(*s, "beta_slow", 1.0);
    r.mscale = get_num(*s, "mscale", 1.0);
    r.mscale_all_dim = get_num(*s, "mscale_all_dim", 0.0);
    r.attention_factor = get_num(*s, "attention_factor", 0.0);
    r.truncate = get_bool(*s, "truncate", true);
  }
  return r;
}

struct KnownSize {
  const char* family;
  const char* size;
  int hidden, intermediate, layers, q_heads, kv_heads;
};
// Published geometries of the checkpoints each family serves by name.
const KnownSize kSizes[] = {
    {"qwen3", "0.6B", 1024, 3072, 28, 16, 8},   {"qwen3", "1.7B", 2048, 6144, 28, 16, 8},
    {"qwen3", "4B", 2560, 9728, 36, 32, 8},     {"qwen3", "8B", 4096, 12288, 36, 32, 8},
    {"qwen3", "14B", 5120, 17408, 40, 40, 8},   {"qwen3", "32B", 5120, 25600, 64, 64, 8},
    {"llama", "1B", 2048, 8192, 16, 32, 8},     {"llama", "3B", 3072, 8192, 28, 24, 8},
    {"llama", "8B", 4096, 14336, 32, 32, 8},    {"llama", "70B", 8192, 28672, 80, 64, 8},
    {"mistral", "7B", 4096, 14336, 32, 32, 8},  {"mistral", "12B", 5120, 14336, 40, 32, 8},
    {"qwen3_moe", "30B-A3B", 2048, 6144, 48, 32, 4}, {"qwen3_moe", "235B-A22B", 4096, 12288, 94, 64, 4},
    {"mixtral", "8x7B", 4096, 14336, 32, 32, 8},  {"mixtral", "8x22B", 6144, 16384, 56, 48, 8},
};

std::string size_of(const std::string& family, const ModelConfig& m) {
  for (const auto& k : kSizes)
    if (family == k.family && m.hidden == k.hidden && m.layers == k.layers &&
        m.q_heads == k.q_heads && m.kv_heads == k.kv_heads &&
        (family == "qwen3_moe" || m.intermediate == k.intermediate))
      return k.size;
  return "custom";
}

// The decoder geometry every family shares, from an HF config.
ModelConfig decoder_config(const Checkpoint& ck, const std::string& family, double theta, float eps_default) {
  const Json& c = ck.config();
  ModelConfig m;
  m.family = family;
  m.hidden = static_cast<int>(need_int(c, "hidden_size"));
  m.layers = static_cast<int>(need_int(c, "num_hidden_layers"));
  m.q_heads = static_cast<int>(need_int(c, "num_attention_heads"));
  m.kv_heads = c["num_key_value_heads"].is_number() ? static_cast<int>(c["num_key_value_heads"].as_int())
                                                   : m.q_heads;
  m.head_dim = c["head_dim"].is_number() ? static_cast<int>(c["head_dim"].as_int()) : m.hidden / m.q_heads;
  m.vocab = static_cast<int>(need_int(c, "vocab_size"));
  m.intermediate = c["intermediate_size"].is_number() ? static_cast<int>(c["intermediate_size"].as_int()) : 0;
  m.eps = static_cast<float>(get_num(c, "rms_norm_eps", eps_default));
  m.tied = get_bool(c, "tie_word_embeddings", false);
  m.rope = rope_of(c, theta);
  const int64_t positions = c["max_position_embeddings"].is_number() ? c["max_position_embeddings"].as_int() : 32768;
  m.window = static_cast<int>(std::min<int64_t>(positions, 131072));
  m.rows = 8192;
  if (m.head_dim != 64 && m.head_dim != 128)
    unsupported("head_dim", std::to_string(m.head_dim) + ", the attention kernels hold 64 or 128");
  if (m.q_heads % m.kv_heads != 0 || m.q_heads / m.kv_heads > 16)
    unsupported("num_key_value_heads", "query heads do not group evenly over at most 16 per key/value head");
  if (m.hidden % 64 != 0) unsupported("hidden_size", "not a multiple of 64");
  if (get_bool(c, "attention_bias", false)) unsupported("attention_bias", family + " projects without biases");
  if (get_bool(c, "mlp_bias", false)) unsupported("mlp_bias", family + " projects without biases");
  return m;
}

// ------------------------------------------------------------------------------------ scopes
ModelConfig qwen3_scope(const Checkpoint& ck, Output output, const std::string& form) {
  ModelConfig m = decoder_config(ck, "qwen3", 1000000.0, 1e-6f);
  const Json& c = ck.config();
  m.qk_norm = true;
  if (get_bool(c, "use_sliding_window", false))
    unsupported("use_sliding_window", "Qwen3 attends the whole history");
  const Json& q = ck.declaration();
  if (form == "bf16" && !q.is_null() && ck.quantization().empty())
    unsupported("quantization_config", "the BF16 line reads unquantized checkpoints");
  if (form == "fp8_block") {
    if (q.is_null() || !q["weight_block_size"].is_array())
      invalid("config.json:quantization_config", "not a block-scaled FP8 declaration");
    m.precision = "float8_e4m3fn";
  }
  if (m.intermediate % 128 != 0) unsupported("intermediate_size", "not a multiple of 128");
  m.output = output;
  if (output == Output::Scores) m.labels = 256;
  m.size = size_of("qwen3", m);
  return m;
}

ModelConfig llama_scope(const Checkpoint& ck, const std::string& family, const std::string& form) {
  ModelConfig m = decoder_config(ck, family, family == "mistral" ? 1000000.0 : 500000.0, 1e-5f);
  const Json& c = ck.config();
  if (family == "mistral" && c["sliding_window"].is_number())
    unsupported("sliding_window", "Mistral attends the whole history here");
  const Json& q = ck.declaration();
  if (form == "bf16" && !q.is_null() && ck.quantization().empty())
    unsupported("quantization_config", "the BF16 line reads unquantized checkpoints");
  if (form == "nvfp4") {
    const bool nvfp4 = q.is_object() && ((q["quant_algo"].is_string() && q["quant_algo"].as_string() == "NVFP4") ||
                                         (q["quantization"].is_object() && q["quantization"]["quant_algo"].is_string() &&
                                          q["quantization"]["quant_algo"].as_string() == "NVFP4"));
    if (!nvfp4) invalid("config.json:quantization_config", "not an NVFP4 declaration");
    m.precision = "uint8";
  }
  if (form == "fp8_block") {
    if (q.is_null() || !q["weight_block_size"].is_array())
      invalid("config.json:quantization_config", "not a block-scaled FP8 declaration");
    m.precision = "float8_e4m3fn";
  }
  if (form == "fp8_static") {
    // Static per-tensor FP8 (Mistral NeMo FP8 and the like): E4M3 codes with one weight_scale a
    // projection; the input_scale a static scheme calibrates is read and the inputs stay BF16.
    const bool fp8 = q.is_object() && q["quant_method"].is_string() && q["quant_method"].as_string() == "fp8";
    if (!fp8 || q["weight_block_size"].is_array() || !q["activation_scheme"].is_string() ||
        q["activation_scheme"].as_string() != "static")
      invalid("config.json:quantization_config", "not a static per-tensor FP8 declaration");
    m.precision = "float8_e4m3fn";
  }
  if (m.intermediate % 128 != 0) unsupported("intermediate_size", "not a multiple of 128");
  m.size = size_of(family, m);
  return m;
}

ModelConfig qwen3_moe_scope(const Checkpoint& ck) {
  ModelConfig m = decoder_config(ck, "qwen3_moe", 1000000.0, 1e-6f);
  const Json& c = ck.config();
  m.qk_norm = true;
  m.experts = static_cast<int>(need_int(c, "num_experts"));
  m.top_k = static_cast<int>(need_int(c, "num_experts_per_tok"));
  m.expert_intermediate = static_cast<int>(need_int(c, "moe_intermediate_size"));
  m.norm_topk = get_bool(c, "norm_topk_prob", true);
  if (c["mlp_only_layers"].is_array() && c["mlp_only_layers"].size() > 0)
    unsupported("mlp_only_layers", "every layer routes to experts here");
  if (get_num(c, "decoder_sparse_step", 1) != 1) unsupported("decoder_sparse_step", "every layer routes to experts here");
  if (!ck.declaration().is_null()) unsupported("quantization_config", "the MoE line reads BF16 checkpoints");
  m.size = size_of("qwen3_moe", m);
  m.precision = "bfloat16";
  return m;
}

// Mixtral: Llama attention (no QK-norm) and a routed SwiGLU of num_local_experts experts a layer,
// softmax over every expert then the top num_experts_per_tok renormalised (the routing of the MoE
// line with its top-k weights normalised); intermediate_size is an expert's width.
ModelConfig mixtral_scope(const Checkpoint& ck) {
  ModelConfig m = decoder_config(ck, "mixtral", 1000000.0, 1e-5f);
  const Json& c = ck.config();
  if (c["sliding_window"].is_number()) unsupported("sliding_window", "Mixtral attends the whole history here");
  m.experts = static_cast<int>(need_int(c, "num_local_experts"));
  m.top_k = static_cast<int>(need_int(c, "num_experts_per_tok"));
  m.expert_intermediate = m.intermediate;
  m.norm_topk = true;
  if (m.expert_intermediate % 128 != 0) unsupported("intermediate_size", "not a multiple of 128");
  if (get_num(c, "router_jitter_noise", 0.0) != 0.0) unsupported("router_jitter_noise", "routing is deterministic here");
  if (!ck.declaration().is_null()) unsupported("quantization_config", "the MoE line reads BF16 checkpoints");
  m.size = size_of("mixtral", m);
  m.precision = "bfloat16";
  return m;
}

Implementation make(const char* family, const char* cls, const char* form, Output out,
                    std::function<ModelConfig(const Checkpoint&)> scope) {
  Implementation i;
  i.family = family;
  i.cls = cls;
  i.form = form;
  i.output = out;
  i.scope = std::move(scope);
  // Dense BF16 decoders take LoRA adapters (two slots a call).
  const bool moe = std::string(family) == "qwen3_moe" || std::string(family) == "mixtral";
  i.adapters = (std::string(form) == "bf16" && !moe && out != Output::Scores) ? 2 : 0;
  return i;
}

const std::map<std::string, std::vector<Implementation>>& served() {
  static const std::map<std::string, std::vector<Implementation>> table = [] {
    std::map<std::string, std::vector<Implementation>> t;
    t["Qwen3ForCausalLM"] = {
        make("qwen3", "qwen3.ForCausalLM", "bf16", Output::Tokens,
             [](const Checkpoint& c) { return qwen3_scope(c, Output::Tokens, "bf16"); }),
        make("qwen3", "qwen3.ForCausalLM", "fp8_block", Output::Tokens,
             [](const Checkpoint& c) { return qwen3_scope(c, Output::Tokens, "fp8_block"); }),
    };
    t["Qwen3ForSequenceClassification"] = {
        make("qwen3", "qwen3.ForSequenceClassification", "bf16", Output::Scores,
             [](const Checkpoint& c) { return qwen3_scope(c, Output::Scores, "bf16"); })};
    t["Qwen3Model"] = {make("qwen3", "qwen3.Model", "bf16", Output::Hidden,
                            [](const Checkpoint& c) { return qwen3_scope(c, Output::Hidden, "bf16"); })};
    t["LlamaForCausalLM"] = {
        make("llama", "llama.ForCausalLM", "bf16", Output::Tokens,
             [](const Checkpoint& c) { return llama_scope(c, "llama", "bf16"); }),
        make("llama", "llama.ForCausalLM", "nvfp4", Output::Tokens,
             [](const Checkpoint& c) { return llama_scope(c, "llama", "nvfp4"); }),
        make("llama", "llama.ForCausalLM", "fp8_block", Output::Tokens,
             [](const Checkpoint& c) { return llama_scope(c, "llama", "fp8_block"); }),
        make("llama", "llama.ForCausalLM", "fp8_static", Output::Tokens,
             [](const Checkpoint& c) { return llama_scope(c, "llama", "fp8_static"); }),
    };
    t["MistralForCausalLM"] = {
        make("mistral", "mistral.ForCausalLM", "bf16", Output::Tokens,
             [](const Checkpoint& c) { return llama_scope(c, "mistral", "bf16"); }),
        make("mistral", "mistral.ForCausalLM", "fp8_static", Output::Tokens,
             [](const Checkpoint& c) { return llama_scope(c, "mistral", "fp8_static"); }),
    };
    t["Qwen3MoeForCausalLM"] = {make("qwen3_moe", "qwen3_moe.ForCausalLM", "bf16", Output::Tokens,
                                     [](const Checkpoint& c) { return qwen3_moe_scope(c); })};
    t["MixtralForCausalLM"] = {make("mixtral", "mixtral.ForCausalLM", "bf16", Output::Tokens,
                                    [](const Checkpoint& c) { return mixtral_scope(c); })};
    // Gemma 4 unified's media embedders, loaded alone (registry.rs:571): an Encoder.
    t["Gemma4UnifiedForConditionalGeneration"] = {
        make("gemma4_unified", "Encoder", "bf16", Output::Hidden, [](const Checkpoint& c) {
          const EncoderConfig e = encoder_config(c);
          ModelConfig m;
          m.family = "gemma4_unified";
          m.size = e.size;
          m.hidden = e.text;
          return m;
        })};
    return t;
  }();
  return table;
}

}  // namespace

const std::vector<std::string>& architecture_names() { return kNames; }

Listed listed(const std::vector<std::string>& names) {
  for (const auto& n : names) {
    for (const auto& k : kNames) {
      if (k != n) continue;
      Listed l;
      l.name = k;
      auto it = served().find(k);
      if (it == served().end() || it->second.empty()) unsupported(k, "no model type is implemented");
      for (const auto& i : it->second) l.implementations.push_back(&i);
      return l;
    }
  }
  std::string joined;
  for (size_t i = 0; i < names.size(); ++i) joined += (i ? ", " : "") + names[i];
  invalid(joined, "unknown architecture");
}

const Implementation* choose(const Listed& l, const Checkpoint& c, ModelConfig* config) {
  std::vector<std::pair<const Implementation*, ModelConfig>> ok;
  std::vector<std::pair<bool, std::string>> refused;
  for (const Implementation* i : l.implementations) {
    try {
      ModelConfig m = i->scope(c);
      ok.emplace_back(i, m);
    } catch (const Unsupported& e) {
      refused.emplace_back(true, e.what());
    } catch (const ValueError& e) {
      refused.emplace_back(false, e.what());
    }
  }
  if (ok.size() == 1) {
    *config = ok[0].second;
    config->architecture = l.name;
    return ok[0].first;
  }
  if (ok.empty() && refused.size() == 1) {
    if (refused[0].first) throw Unsupported(refused[0].second);
    throw ValueError(refused[0].second);
  }
  if (ok.empty()) {
    // Report the refusal of the line that reads the checkpoint's own form first.
    for (const auto& r : refused)
      if (r.first) throw Unsupported(r.second);
    std::string joined;
    for (size_t i = 0; i < refused.size(); ++i) joined += (i ? "; " : "") + refused[i].second;
    invalid(l.name, "no implementation serves the checkpoint: " + joined);
  }
  std::string sizes;
  for (size_t i = 0; i < ok.size(); ++i) sizes += (i ? "; " : "") + ok[i].second.size;
  invalid(l.name, "implementations of sizes " + sizes + " all serve the checkpoint");
}

Selection select(const LoadOptions& o, const Checkpoint& ck) {
  std::vector<std::string> names;
  if (o.architecture) {
    names.push_back(*o.architecture);
  } else {
    for (const auto& a : ck.config()["architectures"].items())
      if (a.is_string()) names.push_back(a.as_string());
    if (ck.config()["_class_name"].is_string()) names.push_back(ck.config()["_class_name"].as_string());
  }
  if (names.empty()) invalid("config.json:architectures", "the config names no architecture");
  const Listed l = listed(names);
  Selection s;
  s.architecture = l.name;
  const Checkpoint* read = &ck;
  Checkpoint quantized;
  if (o.quantization) {
    quantized = ck.quantized(*o.quantization == "fp8_per_tensor" ? "tensor" : "channel");
    read = &quantized;
  }
  s.implementation = choose(l, *read, &s.config);
  // A media encoder loads alone, and a decoder holds none that does (the reference's
  // `Listed::reads(Part)`: vision_language/gemma4_unified.rs:25-33 and the decoders').
  const bool encoder = s.implementation->family == "gemma4_unified";
  if (encoder && !o.encoder) unsupported("encoder", "a media encoder loads alone, so choose the encoder");
  if (!encoder && o.encoder) unsupported("encoder", "a decoder holds no media encoder that loads alone");
  if (encoder) {
    s.chips = o.chips.value_or(1);
    if (s.chips != 1) unsupported("chips", "a media encoder runs on one chip");
    if (o.adapters) unsupported("adapters", "a media encoder takes no adapters");
    return s;
  }
  const ModelConfig& m = s.config;
  s.chips = o.chips.value_or(1);
  if (s.chips != 1 && s.chips != 2 && s.chips != 4 && s.chips != 8)
    unsupported("chips", "a load runs on 1, 2, 4 or 8 chips");
  if (s.chips > 1) {
    const int inter = m.experts > 0 ? 128 * s.chips : m.intermediate;
    const bool split = m.q_heads % s.chips == 0 &&
                       (m.kv_heads % s.chips == 0 || s.chips % m.kv_heads == 0) &&
                       inter % s.chips == 0 && (inter / s.chips) % 128 == 0;
    if (!split)
      unsupported("chips", "the " + l.name + " " + m.size + " geometry does not split over " +
                               std::to_string(s.chips) + " chips");
  }
  if (o.kv_cache && *o.kv_cache != "bfloat16")
    unsupported("kv_cache", "every implementation caches keys and values in BF16");
  if (o.layers) unsupported("layers", "every implementation loads whole");
  if (o.adapters && s.implementation->adapters == 0)
    unsupported("adapters", "the " + l.name + " " + m.size + " implementation takes no adapter");
  if (o.quantization) {
    if (s.implementation->form != "bf16" || m.experts > 0)
      unsupported("quantization", "load-time FP8 quantization reads dense BF16 checkpoints");
    s.config.weight_format = *o.quantization == "fp8_per_tensor" ? "fp8_tensor" : "fp8_channel";
  }
  if (s.implementation->form == "fp8_block") s.config.weight_format = "fp8_block";
  if (s.implementation->form == "fp8_static") s.config.weight_format = "fp8_static";
  if (s.implementation->form == "nvfp4") {
    // ModelOpt NVFP4 checkpoints with calibrated input scales run W4A4 on the block-scaled MMA;
    // without them (or with FOA_NVFP4_W4A16=1) the inputs stay BF16 (W4A16).
    const char* a16 = std::getenv("FOA_NVFP4_W4A16");
    const bool inputs = ck.get("model.layers.0.self_attn.q_proj.input_scale") != nullptr;
    s.config.weight_format = (inputs && !(a16 && a16[0] == '1')) ? "nvfp4_a4" : "nvfp4";
  }
  if (m.experts > 0 && m.experts % s.chips != 0)
    unsupported("chips", "the " + std::to_string(m.experts) + " experts do not split over " +
                             std::to_string(s.chips) + " chips");
  return s;
}

// ------------------------------------------------------------------------------------ weights
namespace {

uint16_t f32_to_bf16(float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  if ((b & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((b >> 16) | 0x40);  // NaN
  b += 0x7fffu + ((b >> 16) & 1u);
  return static_cast<uint16_t>(b >> 16);
}

float f16_to_f32(uint16_t h) {
  const uint32_t s = (h & 0x8000u) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ff;
  uint32_t b;
  if (e == 0) {
    if (m == 0) {
      b = s;
    } else {  // subnormal
      float f = std::ldexp(static_cast<float>(m), -24);
      std::memcpy(&b, &f, 4);
      b |= s;
    }
  } else if (e == 31) {
    b = s | 0x7f800000u | (m << 13);
  } else {
    b = s | ((e + 112) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

// Element (r, c) of a 2-D (or 1-D) checkpoint tensor as BF16 bits.
struct Source {
  const StoredTensor* t;
  int64_t rows, cols;
  Source(const StoredTensor* s) : t(s) {
    rows = s->shape.size() == 2 ? s->shape[0] : 1;
    cols = s->shape.empty() ? 1 : s->shape.back();
  }
  void row(int64_t r, int64_t c0, int64_t n, uint16_t* out) const {
    const uint8_t* base = t->data();
    const int64_t off = r * cols + c0;
    switch (t->dtype) {
      case StDType::BF16: std::memcpy(out, base + off * 2, n * 2); break;
      case StDType::F16:
        for (int64_t i = 0; i < n; ++i) {
          uint16_t h;
          std::memcpy(&h, base + (off + i) * 2, 2);
          out[i] = f32_to_bf16(f16_to_f32(h));
        }
        break;
      case StDType::F32:
        for (int64_t i = 0; i < n; ++i) {
          float f;
          std::memcpy(&f, base + (off + i) * 4, 4);
          out[i] = f32_to_bf16(f);
        }
        break;
      default: throw ValueError("a projection of dtype " + std::string(st_dtype_name(t->dtype)) + " does not load as BF16");
    }
  }
};

}  // namespace

std::vector<uint16_t> tensor_bf16(const StoredTensor& t) {
  const int64_t n = t.numel();
  std::vector<uint16_t> out(static_cast<size_t>(n));
  const uint8_t* base = t.data();
  switch (t.dtype) {
    case StDType::BF16: std::memcpy(out.data(), base, n * 2); break;
    case StDType::F16:
      for (int64_t i = 0; i < n; ++i) {
        uint16_t h;
        std::memcpy(&h, base + i * 2, 2);
        out[i] = f32_to_bf16(f16_to_f32(h));
      }
      break;
    case StDType::F32:
      for (int64_t i = 0; i < n; ++i) {
        float f;
        std::memcpy(&f, base + i * 4, 4);
        out[i] = f32_to_bf16(f);
      }
      break;
    default: throw ValueError("a tensor of dtype " + std::string(st_dtype_name(t.dtype)) + " does not load as BF16");
  }
  return out;
}

std::vector<float> tensor_f32(const StoredTensor& t) {
  const int64_t n = t.numel();
  std::vector<float> out(static_cast<size_t>(n));
  const uint8_t* base = t.data();
  for (int64_t i = 0; i < n; ++i) {
    switch (t.dtype) {
      case StDType::BF16: {
        uint16_t h;
        std::memcpy(&h, base + i * 2, 2);
        const uint32_t b = static_cast<uint32_t>(h) << 16;
        std::memcpy(&out[i], &b, 4);
        break;
      }
      case StDType::F16: {
        uint16_t h;
        std::memcpy(&h, base + i * 2, 2);
        out[i] = f16_to_f32(h);
        break;
      }
      case StDType::F32: std::memcpy(&out[i], base + i * 4, 4); break;
      default: throw ValueError("a tensor of dtype " + std::string(st_dtype_name(t.dtype)) + " does not load as FP32");
    }
  }
  return out;
}

void load_weights(DecoderModel& model, const Checkpoint& ck) {
  const ModelConfig& cfg = model.config();
  const int H = cfg.hidden, D = cfg.head_dim;
  const int qh_l = model.q_heads_local(), kvh_l = model.kv_heads_local();
  const int qh0 = model.q_head_first(), kvh0 = model.kv_head_first();
  const int inter_l = model.intermediate_local(), rank = model.rank();
  std::map<std::string, bool> used;
  for (const auto& n : ck.names()) used[n] = false;
  std::vector<std::string> missing;
  auto take = [&](const std::string& name, std::vector<int64_t> shape) -> const StoredTensor* {
    const StoredTensor* t = ck.get(name);
    if (!t) {
      missing.push_back(name);
      return nullptr;
    }
    if (t->shape != shape) {
      std::string s;
      for (auto x : t->shape) s += (s.empty() ? "" : ", ") + std::to_string(x);
      invalid(name, "shape [" + s + "] is not the model's");
    }
    used[name] = true;
    return t;
  };
  auto st = model.device().state();
  std::vector<uint16_t> host;
  // A BF16 image into its slot; a slot quantized at load takes it through the device quantizer
  // (`amax`: the fused tensor's magnitude a per-tensor scale covers).
  float fused_amax = -1.f;
  auto upload = [&](const std::string& slot) {
    WeightSlot& w = model.weight_slot(slot);
    if (w.format == foa::kWeightBf16) {
      st->check_cuda(cudaMemcpy(w.ptr, host.data(), host.size() * 2, cudaMemcpyHostToDevice), "weight upload");
      return;
    }
    HbmBuffer tmp(model.device(), host.size() * 2);
    st->check_cuda(cudaMemcpy(tmp.data(), host.data(), host.size() * 2, cudaMemcpyHostToDevice), "weight upload");
    model.quantize_slot(w, static_cast<const __nv_bfloat16*>(tmp.data()), 0.f, fused_amax);
  };
  // The largest magnitude over whole checkpoint tensors (every rank's shard of them).
  auto amax_of = [&](std::initializer_list<const StoredTensor*> parts) {
    float m = 0.f;
    std::vector<uint16_t> row;
    for (const StoredTensor* t : parts) {
      if (!t) continue;
      const Source src(t);
      row.resize(static_cast<size_t>(src.cols));
      for (int64_t r = 0; r < src.rows; ++r) {
        src.row(r, 0, src.cols, row.data());
        for (uint16_t b : row) {
          const uint32_t bits = static_cast<uint32_t>(b & 0x7fff) << 16;
          float f;
          std::memcpy(&f, &bits, 4);
          m = std::max(m, f);
        }
      }
    }
    return m;
  };
  const bool per_tensor = cfg.weight_format == "fp8_tensor";
  auto image = [&](const std::string& slot) {
    const WeightSlot& w = model.weights().at(slot);
    size_t n = 1;
    for (auto s : w.shape) n *= static_cast<size_t>(s);
    host.assign(n, 0);
    return w.shape;
  };
  // Rows [src0, src0 + n) of `s`, columns [c0, c0 + ncols), into image rows from dst0.
  auto copy_rows = [&](const Source& s, int64_t src0, int64_t n, int64_t dst0, int64_t c0, int64_t ncols,
                       int64_t dst_cols) {
    for (int64_t r = 0; r < n; ++r) s.row(src0 + r, c0, ncols, host.data() + (dst0 + r) * dst_cols);
  };
  // ---- quantized projections: codes and scales sliced and stacked like the BF16 rows.
  // One part of a fused projection: rows [r0, r0 + n) and columns [c0, c0 + nc) of the
  // checkpoint's q/k/v, gate/up, o or down, placed at image rows `dst` (a list of 128-row blocks
  // or a contiguous range).
  struct Part {
    std::string base;          // "model.layers.3.self_attn.q_proj"
    int64_t rows, cols;        // the checkpoint's logical shape
    int64_t r0, n;             // source rows
    std::vector<int64_t> dst;  // destination row of each source row block of 128 (or one entry)
    bool blocked;              // dst holds one entry per 128 source rows
  };
  auto f32_of = [&](const StoredTensor* t, int64_t i) -> float {
    float f = 0.f;
    if (t->dtype == StDType::F32) std::memcpy(&f, t->data() + i * 4, 4);
    else if (t->dtype == StDType::BF16) {
      uint16_t h;
      std::memcpy(&h, t->data() + i * 2, 2);
      const uint32_t b = static_cast<uint32_t>(h) << 16;
      std::memcpy(&f, &b, 4);
    } else {
      invalid(t->file, "a scale of dtype " + std::string(st_dtype_name(t->dtype)) + " does not load");
    }
    return f;
  };
  auto scalar = [&](const std::string& name) -> float {
    const StoredTensor* t = ck.get(name);
    if (!t) {
      missing.push_back(name);
      return 1.f;
    }
    if (t->numel() != 1) invalid(name, "a tensor scale holds one value");
    used[name] = true;
    return f32_of(t, 0);
  };
  auto load_quantized = [&](const std::string& slot, const std::vector<Part>& parts, int64_t c0, int64_t nc) {
    WeightSlot& w = model.weight_slot(slot);
    const int64_t R = w.shape[0], C = w.shape[1];
    if (w.format == foa::kWeightFp8Block && w.scale_rows == 1) {
      // Static per-tensor FP8: each part's codes, and its weight_scale on every one of its rows.
      std::vector<uint8_t> codes(static_cast<size_t>(R * C), 0);
      std::vector<float> rows_scale(static_cast<size_t>(R), 0.f);
      for (const Part& p : parts) {
        const StoredTensor* wt = take(p.base + ".weight", {p.rows, p.cols});
        if (wt && wt->dtype != StDType::F8_E4M3)
          invalid(p.base + ".weight", std::string("codes of dtype ") + st_dtype_name(wt->dtype) + " are not F8_E4M3");
        const float ws = scalar(p.base + ".weight_scale");
        if (ck.get(p.base + ".input_scale")) scalar(p.base + ".input_scale");  // calibrated, inputs stay BF16
        for (int64_t i = 0; i < p.n; ++i) {
          const int64_t d = p.blocked ? p.dst[i / 128] + i % 128 : p.dst[0] + i;
          if (wt) std::memcpy(codes.data() + d * C, wt->data() + (p.r0 + i) * p.cols + c0, C);
          rows_scale[static_cast<size_t>(d)] = ws;
        }
      }
      st->check_cuda(cudaMemcpy(w.codes, codes.data(), codes.size(), cudaMemcpyHostToDevice), "weight upload");
      st->check_cuda(cudaMemcpy(w.scales, rows_scale.data(), rows_scale.size() * 4, cudaMemcpyHostToDevice),
                     "weight upload");
      return;
    }
    const bool fp8 = w.format == foa::kWeightFp8A8;
    const int64_t code_bytes = fp8 ? C : C / 2;
    std::vector<uint8_t> codes(static_cast<size_t>(R * code_bytes), 0);
    // FP8: FP32 block scales [R/128][C/128]; NVFP4: E4M3 [R][C/16] (atoms built on the device).
    std::vector<float> fscales;
    std::vector<uint8_t> bscales;
    if (fp8) fscales.assign(static_cast<size_t>((R + 127) / 128 * (C / 128)), 0.f);
    else bscales.assign(static_cast<size_t>(R * (C / 16)), 0);
    float tensor_scale = 0.f, input_scale = 0.f;
    for (const Part& p : parts) {
      const int64_t src_code_bytes = fp8 ? p.cols : p.cols / 2;
      const StoredTensor* wt = take(p.base + ".weight", {p.rows, src_code_bytes});
      if (wt && wt->dtype != (fp8 ? StDType::F8_E4M3 : StDType::U8))
        invalid(p.base + ".weight", std::string("codes of dtype ") + st_dtype_name(wt->dtype) + " are not " + (fp8 ? "F8_E4M3" : "U8"));
      auto dst_row = [&](int64_t i) {  // image row of source row r0 + i
        return p.blocked ? p.dst[i / 128] + i % 128 : p.dst[0] + i;
      };
      const int64_t cb0 = fp8 ? c0 : c0 / 2, cbn = fp8 ? nc : nc / 2;
      if (wt)
        for (int64_t i = 0; i < p.n; ++i)
          std::memcpy(codes.data() + dst_row(i) * code_bytes, wt->data() + (p.r0 + i) * src_code_bytes + cb0, cbn);
      if (fp8) {
        const StoredTensor* sc = ck.get(p.base + ".weight_scale_inv");
        std::string sname = p.base + ".weight_scale_inv";
        if (!sc) {
          sc = ck.get(p.base + ".weight_scale");
          sname = p.base + ".weight_scale";
        }
        const int64_t srows = (p.rows + 127) / 128, scols = (p.cols + 127) / 128;
        if (!sc) {
          missing.push_back(p.base + ".weight_scale_inv");
          continue;
        }
        if (sc->shape != std::vector<int64_t>{srows, scols}) invalid(sname, "not one scale per 128x128 block");
        if (p.r0 % 128 != 0 || p.n % 128 != 0 || c0 % 128 != 0 || nc % 128 != 0)
          unsupported(sname, "a shard boundary falls inside a 128x128 scale block");
        used[sname] = true;
        for (int64_t i = 0; i < p.n; i += 128)
          for (int64_t j = 0; j < nc / 128; ++j)
            fscales[static_cast<size_t>((dst_row(i) / 128) * (C / 128) + j)] =
                f32_of(sc, (p.r0 + i) / 128 * scols + c0 / 128 + j);
      } else {
        const StoredTensor* sc = take(p.base + ".weight_scale", {p.rows, p.cols / 16});
        if (sc && sc->dtype != StDType::F8_E4M3) invalid(p.base + ".weight_scale", "block scales are F8_E4M3");
        if (sc)
          for (int64_t i = 0; i < p.n; ++i)
            std::memcpy(bscales.data() + dst_row(i) * (C / 16), sc->data() + (p.r0 + i) * (p.cols / 16) + c0 / 16, nc / 16);
        const float ts = scalar(p.base + ".weight_scale_2");
        const bool has_in = ck.get(p.base + ".input_scale") != nullptr;
        const float is = has_in ? scalar(p.base + ".input_scale") : 1.f;
        if (tensor_scale != 0.f && (ts != tensor_scale || (has_in && is != input_scale)))
          unsupported(p.base, "fused projections with different tensor scales");
        tensor_scale = ts;
        input_scale = is;
      }
    }
    st->check_cuda(cudaMemcpy(w.codes, codes.data(), codes.size(), cudaMemcpyHostToDevice), "weight upload");
    if (fp8) {
      // The W8A8 GEMM stages each block scale as a 16-byte entry (the value four times).
      std::vector<float> padded(fscales.size() * 4);
      for (size_t i = 0; i < fscales.size(); ++i)
        for (int j = 0; j < 4; ++j) padded[i * 4 + j] = fscales[i];
      st->check_cuda(cudaMemcpy(w.scales, padded.data(), padded.size() * 4, cudaMemcpyHostToDevice), "weight upload");
      return;
    }
    w.tensor_scale = tensor_scale;
    w.input_scale = input_scale;
    if (w.format == foa::kWeightNvfp4) {
      st->check_cuda(cudaMemcpy(w.scales, bscales.data(), bscales.size(), cudaMemcpyHostToDevice), "weight upload");
      return;
    }
    HbmBuffer tmp(model.device(), bscales.size());
    st->check_cuda(cudaMemcpy(tmp.data(), bscales.data(), bscales.size(), cudaMemcpyHostToDevice), "weight upload");
    if (foa::nvfp4_scale_atoms(static_cast<const uint8_t*>(tmp.data()), C / 16, static_cast<int>(R),
                               static_cast<int>(C), static_cast<uint8_t*>(w.scales), st->stream) != 0)
      st->fail("scale repack launch failed");
    st->check_cuda(cudaStreamSynchronize(st->stream), "scale repack");
  };
  // Checkpoints that hold their own codes and scales (load-time FP8 reads BF16 and quantizes).
  const bool quantized = cfg.weight_format == "fp8_block" || cfg.weight_format == "nvfp4" ||
                         cfg.weight_format == "nvfp4_a4" || cfg.weight_format == "fp8_static";

  // Names under "model." (a causal or classifier checkpoint); a base model saved on its own
  // (sentence-embedding checkpoints) names its tensors from the root.
  const std::string pre = (cfg.output == Output::Hidden && ck.get("model.embed_tokens.weight") == nullptr &&
                           ck.get("embed_tokens.weight") != nullptr)
                              ? ""
                              : "model.";
  // Embedding (whole on every chip) and head (this chip's vocabulary rows).
  if (auto* t = take(pre + "embed_tokens.weight", {cfg.vocab, H})) {
    image("embed");
    copy_rows(Source(t), 0, cfg.vocab, 0, 0, H, H);
    upload("embed");
  }
  if (!cfg.tied && cfg.output == Output::Tokens) {
    if (auto* t = take("lm_head.weight", {cfg.vocab, H})) {
      image("lm_head");
      const int64_t n = model.vocab_end() - model.vocab_begin();
      copy_rows(Source(t), model.vocab_begin(), n, 0, 0, H, H);
      upload("lm_head");
    }
  } else if (ck.get("lm_head.weight")) {
    // A tied head the checkpoint also stores, or the head of a causal checkpoint loaded as its
    // base model: read by no call.
    used["lm_head.weight"] = true;
  }
  if (auto* t = take(pre + "norm.weight", {H})) {
    image("final_norm");
    Source(t).row(0, 0, H, host.data());
    upload("final_norm");
  }
  if (cfg.output == Output::Scores) {
    const StoredTensor* t = ck.get("score.weight");
    if (!t) {
      missing.push_back("score.weight");
    } else {
      used["score.weight"] = true;
      image("score");
      copy_rows(Source(t), 0, t->shape[0], 0, 0, H, H);
      upload("score");
    }
  }
  for (int l = 0; l < cfg.layers; ++l) {
    const std::string hf = pre + "layers." + std::to_string(l) + ".";
    const std::string en = "layers." + std::to_string(l) + ".";
    if (auto* t = take(hf + "input_layernorm.weight", {H})) {
      image(en + "in_norm");
      Source(t).row(0, 0, H, host.data());
      upload(en + "in_norm");
    }
    if (auto* t = take(hf + "post_attention_layernorm.weight", {H})) {
      image(en + "post_norm");
      Source(t).row(0, 0, H, host.data());
      upload(en + "post_norm");
    }
    if (quantized) {
      const int64_t qr = static_cast<int64_t>(cfg.q_heads) * D, kr = static_cast<int64_t>(cfg.kv_heads) * D;
      const int64_t ql = static_cast<int64_t>(qh_l) * D, kl = static_cast<int64_t>(kvh_l) * D;
      load_quantized(en + "qkv",
                     {Part{hf + "self_attn.q_proj", qr, H, static_cast<int64_t>(qh0) * D, ql, {0}, false},
                      Part{hf + "self_attn.k_proj", kr, H, static_cast<int64_t>(kvh0) * D, kl, {ql}, false},
                      Part{hf + "self_attn.v_proj", kr, H, static_cast<int64_t>(kvh0) * D, kl, {ql + kl}, false}},
                     0, H);
    }
    const auto* q = quantized ? nullptr : take(hf + "self_attn.q_proj.weight", {static_cast<int64_t>(cfg.q_heads) * D, H});
    const auto* k = quantized ? nullptr : take(hf + "self_attn.k_proj.weight", {static_cast<int64_t>(cfg.kv_heads) * D, H});
    const auto* v = quantized ? nullptr : take(hf + "self_attn.v_proj.weight", {static_cast<int64_t>(cfg.kv_heads) * D, H});
    if (q && k && v) {
      fused_amax = per_tensor ? amax_of({q, k, v}) : -1.f;
      image(en + "qkv");
      copy_rows(Source(q), static_cast<int64_t>(qh0) * D, static_cast<int64_t>(qh_l) * D, 0, 0, H, H);
      copy_rows(Source(k), static_cast<int64_t>(kvh0) * D, static_cast<int64_t>(kvh_l) * D,
                static_cast<int64_t>(qh_l) * D, 0, H, H);
      copy_rows(Source(v), static_cast<int64_t>(kvh0) * D, static_cast<int64_t>(kvh_l) * D,
                static_cast<int64_t>(qh_l + kvh_l) * D, 0, H, H);
      upload(en + "qkv");
    }
    if (cfg.qk_norm) {
      for (const char* which : {"q_norm", "k_norm"}) {
        if (auto* t = take(hf + "self_attn." + which + ".weight", {D})) {
          image(en + which);
          Source(t).row(0, 0, D, host.data());
          upload(en + which);
        }
      }
    }
    if (quantized) {
      load_quantized(en + "o",
                     {Part{hf + "self_attn.o_proj", H, static_cast<int64_t>(cfg.q_heads) * D, 0, H, {0}, false}},
                     static_cast<int64_t>(qh0) * D, static_cast<int64_t>(qh_l) * D);
    } else if (auto* t = take(hf + "self_attn.o_proj.weight", {H, static_cast<int64_t>(cfg.q_heads) * D})) {
      fused_amax = per_tensor ? amax_of({t}) : -1.f;
      image(en + "o");
      copy_rows(Source(t), 0, H, 0, static_cast<int64_t>(qh0) * D, static_cast<int64_t>(qh_l) * D,
                static_cast<int64_t>(qh_l) * D);
      upload(en + "o");
    }
    if (cfg.experts > 0) {
      // Router (every expert) and this rank's experts, gate/up interleaved in 128-row blocks.
      const int E = cfg.experts, El = model.experts_local(), e0 = model.expert_first();
      const int64_t I = cfg.expert_intermediate;
      // Expert block names: Qwen3-MoE `mlp.gate`, `mlp.experts.e.{gate,up,down}_proj`; Mixtral
      // `block_sparse_moe.gate`, `block_sparse_moe.experts.e.{w1,w3,w2}`.
      const bool mixtral = cfg.family == "mixtral";
      const std::string block = hf + (mixtral ? "block_sparse_moe." : "mlp.");
      const char* gate_name = mixtral ? "w1.weight" : "gate_proj.weight";
      const char* up_name = mixtral ? "w3.weight" : "up_proj.weight";
      const char* down_name = mixtral ? "w2.weight" : "down_proj.weight";
      if (auto* t = take(block + "gate.weight", {E, H})) {
        image(en + "router");
        copy_rows(Source(t), 0, E, 0, 0, H, H);
        upload(en + "router");
      }
      image(en + "experts_gate_up");
      bool complete = true;
      for (int x = 0; x < El; ++x) {
        const std::string ep = block + "experts." + std::to_string(e0 + x) + ".";
        const auto* g = take(ep + gate_name, {I, H});
        const auto* u = take(ep + up_name, {I, H});
        if (!g || !u) {
          complete = false;
          continue;
        }
        const Source sg(g), su(u);
        for (int64_t j = 0; j < I; ++j) {
          const int64_t block = j / 128, in = j % 128, base = static_cast<int64_t>(x) * 2 * I;
          sg.row(j, 0, H, host.data() + (base + block * 256 + in) * H);
          su.row(j, 0, H, host.data() + (base + block * 256 + 128 + in) * H);
        }
      }
      if (complete) upload(en + "experts_gate_up");
      image(en + "experts_down");
      complete = true;
      for (int x = 0; x < El; ++x) {
        const std::string ep = block + "experts." + std::to_string(e0 + x) + ".";
        if (auto* t = take(ep + down_name, {H, I}))
          copy_rows(Source(t), 0, H, static_cast<int64_t>(x) * H, 0, I, I);
        else
          complete = false;
      }
      if (complete) upload(en + "experts_down");
      // Other ranks' experts are theirs to load.
      for (int x = 0; x < E; ++x) {
        if (x >= e0 && x < e0 + El) continue;
        const std::string ep = block + "experts." + std::to_string(x) + ".";
        for (const char* n : {gate_name, up_name, down_name})
          if (used.count(ep + n)) used[ep + n] = true;
      }
    }
    if (cfg.experts == 0 && quantized) {
      // Gate and up rows alternate in 128-row blocks (see the BF16 path below).
      std::vector<int64_t> gate_dst, up_dst;
      for (int64_t b = 0; b < inter_l / 128; ++b) {
        gate_dst.push_back(b * 256);
        up_dst.push_back(b * 256 + 128);
      }
      const int64_t r0 = static_cast<int64_t>(rank) * inter_l;
      load_quantized(en + "gate_up",
                     {Part{hf + "mlp.gate_proj", cfg.intermediate, H, r0, inter_l, gate_dst, true},
                      Part{hf + "mlp.up_proj", cfg.intermediate, H, r0, inter_l, up_dst, true}},
                     0, H);
      load_quantized(en + "down", {Part{hf + "mlp.down_proj", H, cfg.intermediate, 0, H, {0}, false}},
                     static_cast<int64_t>(rank) * inter_l, inter_l);
    }
    if (cfg.experts == 0 && !quantized) {
      const auto* g = take(hf + "mlp.gate_proj.weight", {cfg.intermediate, H});
      const auto* u = take(hf + "mlp.up_proj.weight", {cfg.intermediate, H});
      if (g && u) {
        // Gate and up rows alternate in 128-row blocks, so one GEMM tile holds both halves of
        // the SwiGLU it feeds.
        fused_amax = per_tensor ? amax_of({g, u}) : -1.f;
        image(en + "gate_up");
        const Source sg(g), su(u);
        for (int64_t j = 0; j < inter_l; ++j) {
          const int64_t src = static_cast<int64_t>(rank) * inter_l + j;
          const int64_t block = j / 128, in = j % 128;
          sg.row(src, 0, H, host.data() + ((block * 256) + in) * H);
          su.row(src, 0, H, host.data() + ((block * 256) + 128 + in) * H);
        }
        upload(en + "gate_up");
      }
      if (auto* t = take(hf + "mlp.down_proj.weight", {H, cfg.intermediate})) {
        fused_amax = per_tensor ? amax_of({t}) : -1.f;
        image(en + "down");
        copy_rows(Source(t), 0, H, 0, static_cast<int64_t>(rank) * inter_l, inter_l, inter_l);
        upload(en + "down");
      }
    }
  }
  if (!missing.empty()) {
    std::string s;
    for (size_t i = 0; i < missing.size() && i < 8; ++i) s += (i ? ", " : "") + missing[i];
    if (missing.size() > 8) s += ", ... (" + std::to_string(missing.size()) + " in all)";
    invalid("checkpoint", "missing tensors: " + s);
  }
  std::vector<std::string> extra;
  for (const auto& [n, u] : used)
    if (!u) extra.push_back(n);
  if (!extra.empty()) {
    std::string s;
    for (size_t i = 0; i < extra.size() && i < 8; ++i) s += (i ? ", " : "") + extra[i];
    if (extra.size() > 8) s += ", ... (" + std::to_string(extra.size()) + " in all)";
    invalid("checkpoint", "unexpected tensors: " + s);
  }
}

}  // namespace foa::engine
