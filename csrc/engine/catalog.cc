#include "catalog.h"

#include <functional>
#include <map>
#include <set>

#include "runtime.h"

namespace foa::engine::catalog {
namespace {

[[noreturn]] void refuse(const std::string& what) { throw ValueError(what); }

int64_t need(const Json& c, const char* key) {
  const Json& v = c[key];
  if (!v.is_number()) refuse(std::string("config.json:") + key + ": missing or not a number");
  return v.as_int();
}

int64_t get(const Json& c, const char* key, int64_t def) {
  const Json& v = c[key];
  return v.is_number() ? v.as_int() : def;
}

bool flag(const Json& c, const char* key, bool def) {
  const Json& v = c[key];
  return v.is_bool() ? v.as_bool() : def;
}

std::string text(const Json& c, const char* key, const std::string& def) {
  const Json& v = c[key];
  return v.is_string() ? v.as_string() : def;
}

// Accumulates a composition: modules (tree lines) and their weights under a name prefix.
struct Builder {
  Composition c;
  int depth = 0;
  void module(const std::string& line) { c.tree.push_back(std::string(2 * depth, ' ') + line); }
  void weight(const std::string& name, std::vector<int64_t> shape) { c.weights.push_back({name, std::move(shape)}); }
  void alias(const std::string& name, std::vector<int64_t> shape) { c.aliases.push_back({name, std::move(shape)}); }
  // A head that shares the embedding's values when `tied`, else a weight of its own.
  void head(const std::string& name, std::vector<int64_t> shape, bool tied) {
    if (tied) alias(name, std::move(shape));
    else weight(name, std::move(shape));
  }
  void linear(const std::string& p, int64_t out, int64_t in, bool bias) {
    weight(p + ".weight", {out, in});
    if (bias) weight(p + ".bias", {out});
  }
  void layer_norm(const std::string& p, int64_t n, bool bias = true) {
    weight(p + ".weight", {n});
    if (bias) weight(p + ".bias", {n});
  }
  template <typename F>
  void nest(const std::string& line, F body) {
    module(line);
    ++depth;
    body();
    --depth;
  }
};

// BERT encoder (post-norm, learned positions, token types, GELU MLP, pooler).
Composition bert(const Json& cfg, const std::string& arch, const std::string& prefix) {
  const int64_t H = need(cfg, "hidden_size"), L = need(cfg, "num_hidden_layers"),
                heads = need(cfg, "num_attention_heads"), I = need(cfg, "intermediate_size"),
                V = need(cfg, "vocab_size"), P = get(cfg, "max_position_embeddings", 512),
                T = get(cfg, "type_vocab_size", 2);
  if (H % heads != 0) refuse("config.json:num_attention_heads: does not divide hidden_size");
  Builder b;
  b.c.family = "bert";
  b.c.architecture = arch;
  b.nest("BertModel (post-norm encoder, bidirectional attention)", [&] {
    b.nest("Embeddings (word + position + token type, LayerNorm)", [&] {
      b.weight(prefix + "embeddings.word_embeddings.weight", {V, H});
      b.weight(prefix + "embeddings.position_embeddings.weight", {P, H});
      b.weight(prefix + "embeddings.token_type_embeddings.weight", {T, H});
      b.layer_norm(prefix + "embeddings.LayerNorm", H);
    });
    b.nest("Layers x " + std::to_string(L) + " (self-attention, add & LayerNorm, GELU MLP, add & LayerNorm)", [&] {
      for (int64_t l = 0; l < L; ++l) {
        const std::string p = prefix + "encoder.layer." + std::to_string(l) + ".";
        for (const char* q : {"query", "key", "value"}) b.linear(p + "attention.self." + q, H, H, true);
        b.linear(p + "attention.output.dense", H, H, true);
        b.layer_norm(p + "attention.output.LayerNorm", H);
        b.linear(p + "intermediate.dense", I, H, true);
        b.linear(p + "output.dense", H, I, true);
        b.layer_norm(p + "output.LayerNorm", H);
      }
    });
    b.nest("Pooler (first token, dense, tanh)", [&] { b.linear(prefix + "pooler.dense", H, H, true); });
  });
  return b.c;
}

// T5 / mT5 encoder-decoder (pre-norm RMSNorm, relative position buckets in the first block of each
// stack, ReLU or gated-GELU feed-forward).
Composition t5(const Json& cfg, const std::string& arch) {
  const int64_t d = need(cfg, "d_model"), d_kv = need(cfg, "d_kv"), ff = need(cfg, "d_ff"),
                heads = need(cfg, "num_heads"), L = need(cfg, "num_layers"),
                Ld = get(cfg, "num_decoder_layers", L), V = need(cfg, "vocab_size"),
                buckets = get(cfg, "relative_attention_num_buckets", 32);
  const std::string ffp = text(cfg, "feed_forward_proj", "relu");
  const bool gated = ffp.rfind("gated-", 0) == 0;
  const bool tied = flag(cfg, "tie_word_embeddings", true);
  const int64_t inner = heads * d_kv;
  Builder b;
  b.c.family = "t5";
  b.c.architecture = arch;
  auto attention = [&](const std::string& p, bool relative) {
    for (const char* q : {"q", "k", "v"}) b.weight(p + "." + q + ".weight", {inner, d});
    b.weight(p + ".o.weight", {d, inner});
    if (relative) b.weight(p + ".relative_attention_bias.weight", {buckets, heads});
  };
  auto feed_forward = [&](const std::string& p) {
    if (gated) {
      b.weight(p + ".DenseReluDense.wi_0.weight", {ff, d});
      b.weight(p + ".DenseReluDense.wi_1.weight", {ff, d});
    } else {
      b.weight(p + ".DenseReluDense.wi.weight", {ff, d});
    }
    b.weight(p + ".DenseReluDense.wo.weight", {d, ff});
    b.weight(p + ".layer_norm.weight", {d});
  };
  b.nest(arch + " (" + (gated ? "gated " : "") + ffp + " feed-forward)", [&] {
    b.weight("shared.weight", {V, d});
    b.alias("encoder.embed_tokens.weight", {V, d});  // each stack's embedding is the shared one
    b.alias("decoder.embed_tokens.weight", {V, d});
    b.nest("Encoder x " + std::to_string(L) + " (self-attention, feed-forward; RMSNorm before each)", [&] {
      for (int64_t l = 0; l < L; ++l) {
        const std::string p = "encoder.block." + std::to_string(l) + ".layer.";
        attention(p + "0.SelfAttention", l == 0);
        b.weight(p + "0.layer_norm.weight", {d});
        feed_forward(p + "1");
      }
      b.weight("encoder.final_layer_norm.weight", {d});
    });
    b.nest("Decoder x " + std::to_string(Ld) + " (causal self-attention, cross-attention, feed-forward)", [&] {
      for (int64_t l = 0; l < Ld; ++l) {
        const std::string p = "decoder.block." + std::to_string(l) + ".layer.";
        attention(p + "0.SelfAttention", l == 0);
        b.weight(p + "0.layer_norm.weight", {d});
        attention(p + "1.EncDecAttention", false);
        b.weight(p + "1.layer_norm.weight", {d});
        feed_forward(p + "2");
      }
      b.weight("decoder.final_layer_norm.weight", {d});
    });
    b.nest(tied ? "Head (tied to the shared embedding, scaled by d_model^-0.5)" : "Head (untied)",
           [&] { b.head("lm_head.weight", {V, d}, tied); });
  });
  return b.c;
}

// Whisper encoder-decoder (two convolutions over log-mel frames, learned positions, pre-norm
// LayerNorm blocks; key projections without bias).
Composition whisper(const Json& cfg, const std::string& arch) {
  const int64_t d = need(cfg, "d_model"), mels = get(cfg, "num_mel_bins", 80),
                Le = need(cfg, "encoder_layers"), Ld = need(cfg, "decoder_layers"),
                ffe = need(cfg, "encoder_ffn_dim"), ffd = need(cfg, "decoder_ffn_dim"), V = need(cfg, "vocab_size"),
                src = get(cfg, "max_source_positions", 1500), tgt = get(cfg, "max_target_positions", 448);
  Builder b;
  b.c.family = "whisper";
  b.c.architecture = arch;
  auto attention = [&](const std::string& p) {
    b.linear(p + ".q_proj", d, d, true);
    b.linear(p + ".k_proj", d, d, false);
    b.linear(p + ".v_proj", d, d, true);
    b.linear(p + ".out_proj", d, d, true);
  };
  b.nest(arch, [&] {
    b.nest("Encoder (conv k3 from " + std::to_string(mels) + " mel bins, GELU, conv k3 stride 2, GELU, positions) x " +
                 std::to_string(Le),
           [&] {
             b.weight("model.encoder.conv1.weight", {d, mels, 3});
             b.weight("model.encoder.conv1.bias", {d});
             b.weight("model.encoder.conv2.weight", {d, d, 3});
             b.weight("model.encoder.conv2.bias", {d});
             b.weight("model.encoder.embed_positions.weight", {src, d});
             for (int64_t l = 0; l < Le; ++l) {
               const std::string p = "model.encoder.layers." + std::to_string(l) + ".";
               attention(p + "self_attn");
               b.layer_norm(p + "self_attn_layer_norm", d);
               b.linear(p + "fc1", ffe, d, true);
               b.linear(p + "fc2", d, ffe, true);
               b.layer_norm(p + "final_layer_norm", d);
             }
             b.layer_norm("model.encoder.layer_norm", d);
           });
    b.nest("Decoder (tokens, positions; causal self-attention, cross-attention, GELU MLP) x " + std::to_string(Ld),
           [&] {
             b.weight("model.decoder.embed_tokens.weight", {V, d});
             b.weight("model.decoder.embed_positions.weight", {tgt, d});
             for (int64_t l = 0; l < Ld; ++l) {
               const std::string p = "model.decoder.layers." + std::to_string(l) + ".";
               attention(p + "self_attn");
               b.layer_norm(p + "self_attn_layer_norm", d);
               attention(p + "encoder_attn");
               b.layer_norm(p + "encoder_attn_layer_norm", d);
               b.linear(p + "fc1", ffd, d, true);
               b.linear(p + "fc2", d, ffd, true);
               b.layer_norm(p + "final_layer_norm", d);
             }
             b.layer_norm("model.decoder.layer_norm", d);
           });
    b.head("proj_out.weight", {V, d}, flag(cfg, "tie_word_embeddings", true));
  });
  return b.c;
}

// Mamba-2 (selective state-space mixer: one input projection into z, x, B, C and dt, a causal
// depthwise convolution over x, B and C, the scan with per-head A and D, a gated RMSNorm, the
// output projection).
Composition mamba2(const Json& cfg, const std::string& arch) {
  const int64_t d = need(cfg, "hidden_size"), L = need(cfg, "num_hidden_layers"), V = need(cfg, "vocab_size"),
                state = need(cfg, "state_size"), groups = get(cfg, "n_groups", 1), conv = get(cfg, "conv_kernel", 4),
                expand = get(cfg, "expand", 2), head_dim = get(cfg, "head_dim", 64);
  const int64_t inner = expand * d;
  if (inner % head_dim != 0) refuse("config.json:head_dim: does not divide expand * hidden_size");
  const int64_t heads = get(cfg, "num_heads", inner / head_dim);
  if (heads * head_dim != inner) refuse("config.json:num_heads: num_heads * head_dim differs from expand * hidden_size");
  const bool bias = flag(cfg, "use_bias", false), conv_bias = flag(cfg, "use_conv_bias", true);
  const bool tied = flag(cfg, "tie_word_embeddings", false);
  const int64_t conv_dim = inner + 2 * groups * state;
  Builder b;
  b.c.family = "mamba2";
  b.c.architecture = arch;
  b.nest(arch + " (RMSNorm, Mamba-2 mixer, residual) x " + std::to_string(L), [&] {
    b.nest("Embedding " + std::to_string(V) + " x " + std::to_string(d), [&] {
      b.weight("backbone.embeddings.weight", {V, d});
    });
    b.nest("Mixer: in_proj to z, x, B, C (" + std::to_string(groups) + " groups of state " + std::to_string(state) +
               ") and dt (" + std::to_string(heads) + " heads of " + std::to_string(head_dim) + "); causal conv " +
               std::to_string(conv) + " over x, B, C; SiLU; SSD scan with A = -exp(A_log), D skip; RMSNorm gated "
               "by SiLU(z); out_proj",
           [] {});
    for (int64_t l = 0; l < L; ++l) {
      const std::string p = "backbone.layers." + std::to_string(l) + ".";
      b.weight(p + "norm.weight", {d});
      b.linear(p + "mixer.in_proj", 2 * inner + 2 * groups * state + heads, d, bias);
      b.weight(p + "mixer.conv1d.weight", {conv_dim, 1, conv});
      if (conv_bias) b.weight(p + "mixer.conv1d.bias", {conv_dim});
      b.weight(p + "mixer.dt_bias", {heads});
      b.weight(p + "mixer.A_log", {heads});
      b.weight(p + "mixer.D", {heads});
      b.weight(p + "mixer.norm.weight", {inner});
      b.linear(p + "mixer.out_proj", d, inner, bias);
    }
    b.nest("Final RMSNorm, head" + std::string(tied ? " (tied to the embedding)" : ""), [&] {
      b.weight("backbone.norm_f.weight", {d});
      b.head("lm_head.weight", {V, d}, tied);
    });
  });
  return b.c;
}

// Gemma-3 text decoder (GQA with QK RMSNorm, sandwich norms around attention and MLP, GeGLU MLP,
// local sliding-window and global layers, tied embeddings).
Composition gemma3_text(const Json& cfg, const std::string& arch) {
  const int64_t d = need(cfg, "hidden_size"), L = need(cfg, "num_hidden_layers"), V = need(cfg, "vocab_size"),
                heads = need(cfg, "num_attention_heads"), kv = get(cfg, "num_key_value_heads", heads),
                I = need(cfg, "intermediate_size"), hd = get(cfg, "head_dim", 256);
  if (heads % kv != 0) refuse("config.json:num_key_value_heads: does not divide num_attention_heads");
  // The layers' attention: `layer_types` when listed, else one global layer every
  // `sliding_window_pattern` (6).
  int64_t global = 0;
  const Json& types = cfg["layer_types"];
  if (types.is_array()) {
    if (static_cast<int64_t>(types.size()) != L) refuse("config.json:layer_types: one entry a layer");
    for (const auto& t : types.items()) {
      if (!t.is_string() || (t.as_string() != "full_attention" && t.as_string() != "sliding_attention"))
        refuse("config.json:layer_types: full_attention or sliding_attention");
      global += t.as_string() == "full_attention";
    }
  } else {
    const int64_t pattern = get(cfg, "sliding_window_pattern", 6);
    if (pattern <= 0) refuse("config.json:sliding_window_pattern: at least 1");
    global = L / pattern;
  }
  const int64_t window = get(cfg, "sliding_window", 4096);
  Builder b;
  b.c.family = "gemma3_text";
  b.c.architecture = arch;
  b.nest(arch + " x " + std::to_string(L) + " (" + std::to_string(global) + " global, " + std::to_string(L - global) +
             " sliding-window of " + std::to_string(window) + "; sandwich RMSNorms, QK RMSNorm, GeGLU MLP)",
         [&] {
           b.nest("Embedding " + std::to_string(V) + " x " + std::to_string(d) + ", scaled by sqrt(hidden_size)",
                  [&] { b.weight("model.embed_tokens.weight", {V, d}); });
           b.nest("Attention: " + std::to_string(heads) + " query heads, " + std::to_string(kv) + " KV heads of " +
                      std::to_string(hd) + "; RMSNorm of q and k; RoPE (local and global bases)",
                  [] {});
           b.nest("MLP: gelu_tanh(gate) * up, down (" + std::to_string(I) + ")", [] {});
           for (int64_t l = 0; l < L; ++l) {
             const std::string p = "model.layers." + std::to_string(l) + ".";
             b.weight(p + "input_layernorm.weight", {d});
             b.weight(p + "self_attn.q_proj.weight", {heads * hd, d});
             b.weight(p + "self_attn.k_proj.weight", {kv * hd, d});
             b.weight(p + "self_attn.v_proj.weight", {kv * hd, d});
             b.weight(p + "self_attn.o_proj.weight", {d, heads * hd});
             b.weight(p + "self_attn.q_norm.weight", {hd});
             b.weight(p + "self_attn.k_norm.weight", {hd});
             b.weight(p + "post_attention_layernorm.weight", {d});
             b.weight(p + "pre_feedforward_layernorm.weight", {d});
             b.weight(p + "mlp.gate_proj.weight", {I, d});
             b.weight(p + "mlp.up_proj.weight", {I, d});
             b.weight(p + "mlp.down_proj.weight", {d, I});
             b.weight(p + "post_feedforward_layernorm.weight", {d});
           }
           const bool tied = flag(cfg, "tie_word_embeddings", true);
           b.nest("Final RMSNorm, head" + std::string(tied ? " (tied to the embedding)" : ""), [&] {
             b.weight("model.norm.weight", {d});
             b.head("lm_head.weight", {V, d}, tied);
           });
         });
  return b.c;
}

using Maker = std::function<Composition(const Json&, const std::string&, const Checkpoint&)>;

const std::map<std::string, Maker>& makers() {
  static const std::map<std::string, Maker> m = {
      {"BertModel",
       [](const Json& c, const std::string& a, const Checkpoint& ck) {
         // Checkpoints saved from the pretraining heads name the encoder under "bert.".
         const bool nested = ck.get("bert.embeddings.word_embeddings.weight") != nullptr;
         return bert(c, a, nested ? "bert." : "");
       }},
      {"T5ForConditionalGeneration", [](const Json& c, const std::string& a, const Checkpoint&) { return t5(c, a); }},
      {"MT5ForConditionalGeneration", [](const Json& c, const std::string& a, const Checkpoint&) { return t5(c, a); }},
      {"WhisperForConditionalGeneration",
       [](const Json& c, const std::string& a, const Checkpoint&) { return whisper(c, a); }},
      {"Mamba2ForCausalLM", [](const Json& c, const std::string& a, const Checkpoint&) { return mamba2(c, a); }},
      {"Gemma3ForCausalLM", [](const Json& c, const std::string& a, const Checkpoint&) { return gemma3_text(c, a); }},
  };
  return m;
}

}  // namespace

bool composes(const std::string& architecture) { return makers().count(architecture) > 0; }

Composition compose(const Checkpoint& ck) {
  const Json& cfg = ck.config();
  for (const auto& a : cfg["architectures"].items()) {
    if (!a.is_string()) continue;
    const auto it = makers().find(a.as_string());
    if (it != makers().end()) return it->second(cfg, a.as_string(), ck);
  }
  refuse("config.json:architectures: no catalog composition (bert, t5, mt5, whisper, mamba2, gemma3 text)");
}

void check(const Composition& c, const Checkpoint& ck) {
  std::set<std::string> read;
  for (const auto& w : c.weights) {
    const StoredTensor* t = ck.get(w.name);
    if (t == nullptr) refuse(w.name + ": missing from the checkpoint (" + c.family + ")");
    if (t->shape != w.shape) {
      std::string want, got;
      for (auto v : w.shape) want += (want.empty() ? "" : ", ") + std::to_string(v);
      for (auto v : t->shape) got += (got.empty() ? "" : ", ") + std::to_string(v);
      refuse(w.name + ": shape [" + got + "], the composition reads [" + want + "]");
    }
    read.insert(w.name);
  }
  for (const auto& w : c.aliases) {
    const StoredTensor* t = ck.get(w.name);
    if (t == nullptr) continue;
    if (t->shape != w.shape) refuse(w.name + ": a tied copy whose shape differs from the weight it copies");
    read.insert(w.name);
  }
  for (const auto& n : ck.names())
    if (!read.count(n)) refuse(n + ": not read by the " + c.family + " composition");
}

}  // namespace foa::engine::catalog
