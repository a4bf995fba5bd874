#include "catalog.h"

#include <map>
#include <set>
#include <utility>

#include "runtime.h"

namespace foa::engine::catalog {
namespace {

[[noreturn]] void refuse(const std::string& what) { throw ValueError(what); }

std::string str(int64_t v) { return std::to_string(v); }

std::string dims(const std::vector<int64_t>& shape) {
  std::string s;
  for (auto v : shape) s += (s.empty() ? "" : ", ") + std::to_string(v);
  return "[" + s + "]";
}

std::string joined(const std::set<int64_t>& v) {
  std::string s;
  for (auto x : v) s += (s.empty() ? "" : ", ") + std::to_string(x);
  return s;
}

// A config (or one of its nested sub-configs) read with the upstream class defaults: configs that
// older exports wrote keep only the sub-config values that differ from the class defaults.
class Config {
 public:
  Config(const Json& j, std::string where, std::map<std::string, Json> defaults = {})
      : j_(j), where_(std::move(where)), defaults_(std::move(defaults)) {}

  const Json& operator[](const std::string& key) const {
    const Json& v = j_[key];
    if (!v.is_null()) return v;
    const auto it = defaults_.find(key);
    return it == defaults_.end() ? v : it->second;
  }
  std::string key(const std::string& k) const { return "config.json:" + where_ + k; }
  int64_t need(const std::string& k) const {
    const Json& v = (*this)[k];
    if (!v.is_number()) refuse(key(k) + ": missing or not a number");
    return v.as_int();
  }
  int64_t get(const std::string& k, int64_t def) const {
    const Json& v = (*this)[k];
    return v.is_number() ? v.as_int() : def;
  }
  bool flag(const std::string& k, bool def) const {
    const Json& v = (*this)[k];
    return v.is_bool() ? v.as_bool() : def;
  }
  std::string text(const std::string& k, const std::string& def) const {
    const Json& v = (*this)[k];
    return v.is_string() ? v.as_string() : def;
  }
  std::vector<int64_t> ints(const std::string& k, std::vector<int64_t> def) const {
    const Json& v = (*this)[k];
    if (!v.is_array()) return def;
    std::vector<int64_t> out;
    for (const auto& x : v.items()) {
      if (!x.is_number()) refuse(key(k) + ": a list of integers");
      out.push_back(x.as_int());
    }
    return out;
  }
  // A nested sub-config, read with its class defaults.
  Config sub(const std::string& k, std::map<std::string, Json> defaults) const {
    const Json& v = j_[k];
    if (!v.is_null() && !v.is_object()) refuse(key(k) + ": an object");
    return Config(v, where_ + k + ".", std::move(defaults));
  }
  // The model type a nested sub-config names, or `def`.
  std::string type_of(const std::string& k, const std::string& def) const {
    const Json& t = j_[k]["model_type"];
    return t.is_string() ? t.as_string() : def;
  }

 private:
  const Json& j_;
  std::string where_;
  std::map<std::string, Json> defaults_;
};

Json I(int64_t v) { return Json::integer(v); }

// Accumulates a composition: modules (tree lines) and their weights by checkpoint name.
struct Builder {
  Composition c;
  int depth = 0;
  void module(const std::string& line) { c.tree.push_back(std::string(2 * depth, ' ') + line); }
  void weight(const std::string& name, std::vector<int64_t> shape) { c.weights.push_back({name, std::move(shape)}); }
  void optional(const std::string& name, std::vector<int64_t> shape) {
    c.optional.push_back({name, std::move(shape)});
  }
  void ignore(const std::string& name) { c.ignored.push_back(name); }
  // A head that shares the embedding's values when `tied`, else a weight of its own.
  void head(const std::string& name, std::vector<int64_t> shape, bool tied) {
    if (tied) optional(name, std::move(shape));
    else weight(name, std::move(shape));
  }
  void linear(const std::string& p, int64_t out, int64_t in, bool bias) {
    weight(p + ".weight", {out, in});
    if (bias) weight(p + ".bias", {out});
  }
  void norm(const std::string& p, int64_t n, bool bias = false) {
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
  void leaf(const std::string& line) { module(line); }
};

Builder start(const std::string& family, const std::string& arch) {
  Builder b;
  b.c.family = family;
  b.c.architecture = arch;
  return b;
}

// ---- Shared blocks ---------------------------------------------------------------------------

// Gated MLP (SiLU or GELU): gate_proj, up_proj, down_proj.
void gated_mlp(Builder& b, const std::string& p, int64_t d, int64_t inner, bool bias = false) {
  b.linear(p + ".gate_proj", inner, d, bias);
  b.linear(p + ".up_proj", inner, d, bias);
  b.linear(p + ".down_proj", d, inner, bias);
}

// Grouped-query attention projections q/k/v/o.
void gqa(Builder& b, const std::string& p, int64_t d, int64_t heads, int64_t kv, int64_t hd, bool qkv_bias,
         bool o_bias = false) {
  b.linear(p + ".q_proj", heads * hd, d, qkv_bias);
  b.linear(p + ".k_proj", kv * hd, d, qkv_bias);
  b.linear(p + ".v_proj", kv * hd, d, qkv_bias);
  b.linear(p + ".o_proj", d, heads * hd, o_bias);
}

// Routed experts as the published checkpoints store them: one gate/up/down triple per expert.
void experts(Builder& b, const std::string& p, int64_t n, int64_t d, int64_t inner) {
  for (int64_t e = 0; e < n; ++e) gated_mlp(b, p + "." + str(e), d, inner);
}

int64_t labels(const Config& c) {
  const Json& m = c["id2label"];
  if (m.is_object() && m.size() > 0) return static_cast<int64_t>(m.size());
  return c.get("num_labels", 2);
}

void heads_divide(const Config& c, int64_t d, int64_t heads, const char* key = "num_attention_heads") {
  if (heads <= 0 || d % heads != 0) refuse(c.key(key) + ": does not divide hidden_size");
}

std::string head_line(bool tied) { return std::string("Final RMSNorm, head") + (tied ? " (tied to the embedding)" : ""); }

// ---- Encoders: BERT, XLM-RoBERTa (BGE-M3) ---------------------------------------------------

// The post-norm encoder stack of BERT and RoBERTa: embeddings, layers, the pooler when asked.
void bert_stack(Builder& b, const Config& cfg, const std::string& p, int64_t positions, bool pooler,
                bool pooler_optional = false) {
  const int64_t H = cfg.need("hidden_size"), L = cfg.need("num_hidden_layers"),
                heads = cfg.need("num_attention_heads"), I = cfg.need("intermediate_size"),
                V = cfg.need("vocab_size"), T = cfg.get("type_vocab_size", 2);
  heads_divide(cfg, H, heads);
  b.nest("Embeddings (word " + str(V) + " + position " + str(positions) + " + token type " + str(T) + ", LayerNorm)",
         [&] {
           b.weight(p + "embeddings.word_embeddings.weight", {V, H});
           b.weight(p + "embeddings.position_embeddings.weight", {positions, H});
           b.weight(p + "embeddings.token_type_embeddings.weight", {T, H});
           b.norm(p + "embeddings.LayerNorm", H, true);
         });
  b.nest("Layers x " + str(L) + " (" + str(heads) + "-head self-attention, add & LayerNorm, GELU MLP " + str(I) +
             ", add & LayerNorm)",
         [&] {
           for (int64_t l = 0; l < L; ++l) {
             const std::string q = p + "encoder.layer." + str(l) + ".";
             for (const char* n : {"query", "key", "value"}) b.linear(q + "attention.self." + n, H, H, true);
             b.linear(q + "attention.output.dense", H, H, true);
             b.norm(q + "attention.output.LayerNorm", H, true);
             b.linear(q + "intermediate.dense", I, H, true);
             b.linear(q + "output.dense", H, I, true);
             b.norm(q + "output.LayerNorm", H, true);
           }
         });
  if (pooler) {
    b.nest(std::string("Pooler (first token, dense, tanh)") + (pooler_optional ? ", optional" : ""), [&] {
      if (pooler_optional) {
        b.optional(p + "pooler.dense.weight", {H, H});
        b.optional(p + "pooler.dense.bias", {H});
      } else {
        b.linear(p + "pooler.dense", H, H, true);
      }
    });
  } else {
    b.ignore(p + "pooler.");
  }
  b.ignore(p + "embeddings.position_ids");
}

Composition bert(const Json& j, const std::string& arch, const Checkpoint& ck) {
  const Config cfg(j, "");
  Builder b = start("bert", arch);
  const int64_t H = cfg.need("hidden_size"), V = cfg.need("vocab_size"),
                P = cfg.get("max_position_embeddings", 512);
  if (arch == "BertModel") {
    // Checkpoints saved from a model with a head name the encoder under "bert.".
    const bool nested = ck.get("bert.embeddings.word_embeddings.weight") != nullptr;
    b.nest("BertModel (post-norm encoder, bidirectional attention)",
           [&] { bert_stack(b, cfg, nested ? "bert." : "", P, true); });
    if (nested) b.ignore("cls.");
  } else if (arch == "BertForMaskedLM") {
    b.nest("BertForMaskedLM", [&] {
      bert_stack(b, cfg, "bert.", P, false);
      b.nest("Masked-token head (dense, GELU, LayerNorm, decoder tied to the word embeddings, bias)", [&] {
        b.linear("cls.predictions.transform.dense", H, H, true);
        b.norm("cls.predictions.transform.LayerNorm", H, true);
        b.weight("cls.predictions.bias", {V});
        b.optional("cls.predictions.decoder.weight", {V, H});
        b.optional("cls.predictions.decoder.bias", {V});
      });
    });
    b.ignore("cls.seq_relationship.");
  } else {
    const bool sequence = arch == "BertForSequenceClassification";
    const int64_t n = labels(cfg);
    b.nest(arch, [&] {
      bert_stack(b, cfg, "bert.", P, sequence);
      b.nest(std::string(sequence ? "Classifier over the pooled first token" : "Classifier per token") + " (" +
                 str(n) + " labels)",
             [&] { b.linear("classifier", n, H, true); });
    });
  }
  return b.c;
}

Composition xlm_roberta(const Json& j, const std::string& arch, const Checkpoint& ck) {
  const Config cfg(j, "");
  Builder b = start("xlm_roberta", arch);
  // RoBERTa's positions start after the padding index: the table has max_position_embeddings rows.
  const int64_t P = cfg.get("max_position_embeddings", 514), H = cfg.need("hidden_size");
  if (arch == "XLMRobertaModel") {
    const bool nested = ck.get("roberta.embeddings.word_embeddings.weight") != nullptr;
    b.nest("XLMRobertaModel (BGE-M3's dense, sparse and multi-vector scores read its last hidden rows)",
           [&] { bert_stack(b, cfg, nested ? "roberta." : "", P, true, true); });
    if (nested) b.ignore("lm_head.");
  } else {
    const int64_t n = labels(cfg);
    b.nest(arch + " (cross-encoder reranker)", [&] {
      bert_stack(b, cfg, "roberta.", P, false);
      b.nest("Classification head over the first token (dense, tanh, out_proj to " + str(n) + ")", [&] {
        b.linear("classifier.dense", H, H, true);
        b.linear("classifier.out_proj", n, H, true);
      });
    });
  }
  return b.c;
}

// ---- Contrastive encoders: CLIP, SigLIP -----------------------------------------------------

std::map<std::string, Json> clip_text_defaults(bool siglip) {
  if (siglip)
    return {{"hidden_size", I(768)}, {"intermediate_size", I(3072)}, {"num_hidden_layers", I(12)},
            {"num_attention_heads", I(12)}, {"vocab_size", I(32000)}, {"max_position_embeddings", I(64)}};
  return {{"hidden_size", I(512)}, {"intermediate_size", I(2048)}, {"num_hidden_layers", I(12)},
          {"num_attention_heads", I(8)}, {"vocab_size", I(49408)}, {"max_position_embeddings", I(77)},
          {"projection_dim", I(512)}};
}

std::map<std::string, Json> clip_vision_defaults(bool siglip) {
  return {{"hidden_size", I(768)}, {"intermediate_size", I(3072)}, {"num_hidden_layers", I(12)},
          {"num_attention_heads", I(12)}, {"image_size", I(224)}, {"patch_size", I(siglip ? 16 : 32)},
          {"num_channels", I(3)}, {"projection_dim", I(512)}};
}

// Pre-norm encoder layers of CLIP and SigLIP (and of LLaVA's vision towers).
void clip_layers(Builder& b, const std::string& p, int64_t d, int64_t inner, int64_t L) {
  for (int64_t l = 0; l < L; ++l) {
    const std::string q = p + str(l) + ".";
    for (const char* n : {"q_proj", "k_proj", "v_proj", "out_proj"}) b.linear(q + "self_attn." + n, d, d, true);
    b.norm(q + "layer_norm1", d, true);
    b.linear(q + "mlp.fc1", inner, d, true);
    b.linear(q + "mlp.fc2", d, inner, true);
    b.norm(q + "layer_norm2", d, true);
  }
}

// A CLIP or SigLIP text tower under `p` ("text_model."); returns its width.
int64_t clip_text(Builder& b, const Config& c, const std::string& p, bool siglip) {
  const int64_t d = c.need("hidden_size"), I = c.need("intermediate_size"), L = c.need("num_hidden_layers"),
                heads = c.need("num_attention_heads"), V = c.need("vocab_size"), P = c.need("max_position_embeddings");
  heads_divide(c, d, heads);
  b.nest(std::string(siglip ? "SigLIP" : "CLIP") + " text tower (" + str(V) + " tokens, " + str(P) + " positions, " +
             str(L) + " pre-norm layers of " + str(heads) + " heads, " +
             (siglip ? "last token, head)" : "causal mask, end-of-text token)"),
         [&] {
           b.weight(p + "embeddings.token_embedding.weight", {V, d});
           b.weight(p + "embeddings.position_embedding.weight", {P, d});
           clip_layers(b, p + "encoder.layers.", d, I, L);
           b.norm(p + "final_layer_norm", d, true);
           if (siglip) b.linear(p + "head", c.get("projection_size", d), d, true);
         });
  b.ignore(p + "embeddings.position_ids");
  return d;
}

// A CLIP or SigLIP vision tower under `p` ("vision_model."); returns its width.
int64_t clip_vision(Builder& b, const Config& c, const std::string& p, bool siglip) {
  const int64_t d = c.need("hidden_size"), I = c.need("intermediate_size"), L = c.need("num_hidden_layers"),
                heads = c.need("num_attention_heads"), image = c.need("image_size"), patch = c.need("patch_size"),
                ch = c.get("num_channels", 3);
  heads_divide(c, d, heads);
  if (patch <= 0 || image % patch != 0) refuse(c.key("patch_size") + ": does not divide image_size");
  const int64_t patches = (image / patch) * (image / patch);
  const bool probe = siglip && c.flag("vision_use_head", true);
  b.nest(std::string(siglip ? "SigLIP" : "CLIP") + " vision tower (" + str(image) + "px, patches of " + str(patch) +
             ", " + str(L) + " pre-norm layers of " + str(heads) + " heads" +
             (siglip ? (probe ? ", attention-pooling head)" : ")") : ", class token)"),
         [&] {
           if (siglip) {
             b.weight(p + "embeddings.patch_embedding.weight", {d, ch, patch, patch});
             b.weight(p + "embeddings.patch_embedding.bias", {d});
             b.weight(p + "embeddings.position_embedding.weight", {patches, d});
           } else {
             b.weight(p + "embeddings.class_embedding", {d});
             b.weight(p + "embeddings.patch_embedding.weight", {d, ch, patch, patch});
             b.weight(p + "embeddings.position_embedding.weight", {patches + 1, d});
             b.norm(p + "pre_layrnorm", d, true);
           }
           clip_layers(b, p + "encoder.layers.", d, I, L);
           b.norm(p + "post_layernorm", d, true);
           if (probe) {
             b.weight(p + "head.probe", {1, 1, d});
             b.weight(p + "head.attention.in_proj_weight", {3 * d, d});
             b.weight(p + "head.attention.in_proj_bias", {3 * d});
             b.linear(p + "head.attention.out_proj", d, d, true);
             b.norm(p + "head.layernorm", d, true);
             b.linear(p + "head.mlp.fc1", I, d, true);
             b.linear(p + "head.mlp.fc2", d, I, true);
           }
         });
  b.ignore(p + "embeddings.position_ids");
  return d;
}

Composition clip(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const bool siglip = arch.rfind("Siglip", 0) == 0;
  Builder b = start(siglip ? "siglip" : "clip", arch);
  b.nest(arch, [&] {
    if (arch == "CLIPModel" || arch == "SiglipModel") {
      const int64_t dt = clip_text(b, cfg.sub("text_config", clip_text_defaults(siglip)), "text_model.", siglip);
      const int64_t dv = clip_vision(b, cfg.sub("vision_config", clip_vision_defaults(siglip)), "vision_model.", siglip);
      if (siglip) {
        b.nest("Sigmoid loss scale and bias", [&] {
          b.weight("logit_scale", {1});
          b.weight("logit_bias", {1});
        });
      } else {
        const int64_t proj = cfg.get("projection_dim", 512);
        b.nest("Projections to a shared space of " + str(proj) + " (no bias), logit scale", [&] {
          b.weight("visual_projection.weight", {proj, dv});
          b.weight("text_projection.weight", {proj, dt});
          b.weight("logit_scale", {});
        });
      }
    } else if (arch.find("Text") != std::string::npos) {
      const Config c(j, "", clip_text_defaults(siglip));
      const int64_t d = clip_text(b, c, "text_model.", siglip);
      if (arch == "CLIPTextModelWithProjection")
        b.nest("Projection (no bias)", [&] { b.weight("text_projection.weight", {c.need("projection_dim"), d}); });
    } else {
      const Config c(j, "", clip_vision_defaults(siglip));
      const int64_t d = clip_vision(b, c, "vision_model.", siglip);
      if (arch == "CLIPVisionModelWithProjection")
        b.nest("Projection (no bias)", [&] { b.weight("visual_projection.weight", {c.need("projection_dim"), d}); });
    }
  });
  return b.c;
}

// ---- Encoder-decoders: T5 / mT5, Whisper ---------------------------------------------------

// T5 / mT5 (pre-norm RMSNorm, relative position buckets in the first block of each stack, ReLU or
// gated-GELU feed-forward).
Composition t5(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const int64_t d = cfg.need("d_model"), d_kv = cfg.need("d_kv"), ff = cfg.need("d_ff"),
                heads = cfg.need("num_heads"), L = cfg.need("num_layers"), Ld = cfg.get("num_decoder_layers", L),
                V = cfg.need("vocab_size"), buckets = cfg.get("relative_attention_num_buckets", 32);
  const std::string ffp = cfg.text("feed_forward_proj", "relu");
  const bool gated = ffp.rfind("gated-", 0) == 0;
  const bool tied = cfg.flag("tie_word_embeddings", true);
  const bool encoder_only = arch == "T5EncoderModel";
  const int64_t inner = heads * d_kv;
  Builder b = start("t5", arch);
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
  b.nest(arch + " (" + ffp + " feed-forward " + str(ff) + ", " + str(heads) + " heads of " + str(d_kv) + ")", [&] {
    b.weight("shared.weight", {V, d});
    b.optional("encoder.embed_tokens.weight", {V, d});  // each stack's embedding is the shared one
    b.nest("Encoder x " + str(L) + " (self-attention, feed-forward; RMSNorm before each)", [&] {
      for (int64_t l = 0; l < L; ++l) {
        const std::string p = "encoder.block." + str(l) + ".layer.";
        attention(p + "0.SelfAttention", l == 0);
        b.weight(p + "0.layer_norm.weight", {d});
        feed_forward(p + "1");
      }
      b.weight("encoder.final_layer_norm.weight", {d});
    });
    if (encoder_only) return;
    b.optional("decoder.embed_tokens.weight", {V, d});
    b.nest("Decoder x " + str(Ld) + " (causal self-attention, cross-attention, feed-forward)", [&] {
      for (int64_t l = 0; l < Ld; ++l) {
        const std::string p = "decoder.block." + str(l) + ".layer.";
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

// Whisper (two convolutions over log-mel frames, learned positions, pre-norm LayerNorm blocks;
// key projections without bias).
Composition whisper(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const int64_t d = cfg.need("d_model"), mels = cfg.get("num_mel_bins", 80), Le = cfg.need("encoder_layers"),
                Ld = cfg.need("decoder_layers"), ffe = cfg.need("encoder_ffn_dim"), ffd = cfg.need("decoder_ffn_dim"),
                V = cfg.need("vocab_size"), src = cfg.get("max_source_positions", 1500),
                tgt = cfg.get("max_target_positions", 448);
  Builder b = start("whisper", arch);
  auto attention = [&](const std::string& p) {
    b.linear(p + ".q_proj", d, d, true);
    b.linear(p + ".k_proj", d, d, false);
    b.linear(p + ".v_proj", d, d, true);
    b.linear(p + ".out_proj", d, d, true);
  };
  b.nest(arch, [&] {
    b.nest("Encoder (conv k3 from " + str(mels) + " mel bins, GELU, conv k3 stride 2, GELU, positions) x " + str(Le),
           [&] {
             b.weight("model.encoder.conv1.weight", {d, mels, 3});
             b.weight("model.encoder.conv1.bias", {d});
             b.weight("model.encoder.conv2.weight", {d, d, 3});
             b.weight("model.encoder.conv2.bias", {d});
             b.weight("model.encoder.embed_positions.weight", {src, d});
             for (int64_t l = 0; l < Le; ++l) {
               const std::string p = "model.encoder.layers." + str(l) + ".";
               attention(p + "self_attn");
               b.norm(p + "self_attn_layer_norm", d, true);
               b.linear(p + "fc1", ffe, d, true);
               b.linear(p + "fc2", d, ffe, true);
               b.norm(p + "final_layer_norm", d, true);
             }
             b.norm("model.encoder.layer_norm", d, true);
           });
    b.nest("Decoder (tokens, positions; causal self-attention, cross-attention, GELU MLP) x " + str(Ld), [&] {
      b.weight("model.decoder.embed_tokens.weight", {V, d});
      b.weight("model.decoder.embed_positions.weight", {tgt, d});
      for (int64_t l = 0; l < Ld; ++l) {
        const std::string p = "model.decoder.layers." + str(l) + ".";
        attention(p + "self_attn");
        b.norm(p + "self_attn_layer_norm", d, true);
        attention(p + "encoder_attn");
        b.norm(p + "encoder_attn_layer_norm", d, true);
        b.linear(p + "fc1", ffd, d, true);
        b.linear(p + "fc2", d, ffd, true);
        b.norm(p + "final_layer_norm", d, true);
      }
      b.norm("model.decoder.layer_norm", d, true);
    });
    b.head("proj_out.weight", {V, d}, cfg.flag("tie_word_embeddings", true));
  });
  return b.c;
}

// ---- Recurrent and hybrid decoders: Mamba, Mamba-2, Bamba ----------------------------------

// One Mamba-2 mixer under `p` (in_proj to z, x, B, C, dt; causal depthwise conv over x, B, C;
// per-head A, D and dt bias; gated RMSNorm; out_proj).
void mamba2_mixer(Builder& b, const std::string& p, int64_t d, int64_t inner, int64_t heads, int64_t groups,
                  int64_t state, int64_t conv, bool bias, bool conv_bias) {
  const int64_t conv_dim = inner + 2 * groups * state;
  b.linear(p + "in_proj", 2 * inner + 2 * groups * state + heads, d, bias);
  b.weight(p + "conv1d.weight", {conv_dim, 1, conv});
  if (conv_bias) b.weight(p + "conv1d.bias", {conv_dim});
  b.weight(p + "dt_bias", {heads});
  b.weight(p + "A_log", {heads});
  b.weight(p + "D", {heads});
  b.weight(p + "norm.weight", {inner});
  b.linear(p + "out_proj", d, inner, bias);
}

std::string mamba2_line(int64_t heads, int64_t head_dim, int64_t groups, int64_t state, int64_t conv) {
  return "Mixer: in_proj to z, x, B, C (" + str(groups) + " groups of state " + str(state) + ") and dt (" +
         str(heads) + " heads of " + str(head_dim) + "); causal conv " + str(conv) +
         " over x, B, C; SiLU; SSD scan with A = -exp(A_log), D skip; RMSNorm gated by SiLU(z); out_proj";
}

Composition mamba(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const int64_t d = cfg.need("hidden_size"), L = cfg.need("num_hidden_layers"), V = cfg.need("vocab_size"),
                state = cfg.get("state_size", 16), conv = cfg.get("conv_kernel", 4), expand = cfg.get("expand", 2),
                inner = cfg.get("intermediate_size", expand * d);
  const Json& r = cfg["time_step_rank"];
  const int64_t rank = r.is_number() ? r.as_int() : (d + 15) / 16;  // "auto": ceil(hidden / 16)
  const bool bias = cfg.flag("use_bias", false), conv_bias = cfg.flag("use_conv_bias", true),
             tied = cfg.flag("tie_word_embeddings", true);
  Builder b = start("mamba", arch);
  b.nest(arch + " (RMSNorm, Mamba mixer, residual) x " + str(L), [&] {
    b.nest("Embedding " + str(V) + " x " + str(d), [&] { b.weight("backbone.embeddings.weight", {V, d}); });
    b.leaf("Mixer: in_proj to x and z (" + str(inner) + "); causal conv " + str(conv) +
           " over x; SiLU; x_proj to dt (rank " + str(rank) + "), B, C (state " + str(state) +
           "); dt_proj, softplus; selective scan with A = -exp(A_log), D skip; gate SiLU(z); out_proj");
    for (int64_t l = 0; l < L; ++l) {
      const std::string p = "backbone.layers." + str(l) + ".";
      b.weight(p + "norm.weight", {d});
      b.linear(p + "mixer.in_proj", 2 * inner, d, bias);
      b.weight(p + "mixer.conv1d.weight", {inner, 1, conv});
      if (conv_bias) b.weight(p + "mixer.conv1d.bias", {inner});
      b.weight(p + "mixer.x_proj.weight", {rank + 2 * state, inner});
      b.linear(p + "mixer.dt_proj", inner, rank, true);
      b.weight(p + "mixer.A_log", {inner, state});
      b.weight(p + "mixer.D", {inner});
      b.linear(p + "mixer.out_proj", d, inner, bias);
    }
    b.nest(head_line(tied), [&] {
      b.weight("backbone.norm_f.weight", {d});
      b.head("lm_head.weight", {V, d}, tied);
    });
  });
  return b.c;
}

Composition mamba2(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const int64_t d = cfg.need("hidden_size"), L = cfg.need("num_hidden_layers"), V = cfg.need("vocab_size"),
                state = cfg.need("state_size"), groups = cfg.get("n_groups", 1), conv = cfg.get("conv_kernel", 4),
                expand = cfg.get("expand", 2), head_dim = cfg.get("head_dim", 64);
  const int64_t inner = expand * d;
  if (head_dim <= 0 || inner % head_dim != 0) refuse(cfg.key("head_dim") + ": does not divide expand * hidden_size");
  const int64_t heads = cfg.get("num_heads", inner / head_dim);
  if (heads * head_dim != inner)
    refuse(cfg.key("num_heads") + ": num_heads * head_dim differs from expand * hidden_size");
  const bool bias = cfg.flag("use_bias", false), conv_bias = cfg.flag("use_conv_bias", true),
             tied = cfg.flag("tie_word_embeddings", false);
  Builder b = start("mamba2", arch);
  b.nest(arch + " (RMSNorm, Mamba-2 mixer, residual) x " + str(L), [&] {
    b.nest("Embedding " + str(V) + " x " + str(d), [&] { b.weight("backbone.embeddings.weight", {V, d}); });
    b.leaf(mamba2_line(heads, head_dim, groups, state, conv));
    for (int64_t l = 0; l < L; ++l) {
      const std::string p = "backbone.layers." + str(l) + ".";
      b.weight(p + "norm.weight", {d});
      mamba2_mixer(b, p + "mixer.", d, inner, heads, groups, state, conv, bias, conv_bias);
    }
    b.nest(head_line(tied), [&] {
      b.weight("backbone.norm_f.weight", {d});
      b.head("lm_head.weight", {V, d}, tied);
    });
  });
  return b.c;
}

// Bamba: Mamba-2 mixers with attention at the listed layers, a gated MLP after every mixer.
Composition bamba(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const int64_t d = cfg.need("hidden_size"), L = cfg.need("num_hidden_layers"), V = cfg.need("vocab_size"),
                heads = cfg.need("num_attention_heads"), kv = cfg.get("num_key_value_heads", heads),
                I = cfg.need("intermediate_size"), mh = cfg.need("mamba_n_heads"), mhd = cfg.get("mamba_d_head", 64),
                groups = cfg.get("mamba_n_groups", 1), state = cfg.get("mamba_d_state", 256),
                conv = cfg.get("mamba_d_conv", 4), expand = cfg.get("mamba_expand", 2);
  const int64_t inner = expand * d;
  if (mh * mhd != inner)
    refuse(cfg.key("mamba_n_heads") + ": mamba_n_heads * mamba_d_head differs from mamba_expand * hidden_size");
  heads_divide(cfg, d, heads);
  const std::vector<int64_t> attn = cfg.ints("attn_layer_indices", {});
  const std::set<int64_t> at(attn.begin(), attn.end());
  for (auto l : at)
    if (l < 0 || l >= L) refuse(cfg.key("attn_layer_indices") + ": layer " + str(l) + " out of range");
  const bool tied = cfg.flag("tie_word_embeddings", false), ab = cfg.flag("attention_bias", false),
             mb = cfg.flag("mlp_bias", false);
  const int64_t n_attn = static_cast<int64_t>(at.size());
  Builder b = start("bamba", arch);
  b.nest(arch + " x " + str(L) + " (" + str(n_attn) + " attention, " + str(L - n_attn) +
             " Mamba-2; each followed by a gated MLP " + str(I) + ")",
         [&] {
           b.nest("Embedding " + str(V) + " x " + str(d), [&] { b.weight("model.embed_tokens.weight", {V, d}); });
           b.leaf(mamba2_line(mh, mhd, groups, state, conv));
           b.leaf("Attention at layers " + joined(at) + ": " + str(heads) + " query heads, " + str(kv) +
                  " KV heads of " + str(d / heads) + "; partial RoPE");
           for (int64_t l = 0; l < L; ++l) {
             const std::string p = "model.layers." + str(l) + ".";
             b.weight(p + "input_layernorm.weight", {d});
             if (at.count(l))
               gqa(b, p + "self_attn", d, heads, kv, d / heads, ab, ab);
             else
               mamba2_mixer(b, p + "mamba.", d, inner, mh, groups, state, conv, cfg.flag("mamba_proj_bias", false),
                            cfg.flag("mamba_conv_bias", true));
             b.weight(p + "pre_ff_layernorm.weight", {d});
             gated_mlp(b, p + "feed_forward", d, I, mb);
           }
           b.nest(head_line(tied), [&] {
             b.weight("model.final_layernorm.weight", {d});
             b.head("lm_head.weight", {V, d}, tied);
           });
         });
  return b.c;
}

// ---- Attention decoders: Gemma-3 and Gemma-4 text, OLMoE, DeepSeek-V2 -----------------------

// Marks the config's full-attention layers (from `layer_types`, else one every
// `sliding_window_pattern`) and returns their count.
int64_t global_layers(const Config& cfg, int64_t L, std::vector<bool>* full) {
  full->assign(L, false);
  const Json& types = cfg["layer_types"];
  int64_t global = 0;
  if (types.is_array()) {
    if (static_cast<int64_t>(types.size()) != L) refuse(cfg.key("layer_types") + ": one entry a layer");
    for (int64_t l = 0; l < L; ++l) {
      const Json& t = types.at(l);
      if (!t.is_string() || (t.as_string() != "full_attention" && t.as_string() != "sliding_attention"))
        refuse(cfg.key("layer_types") + ": full_attention or sliding_attention");
      (*full)[l] = t.as_string() == "full_attention";
      global += (*full)[l];
    }
  } else {
    const int64_t pattern = cfg.get("sliding_window_pattern", 6);
    if (pattern <= 0) refuse(cfg.key("sliding_window_pattern") + ": at least 1");
    for (int64_t l = 0; l < L; ++l) {
      (*full)[l] = (l + 1) % pattern == 0;
      global += (*full)[l];
    }
  }
  return global;
}

// Gemma-3 text decoder (GQA with QK RMSNorm, sandwich norms around attention and MLP, GeGLU MLP,
// local sliding-window and global layers, tied embeddings).
Composition gemma3_text(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const int64_t d = cfg.need("hidden_size"), L = cfg.need("num_hidden_layers"), V = cfg.need("vocab_size"),
                heads = cfg.need("num_attention_heads"), kv = cfg.get("num_key_value_heads", heads),
                I = cfg.need("intermediate_size"), hd = cfg.get("head_dim", 256);
  if (kv <= 0 || heads % kv != 0) refuse(cfg.key("num_key_value_heads") + ": does not divide num_attention_heads");
  std::vector<bool> full;
  const int64_t global = global_layers(cfg, L, &full);
  const int64_t window = cfg.get("sliding_window", 4096);
  const bool tied = cfg.flag("tie_word_embeddings", true);
  Builder b = start("gemma3_text", arch);
  b.nest(arch + " x " + str(L) + " (" + str(global) + " global, " + str(L - global) + " sliding-window of " +
             str(window) + "; sandwich RMSNorms, QK RMSNorm, GeGLU MLP)",
         [&] {
           b.nest("Embedding " + str(V) + " x " + str(d) + ", scaled by sqrt(hidden_size)",
                  [&] { b.weight("model.embed_tokens.weight", {V, d}); });
           b.leaf("Attention: " + str(heads) + " query heads, " + str(kv) + " KV heads of " + str(hd) +
                  "; RMSNorm of q and k; RoPE (local and global bases)");
           b.leaf("MLP: gelu_tanh(gate) * up, down (" + str(I) + ")");
           for (int64_t l = 0; l < L; ++l) {
             const std::string p = "model.layers." + str(l) + ".";
             b.weight(p + "input_layernorm.weight", {d});
             gqa(b, p + "self_attn", d, heads, kv, hd, false);
             b.weight(p + "self_attn.q_norm.weight", {hd});
             b.weight(p + "self_attn.k_norm.weight", {hd});
             b.weight(p + "post_attention_layernorm.weight", {d});
             b.weight(p + "pre_feedforward_layernorm.weight", {d});
             gated_mlp(b, p + "mlp", d, I);
             b.weight(p + "post_feedforward_layernorm.weight", {d});
           }
           b.nest(head_line(tied), [&] {
             b.weight("model.norm.weight", {d});
             b.head("lm_head.weight", {V, d}, tied);
           });
         });
  return b.c;
}

// Gemma-4 text decoder: Gemma-3's layer plus global layers of a wider head (optionally keys as
// values, with their own KV head count), per-layer input embeddings gated into every layer, a
// learned per-layer scalar, KV shared by the last layers (whose MLP may be twice as wide), and an
// optional mixture-of-experts block beside the MLP.
Composition gemma4_text(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const int64_t d = cfg.need("hidden_size"), L = cfg.need("num_hidden_layers"), V = cfg.need("vocab_size"),
                heads = cfg.need("num_attention_heads"), kv = cfg.get("num_key_value_heads", heads),
                I = cfg.need("intermediate_size"), hd = cfg.get("head_dim", 256), ghd = cfg.get("global_head_dim", hd),
                gkv = cfg.get("num_global_key_value_heads", kv), ple = cfg.get("hidden_size_per_layer_input", 0),
                ple_vocab = cfg.get("vocab_size_per_layer_input", V), shared = cfg.get("num_kv_shared_layers", 0);
  const bool k_eq_v = cfg.flag("attention_k_eq_v", false), bias = cfg.flag("attention_bias", false),
             wide = cfg.flag("use_double_wide_mlp", false), moe = cfg.flag("enable_moe_block", false),
             tied = cfg.flag("tie_word_embeddings", true);
  if (shared < 0 || shared > L) refuse(cfg.key("num_kv_shared_layers") + ": between 0 and num_hidden_layers");
  std::vector<bool> full;
  const int64_t global = global_layers(cfg, L, &full);
  const int64_t first_shared = L - shared;
  Builder b = start("gemma4_text", arch);
  b.nest(arch + " x " + str(L) + " (" + str(global) + " global with heads of " + str(ghd) + ", " + str(L - global) +
             " sliding-window of " + str(cfg.get("sliding_window", 512)) + " with heads of " + str(hd) +
             (shared > 0 ? "; the last " + str(shared) + " reuse earlier layers' KV" : "") +
             (moe ? "; MoE block" : "") + ")",
         [&] {
           b.nest("Embedding " + str(V) + " x " + str(d) + ", scaled by sqrt(hidden_size)",
                  [&] { b.weight("model.embed_tokens.weight", {V, d}); });
           if (ple > 0) {
             b.nest("Per-layer inputs: embedding " + str(ple_vocab) + " x " + str(L) + "*" + str(ple) +
                        " plus a projection of the embedded rows, RMSNorm",
                    [&] {
                      b.weight("model.embed_tokens_per_layer.weight", {ple_vocab, L * ple});
                      b.weight("model.per_layer_model_projection.weight", {L * ple, d});
                      b.weight("model.per_layer_projection_norm.weight", {ple});
                    });
           }
           for (int64_t l = 0; l < L; ++l) {
             const std::string p = "model.layers." + str(l) + ".";
             const bool g = full[l];
             const int64_t h = g ? ghd : hd;
             const bool alt = k_eq_v && g;  // keys double as values
             const int64_t nkv = alt ? gkv : kv;
             if (nkv <= 0 || heads % nkv != 0)
               refuse(cfg.key(alt ? "num_global_key_value_heads" : "num_key_value_heads") +
                      ": does not divide num_attention_heads");
             b.weight(p + "layer_scalar", {1});
             b.weight(p + "input_layernorm.weight", {d});
             b.linear(p + "self_attn.q_proj", heads * h, d, bias);
             b.linear(p + "self_attn.k_proj", nkv * h, d, bias);
             if (!alt) b.linear(p + "self_attn.v_proj", nkv * h, d, bias);
             b.linear(p + "self_attn.o_proj", d, heads * h, bias);
             b.weight(p + "self_attn.q_norm.weight", {h});
             b.weight(p + "self_attn.k_norm.weight", {h});
             b.weight(p + "post_attention_layernorm.weight", {d});
             b.weight(p + "pre_feedforward_layernorm.weight", {d});
             gated_mlp(b, p + "mlp", d, (wide && first_shared > 0 && l >= first_shared) ? 2 * I : I);
             b.weight(p + "post_feedforward_layernorm.weight", {d});
             if (ple > 0) {
               b.weight(p + "per_layer_input_gate.weight", {ple, d});
               b.weight(p + "per_layer_projection.weight", {d, ple});
               b.weight(p + "post_per_layer_input_norm.weight", {d});
             }
             if (moe) {
               const int64_t E = cfg.need("num_experts"), mi = cfg.need("moe_intermediate_size");
               b.weight(p + "router.proj.weight", {E, d});
               b.weight(p + "router.scale", {d});
               b.weight(p + "router.per_expert_scale", {E});
               b.weight(p + "experts.gate_up_proj", {E, 2 * mi, d});
               b.weight(p + "experts.down_proj", {E, d, mi});
               for (const char* n :
                    {"post_feedforward_layernorm_1", "post_feedforward_layernorm_2", "pre_feedforward_layernorm_2"})
                 b.weight(p + n + ".weight", {d});
             }
           }
           b.nest(head_line(tied), [&] {
             b.weight("model.norm.weight", {d});
             b.head("lm_head.weight", {V, d}, tied);
           });
         });
  return b.c;
}

// OLMoE: Llama-style attention with RMSNorm over the whole q and k projections, a routed SwiGLU
// expert block in every layer.
Composition olmoe(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const int64_t d = cfg.need("hidden_size"), L = cfg.need("num_hidden_layers"), V = cfg.need("vocab_size"),
                heads = cfg.need("num_attention_heads"), kv = cfg.get("num_key_value_heads", heads),
                I = cfg.need("intermediate_size"), E = cfg.need("num_experts"), k = cfg.get("num_experts_per_tok", 8);
  heads_divide(cfg, d, heads);
  const int64_t hd = d / heads;
  const bool tied = cfg.flag("tie_word_embeddings", false), bias = cfg.flag("attention_bias", false);
  Builder b = start("olmoe", arch);
  b.nest(arch + " x " + str(L) + " (" + str(E) + " experts of " + str(I) + ", top " + str(k) +
             "; RMSNorm over the whole q and k projections)",
         [&] {
           b.weight("model.embed_tokens.weight", {V, d});
           b.leaf("Attention: " + str(heads) + " query heads, " + str(kv) + " KV heads of " + str(hd) + "; RoPE");
           b.leaf("Experts: router softmax over " + str(E) + ", top " + str(k) + (cfg.flag("norm_topk_prob", false)
                                                                                  ? " renormalised"
                                                                                  : " unnormalised") +
                  ", SwiGLU " + str(I));
           for (int64_t l = 0; l < L; ++l) {
             const std::string p = "model.layers." + str(l) + ".";
             b.weight(p + "input_layernorm.weight", {d});
             gqa(b, p + "self_attn", d, heads, kv, hd, bias, bias);
             b.weight(p + "self_attn.q_norm.weight", {heads * hd});
             b.weight(p + "self_attn.k_norm.weight", {kv * hd});
             b.weight(p + "post_attention_layernorm.weight", {d});
             b.weight(p + "mlp.gate.weight", {E, d});
             experts(b, p + "mlp.experts", E, d, I);
           }
           b.weight("model.norm.weight", {d});
           b.head("lm_head.weight", {V, d}, tied);
         });
  return b.c;
}

// DeepSeek-V2: multi-head latent attention (low-rank KV with a shared rotary key, optional
// low-rank queries) and a mixture of routed and shared experts after the first dense layers.
Composition deepseek_v2(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const int64_t d = cfg.need("hidden_size"), L = cfg.need("num_hidden_layers"), V = cfg.need("vocab_size"),
                heads = cfg.need("num_attention_heads"), I = cfg.need("intermediate_size"),
                kv_rank = cfg.need("kv_lora_rank"), nope = cfg.need("qk_nope_head_dim"),
                rope = cfg.need("qk_rope_head_dim"), vd = cfg.need("v_head_dim"), E = cfg.get("n_routed_experts", 0),
                shared = cfg.get("n_shared_experts", 0), mi = cfg.get("moe_intermediate_size", 0),
                dense = cfg.get("first_k_dense_replace", 0), freq = cfg.get("moe_layer_freq", 1),
                q_rank = cfg.get("q_lora_rank", 0);
  if (freq <= 0) refuse(cfg.key("moe_layer_freq") + ": at least 1");
  const bool tied = cfg.flag("tie_word_embeddings", false), bias = cfg.flag("attention_bias", false);
  Builder b = start("deepseek_v2", arch);
  b.nest(arch + " x " + str(L) + " (latent attention: KV rank " + str(kv_rank) +
             (q_rank > 0 ? ", query rank " + str(q_rank) : std::string()) + "; " + str(E) + " routed + " +
             str(shared) + " shared experts of " + str(mi) + " after " + str(dense) + " dense layers)",
         [&] {
           b.weight("model.embed_tokens.weight", {V, d});
           b.leaf("Latent attention: " + str(heads) + " heads; keys " + str(nope) + " + rotary " + str(rope) +
                  ", values " + str(vd) + "; the cache holds the " + str(kv_rank) + "-wide latent and one rotary key");
           b.leaf("Experts: router over " + str(E) + " (" + cfg.text("topk_method", "greedy") + "), top " +
                  str(cfg.get("num_experts_per_tok", 6)) + ", plus " + str(shared) + " shared, SwiGLU " + str(mi));
           for (int64_t l = 0; l < L; ++l) {
             const std::string p = "model.layers." + str(l) + ".";
             b.weight(p + "input_layernorm.weight", {d});
             if (q_rank > 0) {
               b.linear(p + "self_attn.q_a_proj", q_rank, d, bias);
               b.weight(p + "self_attn.q_a_layernorm.weight", {q_rank});
               b.weight(p + "self_attn.q_b_proj.weight", {heads * (nope + rope), q_rank});
             } else {
               b.weight(p + "self_attn.q_proj.weight", {heads * (nope + rope), d});
             }
             b.linear(p + "self_attn.kv_a_proj_with_mqa", kv_rank + rope, d, bias);
             b.weight(p + "self_attn.kv_a_layernorm.weight", {kv_rank});
             b.weight(p + "self_attn.kv_b_proj.weight", {heads * (nope + vd), kv_rank});
             b.linear(p + "self_attn.o_proj", d, heads * vd, bias);
             b.weight(p + "post_attention_layernorm.weight", {d});
             if (E > 0 && l >= dense && l % freq == 0) {
               b.weight(p + "mlp.gate.weight", {E, d});
               experts(b, p + "mlp.experts", E, d, mi);
               if (shared > 0) gated_mlp(b, p + "mlp.shared_experts", d, mi * shared);
             } else {
               gated_mlp(b, p + "mlp", d, I);
             }
           }
           b.weight("model.norm.weight", {d});
           b.head("lm_head.weight", {V, d}, tied);
         });
  return b.c;
}

// ---- Vision-language: LLaVA, Mllama, Qwen3-VL ----------------------------------------------

std::map<std::string, Json> text_defaults(const std::string& type) {
  if (type == "mistral")
    return {{"hidden_size", I(4096)}, {"intermediate_size", I(14336)}, {"num_hidden_layers", I(32)},
            {"num_attention_heads", I(32)}, {"num_key_value_heads", I(8)}, {"vocab_size", I(32000)}};
  if (type == "qwen2")
    return {{"hidden_size", I(4096)}, {"intermediate_size", I(22016)}, {"num_hidden_layers", I(32)},
            {"num_attention_heads", I(32)}, {"num_key_value_heads", I(32)}, {"vocab_size", I(151936)}};
  return {{"hidden_size", I(4096)}, {"intermediate_size", I(11008)}, {"num_hidden_layers", I(32)},
          {"num_attention_heads", I(32)}, {"vocab_size", I(32000)}};
}

// A Llama, Mistral, Qwen2 or Qwen3 text decoder whose embedding, layers and final norm sit under
// `model` ("...embed_tokens", "...layers.N", "...norm"), its head at `head`.
void text_decoder(Builder& b, const Config& t, const std::string& type, const std::string& model,
                  const std::string& head, bool tied) {
  const int64_t d = t.need("hidden_size"), L = t.need("num_hidden_layers"), V = t.need("vocab_size"),
                heads = t.need("num_attention_heads"), kv = t.get("num_key_value_heads", heads),
                I = t.need("intermediate_size");
  heads_divide(t, d, heads);
  const int64_t hd = t.get("head_dim", d / heads);
  if (kv <= 0 || heads % kv != 0) refuse(t.key("num_key_value_heads") + ": does not divide num_attention_heads");
  const bool qwen2 = type == "qwen2", qk_norm = type.rfind("qwen3", 0) == 0;
  const bool ab = t.flag("attention_bias", false);
  b.nest("Text decoder (" + type + ") x " + str(L) + ": " + str(heads) + " query heads, " + str(kv) +
             " KV heads of " + str(hd) + (qk_norm ? ", QK RMSNorm" : "") + ", SwiGLU MLP " + str(I),
         [&] {
           b.weight(model + "embed_tokens.weight", {V, d});
           for (int64_t l = 0; l < L; ++l) {
             const std::string p = model + "layers." + str(l) + ".";
             b.weight(p + "input_layernorm.weight", {d});
             gqa(b, p + "self_attn", d, heads, kv, hd, qwen2 || ab, !qwen2 && ab);
             if (qk_norm) {
               b.weight(p + "self_attn.q_norm.weight", {hd});
               b.weight(p + "self_attn.k_norm.weight", {hd});
             }
             b.weight(p + "post_attention_layernorm.weight", {d});
             gated_mlp(b, p + "mlp", d, I, t.flag("mlp_bias", false));
           }
           b.weight(model + "norm.weight", {d});
           b.head(head, {V, d}, tied);
         });
}

// Where a vision-language checkpoint keeps its parts: transformers' own layout ("model.…") or the
// layout the hub's first exports used ("language_model.model.…").
struct Layout {
  std::string vision, projector, text, head;
};

Layout layout(const Checkpoint& ck, const std::string& vision) {
  if (ck.get("language_model.model.embed_tokens.weight") != nullptr)
    return {vision, "multi_modal_projector", "language_model.model.", "language_model.lm_head.weight"};
  return {"model." + vision, "model.multi_modal_projector", "model.language_model.", "lm_head.weight"};
}

Composition llava(const Json& j, const std::string& arch, const Checkpoint& ck) {
  const Config cfg(j, "");
  const std::string ttype = cfg.type_of("text_config", "llama");
  if (ttype != "llama" && ttype != "mistral" && ttype != "qwen2")
    refuse("config.json:text_config.model_type: llama, mistral or qwen2");
  const Config tc = cfg.sub("text_config", text_defaults(ttype));
  const std::string vtype = cfg.type_of("vision_config", "clip_vision_model");
  const bool siglip = vtype == "siglip_vision_model";
  if (!siglip && vtype != "clip_vision_model")
    refuse("config.json:vision_config.model_type: clip_vision_model or siglip_vision_model");
  const Config vc = cfg.sub("vision_config", clip_vision_defaults(siglip));
  const Layout at = layout(ck, "vision_tower.");
  const bool tied = cfg.flag("tie_word_embeddings", tc.flag("tie_word_embeddings", false));
  const bool pbias = cfg.flag("multimodal_projector_bias", true);
  Builder b = start("llava", arch);
  b.nest(arch + " (image features from vision layer " + str(cfg.get("vision_feature_layer", -2)) +
             ", projected into the text decoder's rows)",
         [&] {
           const int64_t dv = clip_vision(b, vc, at.vision + "vision_model.", siglip);
           const int64_t dt = tc.need("hidden_size");
           b.nest("Projector (linear, " + cfg.text("projector_hidden_act", "gelu") + ", linear)", [&] {
             b.linear(at.projector + ".linear_1", dt, dv, pbias);
             b.linear(at.projector + ".linear_2", dt, dt, pbias);
           });
           text_decoder(b, tc, ttype, at.text, at.head, tied);
         });
  return b.c;
}

Composition mllama(const Json& j, const std::string& arch, const Checkpoint& ck) {
  const Config cfg(j, "");
  const Config vc = cfg.sub("vision_config",
                            {{"hidden_size", I(1280)}, {"intermediate_size", I(5120)}, {"num_hidden_layers", I(32)},
                             {"num_global_layers", I(8)}, {"attention_heads", I(16)}, {"num_channels", I(3)},
                             {"image_size", I(448)}, {"patch_size", I(14)}, {"max_num_tiles", I(4)},
                             {"vision_output_dim", I(7680)}});
  const Config tc = cfg.sub("text_config",
                            {{"hidden_size", I(4096)}, {"intermediate_size", I(14336)}, {"num_hidden_layers", I(40)},
                             {"num_attention_heads", I(32)}, {"num_key_value_heads", I(8)}, {"vocab_size", I(128256)}});
  const int64_t dv = vc.need("hidden_size"), Iv = vc.need("intermediate_size"), Lv = vc.need("num_hidden_layers"),
                Lg = vc.need("num_global_layers"), ch = vc.need("num_channels"), image = vc.need("image_size"),
                patch = vc.need("patch_size"), tiles = vc.need("max_num_tiles"), out = vc.need("vision_output_dim");
  if (patch <= 0 || image % patch != 0) refuse(vc.key("patch_size") + ": does not divide image_size");
  const Json& ratios = vc["supported_aspect_ratios"];
  const int64_t aspect_ids = (ratios.is_array() ? static_cast<int64_t>(ratios.size()) : 8) + 1;
  const int64_t patches = (image / patch) * (image / patch) + 1;
  const int64_t d = tc.need("hidden_size"), L = tc.need("num_hidden_layers"), V = tc.need("vocab_size"),
                heads = tc.need("num_attention_heads"), kv = tc.get("num_key_value_heads", heads),
                I = tc.need("intermediate_size");
  heads_divide(tc, d, heads);
  const int64_t hd = d / heads;
  const std::vector<int64_t> cross = tc.ints("cross_attention_layers", {3, 8, 13, 18, 23, 28, 33, 38});
  const std::set<int64_t> xl(cross.begin(), cross.end());
  for (auto l : xl)
    if (l < 0 || l >= L) refuse(tc.key("cross_attention_layers") + ": layer " + str(l) + " out of range");
  const Layout at = layout(ck, "vision_model.");
  Builder b = start("mllama", arch);
  auto vision_layers = [&](const std::string& p, int64_t n, bool gated) {
    for (int64_t l = 0; l < n; ++l) {
      const std::string q = p + str(l) + ".";
      if (gated) {
        b.weight(q + "gate_attn", {1});
        b.weight(q + "gate_ffn", {1});
      }
      for (const char* m : {"q_proj", "k_proj", "v_proj", "o_proj"})
        b.weight(q + "self_attn." + m + ".weight", {dv, dv});
      b.linear(q + "mlp.fc1", Iv, dv, true);
      b.linear(q + "mlp.fc2", dv, Iv, true);
      b.norm(q + "input_layernorm", dv, true);
      b.norm(q + "post_attention_layernorm", dv, true);
    }
  };
  b.nest(arch + " (tiled image encoder; cross-attention at " + str(static_cast<int64_t>(xl.size())) + " of " +
             str(L) + " text layers)",
         [&] {
           b.nest("Vision (up to " + str(tiles) + " tiles of " + str(image) + "px, " + str(Lv) + " local + " +
                      str(Lg) + " gated global layers, intermediate layers concatenated to " + str(out) + ")",
                  [&] {
                    const std::string p = at.vision;
                    b.weight(p + "class_embedding", {dv});
                    b.weight(p + "patch_embedding.weight", {dv, ch, patch, patch});
                    b.weight(p + "gated_positional_embedding.gate", {1});
                    b.weight(p + "gated_positional_embedding.embedding", {patches, dv});
                    b.weight(p + "gated_positional_embedding.tile_embedding.weight",
                             {aspect_ids, tiles * patches * dv});
                    for (const char* t : {"pre_tile_positional_embedding", "post_tile_positional_embedding"}) {
                      b.weight(p + t + ".gate", {1});
                      b.weight(p + t + ".embedding.weight", {aspect_ids, tiles * dv});
                    }
                    b.norm(p + "layernorm_pre", dv, true);
                    b.norm(p + "layernorm_post", dv, true);
                    vision_layers(p + "transformer.layers.", Lv, false);
                    vision_layers(p + "global_transformer.layers.", Lg, true);
                  });
           b.nest("Projector (linear " + str(out) + " to " + str(d) + ")",
                  [&] { b.linear(at.projector, d, out, true); });
           b.nest("Text decoder x " + str(L) + " (gated cross-attention with QK RMSNorm at layers " + joined(xl) +
                      ", self-attention elsewhere)",
                  [&] {
                    const std::string m = at.text;
                    b.weight(m + "embed_tokens.weight", {V + 8, d});  // 8 more rows for the image tokens
                    for (int64_t l = 0; l < L; ++l) {
                      const std::string p = m + "layers." + str(l) + ".";
                      b.weight(p + "input_layernorm.weight", {d});
                      if (xl.count(l)) {
                        b.weight(p + "cross_attn_attn_gate", {1});
                        b.weight(p + "cross_attn_mlp_gate", {1});
                        gqa(b, p + "cross_attn", d, heads, kv, hd, false);
                        b.weight(p + "cross_attn.q_norm.weight", {hd});
                        b.weight(p + "cross_attn.k_norm.weight", {hd});
                      } else {
                        gqa(b, p + "self_attn", d, heads, kv, hd, false);
                      }
                      b.weight(p + "post_attention_layernorm.weight", {d});
                      gated_mlp(b, p + "mlp", d, I);
                    }
                    b.weight(m + "norm.weight", {d});
                    b.head(at.head, {V, d}, tc.flag("tie_word_embeddings", false));
                  });
         });
  return b.c;
}

Composition qwen3_vl(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const Config vc = cfg.sub("vision_config",
                            {{"depth", I(27)}, {"hidden_size", I(1152)}, {"intermediate_size", I(4304)},
                             {"num_heads", I(16)}, {"in_channels", I(3)}, {"patch_size", I(16)},
                             {"temporal_patch_size", I(2)}, {"spatial_merge_size", I(2)},
                             {"out_hidden_size", I(3584)}, {"num_position_embeddings", I(2304)}});
  const Config tc = cfg.sub("text_config",
                            {{"hidden_size", I(4096)}, {"intermediate_size", I(22016)}, {"num_hidden_layers", I(32)},
                             {"num_attention_heads", I(32)}, {"num_key_value_heads", I(32)},
                             {"vocab_size", I(151936)}, {"head_dim", I(128)}});
  const int64_t dv = vc.need("hidden_size"), Iv = vc.need("intermediate_size"), depth = vc.need("depth"),
                ch = vc.need("in_channels"), patch = vc.need("patch_size"), tp = vc.need("temporal_patch_size"),
                merge = vc.need("spatial_merge_size"), out = vc.need("out_hidden_size"),
                pos = vc.need("num_position_embeddings"), vh = vc.need("num_heads");
  const std::vector<int64_t> deep = vc.ints("deepstack_visual_indexes", {8, 16, 24});
  for (auto l : deep)
    if (l < 0 || l >= depth) refuse(vc.key("deepstack_visual_indexes") + ": block " + str(l) + " out of range");
  if (tc.need("hidden_size") != out) refuse(vc.key("out_hidden_size") + ": differs from text_config.hidden_size");
  const int64_t merged = dv * merge * merge;
  const std::set<int64_t> deep_set(deep.begin(), deep.end());
  Builder b = start("qwen3_vl", arch);
  b.nest(arch + " (" + str(merge) + "x" + str(merge) + " patch merge; DeepStack features from vision blocks " +
             joined(deep_set) + " added to the first text layers)",
         [&] {
           b.nest("Vision x " + str(depth) + " (" + str(tp) + "x" + str(patch) + "x" + str(patch) +
                      " patches, learned positions " + str(pos) + " interpolated, 2-D RoPE, " + str(vh) + " heads)",
                  [&] {
                    const std::string p = "model.visual.";
                    b.weight(p + "patch_embed.proj.weight", {dv, ch, tp, patch, patch});
                    b.weight(p + "patch_embed.proj.bias", {dv});
                    b.weight(p + "pos_embed.weight", {pos, dv});
                    for (int64_t l = 0; l < depth; ++l) {
                      const std::string q = p + "blocks." + str(l) + ".";
                      b.norm(q + "norm1", dv, true);
                      b.norm(q + "norm2", dv, true);
                      b.linear(q + "attn.qkv", 3 * dv, dv, true);
                      b.linear(q + "attn.proj", dv, dv, true);
                      b.linear(q + "mlp.linear_fc1", Iv, dv, true);
                      b.linear(q + "mlp.linear_fc2", dv, Iv, true);
                    }
                    b.norm(p + "merger.norm", dv, true);
                    b.linear(p + "merger.linear_fc1", merged, merged, true);
                    b.linear(p + "merger.linear_fc2", out, merged, true);
                    for (size_t i = 0; i < deep.size(); ++i) {
                      const std::string q = p + "deepstack_merger_list." + str(static_cast<int64_t>(i)) + ".";
                      b.norm(q + "norm", merged, true);
                      b.linear(q + "linear_fc1", merged, merged, true);
                      b.linear(q + "linear_fc2", out, merged, true);
                    }
                  });
           text_decoder(b, tc, "qwen3_vl_text", "model.language_model.", "lm_head.weight",
                        cfg.flag("tie_word_embeddings", tc.flag("tie_word_embeddings", false)));
         });
  return b.c;
}

// ---- Diffusion: AutoencoderKL, DiT, FLUX, pipelines -----------------------------------------

void conv(Builder& b, const std::string& p, int64_t out, int64_t in, int64_t k) {
  b.weight(p + ".weight", {out, in, k, k});
  b.weight(p + ".bias", {out});
}

// A ResNet block of the autoencoder: GroupNorm, SiLU, 3x3 convolution, twice; a 1x1 shortcut
// when the width changes.
void resnet(Builder& b, const std::string& p, int64_t in, int64_t out) {
  b.norm(p + "norm1", in, true);
  conv(b, p + "conv1", out, in, 3);
  b.norm(p + "norm2", out, true);
  conv(b, p + "conv2", out, out, 3);
  if (in != out) conv(b, p + "conv_shortcut", out, in, 1);
}

// The autoencoder's middle block: a ResNet block, one-head self-attention over the spatial
// positions (GroupNorm, q/k/v and output projections), a ResNet block.
void vae_middle(Builder& b, const std::string& p, int64_t c, bool attention) {
  resnet(b, p + "resnets.0.", c, c);
  if (attention) {
    b.norm(p + "attentions.0.group_norm", c, true);
    for (const char* n : {"to_q", "to_k", "to_v"}) b.linear(p + "attentions.0." + n, c, c, true);
    b.linear(p + "attentions.0.to_out.0", c, c, true);
  }
  resnet(b, p + "resnets.1.", c, c);
}

// The KL autoencoder of latent diffusion (Stable Diffusion, FLUX): a convolutional encoder to the
// latent's mean and log-variance, a decoder back to pixels.
Composition autoencoder_kl(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const int64_t in = cfg.get("in_channels", 3), out = cfg.get("out_channels", 3), latent = cfg.get("latent_channels", 4),
                layers = cfg.get("layers_per_block", 1), groups = cfg.get("norm_num_groups", 32);
  const std::vector<int64_t> widths = cfg.ints("block_out_channels", {64});
  if (widths.empty()) refuse(cfg.key("block_out_channels") + ": at least one block");
  for (auto w : widths)
    if (w <= 0 || w % groups != 0) refuse(cfg.key("block_out_channels") + ": " + str(w) + " channels in groups of " + str(groups));
  auto types = [&](const char* key, const char* want) {
    const Json& v = cfg[key];
    if (v.is_null()) return;
    if (!v.is_array() || v.size() != widths.size()) refuse(cfg.key(key) + ": one a block");
    for (const auto& t : v.items())
      if (!t.is_string() || t.as_string() != want) refuse(cfg.key(key) + ": every block is " + std::string(want));
  };
  types("down_block_types", "DownEncoderBlock2D");
  types("up_block_types", "UpDecoderBlock2D");
  const bool quant = cfg.flag("use_quant_conv", true), post = cfg.flag("use_post_quant_conv", true),
             mid_attention = cfg.flag("mid_block_add_attention", true);
  const int64_t n = static_cast<int64_t>(widths.size()), top = widths.back();
  Builder b = start("autoencoder_kl", arch);
  std::string chans;
  for (auto w : widths) chans += (chans.empty() ? "" : ", ") + str(w);
  b.nest(arch + " (" + str(latent) + " latent channels, blocks of " + chans + ", " + str(layers) +
             " ResNet blocks each, GroupNorm " + str(groups) + ")",
         [&] {
           b.nest("Encoder (downsampling by " + str(int64_t{1} << (n - 1)) + "; mean and log-variance out)", [&] {
             conv(b, "encoder.conv_in", widths[0], in, 3);
             for (int64_t i = 0; i < n; ++i) {
               const std::string p = "encoder.down_blocks." + str(i) + ".";
               const int64_t from = i == 0 ? widths[0] : widths[i - 1];
               for (int64_t r = 0; r < layers; ++r) resnet(b, p + "resnets." + str(r) + ".", r == 0 ? from : widths[i], widths[i]);
               if (i + 1 < n) conv(b, p + "downsamplers.0.conv", widths[i], widths[i], 3);
             }
             vae_middle(b, "encoder.mid_block.", top, mid_attention);
             b.norm("encoder.conv_norm_out", top, true);
             conv(b, "encoder.conv_out", 2 * latent, top, 3);
             if (quant) conv(b, "quant_conv", 2 * latent, 2 * latent, 1);
           });
           b.nest("Decoder (upsampling, " + str(layers + 1) + " ResNet blocks a level)", [&] {
             if (post) conv(b, "post_quant_conv", latent, latent, 1);
             conv(b, "decoder.conv_in", top, latent, 3);
             vae_middle(b, "decoder.mid_block.", top, mid_attention);
             int64_t prev = top;
             for (int64_t i = 0; i < n; ++i) {
               const std::string p = "decoder.up_blocks." + str(i) + ".";
               const int64_t w = widths[n - 1 - i];
               for (int64_t r = 0; r <= layers; ++r) resnet(b, p + "resnets." + str(r) + ".", r == 0 ? prev : w, w);
               if (i + 1 < n) conv(b, p + "upsamplers.0.conv", w, w, 3);
               prev = w;
             }
             b.norm("decoder.conv_norm_out", widths[0], true);
             conv(b, "decoder.conv_out", out, widths[0], 3);
           });
         });
  return b.c;
}

// A timestep (or guidance) embedding: sinusoidal features of 256, linear, SiLU, linear.
void timestep_embedder(Builder& b, const std::string& p, int64_t d, int64_t in = 256) {
  b.linear(p + ".linear_1", d, in, true);
  b.linear(p + ".linear_2", d, d, true);
}

// DiT: patch embedding, transformer blocks modulated by the timestep and class (adaLN-Zero, each
// block with its own embedders), a modulated linear head to the patch's noise and variance.
Composition dit(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const std::string norm = cfg.text("norm_type", "ada_norm_zero");
  if (norm != "ada_norm_zero")
    refuse(cfg.key("norm_type") + ": " + norm + "; DiT modulates its norms by the timestep and class (ada_norm_zero)");
  const int64_t heads = cfg.get("num_attention_heads", 16), hd = cfg.get("attention_head_dim", 72),
                in = cfg.get("in_channels", 4), out = cfg.get("out_channels", in), L = cfg.get("num_layers", 28),
                patch = cfg.get("patch_size", 2), classes = cfg.get("num_embeds_ada_norm", 1000),
                sample = cfg.get("sample_size", 32);
  if (patch <= 0 || sample % patch != 0) refuse(cfg.key("patch_size") + ": does not divide sample_size");
  const int64_t d = heads * hd, ff = cfg.get("ff_inner_dim", 4 * d);
  Builder b = start("dit", arch);
  b.nest(arch + " x " + str(L) + " (" + str(sample) + "x" + str(sample) + " latents in patches of " + str(patch) + ", " +
             str(heads) + " heads of " + str(hd) + ", " + str(classes) + " classes and a null class)",
         [&] {
           conv(b, "pos_embed.proj", d, in, patch);
           b.ignore("pos_embed.pos_embed");
           b.leaf("Block: adaLN-Zero (timestep and class embedded, SiLU, linear to 6 modulations), "
                  "self-attention, tanh-GELU MLP " + str(ff));
           for (int64_t l = 0; l < L; ++l) {
             const std::string p = "transformer_blocks." + str(l) + ".";
             timestep_embedder(b, p + "norm1.emb.timestep_embedder", d);
             b.weight(p + "norm1.emb.class_embedder.embedding_table", {classes + 1, d});
             b.linear(p + "norm1.linear", 6 * d, d, true);
             for (const char* n : {"to_q", "to_k", "to_v"}) b.linear(p + "attn1." + n, d, d, true);
             b.linear(p + "attn1.to_out.0", d, d, true);
             b.linear(p + "ff.net.0.proj", ff, d, true);
             b.linear(p + "ff.net.2", d, ff, true);
           }
           b.nest("Head: modulated LayerNorm, linear to " + str(patch) + "x" + str(patch) + "x" + str(out), [&] {
             b.linear("proj_out_1", 2 * d, d, true);
             b.linear("proj_out_2", patch * patch * out, d, true);
           });
         });
  return b.c;
}

// FLUX.1's transformer: double-stream blocks (image and text rows with their own modulations,
// projections and MLPs, attending jointly with QK RMSNorm and 3-axis RoPE), then single-stream
// blocks over the joined rows (parallel attention and MLP), a modulated head.
Composition flux(const Json& j, const std::string& arch, const Checkpoint&) {
  const Config cfg(j, "");
  const int64_t heads = cfg.get("num_attention_heads", 24), hd = cfg.get("attention_head_dim", 128),
                in = cfg.get("in_channels", 64), out = cfg.get("out_channels", in), patch = cfg.get("patch_size", 1),
                L = cfg.get("num_layers", 19), Ls = cfg.get("num_single_layers", 38),
                joint = cfg.get("joint_attention_dim", 4096), pooled = cfg.get("pooled_projection_dim", 768);
  const bool guidance = cfg.flag("guidance_embeds", false);
  const std::vector<int64_t> axes = cfg.ints("axes_dims_rope", {16, 56, 56});
  int64_t rope = 0;
  for (auto a : axes) rope += a;
  if (rope != hd) refuse(cfg.key("axes_dims_rope") + ": the axes rotate " + str(rope) + " of a head's " + str(hd));
  const int64_t d = heads * hd, mlp = 4 * d;
  Builder b = start("flux", arch);
  b.nest(arch + " (" + str(L) + " double-stream + " + str(Ls) + " single-stream blocks, " + str(heads) + " heads of " +
             str(hd) + (guidance ? ", guidance embedded" : "") + ")",
         [&] {
           b.nest("Embeddings: image rows, text rows, timestep" + std::string(guidance ? " + guidance" : "") +
                      " + pooled text",
                  [&] {
                    b.linear("x_embedder", d, in * patch * patch, true);
                    b.linear("context_embedder", d, joint, true);
                    timestep_embedder(b, "time_text_embed.timestep_embedder", d);
                    if (guidance) timestep_embedder(b, "time_text_embed.guidance_embedder", d);
                    b.linear("time_text_embed.text_embedder.linear_1", d, pooled, true);
                    b.linear("time_text_embed.text_embedder.linear_2", d, d, true);
                  });
           b.leaf("Double-stream block: per stream adaLN-Zero (6 modulations), q/k/v with RMSNorm of q and k, "
                  "joint attention, output projection, tanh-GELU MLP " + str(mlp));
           for (int64_t l = 0; l < L; ++l) {
             const std::string p = "transformer_blocks." + str(l) + ".";
             b.linear(p + "norm1.linear", 6 * d, d, true);
             b.linear(p + "norm1_context.linear", 6 * d, d, true);
             for (const char* n : {"to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj"})
               b.linear(p + "attn." + n, d, d, true);
             for (const char* n : {"norm_q", "norm_k", "norm_added_q", "norm_added_k"}) b.weight(p + "attn." + n + ".weight", {hd});
             b.linear(p + "attn.to_out.0", d, d, true);
             b.linear(p + "attn.to_add_out", d, d, true);
             for (const char* s : {"ff", "ff_context"}) {
               b.linear(p + s + ".net.0.proj", mlp, d, true);
               b.linear(p + s + ".net.2", d, mlp, true);
             }
           }
           b.leaf("Single-stream block: adaLN-Zero (3 modulations), q/k/v with RMSNorm and a parallel MLP " +
                  str(mlp) + ", one output projection of both");
           for (int64_t l = 0; l < Ls; ++l) {
             const std::string p = "single_transformer_blocks." + str(l) + ".";
             b.linear(p + "norm.linear", 3 * d, d, true);
             for (const char* n : {"to_q", "to_k", "to_v"}) b.linear(p + "attn." + n, d, d, true);
             b.weight(p + "attn.norm_q.weight", {hd});
             b.weight(p + "attn.norm_k.weight", {hd});
             b.linear(p + "proj_mlp", mlp, d, true);
             b.linear(p + "proj_out", d, d + mlp, true);
           }
           b.nest("Head: modulated LayerNorm, linear to the patch's " + str(out * patch * patch) + " channels", [&] {
             b.linear("norm_out.linear", 2 * d, d, true);
             b.linear("proj_out", patch * patch * out, d, true);
           });
         });
  return b.c;
}

// The class a (component) config names: diffusers' `_class_name`, else its first architecture.
std::string class_of(const Json& cfg) {
  if (cfg["_class_name"].is_string()) return cfg["_class_name"].as_string();
  const Json& a = cfg["architectures"];
  if (a.is_array() && a.size() > 0 && a.at(0).is_string()) return a.at(0).as_string();
  return "";
}

using Maker = Composition (*)(const Json&, const std::string&, const Checkpoint&);
const std::map<std::string, Maker>& makers();

// A diffusers pipeline: each component folder with a config composes on its own, its tensors
// under the folder's name (the tokenizers and the scheduler hold no weights).
Composition pipeline(const Json& j, const std::string& arch, const Checkpoint& ck) {
  Builder b = start("pipeline", arch);
  b.nest(arch, [&] {
    for (const auto& [name, v] : j.members()) {
      if (!v.is_object()) continue;
      const std::string cls = class_of(v);
      if (cls.empty()) continue;
      const auto it = makers().find(cls);
      if (it == makers().end() || it->second == pipeline)
        refuse("config.json:" + name + ": " + cls + " has no catalog composition");
      const Composition c = it->second(v, cls, ck);
      b.module(name + ": " + c.family);
      for (const auto& line : c.tree) b.c.tree.push_back(std::string(2 * (b.depth + 1), ' ') + line);
      const std::string p = name + ".";
      for (const auto& w : c.weights) b.weight(p + w.name, w.shape);
      for (const auto& w : c.optional) b.optional(p + w.name, w.shape);
      for (const auto& n : c.ignored) b.ignore(p + n);
    }
  });
  return b.c;
}

// ---- Dispatch --------------------------------------------------------------------------------


const std::map<std::string, Maker>& makers() {
  static const std::map<std::string, Maker> m = {
      {"BertModel", bert},
      {"BertForMaskedLM", bert},
      {"BertForSequenceClassification", bert},
      {"BertForTokenClassification", bert},
      {"XLMRobertaModel", xlm_roberta},
      {"XLMRobertaForSequenceClassification", xlm_roberta},
      {"CLIPModel", clip},
      {"CLIPTextModel", clip},
      {"CLIPTextModelWithProjection", clip},
      {"CLIPVisionModel", clip},
      {"CLIPVisionModelWithProjection", clip},
      {"SiglipModel", clip},
      {"SiglipVisionModel", clip},
      {"T5ForConditionalGeneration", t5},
      {"MT5ForConditionalGeneration", t5},
      {"T5EncoderModel", t5},
      {"WhisperForConditionalGeneration", whisper},
      {"MambaForCausalLM", mamba},
      {"Mamba2ForCausalLM", mamba2},
      {"BambaForCausalLM", bamba},
      {"Gemma3ForCausalLM", gemma3_text},
      {"Gemma4ForCausalLM", gemma4_text},
      {"OlmoeForCausalLM", olmoe},
      {"DeepseekV2ForCausalLM", deepseek_v2},
      {"LlavaForConditionalGeneration", llava},
      {"MllamaForConditionalGeneration", mllama},
      {"Qwen3VLForConditionalGeneration", qwen3_vl},
      {"AutoencoderKL", autoencoder_kl},
      {"DiTTransformer2DModel", dit},
      {"Transformer2DModel", dit},
      {"FluxTransformer2DModel", flux},
      {"FluxPipeline", pipeline},
      {"DiTPipeline", pipeline},
  };
  return m;
}

bool is_ignored(const Composition& c, const std::string& name) {
  for (const auto& n : c.ignored) {
    if (n.empty()) continue;
    if (n.back() == '.' ? name.rfind(n, 0) == 0 : name == n) return true;
  }
  return false;
}

}  // namespace

bool composes(const std::string& architecture) { return makers().count(architecture) > 0; }

std::vector<std::string> architectures() {
  std::vector<std::string> out;
  for (const auto& entry : makers()) out.push_back(entry.first);
  return out;
}

Composition compose(const Checkpoint& ck) {
  const Json& cfg = ck.config();
  for (const auto& a : cfg["architectures"].items()) {
    if (!a.is_string()) continue;
    const auto it = makers().find(a.as_string());
    if (it != makers().end()) return it->second(cfg, a.as_string(), ck);
  }
  // Diffusers names a model's (or a pipeline's) class in `_class_name`.
  if (cfg["_class_name"].is_string()) {
    const auto it = makers().find(cfg["_class_name"].as_string());
    if (it != makers().end()) return it->second(cfg, cfg["_class_name"].as_string(), ck);
  }
  refuse("config.json:architectures: no catalog composition");
}

void check(const Composition& c, const Checkpoint& ck) {
  std::set<std::string> read;
  auto fits = [&](const Weight& w, const StoredTensor* t) {
    if (t->shape != w.shape) refuse(w.name + ": shape " + dims(t->shape) + ", the composition reads " + dims(w.shape));
    read.insert(w.name);
  };
  for (const auto& w : c.weights) {
    const StoredTensor* t = ck.get(w.name);
    if (t == nullptr) refuse(w.name + ": missing from the checkpoint (" + c.family + ")");
    fits(w, t);
  }
  for (const auto& w : c.optional)
    if (const StoredTensor* t = ck.get(w.name)) fits(w, t);
  for (const auto& n : ck.names())
    if (!read.count(n) && !is_ignored(c, n)) refuse(n + ": not read by the " + c.family + " composition");
}

}  // namespace foa::engine::catalog
