#include "encoder.h"

#include <cmath>
#include <map>

#include "kernels/gemm.cuh"
#include "kernels/media.cuh"
#include "registry.h"
#include "trace.h"

namespace foa::engine {

namespace {

[[noreturn]] void invalid_data(const std::string& name, const std::string& reason) {
  throw ValueError(name + ": " + reason);
}
[[noreturn]] void refuse(const std::string& name, const std::string& reason) {
  throw Unsupported(name + ": " + reason);
}

int width(const Json& section, const char* key, const std::string& where) {
  const Json& v = section[key];
  if (!v.is_int() || v.as_int() <= 0) invalid_data("config.json:" + where + "." + key, "missing or not a positive integer");
  return static_cast<int>(v.as_int());
}

}  // namespace

EncoderConfig encoder_config(const Checkpoint& ck) {
  const Json& c = ck.config();
  if (!ck.quantization().empty() || !ck.declaration().is_null())
    refuse("quantization", "the media encoder's projections stay BF16");
  if (!c["model_type"].is_string() || c["model_type"].as_string() != "gemma4_unified")
    invalid_data("config.json:model_type", "the media encoder reads a gemma4_unified config");
  const Json& text = c["text_config"];
  const Json& vision = c["vision_config"];
  const Json& audio = c["audio_config"];
  if (!text.is_object() || !vision.is_object() || !audio.is_object())
    invalid_data("config.json", "the config declares no text, vision and audio sections");
  EncoderConfig e;
  e.text = width(text, "hidden_size", "text_config");
  e.embed = width(vision, "mm_embed_dim", "vision_config");
  e.positions = width(vision, "mm_posemb_size", "vision_config");
  const int patch = width(vision, "patch_size", "vision_config");
  const int pool = width(vision, "pooling_kernel_size", "vision_config");
  e.patch = 3 * (patch * pool) * (patch * pool);
  e.samples = width(audio, "audio_embed_dim", "audio_config");
  if (vision["rms_norm_eps"].is_number()) e.vision_eps = static_cast<float>(vision["rms_norm_eps"].as_double());
  if (audio["rms_norm_eps"].is_number()) e.audio_eps = static_cast<float>(audio["rms_norm_eps"].as_double());
  // The projections' inner dimensions run in 64-element k-blocks; the row kernels stage a row of
  // at most 12288 values.
  for (const auto& [name, v] : std::vector<std::pair<std::string, int>>{
           {"patch", e.patch}, {"mm_embed_dim", e.embed}, {"audio_embed_dim", e.samples}, {"hidden_size", e.text}})
    if (v % 64 != 0 || v > 12288)
      refuse("config.json", name + " " + std::to_string(v) + " is not a multiple of 64 up to 12288");
  const bool published = e.text == 3840 && e.embed == 3840 && e.positions == 1120 && e.patch == 6912 &&
                         e.samples == 640;
  e.size = published ? "12B" : "custom";
  return e;
}

MediaEncoder::MediaEncoder(const Device& device, EncoderConfig cfg) : device_(device), cfg_(std::move(cfg)) {}

void MediaEncoder::load(const Checkpoint& ck) {
  std::map<std::string, bool> used;
  for (const auto& n : ck.names())
    if (n.rfind("model.", 0) == 0 && n.rfind("model.language_model.", 0) != 0) used[n] = false;
  std::vector<std::string> missing;
  auto st = device_.state();
  auto take = [&](const std::string& name, std::vector<std::vector<int64_t>> shapes) -> const StoredTensor* {
    const StoredTensor* t = ck.get(name);
    if (t == nullptr) {
      missing.push_back(name);
      return nullptr;
    }
    bool ok = false;
    for (const auto& s : shapes) ok = ok || t->shape == s;
    if (!ok) {
      std::string s;
      for (auto x : t->shape) s += (s.empty() ? "" : ", ") + std::to_string(x);
      invalid_data(name, "shape [" + s + "] is not the model's");
    }
    used[name] = true;
    return t;
  };
  auto bf16 = [&](const std::string& name, std::vector<std::vector<int64_t>> shapes) {
    const StoredTensor* t = take(name, std::move(shapes));
    if (t == nullptr) return HbmBuffer();
    const std::vector<uint16_t> host = tensor_bf16(*t);
    HbmBuffer b(device_, host.size() * 2);
    st->check_cuda(cudaMemcpy(b.data(), host.data(), host.size() * 2, cudaMemcpyHostToDevice), "encoder weight upload");
    return b;
  };
  auto f32 = [&](const std::string& name, std::vector<std::vector<int64_t>> shapes) {
    const StoredTensor* t = take(name, std::move(shapes));
    if (t == nullptr) return HbmBuffer();
    const std::vector<float> host = tensor_f32(*t);
    HbmBuffer b(device_, host.size() * 4);
    st->check_cuda(cudaMemcpy(b.data(), host.data(), host.size() * 4, cudaMemcpyHostToDevice), "encoder weight upload");
    return b;
  };
  const std::string v = "model.vision_embedder.";
  const int64_t P = cfg_.patch, E = cfg_.embed, T = cfg_.text, S = cfg_.samples, N = cfg_.positions;
  ln1_w_ = bf16(v + "patch_ln1.weight", {{P}});
  ln1_b_ = bf16(v + "patch_ln1.bias", {{P}});
  dense_w_ = bf16(v + "patch_dense.weight", {{E, P}});
  dense_b_ = f32(v + "patch_dense.bias", {{E}});
  ln2_w_ = bf16(v + "patch_ln2.weight", {{E}});
  ln2_b_ = bf16(v + "patch_ln2.bias", {{E}});
  table_ = bf16(v + "pos_embedding", {{N, 2, E}, {2 * N, E}});
  pn_w_ = bf16(v + "pos_norm.weight", {{E}});
  pn_b_ = bf16(v + "pos_norm.bias", {{E}});
  vision_proj_ = bf16("model.embed_vision.embedding_projection.weight", {{T, E}});
  audio_proj_ = bf16("model.embed_audio.embedding_projection.weight", {{T, S}});
  if (!missing.empty()) {
    std::string s;
    for (size_t i = 0; i < missing.size() && i < 8; ++i) s += (i ? ", " : "") + missing[i];
    invalid_data("checkpoint", "missing tensors: " + s);
  }
  std::vector<std::string> extra;
  for (const auto& [n, u] : used)
    if (!u) extra.push_back(n);
  if (!extra.empty()) {
    std::string s;
    for (size_t i = 0; i < extra.size() && i < 8; ++i) s += (i ? ", " : "") + extra[i];
    if (extra.size() > 8) s += ", ... (" + std::to_string(extra.size()) + " in all)";
    invalid_data("checkpoint", "unexpected tensors: " + s);
  }
}

std::vector<std::vector<size_t>> MediaEncoder::launches(const std::vector<int64_t>& rows) {
  std::vector<std::vector<size_t>> out;
  int64_t filled = 0;
  for (size_t i = 0; i < rows.size(); ++i) {
    if (rows[i] > kLaunchRows)
      throw Unsupported("item " + std::to_string(i) + " holds " + std::to_string(rows[i]) +
                        " rows; a launch takes at most " + std::to_string(kLaunchRows));
    if (!out.empty() && filled + rows[i] <= kLaunchRows) {
      filled += rows[i];
      out.back().push_back(i);
    } else {
      out.push_back({i});
      filled = rows[i];
    }
  }
  return out;
}

namespace {

// C = A . W^T on the tcgen05 GEMM (BF16 operands; FP32 or BF16 output).
void project(DeviceState& st, const void* a, int M, int K, const void* w, int N, void* c, int epi) {
  foa::GemmArgs g;
  g.a = a;
  g.lda = K;
  g.w = w;
  g.ldw = K;
  g.M = M;
  g.N = N;
  g.K = K;
  g.c = c;
  g.ldc = N;
  g.epilogue = epi;
  g.status = st.status;
  if (foa::gemm_bf16(g, st.stream) != 0) st.fail("media encoder projection launch failed");
}

void rows_of(const HbmBuffer& b, int64_t count, int width, const std::string& what) {
  if (static_cast<int64_t>(b.size()) != count * width * 2)
    throw ValueError(std::to_string(b.size()) + " bytes do not hold " + std::to_string(count) + " rows of " +
                     std::to_string(width) + " BF16 values" + what);
}

}  // namespace

std::vector<HbmTensor> MediaEncoder::vision(const std::vector<ImageInput>& images) {
  TraceScope span("encoder.vision", "call");
  for (const auto& im : images) {
    rows_of(im.patches, static_cast<int64_t>(im.positions.size()), cfg_.patch, "");
    for (const auto& xy : im.positions) {
      if (xy[0] < 0 || xy[1] < 0)
        throw ValueError("a patch position is negative: pass the image's valid patches only");
      if (xy[0] >= cfg_.positions || xy[1] >= cfg_.positions)
        throw ValueError("a patch position reaches past the " + std::to_string(cfg_.positions) + " positions");
    }
  }
  std::vector<int64_t> counts;
  for (const auto& im : images) counts.push_back(static_cast<int64_t>(im.positions.size()));
  auto st = device_.state();
  st->check();
  st->activate();
  cudaStream_t s = st->stream;
  std::vector<HbmTensor> out;
  for (const auto& items : launches(counts)) {
    int64_t R = 0;
    for (size_t i : items) R += counts[i];
    if (R == 0) {
      for (size_t i : items) out.push_back(HbmTensor(HbmBuffer(device_, 0), {0, cfg_.text}, DType::BF16));
      continue;
    }
    const int rows = static_cast<int>(R);
    HbmBuffer inputs(device_, R * cfg_.patch * 2);
    std::vector<int32_t> xy;
    int64_t at = 0;
    for (size_t i : items) {
      const auto& im = images[i];
      if (counts[i] > 0)
        st->check_cuda(cudaMemcpyAsync(static_cast<char*>(inputs.data()) + at * cfg_.patch * 2, im.patches.data(),
                                       counts[i] * cfg_.patch * 2, cudaMemcpyDeviceToDevice, s),
                       "patch copy");
      for (const auto& p : im.positions) {
        xy.push_back(p[0]);
        xy.push_back(p[1]);
      }
      at += counts[i];
    }
    HbmBuffer positions(device_, xy.size() * 4);
    st->check_cuda(cudaMemcpyAsync(positions.data(), xy.data(), xy.size() * 4, cudaMemcpyHostToDevice, s),
                   "patch positions");
    HbmBuffer x1(device_, R * cfg_.patch * 2), acc(device_, R * cfg_.embed * 4), u(device_, R * cfg_.embed * 2);
    HbmBuffer rows_out(device_, R * cfg_.text * 2);
    auto bf = [](const HbmBuffer& b) { return static_cast<__nv_bfloat16*>(b.data()); };
    if (foa::media_layernorm(bf(inputs), cfg_.patch, bf(ln1_w_), bf(ln1_b_), cfg_.ln_eps, bf(x1), cfg_.patch, rows,
                             cfg_.patch, s) != 0)
      st->fail("patch norm launch failed");
    project(*st, x1.data(), rows, cfg_.patch, dense_w_.data(), cfg_.embed, acc.data(), foa::kEpiF32);
    if (foa::media_vision_tail(static_cast<const float*>(acc.data()), cfg_.embed,
                               static_cast<const float*>(dense_b_.data()), bf(ln2_w_), bf(ln2_b_), bf(table_),
                               static_cast<const int32_t*>(positions.data()), bf(pn_w_), bf(pn_b_), cfg_.ln_eps,
                               cfg_.vision_eps, bf(u), cfg_.embed, rows, cfg_.embed, s) != 0)
      st->fail("patch embedding launch failed");
    project(*st, u.data(), rows, cfg_.embed, vision_proj_.data(), cfg_.text, rows_out.data(), foa::kEpiBf16);
    const HbmTensor all(rows_out, {R, cfg_.text}, DType::BF16);
    at = 0;
    for (size_t i : items) {
      out.push_back(all.rows(at, at + counts[i]));
      at += counts[i];
    }
    // The host positions were copied from pageable memory: the copy is done once the call returns.
  }
  return out;
}

std::vector<HbmTensor> MediaEncoder::audio(const std::vector<AudioInput>& clips) {
  TraceScope span("encoder.audio", "call");
  std::vector<int64_t> counts;
  for (const auto& c : clips) {
    rows_of(c.frames, c.count, cfg_.samples, "");
    counts.push_back(c.count);
  }
  auto st = device_.state();
  st->check();
  st->activate();
  cudaStream_t s = st->stream;
  std::vector<HbmTensor> out;
  for (const auto& items : launches(counts)) {
    int64_t R = 0;
    for (size_t i : items) R += counts[i];
    if (R == 0) {
      for (size_t i : items) out.push_back(HbmTensor(HbmBuffer(device_, 0), {0, cfg_.text}, DType::BF16));
      continue;
    }
    const int rows = static_cast<int>(R);
    HbmBuffer inputs(device_, R * cfg_.samples * 2), normed(device_, R * cfg_.samples * 2);
    int64_t at = 0;
    for (size_t i : items) {
      if (counts[i] > 0)
        st->check_cuda(cudaMemcpyAsync(static_cast<char*>(inputs.data()) + at * cfg_.samples * 2,
                                       clips[i].frames.data(), counts[i] * cfg_.samples * 2,
                                       cudaMemcpyDeviceToDevice, s),
                       "frame copy");
      at += counts[i];
    }
    if (foa::media_unit_rmsnorm(static_cast<const __nv_bfloat16*>(inputs.data()), cfg_.samples, cfg_.audio_eps,
                                static_cast<__nv_bfloat16*>(normed.data()), cfg_.samples, rows, cfg_.samples,
                                s) != 0)
      st->fail("frame norm launch failed");
    HbmBuffer rows_out(device_, R * cfg_.text * 2);
    project(*st, normed.data(), rows, cfg_.samples, audio_proj_.data(), cfg_.text, rows_out.data(), foa::kEpiBf16);
    const HbmTensor all(rows_out, {R, cfg_.text}, DType::BF16);
    at = 0;
    for (size_t i : items) {
      out.push_back(all.rows(at, at + counts[i]));
      at += counts[i];
    }
  }
  return out;
}

}  // namespace foa::engine
