// The registry: every upstream architecture name once, with the implementations that serve it on
// Blackwell, or none when the name is refused; and the load options checked against it before
// any weight is read.
//
// Reference: crates/furiosa-opt-engine/src/registry.rs (ARCHITECTURES :28, Implementation::listed
// :967, choose :985-1014) and load.rs (LoadOptions :35-262). The same lookup rules hold: the
// options' architecture, else the first of the config's `architectures` then `_class_name` the
// registry lists; an unknown name is invalid data, a listed name without implementations is
// unsupported; the one implementation whose scope serves the checkpoint is chosen.
#pragma once

#include <functional>
#include <optional>
#include <string>
#include <vector>

#include "checkpoint.h"
#include "model.h"

namespace foa::engine {

// A load refusal: the Python class is ValueError for invalid data, NotImplementedError for an
// unsupported choice; the message is "<name>: <reason>".
struct LoadRefusal {
  bool unsupported = false;
  std::string name, reason;
  [[noreturn]] void raise() const;
};

// A checkpoint tensor's values (BF16, F16 or F32 in the file) as BF16 bits, or as FP32.
std::vector<uint16_t> tensor_bf16(const StoredTensor& t);
std::vector<float> tensor_f32(const StoredTensor& t);

struct Implementation {
  std::string family;      // qwen3 | llama | mistral | qwen3_moe
  std::string cls;         // Python class path, e.g. "qwen3.ForCausalLM"
  std::string form;        // bf16 | fp8_block | nvfp4
  Output output = Output::Tokens;
  int adapters = 0;
  // The model config this implementation serves `checkpoint` as, or a refusal (from the config
  // and names alone).
  std::function<ModelConfig(const Checkpoint&)> scope;
};

struct Listed {
  std::string name;
  std::vector<const Implementation*> implementations;
};

// Every registry name (670), in registry order.
const std::vector<std::string>& architecture_names();
// The first of `names` the registry lists, with its implementations; throws the reference's
// refusals (unknown: invalid data; no implementation: unsupported).
Listed listed(const std::vector<std::string>& names);
// The one implementation of `l` whose scope serves `c`.
const Implementation* choose(const Listed& l, const Checkpoint& c, ModelConfig* config);

struct LoadOptions {
  std::optional<int> chips;
  std::optional<std::string> kv_cache;
  std::optional<std::string> architecture;
  std::optional<std::pair<int64_t, int64_t>> layers;
  bool batch_invariant = false;
  std::optional<std::string> quantization;  // fp8_per_tensor | fp8_per_channel
  bool encoder = false;
  bool adapters = false;
};

struct Selection {
  std::string architecture;
  const Implementation* implementation = nullptr;
  ModelConfig config;
  int chips = 1;
};

// The implementation `checkpoint` loads as with `options`, from its config and names alone.
Selection select(const LoadOptions& options, const Checkpoint& checkpoint);

// Copies the checkpoint's tensors strictly (every name read once, none missing) into the model's
// weight slots, this rank's shard of each.
void load_weights(DecoderModel& model, const Checkpoint& checkpoint);

}  // namespace foa::engine
