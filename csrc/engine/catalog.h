// Catalog compositions: families the registry lists but no kernels serve yet (encoders,
// encoder-decoders, contrastive and vision-language models, recurrent, hybrid and further decoder
// families). Each is a typed description built from config.json alone: the module tree and every
// weight it reads, by checkpoint name and shape, so a checkpoint (its values or only its
// safetensors headers) can be checked strictly against it without a device. The reference keeps
// such families as typed compositions too
// (crates/furiosa-opt-models/src/models/{encoder,encoder_decoder,vision_language,decoder/recurrent,
// decoder/hybrid,decoder/attention}); its registry, like this one, refuses to load them (no model
// type is implemented).
#pragma once

#include <string>
#include <vector>

#include "checkpoint.h"

namespace foa::engine::catalog {

struct Weight {
  std::string name;            // the checkpoint's tensor name
  std::vector<int64_t> shape;  // its logical shape
};

struct Composition {
  std::string family;        // "bert", "t5", "whisper", "clip", "mamba2", "llava", ...
  std::string architecture;  // the config's architecture it composes
  std::vector<std::string> tree;  // the module tree, one line a module (indented by depth)
  std::vector<Weight> weights;    // every weight, strict
  // Weights a checkpoint may hold or leave out: tied copies (a head or a stack's embedding that
  // shares another weight's values) and parts the model does not use. Held, they must have the shape.
  std::vector<Weight> optional;
  // Names a checkpoint may hold that nothing reads (exact, or a prefix when it ends in '.'):
  // buffers older exports saved, and heads of the pretraining objective.
  std::vector<std::string> ignored;
};

// Whether `architecture` has a catalog composition.
bool composes(const std::string& architecture);

// Every architecture with a catalog composition.
std::vector<std::string> architectures();

// The composition of the config's first listed catalog architecture. Refuses (ValueError) a
// config without one, or an inconsistent geometry, naming the config key.
Composition compose(const Checkpoint& ck);

// Checks `ck` against `c`: every weight present with its shape, every optional weight held with
// its shape, and no other tensor but the ignored names. Refuses (ValueError) with the first
// missing, misshaped or unread name.
void check(const Composition& c, const Checkpoint& ck);

}  // namespace foa::engine::catalog
