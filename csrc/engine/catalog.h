// Catalog compositions: families the registry lists but no kernels serve yet (encoders,
// encoder-decoders, recurrent and further decoder families). Each is a typed description built
// from config.json alone: the module tree and every weight it reads, by checkpoint name and shape,
// so a checkpoint (its values or only its safetensors headers) can be checked strictly against it
// without a device. The reference keeps such families as typed compositions too
// (crates/furiosa-opt-models/src/models/{encoder,encoder_decoder,decoder/recurrent,...}); its
// registry, like this one, refuses to load them (no model type is implemented).
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
  std::string family;        // "bert", "t5", "whisper", "mamba2", "gemma3_text"
  std::string architecture;  // the config's architecture it composes
  std::vector<std::string> tree;  // the module tree, one line a module (indented by depth)
  std::vector<Weight> weights;    // every weight, strict
  // Tied copies (a head or a stack's embedding that shares another weight's values): a checkpoint
  // may hold them or leave them out; held, they must have the shape.
  std::vector<Weight> aliases;
};

// Whether `architecture` has a catalog composition.
bool composes(const std::string& architecture);

// The composition of the config's first listed catalog architecture. Refuses (ValueError) a
// config without one, or a missing or inconsistent geometry key, naming the key.
Composition compose(const Checkpoint& ck);

// Checks `ck` against `c`: every weight present with its shape, every alias held with its shape,
// and no other tensor. Refuses (ValueError) with the first missing, misshaped or unread name.
void check(const Composition& c, const Checkpoint& ck);

}  // namespace foa::engine::catalog
