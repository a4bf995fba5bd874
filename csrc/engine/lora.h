// LoRA adapters of a loaded decoder: a PEFT checkpoint's lora_A / lora_B factors on the device in
// the layout the projection GEMMs read as extra K segments (the reference's adapter slots,
// crates/furiosa-opt-engine/src/decoder/adapters.rs:21-102, crates/furiosa-opt-models/src/
// modules/lora.rs:1-12, 33, 349-402).
//
// Per layer and fused projection (q/k/v, o, gate/up, down) an adapter holds
//   A [kpad, in]  : each part's lora_A rows, each zero-padded to RANK rows (q, k, v: 3 x 32 rows,
//                   padded to 128; gate, up: 2 x 32; o, down: 32, padded to 64), this rank's
//                   input columns for the row-parallel o and down;
//   B [out, kpad] : each output row's lora_B row in its part's columns, scaled by
//                   lora_alpha / r (or / sqrt(r) with rsLoRA) and rounded once to BF16, this
//                   rank's output rows for the column-parallel projections.
// A call computes Z = X A^T per slot, zeroes the rows of other slots, and adds Z B^T into the
// projection's FP32 sums (one rounding with the base projection).
#pragma once

#include <array>
#include <memory>
#include <vector>

#include "checkpoint.h"
#include "model.h"
#include "runtime.h"

namespace foa::engine {

struct LoraFactor {
  HbmBuffer a, b;
  int kpad = 0;       // K columns of B and rows of A (a multiple of 64), 0: module not adapted
  int in = 0, out = 0;
};

class LoraAdapter {
 public:
  static constexpr int kRank = 32;
  static constexpr int kSlots = 2;
  // Modules of a layer in the order the decoder projects.
  enum Module { kQkv = 0, kO = 1, kGateUp = 2, kDown = 3 };

  LoraAdapter(const DecoderModel& model, const Checkpoint& ck);
  const DecoderModel* owner() const { return owner_; }
  const LoraFactor& factor(int layer, int module) const { return layers_[layer][module]; }

 private:
  const DecoderModel* owner_;
  std::vector<std::array<LoraFactor, 4>> layers_;
};

}  // namespace foa::engine
