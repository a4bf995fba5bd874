// Objects the Python binding hands out, shared by its translation units.
#pragma once

#include <memory>
#include <string>

#include "engine/encoder.h"
#include "engine/lora.h"
#include "engine/model.h"

// Hands the engine's queued log records to Python's `logging` (logger "furiosa_opt_engine"); the
// GIL is held. `LogsOnExit` does it when a binding call returns or raises: declare it first in the
// call's body, so that it runs after any `gil_scoped_release` in the body has ended.
void emit_logs();
struct LogsOnExit {
  ~LogsOnExit();
};

// A loaded decoder: the model, and its load's descriptive fields.
struct PyDecoder {
  std::shared_ptr<foa::engine::DecoderModel> model;
  std::string size, precision, kv_cache = "bfloat16";
  int parallel = 1;
  bool batch_invariant = false;
};
struct PyQwen3ForCausalLM : PyDecoder {};
struct PyQwen3ForSequenceClassification : PyDecoder {};
struct PyQwen3Model : PyDecoder {};
struct PyLlamaForCausalLM : PyDecoder {};
struct PyMistralForCausalLM : PyDecoder {};
struct PyQwen3MoeForCausalLM : PyDecoder {};
struct PyMixtralForCausalLM : PyDecoder {};
// A media encoder (a load of a vision-language model's encoder alone).
struct PyEncoder {
  std::shared_ptr<foa::engine::MediaEncoder> encoder;
};

// The LoRA adapters a decoder's calls run with, and one loaded adapter.
struct PyAdapterSpec {
  std::shared_ptr<foa::engine::DecoderModel> model;
};
struct PyAdapter {
  std::shared_ptr<const foa::engine::LoraAdapter> adapter;
  std::shared_ptr<foa::engine::DecoderModel> model;  // keeps the decoder alive
};
