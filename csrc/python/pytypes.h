// Objects the Python binding hands out, shared by its translation units.
#pragma once

#include <memory>
#include <string>

#include "engine/model.h"

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
