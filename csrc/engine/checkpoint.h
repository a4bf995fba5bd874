// Checkpoints: the tensors of a Hugging Face model (or diffusers pipeline) directory, mapped from
// their safetensors files or copied into host memory, and the model's config.
//
// Behaviour follows the reference loader (crates/furiosa-opt-models/src/load/checkpoint.rs):
// a model's folder holds the files `model.safetensors.index.json` names, else its `.safetensors`
// files, and `config.json`; a pipeline's folder holds `model_index.json` and a folder per
// component, whose tensors are named by the folder's dotted path; a tensor held by two files is
// refused; `read()` copies every tensor so later changes to the files do not reach it.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "json.h"
#include "runtime.h"

namespace foa::engine {

// Safetensors element types (the file format's names).
enum class StDType { BOOL, U8, I8, I16, U16, I32, U32, I64, U64, F16, BF16, F32, F64, F8_E4M3, F8_E5M2, F8_E8M0, F4 };
StDType st_dtype(const std::string& name);
const char* st_dtype_name(StDType d);
size_t st_dtype_bits(StDType d);

struct Mapping;  // a mapped file or a host copy

struct StoredTensor {
  StDType dtype;
  std::vector<int64_t> shape;
  std::shared_ptr<Mapping> bytes;  // null for a declared-only tensor
  size_t begin = 0, end = 0;
  std::string file;
  const uint8_t* data() const;
  size_t nbytes() const { return end - begin; }
  int64_t numel() const;
};

enum class Part { Whole, Encoder };

class Checkpoint {
 public:
  Checkpoint() = default;
  // Maps `directory`; `config` replaces the directory's config when given. `declared` reads the
  // files' headers only (no value can be read then).
  static Checkpoint open(const std::string& directory, const Json* config, bool declared = false);
  Checkpoint read() const;                       // every tensor copied into host memory
  Checkpoint encoder() const;                    // the media-encoder part of the checkpoint
  // Quantized at load ("tensor" or "channel"): refused for a checkpoint that declares its own.
  Checkpoint quantized(const std::string& granularity) const;

  const Json& config() const { return config_; }
  const std::map<std::string, StoredTensor>& tensors() const { return tensors_; }
  const StoredTensor* get(const std::string& name) const;
  std::vector<std::string> names() const;
  const std::string& directory() const { return directory_; }
  Part part() const { return part_; }
  const std::string& quantization() const { return quantization_; }  // "" when none
  // The config's quantization declaration, or null.
  const Json& declaration() const { return config_["quantization_config"]; }
  bool declared_only() const { return declared_; }

 private:
  Json config_;
  std::map<std::string, StoredTensor> tensors_;
  std::string directory_;
  std::string quantization_;
  Part part_ = Part::Whole;
  bool declared_ = false;
  void add_file(const std::string& path, const std::string& prefix, bool declared);
};

}  // namespace foa::engine
