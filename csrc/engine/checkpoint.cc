#include "checkpoint.h"

#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <fstream>
#include <sstream>

namespace foa::engine {

// ------------------------------------------------------------------------------------ dtypes
namespace {
struct StInfo {
  StDType d;
  const char* name;
  size_t bits;
};
constexpr StInfo kSt[] = {
    {StDType::BOOL, "BOOL", 8},  {StDType::U8, "U8", 8},       {StDType::I8, "I8", 8},
    {StDType::I16, "I16", 16},   {StDType::U16, "U16", 16},    {StDType::I32, "I32", 32},
    {StDType::U32, "U32", 32},   {StDType::I64, "I64", 64},    {StDType::U64, "U64", 64},
    {StDType::F16, "F16", 16},   {StDType::BF16, "BF16", 16},  {StDType::F32, "F32", 32},
    {StDType::F64, "F64", 64},   {StDType::F8_E4M3, "F8_E4M3", 8}, {StDType::F8_E5M2, "F8_E5M2", 8},
    {StDType::F8_E8M0, "F8_E8M0", 8}, {StDType::F4, "F4", 4},
};
}  // namespace

StDType st_dtype(const std::string& name) {
  for (const auto& i : kSt)
    if (name == i.name) return i.d;
  throw ValueError("unknown safetensors dtype " + name);
}
const char* st_dtype_name(StDType d) { return kSt[static_cast<int>(d)].name; }
size_t st_dtype_bits(StDType d) { return kSt[static_cast<int>(d)].bits; }

// ------------------------------------------------------------------------------------ mapping
struct Mapping {
  const uint8_t* ptr = nullptr;
  size_t size = 0;
  bool mapped = false;
  std::vector<uint8_t> owned;
  ~Mapping() {
    if (mapped && ptr) munmap(const_cast<uint8_t*>(ptr), size);
  }
};

const uint8_t* StoredTensor::data() const {
  if (!bytes) throw ValueError("the checkpoint declares this tensor without values");
  return bytes->ptr + begin;
}

int64_t StoredTensor::numel() const {
  int64_t n = 1;
  for (auto s : shape) n *= s;
  return n;
}

namespace {
bool exists(const std::string& p) {
  struct stat s;
  return ::stat(p.c_str(), &s) == 0;
}
bool is_dir(const std::string& p) {
  struct stat s;
  return ::stat(p.c_str(), &s) == 0 && S_ISDIR(s.st_mode);
}
std::string slurp(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw IoError(path + ": " + std::strerror(errno));
  std::stringstream ss;
  ss << f.rdbuf();
  return ss.str();
}
std::vector<std::string> list(const std::string& dir) {
  std::vector<std::string> out;
  DIR* d = ::opendir(dir.c_str());
  if (!d) return out;
  while (dirent* e = ::readdir(d)) {
    const std::string n = e->d_name;
    if (n != "." && n != "..") out.push_back(n);
  }
  ::closedir(d);
  std::sort(out.begin(), out.end());
  return out;
}
bool ends_with(const std::string& s, const std::string& suffix) {
  return s.size() >= suffix.size() && s.compare(s.size() - suffix.size(), suffix.size(), suffix) == 0;
}
}  // namespace

void Checkpoint::add_file(const std::string& path, const std::string& prefix, bool declared) {
  auto m = std::make_shared<Mapping>();
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw IoError(path + ": " + std::strerror(errno));
  struct stat s;
  ::fstat(fd, &s);
  const size_t size = static_cast<size_t>(s.st_size);
  if (size < 8) {
    ::close(fd);
    throw ValueError(path + ": not a safetensors file");
  }
  uint64_t header_len = 0;
  if (::pread(fd, &header_len, 8, 0) != 8) {
    ::close(fd);
    throw IoError(path + ": cannot read the header");
  }
  if (header_len > size - 8 && !declared) {
    ::close(fd);
    throw ValueError(path + ": the header runs past the file");
  }
  std::string header(header_len, '\0');
  if (::pread(fd, header.data(), header_len, 8) != static_cast<ssize_t>(header_len)) {
    ::close(fd);
    throw IoError(path + ": cannot read the header");
  }
  if (!declared) {
    void* p = ::mmap(nullptr, size, PROT_READ, MAP_SHARED, fd, 0);
    if (p == MAP_FAILED) {
      ::close(fd);
      throw IoError(path + ": " + std::strerror(errno));
    }
    m->ptr = static_cast<const uint8_t*>(p);
    m->size = size;
    m->mapped = true;
  }
  ::close(fd);
  const Json h = Json::parse(header);
  if (!h.is_object()) throw ValueError(path + ": the header is not an object");
  const size_t base = 8 + header_len;
  for (const auto& [name, info] : h.members()) {
    if (name == "__metadata__") continue;
    StoredTensor t;
    t.dtype = st_dtype(info["dtype"].as_string());
    for (const auto& d : info["shape"].items()) t.shape.push_back(d.as_int());
    const auto& off = info["data_offsets"];
    if (!off.is_array() || off.size() != 2) throw ValueError(path + ": " + name + " has no data offsets");
    t.begin = base + static_cast<size_t>(off.at(0).as_int());
    t.end = base + static_cast<size_t>(off.at(1).as_int());
    const size_t expect = (static_cast<size_t>(t.numel()) * st_dtype_bits(t.dtype) + 7) / 8;
    if (t.end < t.begin || t.end - t.begin != expect)
      throw ValueError(path + ": " + name + " spans other than its shape's bytes");
    if (!declared && t.end > size) throw ValueError(path + ": " + name + " runs past the file");
    t.bytes = declared ? nullptr : m;
    t.file = path;
    const std::string full = prefix + name;
    auto it = tensors_.find(full);
    if (it != tensors_.end())
      throw ValueError(full + ": held by two files, " + it->second.file + " and " + path);
    tensors_.emplace(full, std::move(t));
  }
}

Checkpoint Checkpoint::open(const std::string& directory, const Json* config, bool declared) {
  Checkpoint c;
  c.directory_ = directory;
  c.declared_ = declared;
  const std::string pipeline = directory + "/model_index.json";
  if (exists(pipeline)) {
    // A pipeline: model_index.json, and each component folder's files and config at its path.
    Json index = Json::parse(slurp(pipeline));
    std::vector<std::pair<std::string, std::string>> stack = {{directory, ""}};
    while (!stack.empty()) {
      auto [dir, rel] = stack.back();
      stack.pop_back();
      for (const auto& n : list(dir)) {
        const std::string path = dir + "/" + n;
        if (is_dir(path)) {
          stack.push_back({path, rel.empty() ? n : rel + "." + n});
          continue;
        }
        if (rel.empty()) continue;
        if (n == "config.json") index.set(rel, Json::parse(slurp(path)));
        if (ends_with(n, ".safetensors")) c.add_file(path, rel + ".", declared);
      }
    }
    c.config_ = config ? *config : index;
    return c;
  }
  if (!is_dir(directory)) throw IoError(directory + ": no such checkpoint directory");
  const std::string index = directory + "/model.safetensors.index.json";
  if (exists(index)) {
    const Json idx = Json::parse(slurp(index));
    std::vector<std::string> files;
    for (const auto& [name, file] : idx["weight_map"].members())
      if (std::find(files.begin(), files.end(), file.as_string()) == files.end())
        files.push_back(file.as_string());
    std::sort(files.begin(), files.end());
    for (const auto& f : files) c.add_file(directory + "/" + f, "", declared);
  } else {
    for (const auto& n : list(directory))
      if (ends_with(n, ".safetensors")) c.add_file(directory + "/" + n, "", declared);
  }
  if (config) {
    c.config_ = *config;
  } else if (exists(directory + "/config.json")) {
    c.config_ = Json::parse(slurp(directory + "/config.json"));
  } else if (exists(directory + "/adapter_config.json")) {
    c.config_ = Json::parse(slurp(directory + "/adapter_config.json"));
  } else {
    c.config_ = Json::object({});
  }
  return c;
}

Checkpoint Checkpoint::read() const {
  Checkpoint c = *this;
  for (auto& [name, t] : c.tensors_) {
    if (!t.bytes) continue;
    auto m = std::make_shared<Mapping>();
    m->owned.assign(t.data(), t.data() + t.nbytes());
    m->ptr = m->owned.data();
    m->size = m->owned.size();
    t.bytes = m;
    t.begin = 0;
    t.end = m->size;
  }
  return c;
}

Checkpoint Checkpoint::encoder() const {
  Checkpoint c = *this;
  c.part_ = Part::Encoder;
  return c;
}

Checkpoint Checkpoint::quantized(const std::string& granularity) const {
  if (!declaration().is_null())
    throw ValueError(
        "config.json:quantization_config: the checkpoint is quantized already, so it loads its own "
        "weights");
  Checkpoint c = *this;
  c.quantization_ = granularity;
  return c;
}

const StoredTensor* Checkpoint::get(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

std::vector<std::string> Checkpoint::names() const {
  std::vector<std::string> out;
  for (const auto& [n, t] : tensors_) out.push_back(n);
  return out;
}

}  // namespace foa::engine
