#include "runtime.h"

#include <cstdio>

#include "trace.h"

#include <cstdlib>

#include <algorithm>
#include <cstring>

namespace foa::engine {

// ------------------------------------------------------------------------------------ dtypes
namespace {
struct DTypeInfo {
  DType d;
  const char* name;
  size_t size;
};
constexpr DTypeInfo kDTypes[] = {
    {DType::Bool, "bool", 1},           {DType::U8, "uint8", 1},
    {DType::I8, "int8", 1},             {DType::I16, "int16", 2},
    {DType::I32, "int32", 4},           {DType::I64, "int64", 8},
    {DType::F16, "float16", 2},         {DType::BF16, "bfloat16", 2},
    {DType::F32, "float32", 4},         {DType::F64, "float64", 8},
    {DType::F8E4M3, "float8_e4m3fn", 1}, {DType::F8E5M2, "float8_e5m2", 1},
};
}  // namespace

DType dtype_from_name(const std::string& name) {
  for (const auto& i : kDTypes)
    if (name == i.name) return i.d;
  throw ValueError("unknown dtype: " + name);
}
const char* dtype_name(DType d) { return kDTypes[static_cast<int>(d)].name; }
size_t dtype_size(DType d) { return kDTypes[static_cast<int>(d)].size; }

// ------------------------------------------------------------------------------------ device
namespace {
size_t size_class(size_t bytes) {
  if (bytes <= (1u << 20)) return (bytes + 511) / 512 * 512;
  return (bytes + (2u << 20) - 1) / (2u << 20) * (2u << 20);
}
}  // namespace

void* DeviceState::allocate(size_t bytes, size_t* rounded) {
  const size_t r = size_class(std::max<size_t>(bytes, 1));
  *rounded = r;
  {
    std::lock_guard<std::mutex> g(pool_mu);
    auto it = pool.find(r);
    if (it != pool.end() && !it->second.empty()) {
      void* p = it->second.back();
      it->second.pop_back();
      pooled_bytes -= r;
      return p;
    }
  }
  activate();
  void* p = nullptr;
  if (cudaMalloc(&p, r) != cudaSuccess) {
    cudaGetLastError();
    // Give the cached blocks back to the driver and retry once.
    std::lock_guard<std::mutex> g(pool_mu);
    cudaStreamSynchronize(stream);
    for (auto& [sz, v] : pool)
      for (void* q : v) cudaFree(q);
    pool.clear();
    pooled_bytes = 0;
    if (cudaMalloc(&p, r) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
  }
  return p;
}

void DeviceState::release(void* ptr, size_t rounded) {
  std::lock_guard<std::mutex> g(pool_mu);
  pool[rounded].push_back(ptr);
  pooled_bytes += rounded;
}

size_t DeviceState::trim() {
  activate();
  cudaStreamSynchronize(stream);
  std::lock_guard<std::mutex> g(pool_mu);
  size_t freed = 0;
  for (auto& [sz, v] : pool) {
    for (void* q : v) cudaFree(q);
    freed += sz * v.size();
  }
  pool.clear();
  pooled_bytes = 0;
  return freed;
}

DeviceState::~DeviceState() {
  if (ordinal >= 0) {
    cudaSetDevice(ordinal);
    cudaStreamSynchronize(stream);
    for (auto& [sz, v] : pool)
      for (void* q : v) cudaFree(q);
    if (status) cudaFree(status);
    if (stream) cudaStreamDestroy(stream);
  }
}

void DeviceState::check() const {
  if (!poison.empty()) throw DeviceError("the device failed earlier: " + poison);
}

void DeviceState::fail(const std::string& what) {
  if (poison.empty()) log_event(LogLevel::Error, "GPU " + std::to_string(ordinal) + " failed: " + what);
  if (poison.empty()) poison = what;
  throw DeviceError(what);
}

void DeviceState::check_cuda(cudaError_t err, const char* what) {
  if (err != cudaSuccess) fail(std::string(what) + ": " + cudaGetErrorString(err));
}

void DeviceState::check_status() {
  int code = 0;
  check_cuda(cudaMemcpyAsync(&code, status, sizeof(int), cudaMemcpyDeviceToHost, stream),
             "status read");
  check_cuda(cudaStreamSynchronize(stream), "status wait");
  raise_status(code);
}

void DeviceState::raise_status(int code) {
  if (code == 0) return;
  static const char* what[] = {"",
                               "a TMA stage never landed",
                               "a pipeline stage was never released",
                               "an accumulator was never completed",
                               "an accumulator was never released",
                               "a peer rank never raised its flag",
                               "copies in flight did not land while aborting",
                               "a launch argument failed a device-side check",
                               "an index read from device memory (a block ID or cache slot) was out of range"};
  const std::string reason = code > 0 && code < 9 ? what[code] : "unknown";
  cudaMemsetAsync(status, 0, sizeof(int), stream);
  fail(std::string(code >= 7 && code <= 8 ? "a kernel refused its input: " : "a kernel gave up a bounded wait: ") +
       reason + " (status " + std::to_string(code) + ")");
}

bool DeviceState::injected(const char* kind) {
  if (fault_countdown < 0 || fault_kind != kind) return false;
  if (fault_countdown-- > 0) return false;
  fault_kind.clear();
  return true;
}

void DeviceState::activate() const { cudaSetDevice(ordinal); }

Device::Device(std::vector<int> chips, int pes_begin, int pes_end, int rank) {
  if (chips.empty()) throw ValueError("a placement holds at least one chip");
  if (rank < 0 || rank >= static_cast<int>(chips.size()))
    throw ValueError("the process rank is outside the placement's chips");
  state_ = std::make_shared<DeviceState>();
  state_->chips = chips;
  state_->pes_begin = pes_begin;
  state_->pes_end = pes_end;
  state_->rank = rank;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    state_->ordinal = -1;
    throw DeviceError("no CUDA device is visible");
  }
  // With one GPU visible per process (CUDA_VISIBLE_DEVICES narrowed by the launcher) the chip is
  // ordinal 0; otherwise it is the placement's chip ordinal.
  const int chip = chips[rank];
  state_->ordinal = chip < count ? chip : (count == 1 ? 0 : -1);
  if (state_->ordinal < 0) throw DeviceError("chip " + std::to_string(chip) + " is not visible");
  state_->check_cuda(cudaSetDevice(state_->ordinal), "open device");
  state_->check_cuda(cudaStreamCreateWithFlags(&state_->stream, cudaStreamNonBlocking), "stream");
  state_->check_cuda(cudaMalloc(&state_->status, 64), "status word");
  state_->check_cuda(cudaMemset(state_->status, 0, 64), "status word");
  {
    cudaDeviceProp prop{};
    size_t free_b = 0, total = 0;
    if (cudaGetDeviceProperties(&prop, state_->ordinal) == cudaSuccess && cudaMemGetInfo(&free_b, &total) == cudaSuccess) {
      char line[256];
      std::snprintf(line, sizeof(line), "GPU %d (%s, %d SMs): %.1f of %.1f GiB free; rank %d of %zu", state_->ordinal,
                    prop.name, prop.multiProcessorCount, free_b / 1073741824.0, total / 1073741824.0, rank,
                    chips.size());
      log_event(LogLevel::Info, line);
    }
    cudaGetLastError();
  }
  if (const char* f = std::getenv("FOA_FAULT")) {
    // <kind>:<countdown>, e.g. "launch:10": the eleventh kernel launch fails.
    const std::string spec(f);
    const size_t colon = spec.find(':');
    state_->fault_kind = spec.substr(0, colon);
    state_->fault_countdown = colon == std::string::npos ? 0 : std::atoll(spec.c_str() + colon + 1);
  }
}

size_t Device::capacity() const {
  state_->activate();
  size_t free_b = 0, total = 0;
  cudaMemGetInfo(&free_b, &total);
  return total;
}

size_t Device::available() const {
  state_->activate();
  size_t free_b = 0, total = 0;
  cudaMemGetInfo(&free_b, &total);
  return free_b;
}

void Device::synchronize() const {
  state_->check();
  state_->activate();
  state_->check_cuda(cudaStreamSynchronize(state_->stream), "synchronize");
}

// ------------------------------------------------------------------------------------ buffers
DeviceAllocation::~DeviceAllocation() {
  if (ptr) device->release(ptr, bytes);
}

HbmBuffer::HbmBuffer(const Device& device, size_t bytes) {
  auto st = device.state();
  st->check();
  st->activate();
  auto a = std::make_shared<DeviceAllocation>();
  a->device = st;
  if (bytes > 0) {
    a->ptr = st->allocate(bytes, &a->bytes);
    if (a->ptr == nullptr)
      throw DeviceError("device allocation of " + std::to_string(bytes) + " bytes failed");
  }
  alloc_ = std::move(a);
  offset_ = 0;
  size_ = bytes;
}

HbmBuffer HbmBuffer::slice(size_t offset, size_t bytes) const {
  if (offset % 8 != 0 || bytes % 8 != 0)
    throw ValueError("a device range starts and ends on 8-byte boundaries");
  if (offset > size_ || bytes > size_ - offset) throw ValueError("the range is outside the allocation");
  return HbmBuffer(alloc_, offset_ + offset, bytes);
}

HbmBuffer HbmBuffer::slice_unchecked(size_t offset, size_t bytes) const {
  if (offset > size_ || bytes > size_ - offset) throw ValueError("the range is outside the allocation");
  return HbmBuffer(alloc_, offset_ + offset, bytes);
}

HostAllocation::~HostAllocation() {
  if (ptr) {
    if (pinned)
      cudaFreeHost(ptr);
    else
      free(ptr);
  }
}

HostBuffer::HostBuffer(size_t bytes) {
  alloc_ = std::make_shared<HostAllocation>();
  alloc_->bytes = bytes;
  const size_t n = bytes == 0 ? 1 : bytes;
  if (cudaHostAlloc(&alloc_->ptr, n, cudaHostAllocPortable) == cudaSuccess) {
    alloc_->pinned = true;
  } else {
    cudaGetLastError();
    alloc_->ptr = malloc(n);
    if (!alloc_->ptr) throw std::bad_alloc();
  }
  std::memset(alloc_->ptr, 0, n);
  size_ = bytes;
}

HostBuffer::HostBuffer(const void* src, size_t bytes) : HostBuffer(bytes) {
  if (bytes) std::memcpy(alloc_->ptr, src, bytes);
}

HostBuffer HostBuffer::slice(size_t offset, size_t bytes) const {
  if (bytes == 0) throw ValueError("a host range is not empty");
  if (offset > size_ || bytes > size_ - offset) throw ValueError("the range is outside the buffer");
  HostBuffer h;
  h.alloc_ = alloc_;
  h.offset_ = offset_ + offset;
  h.size_ = bytes;
  h.last_ = last_;
  return h;
}

std::shared_ptr<TransferState> HostBuffer::last() const { return *last_; }

TransferState::~TransferState() {
  if (done) {
    if (device) device->activate();
    cudaEventDestroy(done);
  }
}

namespace {
std::shared_ptr<TransferState> submit_copy(const std::shared_ptr<DeviceState>& dev, void* dst,
                                           const void* src, size_t bytes, cudaMemcpyKind kind) {
  dev->check();
  dev->activate();
  auto t = std::make_shared<TransferState>();
  t->device = dev;
  dev->check_cuda(cudaEventCreateWithFlags(&t->done, cudaEventDisableTiming), "transfer event");
  if (dev->injected("copy")) dev->fail("transfer failed (injected fault)");
  if (bytes) dev->check_cuda(cudaMemcpyAsync(dst, src, bytes, kind, dev->stream), "transfer");
  dev->check_cuda(cudaEventRecord(t->done, dev->stream), "transfer event");
  return t;
}
}  // namespace

Transfer HostBuffer::to_hbm(const HbmBuffer& dst) const {
  const size_t chips = dst.device()->chips.size();
  if (size_ != dst.size() * chips)
    throw ValueError("the host range holds " + std::to_string(size_) + " bytes, not " +
                     std::to_string(dst.size() * chips));
  // In a process per chip, this process moves its own chip's bytes: the rank's slice.
  const char* src = static_cast<const char*>(data()) + dst.size() * dst.device()->rank;
  auto t = submit_copy(dst.device(), dst.data(), src, dst.size(), cudaMemcpyHostToDevice);
  *last_ = t;
  return Transfer(t);
}

Transfer copy_to_host(const HbmBuffer& src, const HostBuffer& dst) {
  const size_t chips = src.device()->chips.size();
  if (dst.size() != src.size() * chips)
    throw ValueError("the host range holds " + std::to_string(dst.size()) + " bytes, not " +
                     std::to_string(src.size() * chips));
  char* out = static_cast<char*>(dst.data()) + src.size() * src.device()->rank;
  auto t = submit_copy(src.device(), out, src.data(), src.size(), cudaMemcpyDeviceToHost);
  *dst.last_ = t;
  return Transfer(t);
}

bool Transfer::done() const {
  if (!s_) return true;
  if (!s_->error.empty()) throw DeviceError(s_->error);
  s_->device->activate();
  const cudaError_t e = cudaEventQuery(s_->done);
  if (e == cudaErrorNotReady) {
    cudaGetLastError();
    return false;
  }
  if (e != cudaSuccess) {
    s_->error = std::string("transfer failed: ") + cudaGetErrorString(e);
    s_->device->poison = s_->error;
    throw DeviceError(s_->error);
  }
  return true;
}

void Transfer::wait() const {
  if (!s_) return;
  if (!s_->error.empty()) throw DeviceError(s_->error);
  s_->device->activate();
  const cudaError_t e = cudaEventSynchronize(s_->done);
  if (e != cudaSuccess) {
    s_->error = std::string("transfer failed: ") + cudaGetErrorString(e);
    s_->device->poison = s_->error;
    throw DeviceError(s_->error);
  }
}

// ------------------------------------------------------------------------------------ tensors
namespace {
int64_t product(const std::vector<int64_t>& shape) {
  int64_t n = 1;
  for (auto s : shape) {
    if (s < 0) throw ValueError("a dimension is negative");
    n *= s;
  }
  return n;
}
}  // namespace

HbmTensor::HbmTensor(HbmBuffer buffer, std::vector<int64_t> shape, DType dtype)
    : buffer_(std::move(buffer)), shape_(std::move(shape)), dtype_(dtype) {
  if (nbytes() > buffer_.size()) throw ValueError("the buffer is too small for the shape and dtype");
}

int64_t HbmTensor::numel() const { return product(shape_); }
size_t HbmTensor::nbytes() const { return static_cast<size_t>(numel()) * dtype_size(dtype_); }

void HbmTensor::wait() const {
  auto dev = buffer_.device();
  dev->check();
  dev->activate();
  // The kernels' status word travels with the same synchronisation: a bounded wait that gave up
  // raises here, when the result is read.
  int code = 0;
  dev->check_cuda(cudaMemcpyAsync(&code, dev->status, sizeof(int), cudaMemcpyDeviceToHost, dev->stream),
                  "status read");
  dev->check_cuda(cudaStreamSynchronize(dev->stream), "wait");
  dev->raise_status(code);
}

std::vector<uint8_t> HbmTensor::to_host_bytes() const {
  auto dev = buffer_.device();
  dev->check();
  dev->activate();
  if (dev->injected("copy")) dev->fail("copy to host failed (injected fault)");
  std::vector<uint8_t> out(nbytes());
  int code = 0;
  if (!out.empty())
    dev->check_cuda(cudaMemcpyAsync(out.data(), buffer_.data(), out.size(), cudaMemcpyDeviceToHost,
                                    dev->stream),
                    "copy to host");
  dev->check_cuda(cudaMemcpyAsync(&code, dev->status, sizeof(int), cudaMemcpyDeviceToHost, dev->stream),
                  "status read");
  dev->check_cuda(cudaStreamSynchronize(dev->stream), "copy to host");
  dev->raise_status(code);
  return out;
}

HbmTensor HbmTensor::rows(int64_t start, int64_t stop) const {
  if (shape_.empty()) throw ValueError("the tensor has no axes");
  const int64_t n = shape_[0];
  start = std::max<int64_t>(0, std::min(start, n));
  stop = std::max<int64_t>(start, std::min(stop, n));
  int64_t row = 1;
  for (size_t i = 1; i < shape_.size(); ++i) row *= shape_[i];
  const size_t rb = static_cast<size_t>(row) * dtype_size(dtype_);
  auto shape = shape_;
  shape[0] = stop - start;
  // Row views need not be 8-byte aligned: the view keeps the storage and a byte offset.
  return HbmTensor(buffer_.slice_unchecked(start * rb, (stop - start) * rb), shape, dtype_);
}

int64_t HostTensor::numel() const { return product(shape_); }

HostTensor::HostTensor(std::vector<int64_t> shape, DType dtype)
    : shape_(std::move(shape)), dtype_(dtype) {
  bytes_.assign(static_cast<size_t>(product(shape_)) * dtype_size(dtype_), 0);
}

HostTensor::HostTensor(std::vector<int64_t> shape, DType dtype, const void* bytes)
    : HostTensor(std::move(shape), dtype) {
  if (!bytes_.empty()) std::memcpy(bytes_.data(), bytes, bytes_.size());
}

void HostTensor::write(const void* bytes, size_t n) {
  if (n != bytes_.size())
    throw ValueError("the bytes hold " + std::to_string(n) + ", the tensor " +
                     std::to_string(bytes_.size()));
  std::memcpy(bytes_.data(), bytes, n);
}

HbmTensor HostTensor::to_hbm(const Device& device) const {
  HbmBuffer buf(device, std::max<size_t>(bytes_.size(), 8));
  auto dev = device.state();
  dev->activate();
  if (dev->injected("copy")) dev->fail("copy to device failed (injected fault)");
  if (!bytes_.empty())
    dev->check_cuda(cudaMemcpyAsync(buf.data(), bytes_.data(), bytes_.size(), cudaMemcpyHostToDevice,
                                    dev->stream),
                    "copy to device");
  dev->check_cuda(cudaStreamSynchronize(dev->stream), "copy to device");
  return HbmTensor(buf, shape_, dtype_);
}

}  // namespace foa::engine
