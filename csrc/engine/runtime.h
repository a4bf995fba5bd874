// Runtime memory of the engine: devices, device and pinned host buffers, transfers and typed
// tensors (the layer the reference takes from its SDK and wraps in
// crates/furiosa-opt-python/src/tensor.rs).
//
// One process drives one GPU. A placement of N chips is served by N processes (one per GPU, the
// ranks of a torch.distributed group); each opens chips[rank]. Every device keeps one in-order
// stream, so calls and copies run in submission order, and a sticky error: after a failed
// launch or copy every later call raises.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <map>
#include <cstddef>
#include <cstdint>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

namespace foa::engine {

// Errors carry the Python exception class they map to.
struct ValueError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct Unsupported : std::runtime_error {  // NotImplementedError
  using std::runtime_error::runtime_error;
};
struct DeviceError : std::runtime_error {  // RuntimeError
  using std::runtime_error::runtime_error;
};
struct IoError : std::runtime_error {  // OSError
  using std::runtime_error::runtime_error;
};

// ------------------------------------------------------------------------------------ dtypes
enum class DType : int {
  Bool, U8, I8, I16, I32, I64, F16, BF16, F32, F64, F8E4M3, F8E5M2,
};
DType dtype_from_name(const std::string& name);  // engine names (torch-style); throws ValueError
const char* dtype_name(DType d);
size_t dtype_size(DType d);

// ------------------------------------------------------------------------------------ device
struct DeviceState {
  int ordinal = 0;             // CUDA ordinal this process opened
  std::vector<int> chips;      // placement chips in rank order
  int pes_begin = 0, pes_end = 8;
  int rank = 0;                // this process's index in `chips`
  cudaStream_t stream = nullptr;
  std::mutex mu;               // serialises calls on the device (the binding's device lock)
  std::string poison;          // first failure; non-empty poisons every later call
  int* status = nullptr;       // device status word the kernels write
  // Caching allocator: freed device blocks by size class, reused in stream order (every use of
  // device memory is ordered on `stream`, so a block freed by the host is reused only by work
  // submitted after every earlier use).
  std::mutex pool_mu;
  std::map<size_t, std::vector<void*>> pool;
  size_t pooled_bytes = 0;
  void* allocate(size_t bytes, size_t* rounded);
  void release(void* ptr, size_t rounded);
  // Returns every cached free block to the driver (after the stream's work): memory a dropped
  // model or cache held becomes the GPU's again (sleep mode). Returns the bytes freed.
  size_t trim();
  ~DeviceState();

  void check() const;                              // raises when poisoned
  void fail(const std::string& what);              // poisons and raises DeviceError
  void check_cuda(cudaError_t err, const char* what);
  void check_status();                             // reads the kernel status word (synchronises)
  // Raises (and poisons) when `code`, a status word read after the work that wrote it, is set.
  void raise_status(int code);
  void activate() const;                           // cudaSetDevice(ordinal)

  // Host-side fault injection (failure drills and tests; no GPU fault is made): after `countdown`
  // more events of `fault_kind` the next one fails as the real failure would. Kinds: "launch" (the
  // driver rejects a kernel launch), "copy" (a host-device copy fails), "peer" (a peer never
  // answers a collective: its bounded wait gives up). FOA_FAULT=<kind>:<countdown> sets it at open.
  std::string fault_kind;
  int64_t fault_countdown = -1;
  bool injected(const char* kind);
};

class Device {
 public:
  // Opens chips[rank] of the placement, `rank` being this process's rank among `chips.size()`.
  Device(std::vector<int> chips, int pes_begin, int pes_end, int rank);
  size_t capacity() const;
  size_t available() const;
  void synchronize() const;
  const std::shared_ptr<DeviceState>& state() const { return state_; }
  int chips() const { return static_cast<int>(state_->chips.size()); }

 private:
  std::shared_ptr<DeviceState> state_;
};

// ------------------------------------------------------------------------------------ buffers
struct DeviceAllocation {
  std::shared_ptr<DeviceState> device;
  void* ptr = nullptr;
  size_t bytes = 0;
  ~DeviceAllocation();
};

class HbmBuffer {
 public:
  HbmBuffer() = default;
  HbmBuffer(const Device& device, size_t bytes);
  HbmBuffer(std::shared_ptr<DeviceAllocation> alloc, size_t offset, size_t bytes)
      : alloc_(std::move(alloc)), offset_(offset), size_(bytes) {}
  size_t size() const { return size_; }
  void* data() const { return alloc_ ? static_cast<char*>(alloc_->ptr) + offset_ : nullptr; }
  HbmBuffer slice(size_t offset, size_t bytes) const;  // 8-byte aligned ranges
  HbmBuffer slice_unchecked(size_t offset, size_t bytes) const;
  const std::shared_ptr<DeviceState>& device() const { return alloc_->device; }
  bool valid() const { return alloc_ != nullptr; }
  bool same_storage(const HbmBuffer& o) const { return alloc_ == o.alloc_; }

 private:
  std::shared_ptr<DeviceAllocation> alloc_;
  size_t offset_ = 0, size_ = 0;
};

struct HostAllocation {
  void* ptr = nullptr;
  size_t bytes = 0;
  bool pinned = false;
  ~HostAllocation();
};

class Transfer;

class HostBuffer {
 public:
  HostBuffer() = default;
  explicit HostBuffer(size_t bytes);                    // zeroed, page-locked
  HostBuffer(const void* src, size_t bytes);            // a copy of `src`
  size_t size() const { return size_; }
  void* data() const { return alloc_ ? static_cast<char*>(alloc_->ptr) + offset_ : nullptr; }
  HostBuffer slice(size_t offset, size_t bytes) const;
  Transfer to_hbm(const HbmBuffer& dst) const;
  // The last transfer submitted on these bytes; exporting waits for it.
  std::shared_ptr<struct TransferState> last() const;

 private:
  friend class HbmBuffer;
  friend Transfer copy_to_host(const HbmBuffer& src, const HostBuffer& dst);
  std::shared_ptr<HostAllocation> alloc_;
  size_t offset_ = 0, size_ = 0;
  std::shared_ptr<std::shared_ptr<struct TransferState>> last_ = std::make_shared<std::shared_ptr<struct TransferState>>();
};

struct TransferState {
  std::shared_ptr<DeviceState> device;
  cudaEvent_t done = nullptr;
  std::string error;
  ~TransferState();
};

class Transfer {
 public:
  Transfer() = default;
  explicit Transfer(std::shared_ptr<TransferState> s) : s_(std::move(s)) {}
  bool done() const;
  void wait() const;
  const std::shared_ptr<TransferState>& state() const { return s_; }

 private:
  std::shared_ptr<TransferState> s_;
};

Transfer copy_to_host(const HbmBuffer& src, const HostBuffer& dst);

// ------------------------------------------------------------------------------------ tensors
class HbmTensor {
 public:
  HbmTensor(HbmBuffer buffer, std::vector<int64_t> shape, DType dtype);
  const std::vector<int64_t>& shape() const { return shape_; }
  DType dtype() const { return dtype_; }
  const HbmBuffer& buffer() const { return buffer_; }
  size_t nbytes() const;
  int64_t numel() const;
  void wait() const;
  std::vector<uint8_t> to_host_bytes() const;
  HbmTensor rows(int64_t start, int64_t stop) const;

 private:
  HbmBuffer buffer_;
  std::vector<int64_t> shape_;
  DType dtype_;
};

class HostTensor {
 public:
  HostTensor(std::vector<int64_t> shape, DType dtype);  // zeroed
  HostTensor(std::vector<int64_t> shape, DType dtype, const void* bytes);
  const std::vector<int64_t>& shape() const { return shape_; }
  DType dtype() const { return dtype_; }
  size_t nbytes() const { return bytes_.size(); }
  int64_t numel() const;
  const uint8_t* data() const { return bytes_.data(); }
  uint8_t* data() { return bytes_.data(); }
  void write(const void* bytes, size_t n);
  HbmTensor to_hbm(const Device& device) const;

 private:
  std::vector<int64_t> shape_;
  DType dtype_;
  std::vector<uint8_t> bytes_;
};

}  // namespace foa::engine
