// foa_paged_decode_noalloc: paged decode attention that allocates no memory. The interface, its
// return codes and the size limit are declared in noalloc.h; this file has no counterpart in the
// reference (furiosa-ai/furiosa-opt-models).
//
// What it does: the same flash-decoding kernels as `paged_decode` (attention.cu) on one-row
// segments over the paged KV cache. When a history is longer than one split (`keys_per_split`
// keys), the per-split partial outputs and log-sum-exps go to a fixed scratch array declared in
// this file, `g_noalloc_scratch`, instead of caller- or engine-allocated buffers. The array is a
// file-scope `__device__` variable: it is part of the loaded library, every GPU that loads the
// library holds one copy of it until the process exits, and nothing allocates it at run time.
//
// Set-up: the first call on each device, with that device current, looks up the device address of
// the scratch array with cudaGetSymbolAddress and keeps it for later calls on that device. Make
// that first call before capturing any stream into a graph. The address belongs to the device's
// current context: after cudaDeviceReset (or any teardown of the primary context) the module is
// loaded again at another address, so a process that resets a device must not call this entry
// point on that device afterwards (the kept address would be stale).
//
// Sharing: every call on a device uses the same scratch array, and the array keeps whatever the
// last call left in it. Nothing in it has to start at zero: each call writes every partial before
// it reads it. Two calls whose kernels overlap on the GPU (different streams without ordering, or
// different host threads) race on the array; order them on one stream.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "attention.cuh"
#include "noalloc.h"

namespace {

constexpr size_t kNoAllocScratchBytes = FOA_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

std::mutex g_setup_mu;
float* g_scratch_address[kMaxDevices] = {};

void report(char* error, int error_len, const char* msg) {
  if (error == nullptr || error_len <= 0) return;
  std::strncpy(error, msg, static_cast<size_t>(error_len) - 1);
  error[error_len - 1] = '\0';
}

}  // namespace

// Declared in noalloc.h (return codes and the size limit there too).
extern "C" __attribute__((visibility("default"))) int foa_paged_decode_noalloc(
    const void* q, void* o, const void* cache, const int32_t* table, const int32_t* segments,
    int num_segments, int q_heads, int kv_heads, int head_dim, float scale, int max_keys,
    int keys_per_split, void* stream, char* error, int error_len) {
  if (q == nullptr || o == nullptr || cache == nullptr || table == nullptr || segments == nullptr ||
      num_segments <= 0 || q_heads <= 0 || kv_heads <= 0 || max_keys <= 0 || keys_per_split <= 0 ||
      (head_dim != 64 && head_dim != 128)) {
    report(error, error_len, "foa_paged_decode_noalloc: invalid argument");
    return FOA_NOALLOC_BAD_ARGUMENT;
  }
  const long long splits = (static_cast<long long>(max_keys) + keys_per_split - 1) / keys_per_split;
  const long long entries = static_cast<long long>(num_segments) * q_heads * splits;
  const long long need = entries * (head_dim + 1) * static_cast<long long>(sizeof(float));
  if (splits > 1 && need > static_cast<long long>(kNoAllocScratchBytes)) {
    report(error, error_len,
           "foa_paged_decode_noalloc: the call needs more scratch than the 16 MiB this entry point "
           "holds (segments * q_heads * splits * (head_dim + 1) * 4 bytes)");
    return FOA_NOALLOC_TOO_LARGE;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    report(error, error_len, "foa_paged_decode_noalloc: no current device");
    return FOA_NOALLOC_SETUP_FAILED;
  }
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (g_scratch_address[dev] == nullptr) {
      void* ptr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (e != cudaSuccess || ptr == nullptr) {
        cudaGetLastError();
        report(error, error_len, "foa_paged_decode_noalloc: cannot find the scratch array's address");
        return FOA_NOALLOC_SETUP_FAILED;
      }
      g_scratch_address[dev] = static_cast<float*>(ptr);
    }
    scratch = g_scratch_address[dev];
  }
  foa::PagedAttention a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.o = static_cast<__nv_bfloat16*>(o);
  a.cache = static_cast<const __nv_bfloat16*>(cache);
  a.table = table;
  a.segments = reinterpret_cast<const foa::Segment*>(segments);
  a.num_segments = num_segments;
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  a.head_dim = head_dim;
  a.scale = scale;
  // Log-sum-exps first, then the outputs, 256-byte aligned.
  const size_t lse_floats = (static_cast<size_t>(entries) + 63) / 64 * 64;
  a.partial_lse = scratch;
  a.partial_o = scratch + lse_floats;
  a.partial_capacity = static_cast<size_t>(entries);
  a.max_keys = max_keys;
  a.keys_per_split = keys_per_split;
  a.status = nullptr;
  if (splits > 1 && (lse_floats + static_cast<size_t>(entries) * head_dim) * sizeof(float) > kNoAllocScratchBytes) {
    report(error, error_len, "foa_paged_decode_noalloc: the call needs more scratch than this entry point holds");
    return FOA_NOALLOC_TOO_LARGE;
  }
  const int rc = foa::paged_decode(a, static_cast<cudaStream_t>(stream));
  if (rc != 0) {
    report(error, error_len, "foa_paged_decode_noalloc: the launch was rejected");
    return rc == -2 ? FOA_NOALLOC_BAD_ARGUMENT : FOA_NOALLOC_LAUNCH_FAILED;
  }
  return FOA_NOALLOC_OK;
}
