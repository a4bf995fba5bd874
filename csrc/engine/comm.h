// Tensor-parallel collectives of one rank: a symmetric heap in device memory, exported through
// CUDA IPC and opened by every peer, and the fused collective kernels over it.
#pragma once

#include <string>
#include <vector>

#include "kernels/comm.cuh"
#include "model.h"
#include "runtime.h"

namespace foa::engine {

class PeerCollectives : public Collectives {
 public:
  // A heap for calls of up to `rows` rows of `cols` columns and `kept` returned rows, and (mixture
  // of experts) two buffers of `moe_rows` expert rows.
  PeerCollectives(const Device& device, int world, int rank, int64_t rows, int cols, int64_t kept,
                  int64_t moe_rows = 0);
  ~PeerCollectives() override;

  // This rank's heap as an opaque IPC handle; `connect` opens every rank's handle (in rank order).
  std::string handle() const;
  void connect(const std::vector<std::string>& handles);
  bool connected() const { return connected_; }

  int rank() const override { return rank_; }
  int world() const override { return world_; }
  void begin_call(cudaStream_t stream) override;
  float* partial_buffer() override;
  int add_norm(__nv_bfloat16* residual, const __nv_bfloat16* weight, float eps,
               __nv_bfloat16* out, int rows, int cols, cudaStream_t stream,
               const foa::GemmSplits* splits = nullptr) override;
  bool inline_scatter(int rows) const override;
  void argmax(const float* value, const int32_t* index, int rows, int32_t* out,
              cudaStream_t stream) override;
  __nv_bfloat16* residual_buffer() override;
  __nv_bfloat16* hidden_buffer() override;
  __nv_bfloat16* moe_rows(int which, size_t rows) override;
  void moe_combine_norm(int which, const int32_t* pos_all, const int32_t* ids, const float* weights,
                        int experts_local, const __nv_bfloat16* norm, float eps, int rows, int k,
                        int cols, cudaStream_t stream) override;
  // A device-side barrier of every rank (used before the heap is released).
  void barrier(cudaStream_t stream);
  // The reference's AllGather (exchange false: `dst` [rows * world, cols], the parts in rank
  // order) or Exchange (true: `dst` [rows / world, cols * world], rank t holding rows t * rows /
  // world .. of every rank's columns) of BF16 rows, between calls; every rank calls it in the same
  // order with the same shape. The parts land in the heap's hidden buffers between two barriers,
  // after one that keeps a rank from writing into a peer still in its call.
  void gather_rows(const __nv_bfloat16* src, int rows, int cols, bool exchange, __nv_bfloat16* dst,
                   cudaStream_t stream);
  // Reduce-scatter (two-shot) rather than one-shot for a call of `rows` rows.
  bool two_shot(int rows) const;
  // Measurement: the add_norm kernels write milestone timestamps here (null: none).
  void set_trace(unsigned long long* trace) { trace_ = trace; }
  // Fault drill (DeviceState::injected "peer"): the next collective reports a silent peer.
  void inject_peer(cudaStream_t stream);

 private:
  Device device_;
  int world_, rank_;
  int64_t rows_, kept_, moe_rows_;
  int cols_;
  void* heap_ = nullptr;
  size_t heap_bytes_ = 0;

  size_t off_signal_, off_arrivals_, off_seq_, off_epoch_, off_recv_, off_partial_, off_residual_, off_hidden_,
      off_gvalue_, off_gindex_, off_moe_;
  int64_t slot_rows_ = 0;          // rows of one source slot of the receive region
  size_t one_shot_limit_ = 0;      // bytes a one-shot call may push to its peers
  std::vector<void*> peer_base_;   // every rank's heap as mapped here (own heap at rank_)
  std::vector<bool> opened_;
  foa::PeerBuffers peers_{};
  bool connected_ = false;
  unsigned long long epoch_ = 0;
  int site_ = 0;
  int* status_ = nullptr;
  unsigned long long* trace_ = nullptr;
};

}  // namespace foa::engine
