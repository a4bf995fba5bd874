#include "comm.h"

#include <cstdlib>
#include <cstring>

namespace foa::engine {

namespace {
size_t align_to(size_t v, size_t a) { return (v + a - 1) / a * a; }
}  // namespace

PeerCollectives::PeerCollectives(const Device& device, int world, int rank, int64_t rows, int cols,
                                 int64_t kept, int64_t moe_rows)
    : device_(device), world_(world), rank_(rank), rows_(rows), kept_(kept), moe_rows_(moe_rows), cols_(cols) {
  if (world < 2 || world > foa::kMaxRanks) throw Unsupported("tensor parallelism takes 2 to 8 chips");
  auto st = device_.state();
  st->activate();
  status_ = st->status;
  size_t off = 0;
  off_signal_ = off;
  off = align_to(off + 64 * sizeof(unsigned long long), 4096);
  off_arrivals_ = off;
  off = align_to(off + 64, 256);
  off_seq_ = off;
  off = align_to(off + 64, 256);
  off_epoch_ = off;
  off = align_to(off + 64, 256);
  // Receive region: [2 buffers][world source slots][slot rows][cols] FP32. One-shot calls use
  // `rows` slot rows of every slot, reduce-scatter calls ceil(rows / world).
  slot_rows_ = (rows + world - 1) / world;
  off_recv_ = off;
  const size_t recv_floats = 2 * static_cast<size_t>(world) * slot_rows_ * cols;
  off = align_to(off + recv_floats * sizeof(float), 4096);
  // This rank's FP32 partial [rows][cols]: the row-parallel GEMM's local output, scattered from.
  off_partial_ = off;
  off = align_to(off + static_cast<size_t>(rows) * cols * sizeof(float), 4096);
  off_residual_ = off;
  off = align_to(off + static_cast<size_t>(rows) * cols * 2, 4096);
  off_hidden_ = off;
  off = align_to(off + static_cast<size_t>(rows) * cols * 2, 4096);
  off_gvalue_ = off;
  off = align_to(off + static_cast<size_t>(world) * kept * 4, 256);
  off_gindex_ = off;
  off = align_to(off + static_cast<size_t>(world) * kept * 4, 4096);
  off_moe_ = off;
  off = align_to(off + 2 * static_cast<size_t>(moe_rows) * cols * 2, 4096);
  heap_bytes_ = off;
  st->check_cuda(cudaMalloc(&heap_, heap_bytes_), "tensor-parallel heap");
  st->check_cuda(cudaMemset(heap_, 0, heap_bytes_), "tensor-parallel heap");
  // Every receive slot starts unwritten; peers write into it only after `connect`.
  if (foa::tp_clear_recv(reinterpret_cast<float*>(static_cast<char*>(heap_) + off_recv_), recv_floats,
                         st->stream) != 0)
    st->fail("receive region launch failed");
  st->check_cuda(cudaStreamSynchronize(st->stream), "tensor-parallel heap");
  const char* lim = std::getenv("FOA_TP_ONESHOT_BYTES");
  // One-shot pushes (world - 1) copies of the call's partials; up to 4 MiB of them it beats the
  // reduce-scatter's second hop and barrier (2 B200s, Qwen3-1.7B o_proj: 256 rows 17.6 against
  // 28.0 us; 1024 rows 61.8 against 43.2 us).
  one_shot_limit_ = lim ? static_cast<size_t>(std::strtoull(lim, nullptr, 10)) : (size_t{4} << 20);
  peer_base_.assign(world, nullptr);
  opened_.assign(world, false);
  peer_base_[rank] = heap_;
}

PeerCollectives::~PeerCollectives() {
  device_.state()->activate();
  cudaStreamSynchronize(device_.state()->stream);
  for (int p = 0; p < world_; ++p)
    if (opened_[p]) cudaIpcCloseMemHandle(peer_base_[p]);
  if (heap_) cudaFree(heap_);
}

std::string PeerCollectives::handle() const {
  cudaIpcMemHandle_t h;
  device_.state()->activate();
  if (cudaIpcGetMemHandle(&h, heap_) != cudaSuccess) {
    cudaGetLastError();
    throw DeviceError("cannot export the tensor-parallel heap");
  }
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

void PeerCollectives::connect(const std::vector<std::string>& handles) {
  if (static_cast<int>(handles.size()) != world_) throw ValueError("one handle per rank");
  auto st = device_.state();
  st->activate();
  for (int p = 0; p < world_; ++p) {
    if (p == rank_) continue;
    cudaIpcMemHandle_t h;
    if (handles[p].size() != sizeof(h)) throw ValueError("malformed peer handle");
    std::memcpy(&h, handles[p].data(), sizeof(h));
    void* ptr = nullptr;
    st->check_cuda(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess), "open peer heap");
    peer_base_[p] = ptr;
    opened_[p] = true;
  }
  for (int p = 0; p < world_; ++p) {
    char* b = static_cast<char*>(peer_base_[p]);
    peers_.signal[p] = reinterpret_cast<unsigned long long*>(b + off_signal_);
    peers_.recv[p] = reinterpret_cast<float*>(b + off_recv_);
    peers_.residual[p] = reinterpret_cast<__nv_bfloat16*>(b + off_residual_);
    peers_.hidden[p] = reinterpret_cast<__nv_bfloat16*>(b + off_hidden_);
    peers_.gather_value[p] = reinterpret_cast<float*>(b + off_gvalue_);
    peers_.gather_index[p] = reinterpret_cast<int32_t*>(b + off_gindex_);
  }
  connected_ = true;
}

void PeerCollectives::begin_call(cudaStream_t stream) {
  if (!connected_) throw DeviceError("tensor-parallel peers are not connected");
  ++epoch_;
  site_ = 0;
  auto* ep = reinterpret_cast<unsigned long long*>(static_cast<char*>(heap_) + off_epoch_);
  if (foa::tp_set_epoch(ep, epoch_, stream) != 0) device_.state()->fail("epoch launch failed");
}

bool PeerCollectives::two_shot(int rows) const {
  // Little data: every rank receives every row (one NVLink hop, no barrier). More: each row goes
  // to the rank that reduces its slice, which stores the results into every rank (1/world of the
  // traffic, plus a closing barrier).
  const size_t one_shot_bytes = static_cast<size_t>(rows) * cols_ * 4 * (world_ - 1);
  return one_shot_bytes > one_shot_limit_ || rows > slot_rows_;
}

float* PeerCollectives::partial_buffer() {
  return reinterpret_cast<float*>(static_cast<char*>(heap_) + off_partial_);
}

__nv_bfloat16* PeerCollectives::residual_buffer() {
  return reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(heap_) + off_residual_);
}

__nv_bfloat16* PeerCollectives::hidden_buffer() {
  return reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(heap_) + off_hidden_);
}

__nv_bfloat16* PeerCollectives::moe_rows(int which, size_t rows) {
  if (rows > static_cast<size_t>(moe_rows_)) throw ValueError("call exceeds the expert-parallel heap");
  return reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(heap_) + off_moe_) +
         static_cast<size_t>(which & 1) * moe_rows_ * cols_;
}

void PeerCollectives::moe_combine_norm(int which, const int32_t* pos_all, const int32_t* ids,
                                       const float* weights, int experts_local,
                                       const __nv_bfloat16* norm, float eps, int rows, int k, int cols,
                                       cudaStream_t stream) {
  foa::MoeCombineArgs a{};
  a.peers = peers_;
  for (int p = 0; p < world_; ++p)
    a.y[p] = reinterpret_cast<const __nv_bfloat16*>(static_cast<char*>(peer_base_[p]) + off_moe_) +
             static_cast<size_t>(which & 1) * moe_rows_ * cols_;
  a.ldy = cols;
  a.pos = pos_all;
  a.ids = ids;
  a.weights = weights;
  a.experts_local = experts_local;
  a.norm = norm;
  a.eps = eps;
  a.epoch = reinterpret_cast<const unsigned long long*>(static_cast<char*>(heap_) + off_epoch_);
  a.rows = rows;
  a.k = k;
  a.cols = cols;
  a.rank = rank_;
  a.world = world_;
  a.site = site_++;
  a.status = status_;
  if (foa::tp_moe_combine_norm(a, stream) != 0) device_.state()->fail("expert-parallel combine launch failed");
}

bool PeerCollectives::inline_scatter(int rows) const {
  const int grid = two_shot(rows) ? (rows + world_ - 1) / world_ : rows;
  return grid <= foa::kInlineScatterCtas;
}

int PeerCollectives::add_norm(__nv_bfloat16* residual, const __nv_bfloat16* weight, float eps,
                              __nv_bfloat16* out, int rows, int cols, cudaStream_t stream,
                              const foa::GemmSplits* splits) {
  if (residual != residual_buffer() || out != hidden_buffer())
    throw DeviceError("tensor-parallel add_norm takes the heap's own buffers");
  if (cols != cols_ || rows > rows_) throw ValueError("call exceeds the tensor-parallel heap");
  if (!connected_) throw DeviceError("tensor-parallel peers are not connected");
  const bool two = two_shot(rows);
  // Small calls (decode): each reducer CTA first stores its rows of this rank's partial into the
  // peers, all CTAs resident at once, which saves the scatter's launch. Larger calls: the
  // partial goes out from every SM in a scatter kernel, and the reducer behind it polls.
  const bool inline_scatter = this->inline_scatter(rows);
  if (splits != nullptr && splits->splits > 1 && !inline_scatter)
    throw DeviceError("GEMM K splits reach add_norm only in calls whose reducer scatters");
  if (!inline_scatter) {
  foa::ScatterArgs sc{};
  sc.peers = peers_;
  sc.partial = partial_buffer();
  sc.rows = rows;
  sc.cols = cols;
  sc.rank = rank_;
  sc.world = world_;
  sc.owner_rows = two ? (rows + world_ - 1) / world_ : 0;
  sc.slot_stride = static_cast<long>(slot_rows_) * cols_;
  sc.buf_stride = sc.slot_stride * world_;
  sc.seq = reinterpret_cast<const unsigned int*>(static_cast<char*>(heap_) + off_seq_);
  if (foa::tp_scatter(sc, stream) != 0) device_.state()->fail("tensor-parallel scatter launch failed");
  }
  foa::AddNormArgs a{};
  a.partial = inline_scatter ? partial_buffer() : nullptr;
  if (inline_scatter && splits != nullptr && splits->splits > 1) a.splits = *splits;
  a.peers = peers_;
  a.epoch = reinterpret_cast<const unsigned long long*>(static_cast<char*>(heap_) + off_epoch_);
  a.arrivals = reinterpret_cast<unsigned int*>(static_cast<char*>(heap_) + off_arrivals_);
  a.seq = reinterpret_cast<unsigned int*>(static_cast<char*>(heap_) + off_seq_);
  a.recv = peers_.recv[rank_];
  a.slot_stride = static_cast<long>(slot_rows_) * cols_;
  a.buf_stride = a.slot_stride * world_;
  a.weight = weight;
  a.eps = eps;
  a.rows = rows;
  a.cols = cols;
  a.rank = rank_;
  a.world = world_;
  a.site = site_++;
  a.two_shot = two ? 1 : 0;
  a.gather_residual = moe_rows_ > 0 ? 1 : 0;  // the expert combine reads every row's residual
  a.status = status_;
  a.trace = trace_;
  if (foa::tp_add_norm(a, stream) != 0) device_.state()->fail("tensor-parallel add_norm launch failed");
  inject_peer(stream);
  return inline_scatter ? 1 : 2;
}

void PeerCollectives::inject_peer(cudaStream_t stream) {
  // Host-side drill of a peer that never answers: the status word the kernel's bounded wait
  // would write, read when the call's result is.
  static const int kPeerTimeout = 5;
  if (device_.state()->injected("peer"))
    cudaMemcpyAsync(status_, &kPeerTimeout, sizeof(int), cudaMemcpyHostToDevice, stream);
}

void PeerCollectives::argmax(const float* value, const int32_t* index, int rows, int32_t* out,
                             cudaStream_t stream) {
  if (rows > kept_) throw ValueError("call keeps more rows than the tensor-parallel heap holds");
  foa::ArgmaxArgs a{};
  a.peers = peers_;
  a.epoch = reinterpret_cast<const unsigned long long*>(static_cast<char*>(heap_) + off_epoch_);
  a.value = value;
  a.index = index;
  a.out = out;
  a.rows = rows;
  a.rank = rank_;
  a.world = world_;
  a.site = site_++;
  a.status = status_;
  if (foa::tp_argmax(a, stream) != 0) device_.state()->fail("tensor-parallel argmax launch failed");
}

void PeerCollectives::barrier(cudaStream_t stream) {
  auto* ep = reinterpret_cast<const unsigned long long*>(static_cast<char*>(heap_) + off_epoch_);
  ++epoch_;
  foa::tp_set_epoch(const_cast<unsigned long long*>(ep), epoch_, stream);
  if (foa::tp_barrier(peers_, ep, rank_, world_, 0, status_, stream) != 0)
    device_.state()->fail("tensor-parallel barrier launch failed");
}

void PeerCollectives::gather_rows(const __nv_bfloat16* src, int rows, int cols, bool exchange,
                                  __nv_bfloat16* dst, cudaStream_t stream) {
  if (!connected_) throw ValueError("gather_rows: the collectives are not connected");
  if (rows <= 0 || cols <= 0 || cols % 8 != 0)
    throw ValueError("gather_rows: rows and columns positive, columns a multiple of 8");
  if (exchange && rows % world_ != 0)
    throw ValueError("gather_rows: an exchange splits its rows evenly over the ranks");
  const int64_t elems = static_cast<int64_t>(rows) * cols * world_;
  if (elems > rows_ * cols_)
    throw ValueError("gather_rows: " + std::to_string(elems) + " gathered values pass the landing buffer of " +
                     std::to_string(rows_ * cols_));
  barrier(stream);
  foa::RowsArgs a{};
  a.peers = peers_;
  a.src = src;
  a.rows = rows;
  a.cols = cols;
  a.rank = rank_;
  a.world = world_;
  a.exchange = exchange ? 1 : 0;
  if (foa::tp_push_rows(a, stream) != 0) device_.state()->fail("tensor-parallel row push launch failed");
  barrier(stream);
  device_.state()->check_cuda(cudaMemcpyAsync(dst, peers_.hidden[rank_], static_cast<size_t>(elems) * 2,
                                              cudaMemcpyDeviceToDevice, stream),
                              "gathered rows copy");
  barrier(stream);
}

}  // namespace foa::engine
