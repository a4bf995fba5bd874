// Tensor-parallel collectives over NVLink peer memory.
//
// The reference's all-reduce is a deterministic FP32 recursive doubling over chip DMA, narrowed
// to BF16 once at the end (crates/furiosa-opt-models/src/ops/collective/mod.rs:22-141); its
// all-gather joins parts in chip order (gather.rs:17-99). Here the row-parallel GEMM writes its FP32
// partial into this rank's memory at full speed; a scatter kernel on every SM then stores it over
// NVLink into the receive buffers of the reducing ranks, and the reducer (launched while the
// scatter runs) adds the landed partials in rank order, so every rank computes the same bits (in
// small calls, whose reducer CTAs are all resident at once, each reducer CTA first stores its own
// rows to the peers, with no scatter launch); the
// sum is fused with the residual add (one rounding) and the RMSNorm that follows. Small calls push
// every row to every rank (one-shot: one NVLink hop, no barrier); large calls push each row to the
// rank that owns its slice (reduce-scatter), and the owner stores the normed rows into every rank
// (all-gather) before a closing barrier.
//
// Arrival is detected without flags: a receive slot holds -0.0 until its value lands (the scatter
// never sends -0.0), and the reducer writes -0.0 back after reading. Ranks meet at device-side
// barriers elsewhere: a rank stores a monotonically increasing value into its slot of every
// peer's signal array (release, system scope) and waits, bounded, until every slot of its own
// array has reached the value. A wait that gives up records kTimeoutPeer and returns.

#include <algorithm>

#include "comm.cuh"
#include "launch.cuh"
#include "sm100.cuh"

namespace foa {
namespace {

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long barrier_value(const unsigned long long* epoch,
                                                            int site, int phase) {
  return (*epoch) * 4096ull + (unsigned long long)site * 2ull + (unsigned long long)phase + 1ull;
}

__device__ void signal_all(const PeerBuffers& pb, int rank, int world, unsigned long long v) {
  __threadfence_system();
  for (int p = 0; p < world; ++p) st_release_sys(pb.signal[p] + rank, v);
}

// Waits until `*flag` reaches `v` (acquire, system scope); gives up after `limit_ns`, recording
// kTimeoutPeer.
__device__ bool wait_flag(const unsigned long long* flag, unsigned long long v, uint64_t start,
                          uint64_t limit_ns, int* status) {
  uint32_t spins = 0;
  while (ld_acquire_sys(flag) < v) {
    if ((++spins & 255u) == 0 && global_ns() - start > limit_ns) {
      record_status(status, kTimeoutPeer);
      return false;
    }
  }
  return true;
}

__device__ bool wait_all(const PeerBuffers& pb, int rank, int world, unsigned long long v,
                         int* status) {
  const unsigned long long* s = pb.signal[rank];
  const uint64_t start = global_ns();
  for (int p = 0; p < world; ++p)
    if (!wait_flag(s + p, v, start, kWaitLimitNs, status)) return false;
  return true;
}

// The peers' bounded wait on one flag, with its own limit: a test makes it run out (a flag nothing
// sets) and reads the status the kernel leaves, the context still usable.
__global__ void wait_probe_kernel(const unsigned long long* flag, unsigned long long v, uint64_t limit_ns,
                                  int* status) {
  wait_flag(flag, v, global_ns(), limit_ns, status);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  return t;
}

constexpr uint32_t kUnwritten = 0x80000000u;  // -0.0: a receive slot whose value has not landed

__device__ __forceinline__ float4 ld_volatile_f4(const float* p) {
  float4 v;
  asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ bool unwritten(const float4& v) {
  return (__float_as_uint(v.x) == kUnwritten) | (__float_as_uint(v.y) == kUnwritten) |
         (__float_as_uint(v.z) == kUnwritten) | (__float_as_uint(v.w) == kUnwritten);
}

// One CTA of 256 threads per row; each thread holds kVec vectors of 8 columns. The partials are
// pushed here by the scatter kernels of every rank; each thread polls its 8 values of every source
// slot, adds them in rank order and marks the slot unwritten again. It follows this rank's scatter,
// which lets it launch only after the kernels before the scatter completed (so the previous
// reducer's sequence advance and every earlier read of the residual and normed rows are done); the
// partials themselves are polled for, so this kernel does not wait for the scatter to finish.
template <int kVec>
__global__ void __launch_bounds__(256) tp_add_norm_kernel(const AddNormArgs a) {
  if (a.partial != nullptr) pdl_wait();  // inline scatter: this rank's partial is complete
  pdl_trigger();
  __shared__ float red[8];
  const int rs = a.two_shot ? (a.rows + a.world - 1) / a.world : a.rows;
  const int slot_row = blockIdx.x;
  const int row = a.two_shot ? a.rank * rs + slot_row : slot_row;
  const unsigned int parity = __ldcg(a.seq) & 1u;
  if (a.partial != nullptr) {
    // Every rank's CTA `slot_row` reduces slot row `slot_row`: store this rank's rows of it there
    // (one-shot: row slot_row to every rank; two-shot: row q * rs + slot_row to rank q), -0.0 as
    // +0.0 so the unwritten mark stays unambiguous.
    const long off = (long)parity * a.buf_stride + (long)a.rank * a.slot_stride + (long)slot_row * a.cols;
    for (int q = 0; q < a.world; ++q) {
      const int src_row = a.two_shot ? q * rs + slot_row : slot_row;
      if (src_row >= a.rows) continue;
      const float4* src = reinterpret_cast<const float4*>(a.partial + (long)src_row * a.cols);
      float4* dst = reinterpret_cast<float4*>(a.peers.recv[q] + off);
      for (int v = threadIdx.x; v < a.cols / 4; v += blockDim.x) {
        float4 x;
        if (a.splits.splits > 1) {
          // The GEMM's K splits, added in split order (what its reduction would have stored); the
          // loads all go out first.
          float4 p[GemmSplits::kMax];
#pragma unroll
          for (int s = 0; s < GemmSplits::kMax; ++s)
            if (s < a.splits.splits)
              p[s] = __ldcg(reinterpret_cast<const float4*>(a.splits.ws + a.splits.at(s, src_row, 4L * v)));
          x = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int s = 0; s < GemmSplits::kMax; ++s)
            if (s < a.splits.splits) {
              x.x += p[s].x; x.y += p[s].y; x.z += p[s].z; x.w += p[s].w;
            }
        } else {
          x = __ldcg(src + v);
        }
        x.x = __float_as_uint(x.x) == kUnwritten ? 0.f : x.x;
        x.y = __float_as_uint(x.y) == kUnwritten ? 0.f : x.y;
        x.z = __float_as_uint(x.z) == kUnwritten ? 0.f : x.z;
        x.w = __float_as_uint(x.w) == kUnwritten ? 0.f : x.w;
        dst[v] = x;
      }
    }
  }
  float* recv = a.recv + (long)parity * a.buf_stride + (long)slot_row * a.cols;
  const int nvec = a.cols / 8;
  const bool tracer = a.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0;
  if (tracer) a.trace[0] = global_ns();
  if (row < a.rows) {
    const uint64_t start = global_ns();
    bool late = false;
    float h[kVec][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
      const int v = threadIdx.x + i * 256;
      if (v >= nvec) continue;
      float acc[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) acc[t] = 0.f;
      for (int p = 0; p < a.world; ++p) {
        float* src = recv + (long)p * a.slot_stride + v * 8;
        float4 x0, x1;
        uint32_t spins = 0;
        for (;;) {
          x0 = ld_volatile_f4(src);
          x1 = ld_volatile_f4(src + 4);
          if (!(unwritten(x0) || unwritten(x1)) || late) break;
          __nanosleep(100);  // polled while the pushing GEMM runs: leave it the issue slots
          if ((++spins & 63u) == 0 && global_ns() - start > kWaitLimitNs) {
            record_status(a.status, kTimeoutPeer);
            late = true;
          }
        }
        acc[0] += x0.x; acc[1] += x0.y; acc[2] += x0.z; acc[3] += x0.w;
        acc[4] += x1.x; acc[5] += x1.y; acc[6] += x1.z; acc[7] += x1.w;
        const float m = __uint_as_float(kUnwritten);
        reinterpret_cast<float4*>(src)[0] = make_float4(m, m, m, m);
        reinterpret_cast<float4*>(src)[1] = make_float4(m, m, m, m);
      }
      const __nv_bfloat16* rp = a.peers.residual[a.rank] + (long)row * a.cols + v * 8;
      const uint4 rv = *reinterpret_cast<const uint4*>(rp);
      const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
      uint32_t packed[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        packed[t] = pack_bf16x2(acc[2 * t] + bf16_lo(rw[t]), acc[2 * t + 1] + bf16_hi(rw[t]));
        h[i][2 * t] = bf16_lo(packed[t]);
        h[i][2 * t + 1] = bf16_hi(packed[t]);
        ss += h[i][2 * t] * h[i][2 * t] + h[i][2 * t + 1] * h[i][2 * t + 1];
      }
      const uint4 out = make_uint4(packed[0], packed[1], packed[2], packed[3]);
      if (a.two_shot && a.gather_residual) {
        for (int p = 0; p < a.world; ++p)
          *reinterpret_cast<uint4*>(a.peers.residual[p] + (long)row * a.cols + v * 8) = out;
      } else {
        *reinterpret_cast<uint4*>(a.peers.residual[a.rank] + (long)row * a.cols + v * 8) = out;
      }
    }
    const float total = block_sum(ss, red);
    if (tracer) a.trace[1] = global_ns();
    const float inv = rsqrtf(total / (float)a.cols + a.eps);
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
      const int v = threadIdx.x + i * 256;
      if (v >= nvec) continue;
      const uint4 wv = *reinterpret_cast<const uint4*>(a.weight + v * 8);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int t = 0; t < 4; ++t)
        o[t] = pack_bf16x2(h[i][2 * t] * inv * bf16_lo(ww[t]), h[i][2 * t + 1] * inv * bf16_hi(ww[t]));
      const uint4 out = make_uint4(o[0], o[1], o[2], o[3]);
      if (a.two_shot) {
        for (int p = 0; p < a.world; ++p)
          *reinterpret_cast<uint4*>(a.peers.hidden[p] + (long)row * a.cols + v * 8) = out;
      } else {
        *reinterpret_cast<uint4*>(a.peers.hidden[a.rank] + (long)row * a.cols + v * 8) = out;
      }
    }
  }
  // The last CTA to finish advances the receive sequence (every CTA has read it) and, two-shot,
  // tells every peer its slice has landed and waits until every peer's slice has landed here, so
  // the kernel ends only with every row in place.
  __syncthreads();
  if (threadIdx.x == 0) {
    if (a.two_shot)
      __threadfence_system();
    else
      __threadfence();
    const unsigned int done = atomicAdd(a.arrivals, 1u);
    if (done == gridDim.x - 1) {
      *a.arrivals = 0;
      *a.seq += 1u;
      if (a.two_shot) {
        const unsigned long long v = barrier_value(a.epoch, a.site, 1);
        signal_all(a.peers, a.rank, a.world, v);
        wait_all(a.peers, a.rank, a.world, v, a.status);
      }
    }
    if (tracer) a.trace[2] = global_ns();
  }
}

// Stores this rank's FP32 partial (the row-parallel GEMM's local output) into the receive slots
// of the ranks that reduce it, from every SM: each thread moves 16 bytes of a row (consecutive
// threads, consecutive columns: a warp's stores to one rank cover 512 contiguous bytes), with a
// -0.0 value sent as +0.0 so the slot's unwritten mark stays unambiguous.
__global__ void __launch_bounds__(256) tp_scatter_kernel(const ScatterArgs a) {
  pdl_wait();     // the GEMM's partial is complete (and every kernel before it)
  pdl_trigger();  // the reducer may launch now and poll for what lands
  const long off = (long)(__ldcg(a.seq) & 1u) * a.buf_stride + (long)a.rank * a.slot_stride;
  const int vec = a.cols / 4;
  const long total = (long)a.rows * vec;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int r = static_cast<int>(i / vec), c = static_cast<int>(i % vec) * 4;
    float4 v = __ldcg(reinterpret_cast<const float4*>(a.partial + (long)r * a.cols + c));
    const float z = 0.f;
    v.x = __float_as_uint(v.x) == kUnwritten ? z : v.x;
    v.y = __float_as_uint(v.y) == kUnwritten ? z : v.y;
    v.z = __float_as_uint(v.z) == kUnwritten ? z : v.z;
    v.w = __float_as_uint(v.w) == kUnwritten ? z : v.w;
    if (a.owner_rows > 0) {
      const int q = r / a.owner_rows;
      *reinterpret_cast<float4*>(a.peers.recv[q] + off + (long)(r - q * a.owner_rows) * a.cols + c) = v;
    } else {
      for (int q = 0; q < a.world; ++q)
        *reinterpret_cast<float4*>(a.peers.recv[q] + off + (long)r * a.cols + c) = v;
    }
  }
}

__global__ void fill_u32_kernel(uint32_t* p, size_t n, uint32_t v) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    p[i] = v;
}

template <int kVec>
__global__ void __launch_bounds__(256) tp_moe_combine_kernel(const MoeCombineArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8];
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    const unsigned long long v = barrier_value(a.epoch, a.site, 0);
    if (blockIdx.x == 0) signal_all(a.peers, a.rank, a.world, v);
    ok_s = wait_all(a.peers, a.rank, a.world, v, a.status);
  }
  __syncthreads();
  if (!ok_s) return;
  const int r = blockIdx.x;
  const long n = (long)a.rows * a.k;
  float xs[kVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c >= a.cols) continue;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < a.k; ++j) {
      const long sel = (long)r * a.k + j;
      const int owner = a.ids[sel] / a.experts_local;
      if (owner < 0 || owner >= a.world) continue;
      const int p = a.pos[owner * n + sel];
      if (p < 0) continue;
      const float w = a.weights[sel];
      const uint4 q = *reinterpret_cast<const uint4*>(a.y[owner] + (long)p * a.ldy + c);
      const uint32_t v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        acc[2 * t] = __fadd_rn(acc[2 * t], __fmul_rn(w, bf16_lo(v[t])));
        acc[2 * t + 1] = __fadd_rn(acc[2 * t + 1], __fmul_rn(w, bf16_hi(v[t])));
      }
    }
    __nv_bfloat16* xr = a.peers.residual[a.rank] + (long)r * a.cols + c;
    const uint4 q = *reinterpret_cast<const uint4*>(xr);
    const uint32_t v[4] = {q.x, q.y, q.z, q.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float m0 = __bfloat162float(__float2bfloat16_rn(acc[2 * t]));
      const float m1 = __bfloat162float(__float2bfloat16_rn(acc[2 * t + 1]));
      o[t] = pack_bf16x2(bf16_lo(v[t]) + m0, bf16_hi(v[t]) + m1);
      xs[i][2 * t] = bf16_lo(o[t]);
      xs[i][2 * t + 1] = bf16_hi(o[t]);
      ss += xs[i][2 * t] * xs[i][2 * t] + xs[i][2 * t + 1] * xs[i][2 * t + 1];
    }
    *reinterpret_cast<uint4*>(xr) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  const float total = block_sum(ss, red);
  const float inv = rsqrtf(total / (float)a.cols + a.eps);
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int c = (threadIdx.x + i * 256) * 8;
    if (c >= a.cols) continue;
    const uint4 wv = *reinterpret_cast<const uint4*>(a.norm + c);
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t)
      o[t] = pack_bf16x2(xs[i][2 * t] * inv * bf16_lo(ww[t]), xs[i][2 * t + 1] * inv * bf16_hi(ww[t]));
    *reinterpret_cast<uint4*>(a.peers.hidden[a.rank] + (long)r * a.cols + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void __launch_bounds__(256) tp_argmax_kernel(const ArgmaxArgs a) {
  pdl_wait();
  pdl_trigger();
  // Push this rank's candidates into every rank's gather arrays.
  for (int i = threadIdx.x; i < a.rows; i += blockDim.x) {
    const float v = a.value[i];
    const int32_t x = a.index[i];
    for (int p = 0; p < a.world; ++p) {
      a.peers.gather_value[p][(long)a.rank * a.rows + i] = v;
      a.peers.gather_index[p][(long)a.rank * a.rows + i] = x;
    }
  }
  __syncthreads();
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    const unsigned long long v = barrier_value(a.epoch, a.site, 0);
    signal_all(a.peers, a.rank, a.world, v);
    ok_s = wait_all(a.peers, a.rank, a.world, v, a.status);
  }
  __syncthreads();
  if (!ok_s) return;
  const float* gv = a.peers.gather_value[a.rank];
  const int32_t* gi = a.peers.gather_index[a.rank];
  for (int i = threadIdx.x; i < a.rows; i += blockDim.x) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int p = 0; p < a.world; ++p) {
      const float v = gv[(long)p * a.rows + i];
      const int x = gi[(long)p * a.rows + i];
      if (v > bv || (v == bv && x < bi)) {
        bv = v;
        bi = x;
      }
    }
    a.out[i] = bi == 0x7fffffff ? 0 : bi;
  }
}

__global__ void tp_barrier_kernel(PeerBuffers peers, const unsigned long long* epoch, int rank,
                                  int world, int site, int* status) {
  pdl_wait();
  const unsigned long long v = barrier_value(epoch, site, 0);
  signal_all(peers, rank, world, v);
  wait_all(peers, rank, world, v, status);
}

__global__ void set_u64_kernel(unsigned long long* p, unsigned long long v) { *p = v; }

__global__ void __launch_bounds__(256) tp_push_rows_kernel(const RowsArgs a) {
  pdl_wait();
  const int vec = a.cols / 8;  // 16-byte vectors a row
  const long total = (long)a.rows * vec;
  const int part = a.exchange ? a.rows / a.world : a.rows;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int r = static_cast<int>(i / vec);
    const int c = static_cast<int>(i % vec) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(a.src + (long)r * a.cols + c);
    if (a.exchange) {
      // Row r goes to rank r / part, at its row r % part, in the column block of this rank.
      const int t = r / part;
      __nv_bfloat16* dst = a.peers.hidden[t] + (long)(r % part) * a.world * a.cols + (long)a.rank * a.cols + c;
      *reinterpret_cast<uint4*>(dst) = v;
    } else {
      for (int p = 0; p < a.world; ++p) {
        __nv_bfloat16* dst = a.peers.hidden[p] + ((long)a.rank * a.rows + r) * a.cols + c;
        *reinterpret_cast<uint4*>(dst) = v;
      }
    }
  }
  __threadfence_system();
}

}  // namespace

int tp_moe_combine_norm(const MoeCombineArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return 0;
  if (a.cols % 8 != 0 || a.cols > 8 * 256 * 4 || a.world < 1 || a.world > kMaxRanks) return -2;
  const int vec = (a.cols / 8 + 255) / 256;
  auto kernel = vec <= 1 ? tp_moe_combine_kernel<1> : vec <= 2 ? tp_moe_combine_kernel<2> : tp_moe_combine_kernel<4>;
  return launch_pdl(kernel, dim3(a.rows), dim3(256), 0, stream, a) == cudaSuccess ? 0 : -5;
}

int wait_probe(const unsigned long long* flag, unsigned long long value, uint64_t limit_ns, int* status,
               cudaStream_t stream) {
  if (limit_ns > kWaitLimitNs) return -2;
  wait_probe_kernel<<<1, 1, 0, stream>>>(flag, value, limit_ns, status);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int tp_set_epoch(unsigned long long* epoch, unsigned long long value, cudaStream_t stream) {
  set_u64_kernel<<<1, 1, 0, stream>>>(epoch, value);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int tp_add_norm(const AddNormArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return 0;
  if (a.world < 1 || a.world > kMaxRanks || a.cols % 8 != 0) return -2;
  const int vec = (a.cols / 8 + 255) / 256;
  const int grid = a.two_shot ? (a.rows + a.world - 1) / a.world : a.rows;
  if (a.partial != nullptr && (grid > kInlineScatterCtas || a.cols % 4 != 0 || a.splits.splits > GemmSplits::kMax))
    return -2;
  cudaError_t e;
  switch (vec) {
    case 1: e = launch_pdl(tp_add_norm_kernel<1>, dim3(grid), dim3(256), 0, stream, a); break;
    case 2: e = launch_pdl(tp_add_norm_kernel<2>, dim3(grid), dim3(256), 0, stream, a); break;
    case 3:
    case 4: e = launch_pdl(tp_add_norm_kernel<4>, dim3(grid), dim3(256), 0, stream, a); break;
    default: return -2;
  }
  return e == cudaSuccess ? 0 : -5;
}

int tp_scatter(const ScatterArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return 0;
  if (a.world < 1 || a.world > kMaxRanks || a.cols % 4 != 0) return -2;
  const long vecs = (long)a.rows * (a.cols / 4);
  const int blocks = static_cast<int>(std::min<long>((vecs + 255) / 256, 148 * 8));
  return launch_pdl(tp_scatter_kernel, dim3(blocks), dim3(256), 0, stream, a) == cudaSuccess ? 0 : -5;
}

int tp_clear_recv(float* recv, size_t floats, cudaStream_t stream) {
  if (floats == 0) return 0;
  fill_u32_kernel<<<296, 256, 0, stream>>>(reinterpret_cast<uint32_t*>(recv), floats, kUnwritten);
  return cudaGetLastError() == cudaSuccess ? 0 : -5;
}

int tp_argmax(const ArgmaxArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return 0;
  return launch_pdl(tp_argmax_kernel, dim3(1), dim3(256), 0, stream, a) == cudaSuccess ? 0 : -5;
}

int tp_push_rows(const RowsArgs& a, cudaStream_t stream) {
  if (a.rows <= 0 || a.cols <= 0 || a.cols % 8 != 0 || a.world < 1 || a.world > kMaxRanks ||
      (a.exchange && a.rows % a.world != 0) ||
      reinterpret_cast<uintptr_t>(a.src) % 16 != 0)
    return -2;
  const long vecs = (long)a.rows * (a.cols / 8);
  const int blocks = static_cast<int>(std::min<long>((vecs + 255) / 256, 148 * 4));
  return launch_pdl(tp_push_rows_kernel, dim3(blocks), dim3(256), 0, stream, a) == cudaSuccess ? 0 : -5;
}

int tp_barrier(const PeerBuffers& peers, const unsigned long long* epoch, int rank, int world,
               int site, int* status, cudaStream_t stream) {
  return launch_pdl(tp_barrier_kernel, dim3(1), dim3(1), 0, stream, peers, epoch, rank, world,
                    site, status) == cudaSuccess
             ? 0
             : -5;
}

}  // namespace foa
