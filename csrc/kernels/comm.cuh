// Tensor-parallel collectives over NVLink peer memory, fused with the work around them.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gemm.cuh"

namespace foa {

constexpr int kMaxRanks = 8;

// Every rank's symmetric buffers, as this rank addresses them (peer pointers through CUDA IPC).
struct PeerBuffers {
  float* recv[kMaxRanks];               // FP32 partial receive regions (see AddNormArgs)
  __nv_bfloat16* residual[kMaxRanks];   // the residual stream [rows, cols]
  __nv_bfloat16* hidden[kMaxRanks];     // normed rows [rows, cols]
  unsigned long long* signal[kMaxRanks];  // barrier slots: slot i is written by rank i
  float* gather_value[kMaxRanks];       // argmax candidates [ranks][rows]
  int32_t* gather_index[kMaxRanks];
};

// The FP32 partial sums arrive in this rank's receive region, pushed there over NVLink by every
// rank's scatter (tp_scatter): [2 buffers][world source slots][slot rows][cols], the buffer
// picked by the low bit of `seq`. A slot holds -0.0 until its value lands; the reducer polls
// (bounded) until none of the values it needs is -0.0, then writes -0.0 back. `seq` advances once
// per call (by the last CTA to finish), so consecutive calls alternate buffers and a rank that
// runs ahead writes the buffer its peer is not reading.
struct AddNormArgs {
  PeerBuffers peers;
  const unsigned long long* epoch;  // this call's epoch (device memory, written per call)
  unsigned int* arrivals;           // this rank's CTA arrival counter (zero between calls)
  unsigned int* seq;                // this rank's receive sequence
  float* recv;                      // this rank's receive region
  long slot_stride, buf_stride;     // floats between source slots, between buffers
  const __nv_bfloat16* weight;
  float eps;
  int rows, cols, rank, world, site;
  // 0: every rank received every row (one-shot all-reduce) at slot row = row.
  // 1: rank r received rows [r * s, (r + 1) * s) at slot rows 0..s-1, s = ceil(rows / world)
  //    (reduce-scatter); it reduces them and stores the results into every rank (all-gather).
  int two_shot;
  // Reduce-scatter only: 1 stores the owner's residual rows into every rank too (callers that read
  // every row's residual, such as the mixture-of-experts combine); 0 keeps each residual row on
  // its owner alone, which is the only rank that adds to it again within the call.
  int gather_residual;
  int* status;
  // Optional: CTA 0 writes %globaltimer here at entry (after the grid dependency wait), once its
  // row's partials have all landed, and at exit.
  unsigned long long* trace;
  // Small calls (the grid at most kInlineScatterCtas CTAs): this rank's FP32 partial [rows, cols],
  // which each CTA first stores into the receive slots of the rows it reduces on every rank (the
  // scatter of tp_scatter, without its launch). Null: the partials arrive from tp_scatter.
  const float* partial;
  // With `partial` and splits.splits > 1: this rank's partial is the sum, in split order, of a
  // GEMM's K splits in its workspace (GemmSplits layout); `partial` is then not read.
  GemmSplits splits;
};

// The largest grid whose CTAs push their own rows before polling (they must all be resident, on
// every rank, at once).
constexpr int kInlineScatterCtas = 148;

// residual = bf16(sum over ranks in rank order of partial + residual); hidden = RMSNorm(residual)
// * weight; every rank ends with the same hidden rows, and with the same residual rows where it
// holds them (all of them one-shot; its own slice, or all with gather_residual, two-shot).
int tp_add_norm(const AddNormArgs& args, cudaStream_t stream);

// Stores this rank's FP32 partial [rows, cols] (cols a multiple of 4) into the receive slots that
// AddNormArgs describes: slot `rank` of buffer (*seq & 1) of every rank (owner_rows == 0), or of
// rank r / owner_rows at slot row r % owner_rows (reduce-scatter).
struct ScatterArgs {
  PeerBuffers peers;
  const float* partial;
  int rows, cols, rank, world, owner_rows;
  long slot_stride, buf_stride;
  const unsigned int* seq;
};
int tp_scatter(const ScatterArgs& args, cudaStream_t stream);

// Writes the not-yet-written mark (-0.0) over `floats` floats of a receive region.
int tp_clear_recv(float* recv, size_t floats, cudaStream_t stream);

struct ArgmaxArgs {
  PeerBuffers peers;
  const unsigned long long* epoch;
  const float* value;     // this rank's candidates [rows]
  const int32_t* index;
  int32_t* out;           // tokens [rows]
  int rows, rank, world, site;
  int* status;
};

// Row collectives between calls (reference: ops/collective/gather.rs:17-99 `AllGather`, parts
// joined in chip order, rows stacked [N*S, W] on every chip; ops/collective/mod.rs:313-344
// `Exchange`, chip t receives rows t*S.. of every chip's columns, [S, N*C]). This rank stores its
// BF16 part straight into every receiver's landing buffer (peers.hidden) over NVLink, 16 bytes a
// store, and fences them system-wide before it ends; a barrier then tells the receivers.
struct RowsArgs {
  PeerBuffers peers;
  const __nv_bfloat16* src;  // this rank's part [rows, cols]
  int rows, cols;            // cols a multiple of 8; for an exchange rows a multiple of world
  int rank, world;
  int exchange;              // 0: all-gather, 1: exchange
};
int tp_push_rows(const RowsArgs& args, cudaStream_t stream);

// Exchanges every rank's (value, index) candidates and keeps the first maximum.
int tp_argmax(const ArgmaxArgs& args, cudaStream_t stream);

struct MoeCombineArgs {
  PeerBuffers peers;                       // residual, hidden and signal slots
  const __nv_bfloat16* y[kMaxRanks];       // every rank's expert rows [capacity, cols] (BF16)
  long ldy;
  const int32_t* pos;                      // [world][rows * k]: a selection's row on its expert's rank
  const int32_t* ids;                      // [rows, k] experts, best first
  const float* weights;                    // [rows, k]
  int experts_local;                       // experts per rank (rank of expert e: e / experts_local)
  const __nv_bfloat16* norm;
  float eps;
  const unsigned long long* epoch;
  int rows, k, cols, rank, world, site;
  int* status;
};

// Expert-parallel combine over NVLink: after a barrier (every rank's expert rows in place), each
// rank reads every selection's BF16 row from the rank that computed it and forms
// residual = bf16(residual + bf16(sum_j w_j * y_j)) in choice order, then hidden = RMSNorm(residual)
// * norm; every rank ends with the same rows.
int tp_moe_combine_norm(const MoeCombineArgs& args, cudaStream_t stream);

// One thread waits, bounded by `limit_ns` (at most the kernels' 2 s), until `*flag` reaches
// `value`, recording the peer-timeout status when it gives up: the wait every peer flag uses.
int wait_probe(const unsigned long long* flag, unsigned long long value, uint64_t limit_ns, int* status,
               cudaStream_t stream);

// Writes this call's epoch (stream-ordered, outside any captured graph).
int tp_set_epoch(unsigned long long* epoch, unsigned long long value, cudaStream_t stream);

// Every rank waits for every other at this site (a device-side barrier, bounded).
int tp_barrier(const PeerBuffers& peers, const unsigned long long* epoch, int rank, int world,
               int site, int* status, cudaStream_t stream);

}  // namespace foa
