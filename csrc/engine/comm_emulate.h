// Host-thread emulation of the tensor-parallel add+norm all-reduce (csrc/kernels/comm.cu
// `tp_scatter_kernel`, `tp_add_norm_kernel`): one thread per rank runs the kernels' schedule on
// host memory, concurrently, so the protocol is exercised under real interleavings on a CPU.
//
// What is emulated, as the kernels do it:
// - every rank's receive region: [2 buffers][world source slots][slot rows][cols] FP32 values,
//   "-0.0" meaning not yet written; the buffer is the low bit of the rank's call sequence;
// - the scatter: a rank stores its partial rows into the slots of the ranks that reduce them
//   (every rank one-shot; the owner of the row's slice two-shot), a -0.0 value sent as +0.0; either
//   all rows before reducing, or (small calls) each slot row right before reducing it (inline);
// - the reducer: for each 8-value vector it polls every source slot in rank order until none of
//   its values is -0.0, with a time limit after which it records a timeout and goes on (the
//   kernels' bounded waits), adds them in FP32 from +0.0, writes -0.0 back, adds the BF16 residual
//   with one rounding and normalises the row;
// - two-shot: the owner stores the normed rows (and, when asked, the residual rows) into every
//   rank, and the ranks meet at an epoch barrier before the call ends; each rank advances its
//   sequence once per call.
// The norm's inverse is computed as 1 / sqrt(mean + eps) in FP32 from an FP64 mean (the device
// uses rsqrtf); the residual, which carries every partial, is the bitwise contract.
#pragma once

#include <cstdint>
#include <vector>

namespace foa::engine::emulate {

struct AllReduceCall {
  int rows = 0, cols = 0;
  std::vector<std::vector<float>> partials;  // [world][rows * cols]
  std::vector<uint16_t> residual;            // BF16 bits [rows * cols], the same on every rank
  std::vector<uint16_t> weight;              // BF16 bits [cols]
  float eps = 1e-6f;
  bool gather_residual = false;              // two-shot: store residual rows into every rank
};

struct AllReduceOptions {
  int slot_rows = 0;             // rows a receive slot holds (one-shot needs rows <= slot_rows)
  long one_shot_bytes = 4 << 20;  // pushed bytes up to which a call is one-shot
  int inline_rows = 148;          // calls of at most this many reducer rows scatter inline
  double wait_limit_s = 2.0;      // a poll's time limit
  unsigned jitter_seed = 0;       // nonzero: random yields between vectors, to vary interleavings
  int drop_rank = -1;             // a rank that never scatters (its peers' waits run out)
};

struct AllReduceRank {
  std::vector<uint16_t> hidden;    // BF16 bits [rows * cols]
  std::vector<uint16_t> residual;  // BF16 bits [rows * cols]
};

struct AllReduceResult {
  std::vector<std::vector<AllReduceRank>> calls;  // [call][rank]
  std::vector<int> timeouts;                      // per rank: polls and barrier waits that ran out
  std::vector<bool> two_shot;                     // per call
};

// Runs `calls` one after another on every rank (each rank a thread of its own) and returns every
// rank's rows after each call.
AllReduceResult all_reduce(int world, const std::vector<AllReduceCall>& calls, const AllReduceOptions& options);

uint16_t bf16_bits(float x);  // round to nearest even
float bf16_value(uint16_t bits);

}  // namespace foa::engine::emulate
