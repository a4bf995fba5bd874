#include "comm_emulate.h"

#include <atomic>
#include <chrono>
#include <cmath>
#include <cstring>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <thread>

namespace foa::engine::emulate {

uint16_t bf16_bits(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return static_cast<uint16_t>((u >> 16) | 0x40u);  // NaN
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

float bf16_value(uint16_t bits) {
  const uint32_t u = static_cast<uint32_t>(bits) << 16;
  float x;
  std::memcpy(&x, &u, 4);
  return x;
}

namespace {

constexpr uint32_t kMark = 0x80000000u;  // -0.0: not written

template <typename T>
std::unique_ptr<std::atomic<T>[]> atomics(size_t n, T value) {
  std::unique_ptr<std::atomic<T>[]> p(new std::atomic<T>[n]);
  for (size_t i = 0; i < n; ++i) p[i].store(value, std::memory_order_relaxed);
  return p;
}

uint32_t bits_of(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  return u;
}

float float_of(uint32_t u) {
  float x;
  std::memcpy(&x, &u, 4);
  return x;
}

// One rank's memory that its peers write: receive slots, the rows the reducers store, barrier flags.
struct RankMemory {
  std::unique_ptr<std::atomic<uint32_t>[]> recv;
  std::unique_ptr<std::atomic<uint16_t>[]> residual, hidden;
  std::unique_ptr<std::atomic<uint64_t>[]> flags;  // [world]: the last barrier epoch each peer signalled
  std::atomic<uint32_t> seq{0};
};

class Emulation {
 public:
  Emulation(int world, const std::vector<AllReduceCall>& calls, const AllReduceOptions& o)
      : world_(world), calls_(calls), o_(o) {
    int max_rows = 0, max_cols = 0;
    for (const auto& c : calls) {
      if (static_cast<int>(c.partials.size()) != world) throw std::invalid_argument("one partial a rank");
      if (c.cols % 8 != 0) throw std::invalid_argument("cols: a multiple of 8");
      if (c.residual.size() != static_cast<size_t>(c.rows) * c.cols || c.weight.size() != static_cast<size_t>(c.cols))
        throw std::invalid_argument("residual [rows, cols] and weight [cols]");
      for (const auto& p : c.partials)
        if (p.size() != static_cast<size_t>(c.rows) * c.cols) throw std::invalid_argument("partials [rows, cols]");
      max_rows = std::max(max_rows, c.rows);
      max_cols = std::max(max_cols, c.cols);
    }
    slot_rows_ = o.slot_rows > 0 ? o.slot_rows : max_rows;
    cols_cap_ = max_cols;
    for (const auto& c : calls) {
      if (two_shot(c) ? (c.rows + world - 1) / world > slot_rows_ : c.rows > slot_rows_)
        throw std::invalid_argument("a call's rows do not fit the receive slots");
    }
    const size_t recv = static_cast<size_t>(2) * world * slot_rows_ * cols_cap_;
    const size_t rows = static_cast<size_t>(max_rows) * max_cols;
    for (int r = 0; r < world; ++r) {
      auto m = std::make_unique<RankMemory>();
      m->recv = atomics<uint32_t>(recv, kMark);
      m->residual = atomics<uint16_t>(rows, 0);
      m->hidden = atomics<uint16_t>(rows, 0);
      m->flags = atomics<uint64_t>(world, 0);
      mem_.push_back(std::move(m));
    }
    result_.calls.assign(calls.size(), std::vector<AllReduceRank>(world));
    result_.timeouts.assign(world, 0);
    for (const auto& c : calls) result_.two_shot.push_back(two_shot(c));
  }

  AllReduceResult run() {
    std::vector<std::thread> threads;
    std::vector<std::string> errors(world_);
    for (int r = 0; r < world_; ++r)
      threads.emplace_back([this, r, &errors] {
        try {
          rank_main(r);
        } catch (const std::exception& e) {
          errors[r] = e.what();
        }
      });
    for (auto& t : threads) t.join();
    for (const auto& e : errors)
      if (!e.empty()) throw std::runtime_error(e);
    return std::move(result_);
  }

 private:
  int world_, slot_rows_ = 0, cols_cap_ = 0;
  const std::vector<AllReduceCall>& calls_;
  AllReduceOptions o_;
  std::vector<std::unique_ptr<RankMemory>> mem_;
  AllReduceResult result_;

  bool two_shot(const AllReduceCall& c) const {
    const long pushed = static_cast<long>(c.rows) * c.cols * 4 * (world_ - 1);
    return pushed > o_.one_shot_bytes || c.rows > (o_.slot_rows > 0 ? o_.slot_rows : c.rows);
  }

  size_t slot(int parity, int source, int slot_row, int cols) const {
    return ((static_cast<size_t>(parity) * world_ + source) * slot_rows_ + slot_row) * static_cast<size_t>(cols);
  }

  // Rank `me`'s row `row` of its partial into slot row `slot_row` of rank `q` (scatter).
  void push(int me, const AllReduceCall& c, int parity, int row, int q, int slot_row) {
    if (me == o_.drop_rank) return;
    const float* src = c.partials[me].data() + static_cast<size_t>(row) * c.cols;
    std::atomic<uint32_t>* dst = mem_[q]->recv.get() + slot(parity, me, slot_row, c.cols);
    for (int j = 0; j < c.cols; ++j) {
      const uint32_t b = bits_of(src[j]);
      dst[j].store(b == kMark ? 0u : b, std::memory_order_release);
    }
  }

  void rank_main(int me) {
    std::mt19937 rng(o_.jitter_seed * 1000003u + static_cast<unsigned>(me));
    auto jitter = [&] {
      if (o_.jitter_seed != 0 && (rng() & 7u) == 0) std::this_thread::yield();
    };
    RankMemory& m = *mem_[me];
    for (size_t n = 0; n < calls_.size(); ++n) {
      const AllReduceCall& c = calls_[n];
      const bool two = two_shot(c);
      const int rs = two ? (c.rows + world_ - 1) / world_ : c.rows;  // slot rows this call uses
      const int parity = static_cast<int>(m.seq.load(std::memory_order_relaxed) & 1u);
      for (size_t i = 0; i < c.residual.size(); ++i) m.residual[i].store(c.residual[i], std::memory_order_relaxed);
      const bool inline_scatter = rs <= o_.inline_rows;
      if (!inline_scatter) {
        for (int row = 0; row < c.rows; ++row) {
          if (two) {
            const int q = row / rs;
            push(me, c, parity, row, q, row - q * rs);
          } else {
            for (int q = 0; q < world_; ++q) push(me, c, parity, row, q, row);
          }
          jitter();
        }
      }
      for (int s = 0; s < rs; ++s) {
        if (inline_scatter)
          for (int q = 0; q < world_; ++q) {
            const int row = two ? q * rs + s : s;
            if (row < c.rows) push(me, c, parity, row, q, s);
          }
        reduce(me, c, parity, two, rs, s, jitter);
      }
      m.seq.fetch_add(1u, std::memory_order_relaxed);
      if (two) barrier(me, n + 1);
      AllReduceRank& out = result_.calls[n][me];
      const size_t count = static_cast<size_t>(c.rows) * c.cols;
      out.hidden.resize(count);
      out.residual.resize(count);
      for (size_t i = 0; i < count; ++i) {
        out.hidden[i] = m.hidden[i].load(std::memory_order_relaxed);
        out.residual[i] = m.residual[i].load(std::memory_order_relaxed);
      }
    }
  }

  template <typename J>
  void reduce(int me, const AllReduceCall& c, int parity, bool two, int rs, int s, J& jitter) {
    const int row = two ? me * rs + s : s;
    if (row >= c.rows) return;
    const auto start = std::chrono::steady_clock::now();
    bool late = false;
    std::vector<float> acc(c.cols, 0.0f);
    for (int v = 0; v < c.cols / 8; ++v) {
      for (int p = 0; p < world_; ++p) {
        std::atomic<uint32_t>* src = mem_[me]->recv.get() + slot(parity, p, s, c.cols) + v * 8;
        uint32_t x[8];
        for (;;) {
          bool ready = true;
          for (int t = 0; t < 8; ++t) {
            x[t] = src[t].load(std::memory_order_acquire);
            ready &= x[t] != kMark;
          }
          if (ready || late) break;
          std::this_thread::yield();
          if (std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count() > o_.wait_limit_s) {
            ++result_.timeouts[me];
            late = true;
          }
        }
        for (int t = 0; t < 8; ++t) {
          acc[v * 8 + t] += float_of(x[t]);
          src[t].store(kMark, std::memory_order_relaxed);
        }
      }
      jitter();
    }
    const size_t base = static_cast<size_t>(row) * c.cols;
    std::vector<uint16_t> x(c.cols);
    double squares = 0.0;
    for (int j = 0; j < c.cols; ++j) {
      x[j] = bf16_bits(acc[j] + bf16_value(mem_[me]->residual[base + j].load(std::memory_order_relaxed)));
      const double h = bf16_value(x[j]);
      squares += h * h;
    }
    const float inv = 1.0f / std::sqrt(static_cast<float>(squares / c.cols) + c.eps);
    for (int j = 0; j < c.cols; ++j) {
      const uint16_t h = bf16_bits(bf16_value(x[j]) * inv * bf16_value(c.weight[j]));
      for (int q = 0; q < world_; ++q) {
        const bool mine = q == me;
        if (two || mine) mem_[q]->hidden[base + j].store(h, std::memory_order_relaxed);
        if (mine || (two && c.gather_residual)) mem_[q]->residual[base + j].store(x[j], std::memory_order_relaxed);
      }
    }
  }

  // Two-shot calls end at an epoch barrier: a rank signals every peer, then waits for every peer.
  void barrier(int me, uint64_t epoch) {
    std::atomic_thread_fence(std::memory_order_release);
    for (int q = 0; q < world_; ++q) mem_[q]->flags[me].store(epoch, std::memory_order_release);
    const auto start = std::chrono::steady_clock::now();
    for (int p = 0; p < world_; ++p) {
      while (mem_[me]->flags[p].load(std::memory_order_acquire) < epoch) {
        std::this_thread::yield();
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count() > o_.wait_limit_s) {
          ++result_.timeouts[me];
          break;
        }
      }
    }
  }
};

}  // namespace

AllReduceResult all_reduce(int world, const std::vector<AllReduceCall>& calls, const AllReduceOptions& options) {
  if (world < 1) throw std::invalid_argument("world: at least one rank");
  return Emulation(world, calls, options).run();
}

}  // namespace foa::engine::emulate
