// Tracing of engine calls: host spans (wall clock) and device spans (CUDA events on the call's
// stream), written as a Chrome trace (the JSON that chrome://tracing and Perfetto read) and marked
// as NVTX ranges for Nsight tools.
//
// Reference: FURIOSA_OPT_PROFILE=info|debug|trace records device spans for a `tracing` subscriber
// (docs/reference/environment.md:19); the benchmark writes them with `tracing_chrometrace`
// (crates/furiosa-opt-engine/tests/forward.rs:340-357) and its metrics action aggregates the
// `forward` spans' step time and the kernels' cycles (.github/actions/metrics/action.yml:10-67).
// Here the same switch (FURIOSA_OPT_PROFILE, or FOA_PROFILE) takes the same levels:
//   info:  a host span per call ("forward", "encoder.vision", ...) and the call's device span
//          ("forward.device"), whose args carry step_ms;
//   debug: also the call's host phases (plan, stage, launch);
//   trace: also a device span per kernel launch ("GPU" category, args ns); calls then run eagerly
//          (no CUDA graph) and an event between two launches serializes them.
// The trace is written to FURIOSA_OPT_OUT_DIR (default ".") as trace-<pid>.json by flush(), which
// the Python package calls at exit.
#pragma once

#include <cuda_runtime.h>

#include <chrono>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

namespace foa::engine {

// Engine log records for Python's `logging` (logger "furiosa_opt_engine"). Engine code queues them
// from any thread and under any lock: queuing calls no Python and takes only the queue's own lock.
// The binding hands the queue to `logging` on the calling thread when a public call returns or
// raises. Levels are Python's numbers; the queue keeps the newest kLogQueue records.
enum class LogLevel : int { Debug = 10, Info = 20, Warning = 30, Error = 40 };
constexpr size_t kLogQueue = 1024;
void log_event(LogLevel level, std::string message);
bool logs_pending();
std::vector<std::pair<int, std::string>> take_logs();

enum class TraceLevel : int { Off = 0, Info = 1, Debug = 2, Trace = 3 };

TraceLevel trace_level();
void set_trace_level(TraceLevel level);  // overrides the environment (tests, tools)
TraceLevel parse_trace_level(const std::string& name);

uint64_t trace_now_ns();  // host clock of the spans (steady, nanoseconds)

class Tracer {
 public:
  static Tracer& get();
  void host_span(const std::string& name, const std::string& cat, uint64_t t0_ns, uint64_t t1_ns,
                 const std::string& args_json = "");
  // A device span between two events recorded on `stream` of device `ordinal` (resolved at flush).
  void device_span(const std::string& name, const std::string& cat, int ordinal, cudaEvent_t begin,
                   cudaEvent_t end);
  // An event recorded now on `stream` (from a pool; returned at flush).
  cudaEvent_t record(int ordinal, cudaStream_t stream);
  // Writes every span so far as Chrome trace JSON to `path` (empty: the default path) and clears
  // them; returns the path written, or "" when there was nothing to write.
  std::string flush(const std::string& path = "");
  size_t pending() const;

 private:
  struct Host {
    std::string name, cat, args;
    uint64_t t0, t1;
  };
  struct Dev {
    std::string name, cat;
    int ordinal;
    cudaEvent_t a, b;
  };
  struct Base {
    int ordinal;
    cudaEvent_t event;
    uint64_t host_ns;
  };
  mutable std::mutex mu_;
  std::vector<Host> host_;
  std::vector<Dev> dev_;
  std::vector<Base> bases_;
  std::vector<std::pair<int, cudaEvent_t>> events_;  // every event handed out (destroyed at flush)
  const Base& base(int ordinal, cudaStream_t stream);
};

// A host span from construction to destruction, recorded when the level reaches `level`, with an
// NVTX range around it.
class TraceScope {
 public:
  TraceScope(const char* name, const char* cat, TraceLevel level = TraceLevel::Info);
  ~TraceScope() { end(); }
  void end();  // records the span now (once)
  void args(std::string json) { args_ = std::move(json); }
  bool on() const { return on_; }

 private:
  const char* name_;
  const char* cat_;
  bool on_;
  uint64_t t0_ = 0;
  std::string args_;
};

}  // namespace foa::engine
