#include "trace.h"

#include <nvtx3/nvToolsExt.h>
#include <unistd.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <deque>
#include <fstream>
#include <iomanip>
#include <sstream>

namespace foa::engine {

namespace {
std::mutex g_log_mu;
std::deque<std::pair<int, std::string>> g_logs;
size_t g_dropped = 0;
std::atomic<bool> g_log_pending{false};
}  // namespace

void log_event(LogLevel level, std::string message) {
  std::lock_guard<std::mutex> g(g_log_mu);
  if (g_logs.size() >= kLogQueue) {
    g_logs.pop_front();
    ++g_dropped;
  }
  g_logs.emplace_back(static_cast<int>(level), std::move(message));
  g_log_pending.store(true, std::memory_order_release);
}

bool logs_pending() { return g_log_pending.load(std::memory_order_acquire); }

std::vector<std::pair<int, std::string>> take_logs() {
  std::lock_guard<std::mutex> g(g_log_mu);
  std::vector<std::pair<int, std::string>> out;
  if (g_dropped > 0) {
    out.emplace_back(static_cast<int>(LogLevel::Warning),
                     std::to_string(g_dropped) + " older engine log records were dropped (queue full)");
    g_dropped = 0;
  }
  out.insert(out.end(), std::make_move_iterator(g_logs.begin()), std::make_move_iterator(g_logs.end()));
  g_logs.clear();
  g_log_pending.store(false, std::memory_order_release);
  return out;
}

namespace {

std::atomic<int> g_level{-1};

std::string escape(const std::string& s) {
  std::string o;
  for (char c : s) {
    if (c == '"' || c == '\\') o += '\\';
    if (static_cast<unsigned char>(c) < 0x20) continue;
    o += c;
  }
  return o;
}

}  // namespace

TraceLevel parse_trace_level(const std::string& name) {
  if (name == "info") return TraceLevel::Info;
  if (name == "debug") return TraceLevel::Debug;
  if (name == "trace") return TraceLevel::Trace;
  return TraceLevel::Off;
}

TraceLevel trace_level() {
  int v = g_level.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* e = std::getenv("FURIOSA_OPT_PROFILE");
    if (e == nullptr) e = std::getenv("FOA_PROFILE");
    v = static_cast<int>(parse_trace_level(e ? e : ""));
    g_level.store(v, std::memory_order_relaxed);
  }
  return static_cast<TraceLevel>(v);
}

void set_trace_level(TraceLevel level) { g_level.store(static_cast<int>(level), std::memory_order_relaxed); }

uint64_t trace_now_ns() {
  return static_cast<uint64_t>(
      std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now().time_since_epoch())
          .count());
}

Tracer& Tracer::get() {
  static Tracer t;
  return t;
}

void Tracer::host_span(const std::string& name, const std::string& cat, uint64_t t0, uint64_t t1,
                       const std::string& args) {
  std::lock_guard<std::mutex> g(mu_);
  host_.push_back(Host{name, cat, args, t0, t1});
}

const Tracer::Base& Tracer::base(int ordinal, cudaStream_t stream) {
  for (const auto& b : bases_)
    if (b.ordinal == ordinal) return b;
  // Align the device clock with the host's: an event recorded on an idle stream.
  cudaStreamSynchronize(stream);
  cudaEvent_t e;
  cudaEventCreate(&e);
  cudaEventRecord(e, stream);
  cudaEventSynchronize(e);
  bases_.push_back(Base{ordinal, e, trace_now_ns()});
  return bases_.back();
}

cudaEvent_t Tracer::record(int ordinal, cudaStream_t stream) {
  std::lock_guard<std::mutex> g(mu_);
  base(ordinal, stream);
  cudaEvent_t e;
  cudaEventCreate(&e);
  cudaEventRecord(e, stream);
  events_.emplace_back(ordinal, e);
  return e;
}

void Tracer::device_span(const std::string& name, const std::string& cat, int ordinal, cudaEvent_t a,
                         cudaEvent_t b) {
  std::lock_guard<std::mutex> g(mu_);
  dev_.push_back(Dev{name, cat, ordinal, a, b});
}

size_t Tracer::pending() const {
  std::lock_guard<std::mutex> g(mu_);
  return host_.size() + dev_.size();
}

std::string Tracer::flush(const std::string& path_in) {
  std::lock_guard<std::mutex> g(mu_);
  if (host_.empty() && dev_.empty()) return "";
  std::string path = path_in;
  if (path.empty()) {
    const char* dir = std::getenv("FURIOSA_OPT_OUT_DIR");
    path = std::string(dir ? dir : ".") + "/trace-" + std::to_string(getpid()) + ".json";
  }
  const long pid = static_cast<long>(getpid());
  std::ostringstream out;
  out << std::fixed << std::setprecision(3);  // microseconds with nanosecond digits
  out << "{\"traceEvents\": [";
  bool first = true;
  auto sep = [&]() {
    if (!first) out << ",\n";
    first = false;
  };
  for (const auto& h : host_) {
    sep();
    out << "{\"name\": \"" << escape(h.name) << "\", \"cat\": \"" << escape(h.cat) << "\", \"ph\": \"X\", \"ts\": "
        << h.t0 / 1000.0 << ", \"dur\": " << (h.t1 - h.t0) / 1000.0 << ", \"pid\": " << pid << ", \"tid\": 0";
    if (!h.args.empty()) out << ", \"args\": " << h.args;
    out << "}";
  }
  for (const auto& d : dev_) {
    const Base* b = nullptr;
    for (const auto& x : bases_)
      if (x.ordinal == d.ordinal) b = &x;
    if (b == nullptr) continue;
    cudaSetDevice(d.ordinal);
    if (cudaEventSynchronize(d.b) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    float start_ms = 0.f, dur_ms = 0.f;
    if (cudaEventElapsedTime(&start_ms, b->event, d.a) != cudaSuccess ||
        cudaEventElapsedTime(&dur_ms, d.a, d.b) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    sep();
    const double ts = b->host_ns / 1000.0 + start_ms * 1000.0;
    out << "{\"name\": \"" << escape(d.name) << "\", \"cat\": \"" << escape(d.cat) << "\", \"ph\": \"X\", \"ts\": "
        << ts << ", \"dur\": " << dur_ms * 1000.0 << ", \"pid\": " << pid << ", \"tid\": " << 1 + d.ordinal
        << ", \"args\": {\"ns\": " << static_cast<long long>(dur_ms * 1e6) << ", \"step_ms\": " << dur_ms << "}}";
  }
  out << "]}\n";
  std::ofstream f(path);
  f << out.str();
  host_.clear();
  dev_.clear();
  for (auto& [ord, e] : events_) {
    cudaSetDevice(ord);
    cudaEventDestroy(e);
  }
  events_.clear();
  if (!f.good()) {
    log_event(LogLevel::Warning, "trace: could not write " + path);
    return "";
  }
  log_event(LogLevel::Info, "trace written to " + path);
  return path;
}

TraceScope::TraceScope(const char* name, const char* cat, TraceLevel level)
    : name_(name), cat_(cat), on_(trace_level() >= level && level != TraceLevel::Off) {
  if (on_) {
    t0_ = trace_now_ns();
    nvtxRangePushA(name);
  }
}

void TraceScope::end() {
  if (!on_) return;
  on_ = false;
  nvtxRangePop();
  Tracer::get().host_span(name_, cat_, t0_, trace_now_ns(), args_);
}

}  // namespace foa::engine
