// The engine's Python classes: the surface of the `furiosa_opt_engine` wheel (its generated stubs
// name every class and method: crates/furiosa-opt-engine/python/furiosa_opt_engine/*.pyi).
//
// Calls release the GIL around device work. Errors map to Python classes by kind: invalid input
// to ValueError, a refused feature to NotImplementedError, a device failure to RuntimeError, a
// file failure to OSError.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>
#include <optional>

#include "engine/batch.h"
#include "engine/comm.h"
#include "engine/model.h"
#include "engine/registry.h"
#include "engine/runtime.h"
#include "engine/trace.h"
#include "kernels/gemm.cuh"
#include "python/pytypes.h"

namespace py = pybind11;
using namespace foa::engine;

void emit_logs() {
  if (!logs_pending()) return;
  const auto records = take_logs();
  try {
    py::object logger = py::module_::import("logging").attr("getLogger")("furiosa_opt_engine");
    for (const auto& [level, message] : records) logger.attr("log")(level, message);
  } catch (py::error_already_set& e) {
    e.discard_as_unraisable("furiosa_opt_engine log");
  }
}

LogsOnExit::~LogsOnExit() {
  try {
    emit_logs();
  } catch (...) {
  }
}

namespace {

// ------------------------------------------------------------------------------------ helpers
struct Range {
  int64_t start = 0, stop = 0, step = 1;
};

Range to_range(const py::object& r) {
  if (!py::isinstance(r, py::module_::import("builtins").attr("range")))
    throw py::type_error("expected a range");
  return Range{r.attr("start").cast<int64_t>(), r.attr("stop").cast<int64_t>(),
               r.attr("step").cast<int64_t>()};
}

py::object make_range(int64_t a, int64_t b) {
  return py::module_::import("builtins").attr("range")(a, b);
}

int process_rank(size_t chips) {
  // A placement of N chips runs as N processes, one per GPU: this process serves chips[rank].
  if (chips <= 1) return 0;
  py::object tp = py::module_::import("furiosa_opt_models_b200.parallel.tp");
  return tp.attr("rank_for_chips")(chips).cast<int>();
}

// ------------------------------------------------------------------------------------ Placement
struct Placement {
  std::vector<int> chips;
  int64_t pes_begin = 0, pes_end = 0;
};

// ------------------------------------------------------------------------------------ tensors
py::array host_numpy(const std::vector<int64_t>& shape, DType dtype, const uint8_t* data) {
  std::vector<py::ssize_t> dims(shape.begin(), shape.end());
  auto np = py::module_::import("numpy");
  size_t n = 1;
  for (auto s : shape) n *= static_cast<size_t>(s);
  auto copy = [&](const char* fmt) {
    py::array a(py::dtype(fmt), dims);
    std::memcpy(a.mutable_data(), data, n * dtype_size(dtype));
    return a;
  };
  switch (dtype) {
    case DType::Bool: return copy("?");
    case DType::U8: return copy("u1");
    case DType::I8: return copy("i1");
    case DType::I16: return copy("i2");
    case DType::I32: return copy("i4");
    case DType::I64: return copy("i8");
    case DType::F16: return copy("f2");
    case DType::F32: return copy("f4");
    case DType::F64: return copy("f8");
    case DType::BF16: {
      // NumPy has no BF16: observe the values as lossless F32.
      py::array_t<float> a(dims);
      auto* out = a.mutable_data();
      for (size_t i = 0; i < n; ++i) {
        uint32_t bits = static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(data)[i]) << 16;
        std::memcpy(out + i, &bits, 4);
      }
      return a;
    }
    case DType::F8E4M3:
    case DType::F8E5M2: return copy("u1");
  }
  return copy("u1");
}

}  // namespace

struct PyCacheSpec {
  CacheSpec spec;
  Device device;
};
struct PyCache {
  std::shared_ptr<Cache> cache;
  Device device;
};

struct PyRequest {
  std::vector<std::vector<int64_t>> rows;
  int64_t cached = 0;
  std::shared_ptr<HbmTensor> tokens;
  Keep keep;
  py::object keep_obj;
  std::optional<int64_t> adapter;
  py::object positions = py::none(), mask = py::none();
  std::vector<std::pair<int64_t, py::object>> overrides;
};

enum class PyKeep { NONE, LAST, ALL };
enum class PyOutput { TOKENS, HIDDEN, SCORES };

struct PyKind {
  KindTag tag = KindTag::Paged;
  int64_t length = 0;
};
struct PyKindPaged : PyKind {};
struct PyKindState : PyKind {};
struct PyKindCross : PyKind {};

ModelConfig model_config_from_dict(const py::dict& d) {
  ModelConfig c;
  auto get = [&](const char* k, auto def) {
    using T = decltype(def);
    return d.contains(k) ? d[k].cast<T>() : def;
  };
  c.architecture = get("architecture", std::string("Qwen3ForCausalLM"));
  c.family = get("family", std::string("qwen3"));
  c.size = get("size", std::string("custom"));
  c.precision = get("precision", std::string("bfloat16"));
  c.weight_format = get("weight_format", std::string("bf16"));
  c.hidden = get("hidden", 0);
  c.intermediate = get("intermediate", 0);
  c.layers = get("layers", 0);
  c.q_heads = get("q_heads", 0);
  c.kv_heads = get("kv_heads", 0);
  c.head_dim = get("head_dim", 128);
  c.vocab = get("vocab", 0);
  c.eps = get("eps", 1e-6f);
  c.qk_norm = get("qk_norm", false);
  c.tied = get("tied", false);
  c.window = get("window", 32768);
  c.rows = get("rows", 8192);
  c.labels = get("labels", 0);
  c.experts = get("experts", 0);
  c.top_k = get("top_k", 0);
  c.expert_intermediate = get("expert_intermediate", 0);
  c.norm_topk = get("norm_topk", true);
  const std::string out = get("output", std::string("tokens"));
  c.output = out == "hidden" ? Output::Hidden : out == "scores" ? Output::Scores : Output::Tokens;
  if (d.contains("rope")) {
    py::dict r = d["rope"];
    auto rg = [&](const char* k, auto def) {
      using T = decltype(def);
      return r.contains(k) && !r[k].is_none() ? r[k].cast<T>() : def;
    };
    c.rope.type = rg("type", std::string("default"));
    c.rope.theta = rg("theta", 10000.0);
    c.rope.factor = rg("factor", 1.0);
    c.rope.low_freq_factor = rg("low_freq_factor", 1.0);
    c.rope.high_freq_factor = rg("high_freq_factor", 4.0);
    c.rope.original_max_positions = rg("original_max_positions", 0.0);
    c.rope.beta_fast = rg("beta_fast", 32.0);
    c.rope.beta_slow = rg("beta_slow", 1.0);
    c.rope.mscale = rg("mscale", 1.0);
    c.rope.mscale_all_dim = rg("mscale_all_dim", 0.0);
    c.rope.attention_factor = rg("attention_factor", 0.0);
    c.rope.truncate = rg("truncate", true);
  }
  return c;
}

void bind_checkpoint_and_load(py::module_& m);

void bind_engine(py::module_& m) {
  // Exception classes by kind.
  py::register_exception_translator([](std::exception_ptr p) {
    try {
      if (p) std::rethrow_exception(p);
    } catch (const ValueError& e) {
      PyErr_SetString(PyExc_ValueError, e.what());
    } catch (const Unsupported& e) {
      PyErr_SetString(PyExc_NotImplementedError, e.what());
    } catch (const DeviceError& e) {
      PyErr_SetString(PyExc_RuntimeError, e.what());
    } catch (const IoError& e) {
      PyErr_SetString(PyExc_OSError, e.what());
    }
  });

  py::module_ decoder = m.def_submodule("decoder", "Decoder calls: requests, caches and outputs.");
  py::module_ qwen3 = m.def_submodule("qwen3", "Qwen3 decoders.");
  py::module_ llama = m.def_submodule("llama", "Llama decoders.");
  py::module_ mistral = m.def_submodule("mistral", "Mistral decoders.");
  py::module_ qwen3_moe = m.def_submodule("qwen3_moe", "Qwen3 mixture-of-experts decoders.");
  py::module_ mixtral = m.def_submodule("mixtral", "Mixtral mixture-of-experts decoders.");

  // ---------------------------------------------------------------- Placement / Device
  py::class_<Placement>(m, "Placement", "Physical chips, in rank order, and the PEs used on each.")
      .def(py::init([](const std::vector<int>& chips, const py::object& pes) {
             Range r = to_range(pes);
             if (r.step != 1) throw ValueError("pes has a step other than 1");
             return Placement{chips, r.start, r.stop};
           }),
           py::arg("chips"), py::arg("pes"))
      .def_property_readonly("chips", [](const Placement& p) { return p.chips; })
      .def_property_readonly("pes", [](const Placement& p) { return make_range(p.pes_begin, p.pes_end); })
      .def("__eq__", [](const Placement& a, const py::object& o) {
        if (!py::isinstance<Placement>(o)) return false;
        const auto& b = o.cast<const Placement&>();
        return a.chips == b.chips && a.pes_begin == b.pes_begin && a.pes_end == b.pes_end;
      })
      .def("__repr__", [](const Placement& p) {
        std::string s = "Placement(chips=[";
        for (size_t i = 0; i < p.chips.size(); ++i) s += (i ? ", " : "") + std::to_string(p.chips[i]);
        return s + "], pes=range(" + std::to_string(p.pes_begin) + ", " + std::to_string(p.pes_end) + "))";
      });

  py::class_<Device>(m, "Device", "An opened device; memory sizes are bytes per chip.")
      .def(py::init([](const Placement& p, std::optional<int> rank) {
             LogsOnExit logs;
             // The process's rank among the placement's chips: given (a framework that runs several
             // replicas in one process group), else the process group's rank.
             const int r = rank ? *rank : process_rank(p.chips.size());
             py::gil_scoped_release nogil;
             return Device(p.chips, static_cast<int>(p.pes_begin), static_cast<int>(p.pes_end), r);
           }),
           py::arg("placement"), py::arg("rank") = py::none())
      .def_property_readonly("capacity", &Device::capacity)
      .def_property_readonly("available", &Device::available)
      .def_property_readonly("chips", &Device::chips)
      .def_property_readonly("rank", [](const Device& d) { return d.state()->rank; })
      .def_property_readonly("ordinal", [](const Device& d) { return d.state()->ordinal; })
      .def_property_readonly("stream", [](const Device& d) { return reinterpret_cast<uint64_t>(d.state()->stream); })
      .def("synchronize", [](const Device& d) {
        py::gil_scoped_release nogil;
        d.synchronize();
      })
      .def("check", [](const Device& d) {
        // Without waiting: raises when an earlier failure poisoned the device, or when the stream
        // reports an error (a fault of work already finished); work still running is not waited for.
        d.state()->check();
        const cudaError_t e = cudaStreamQuery(d.state()->stream);
        if (e != cudaSuccess && e != cudaErrorNotReady) d.state()->check_cuda(e, "device health check");
      }, "Raises when the device failed, without waiting for the work in flight.");

  // ---------------------------------------------------------------- buffers / transfers
  py::class_<Transfer>(m, "Transfer", "A submitted copy between a HostBuffer and an HbmBuffer.")
      .def("done", &Transfer::done)
      .def("wait", [](const Transfer& t) {
        py::gil_scoped_release nogil;
        t.wait();
      });

  py::class_<HostBuffer>(m, "HostBuffer", py::buffer_protocol(),
                         "Page-locked host memory that copies read and write.")
      .def(py::init([](const py::object& source) {
             if (py::isinstance<py::int_>(source)) {
               const int64_t n = source.cast<int64_t>();
               if (n < 0) throw py::value_error("negative size");
               return HostBuffer(static_cast<size_t>(n));
             }
             if (!PyObject_CheckBuffer(source.ptr()))
               throw py::type_error("source is neither an integer nor a C-contiguous buffer");
             py::buffer_info info = py::buffer(source).request();
             Py_buffer view;
             if (PyObject_GetBuffer(source.ptr(), &view, PyBUF_C_CONTIGUOUS) != 0) {
               PyErr_Clear();
               throw py::type_error("source is not C-contiguous");
             }
             HostBuffer b(view.buf, static_cast<size_t>(view.len));
             PyBuffer_Release(&view);
             return b;
           }),
           py::arg("source"))
      .def("__len__", &HostBuffer::size)
      .def("slice", &HostBuffer::slice, py::arg("offset"), py::arg("size"))
      .def("to_hbm", &HostBuffer::to_hbm, py::arg("buffer"))
      .def_buffer([](HostBuffer& b) -> py::buffer_info {
        // Exporting waits for the copies already submitted on the bytes.
        if (auto t = b.last()) Transfer(t).wait();
        return py::buffer_info(b.data(), 1, py::format_descriptor<uint8_t>::format(), 1,
                               {static_cast<py::ssize_t>(b.size())}, {1});
      });

  py::class_<HbmBuffer>(m, "HbmBuffer", "Device memory of len bytes on each chip.")
      .def(py::init([](const Device& d, int64_t size) {
             if (size < 0) throw ValueError("negative size");
             return HbmBuffer(d, static_cast<size_t>(size));
           }),
           py::arg("device"), py::arg("size"))
      .def("__len__", &HbmBuffer::size)
      .def("slice", &HbmBuffer::slice, py::arg("offset"), py::arg("size"))
      .def("to_host", [](const HbmBuffer& b, const HostBuffer& h) { return copy_to_host(b, h); },
           py::arg("host"))
      .def_property_readonly("data_ptr", [](const HbmBuffer& b) { return reinterpret_cast<uint64_t>(b.data()); });

  // ---------------------------------------------------------------- tensors
  py::class_<HbmTensor, std::shared_ptr<HbmTensor>>(m, "HbmTensor",
                                                   "Dense row-major elements in an HbmBuffer.")
      .def(py::init([](const HbmBuffer& b, const std::vector<int64_t>& shape, const std::string& dtype) {
             return std::make_shared<HbmTensor>(b, shape, dtype_from_name(dtype));
           }),
           py::arg("buffer"), py::arg("shape"), py::arg("dtype"))
      .def_property_readonly("shape", &HbmTensor::shape)
      .def_property_readonly("dtype", [](const HbmTensor& t) { return std::string(dtype_name(t.dtype())); })
      .def_property_readonly("buffer", &HbmTensor::buffer)
      .def_property_readonly("data_ptr", [](const HbmTensor& t) { return reinterpret_cast<uint64_t>(t.buffer().data()); })
      .def("wait", [](const HbmTensor& t) {
        py::gil_scoped_release nogil;
        t.wait();
      })
      .def("to_host", [](const HbmTensor& t) {
        std::vector<uint8_t> bytes;
        {
          py::gil_scoped_release nogil;
          bytes = t.to_host_bytes();
        }
        return HostTensor(t.shape(), t.dtype(), bytes.data());
      })
      .def("__getitem__", [](const HbmTensor& t, const py::slice& s) {
        if (t.shape().empty()) throw ValueError("the tensor has no axes");
        py::ssize_t start, stop, step, len;
        if (!s.compute(static_cast<py::ssize_t>(t.shape()[0]), &start, &stop, &step, &len))
          throw py::error_already_set();
        if (step != 1) throw ValueError("the slice steps by other than one row");
        return std::make_shared<HbmTensor>(t.rows(start, std::max(start, stop)));
      });

  py::class_<HostTensor>(m, "HostTensor", "A host tensor, its contents copied on construction.")
      .def(py::init([](const py::object& values, const py::object& dtype) {
             py::object np = py::module_::import("numpy");
             py::object helper = py::module_::import("furiosa_opt_engine._host");
             py::tuple t = helper.attr("from_values")(values, dtype);
             std::vector<int64_t> shape = t[0].cast<std::vector<int64_t>>();
             std::string name = t[1].cast<std::string>();
             py::bytes raw = t[2];
             std::string s = raw;
             return HostTensor(shape, dtype_from_name(name), s.data());
           }),
           py::arg("values"), py::kw_only(), py::arg("dtype") = py::none())
      .def_static("empty", [](const std::vector<int64_t>& shape, const std::string& dtype) {
        return HostTensor(shape, dtype_from_name(dtype));
      }, py::arg("shape"), py::kw_only(), py::arg("dtype"))
      .def_static("from_dlpack", [](const py::object& value) {
        py::object helper = py::module_::import("furiosa_opt_engine._host");
        py::tuple t = helper.attr("from_dlpack")(value);
        std::vector<int64_t> shape = t[0].cast<std::vector<int64_t>>();
        std::string s = t[2].cast<py::bytes>();
        return HostTensor(shape, dtype_from_name(t[1].cast<std::string>()), s.data());
      }, py::arg("value"))
      .def_property_readonly("shape", &HostTensor::shape)
      .def_property_readonly("dtype", [](const HostTensor& t) { return std::string(dtype_name(t.dtype())); })
      .def("write", [](HostTensor& t, const py::bytes& b) {
        std::string s = b;
        t.write(s.data(), s.size());
      }, py::arg("bytes"))
      .def("numpy", [](const HostTensor& t) { return host_numpy(t.shape(), t.dtype(), t.data()); })
      .def("raw", [](const HostTensor& t) { return py::bytes(reinterpret_cast<const char*>(t.data()), t.nbytes()); })
      .def("to_hbm", [](const HostTensor& t, const Device& d) {
        py::gil_scoped_release nogil;
        return std::make_shared<HbmTensor>(t.to_hbm(d));
      }, py::arg("device"));

  // ---------------------------------------------------------------- decoder: cache
  py::class_<Pool>(decoder, "Pool", "A block format.")
      .def(py::init([](int64_t block, int64_t bytes) { return Pool{block, bytes}; }), py::arg("block"), py::arg("bytes"))
      .def_readonly("block", &Pool::block)
      .def_readonly("bytes", &Pool::bytes)
      .def("__eq__", [](const Pool& a, const Pool& b) { return a == b; })
      .def("__repr__", [](const Pool& p) {
        return "Pool(block=" + std::to_string(p.block) + ", bytes=" + std::to_string(p.bytes) + ")";
      });

  py::class_<PyKind> kind(decoder, "Kind", "What the blocks of a group hold.");
  py::class_<PyKindPaged, PyKind>(kind, "Paged", "Paged keys and values: each block caches a page of consecutive positions, read in the order of the request's block table.").def(py::init([]() { return PyKindPaged{{KindTag::Paged, 0}}; }))
      .def("__eq__", [](const PyKind& a, const py::object& o) {
        return py::isinstance<PyKindPaged>(o);
      });
  py::class_<PyKindState, PyKind>(kind, "State", "A recurrent state a block (not served by any decoder here).").def(py::init([]() { return PyKindState{{KindTag::State, 0}}; }))
      .def("__eq__", [](const PyKind& a, const py::object& o) { return py::isinstance<PyKindState>(o); });
  py::class_<PyKindCross, PyKind>(kind, "Cross", "Encoder keys and values: `length` positions that one call writes for every later call to read.")
      .def(py::init([](int64_t length) { return PyKindCross{{KindTag::Cross, length}}; }), py::arg("length"))
      .def_property_readonly("length", [](const PyKindCross& k) { return k.length; })
      .def("__eq__", [](const PyKind& a, const py::object& o) {
        return py::isinstance<PyKindCross>(o) && o.cast<const PyKind&>().length == a.length;
      });

  py::class_<Group>(decoder, "Group", "A set of layers sharing one cache kind and drawing blocks from one pool.")
      .def_readonly("pool", &Group::pool)
      .def_property_readonly("layers", [](const Group& g) { return make_range(g.layers_begin, g.layers_end); })
      .def_property_readonly("kind", [](const Group& g) -> py::object {
        switch (g.kind.tag) {
          case KindTag::Paged: return py::cast(PyKindPaged{{KindTag::Paged, 0}});
          case KindTag::State: return py::cast(PyKindState{{KindTag::State, 0}});
          default: return py::cast(PyKindCross{{KindTag::Cross, g.kind.length}});
        }
      })
      .def_property_readonly("window", [](const Group& g) -> py::object {
        return g.window ? py::cast(*g.window) : py::none();
      });

  py::class_<PyCacheSpec>(decoder, "CacheSpec", "The cache a loaded decoder's calls read.")
      .def_property_readonly("pools", [](const PyCacheSpec& s) { return s.spec.pools; })
      .def_property_readonly("groups", [](const PyCacheSpec& s) { return s.spec.groups; })
      .def("__eq__", [](const PyCacheSpec& a, const PyCacheSpec& b) { return a.spec == b.spec; });

  py::class_<PyCache>(decoder, "Cache", "The storage of a CacheSpec on the decoder's device.")
      .def(py::init([](const PyCacheSpec& spec, int64_t blocks) {
             LogsOnExit logs;
             if (blocks <= 0) throw ValueError("cache blocks must be positive");
             py::gil_scoped_release nogil;
             return PyCache{std::make_shared<Cache>(spec.device, spec.spec, blocks), spec.device};
           }),
           py::arg("spec"), py::arg("blocks"))
      .def_property_readonly("blocks", [](const PyCache& c) { return c.cache->blocks(); })
      .def_property_readonly("spec", [](const PyCache& c) { return PyCacheSpec{c.cache->spec(), c.device}; })
      .def_property_readonly("layers", [](const PyCache& c) { return c.cache->layers(); });

  // ---------------------------------------------------------------- decoder: requests
  py::enum_<PyKeep>(decoder, "Keep", "The appended rows of a request that a call returns.")
      .value("NONE", PyKeep::NONE)
      .value("LAST", PyKeep::LAST)
      .value("ALL", PyKeep::ALL);
  py::enum_<PyOutput>(decoder, "Output", "The output a decoder produces for each kept row: token, hidden row or scores.")
      .value("TOKENS", PyOutput::TOKENS)
      .value("HIDDEN", PyOutput::HIDDEN)
      .value("SCORES", PyOutput::SCORES);

  py::class_<PyAdapterSpec>(decoder, "AdapterSpec",
                            "Adapter limits of a loaded decoder: RANK (the LoRA rank of every update) and SLOTS (how "
                            "many adapters one call can use).")
      .def_property_readonly_static("RANK", [](py::object) { return LoraAdapter::kRank; })
      .def_property_readonly_static("SLOTS", [](py::object) { return LoraAdapter::kSlots; });
  py::class_<PyAdapter>(decoder, "Adapter",
                        "A PEFT LoRA checkpoint loaded onto a decoder's device: each adapted module's "
                        "lora_A and lora_B, the scale folded in.")
      .def(py::init([](const PyAdapterSpec& spec, const py::object& checkpoint) {
             auto ck = py::module_::import("furiosa_opt_engine._native").attr("_checkpoint_ptr")(checkpoint);
             const Checkpoint* c = reinterpret_cast<const Checkpoint*>(ck.cast<uintptr_t>());
             std::shared_ptr<const LoraAdapter> a;
             {
               py::gil_scoped_release nogil;
               a = std::make_shared<LoraAdapter>(*spec.model, *c);
             }
             return PyAdapter{a, spec.model};
           }),
           py::arg("spec"), py::arg("checkpoint"));
  py::class_<PyRequest>(decoder, "Request", "One sequence's tokens after the cached positions its blocks hold.")
      .def(py::init([](const std::vector<std::vector<int64_t>>& rows, int64_t cached,
                       std::shared_ptr<HbmTensor> tokens, const py::object& keep,
                       const py::object& adapter, const py::object& positions,
                       const py::object& mask, const py::object& overrides) {
             if (tokens->dtype() != DType::I32 || tokens->shape().size() != 1)
               throw ValueError("tokens are not one-dimensional I32 IDs");
             if (cached < 0) throw ValueError("cached positions are not negative");
             PyRequest r;
             r.rows = rows;
             r.cached = cached;
             r.tokens = tokens;
             r.keep_obj = keep;
             if (py::isinstance<PyKeep>(keep)) {
               switch (keep.cast<PyKeep>()) {
                 case PyKeep::NONE: r.keep.kind = KeepKind::None; break;
                 case PyKeep::LAST: r.keep.kind = KeepKind::Last; break;
                 case PyKeep::ALL: r.keep.kind = KeepKind::All; break;
               }
             } else {
               Range k = to_range(keep);
               if (k.step != 1 || k.start < 0 || k.stop < 0)
                 throw ValueError("keep is a range with a step other than 1 or a negative bound");
               r.keep = Keep{KeepKind::Range, k.start, k.stop};
             }
             if (!adapter.is_none()) r.adapter = adapter.cast<int64_t>();
             r.positions = positions;
             r.mask = mask;
             for (auto item : overrides) {
               py::tuple t = item.cast<py::tuple>();
               r.overrides.push_back({t[0].cast<int64_t>(), t[1]});
             }
             return r;
           }),
           py::arg("rows"), py::arg("cached"), py::arg("tokens"),
           py::arg("keep") = PyKeep::LAST, py::kw_only(), py::arg("adapter") = py::none(),
           py::arg("positions") = py::none(), py::arg("mask") = py::none(),
           py::arg("overrides") = py::list())
      .def_readonly("rows", &PyRequest::rows)
      .def_readonly("cached", &PyRequest::cached)
      .def_readonly("tokens", &PyRequest::tokens)
      .def_readonly("keep", &PyRequest::keep_obj)
      .def_readonly("adapter", &PyRequest::adapter)
      .def_readonly("positions", &PyRequest::positions)
      .def_readonly("mask", &PyRequest::mask)
      .def_property_readonly("overrides", [](const PyRequest& r) {
        py::list l;
        for (auto& o : r.overrides) l.append(py::make_tuple(o.first, o.second));
        return l;
      });

  // ---------------------------------------------------------------- decoders
  auto forward = [](PyDecoder& d, const std::vector<PyRequest*>& requests, PyCache& cache,
                    const py::object& adapters) {
    LogsOnExit logs;
    std::vector<Request> reqs;
    reqs.reserve(requests.size());
    for (const PyRequest* pr : requests) {
      Request r;
      r.rows = pr->rows;
      r.cached = pr->cached;
      r.tokens = pr->tokens->buffer();
      r.length = pr->tokens->shape()[0];
      if (pr->tokens->buffer().device() != d.model->device().state())
        throw ValueError("a tensor lies on another device");
      r.keep = pr->keep;
      r.adapter = pr->adapter;
      r.positions = !pr->positions.is_none();
      r.mask = !pr->mask.is_none();
      r.overrides = !pr->overrides.empty();
      reqs.push_back(std::move(r));
    }
    std::vector<std::shared_ptr<const LoraAdapter>> slots;
    if (!adapters.is_none() && py::len(adapters) > 0) {
      const Limits lim = d.model->limits();
      if (lim.adapters == 0) throw Unsupported("adapters are not served");
      if (static_cast<int64_t>(py::len(adapters)) > lim.adapters)
        throw ValueError("call holds more adapters than compiled");
      for (auto a : adapters) {
        if (a.is_none()) {
          slots.push_back(nullptr);
          continue;
        }
        const PyAdapter& pa = a.cast<const PyAdapter&>();
        if (pa.model != d.model) throw ValueError("the adapter belongs to another model");
        slots.push_back(pa.adapter);
      }
    }
    py::gil_scoped_release nogil;
    std::lock_guard<std::mutex> g(d.model->device().state()->mu);
    return std::make_shared<HbmTensor>(d.model->forward(reqs, *cache.cache, slots));
  };

  py::class_<PyDecoder>(m, "Decoder", "A decoder loaded on a device, whatever its model.")
      .def_property_readonly("size", [](const PyDecoder& d) { return d.size; })
      .def_property_readonly("precision", [](const PyDecoder& d) { return d.precision; })
      .def_property_readonly("parallel", [](const PyDecoder& d) { return d.parallel; })
      .def_property_readonly("kv_cache", [](const PyDecoder& d) { return d.kv_cache; })
      .def_property_readonly("cache", [](const PyDecoder& d) {
        return PyCacheSpec{d.model->limits().cache, d.model->device()};
      })
      .def_property_readonly("window", [](const PyDecoder& d) { return d.model->limits().window; })
      .def_property_readonly("rows", [](const PyDecoder& d) { return d.model->limits().rows; })
      .def_property_readonly("device", [](const PyDecoder& d) { return d.model->device(); })
      .def_property_readonly("output", [](const PyDecoder& d) {
        switch (d.model->config().output) {
          case Output::Hidden: return PyOutput::HIDDEN;
          case Output::Scores: return PyOutput::SCORES;
          default: return PyOutput::TOKENS;
        }
      })
      .def_property_readonly("adapters", [](const PyDecoder& d) -> py::object {
        if (d.model->limits().adapters == 0) return py::none();
        return py::cast(PyAdapterSpec{d.model});
      })
      .def("forward", forward, py::arg("requests"), py::arg("cache"), py::arg("adapters") = py::none())
      .def("set_graphs", [](PyDecoder& d, bool on) { d.model->set_graphs(on); })
      .def_property_readonly("weight_bytes", [](const PyDecoder& d) { return d.model->weight_bytes(); })
      .def_property_readonly("kernel_launches", [](const PyDecoder& d) { return d.model->kernel_launches(); })
      .def_property_readonly("program", [](const PyDecoder& d) { return d.model->describe(); },
                             "The decoder's launch program: its module tree, one line a module.")
      .def_property_readonly("last_staged_bytes", [](const PyDecoder& d) { return d.model->last_plan().staged.bytes; })
      .def("weight", [](const PyDecoder& d, const std::string& name) {
        const auto& w = d.model->weights().at(name);
        return py::make_tuple(reinterpret_cast<uint64_t>(w.ptr), w.shape);
      })
      .def("quantized_weight", [](const PyDecoder& d, const std::string& name) -> py::object {
        const auto& w = d.model->weights().at(name);
        if (w.format == 0) return py::none();
        py::dict q;
        q["format"] = w.format == foa::kWeightFp8A8     ? "fp8_block"
                      : w.format == foa::kWeightFp8Block ? "fp8_rows"
                      : w.format == foa::kWeightNvfp4    ? "nvfp4"
                                                         : "nvfp4_a4";
        q["codes"] = reinterpret_cast<uint64_t>(w.codes);
        q["scales"] = reinterpret_cast<uint64_t>(w.scales);
        q["scale_ld"] = w.scale_ld;
        q["tensor_scale"] = w.tensor_scale;
        q["input_scale"] = w.input_scale;
        q["shape"] = w.shape;
        return q;
      })
      .def("weight_names", [](const PyDecoder& d) {
        std::vector<std::string> n;
        for (auto& [k, v] : d.model->weights()) n.push_back(k);
        return n;
      })
      .def_property_readonly("geometry", [](const PyDecoder& d) {
        py::dict g;
        g["q_heads"] = d.model->q_heads_local();
        g["kv_heads"] = d.model->kv_heads_local();
        g["q_head_first"] = d.model->q_head_first();
        g["kv_head_first"] = d.model->kv_head_first();
        g["intermediate"] = d.model->intermediate_local();
        g["vocab_begin"] = d.model->vocab_begin();
        g["vocab_end"] = d.model->vocab_end();
        g["vocab_local"] = d.model->vocab_local();
        g["tp"] = d.model->tp();
        g["rank"] = d.model->rank();
        return g;
      });

  py::class_<PyQwen3ForCausalLM, PyDecoder>(qwen3, "ForCausalLM", "HF Qwen3ForCausalLM, loaded on a device.");
  py::class_<PyQwen3ForSequenceClassification, PyDecoder>(qwen3, "ForSequenceClassification",
                                                         "HF Qwen3ForSequenceClassification, loaded on a device.");
  py::class_<PyQwen3Model, PyDecoder>(qwen3, "Model", "HF Qwen3Model, loaded on a device.");
  py::class_<PyLlamaForCausalLM, PyDecoder>(llama, "ForCausalLM", "HF LlamaForCausalLM, loaded on a device.");
  py::class_<PyMistralForCausalLM, PyDecoder>(mistral, "ForCausalLM", "HF MistralForCausalLM, loaded on a device.");
  py::class_<PyQwen3MoeForCausalLM, PyDecoder>(qwen3_moe, "ForCausalLM",
                                               "HF Qwen3MoeForCausalLM, loaded on a device.");
  py::class_<PyMixtralForCausalLM, PyDecoder>(mixtral, "ForCausalLM", "HF MixtralForCausalLM, loaded on a device.");

  // Builds a decoder of `config` (a dict of geometry) with N(0, std) weights: synthetic models
  // of a named architecture for benchmarks and tests.
  m.def("_synthetic_decoder", [](const Device& device, const py::dict& config, int tp, int rank,
                                 uint64_t seed, float stdv, int adapters) -> py::object {
    ModelConfig cfg = model_config_from_dict(config);
    std::shared_ptr<DecoderModel> model;
    {
      py::gil_scoped_release nogil;
      model = std::make_shared<DecoderModel>(device, cfg, tp, rank);
      if (stdv > 0) model->init_random(seed, stdv);
      model->set_adapter_slots(adapters);
    }
    auto fill = [&](PyDecoder& d) {
      d.model = model;
      d.size = cfg.size;
      d.precision = cfg.precision;
      d.parallel = tp;
    };
    if (cfg.family == "llama") { PyLlamaForCausalLM d; fill(d); return py::cast(d); }
    if (cfg.family == "mistral") { PyMistralForCausalLM d; fill(d); return py::cast(d); }
    if (cfg.family == "qwen3_moe") { PyQwen3MoeForCausalLM d; fill(d); return py::cast(d); }
    if (cfg.family == "mixtral") { PyMixtralForCausalLM d; fill(d); return py::cast(d); }
    if (cfg.output == Output::Hidden) { PyQwen3Model d; fill(d); return py::cast(d); }
    if (cfg.output == Output::Scores) { PyQwen3ForSequenceClassification d; fill(d); return py::cast(d); }
    PyQwen3ForCausalLM d;
    fill(d);
    return py::cast(d);
  }, py::arg("device"), py::arg("config"), py::arg("tp") = 1, py::arg("rank") = 0,
     py::arg("seed") = 0, py::arg("std") = 0.02f, py::arg("adapters") = 0);

  m.def("_layout", [](const std::vector<int64_t>& lens) { return layout(lens); });

  // The batch planner without a device: requests as dicts, the model's limits and the cache's
  // spec as tuples. Raises the planner's refusals; returns the plan's host arrays.
  m.def("_plan", [](const py::list& requests, int64_t window, int64_t rows, int64_t adapters_limit,
                    const py::list& spec_pools, const py::list& spec_groups,
                    const py::list& cache_pools, const py::list& cache_groups, int64_t blocks,
                    int64_t adapters_given, const std::vector<bool>& filled, int group) {
    auto spec_of = [](const py::list& pools, const py::list& groups) {
      CacheSpec s;
      for (auto p : pools) {
        auto t = p.cast<py::tuple>();
        s.pools.push_back(Pool{t[0].cast<int64_t>(), t[1].cast<int64_t>()});
      }
      for (auto g : groups) {
        auto t = g.cast<py::tuple>();
        Group gr;
        gr.pool = t[0].cast<int64_t>();
        gr.layers_begin = t[1].cast<int64_t>();
        gr.layers_end = t[2].cast<int64_t>();
        const std::string kind = t[3].cast<std::string>();
        gr.kind.tag = kind == "paged" ? KindTag::Paged : kind == "state" ? KindTag::State : KindTag::Cross;
        gr.kind.length = t[4].cast<int64_t>();
        if (!t[5].is_none()) gr.window = t[5].cast<int64_t>();
        s.groups.push_back(gr);
      }
      return s;
    };
    Limits lim;
    lim.window = window;
    lim.rows = rows;
    lim.adapters = adapters_limit;
    lim.cache = spec_of(spec_pools, spec_groups);
    const CacheSpec cache_spec = spec_of(cache_pools, cache_groups);
    std::vector<Request> reqs;
    for (auto item : requests) {
      py::dict d = item.cast<py::dict>();
      Request r;
      r.rows = d["rows"].cast<std::vector<std::vector<int64_t>>>();
      r.cached = d["cached"].cast<int64_t>();
      r.length = d["length"].cast<int64_t>();
      py::object keep = d.contains("keep") ? py::object(d["keep"]) : py::str("last");
      if (py::isinstance<py::str>(keep)) {
        const std::string k = keep.cast<std::string>();
        r.keep.kind = k == "none" ? KeepKind::None : k == "all" ? KeepKind::All : KeepKind::Last;
      } else {
        auto t = keep.cast<py::tuple>();
        r.keep = Keep{KeepKind::Range, t[0].cast<int64_t>(), t[1].cast<int64_t>()};
      }
      if (d.contains("adapter") && !d["adapter"].is_none()) r.adapter = d["adapter"].cast<int64_t>();
      r.positions = d.contains("positions") && d["positions"].cast<bool>();
      r.mask = d.contains("mask") && d["mask"].cast<bool>();
      r.overrides = d.contains("overrides") && d["overrides"].cast<bool>();
      reqs.push_back(std::move(r));
    }
    std::vector<uint8_t> host;
    const Plan p = plan_call(reqs, lim, cache_spec, blocks, adapters_given, filled, group, 0, host);
    auto arr = [&](size_t off, int64_t n) {
      std::vector<int32_t> v(n);
      std::memcpy(v.data(), host.data() + off, n * 4);
      return v;
    };
    py::dict out;
    out["rows"] = p.rows;
    out["decode"] = p.decode;
    out["prefill"] = p.prefill;
    out["kept"] = p.kept_rows;
    out["positions"] = arr(p.staged.positions, p.rows);
    out["slots"] = arr(p.staged.slots, p.rows);
    out["segments"] = arr(p.staged.segments, 5 * (p.decode + p.prefill));
    out["work"] = arr(p.staged.work, 2 * p.work);
    out["staged_bytes"] = p.staged.bytes;
    return out;
  });

  // Tensor parallelism: a symmetric heap per rank, connected through CUDA IPC handles that the
  // ranks exchange over their process group.
  m.def("_tp_attach", [](PyDecoder& d, int world, int rank) {
    const auto& cfg = d.model->config();
    auto coll = std::make_shared<PeerCollectives>(d.model->device(), world, rank, cfg.rows,
                                                  cfg.hidden, cfg.rows,
                                                  cfg.experts > 0 ? d.model->moe_capacity(cfg.rows) : 0);
    d.model->set_collectives(coll);
    return py::bytes(coll->handle());
  });
  // Device time of layer 0's attention output projection on `rows` rows of `a` (BF16
  // [rows, q_heads_local * head_dim], a device address), in milliseconds per call over `iters`
  // calls on the decoder's stream (every rank calls it in lockstep):
  //   "fused": the GEMM pushing its FP32 partials to the reducing ranks over NVLink, then the
  //            tensor-parallel add+norm that sums them (the decoder's path);
  //   "local": the same GEMM writing its FP32 output to this rank's memory only.
  m.def("_tp_bench_o_proj", [](PyDecoder& d, int rows, uintptr_t a, int iters) {
    auto coll = d.model->collectives();
    if (!coll) throw ValueError("the decoder has no tensor-parallel heap");
    const auto& cfg = d.model->config();
    const WeightSlot& wo = d.model->weights().at("layers.0.o");
    if (wo.format != foa::kWeightBf16 || wo.shape.size() != 2) throw Unsupported("the benchmark takes BF16 weights");
    const int H = cfg.hidden, K = static_cast<int>(wo.shape[1]);
    auto st = d.model->device().state();
    py::gil_scoped_release nogil;
    st->activate();
    cudaStream_t s = st->stream;
    HbmBuffer out(d.model->device(), static_cast<size_t>(rows) * H * 4);
    HbmBuffer ws(d.model->device(), size_t{64} << 20);
    HbmBuffer counters(d.model->device(), 32768 * 4);
    unsigned long long* trace_gemm_ = nullptr;
    st->check_cuda(cudaMemsetAsync(counters.data(), 0, 32768 * 4, s), "counters");
    auto gemm = [&](float* partial) {
      foa::GemmArgs g;
      g.a = reinterpret_cast<const void*>(a);
      g.lda = K;
      g.w = wo.ptr;
      g.ldw = K;
      g.M = rows;
      g.N = H;
      g.K = K;
      g.c = partial ? static_cast<void*>(partial) : out.data();
      g.ldc = H;
      g.epilogue = foa::kEpiF32;
      g.workspace = static_cast<float*>(ws.data());
      g.workspace_bytes = ws.size();
      g.counters = static_cast<int*>(counters.data());
      g.counters_len = 32768;
      g.status = st->status;
      g.trace = trace_gemm_;
      if (foa::gemm_bf16(g, s) != 0) st->fail("benchmark gemm launch failed");
    };
    auto fused = [&]() {
      gemm(coll->partial_buffer());
      coll->add_norm(coll->residual_buffer(), d.model->weights().at("final_norm").ptr, cfg.eps,
                     coll->hidden_buffer(), rows, H, s);
    };
    auto timed = [&](const std::function<void()>& fn) {
      coll->begin_call(s);
      for (int i = 0; i < 3; ++i) fn();
      cudaEvent_t e0, e1;
      cudaEventCreate(&e0);
      cudaEventCreate(&e1);
      coll->begin_call(s);
      cudaEventRecord(e0, s);
      for (int i = 0; i < iters; ++i) fn();
      cudaEventRecord(e1, s);
      cudaEventSynchronize(e1);
      float ms = 0.f;
      cudaEventElapsedTime(&ms, e0, e1);
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
      st->check_status();
      return static_cast<double>(ms) / iters;
    };
    std::map<std::string, double> r;
    r["fused"] = timed(fused);
    r["local"] = timed([&]() { gemm(nullptr); });
    // The scatter and reducer alone on a partial already in place (the collective's own cost).
    r["collective"] = timed([&]() {
      coll->add_norm(coll->residual_buffer(), d.model->weights().at("final_norm").ptr, cfg.eps, coll->hidden_buffer(),
                     rows, H, s);
    });
    {
      // The fused pair again with an event between the GEMM and the collective: the GEMM's share
      // and the scatter + reducer's share (waits for peers included).
      std::vector<cudaEvent_t> ev(3 * iters);
      for (auto& e : ev) cudaEventCreate(&e);
      coll->begin_call(s);
      for (int i = 0; i < iters; ++i) {
        cudaEventRecord(ev[3 * i], s);
        gemm(coll->partial_buffer());
        cudaEventRecord(ev[3 * i + 1], s);
        coll->add_norm(coll->residual_buffer(), d.model->weights().at("final_norm").ptr, cfg.eps,
                       coll->hidden_buffer(), rows, H, s);
        cudaEventRecord(ev[3 * i + 2], s);
      }
      cudaEventSynchronize(ev.back());
      double g = 0, n = 0;
      for (int i = 0; i < iters; ++i) {
        float a0 = 0.f, a1 = 0.f;
        cudaEventElapsedTime(&a0, ev[3 * i], ev[3 * i + 1]);
        cudaEventElapsedTime(&a1, ev[3 * i + 1], ev[3 * i + 2]);
        g += a0;
        n += a1;
      }
      for (auto& e : ev) cudaEventDestroy(e);
      st->check_status();
      r["split_gemm"] = g / iters;
      r["split_norm"] = n / iters;
    }
    {
      // Milestones of one launch (global timer, relative to the GEMM's entry, microseconds): the
      // local GEMM, then the fused pair (GEMM marks 0-7, then the reducer's entry, barrier passed,
      // exit).
      auto* pc = dynamic_cast<PeerCollectives*>(coll.get());
      HbmBuffer tr(d.model->device(), 16 * 8);
      std::vector<unsigned long long> h(16);
      auto read = [&](const char* key, int n) {
        st->check_cuda(cudaMemcpyAsync(h.data(), tr.data(), 16 * 8, cudaMemcpyDeviceToHost, s), "trace");
        st->check_cuda(cudaStreamSynchronize(s), "trace");
        for (int i = 0; i < n; ++i)
          r[std::string(key) + std::to_string(i)] = h[i] ? (static_cast<double>(h[i]) - static_cast<double>(h[0])) / 1000.0 : -1.0;
      };
      coll->begin_call(s);
      st->check_cuda(cudaMemsetAsync(tr.data(), 0, 16 * 8, s), "trace");
      trace_gemm_ = static_cast<unsigned long long*>(tr.data());
      gemm(nullptr);
      trace_gemm_ = nullptr;
      read("trace_local_", 8);
      st->check_cuda(cudaMemsetAsync(tr.data(), 0, 16 * 8, s), "trace");
      if (pc) pc->set_trace(static_cast<unsigned long long*>(tr.data()) + 8);
      trace_gemm_ = static_cast<unsigned long long*>(tr.data());
      fused();
      trace_gemm_ = nullptr;
      if (pc) pc->set_trace(nullptr);
      read("trace_fused_", 11);
    }
    {
      auto* pc = dynamic_cast<PeerCollectives*>(coll.get());
      r["two_shot"] = pc != nullptr && pc->two_shot(rows) ? 1.0 : 0.0;
    }
    return r;
  });
  m.def("_device_trim", [](const Device& d) {
    py::gil_scoped_release nogil;
    return d.state()->trim();
  }, py::arg("device"), "Returns the device's cached free memory to the driver; the bytes freed.");
  m.def("_device_status", [](const Device& d) {
    return py::make_tuple(reinterpret_cast<uint64_t>(d.state()->status), reinterpret_cast<uint64_t>(d.state()->stream));
  }, py::arg("device"), "The device's kernel status word and stream (device addresses), for drills.");
  // Host-side fault drills (see DeviceState::injected): no GPU fault is made.
  m.def("_fault_inject", [](const Device& d, const std::string& kind, int64_t after) {
    if (kind != "launch" && kind != "copy" && kind != "peer" && kind != "")
      throw ValueError(kind + ": a fault is launch, copy or peer");
    d.state()->fault_kind = kind;
    d.state()->fault_countdown = kind.empty() ? -1 : after;
  }, py::arg("device"), py::arg("kind"), py::arg("after") = 0,
     "After `after` more events of `kind` the next one fails as the real failure would.");
  // Tracing (FURIOSA_OPT_PROFILE / FOA_PROFILE = info | debug | trace; see trace.h).
  m.def("_trace_level", []() {
    static const char* names[] = {"off", "info", "debug", "trace"};
    return std::string(names[static_cast<int>(trace_level())]);
  });
  m.def("_trace_set_level", [](const std::string& name) {
    if (name != "off" && parse_trace_level(name) == TraceLevel::Off)
      throw ValueError(name + ": a trace level is off, info, debug or trace");
    set_trace_level(parse_trace_level(name));
  }, py::arg("level"));
  m.def("_trace_now_ns", []() { return trace_now_ns(); });
  m.def("_trace_span", [](const std::string& name, const std::string& cat, uint64_t t0, uint64_t t1,
                          const std::string& args) {
    if (!args.empty() && (args.front() != '{' || args.back() != '}'))
      throw ValueError("_trace_span: args is a JSON object");
    Tracer::get().host_span(name, cat, t0, t1, args);
  }, py::arg("name"), py::arg("cat"), py::arg("t0_ns"), py::arg("t1_ns"), py::arg("args") = std::string(),
     "Adds a host span (the clock of _trace_now_ns) to the trace, for a framework's own phases; "
     "`args` is a JSON object written as the span's args.");
  m.def("_trace_flush", [](const std::string& path) {
    LogsOnExit logs;
    py::gil_scoped_release nogil;
    return Tracer::get().flush(path);
  }, py::arg("path") = std::string(),
     "Writes the spans so far as Chrome trace JSON (default: FURIOSA_OPT_OUT_DIR/trace-<pid>.json) "
     "and clears them; returns the path, or '' when there was nothing to write.");
  m.def("_log", [](int level, const std::string& message, int times) {
    LogsOnExit logs;
    for (int i = 0; i < times; ++i) log_event(static_cast<LogLevel>(level), message);
  }, py::arg("level"), py::arg("message"), py::arg("times") = 1,
     "Queues a record `times` times as engine code does (Python's level numbers); the records reach "
     "`logging` when this call returns.");
  m.def("_tp_connect", [](PyDecoder& d, const std::vector<py::bytes>& handles) {
    std::vector<std::string> hs;
    for (const auto& h : handles) hs.push_back(std::string(h));
    auto* coll = dynamic_cast<PeerCollectives*>(d.model->collectives().get());
    if (coll == nullptr) throw ValueError("the decoder has no tensor-parallel heap");
    py::gil_scoped_release nogil;
    coll->connect(hs);
  });
  m.def("_tp_barrier", [](PyDecoder& d) {
    auto* coll = dynamic_cast<PeerCollectives*>(d.model->collectives().get());
    if (coll == nullptr) return;
    py::gil_scoped_release nogil;
    coll->barrier(d.model->device().state()->stream);
    d.model->device().synchronize();
    d.model->device().state()->check_status();
  });
  // The reference's AllGather / Exchange of BF16 rows over the decoder's peer heap (between calls,
  // every rank in the same order): [rows, cols] -> [rows * world, cols] or [rows / world, cols * world].
  auto gather = [](PyDecoder& d, const HbmTensor& x, bool exchange) {
    auto* coll = dynamic_cast<PeerCollectives*>(d.model->collectives().get());
    if (coll == nullptr) throw ValueError("the decoder has no tensor-parallel collectives attached");
    if (x.dtype() != DType::BF16 || x.shape().size() != 2) throw ValueError("a two-dimensional BF16 tensor");
    const int rows = static_cast<int>(x.shape()[0]), cols = static_cast<int>(x.shape()[1]);
    const int world = coll->world();
    const std::vector<int64_t> shape = exchange ? std::vector<int64_t>{rows / world, static_cast<int64_t>(cols) * world}
                                                : std::vector<int64_t>{static_cast<int64_t>(rows) * world, cols};
    HbmBuffer out(d.model->device(), static_cast<size_t>(rows) * cols * world * 2);
    {
      py::gil_scoped_release nogil;
      auto st = d.model->device().state();
      st->activate();
      coll->gather_rows(static_cast<const __nv_bfloat16*>(x.buffer().data()), rows, cols, exchange,
                        static_cast<__nv_bfloat16*>(out.data()), st->stream);
    }
    return HbmTensor(out, shape, DType::BF16);
  };
  m.def("_tp_all_gather", [gather](PyDecoder& d, const HbmTensor& x) { return gather(d, x, false); },
        py::arg("decoder"), py::arg("rows"));
  m.def("_tp_exchange", [gather](PyDecoder& d, const HbmTensor& x) { return gather(d, x, true); },
        py::arg("decoder"), py::arg("rows"));
  m.def("_tp_detach", [](PyDecoder& d) {
    py::gil_scoped_release nogil;
    d.model->device().synchronize();
    d.model->set_collectives(nullptr);
  });

  bind_checkpoint_and_load(m);
}
