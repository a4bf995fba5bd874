// Checkpoints and load options: the choices of a load, checked against the registry before any
// weight is read, and the strict load into device memory.
#include <pybind11/pybind11.h>

#include <chrono>

#include "engine/lora.h"
#include <pybind11/stl.h>

#include "engine/catalog.h"
#include "engine/checkpoint.h"
#include "engine/encoder.h"
#include "engine/registry.h"
#include "engine/trace.h"
#include "python/pytypes.h"

namespace py = pybind11;
using namespace foa::engine;

namespace {

Json to_json(const py::object& o) {
  const std::string text = py::module_::import("json").attr("dumps")(o).cast<std::string>();
  return Json::parse(text);
}

py::object from_json(const Json& j) {
  return py::module_::import("json").attr("loads")(j.dump());
}

struct PyCheckpoint {
  std::shared_ptr<Checkpoint> ck;
};

py::object make_decoder(const Selection& s, std::shared_ptr<DecoderModel> model, bool invariant) {
  auto fill = [&](PyDecoder& d) {
    d.model = model;
    d.size = s.config.size;
    d.precision = s.config.precision;
    d.parallel = s.chips;
    d.batch_invariant = invariant;
  };
  const std::string& cls = s.implementation->cls;
  if (cls == "qwen3.ForSequenceClassification") {
    PyQwen3ForSequenceClassification d;
    fill(d);
    return py::cast(d);
  }
  if (cls == "qwen3.Model") {
    PyQwen3Model d;
    fill(d);
    return py::cast(d);
  }
  if (cls == "llama.ForCausalLM") {
    PyLlamaForCausalLM d;
    fill(d);
    return py::cast(d);
  }
  if (cls == "mistral.ForCausalLM") {
    PyMistralForCausalLM d;
    fill(d);
    return py::cast(d);
  }
  if (cls == "qwen3_moe.ForCausalLM") {
    PyQwen3MoeForCausalLM d;
    fill(d);
    return py::cast(d);
  }
  if (cls == "mixtral.ForCausalLM") {
    PyMixtralForCausalLM d;
    fill(d);
    return py::cast(d);
  }
  PyQwen3ForCausalLM d;
  fill(d);
  return py::cast(d);
}

}  // namespace

void bind_checkpoint_and_load(py::module_& m) {
  py::class_<PyCheckpoint>(m, "Checkpoint",
                           "A checkpoint directory: its model config and its tensors, memory-mapped or copied into "
                           "host memory.")
      .def(py::init([](const py::object& path, const py::object& config) {
             const std::string p = py::str(py::module_::import("os").attr("fspath")(path));
             std::optional<Json> cfg;
             if (!config.is_none()) cfg = to_json(config);
             LogsOnExit logs;
             auto ck = [&] {
               py::gil_scoped_release nogil;
               return std::make_shared<Checkpoint>(Checkpoint::open(p, cfg ? &*cfg : nullptr));
             }();
             log_event(LogLevel::Debug, p + ": " + std::to_string(ck->tensors().size()) + " tensors");
             return PyCheckpoint{ck};
           }),
           py::arg("path"), py::arg("config") = py::none())
      .def("read", [](const PyCheckpoint& c) {
        py::gil_scoped_release nogil;
        return PyCheckpoint{std::make_shared<Checkpoint>(c.ck->read())};
      })
      .def_property_readonly("config", [](const PyCheckpoint& c) { return from_json(c.ck->config()); })
      .def("names", [](const PyCheckpoint& c) { return c.ck->names(); })
      .def_static("declared", [](const py::object& path, const py::object& config) {
        const std::string p = py::str(py::module_::import("os").attr("fspath")(path));
        std::optional<Json> cfg;
        if (!config.is_none()) cfg = to_json(config);
        return PyCheckpoint{std::make_shared<Checkpoint>(Checkpoint::open(p, cfg ? &*cfg : nullptr, true))};
      }, py::arg("path"), py::arg("config") = py::none());

  py::class_<LoadOptions>(m, "LoadOptions",
                          "A load's architecture, chips, KV cache form, layers, batch invariance, "
                          "quantization and LoRA adapters.")
      .def(py::init<>())
      .def("chips", [](const LoadOptions& o, int64_t chips) {
        if (chips <= 0) throw ValueError("chips: a model loads onto at least one chip");
        LoadOptions n = o;
        n.chips = static_cast<int>(chips);
        return n;
      }, py::arg("chips"))
      .def("kv_cache", [](const LoadOptions& o, const std::string& dtype) {
        dtype_from_name(dtype);
        LoadOptions n = o;
        n.kv_cache = dtype;
        return n;
      }, py::arg("dtype"))
      .def("architecture", [](const LoadOptions& o, const std::string& name) {
        const Listed l = listed({name});
        LoadOptions n = o;
        n.architecture = l.name;
        return n;
      }, py::arg("name"))
      .def("layers", [](const LoadOptions& o, const py::object& r) {
        const int64_t start = r.attr("start").cast<int64_t>(), stop = r.attr("stop").cast<int64_t>(),
                      step = r.attr("step").cast<int64_t>();
        if (step != 1 || start < 0 || stop < 0)
          throw ValueError("layers: a range of step 1 with non-negative bounds");
        LoadOptions n = o;
        n.layers = std::make_pair(start, stop);
        return n;
      }, py::arg("layers"))
      .def("batch_invariant", [](const LoadOptions& o) {
        LoadOptions n = o;
        n.batch_invariant = true;
        return n;
      })
      .def("quantization", [](const LoadOptions& o, const std::string& name) {
        if (name != "fp8_per_tensor" && name != "fp8_per_channel")
          throw ValueError(name + ": a quantization is fp8_per_tensor or fp8_per_channel");
        LoadOptions n = o;
        n.quantization = name;
        return n;
      }, py::arg("name"))
      .def("encoder", [](const LoadOptions& o) {
        LoadOptions n = o;
        n.encoder = true;
        return n;
      })
      .def("adapters", [](const LoadOptions& o) {
        LoadOptions n = o;
        n.adapters = true;
        return n;
      })
      .def("parse", [](const LoadOptions& o, const PyCheckpoint& c) {
        select(o, *c.ck);
      }, py::arg("checkpoint"))
      .def("select", [](const LoadOptions& o, const PyCheckpoint& c) {
        const Selection s = select(o, *c.ck);
        py::dict d;
        d["architecture"] = s.architecture;
        d["class"] = s.implementation->cls;
        d["size"] = s.config.size;
        d["precision"] = s.config.precision;
        d["chips"] = s.chips;
        return d;
      }, py::arg("checkpoint"))
      .def("load", [](const LoadOptions& o, const PyCheckpoint& c, const Device& device) -> py::object {
        LogsOnExit logs;
        const auto t0 = std::chrono::steady_clock::now();
        const Selection s = select(o, *c.ck);
        if (device.chips() != s.chips)
          throw ValueError("the device opens " + std::to_string(device.chips()) + " chips, the load " +
                           std::to_string(s.chips));
        if (s.implementation->family == "gemma4_unified") {
          PyEncoder e;
          {
            py::gil_scoped_release nogil;
            e.encoder = std::make_shared<MediaEncoder>(device, encoder_config(*c.ck));
            e.encoder->load(*c.ck);
          }
          return py::cast(std::move(e));
        }
        std::shared_ptr<DecoderModel> model;
        {
          py::gil_scoped_release nogil;
          model = std::make_shared<DecoderModel>(device, s.config, s.chips, device.state()->rank);
          load_weights(*model, *c.ck);
          model->set_batch_invariant(o.batch_invariant);
          if (o.adapters) model->set_adapter_slots(LoraAdapter::kSlots);
        }
        py::object decoder = make_decoder(s, model, o.batch_invariant);
        if (s.chips > 1)
          py::module_::import("furiosa_opt_models_b200.parallel.tp").attr("attach")(decoder, device);
        const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        log_event(LogLevel::Info, s.architecture + " loaded on " + std::to_string(s.chips) + " GPU(s) from " +
                                      c.ck->directory() + " in " + std::to_string(secs).substr(0, 5) + " s" +
                                      (o.batch_invariant ? " (batch invariant)" : ""));
        return decoder;
      }, py::arg("checkpoint"), py::arg("device"));

  m.def("_architectures", []() { return architecture_names(); });
  m.def("_catalog_composes", [](const std::string& architecture) { return catalog::composes(architecture); });
  m.def("_catalog_architectures", []() { return catalog::architectures(); });
  // The catalog composition of a checkpoint's config (family, module tree, weights and optional
  // weights by name and shape, ignored names), checked strictly against its tensors when `check`.
  m.def("_catalog", [](const PyCheckpoint& c, bool check) {
    const catalog::Composition comp = catalog::compose(*c.ck);
    if (check) catalog::check(comp, *c.ck);
    auto table = [](const std::vector<catalog::Weight>& ws) {
      py::dict d;
      for (const auto& w : ws) d[py::str(w.name)] = py::tuple(py::cast(w.shape));
      return d;
    };
    py::dict out;
    out["family"] = comp.family;
    out["architecture"] = comp.architecture;
    out["tree"] = comp.tree;
    out["weights"] = table(comp.weights);
    out["optional"] = table(comp.optional);
    out["ignored"] = comp.ignored;
    return out;
  }, py::arg("checkpoint"), py::arg("check") = true);
  // The native checkpoint behind a Checkpoint object (for the engine's own classes).
  m.def("_checkpoint_ptr", [](const PyCheckpoint& c) { return reinterpret_cast<uintptr_t>(c.ck.get()); });
}
