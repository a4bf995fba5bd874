// The host-thread emulation of the tensor-parallel all-reduce, for tests of its schedule on a CPU.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "engine/comm_emulate.h"

namespace py = pybind11;
namespace em = foa::engine::emulate;

namespace {

template <typename T>
std::vector<T> flat(const py::handle& obj, size_t want, const char* what) {
  auto a = py::array_t<T, py::array::c_style | py::array::forcecast>::ensure(obj);
  if (!a || static_cast<size_t>(a.size()) != want) throw py::value_error(std::string(what) + ": wrong size");
  return std::vector<T>(a.data(), a.data() + a.size());
}

py::array_t<uint16_t> rows_array(const std::vector<uint16_t>& v, int rows, int cols) {
  py::array_t<uint16_t> a({rows, cols});
  std::copy(v.begin(), v.end(), a.mutable_data());
  return a;
}

}  // namespace

void bind_emulate(py::module_& m) {
  m.def("_tp_emulate", [](int world, const py::list& calls, int slot_rows, long one_shot_bytes, int inline_rows,
                          double wait_limit_s, unsigned jitter_seed, int drop_rank) {
    std::vector<em::AllReduceCall> cs;
    for (const auto& item : calls) {
      const py::dict d = item.cast<py::dict>();
      em::AllReduceCall c;
      c.rows = d["rows"].cast<int>();
      c.cols = d["cols"].cast<int>();
      const size_t n = static_cast<size_t>(c.rows) * c.cols;
      for (const auto& p : d["partials"].cast<py::list>()) c.partials.push_back(flat<float>(p, n, "partials"));
      c.residual = flat<uint16_t>(d["residual"], n, "residual");
      c.weight = flat<uint16_t>(d["weight"], static_cast<size_t>(c.cols), "weight");
      if (d.contains("eps")) c.eps = d["eps"].cast<float>();
      if (d.contains("gather_residual")) c.gather_residual = d["gather_residual"].cast<bool>();
      cs.push_back(std::move(c));
    }
    em::AllReduceOptions o;
    o.slot_rows = slot_rows;
    o.one_shot_bytes = one_shot_bytes;
    o.inline_rows = inline_rows;
    o.wait_limit_s = wait_limit_s;
    o.jitter_seed = jitter_seed;
    o.drop_rank = drop_rank;
    em::AllReduceResult r;
    {
      py::gil_scoped_release nogil;
      r = em::all_reduce(world, cs, o);
    }
    py::list out;
    for (size_t i = 0; i < r.calls.size(); ++i) {
      py::list ranks;
      for (const auto& rk : r.calls[i])
        ranks.append(py::make_tuple(rows_array(rk.hidden, cs[i].rows, cs[i].cols),
                                    rows_array(rk.residual, cs[i].rows, cs[i].cols)));
      out.append(ranks);
    }
    py::dict result;
    result["calls"] = out;
    result["timeouts"] = r.timeouts;
    result["two_shot"] = r.two_shot;
    return result;
  }, py::arg("world"), py::arg("calls"), py::arg("slot_rows") = 0, py::arg("one_shot_bytes") = 4L << 20,
     py::arg("inline_rows") = 148, py::arg("wait_limit_s") = 2.0, py::arg("jitter_seed") = 0u,
     py::arg("drop_rank") = -1,
     "Runs tensor-parallel add+norm all-reduce calls on `world` host threads (one a rank) with the "
     "kernels' schedule; each call is a dict of rows, cols, partials ([world] FP32 [rows, cols]), "
     "residual and weight (BF16 bits), eps and gather_residual. Returns every rank's (hidden, "
     "residual) BF16 bits after each call, per-rank timeout counts and which calls went two-shot.");
}
