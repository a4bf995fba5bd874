// Raw launchers of the engine's kernels for Python: every tensor crosses as a device address and
// its strides, every launch as a CUDA stream handle. The engine's own model code calls the same
// launchers from C++; this surface exists so tests and tools can drive one kernel at a time.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "kernels/comm.cuh"
#include "kernels/gemm.cuh"
#include "kernels/ops.cuh"
#include "kernels/attention.cuh"
#include "kernels/quant.cuh"
#include "kernels/moe.cuh"

namespace py = pybind11;

namespace {

cudaStream_t as_stream(uint64_t s) { return reinterpret_cast<cudaStream_t>(s); }
template <class T>
T* as_ptr(uint64_t p) {
  return reinterpret_cast<T*>(p);
}

void check(int rc, const char* what) {
  if (rc != 0) throw std::runtime_error(std::string(what) + " launch rejected: code " + std::to_string(rc));
}

}  // namespace

void bind_ops(py::module_& m) {
  m.def(
      "gemm",
      [](uint64_t a, long lda, uint64_t w, long ldw, int M, int N, int K, uint64_t c, long ldc,
         uint64_t res, long ldr, int epilogue, int mode, int splits, uint64_t ws, size_t ws_bytes,
         uint64_t counters, int counters_len, uint64_t status, uint64_t stream, uint64_t trace,
         int w_format, uint64_t w_scale, long w_scale_ld, float w_tensor_scale, uint64_t a_scale,
         long a_scale_ld, uint64_t group_tiles, uint64_t tile_group, int group_tile, int groups,
         int w_scale_rows, const std::vector<std::tuple<uint64_t, long, uint64_t, long, int>>& segments,
         uint64_t cta_trace, int reduction, int debug) {
        foa::GemmArgs g;
        g.reduction = reduction;
        g.debug = debug;
        g.cta_trace = reinterpret_cast<unsigned long long*>(cta_trace);
        g.w_scale_rows = w_scale_rows;
        if (segments.size() > 2) throw std::runtime_error("gemm: at most two extra K segments");
        for (size_t i = 0; i < segments.size(); ++i) {
          const auto& [sa, slda, sw, sldw, sk] = segments[i];
          g.seg[i].a = as_ptr<void>(sa);
          g.seg[i].lda = slda;
          g.seg[i].w = as_ptr<void>(sw);
          g.seg[i].ldw = sldw;
          g.seg[i].K = sk;
        }
        g.group_tiles = as_ptr<const int>(group_tiles);
        g.tile_group = as_ptr<const int>(tile_group);
        g.group_tile = group_tile;
        g.groups = groups;
        g.a_scale = as_ptr<void>(a_scale);
        g.a_scale_ld = a_scale_ld;
        g.w_format = w_format;
        g.w_scale = as_ptr<void>(w_scale);
        g.w_scale_ld = w_scale_ld;
        g.w_tensor_scale = w_tensor_scale;
        g.trace = reinterpret_cast<unsigned long long*>(trace);
        g.a = as_ptr<void>(a);
        g.lda = lda;
        g.w = as_ptr<void>(w);
        g.ldw = ldw;
        g.M = M;
        g.N = N;
        g.K = K;
        g.c = as_ptr<void>(c);
        g.ldc = ldc;
        g.residual = as_ptr<void>(res);
        g.ldr = ldr;
        g.epilogue = epilogue;
        g.mode = mode;
        g.splits = splits;
        g.workspace = as_ptr<float>(ws);
        g.workspace_bytes = ws_bytes;
        g.counters = as_ptr<int>(counters);
        g.counters_len = counters_len;
        g.status = as_ptr<int>(status);
        py::gil_scoped_release nogil;
        check(foa::gemm_bf16(g, as_stream(stream)), "gemm");
      },
      py::arg("a"), py::arg("lda"), py::arg("w"), py::arg("ldw"), py::arg("M"), py::arg("N"),
      py::arg("K"), py::arg("c"), py::arg("ldc"), py::arg("res"), py::arg("ldr"),
      py::arg("epilogue"), py::arg("mode"), py::arg("splits"), py::arg("ws"),
      py::arg("ws_bytes"), py::arg("counters"), py::arg("counters_len"), py::arg("status"),
      py::arg("stream"), py::arg("trace") = 0, py::arg("w_format") = 0, py::arg("w_scale") = 0,
      py::arg("w_scale_ld") = 0, py::arg("w_tensor_scale") = 1.0f, py::arg("a_scale") = 0,
      py::arg("a_scale_ld") = 0, py::arg("group_tiles") = 0, py::arg("tile_group") = 0,
      py::arg("group_tile") = 0, py::arg("groups") = 0, py::arg("w_scale_rows") = 128,
      py::arg("segments") = std::vector<std::tuple<uint64_t, long, uint64_t, long, int>>{},
      py::arg("cta_trace") = 0, py::arg("reduction") = 0, py::arg("debug") = 0);

  m.def(
      "quantize_fp8_rows",
      [](uint64_t w, int rows, int cols, float tensor_amax, uint64_t codes, uint64_t scales, uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::quantize_fp8_rows(as_ptr<const __nv_bfloat16>(w), rows, cols, tensor_amax,
                                     as_ptr<uint8_t>(codes), as_ptr<float>(scales), as_stream(stream)),
              "quantize_fp8_rows");
      },
      py::arg("w"), py::arg("rows"), py::arg("cols"), py::arg("tensor_amax"), py::arg("codes"),
      py::arg("scales"), py::arg("stream"));

  m.def(
      "moe_route",
      [](uint64_t logits, long ld, int rows, int experts, int k, bool normalize, uint64_t ids,
         uint64_t weights, uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::moe_route(as_ptr<const __nv_bfloat16>(logits), ld, rows, experts, k, normalize,
                             as_ptr<int32_t>(ids), as_ptr<float>(weights), as_stream(stream)),
              "moe_route");
      },
      py::arg("logits"), py::arg("ld"), py::arg("rows"), py::arg("experts"), py::arg("k"),
      py::arg("normalize"), py::arg("ids"), py::arg("weights"), py::arg("stream"));
  m.def(
      "moe_align",
      [](uint64_t ids, int rows, int k, int experts, int first, int count, int tile, int capacity,
         uint64_t pos, uint64_t src, uint64_t tile_expert, uint64_t tiles, uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::moe_align(as_ptr<const int32_t>(ids), rows, k, experts, first, count, tile, capacity,
                             as_ptr<int32_t>(pos), as_ptr<int32_t>(src), as_ptr<int32_t>(tile_expert),
                             as_ptr<int32_t>(tiles), as_stream(stream)),
              "moe_align");
      },
      py::arg("ids"), py::arg("rows"), py::arg("k"), py::arg("experts"), py::arg("first"),
      py::arg("count"), py::arg("tile"), py::arg("capacity"), py::arg("pos"), py::arg("src"),
      py::arg("tile_expert"), py::arg("tiles"), py::arg("stream"));
  m.def(
      "moe_gather",
      [](uint64_t x, long ldx, uint64_t src, uint64_t tiles, int tile, int capacity, int cols,
         uint64_t out, uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::moe_gather(as_ptr<const __nv_bfloat16>(x), ldx, as_ptr<const int32_t>(src),
                              as_ptr<const int32_t>(tiles), tile, capacity, cols,
                              as_ptr<__nv_bfloat16>(out), as_stream(stream)),
              "moe_gather");
      },
      py::arg("x"), py::arg("ldx"), py::arg("src"), py::arg("tiles"), py::arg("tile"),
      py::arg("capacity"), py::arg("cols"), py::arg("out"), py::arg("stream"));
  m.def(
      "moe_combine",
      [](uint64_t y, long ldy, uint64_t pos, uint64_t weights, int rows, int k, int cols,
         uint64_t residual, long ldr, uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::moe_combine(as_ptr<const __nv_bfloat16>(y), ldy, as_ptr<const int32_t>(pos),
                               as_ptr<const float>(weights), rows, k, cols,
                               as_ptr<__nv_bfloat16>(residual), ldr, as_stream(stream)),
              "moe_combine");
      },
      py::arg("y"), py::arg("ldy"), py::arg("pos"), py::arg("weights"), py::arg("rows"),
      py::arg("k"), py::arg("cols"), py::arg("residual"), py::arg("ldr"), py::arg("stream"));

  m.def(
      "fp8_scales_pad4",
      [](uint64_t scales, long n, uint64_t padded, uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::fp8_scales_pad4(as_ptr<const float>(scales), n, as_ptr<float>(padded), as_stream(stream)),
              "fp8_scales_pad4");
      },
      py::arg("scales"), py::arg("n"), py::arg("padded"), py::arg("stream"));
  m.def(
      "quantize_fp8_act",
      [](uint64_t x, long ldx, int rows, int K, uint64_t codes, long ldc, uint64_t scales,
         int rows_pad, uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::quantize_fp8_act(as_ptr<const __nv_bfloat16>(x), ldx, rows, K,
                                    as_ptr<uint8_t>(codes), ldc, as_ptr<float>(scales), rows_pad,
                                    as_stream(stream)),
              "quantize_fp8_act");
      },
      py::arg("x"), py::arg("ldx"), py::arg("rows"), py::arg("K"), py::arg("codes"), py::arg("ldc"),
      py::arg("scales"), py::arg("rows_pad"), py::arg("stream"));

  m.def(
      "quantize_nvfp4_act",
      [](uint64_t x, long ldx, int rows, int K, float global, uint64_t codes, long ldc,
         uint64_t sf_atoms, uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::quantize_nvfp4_act(as_ptr<const __nv_bfloat16>(x), ldx, rows, K, global,
                                      as_ptr<uint8_t>(codes), ldc, as_ptr<uint8_t>(sf_atoms),
                                      as_stream(stream)),
              "quantize_nvfp4_act");
      },
      py::arg("x"), py::arg("ldx"), py::arg("rows"), py::arg("K"), py::arg("global_scale"),
      py::arg("codes"), py::arg("ldc"), py::arg("sf_atoms"), py::arg("stream"));
  m.def(
      "nvfp4_scale_atoms",
      [](uint64_t scales, long lds, int rows, int K, uint64_t sf_atoms, uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::nvfp4_scale_atoms(as_ptr<const uint8_t>(scales), lds, rows, K,
                                     as_ptr<uint8_t>(sf_atoms), as_stream(stream)),
              "nvfp4_scale_atoms");
      },
      py::arg("scales"), py::arg("lds"), py::arg("rows"), py::arg("K"), py::arg("sf_atoms"),
      py::arg("stream"));

  m.def(
      "quantize_fp8_block",
      [](uint64_t w, int rows, int cols, uint64_t codes, uint64_t scales, uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::quantize_fp8_block(as_ptr<const __nv_bfloat16>(w), rows, cols,
                                      as_ptr<uint8_t>(codes), as_ptr<float>(scales),
                                      as_stream(stream)),
              "quantize_fp8_block");
      },
      py::arg("w"), py::arg("rows"), py::arg("cols"), py::arg("codes"), py::arg("scales"),
      py::arg("stream"));
  m.def(
      "absmax",
      [](uint64_t x, long n, uint64_t out, uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::absmax_bf16(as_ptr<const __nv_bfloat16>(x), n, as_ptr<float>(out),
                               as_stream(stream)),
              "absmax");
      },
      py::arg("x"), py::arg("n"), py::arg("out"), py::arg("stream"));
  m.def(
      "quantize_nvfp4",
      [](uint64_t w, int rows, int cols, uint64_t codes, uint64_t scales, uint64_t amax,
         uint64_t tensor_scale, uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::quantize_nvfp4(as_ptr<const __nv_bfloat16>(w), rows, cols, as_ptr<uint8_t>(codes),
                                  as_ptr<uint8_t>(scales), as_ptr<const float>(amax),
                                  as_ptr<float>(tensor_scale), as_stream(stream)),
              "quantize_nvfp4");
      },
      py::arg("w"), py::arg("rows"), py::arg("cols"), py::arg("codes"), py::arg("scales"),
      py::arg("amax"), py::arg("tensor_scale"), py::arg("stream"));

  m.def(
      "gemm_scratch",
      [](int M, int N, int K, int epilogue, int mode, int splits) {
        foa::GemmArgs g;
        g.M = M;
        g.N = N;
        g.K = K;
        g.epilogue = epilogue;
        g.mode = mode;
        g.splits = splits;
        size_t bytes = 0;
        int counters = 0;
        foa::gemm_bf16_scratch(g, &bytes, &counters);
        return py::make_tuple(bytes, counters);
      },
      py::arg("M"), py::arg("N"), py::arg("K"), py::arg("epilogue"), py::arg("mode"),
      py::arg("splits"));

  m.def(
      "rmsnorm",
      [](uint64_t x, long ldx, uint64_t residual, long ldr, uint64_t weight, uint64_t out,
         long ldo, uint64_t residual_out, long ldro, int rows, int cols, float eps,
         uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::rmsnorm(as_ptr<const __nv_bfloat16>(x), ldx,
                           as_ptr<const __nv_bfloat16>(residual), ldr,
                           as_ptr<const __nv_bfloat16>(weight), as_ptr<__nv_bfloat16>(out), ldo,
                           as_ptr<__nv_bfloat16>(residual_out), ldro, rows, cols, eps,
                           as_stream(stream)),
              "rmsnorm");
      },
      py::arg("x"), py::arg("ldx"), py::arg("residual"), py::arg("ldr"), py::arg("weight"),
      py::arg("out"), py::arg("ldo"), py::arg("residual_out"), py::arg("ldro"), py::arg("rows"),
      py::arg("cols"), py::arg("eps"), py::arg("stream"));
  m.def(
      "embedding",
      [](uint64_t ids, uint64_t table, long ldt, int row_begin, int row_end, uint64_t out,
         long ldo, int rows, int cols, uint64_t stream) {
        py::gil_scoped_release nogil;
        check(foa::embedding(as_ptr<const int32_t>(ids), as_ptr<const __nv_bfloat16>(table), ldt,
                             row_begin, row_end, as_ptr<__nv_bfloat16>(out), ldo, rows, cols,
                             as_stream(stream)),
              "embedding");
      });

  m.def("argmax",
        [](uint64_t logits, long ld, int rows, int cols, int valid, int base, uint64_t idx,
           uint64_t val, uint64_t stream) {
          py::gil_scoped_release nogil;
          check(foa::argmax_rows(as_ptr<const float>(logits), ld, rows, cols, valid, base,
                                 as_ptr<int32_t>(idx), as_ptr<float>(val), as_stream(stream)),
                "argmax");
        });

  m.def("argmax_merge", [](uint64_t values, uint64_t indices, int ranks, int rows, uint64_t out,
                           uint64_t stream) {
    py::gil_scoped_release nogil;
    check(foa::argmax_merge(as_ptr<const float>(values), as_ptr<const int32_t>(indices), ranks,
                            rows, as_ptr<int32_t>(out), as_stream(stream)),
          "argmax_merge");
  });

  m.def("qk_norm_rope_cache",
        [](uint64_t qkv, long ld_qkv, int rows, int q_heads, int kv_heads, int head_dim,
           uint64_t q_norm, uint64_t k_norm, float eps, uint64_t positions, uint64_t inv_freq,
           float attention_factor, uint64_t q_out, uint64_t cache, uint64_t slots,
           uint64_t stream, long cache_slots, uint64_t status) {
          py::gil_scoped_release nogil;
          foa::RopeTable rope{as_ptr<const float>(inv_freq), attention_factor};
          check(foa::qk_norm_rope_cache(
                    as_ptr<const __nv_bfloat16>(qkv), ld_qkv, rows, q_heads, kv_heads, head_dim,
                    as_ptr<const __nv_bfloat16>(q_norm), as_ptr<const __nv_bfloat16>(k_norm), eps,
                    as_ptr<const int32_t>(positions), rope, as_ptr<__nv_bfloat16>(q_out),
                    as_ptr<__nv_bfloat16>(cache), as_ptr<const int32_t>(slots),
                    as_stream(stream), cache_slots, as_ptr<int>(status)),
                "qk_norm_rope_cache");
        },
        py::arg("qkv"), py::arg("ld_qkv"), py::arg("rows"), py::arg("q_heads"), py::arg("kv_heads"),
        py::arg("head_dim"), py::arg("q_norm"), py::arg("k_norm"), py::arg("eps"), py::arg("positions"),
        py::arg("inv_freq"), py::arg("attention_factor"), py::arg("q_out"), py::arg("cache"),
        py::arg("slots"), py::arg("stream"), py::arg("cache_slots") = 0, py::arg("status") = 0);
  auto make_attn = [](uint64_t q, uint64_t o, uint64_t cache, uint64_t table, uint64_t segments,
                      int num_segments, int q_heads, int kv_heads, int head_dim, float scale,
                      uint64_t partial_o, uint64_t partial_lse, size_t capacity, int max_keys,
                      int keys_per_split, uint64_t status) {
    foa::PagedAttention a;
    a.q = as_ptr<const __nv_bfloat16>(q);
    a.o = as_ptr<__nv_bfloat16>(o);
    a.cache = as_ptr<const __nv_bfloat16>(cache);
    a.table = as_ptr<const int32_t>(table);
    a.segments = as_ptr<const foa::Segment>(segments);
    a.num_segments = num_segments;
    a.q_heads = q_heads;
    a.kv_heads = kv_heads;
    a.head_dim = head_dim;
    a.scale = scale;
    a.partial_o = as_ptr<float>(partial_o);
    a.partial_lse = as_ptr<float>(partial_lse);
    a.partial_capacity = capacity;
    a.max_keys = max_keys;
    a.keys_per_split = keys_per_split;
    a.status = as_ptr<int>(status);
    return a;
  };
  m.def("paged_decode",
        [make_attn](uint64_t q, uint64_t o, uint64_t cache, uint64_t table, uint64_t segments,
                    int num_segments, int q_heads, int kv_heads, int head_dim, float scale,
                    uint64_t partial_o, uint64_t partial_lse, size_t capacity, int max_keys,
                    int keys_per_split, uint64_t status, uint64_t stream, uint64_t counters, int warps,
                    int stages, long cache_blocks) {
          auto a = make_attn(q, o, cache, table, segments, num_segments, q_heads, kv_heads,
                             head_dim, scale, partial_o, partial_lse, capacity, max_keys,
                             keys_per_split, status);
          a.cache_blocks = cache_blocks;
          a.decode_warps = warps;
          a.decode_stages = stages;
          a.merge_counters = as_ptr<int>(counters);
          py::gil_scoped_release nogil;
          check(foa::paged_decode(a, as_stream(stream)), "paged_decode");
        },
        py::arg("q"), py::arg("o"), py::arg("cache"), py::arg("table"), py::arg("segments"),
        py::arg("num_segments"), py::arg("q_heads"), py::arg("kv_heads"), py::arg("head_dim"),
        py::arg("scale"), py::arg("partial_o"), py::arg("partial_lse"), py::arg("capacity"),
        py::arg("max_keys"), py::arg("keys_per_split"), py::arg("status"), py::arg("stream"),
        py::arg("counters") = 0, py::arg("warps") = 0, py::arg("stages") = 0, py::arg("cache_blocks") = 0);
  m.def("wait_probe",
        [](uint64_t flag, unsigned long long value, uint64_t limit_ns, uint64_t status, uint64_t stream) {
          check(foa::wait_probe(as_ptr<const unsigned long long>(flag), value, limit_ns, as_ptr<int>(status),
                                as_stream(stream)),
                "wait_probe");
        },
        py::arg("flag"), py::arg("value"), py::arg("limit_ns"), py::arg("status"), py::arg("stream"),
        "A bounded wait on a device flag (the peers' wait) with its own limit; the status word gets "
        "the peer-timeout code when it gives up.");
  m.def("paged_prefill",
        [make_attn](uint64_t q, uint64_t o, uint64_t cache, uint64_t table, uint64_t segments,
                    int num_segments, int q_heads, int kv_heads, int head_dim, float scale,
                    uint64_t work, int num_work, uint64_t status, uint64_t stream, int rows,
                    long cache_blocks, bool bidirectional) {
          auto a = make_attn(q, o, cache, table, segments, num_segments, q_heads, kv_heads,
                             head_dim, scale, 0, 0, 0, 1, 512, status);
          a.rows = rows;
          a.cache_blocks = cache_blocks;
          a.bidirectional = bidirectional ? 1 : 0;
          py::gil_scoped_release nogil;
          check(foa::paged_prefill(a, as_ptr<const int32_t>(work), num_work, as_stream(stream)),
                "paged_prefill");
        },
        py::arg("q"), py::arg("o"), py::arg("cache"), py::arg("table"), py::arg("segments"),
        py::arg("num_segments"), py::arg("q_heads"), py::arg("kv_heads"), py::arg("head_dim"),
        py::arg("scale"), py::arg("work"), py::arg("num_work"), py::arg("status"), py::arg("stream"),
        py::arg("rows") = 0, py::arg("cache_blocks") = 0, py::arg("bidirectional") = false);
}
