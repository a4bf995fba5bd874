// Decoder models on one GPU (one rank of a tensor-parallel group): weights, workspace, and the
// launch sequence of one call, captured into CUDA graphs for decode steps.
//
// The reference composes each decoder from Rust module trees scheduled on its NPU
// (crates/furiosa-opt-models/src/schedule/decoder/mod.rs:398-510, models/decoder/attention/
// qwen3/launch.rs:60-70). Here a call is a fixed sequence of sm_100a kernels per layer:
//   RMSNorm -> packed q/k/v GEMM -> QK-norm + RoPE + paged KV write -> paged attention ->
//   o_proj GEMM (+ residual, or + fused reduce-scatter/all-reduce + residual + RMSNorm across
//   ranks) -> RMSNorm -> gate/up GEMM with SwiGLU epilogue -> down GEMM (+ residual / fused
//   collective) -> next RMSNorm,
// then the kept rows' vocabulary head with a first-maximum argmax.
#pragma once

#include <cuda_bf16.h>

#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "batch.h"
#include "kernels/gemm.cuh"
#include "runtime.h"

namespace foa::engine {

struct RopeSpec {
  std::string type = "default";  // default | linear | llama3 | yarn
  double theta = 10000.0;
  double factor = 1.0;
  double low_freq_factor = 1.0, high_freq_factor = 4.0;  // llama3
  double original_max_positions = 0;                     // llama3 / yarn
  double beta_fast = 32.0, beta_slow = 1.0;              // yarn
  double mscale = 1.0, mscale_all_dim = 0.0;             // yarn
  double attention_factor = 0.0;                         // yarn; 0 derives it
  bool truncate = true;                                  // yarn
};

// Inverse frequencies of the rotated pairs (FP64 on the host, uploaded as FP32) and the factor
// cos/sin are scaled by.
std::vector<float> rope_inv_freq(const RopeSpec& rope, int head_dim, float* attention_factor);

enum class Output { Tokens = 0, Hidden = 1, Scores = 2 };

struct ModelConfig {
  std::string architecture, family, size, precision = "bfloat16";
  // Weight format of the q/k/v, o, gate/up and down projections: "bf16"; "fp8_block" (E4M3 with an
  // FP32 scale per 128x128 block, W8A8); "nvfp4" (E2M1 with E4M3 scales per 16 and an FP32 tensor
  // scale, BF16 inputs: W4A16); "nvfp4_a4" (the same weights, NVFP4 inputs under input_scale:
  // W4A4 on the block-scaled MMA); "fp8_channel" / "fp8_tensor" (BF16 weights quantized at load
  // to E4M3 with one FP32 scale per output row, or per tensor, restored to BF16 in the GEMM: W8A16).
  std::string weight_format = "bf16";
  int hidden = 0, intermediate = 0, layers = 0, q_heads = 0, kv_heads = 0, head_dim = 128;
  int vocab = 0;
  float eps = 1e-6f;
  bool qk_norm = false, tied = false;
  RopeSpec rope;
  int window = 0;   // positions a request reaches at most
  int rows = 8192;  // rows of one call at most
  Output output = Output::Tokens;
  int labels = 0;   // score head rows (sequence classification)
  // Mixture of experts (0 experts: dense)
  int experts = 0, top_k = 0, expert_intermediate = 0;
  bool norm_topk = true;
};

// Tensor-parallel collectives a model's launches need; implemented over NVLink peer memory.
class Collectives {
 public:
  virtual ~Collectives() = default;
  virtual int rank() const = 0;
  virtual int world() const = 0;
  // Where a row-parallel GEMM writes its FP32 partial [rows, cols] (row stride cols) ahead of the
  // add_norm of the same shape.
  virtual float* partial_buffer() = 0;
  // Sums every rank's FP32 partial [rows, cols] (written to partial_buffer) in rank order, adds
  // the BF16 residual (updated in place, rounded once) and writes RMSNorm(residual) * weight to
  // `out` on every rank. Returns the kernels it launched: the reducer, which scatters the partial
  // itself in small calls, or the partial's scatter to the peers and then the reducer. `splits`
  // (small calls only, see inline_scatter): the partial is the sum of a GEMM's K splits left in
  // its workspace, added in split order by the reducer as it scatters them.
  virtual int add_norm(__nv_bfloat16* residual, const __nv_bfloat16* weight, float eps,
                       __nv_bfloat16* out, int rows, int cols, cudaStream_t stream,
                       const foa::GemmSplits* splits = nullptr) = 0;
  // Whether add_norm of `rows` rows scatters the partial from the reducer itself (and so may take
  // a GEMM's K splits in place of the partial).
  virtual bool inline_scatter(int rows) const = 0;
  // The first maximum over ranks of (value, token) candidates [rows]: tokens into `out`.
  virtual void argmax(const float* value, const int32_t* index, int rows, int32_t* out,
                      cudaStream_t stream) = 0;
  // The residual stream and the normed rows, in memory every rank can write.
  virtual __nv_bfloat16* residual_buffer() = 0;
  virtual __nv_bfloat16* hidden_buffer() = 0;
  // Marks the start of a call (before its launches or its graph launch, on the call's stream).
  virtual void begin_call(cudaStream_t stream) = 0;
  // Expert parallelism: this rank's expert-row buffer `which` (0 or 1, alternating by layer) of
  // the symmetric heap, and the combine that reads every rank's rows after a barrier, adds the
  // weighted sum to the residual and writes the next RMSNorm's rows (moe_combine_norm contract).
  virtual __nv_bfloat16* moe_rows(int which, size_t rows) = 0;
  virtual void moe_combine_norm(int which, const int32_t* pos_all, const int32_t* ids,
                                const float* weights, int experts_local, const __nv_bfloat16* norm,
                                float eps, int rows, int k, int cols, cudaStream_t stream) = 0;
};

struct WeightSlot {
  __nv_bfloat16* ptr = nullptr;  // BF16 weights (null for a quantized projection)
  std::vector<int64_t> shape;    // this rank's logical shape
  // A quantized projection (foa::GemmWeightFormat != 0): codes and block scales.
  int format = 0;
  uint8_t* codes = nullptr;      // E4M3 [rows, cols] or packed E2M1 [rows, cols/2]
  void* scales = nullptr;        // FP8: FP32 [ceil(rows/128), scale_ld]; W4A16: E4M3 [rows, cols/16];
                                 // W4A4: 128-row-blocked atoms [ceil(rows/128), cols/64, 512]
  long scale_ld = 0;
  int scale_rows = 128;          // FP8 W8A16: rows one scale covers (128: block scales, 1: per row)
  float tensor_scale = 1.f;      // NVFP4 weight_scale_2
  float input_scale = 1.f;       // W4A4 input_scale
};

class LoraAdapter;
class Module;
struct Launch;
struct DecoderBlocks;

class DecoderModel {
 public:
  DecoderModel(const Device& device, ModelConfig cfg, int tp, int rank);
  ~DecoderModel();
  const ModelConfig& config() const { return cfg_; }
  Limits limits() const;
  int tp() const { return tp_; }
  int rank() const { return rank_; }
  const Device& device() const { return device_; }

  // Weight slots by engine name ("embed", "layers.3.qkv", ...), this rank's shard.
  const std::map<std::string, WeightSlot>& weights() const { return weights_; }
  // A slot to fill (checkpoint loading sets the scales of quantized projections).
  WeightSlot& weight_slot(const std::string& name) { return weights_.at(name); }
  // Fills every weight with N(0, std) (norm weights with 1) from `seed`.
  void init_random(uint64_t seed, float std);
  size_t weight_bytes() const { return arena_bytes_; }

  // Rank geometry.
  int q_heads_local() const { return qh_l_; }
  int kv_heads_local() const { return kvh_l_; }
  int kv_head_first() const { return kvh_first_; }
  int q_head_first() const { return qh_first_; }
  int intermediate_local() const { return inter_l_; }
  int experts_local() const { return experts_l_; }
  int expert_first() const { return expert_first_; }
  // Expert rows of a call of `rows` rows (the grouped GEMM's sorted buffer, padded per expert).
  int64_t moe_capacity(int64_t rows) const;
  int moe_tile(int64_t rows) const;
  int vocab_begin() const { return vocab_begin_; }
  int vocab_end() const { return vocab_end_; }
  int vocab_local() const { return vocab_l_; }

  void set_collectives(std::shared_ptr<Collectives> c) {
    coll_ = std::move(c);
    clear_graphs();
  }
  const std::shared_ptr<Collectives>& collectives() const { return coll_; }
  void set_graphs(bool enabled) { graphs_enabled_ = enabled; }
  // Batch-invariant calls: every projection uses one tiling and one K order whatever the call's
  // row count (no split-K, one operand mapping), and attention tiles each row by its own history.
  void set_batch_invariant(bool on) {
    batch_invariant_ = on;
    clear_graphs();
  }
  bool batch_invariant() const { return batch_invariant_; }

  // One call: plans, stages and launches; returns the kept rows' output (tokens I32 [kept],
  // hidden BF16 [kept, hidden] or scores F32 [kept, labels]) once the launches are submitted.
  HbmTensor forward(const std::vector<Request>& requests, Cache& cache,
                    const std::vector<std::shared_ptr<const LoraAdapter>>& adapters = {});
  // LoRA slots a call may hold (0: the decoder runs no adapter).
  void set_adapter_slots(int slots) {
    adapter_slots_ = slots;
    clear_graphs();
  }

  // Timing hooks for benchmarks: the last call's plan, and the kernels launched so far (graph
  // replays count every kernel node).
  const Plan& last_plan() const { return last_plan_; }
  uint64_t kernel_launches() const { return launches_; }
  // The launch program's module tree, one line a module.
  std::string describe() const;

 private:
  void allocate_weights();
  // Quantizes BF16 weights `src` into the slot's format (synthetic initialisation; `amax`, when
  // >= 0, is the tensor-wide magnitude a per-tensor scale covers).
 public:
  void quantize_slot(WeightSlot& w, const __nv_bfloat16* src, float stdv, float amax = -1.f);

 private:
  void ensure_workspace(int64_t rows, int64_t kept, int64_t decode_splits, int64_t decode_rows);
  int launch(const Plan& plan, const Cache& cache);  // returns the kernels it launched
  int adapter_slots_ = 0;
  std::vector<std::shared_ptr<const LoraAdapter>> call_adapters_;  // the current call's slots
  HbmBuffer ws_lora_z_;
  int64_t graph_bucket(int64_t rows) const;

  Device device_;
  ModelConfig cfg_;
  int tp_, rank_;
  int qh_l_, kvh_l_, qh_first_, kvh_first_, inter_l_, vocab_begin_, vocab_end_, vocab_l_;
  int experts_l_ = 0, expert_first_ = 0;
  std::map<std::string, WeightSlot> weights_;
  HbmBuffer arena_;
  size_t arena_bytes_ = 0;
  std::vector<float> inv_freq_host_;
  float attention_factor_ = 1.f;
  HbmBuffer inv_freq_;

  // Workspace (device), sized for `ws_rows_` rows and `ws_kept_` kept rows.
  int64_t ws_rows_ = 0, ws_kept_ = 0, ws_splits_ = 0, ws_decode_ = 0;
  int keys_per_split_ = 2048;  // decode attention's key chunk and warps a CTA (see the constructor)
  int decode_warps_ = 2;
  HbmBuffer ws_x_, ws_h_, ws_qkv_, ws_q_, ws_attn_, ws_act_, ws_hk_, ws_logits_, ws_idx_, ws_val_,
      ws_tokens_, ws_stage_, ws_part_o_, ws_part_lse_, ws_gemm_, ws_counters_, ws_partial_;
  // Quantized inputs of W8A8 / W4A4 projections: codes and scales of the widest input.
  HbmBuffer ws_qa_, ws_qs_;
  // Mixture of experts: router logits, routing, grouping and the sorted expert rows.
  HbmBuffer ws_logits_e_, ws_ids_, ws_rw_, ws_pos_, ws_src_, ws_tile_e_, ws_tiles_, ws_xs_, ws_eact_, ws_y_;
  int64_t ws_moe_rows_ = 0;
  size_t stage_capacity_ = 0;
  std::vector<uint8_t> host_stage_;
  HostBuffer pinned_stage_[2];
  cudaEvent_t stage_done_[2] = {nullptr, nullptr};
  int stage_slot_ = 0;

  std::shared_ptr<Collectives> coll_;
  bool graphs_enabled_ = true;
  bool batch_invariant_ = false;
  struct GraphKey {
    int64_t rows, splits;
    bool operator<(const GraphKey& o) const {
      return rows < o.rows || (rows == o.rows && splits < o.splits);
    }
  };
  struct GraphEntry {
    cudaGraphExec_t exec = nullptr;
    int kernels = 0;
    const void* cache = nullptr;
  };
  std::map<GraphKey, GraphEntry> graphs_;
  uint64_t launches_ = 0;
  void clear_graphs();
  Plan last_plan_;
  // The launch program (modules.h), built at the first call from the configuration.
  std::unique_ptr<Module> program_;
  friend struct Launch;
  friend struct DecoderBlocks;
};

}  // namespace foa::engine
