// C++ host API of the Qwen3 text-encoder prefill (the Flux2 Klein
// pipeline's prompt encoder).  Mirrors the reference's module surface:
//   Qwen3Config::from_file                 (src/transformers/models/qwen3/Qwen3Config.cpp:26-68)
//   Qwen3Model::forward                    (Qwen3Model.cpp:99-208): embedding, decoder layers,
//                                          final RMSNorm, hidden states extracted before
//                                          chosen layers (Flux2KleinPipeline.cpp:481-491)
//   Qwen3DecoderLayer / Qwen3Attention / Qwen3MLP / Qwen3RMSNorm / Qwen3RotaryEmbedding
// Parameters bind by GGUF name ("model.layers.3.self_attn.q_proj.weight", or
// without the "model." prefix).  Prefill only: causal self-attention over the
// whole prompt with an optional key padding mask, no KV cache.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "plan.hpp"

namespace dcpp {

struct Qwen3Config {
  int64_t vocab_size = 151936;
  int64_t hidden_size = 2560;
  int64_t intermediate_size = 9728;
  int64_t num_hidden_layers = 36;
  int64_t num_attention_heads = 32;
  int64_t num_key_value_heads = 8;
  int64_t head_dim = 128;
  float rms_norm_eps = 1e-6f;
  float rope_theta = 1000000.0f;

  static Qwen3Config from_file(const std::string& path);
  static Qwen3Config from_c(const dcpp_qwen3_config& c);
  void to_c(dcpp_qwen3_config& c) const;
};

class Qwen3Model : public StepPlanner {
 public:
  Qwen3Model(Ctx& ctx, const Qwen3Config& cfg);
  ~Qwen3Model() override;

  const Qwen3Config& config() const { return cfg_; }
  void set_param(const std::string& name, int type, const std::vector<int64_t>& shape, const void* data,
                 size_t nbytes);
  std::vector<std::string> missing() const;

  // Plan buffers / tensor maps / graph for `batch` prompts of `seq` tokens;
  // taps: layer indices t in [0, num_hidden_layers] whose input hidden
  // states (t = num_hidden_layers: the final normed output) forward()
  // returns stacked along the feature axis.
  void prepare(int64_t batch, int64_t seq, const std::vector<int>& taps, bool use_graph);
  // input_ids [B, S] int32; attention_mask [B, S] f32 (nonzero = attend,
  // zero = padding key) or null; last_hidden [B, S, D] f32 (final RMSNorm)
  // or null; taps_out [B, S, n_taps * D] f32 or null.  Host or device pointers.
  void forward(const int32_t* input_ids, const float* attention_mask, float* last_hidden, float* taps_out);
  void set_profiling(bool on);

 private:
  struct Layer {
    DevWeight qkv, o, gate_up, down;  // qkv: q | k | v rows; gate_up: 64-row gate / up blocks
    DevVector in_norm, post_norm, q_norm, k_norm;
  };
  void build_registry();
  void place(DevWeight& w, const std::string& part, int type, const std::vector<int64_t>& shape, const uint8_t* src,
             const std::function<int64_t(int64_t)>& row_map);
  void free_plan();
  void build_plan();

  Qwen3Config cfg_;
  DevWeight embed_;
  DevVector norm_;
  std::vector<Layer> layers_;
  std::map<std::string, std::function<void(int, const std::vector<int64_t>&, const void*, size_t)>> setters_;
  std::vector<DevWeight*> weights_;
  std::vector<DevVector*> vectors_;

  int64_t B_ = 0, S_ = 0;
  std::vector<int> taps_;
  bool planned_ = false;
  std::vector<void*> allocs_;
  float *h_ = nullptr, *last_ = nullptr, *taps_dev_ = nullptr;
  uint16_t *a_ = nullptr, *q_ = nullptr, *k_ = nullptr, *v_ = nullptr, *att_ = nullptr, *mlp_ = nullptr;
  int32_t *ids_dev_ = nullptr, *pos_dev_ = nullptr;
  float* mask_dev_ = nullptr;       // [B, S] attention mask of the call
  uint32_t* mask_bits_ = nullptr;   // [B, words] key bits the attention reads
  float* ones_host_ = nullptr;      // pinned [B, S] of 1 (calls without a mask)
  float2* rope_ = nullptr;
  std::vector<Op> ops_;
  cudaGraphExec_t graph_ = nullptr;
};

}  // namespace dcpp

struct dcpp_qwen3 {
  std::unique_ptr<dcpp::Qwen3Model> model;
  dcpp_ctx* ctx = nullptr;
};
