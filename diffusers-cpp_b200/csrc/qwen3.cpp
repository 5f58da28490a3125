// Qwen3 text-encoder prefill on sm_100a: the C++ model host and its C ABI.
#include "qwen3.hpp"

#include <string.h>

#include <algorithm>
#include <array>
#include <cmath>

#include "attention_tc.cuh"
#include "gguf.hpp"

namespace dcpp {

// ----------------------------------------------------------------- config
Qwen3Config Qwen3Config::from_file(const std::string& path) {
  auto m = read_json_object(path);
  Qwen3Config c;
  auto num = [&](const char* k, auto& dst) {
    auto it = m.find(k);
    if (it == m.end() || it->second == "null") return;
    using T = std::decay_t<decltype(dst)>;
    dst = static_cast<T>(std::stod(it->second));
  };
  num("vocab_size", c.vocab_size);
  num("hidden_size", c.hidden_size);
  num("intermediate_size", c.intermediate_size);
  num("num_hidden_layers", c.num_hidden_layers);
  num("num_attention_heads", c.num_attention_heads);
  num("num_key_value_heads", c.num_key_value_heads);
  num("head_dim", c.head_dim);
  num("rms_norm_eps", c.rms_norm_eps);
  num("rope_theta", c.rope_theta);
  return c;
}

Qwen3Config Qwen3Config::from_c(const dcpp_qwen3_config& s) {
  Qwen3Config c;
  c.vocab_size = s.vocab_size;
  c.hidden_size = s.hidden_size;
  c.intermediate_size = s.intermediate_size;
  c.num_hidden_layers = s.num_hidden_layers;
  c.num_attention_heads = s.num_attention_heads;
  c.num_key_value_heads = s.num_key_value_heads;
  c.head_dim = s.head_dim;
  c.rms_norm_eps = s.rms_norm_eps;
  c.rope_theta = s.rope_theta;
  return c;
}

void Qwen3Config::to_c(dcpp_qwen3_config& s) const {
  s.vocab_size = vocab_size;
  s.hidden_size = hidden_size;
  s.intermediate_size = intermediate_size;
  s.num_hidden_layers = num_hidden_layers;
  s.num_attention_heads = num_attention_heads;
  s.num_key_value_heads = num_key_value_heads;
  s.head_dim = head_dim;
  s.rms_norm_eps = rms_norm_eps;
  s.rope_theta = rope_theta;
}

// ----------------------------------------------------------------- model
Qwen3Model::Qwen3Model(Ctx& ctx, const Qwen3Config& cfg) : StepPlanner(ctx), cfg_(cfg) {
  const auto& c = cfg_;
  if (c.head_dim != 128) fail(DCPP_ERR_UNSUPPORTED, "head_dim must be 128");
  if (c.num_attention_heads < 1 || c.num_key_value_heads < 1 || c.num_attention_heads % c.num_key_value_heads)
    fail(DCPP_ERR_INVALID_ARG, "num_attention_heads must be a multiple of num_key_value_heads");
  if (c.hidden_size % 256 || c.hidden_size > 8192) fail(DCPP_ERR_UNSUPPORTED, "hidden_size must be a multiple of 256, <= 8192");
  if (c.intermediate_size % 64) fail(DCPP_ERR_UNSUPPORTED, "intermediate_size must be a multiple of 64");
  if (c.vocab_size < 1 || c.num_hidden_layers < 0) fail(DCPP_ERR_INVALID_ARG, "bad vocab_size / num_hidden_layers");
  build_registry();
}

Qwen3Model::~Qwen3Model() {
  cudaSetDevice(ctx_.device);
  cudaStreamSynchronize(ctx_.stream);
  free_plan();
  for (auto* w : weights_)
    if (w->data) cudaFree(w->data);
  for (auto* v : vectors_)
    if (v->data) cudaFree(v->data);
}

void Qwen3Model::build_registry() {
  const int64_t D = cfg_.hidden_size, I = cfg_.intermediate_size;
  const int64_t Dq = cfg_.num_attention_heads * 128, Dkv = cfg_.num_key_value_heads * 128;
  using RowMap = std::function<int64_t(int64_t)>;
  auto initw = [&](DevWeight& w, const std::string& name, int64_t rows, int64_t cols, std::set<std::string> parts) {
    w = DevWeight();
    w.name = name;
    w.rows = rows;
    w.cols = cols;
    w.need = std::move(parts);
    weights_.push_back(&w);
  };
  auto initv = [&](DevVector& v, const std::string& name, int64_t n) {
    v = DevVector();
    v.name = name;
    v.n = n;
    vectors_.push_back(&v);
    DevVector* pv = &v;
    setters_[name] = [pv](int type, const std::vector<int64_t>& shape, const void* data, size_t nbytes) {
      set_vector_param(*pv, type, shape, data, nbytes, false);
    };
  };
  auto reg = [&](const std::string& name, DevWeight* w, const std::string& part, int64_t rows, int64_t cols,
                 RowMap map) {
    setters_[name] = [this, w, part, rows, cols, map, name](int type, const std::vector<int64_t>& shape,
                                                           const void* data, size_t nbytes) {
      if (shape.size() != 2 || shape[0] != rows || shape[1] != cols)
        fail(DCPP_ERR_INVALID_ARG, "Error while loading Tensor '" + name + "': Parameter shape mismatch: expected " +
                                       shape_str({rows, cols}) + ", got " + shape_str(shape));
      if (!is_gemm_type(type)) fail(DCPP_ERR_UNSUPPORTED, "Tensor '" + name + "': unsupported type");
      if (nbytes != row_bytes_of(type, cols) * static_cast<size_t>(rows))
        fail(DCPP_ERR_INVALID_ARG, "Tensor '" + name + "': byte size mismatch");
      place(*w, part, type, shape, static_cast<const uint8_t*>(data), map);
    };
  };
  auto offset = [](int64_t base) { return RowMap([base](int64_t i) { return base + i; }); };
  // gate / up rows interleaved in 64-row blocks (the SwiGLU epilogue's layout).
  auto swiglu_rows = [](bool up) {
    return RowMap([up](int64_t j) { return (j / 64) * 128 + (up ? 64 : 0) + (j % 64); });
  };

  initw(embed_, "model.embed_tokens.weight", cfg_.vocab_size, D, {"all"});
  reg(embed_.name, &embed_, "all", cfg_.vocab_size, D, offset(0));
  initv(norm_, "model.norm.weight", D);
  layers_.assign(static_cast<size_t>(cfg_.num_hidden_layers), Layer());
  for (int64_t i = 0; i < cfg_.num_hidden_layers; ++i) {
    Layer& L = layers_[i];
    const std::string p = "model.layers." + std::to_string(i) + ".";
    initw(L.qkv, p + "self_attn.qkv", Dq + 2 * Dkv, D, {"q", "k", "v"});
    reg(p + "self_attn.q_proj.weight", &L.qkv, "q", Dq, D, offset(0));
    reg(p + "self_attn.k_proj.weight", &L.qkv, "k", Dkv, D, offset(Dq));
    reg(p + "self_attn.v_proj.weight", &L.qkv, "v", Dkv, D, offset(Dq + Dkv));
    initw(L.o, p + "self_attn.o_proj.weight", D, Dq, {"all"});
    reg(L.o.name, &L.o, "all", D, Dq, offset(0));
    initw(L.gate_up, p + "mlp.gate_up", 2 * I, D, {"gate", "up"});
    reg(p + "mlp.gate_proj.weight", &L.gate_up, "gate", I, D, swiglu_rows(false));
    reg(p + "mlp.up_proj.weight", &L.gate_up, "up", I, D, swiglu_rows(true));
    initw(L.down, p + "mlp.down_proj.weight", D, I, {"all"});
    reg(L.down.name, &L.down, "all", D, I, offset(0));
    initv(L.in_norm, p + "input_layernorm.weight", D);
    initv(L.post_norm, p + "post_attention_layernorm.weight", D);
    initv(L.q_norm, p + "self_attn.q_norm.weight", 128);
    initv(L.k_norm, p + "self_attn.k_norm.weight", 128);
  }
}

void Qwen3Model::place(DevWeight& w, const std::string& part, int type, const std::vector<int64_t>& shape,
                       const uint8_t* src, const std::function<int64_t(int64_t)>& row_map) {
  if (!w.need.count(part)) fail(DCPP_ERR_STATE, "Tensor '" + w.name + "': part '" + part + "' set twice");
  if (w.type >= 0 && w.type != type)
    fail(DCPP_ERR_UNSUPPORTED, "Tensor '" + w.name + "': parts of one fused weight must share a ggml type");
  if (w.cols % block_size_of(type)) fail(DCPP_ERR_UNSUPPORTED, "Tensor '" + w.name + "': columns not block aligned");
  if (w.type < 0) {
    w.type = type;
    w.row_bytes = row_bytes_of(type, w.cols);
    w.staging.assign(w.row_bytes * static_cast<size_t>(w.rows), 0);
  }
  for (int64_t i = 0; i < shape[0]; ++i) {
    const int64_t d = row_map(i);
    if (d < 0 || d >= w.rows) fail(DCPP_ERR_STATE, "internal: row map out of range for " + w.name);
    memcpy(w.staging.data() + static_cast<size_t>(d) * w.row_bytes, src + static_cast<size_t>(i) * w.row_bytes,
           w.row_bytes);
  }
  w.need.erase(part);
  if (!w.need.empty()) return;
  const size_t bytes = w.staging.size();
  if (cudaMalloc(&w.data, bytes) != cudaSuccess) {
    cudaGetLastError();
    w.data = nullptr;
    fail(DCPP_ERR_OOM, "weight allocation failed for " + w.name);
  }
  cuda_check(cudaMemcpy(w.data, w.staging.data(), bytes, cudaMemcpyHostToDevice), "upload weight");
  std::vector<uint8_t>().swap(w.staging);
  planned_ = false;
}

void Qwen3Model::set_param(const std::string& name, int type, const std::vector<int64_t>& shape, const void* data,
                           size_t nbytes) {
  if (!data) fail(DCPP_ERR_INVALID_ARG, "Tensor '" + name + "': null data");
  if (name == "lm_head.weight") return;  // not used by the prefill
  auto it = setters_.find(name);
  if (it == setters_.end()) it = setters_.find("model." + name);
  if (it == setters_.end()) fail(DCPP_ERR_NOT_FOUND, "Error while loading Tensor '" + name + "': Tensor not found");
  it->second(type, shape, data, nbytes);
  planned_ = false;
}

std::vector<std::string> Qwen3Model::missing() const {
  std::vector<std::string> m;
  for (auto* w : weights_)
    for (auto& p : w->need) m.push_back(w->name + (p == "all" ? "" : " [" + p + "]"));
  for (auto* v : vectors_)
    if (!v->set) m.push_back(v->name);
  return m;
}

// ----------------------------------------------------------------- plan
void Qwen3Model::free_plan() {
  if (graph_) cudaGraphExecDestroy(graph_);
  graph_ = nullptr;
  for (void* p : allocs_) cudaFree(p);
  allocs_.clear();
  if (ones_host_) cudaFreeHost(ones_host_);
  ones_host_ = nullptr;
  ops_.clear();
  last_ops_ = nullptr;
  release_plan_events();
  planned_ = false;
}

void Qwen3Model::prepare(int64_t batch, int64_t seq, const std::vector<int>& taps, bool use_graph) {
  auto miss = missing();
  if (!miss.empty())
    fail(DCPP_ERR_STATE, "parameters not set: " + miss.front() + " (+" + std::to_string(miss.size() - 1) + " more)");
  // One GEMM row group per prompt (the QKV epilogue needs the prompt index).
  if (batch < 1 || batch > kGemmMaxGroups || seq < 1 || batch * seq > (1 << 20))
    fail(DCPP_ERR_UNSUPPORTED, "batch 1..8 and batch * seq <= 2^20");
  for (int t : taps)
    if (t < 0 || t > cfg_.num_hidden_layers) fail(DCPP_ERR_INVALID_ARG, "tap layer out of range");
  if (planned_ && batch == B_ && seq == S_ && taps == taps_ && use_graph == use_graph_) return;
  cudaStreamSynchronize(ctx_.stream);
  free_plan();
  B_ = batch;
  S_ = seq;
  taps_ = taps;
  use_graph_ = use_graph;
  build_plan();
  planned_ = true;
}

void Qwen3Model::build_plan() {
  const int64_t B = B_, S = S_, R = B * S, D = cfg_.hidden_size, I = cfg_.intermediate_size;
  const int64_t Hq = cfg_.num_attention_heads, Hkv = cfg_.num_key_value_heads;
  const int64_t Dq = Hq * 128, Dkv = Hkv * 128;
  const int64_t nt = static_cast<int64_t>(taps_.size());
  auto alloc = [&](size_t bytes) {
    void* p = nullptr;
    if (cudaMalloc(&p, std::max<size_t>(bytes, 256)) != cudaSuccess) {
      cudaGetLastError();
      fail(DCPP_ERR_OOM, "activation allocation of " + std::to_string(bytes) + " bytes failed");
    }
    allocs_.push_back(p);
    return p;
  };
  h_ = static_cast<float*>(alloc(R * D * 4));
  last_ = static_cast<float*>(alloc(R * D * 4));
  taps_dev_ = static_cast<float*>(alloc(std::max<int64_t>(nt, 1) * R * D * 4));
  a_ = static_cast<uint16_t*>(alloc(R * D * 2));
  q_ = static_cast<uint16_t*>(alloc(R * Dq * 2));
  k_ = static_cast<uint16_t*>(alloc(R * Dkv * 2));
  const int64_t sp = attn_vt_stride(S);
  v_ = static_cast<uint16_t*>(alloc(B * Hkv * 128 * sp * 2));
  cuda_check(cudaMemset(v_, 0, B * Hkv * 128 * sp * 2), "memset vt");
  att_ = static_cast<uint16_t*>(alloc(R * Dq * 2));
  mlp_ = static_cast<uint16_t*>(alloc(R * I * 2));
  ids_dev_ = static_cast<int32_t*>(alloc(R * 4));
  pos_dev_ = static_cast<int32_t*>(alloc(S * 4));
  {
    std::vector<int32_t> pos(static_cast<size_t>(S));
    for (int64_t i = 0; i < S; ++i) pos[i] = static_cast<int32_t>(i);
    cuda_check(cudaMemcpy(pos_dev_, pos.data(), S * 4, cudaMemcpyHostToDevice), "positions");
  }
  rope_ = static_cast<float2*>(alloc(S * 64 * sizeof(float2)));
  const int64_t words = (S + 31) / 32;
  mask_dev_ = static_cast<float*>(alloc(R * 4));
  mask_bits_ = static_cast<uint32_t*>(alloc(B * words * 4));
  cuda_check(cudaMallocHost(&ones_host_, R * 4), "pinned ones");
  for (int64_t i = 0; i < R; ++i) ones_host_[i] = 1.0f;
  size_t s0 = 0;
  for (auto& L : layers_)
    for (const DevWeight* w : {&L.qkv, &L.o, &L.gate_up, &L.down})
      if (w->type != kTypeBF16) s0 = std::max(s0, static_cast<size_t>(w->rows * w->cols));
  alloc_expansion_scratch(alloc, s0, 8);

  begin_ops(ops_);
  const float eps = cfg_.rms_norm_eps;
  const int32_t axes[1] = {128};
  const float theta = cfg_.rope_theta;
  float2* rope = rope_;
  int32_t* pos = pos_dev_;
  ops_.push_back({[rope, pos, S, axes, theta](cudaStream_t s) {
                    cuda_check(launch_rope_table(pos, S, 1, axes, theta, rope, s), "rope_table");
                  },
                  1, kOpOther, 0.0, "rope_table"});
  // Key padding bits from the call's attention mask (Qwen3Model.cpp:78-94 adds
  // (1 - mask) * -1e9, which the f16 mask turns into -inf).
  {
    const float* mk = mask_dev_;
    uint32_t* bits = mask_bits_;
    ops_.push_back({[mk, bits, B, S, words](cudaStream_t s) {
                      cuda_check(launch_mask_bits(mk, B, S, words, bits, s), "mask bits");
                    },
                    1, kOpOther, 0.0, "mask_bits"});
  }
  // Embedding::forward (ggml_get_rows).
  {
    const DevWeight* e = &embed_;
    float* h = h_;
    int32_t* ids = ids_dev_;
    int* err = ctx_.d_err;
    ops_.push_back({[e, h, ids, R, err](cudaStream_t s) {
                      cuda_check(launch_get_rows(e->type, e->data, e->rows, e->cols, ids, R, h, err, s), "get_rows");
                    },
                    1, kOpOther, 0.0, "embed_tokens"});
  }
  auto tap_copy = [&](int layer, const float* src) {
    for (int64_t k = 0; k < nt; ++k) {
      if (taps_[k] != layer) continue;
      float* dst = taps_dev_ + k * D;
      ops_.push_back({[dst, src, D, nt, R](cudaStream_t s) {
                        cuda_check(cudaMemcpy2DAsync(dst, nt * D * 4, src, D * 4, D * 4, R, cudaMemcpyDeviceToDevice, s),
                                   "tap copy");
                      },
                      0, kOpOther, 0.0, "tap"});
    }
  };
  auto rms = [&](const DevVector& w, float* y_f32) {
    NormArgs n{};
    n.x = h_;
    n.x_out = h_;
    n.y = a_;
    n.ld_x = D;
    n.ld_y = D;
    n.D = static_cast<int32_t>(D);
    n.eps = eps;
    n.n_segments = 1;
    n.seg[0] = {0, 0, static_cast<int32_t>(R), nullptr, nullptr};
    n.rms = 1;
    n.weight = w.data;
    n.y_f32 = y_f32;
    add_norm(n);
  };
  std::vector<GemmGroup> groups;
  for (int64_t b = 0; b < B; ++b) {
    GemmGroup g{};
    g.row0 = g.orow0 = static_cast<int32_t>(b * S);
    g.rows = static_cast<int32_t>(S);
    g.batch = static_cast<int32_t>(b);
    g.tok0 = 0;
    groups.push_back(g);
  }
  AttnTcArgs at{};
  at.o = att_;
  at.ld_o = Dq;
  at.B = static_cast<int32_t>(B);
  at.H = static_cast<int32_t>(Hq);
  at.S = static_cast<int32_t>(S);
  at.scale = 1.0f / std::sqrt(128.0f);
  at.err = ctx_.d_err;
  at.kernel = ctx_.attn_kernel;
  at.causal = 1;
  at.H_kv = static_cast<int32_t>(Hkv);
  at.key_bits = mask_bits_;
  at.key_words = static_cast<int32_t>(words);
  auto maps = std::make_shared<AttnTcMaps>();
  cuda_check(make_attn_maps(maps.get(), q_, k_, v_, static_cast<int>(B), static_cast<int>(Hq), static_cast<int>(S),
                            static_cast<int>(Hkv)),
             "attention tensor maps");
  const double attn_flops = 2.0 * B * Hq * static_cast<double>(S) * static_cast<double>(S + 1) * 128.0;  // causal
  for (int64_t li = 0; li < cfg_.num_hidden_layers; ++li) {
    Layer& L = layers_[li];
    tap_copy(static_cast<int>(li), h_);
    // Qwen3DecoderLayer.cpp:16-49: h += o_proj(attn(rms(h))); h += mlp(rms(h)).
    rms(L.in_norm, nullptr);
    EpilogueArgs e{};
    e.mode = kEpiQkvMlp;
    e.qkv_cols = static_cast<int32_t>(Dq + 2 * Dkv);
    e.inner = static_cast<int32_t>(Dq);
    e.kv_inner = static_cast<int32_t>(Dkv);
    e.seq = static_cast<int32_t>(S);
    e.heads = static_cast<int32_t>(Hq);
    e.heads_kv = static_cast<int32_t>(Hkv);
    e.rope_neox = 1;
    e.norm_q[0] = e.norm_q[1] = L.q_norm.data;
    e.norm_k[0] = e.norm_k[1] = L.k_norm.data;
    e.eps = eps;
    e.rope = rope_;
    e.q_out = q_;
    e.k_out = k_;
    e.v_out = v_;
    e.vt_stride = sp;
    add_gemm("qkv", a_, D, D, &L.qkv, nullptr, groups, e, Dq + 2 * Dkv);
    ops_.push_back({[at, maps](cudaStream_t s) { cuda_check(launch_attention_tc(*maps, at, s), "attention"); }, 1,
                    kOpAttention, attn_flops, "attention"});
    EpilogueArgs r{};
    r.mode = kEpiResidGate;  // no gate: h += acc
    r.out_f32 = h_;
    r.ld_out = D;
    add_gemm("o_proj", att_, Dq, Dq, &L.o, nullptr, groups, r, D);
    rms(L.post_norm, nullptr);
    EpilogueArgs m{};
    m.mode = kEpiQkvMlp;
    m.qkv_cols = 0;
    m.mlp_out = mlp_;
    m.ld_mlp = I;
    add_gemm("gate_up", a_, D, D, &L.gate_up, nullptr, groups, m, 2 * I);
    add_gemm("down", mlp_, I, I, &L.down, nullptr, groups, r, D);
  }
  rms(norm_, last_);  // Qwen3Model.cpp:195-198; a_ gets the bf16 copy, unused
  tap_copy(static_cast<int>(cfg_.num_hidden_layers), last_);
  end_ops();
  launches_per_step_ = 0;
  for (auto& o : ops_) launches_per_step_ += o.launches;
}

void Qwen3Model::forward(const int32_t* input_ids, const float* attention_mask, float* last_hidden, float* taps_out) {
  if (!planned_) fail(DCPP_ERR_STATE, "forward before prepare");
  if (!input_ids) fail(DCPP_ERR_INVALID_ARG, "forward: null input_ids");
  const int64_t R = B_ * S_, D = cfg_.hidden_size;
  cuda_check(cudaMemcpyAsync(ids_dev_, input_ids, R * 4, cudaMemcpyDefault, ctx_.stream), "copy ids");
  cuda_check(cudaMemcpyAsync(mask_dev_, attention_mask ? attention_mask : ones_host_, R * 4, cudaMemcpyDefault,
                             ctx_.stream),
             "copy mask");
  run_ops(ops_, &graph_);
  if (last_hidden)
    cuda_check(cudaMemcpyAsync(last_hidden, last_, R * D * 4, cudaMemcpyDefault, ctx_.stream), "copy hidden");
  if (taps_out && !taps_.empty())
    cuda_check(cudaMemcpyAsync(taps_out, taps_dev_, static_cast<int64_t>(taps_.size()) * R * D * 4, cudaMemcpyDefault,
                               ctx_.stream),
               "copy taps");
  ctx_.check_device_error();
}

void Qwen3Model::set_profiling(bool on) {
  if (on == profiling_) return;
  cudaStreamSynchronize(ctx_.stream);
  free_plan();
  profiling_ = on;
}

}  // namespace dcpp

// ----------------------------------------------------------------- C ABI
namespace {

template <class F>
dcpp_status qwen_call(dcpp_qwen3* m, const char* entry, F&& f) {
  if (!m || !m->ctx) return DCPP_ERR_INVALID_ARG;
  dcpp_ctx* ctx = m->ctx;
  try {
    ctx->maybe_inject(entry);
    cudaSetDevice(ctx->device);
    f(*m->model);
    return DCPP_OK;
  } catch (const dcpp::Error& e) {
    ctx->last_error = e.what();
    return e.status;
  } catch (const std::exception& e) {
    ctx->last_error = e.what();
    return DCPP_ERR_INVALID_ARG;
  }
}

}  // namespace

extern "C" {

void dcpp_qwen3_config_default(dcpp_qwen3_config* cfg) {
  if (cfg) dcpp::Qwen3Config().to_c(*cfg);
}

dcpp_status dcpp_qwen3_config_from_file(const char* path, dcpp_qwen3_config* cfg) {
  if (!path || !cfg) return DCPP_ERR_INVALID_ARG;
  try {
    dcpp::Qwen3Config::from_file(path).to_c(*cfg);
    return DCPP_OK;
  } catch (const dcpp::Error& e) {
    return e.status;
  } catch (const std::exception&) {
    return DCPP_ERR_INVALID_ARG;
  }
}

dcpp_status dcpp_qwen3_create(dcpp_ctx* ctx, const dcpp_qwen3_config* cfg, dcpp_qwen3** out) {
  if (!ctx || !cfg || !out) return DCPP_ERR_INVALID_ARG;
  *out = nullptr;
  try {
    ctx->maybe_inject("dcpp_qwen3_create");
    cudaSetDevice(ctx->device);
    auto* m = new dcpp_qwen3();
    m->ctx = ctx;
    try {
      m->model.reset(new dcpp::Qwen3Model(*ctx, dcpp::Qwen3Config::from_c(*cfg)));
    } catch (...) {
      delete m;
      throw;
    }
    *out = m;
    return DCPP_OK;
  } catch (const dcpp::Error& e) {
    ctx->last_error = e.what();
    return e.status;
  } catch (const std::exception& e) {
    ctx->last_error = e.what();
    return DCPP_ERR_INVALID_ARG;
  }
}

dcpp_status dcpp_qwen3_destroy(dcpp_qwen3* m) {
  if (!m) return DCPP_ERR_INVALID_ARG;
  if (m->ctx) cudaSetDevice(m->ctx->device);
  delete m;
  return DCPP_OK;
}

dcpp_status dcpp_qwen3_set_param(dcpp_qwen3* m, const char* name, int type, int n_dims, const int64_t* shape,
                                 const void* data, size_t nbytes) {
  return qwen_call(m, "dcpp_qwen3_set_param", [&](dcpp::Qwen3Model& mm) {
    if (!name || !shape || n_dims < 1 || n_dims > 4) dcpp::fail(DCPP_ERR_INVALID_ARG, "set_param: bad name or shape");
    mm.set_param(name, type, std::vector<int64_t>(shape, shape + n_dims), data, nbytes);
  });
}

dcpp_status dcpp_qwen3_missing(dcpp_qwen3* m, int* count, char* first, size_t cap) {
  return qwen_call(m, "dcpp_qwen3_missing", [&](dcpp::Qwen3Model& mm) {
    auto miss = mm.missing();
    if (count) *count = static_cast<int>(miss.size());
    if (first && cap) {
      std::string f = miss.empty() ? "" : miss.front();
      size_t n = std::min(cap - 1, f.size());
      memcpy(first, f.data(), n);
      first[n] = 0;
    }
  });
}

dcpp_status dcpp_qwen3_prepare(dcpp_qwen3* m, int64_t batch, int64_t seq, int n_taps, const int* tap_layers,
                               int use_graph) {
  return qwen_call(m, "dcpp_qwen3_prepare", [&](dcpp::Qwen3Model& mm) {
    if (n_taps < 0 || (n_taps > 0 && !tap_layers)) dcpp::fail(DCPP_ERR_INVALID_ARG, "prepare: bad taps");
    mm.prepare(batch, seq, std::vector<int>(tap_layers, tap_layers + n_taps), use_graph != 0);
  });
}

dcpp_status dcpp_qwen3_forward(dcpp_qwen3* m, const int32_t* ids, const float* attention_mask, float* last_hidden,
                               float* taps) {
  return qwen_call(m, "dcpp_qwen3_forward",
                   [&](dcpp::Qwen3Model& mm) { mm.forward(ids, attention_mask, last_hidden, taps); });
}

dcpp_status dcpp_qwen3_set_profiling(dcpp_qwen3* m, int on) {
  return qwen_call(m, "dcpp_qwen3_set_profiling", [&](dcpp::Qwen3Model& mm) { mm.set_profiling(on != 0); });
}

dcpp_status dcpp_qwen3_profile(dcpp_qwen3* m, int kind, double* ms, double* flops, int64_t* launches) {
  return qwen_call(m, "dcpp_qwen3_profile", [&](dcpp::Qwen3Model& mm) {
    if (kind < 0 || kind >= dcpp::StepPlanner::kOpKinds) dcpp::fail(DCPP_ERR_INVALID_ARG, "bad kind");
    mm.profile(kind, ms, flops, launches);
  });
}

dcpp_status dcpp_qwen3_launches_per_step(dcpp_qwen3* m, int64_t* out) {
  return qwen_call(m, "dcpp_qwen3_launches_per_step", [&](dcpp::Qwen3Model& mm) {
    if (!out) dcpp::fail(DCPP_ERR_INVALID_ARG, "null output");
    *out = mm.launches_per_step();
  });
}

}  // extern "C"

// GGUF checkpoints.
extern "C" {

dcpp_status dcpp_qwen3_load_gguf(dcpp_qwen3* m, const dcpp_gguf* f, int64_t* n_bound, int64_t* n_unused) {
  return qwen_call(m, "dcpp_qwen3_load_gguf", [&](dcpp::Qwen3Model& mm) {
    if (!f || !f->file) dcpp::fail(DCPP_ERR_INVALID_ARG, "load_gguf: null file");
    int64_t unused = 0;
    const int64_t bound = dcpp::gguf_bind_all(
        *f->file,
        [&](const std::string& name, int type, const std::vector<int64_t>& shape, const void* data, size_t nbytes) {
          mm.set_param(name, type, shape, data, nbytes);
        },
        &unused);
    if (n_bound) *n_bound = bound;
    if (n_unused) *n_unused = unused;
    const auto miss = mm.missing();
    if (!miss.empty()) dcpp::fail(DCPP_ERR_NOT_FOUND, "Error while loading Tensor '" + miss.front() + "': Tensor not found");
  });
}

dcpp_status dcpp_qwen3_from_pretrained(dcpp_ctx* ctx, const char* dir, dcpp_qwen3** out) {
  if (!ctx || !dir || !out) return DCPP_ERR_INVALID_ARG;
  *out = nullptr;
  dcpp_qwen3_config cfg;
  try {
    dcpp::Qwen3Config::from_file(std::string(dir) + "/config.json").to_c(cfg);
  } catch (const dcpp::Error& e) {
    ctx->last_error = e.what();
    return e.status;
  } catch (const std::exception& e) {
    ctx->last_error = e.what();
    return DCPP_ERR_INVALID_ARG;
  }
  dcpp_gguf* g = nullptr;
  char err[1024];
  dcpp_status st = dcpp_gguf_open(dir, &g, err, sizeof(err));
  if (st != DCPP_OK) {
    ctx->last_error = err;
    return st;
  }
  st = dcpp_qwen3_create(ctx, &cfg, out);
  if (st == DCPP_OK) st = dcpp_qwen3_load_gguf(*out, g, nullptr, nullptr);
  dcpp_gguf_close(g);
  if (st != DCPP_OK && *out) {
    dcpp_qwen3_destroy(*out);
    *out = nullptr;
  }
  return st;
}

}  // extern "C"
