// Flux2 DiT denoise step on sm_100a: the C++ model host and its C ABI.
#include "flux2.hpp"
#include "attention_tc.cuh"
#include "gguf.hpp"

#include <cuda_fp16.h>

#include <string.h>

#include <algorithm>
#include <array>
#include <cmath>
#include <fstream>
#include <sstream>

namespace dcpp {

// ----------------------------------------------------------------- config
Flux2Config Flux2Config::from_file(const std::string& path) {
  auto m = read_json_object(path);
  Flux2Config c;
  auto num = [&](const char* k, auto& dst) {
    auto it = m.find(k);
    if (it == m.end() || it->second == "null") return;
    using T = std::decay_t<decltype(dst)>;
    dst = static_cast<T>(std::stod(it->second));
  };
  num("patch_size", c.patch_size);
  num("in_channels", c.in_channels);
  {
    auto it = m.find("out_channels");
    if (it != m.end()) c.out_channels = it->second == "null" ? -1 : static_cast<int64_t>(std::stod(it->second));
  }
  num("num_layers", c.num_layers);
  num("num_single_layers", c.num_single_layers);
  num("attention_head_dim", c.attention_head_dim);
  num("num_attention_heads", c.num_attention_heads);
  num("joint_attention_dim", c.joint_attention_dim);
  num("timestep_guidance_channels", c.timestep_guidance_channels);
  num("mlp_ratio", c.mlp_ratio);
  num("rope_theta", c.rope_theta);
  num("eps", c.eps);
  {
    auto it = m.find("axes_dims_rope");
    if (it != m.end() && it->second != "null") c.axes_dims_rope = parse_int_list(it->second);
    it = m.find("guidance_embeds");
    if (it != m.end() && it->second != "null") c.guidance_embeds = it->second == "true";
  }
  return c;
}

Flux2Config Flux2Config::from_c(const dcpp_flux2_config& s) {
  Flux2Config c;
  c.patch_size = s.patch_size;
  c.in_channels = s.in_channels;
  c.out_channels = s.out_channels;
  c.num_layers = s.num_layers;
  c.num_single_layers = s.num_single_layers;
  c.attention_head_dim = s.attention_head_dim;
  c.num_attention_heads = s.num_attention_heads;
  c.joint_attention_dim = s.joint_attention_dim;
  c.timestep_guidance_channels = s.timestep_guidance_channels;
  c.mlp_ratio = s.mlp_ratio;
  if (s.n_axes < 1 || s.n_axes > 8) fail(DCPP_ERR_INVALID_ARG, "n_axes must be 1..8");
  c.axes_dims_rope.assign(s.axes_dims_rope, s.axes_dims_rope + s.n_axes);
  c.rope_theta = s.rope_theta;
  c.eps = s.eps;
  c.guidance_embeds = s.guidance_embeds != 0;
  return c;
}

void Flux2Config::to_c(dcpp_flux2_config& s) const {
  s.patch_size = patch_size;
  s.in_channels = in_channels;
  s.out_channels = out_channels;
  s.num_layers = num_layers;
  s.num_single_layers = num_single_layers;
  s.attention_head_dim = attention_head_dim;
  s.num_attention_heads = num_attention_heads;
  s.joint_attention_dim = joint_attention_dim;
  s.timestep_guidance_channels = timestep_guidance_channels;
  s.mlp_ratio = mlp_ratio;
  s.n_axes = static_cast<int64_t>(std::min<size_t>(axes_dims_rope.size(), 8));
  for (int64_t i = 0; i < s.n_axes; ++i) s.axes_dims_rope[i] = axes_dims_rope[i];
  s.rope_theta = rope_theta;
  s.eps = eps;
  s.guidance_embeds = guidance_embeds ? 1 : 0;
}

// All arithmetic in float, in the reference's order, so the schedule is the
// reference's bit for bit.
void FlowMatchEulerDiscreteScheduler::schedule(int n, float mu, const std::vector<float>& sigmas_in,
                                               std::vector<float>& timesteps, std::vector<float>& sigmas) const {
  if (num_train_timesteps <= 0) fail(DCPP_ERR_INVALID_ARG, "num_train_timesteps must be positive");
  if (n <= 0) fail(DCPP_ERR_INVALID_ARG, "num_inference_steps must be positive");
  const float nt = static_cast<float>(num_train_timesteps);
  if (!sigmas_in.empty()) {
    if (sigmas_in.size() != static_cast<size_t>(n)) fail(DCPP_ERR_INVALID_ARG, "sigmas must have n entries");
    sigmas = sigmas_in;
  } else {
    // timesteps evenly spaced from sigma_max * T down to sigma_min * T
    const float hi = 1.0f * nt, lo = (1.0f / nt) * nt;
    sigmas.assign(static_cast<size_t>(n), 0.0f);
    if (n == 1) {
      sigmas[0] = hi / nt;
    } else {
      const float step_den = static_cast<float>(n - 1);
      for (int i = 0; i < n; ++i) sigmas[i] = (hi - static_cast<float>(i) * (hi - lo) / step_den) / nt;
    }
  }
  for (float& s : sigmas) {
    if (use_dynamic_shifting) {
      // time_shift(mu, 1, s): e / (e + (1/s - 1)^1), e = exp(mu) or mu
      if (s <= 0.0f) fail(DCPP_ERR_INVALID_ARG, "dynamic shifting needs every sigma > 0");
      const float odds = std::pow(1.0f / s - 1.0f, 1.0f);
      const float e = linear_time_shift ? mu : std::exp(mu);
      s = e / (e + odds);
    } else {
      s = shift * s / (1.0f + (shift - 1.0f) * s);
    }
  }
  if (has_shift_terminal) {
    const float stretch = (1.0f - sigmas.back()) / (1.0f - shift_terminal);
    for (float& s : sigmas) s = 1.0f - (1.0f - s) / stretch;
  }
  if (invert_sigmas)
    for (float& s : sigmas) s = 1.0f - s;
  timesteps.resize(static_cast<size_t>(n));
  for (int i = 0; i < n; ++i) timesteps[i] = sigmas[i] * nt;
  sigmas.push_back(invert_sigmas ? 1.0f : 0.0f);
}

void FlowMatchEulerDiscreteScheduler::pipeline_schedule(int n, int64_t image_seq_len, std::vector<float>& timesteps,
                                                        std::vector<float>& sigmas) const {
  if (n <= 0) fail(DCPP_ERR_INVALID_ARG, "num_inference_steps must be positive");
  std::vector<float> base(static_cast<size_t>(n));
  for (int i = 0; i < n; ++i) base[i] = static_cast<float>(1.0 - static_cast<double>(i) / n);
  schedule(n, flux2_empirical_mu(image_seq_len, n), base, timesteps, sigmas);
}

float flux2_empirical_mu(int64_t image_seq_len, int num_steps) {
  // Two linear fits of mu in the sequence length, at 10 and at 200 steps,
  // interpolated linearly in the step count; long sequences use the
  // 200-step fit alone.
  const float len = static_cast<float>(image_seq_len);
  const float at200 = 0.00016927f * len + 0.45666666f;
  if (image_seq_len > 4300) return at200;
  const float at10 = 8.73809524e-05f * len + 1.89833333f;
  const float slope = (at200 - at10) / 190.0f;
  return slope * static_cast<float>(num_steps) + (at200 - 200.0f * slope);
}

// ----------------------------------------------------------------- model
Flux2Transformer2DModel::Flux2Transformer2DModel(Ctx& ctx, const Flux2Config& cfg, bool host_only)
    : StepPlanner(ctx), cfg_(cfg), host_only_(host_only) {
  if (cfg_.attention_head_dim != 128) fail(DCPP_ERR_UNSUPPORTED, "attention_head_dim must be 128");
  if (cfg_.patch_size != 1) fail(DCPP_ERR_UNSUPPORTED, "patch_size must be 1");
  int64_t tot = 0;
  for (auto d : cfg_.axes_dims_rope) tot += d;
  if (tot != cfg_.attention_head_dim) fail(DCPP_ERR_INVALID_ARG, "axes_dims_rope must sum to attention_head_dim");
  if (const char* e = getenv("DCPP_FUSED_DEQUANT")) fused_dequant_ = std::string(e) == "1";
  if (const char* e = getenv("DCPP_TP_COMM")) tp_peer_ = std::string(e) != "nccl";
  if (const char* e = getenv("DCPP_TP_PIECES")) tp_pieces_env_ = std::string(e) == "1" ? 1 : 2;
  if (const char* e = getenv("DCPP_TP_PULL")) tp_pull_ = std::string(e) == "1";
  if (const char* e = getenv("DCPP_TP_OVERLAP")) tp_overlap_ = std::string(e) == "1";
  if (const char* e = getenv("DCPP_BLOCK_PREFETCH")) block_prefetch_ = std::string(e) == "1";
  build_registry();
}

Flux2Transformer2DModel::~Flux2Transformer2DModel() {
  if (host_only_) return;
  cudaSetDevice(ctx_.device);
  cudaStreamSynchronize(ctx_.stream);
  free_plan();
  for (auto* w : weights_) {
    if (w->data) cudaFree(w->data);
    if (w->packed) cudaFree(w->packed);
  }
  for (auto* v : vectors_)
    if (v->data) cudaFree(v->data);
}

// Split `units` indivisible units over the ranks in proportion to `ratios`
// (ShardingRuntime::compute_split_groups, ShardingRuntime.cpp:280-296): with
// c_j = units * f_j / sum f, every rank first gets floor(c_j); the remaining
// units go one by one to the ranks with the largest fractional parts (ties:
// the later rank, as the even split does).  Equal ratios give the even split.
std::vector<int64_t> plan_tensor_split(int64_t units, const std::vector<double>& ratios) {
  const int n = static_cast<int>(ratios.size());
  if (n < 1) fail(DCPP_ERR_INVALID_ARG, "tensor split: no ranks");
  double sum = 0.0;
  for (double f : ratios) {
    if (!(f > 0.0) || !std::isfinite(f)) fail(DCPP_ERR_INVALID_ARG, "tensor split: ratios must be positive");
    sum += f;
  }
  std::vector<int64_t> m(n);
  std::vector<double> frac(n);
  int64_t given = 0;
  for (int j = 0; j < n; ++j) {
    const double c = static_cast<double>(units) * ratios[j] / sum;
    m[j] = static_cast<int64_t>(std::floor(c));
    frac[j] = c - static_cast<double>(m[j]);
    given += m[j];
  }
  for (int64_t left = units - given; left > 0; --left) {
    int best = 0;
    for (int j = 1; j < n; ++j)
      if (frac[j] >= frac[best]) best = j;
    ++m[best];
    frac[best] = -1.0;
  }
  return m;
}

void Flux2Transformer2DModel::set_tensor_parallel(int rank, int nranks, const std::vector<double>& ratios) {
  if (nranks < 1 || rank < 0 || rank >= nranks) fail(DCPP_ERR_INVALID_ARG, "bad tensor-parallel rank");
  if (nranks > 8) fail(DCPP_ERR_UNSUPPORTED, "tensor parallelism over at most 8 GPUs");
  for (auto* w : weights_)
    if (w->type >= 0) fail(DCPP_ERR_STATE, "set_tensor_parallel must come before set_param");
  std::vector<double> f = ratios.empty() ? std::vector<double>(static_cast<size_t>(nranks), 1.0) : ratios;
  if (static_cast<int>(f.size()) != nranks) fail(DCPP_ERR_INVALID_ARG, "tensor split: one ratio per rank");
  const int64_t H = cfg_.num_attention_heads;
  const int64_t F = cfg_.mlp_hidden();
  if (F % 64) fail(DCPP_ERR_UNSUPPORTED, "mlp hidden must be a multiple of 64");
  // Two ratio groups: whole heads (q / k / v rows, to_out columns) and MLP
  // features in units of 64 (the gate / up interleave of the fused GEMM).
  const auto heads = plan_tensor_split(H, f);
  const auto mlp = plan_tensor_split(F / 64, f);
  for (int j = 0; j < nranks; ++j)
    if (heads[j] < 1 || mlp[j] < 1)
      fail(DCPP_ERR_UNSUPPORTED, "tensor split leaves rank " + std::to_string(j) +
                                     " without a head or 64 MLP features (" + std::to_string(H) + " heads over " +
                                     std::to_string(nranks) + " ranks)");
  int64_t h0 = 0, u0 = 0;
  for (int j = 0; j < rank; ++j) {
    h0 += heads[j];
    u0 += mlp[j];
  }
  rank_ = rank;
  nranks_ = nranks;
  h0_ = h0;
  hn_ = heads[rank];
  f0_ = u0 * 64;
  fn_ = mlp[rank] * 64;
  build_registry();
}

void Flux2Transformer2DModel::build_registry() {
  weights_.clear();
  vectors_.clear();
  setters_.clear();
  D_ = cfg_.inner_dim();
  F_ = cfg_.mlp_hidden();
  H_ = cfg_.num_attention_heads;
  if (nranks_ == 1) {
    h0_ = f0_ = 0;
    hn_ = H_;
    fn_ = F_;
  }
  Hl_ = hn_;
  Dl_ = hn_ * cfg_.attention_head_dim;
  Fl_ = fn_;
  const int64_t D = D_, F = F_, Dl = Dl_, Fl = Fl_;
  const int64_t d0 = h0_ * cfg_.attention_head_dim, f0 = f0_;  // this rank's first q/k/v row and MLP feature
  const int64_t tg = cfg_.timestep_guidance_channels;

  auto init = [&](DevWeight& w, const std::string& name, int64_t rows, int64_t cols, std::set<std::string> parts) {
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
  };
  using RowMap = std::function<int64_t(int64_t)>;
  using Cols = std::vector<std::array<int64_t, 3>>;
  auto ident = [](int64_t i) { return i; };
  // Register `name` with full shape [rows, cols] feeding part `part` of w.
  auto reg = [&](const std::string& name, DevWeight* w, const std::string& part, int64_t rows, int64_t cols,
                 RowMap map, Cols cols_ranges) {
    setters_[name] = [this, w, part, rows, cols, map, cols_ranges, name](int type, const std::vector<int64_t>& shape,
                                                                         const void* data, size_t nbytes) {
      if (shape.size() != 2 || shape[0] != rows || shape[1] != cols)
        fail(DCPP_ERR_INVALID_ARG, "Error while loading Tensor '" + name + "': Parameter shape mismatch: expected " +
                                       shape_str({rows, cols}) + ", got " + shape_str(shape));
      if (!is_gemm_type(type)) fail(DCPP_ERR_UNSUPPORTED, "Tensor '" + name + "': unsupported type");
      const size_t need = row_bytes_of(type, cols) * static_cast<size_t>(rows);
      if (nbytes != need)
        fail(DCPP_ERR_INVALID_ARG, "Tensor '" + name + "': expected " + std::to_string(need) + " bytes, got " +
                                       std::to_string(nbytes));
      place_rows(*w, part, type, shape, static_cast<const uint8_t*>(data), map, cols_ranges);
    };
  };
  auto full_cols = [](int64_t c) { return Cols{{0, c, 0}}; };
  // Rows of a [D, *] head-major projection kept by this rank, placed at region g.
  auto head_rows = [=](int g) {
    return RowMap([=](int64_t i) { return (i >= d0 && i < d0 + Dl) ? g * Dl + (i - d0) : -1; });
  };
  // Rows of a [F, *] gate/up projection kept by this rank, interleaved in
  // 64-row blocks (gate block j, up block j, ...) after `base` rows.
  auto mlp_rows = [=](int64_t base, bool up) {
    return RowMap([=](int64_t i) {
      if (i < f0 || i >= f0 + Fl) return int64_t(-1);
      const int64_t j = i - f0;
      return base + (j / 64) * 128 + (up ? 64 : 0) + (j % 64);
    });
  };

  init(time1_, "time_guidance_embed.timestep_embedder.linear_1.weight", D, tg, {"all"});
  init(time2_, "time_guidance_embed.timestep_embedder.linear_2.weight", D, D, {"all"});
  reg(time1_.name, &time1_, "all", D, tg, ident, full_cols(tg));
  reg(time2_.name, &time2_, "all", D, D, ident, full_cols(D));
  if (cfg_.guidance_embeds) {
    init(guid1_, "time_guidance_embed.guidance_embedder.linear_1.weight", D, tg, {"all"});
    init(guid2_, "time_guidance_embed.guidance_embedder.linear_2.weight", D, D, {"all"});
    reg(guid1_.name, &guid1_, "all", D, tg, ident, full_cols(tg));
    reg(guid2_.name, &guid2_, "all", D, D, ident, full_cols(D));
  }
  init(mod_img_, "double_stream_modulation_img.linear.weight", 6 * D, D, {"all"});
  init(mod_txt_, "double_stream_modulation_txt.linear.weight", 6 * D, D, {"all"});
  init(mod_single_, "single_stream_modulation.linear.weight", 3 * D, D, {"all"});
  reg(mod_img_.name, &mod_img_, "all", 6 * D, D, ident, full_cols(D));
  reg(mod_txt_.name, &mod_txt_, "all", 6 * D, D, ident, full_cols(D));
  reg(mod_single_.name, &mod_single_, "all", 3 * D, D, ident, full_cols(D));
  init(x_embed_, "x_embedder.weight", D, cfg_.in_channels, {"all"});
  init(ctx_embed_, "context_embedder.weight", D, cfg_.joint_attention_dim, {"all"});
  reg(x_embed_.name, &x_embed_, "all", D, cfg_.in_channels, ident, full_cols(cfg_.in_channels));
  reg(ctx_embed_.name, &ctx_embed_, "all", D, cfg_.joint_attention_dim, ident, full_cols(cfg_.joint_attention_dim));
  init(norm_out_, "norm_out.linear.weight", 2 * D, D, {"all"});
  init(proj_out_, "proj_out.weight", cfg_.out_ch(), D, {"all"});
  reg(norm_out_.name, &norm_out_, "all", 2 * D, D, ident, full_cols(D));
  reg(proj_out_.name, &proj_out_, "all", cfg_.out_ch(), D, ident, full_cols(D));

  dbl_.assign(static_cast<size_t>(cfg_.num_layers), DoubleBlock());
  for (int64_t b = 0; b < cfg_.num_layers; ++b) {
    DoubleBlock& blk = dbl_[b];
    const std::string p = "transformer_blocks." + std::to_string(b) + ".";
    const char* stream_qkv[2][3] = {{"attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj"},
                                    {"attn.to_q", "attn.to_k", "attn.to_v"}};
    const char* stream_out[2] = {"attn.to_add_out", "attn.to_out.0"};
    const char* stream_ff[2] = {"ff_context", "ff"};
    const char* nq[2] = {"attn.norm_added_q", "attn.norm_q"};
    const char* nk[2] = {"attn.norm_added_k", "attn.norm_k"};
    for (int s = 0; s < 2; ++s) {
      init(blk.qkv[s], p + (s ? "attn.to_qkv" : "attn.add_qkv"), 3 * Dl, D, {"q", "k", "v"});
      for (int g = 0; g < 3; ++g)
        reg(p + stream_qkv[s][g] + ".weight", &blk.qkv[s], std::string(1, "qkv"[g]), D, D, head_rows(g), full_cols(D));
      init(blk.out[s], p + stream_out[s] + ".weight", D, Dl, {"all"});
      reg(p + stream_out[s] + ".weight", &blk.out[s], "all", D, D, ident, Cols{{d0, Dl, 0}});
      const std::string ff = p + stream_ff[s];
      init(blk.ff_in[s], ff + ".linear_in.weight", 2 * Fl, D, {"gate", "up"});
      // fused GGUF tensor [2F, D]: rows [0, F) gate, [F, 2F) up (GGUFLoaderVisitor.cpp:370-408)
      {
        DevWeight* w = &blk.ff_in[s];
        auto gate = mlp_rows(0, false), up = mlp_rows(0, true);
        const std::string fname = ff + ".linear_in.weight";
        setters_[fname] = [this, w, gate, up, D, F, fname](int type, const std::vector<int64_t>& shape,
                                                            const void* data, size_t nbytes) {
          if (shape.size() != 2 || shape[0] != 2 * F || shape[1] != D)
            fail(DCPP_ERR_INVALID_ARG, "Error while loading Tensor '" + fname +
                                           "': Parameter shape mismatch: expected " + shape_str({2 * F, D}) +
                                           ", got " + shape_str(shape));
          const size_t rb = row_bytes_of(type, D);
          if (nbytes != rb * 2 * F) fail(DCPP_ERR_INVALID_ARG, "Tensor '" + fname + "': byte size mismatch");
          const uint8_t* src = static_cast<const uint8_t*>(data);
          place_rows(*w, "gate", type, {F, D}, src, gate, Cols{{0, D, 0}});
          place_rows(*w, "up", type, {F, D}, src + rb * F, up, Cols{{0, D, 0}});
        };
      }
      reg(ff + ".linear_in_gate.weight", &blk.ff_in[s], "gate", F, D, mlp_rows(0, false), full_cols(D));
      reg(ff + ".linear_in_up.weight", &blk.ff_in[s], "up", F, D, mlp_rows(0, true), full_cols(D));
      init(blk.ff_out[s], ff + ".linear_out.weight", D, Fl, {"all"});
      reg(ff + ".linear_out.weight", &blk.ff_out[s], "all", D, F, ident, Cols{{f0, Fl, 0}});
      initv(blk.norm_q[s], p + nq[s] + ".weight", cfg_.attention_head_dim);
      initv(blk.norm_k[s], p + nk[s] + ".weight", cfg_.attention_head_dim);
    }
  }
  sgl_.assign(static_cast<size_t>(cfg_.num_single_layers), SingleBlock());
  for (int64_t b = 0; b < cfg_.num_single_layers; ++b) {
    SingleBlock& blk = sgl_[b];
    const std::string p = "single_transformer_blocks." + std::to_string(b) + ".attn.";
    init(blk.qkv_mlp, p + "to_qkv_mlp_proj.weight", 3 * Dl + 2 * Fl, D, {"q", "k", "v", "gate", "up"});
    {
      DevWeight* w = &blk.qkv_mlp;
      const std::string fname = p + "to_qkv_mlp_proj.weight";
      std::array<RowMap, 3> hr = {head_rows(0), head_rows(1), head_rows(2)};
      auto gate = mlp_rows(3 * Dl, false), up = mlp_rows(3 * Dl, true);
      // fused GGUF tensor [3D + 2F, D]: rows q | k | v | gate | up (GGUFLoaderVisitor.cpp:283-329)
      setters_[fname] = [this, w, hr, gate, up, D, F, fname](int type, const std::vector<int64_t>& shape,
                                                             const void* data, size_t nbytes) {
        if (shape.size() != 2 || shape[0] != 3 * D + 2 * F || shape[1] != D)
          fail(DCPP_ERR_INVALID_ARG, "Error while loading Tensor '" + fname + "': Parameter shape mismatch: expected " +
                                         shape_str({3 * D + 2 * F, D}) + ", got " + shape_str(shape));
        const size_t rb = row_bytes_of(type, D);
        if (nbytes != rb * (3 * D + 2 * F)) fail(DCPP_ERR_INVALID_ARG, "Tensor '" + fname + "': byte size mismatch");
        const uint8_t* src = static_cast<const uint8_t*>(data);
        for (int g = 0; g < 3; ++g) place_rows(*w, std::string(1, "qkv"[g]), type, {D, D}, src + rb * g * D, hr[g], Cols{{0, D, 0}});
        place_rows(*w, "gate", type, {F, D}, src + rb * 3 * D, gate, Cols{{0, D, 0}});
        place_rows(*w, "up", type, {F, D}, src + rb * (3 * D + F), up, Cols{{0, D, 0}});
      };
    }
    for (int g = 0; g < 3; ++g)
      reg(p + "to_qkv_mlp_proj." + std::string(1, "qkv"[g]) + ".weight", &blk.qkv_mlp, std::string(1, "qkv"[g]), D, D,
          head_rows(g), full_cols(D));
    reg(p + "to_qkv_mlp_proj.mlp_in_gate.weight", &blk.qkv_mlp, "gate", F, D, mlp_rows(3 * Dl, false), full_cols(D));
    reg(p + "to_qkv_mlp_proj.mlp_in_up.weight", &blk.qkv_mlp, "up", F, D, mlp_rows(3 * Dl, true), full_cols(D));
    init(blk.out, p + "to_out.weight", D, Dl + Fl, {"attn", "mlp"});
    {
      DevWeight* w = &blk.out;
      const std::string fname = p + "to_out.weight";
      // fused GGUF tensor [D, D + F]: columns attn | mlp (GGUFLoaderVisitor.cpp:331-368)
      setters_[fname] = [this, w, D, F, Dl, Fl, d0, f0, fname](int type, const std::vector<int64_t>& shape,
                                                          const void* data, size_t nbytes) {
        if (shape.size() != 2 || shape[0] != D || shape[1] != D + F)
          fail(DCPP_ERR_INVALID_ARG, "Error while loading Tensor '" + fname + "': Parameter shape mismatch: expected " +
                                         shape_str({D, D + F}) + ", got " + shape_str(shape));
        if (nbytes != row_bytes_of(type, D + F) * D) fail(DCPP_ERR_INVALID_ARG, "Tensor '" + fname + "': byte size mismatch");
        const uint8_t* src = static_cast<const uint8_t*>(data);
        auto id = [](int64_t i) { return i; };
        place_rows(*w, "attn", type, shape, src, id, Cols{{d0, Dl, 0}});
        place_rows(*w, "mlp", type, shape, src, id, Cols{{D + f0, Fl, Dl}});
      };
    }
    reg(p + "to_out.attn.weight", &blk.out, "attn", D, D, ident, Cols{{d0, Dl, 0}});
    reg(p + "to_out.mlp.weight", &blk.out, "mlp", D, F, ident, Cols{{f0, Fl, Dl}});
    initv(blk.norm_q, p + "norm_q.weight", cfg_.attention_head_dim);
    initv(blk.norm_k, p + "norm_k.weight", cfg_.attention_head_dim);
  }
  // The block projections run on the fused-dequant GEMM.
  for (auto& blk : dbl_)
    for (int s = 0; s < 2; ++s)
      for (DevWeight* w : {&blk.qkv[s], &blk.out[s], &blk.ff_in[s], &blk.ff_out[s]}) w->pack = true;
  for (auto& blk : sgl_) {
    blk.qkv_mlp.pack = true;
    blk.out.pack = true;
  }
  for (auto* v : vectors_) {
    DevVector* pv = v;
    setters_[v->name] = [this, pv](int type, const std::vector<int64_t>& shape, const void* data, size_t nbytes) {
      set_vector(*pv, type, shape, data, nbytes);
    };
  }
}

void Flux2Transformer2DModel::place_rows(DevWeight& w, const std::string& part, int type,
                                         const std::vector<int64_t>& shape, const uint8_t* src,
                                         const std::function<int64_t(int64_t)>& row_map,
                                         const std::vector<std::array<int64_t, 3>>& col_ranges) {
  if (!w.need.count(part)) fail(DCPP_ERR_STATE, "Tensor '" + w.name + "': part '" + part + "' set twice");
  {
    // A tensor-parallel column shard that does not fall on quantisation
    // block boundaries (e.g. Q4_K's 256 columns vs 384-column head shards)
    // cannot be sliced in the block format: expand those rows to bf16 on the
    // host (exact dequantised values, rounded once), as the GEMM would.
    const int64_t qbs = block_size_of(type);
    bool unaligned = w.cols % qbs != 0;
    for (auto& cr : col_ranges) unaligned = unaligned || cr[0] % qbs || cr[1] % qbs || cr[2] % qbs;
    // Parts already placed in a quantised type are expanded as well, so one
    // fused weight always ends up in one type.
    if ((unaligned && qbs > 1) || (type == kTypeBF16 && block_size_of(w.type) > 1)) expand_staging_bf16(w);
    if (qbs > 1 && (unaligned || w.type == kTypeBF16)) {
      std::vector<uint16_t> conv(static_cast<size_t>(shape[0]) * shape[1]);
      const size_t src_rb_q = row_bytes_of(type, shape[1]);
      std::vector<float> rowf(static_cast<size_t>(shape[1]));
      for (int64_t i = 0; i < shape[0]; ++i) {
        if (row_map(i) < 0) continue;
        host_dequant_row(type, src + static_cast<size_t>(i) * src_rb_q, shape[1], rowf.data());
        for (int64_t c = 0; c < shape[1]; ++c) conv[static_cast<size_t>(i) * shape[1] + c] = host_f32_to_bf16(rowf[c]);
      }
      place_rows(w, part, kTypeBF16, shape, reinterpret_cast<const uint8_t*>(conv.data()), row_map, col_ranges);
      return;
    }
  }
  if (w.type >= 0 && w.type != type)
    fail(DCPP_ERR_UNSUPPORTED, "Tensor '" + w.name + "': parts of one fused weight must share a ggml type");
  const int64_t bs = block_size_of(type);
  const size_t bb = block_bytes_of(type);
  if (w.cols % bs) fail(DCPP_ERR_UNSUPPORTED, "Tensor '" + w.name + "': columns not block aligned for this type");
  for (auto& cr : col_ranges)
    if (cr[0] % bs || cr[1] % bs || cr[2] % bs)
      fail(DCPP_ERR_UNSUPPORTED, "Tensor '" + w.name + "': column shard not aligned to the quantisation block");
  if (w.type < 0) {
    w.type = type;
    w.row_bytes = row_bytes_of(type, w.cols);
    w.staging.assign(w.row_bytes * static_cast<size_t>(w.rows), 0);
  }
  const size_t src_rb = row_bytes_of(type, shape[1]);
  for (int64_t i = 0; i < shape[0]; ++i) {
    const int64_t d = row_map(i);
    if (d < 0) continue;
    if (d >= w.rows) fail(DCPP_ERR_STATE, "internal: row map out of range for " + w.name);
    for (auto& cr : col_ranges) {
      const size_t so = static_cast<size_t>(cr[0] / bs) * bb;
      const size_t n = static_cast<size_t>(cr[1] / bs) * bb;
      const size_t dof = static_cast<size_t>(cr[2] / bs) * bb;
      memcpy(w.staging.data() + static_cast<size_t>(d) * w.row_bytes + dof, src + static_cast<size_t>(i) * src_rb + so, n);
    }
  }
  w.need.erase(part);
  if (w.need.empty()) finish_weight(w);
}

void Flux2Transformer2DModel::expand_staging_bf16(DevWeight& w) {
  if (w.type < 0 || block_size_of(w.type) == 1) return;
  std::vector<uint8_t> conv(static_cast<size_t>(w.rows) * w.cols * 2);
  std::vector<float> rowf(static_cast<size_t>(w.cols));
  for (int64_t i = 0; i < w.rows; ++i) {
    host_dequant_row(w.type, w.staging.data() + static_cast<size_t>(i) * w.row_bytes, w.cols, rowf.data());
    auto* dst = reinterpret_cast<uint16_t*>(conv.data()) + static_cast<size_t>(i) * w.cols;
    for (int64_t c = 0; c < w.cols; ++c) dst[c] = host_f32_to_bf16(rowf[c]);
  }
  w.type = kTypeBF16;
  w.row_bytes = static_cast<size_t>(w.cols) * 2;
  w.staging.swap(conv);
}

void Flux2Transformer2DModel::finish_weight(DevWeight& w) {
  if (host_only_) {  // keep the assembled rows on the host (read_param)
    w.on_host = true;
    return;
  }
  const size_t bytes = w.staging.size();
  if (cudaMalloc(&w.data, bytes) != cudaSuccess) {
    cudaGetLastError();
    w.data = nullptr;
    fail(DCPP_ERR_OOM, "weight allocation failed for " + w.name);
  }
  cuda_check(cudaMemcpy(w.data, w.staging.data(), bytes, cudaMemcpyHostToDevice), "upload weight");
  std::vector<uint8_t>().swap(w.staging);
  // Block projections in Q4_K / Q8_0 are kept only in the packed stage layout
  // that the fused-dequant GEMM reads (packed once here, on the device).
  const bool packable = (w.type == kTypeQ4_K && w.cols % 256 == 0) || (w.type == kTypeQ8_0 && w.cols % 64 == 0);
  if (w.pack && packable && fused_dequant_) {
    const size_t pb = packed_bytes(w.type, w.rows, w.cols);
    if (cudaMalloc(&w.packed, pb) != cudaSuccess) {
      cudaGetLastError();
      w.packed = nullptr;
      fail(DCPP_ERR_OOM, "packed weight allocation failed for " + w.name);
    }
    cuda_check(launch_pack_weight(w.type, w.data, w.rows, w.cols, w.packed, ctx_.stream), "pack weight");
    cuda_check(cudaStreamSynchronize(ctx_.stream), "pack weight");
    cuda_check(cudaFree(w.data), "free raw weight");
    w.data = nullptr;
  }
  planned_ = false;
}

void Flux2Transformer2DModel::set_vector(DevVector& v, int type, const std::vector<int64_t>& shape, const void* data,
                                         size_t nbytes) {
  set_vector_param(v, type, shape, data, nbytes, host_only_);
  planned_ = false;
}

void Flux2Transformer2DModel::set_param(const std::string& name, int type, const std::vector<int64_t>& shape,
                                        const void* data, size_t nbytes) {
  auto it = setters_.find(name);
  if (it == setters_.end()) fail(DCPP_ERR_NOT_FOUND, "Error while loading Tensor '" + name + "': Tensor not found");
  if (!data) fail(DCPP_ERR_INVALID_ARG, "Tensor '" + name + "': null data");
  it->second(type, shape, data, nbytes);
}

void Flux2Transformer2DModel::require_device(const char* what) const {
  if (host_only_) fail(DCPP_ERR_STATE, std::string(what) + ": a host-only model cannot execute");
}

void Flux2Transformer2DModel::read_param(const std::string& name, int* type, int64_t* rows, int64_t* cols, void* dst,
                                         size_t cap, size_t* nbytes) {
  for (auto* w : weights_) {
    if (w->name != name) continue;
    if (!w->ready()) fail(DCPP_ERR_STATE, "parameter '" + name + "' is not fully set");
    if (w->packed) fail(DCPP_ERR_UNSUPPORTED, "parameter '" + name + "' is held only in the packed GEMM layout");
    const size_t n = w->row_bytes * static_cast<size_t>(w->rows);
    if (type) *type = w->type;
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (nbytes) *nbytes = n;
    if (!dst) return;
    if (cap < n) fail(DCPP_ERR_INVALID_ARG, "read_param: buffer too small for '" + name + "'");
    if (w->on_host) {
      memcpy(dst, w->staging.data(), n);
    } else {
      cuda_check(cudaStreamSynchronize(ctx_.stream), "read_param");
      cuda_check(cudaMemcpy(dst, w->data, n, cudaMemcpyDeviceToHost), "read_param");
    }
    return;
  }
  for (auto* v : vectors_) {
    if (v->name != name) continue;
    if (!v->set) fail(DCPP_ERR_STATE, "parameter '" + name + "' is not set");
    const size_t n = static_cast<size_t>(v->n) * sizeof(float);
    if (type) *type = kTypeF32;
    if (rows) *rows = 1;
    if (cols) *cols = v->n;
    if (nbytes) *nbytes = n;
    if (!dst) return;
    if (cap < n) fail(DCPP_ERR_INVALID_ARG, "read_param: buffer too small for '" + name + "'");
    if (host_only_) {
      memcpy(dst, v->host.data(), n);
    } else {
      cuda_check(cudaStreamSynchronize(ctx_.stream), "read_param");
      cuda_check(cudaMemcpy(dst, v->data, n, cudaMemcpyDeviceToHost), "read_param");
    }
    return;
  }
  fail(DCPP_ERR_NOT_FOUND, "read_param: no parameter named '" + name + "'");
}

std::vector<std::string> Flux2Transformer2DModel::missing() const {
  std::vector<std::string> m;
  for (auto* w : weights_)
    for (auto& p : w->need) m.push_back(w->name + (p == "all" ? "" : " [" + p + "]"));
  for (auto* v : vectors_)
    if (!v->set) m.push_back(v->name);
  return m;
}

// ----------------------------------------------------------------- plan
void Flux2Transformer2DModel::free_plan() {
  if (graph_fwd_) cudaGraphExecDestroy(graph_fwd_);
  for (auto& g : graph_step_)
    if (g) cudaGraphExecDestroy(g);
  graph_fwd_ = nullptr;
  graph_step_[0] = graph_step_[1] = nullptr;
  for (void* p : allocs_) cudaFree(p);
  allocs_.clear();
  sym_.close(ctx_);
  release_plan_events();
  for (int j = 0; j < 8; ++j) {
    ag_flags_peer_[j] = nullptr;
    recv_peer_[j] = nullptr;
    a_peer_[j] = nullptr;
    flags_peer_[0][j] = flags_peer_[1][j] = nullptr;
  }
  epoch_[0] = epoch_[1] = nullptr;
  ag_count_ = step_dev_ = nullptr;
  overlap_ = false;
  ops_fwd_.clear();
  step_ops_[0].clear();
  step_ops_[1].clear();
  last_ops_ = nullptr;
  planned_ = false;
}

void Flux2Transformer2DModel::prepare(int64_t batch, int64_t n_img, int64_t n_txt, bool use_graph, int64_t n_ref) {
  require_device("prepare");
  auto miss = missing();
  if (!miss.empty()) fail(DCPP_ERR_STATE, "parameters not set: " + miss.front() + " (+" + std::to_string(miss.size() - 1) + " more)");
  if (batch < 1 || batch > 4) fail(DCPP_ERR_UNSUPPORTED, "batch must be 1..4");
  if (n_img < 1 || n_txt < 1) fail(DCPP_ERR_INVALID_ARG, "token counts must be positive");
  if (n_ref < 0) fail(DCPP_ERR_INVALID_ARG, "the reference token count must not be negative");
  if ((batch * (n_img + n_ref + n_txt)) > (1 << 24)) fail(DCPP_ERR_UNSUPPORTED, "too many tokens");
  if (planned_ && batch == B_ && n_img == Nl_ && n_ref == Nr_ && n_txt == Nt_ && use_graph == use_graph_) return;
  cudaStreamSynchronize(ctx_.stream);
  free_plan();
  B_ = batch;
  Nl_ = n_img;
  Nr_ = n_ref;
  Ni_ = n_img + n_ref;
  Nt_ = n_txt;
  S_ = Ni_ + n_txt;
  use_graph_ = use_graph;
  build_plan();
  planned_ = true;
}





void Flux2Transformer2DModel::add_allreduce(float* buf, int64_t count) {
  Ctx* c = &ctx_;
  building_->push_back({[buf, count, c](cudaStream_t s) {
                          auto& n = Nccl::get();
                          int r = n.AllReduce(buf, buf, static_cast<size_t>(count), 7, 0, c->comm, s);
                          if (r != 0) fail(DCPP_ERR_NCCL, std::string("ncclAllReduce: ") + n.GetErrorString(r));
                        },
                        0, kOpAllreduce, 0.0, "nccl_allreduce"});
}




std::vector<const DevWeight*> Flux2Transformer2DModel::block_weights(size_t k) const {
  if (k < dbl_.size()) {
    const DoubleBlock& b = dbl_[k];
    return {&b.qkv[0], &b.qkv[1], &b.out[0], &b.out[1], &b.ff_in[0], &b.ff_in[1], &b.ff_out[0], &b.ff_out[1]};
  }
  const SingleBlock& b = sgl_[k - dbl_.size()];
  return {&b.qkv_mlp, &b.out};
}

void Flux2Transformer2DModel::add_tp_barrier(int set, int stream) {
  TpBarrierArgs a{};
  for (int j = 0; j < nranks_; ++j) a.flags[j] = flags_peer_[set][j];
  a.epoch = epoch_[set];
  a.err = ctx_.d_err;
  a.rank = rank_;
  a.nranks = nranks_;
  a.timeout_ns = ctx_.wait_timeout_ns;
  Op o{[a](cudaStream_t s) { cuda_check(launch_tp_barrier(a, s), "tp barrier"); }, 1, kOpAllreduce, 0.0, "tp_barrier"};
  o.stream = stream;
  building_->push_back(o);
}

void Flux2Transformer2DModel::build_plan() {
  const int64_t B = B_, S = S_, Ni = Ni_, Nt = Nt_, Nl = Nl_, D = D_, Dl = Dl_, Fl = Fl_, Hl = Hl_;
  const int64_t R = B * S;
  const int64_t ldc = Dl + Fl;
  const int64_t in_ch = cfg_.in_channels, jd = cfg_.joint_attention_dim, out_ch = cfg_.out_ch();
  const int64_t tg = cfg_.timestep_guidance_channels;
  const bool tp = nranks_ > 1;
  if (tp && !ctx_.comm) fail(DCPP_ERR_STATE, "tensor-parallel model needs dcpp_tp_init on its context");
  if (tp && (ctx_.nranks != nranks_ || ctx_.rank != rank_))
    fail(DCPP_ERR_STATE, "model tensor-parallel rank/size differ from the context's dcpp_tp_init");
  const bool peer = tp && tp_peer_;
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
  part_ = tp && !peer ? static_cast<float*>(alloc(R * D * 4)) : nullptr;
  if (peer) {
    // One IPC-mapped block per rank: a_ | recv slots | barrier flags (2 sets).
    // Two row pieces pay off once the per-site exchange is large and spread
    // over >= 4 GPUs (measured at 8 GPUs: config 3, B*S*D = 37.7 M, gains
    // 2%; config 2, 14.2 M, loses 7%; at 2 GPUs one piece is faster).
    // Overlapped all-gather: the granule flags' epochs give each step
    // kAgSitesPerStep - 1 sites.
    overlap_ = tp_overlap_ && !tp_pull_ && ctx_.use_pair(R) && !fused_dequant_ &&
               2 * cfg_.num_layers + cfg_.num_single_layers < static_cast<int64_t>(kAgSitesPerStep) - 1;
    tp_pieces_ = overlap_ ? 1
                          : (tp_pieces_env_ > 0 ? tp_pieces_env_
                                                : (nranks_ >= 4 && R * D >= (int64_t{24} << 20) ? 2 : 1));
    piece_rows_ = (R + tp_pieces_ - 1) / tp_pieces_;
    chunk_ = (piece_rows_ + nranks_ - 1) / nranks_;
    const int64_t ngr = (R + kGranuleRows - 1) / kGranuleRows;
    own_max_ = (ngr + nranks_ - 1) / nranks_;
    auto up = [](size_t b) { return (b + 255) & ~static_cast<size_t>(255); };
    const size_t off_recv = up(R * D * 2);
    // recv: the push form's receive slots (by chunk or, overlapped, by
    // granule), or the pull form's full-row partials.
    const size_t recv_bytes = std::max<size_t>(
        std::max<size_t>(static_cast<size_t>(nranks_) * tp_pieces_ * chunk_ * D * 2, static_cast<size_t>(R) * D * 2),
        static_cast<size_t>(nranks_) * own_max_ * kGranuleRows * D * 2);
    const size_t off_flags = off_recv + up(recv_bytes);
    const size_t off_ag = off_flags + 512;  // per-granule arrival flags
    sym_.open(ctx_, off_ag + up(static_cast<size_t>(ngr) * 4));
    for (int j = 0; j < nranks_; ++j) {
      a_peer_[j] = reinterpret_cast<uint16_t*>(sym_.peer[j]);
      recv_peer_[j] = reinterpret_cast<uint16_t*>(sym_.peer[j] + off_recv);
      flags_peer_[0][j] = reinterpret_cast<uint32_t*>(sym_.peer[j] + off_flags);
      flags_peer_[1][j] = reinterpret_cast<uint32_t*>(sym_.peer[j] + off_flags + 256);
      ag_flags_peer_[j] = reinterpret_cast<uint32_t*>(sym_.peer[j] + off_ag);
    }
    ag_count_ = static_cast<uint32_t*>(alloc(static_cast<size_t>(kAgSitesPerStep) * own_max_ * 4));
    step_dev_ = static_cast<uint32_t*>(alloc(256));
    cuda_check(cudaMemsetAsync(step_dev_, 0, 256, ctx_.stream), "clear step counter");
    a_ = a_peer_[rank_];
    epoch_[0] = static_cast<uint32_t*>(alloc(256));
    epoch_[1] = epoch_[0] + 32;
    cuda_check(cudaMemsetAsync(epoch_[0], 0, 256, ctx_.stream), "clear epoch");
    // Every rank's flags are zero before any rank's first barrier.
    cuda_check(cudaStreamSynchronize(ctx_.stream), "peer buffers");
    float* one = static_cast<float*>(alloc(256));
    auto& nc = Nccl::get();
    int rc = nc.AllReduce(one, one, 1, 7, 0, ctx_.comm, ctx_.stream);
    if (rc != 0) fail(DCPP_ERR_NCCL, std::string("ncclAllReduce: ") + nc.GetErrorString(rc));
    cuda_check(cudaStreamSynchronize(ctx_.stream), "peer buffers");
  } else {
    a_ = static_cast<uint16_t*>(alloc(R * D * 2));
  }
  q_ = static_cast<uint16_t*>(alloc(R * Dl * 2));
  k_ = static_cast<uint16_t*>(alloc(R * Dl * 2));
  // V is kept transposed, [B, Hl, 128, Sp] with Sp = S rounded up to 64;
  // the padding columns stay zero (finite) for the attention's P.V MMA.
  const int64_t sp = attn_vt_stride(S);
  v_ = static_cast<uint16_t*>(alloc(B * Hl * 128 * sp * 2));
  cuda_check(cudaMemset(v_, 0, B * Hl * 128 * sp * 2), "memset vt");
  cat_ = static_cast<uint16_t*>(alloc(R * ldc * 2));
  xb_ = static_cast<uint16_t*>(alloc(B * Ni * in_ch * 2));
  eb_ = static_cast<uint16_t*>(alloc(B * Nt * jd * 2));
  lat_[0] = static_cast<float*>(alloc(B * Ni * std::max(in_ch, out_ch) * 4));
  lat_[1] = static_cast<float*>(alloc(B * Ni * std::max(in_ch, out_ch) * 4));
  out_dev_ = static_cast<float*>(alloc(B * Ni * out_ch * 4));
  enc_in_ = static_cast<float*>(alloc(B * Nt * jd * 4));
  float* scal = static_cast<float*>(alloc(64 * 4));
  t_dev_ = scal;
  g_dev_ = scal + 8;
  dt_dev_ = scal + 16;
  ids_dev_ = static_cast<int32_t*>(alloc(S * cfg_.axes_dims_rope.size() * 4));
  rope_ = static_cast<float2*>(alloc(S * 64 * sizeof(float2)));
  tproj_ = static_cast<float*>(alloc(B * tg * 4));
  th_ = static_cast<float*>(alloc(B * D * 4));
  temb_ = static_cast<float*>(alloc(B * D * 4));
  gproj_ = static_cast<float*>(alloc(B * tg * 4));
  gh_ = static_cast<float*>(alloc(B * D * 4));
  gemb_ = static_cast<float*>(alloc(B * D * 4));
  mod_img_v_ = static_cast<float*>(alloc(B * 6 * D * 4));
  mod_txt_v_ = static_cast<float*>(alloc(B * 6 * D * 4));
  mod_s_v_ = static_cast<float*>(alloc(B * 3 * D * 4));
  mod_o_v_ = static_cast<float*>(alloc(B * 2 * D * 4));
  // Weight expansion scratch (bf16) for quantised GEMM weights.
  // Only GEMM weights that are neither bf16 nor packed need it; the
  // conditioning GEMVs read their raw GGUF rows directly.
  size_t s0 = 0, s1 = 0;
  auto needs = [](const DevWeight* w) { return w->type != kTypeBF16 && !w->packed; };
  for (const DevWeight* w : {&x_embed_, &ctx_embed_, &proj_out_})
    if (needs(w)) s0 = std::max(s0, static_cast<size_t>(w->rows * w->cols));
  // Block weights: expanded a whole block ahead (block_weights / add_prefetch)
  // into two block-sized sets, or, with block prefetch off, each projection
  // right before its GEMM into the per-GEMM scratch pairs.
  size_t pf = 0;
  for (size_t k = 0; k < dbl_.size() + sgl_.size(); ++k) {
    size_t n = 0;
    for (const DevWeight* w : block_weights(k))
      if (needs(w)) n += (static_cast<size_t>(w->rows * w->cols) + 127) / 128 * 128;
    pf = std::max(pf, n);
  }
  if (block_prefetch_) {
    alloc_prefetch_scratch(alloc, pf);
  } else {
    alloc_prefetch_scratch(alloc, 0);
    for (auto& blk : dbl_)
      for (int s = 0; s < 2; ++s)
        for (const DevWeight* w : {&blk.qkv[s], &blk.out[s], &blk.ff_in[s], &blk.ff_out[s]})
          if (needs(w)) (s == 0 ? s1 : s0) = std::max(s == 0 ? s1 : s0, static_cast<size_t>(w->rows * w->cols));
    for (auto& blk : sgl_)
      for (const DevWeight* w : {&blk.qkv_mlp, &blk.out})
        if (needs(w)) s0 = std::max(s0, static_cast<size_t>(w->rows * w->cols));
  }
  alloc_expansion_scratch(alloc, s0, s1);

  const int n_axes = static_cast<int>(cfg_.axes_dims_rope.size());
  std::array<int32_t, 8> axes{};
  for (int i = 0; i < n_axes; ++i) axes[i] = static_cast<int32_t>(cfg_.axes_dims_rope[i]);
  const float theta = static_cast<float>(cfg_.rope_theta);
  const float eps = cfg_.eps;

  // Row groups over the joint [txt | img] buffer: one per (batch, stream).
  auto stream_groups = [&](bool both_streams) {
    std::vector<GemmGroup> g;
    for (int64_t b = 0; b < B; ++b) {
      GemmGroup t{};
      t.row0 = t.orow0 = static_cast<int32_t>(b * S);
      t.rows = static_cast<int32_t>(Nt);
      t.wsel = 0;
      t.sel = 0;
      t.batch = static_cast<int32_t>(b);
      t.tok0 = 0;
      GemmGroup i = t;
      i.row0 = i.orow0 = static_cast<int32_t>(b * S + Nt);
      i.rows = static_cast<int32_t>(Ni);
      i.wsel = both_streams ? 1 : 0;
      i.sel = 1;
      i.tok0 = static_cast<int32_t>(Nt);
      g.push_back(t);
      g.push_back(i);
    }
    return g;
  };
  // img_only: only the first img_rows image tokens of each batch element
  // (norm_out), written to rows b * Ni of y.
  auto norm_args = [&](const float* const* mods, int64_t mod_stride, int64_t shift_off, int64_t scale_off,
                       bool img_only, uint16_t* y, int64_t dst_ld, const float* resid, int64_t img_rows) {
    NormArgs n{};
    n.x = h_;
    n.x_out = h_;
    n.resid = resid;
    n.y = y;
    n.ld_x = D;
    n.ld_y = dst_ld;
    n.D = static_cast<int32_t>(D);
    n.eps = eps;
    int k = 0;
    for (int64_t b = 0; b < B; ++b) {
      if (!img_only) {
        const float* m = mods[0] + b * mod_stride;
        n.seg[k++] = {static_cast<int32_t>(b * S), static_cast<int32_t>(b * S), static_cast<int32_t>(Nt), m + shift_off,
                      m + scale_off};
      }
      const float* m = mods[1] + b * mod_stride;
      const int32_t dst = img_only ? static_cast<int32_t>(b * Ni) : static_cast<int32_t>(b * S + Nt);
      n.seg[k++] = {static_cast<int32_t>(b * S + Nt), dst, static_cast<int32_t>(img_only ? img_rows : Ni), m + shift_off,
                    m + scale_off};
    }
    n.n_segments = k;
    return n;
  };

  const size_t n_blocks = dbl_.size() + sgl_.size();
  auto build_ops = [&](std::vector<Op>& ops, float* lat_in, float* lat_out, bool euler) {
    begin_ops(ops);
    // Block-ahead expansion: block 0's quantised weights from the start of
    // the step (under the conditioning GEMVs and embedders), block k + 1's
    // while block k's attention runs (after its QKV GEMM, when the set that
    // block k - 1 used is free).  The attention leaves HBM and most issue
    // slots idle; expansions beside a GEMM slow it instead.
    if (overlap_)
      ops.push_back({[=](cudaStream_t s) {
                       cuda_check(launch_step_counter(step_dev_, s), "step counter");
                       cuda_check(cudaMemsetAsync(ag_count_, 0, static_cast<size_t>(kAgSitesPerStep) * own_max_ * 4, s),
                                  "clear all-gather counts");
                     },
                     1});
    size_t blk_idx = 0;
    auto prefetch_next = [&]() {
      if (block_prefetch_ && blk_idx + 1 < n_blocks) add_prefetch(block_weights(blk_idx + 1), static_cast<int>((blk_idx + 1) & 1));
      ++blk_idx;
    };
    if (block_prefetch_ && n_blocks) add_prefetch(block_weights(0), 0);
    // 1. timestep (and guidance) embedding, modulation vectors
    //    (Flux2Transformer2DModel.cpp:130-145).
    ops.push_back({[=](cudaStream_t s) {
                     cuda_check(launch_timestep_proj(t_dev_, static_cast<int>(B), static_cast<int>(tg), 1000.0f, tproj_, s),
                                "timestep_proj");
                   },
                   1});
    add_gemv(time1_, tproj_, static_cast<int>(B), 0, 1, th_);
    add_gemv(time2_, th_, static_cast<int>(B), 0, 0, temb_);
    if (guidance_given_) {
      ops.push_back({[=](cudaStream_t s) {
                       cuda_check(launch_timestep_proj(g_dev_, static_cast<int>(B), static_cast<int>(tg), 1000.0f, gproj_, s),
                                  "guidance_proj");
                     },
                     1});
      add_gemv(guid1_, gproj_, static_cast<int>(B), 0, 1, gh_);
      add_gemv(guid2_, gh_, static_cast<int>(B), 0, 0, gemb_);
      ops.push_back({[=](cudaStream_t s) { cuda_check(launch_add_f32(temb_, gemb_, B * D, s), "add"); }, 1});
    }
    add_gemv(mod_img_, temb_, static_cast<int>(B), 1, 0, mod_img_v_);
    add_gemv(mod_txt_, temb_, static_cast<int>(B), 1, 0, mod_txt_v_);
    add_gemv(mod_single_, temb_, static_cast<int>(B), 1, 0, mod_s_v_);
    add_gemv(norm_out_, temb_, static_cast<int>(B), 1, 0, mod_o_v_);
    // 2. input projections into the joint residual stream h = [txt | img].
    ops.push_back({[=](cudaStream_t s) {
                     cuda_check(launch_f32_to_bf16(lat_in, B * Ni * in_ch, xb_, s), "to_bf16");
                     cuda_check(launch_f32_to_bf16(enc_in_, B * Nt * jd, eb_, s), "to_bf16");
                   },
                   2});
    {
      std::vector<GemmGroup> gi, gt;
      for (int64_t b = 0; b < B; ++b) {
        GemmGroup g{};
        g.row0 = static_cast<int32_t>(b * Ni);
        g.orow0 = static_cast<int32_t>(b * S + Nt);
        g.rows = static_cast<int32_t>(Ni);
        g.batch = static_cast<int32_t>(b);
        gi.push_back(g);
        g.row0 = static_cast<int32_t>(b * Nt);
        g.orow0 = static_cast<int32_t>(b * S);
        g.rows = static_cast<int32_t>(Nt);
        gt.push_back(g);
      }
      EpilogueArgs e{};
      e.mode = kEpiF32;
      e.out_f32 = h_;
      e.ld_out = D;
      add_gemm("x_embedder", xb_, in_ch, in_ch, &x_embed_, nullptr, gi, e, D);
      add_gemm("context_embedder", eb_, jd, jd, &ctx_embed_, nullptr, gt, e, D);
    }
    // 3. rotary table from cat(txt_ids, img_ids) (Flux2Transformer2DModel.cpp:164-169).
    ops.push_back({[=](cudaStream_t s) {
                     cuda_check(launch_rope_table(ids_dev_, S, n_axes, axes.data(), theta, rope_, s), "rope_table");
                   },
                   1});
    AttnTcArgs at{};
    at.o = cat_;
    at.ld_o = ldc;
    at.B = static_cast<int32_t>(B);
    at.H = static_cast<int32_t>(Hl);
    at.S = static_cast<int32_t>(S);
    at.scale = 1.0f / std::sqrt(static_cast<float>(cfg_.attention_head_dim));
    at.err = ctx_.d_err;
    at.kernel = ctx_.attn_kernel;
    auto maps = std::make_shared<AttnTcMaps>();
    cuda_check(make_attn_maps(maps.get(), q_, k_, v_, static_cast<int>(B), static_cast<int>(Hl), static_cast<int>(S)),
               "attention tensor maps");
    auto attn_op = [&]() {
      ops.push_back({[at, maps](cudaStream_t s) { cuda_check(launch_attention_tc(*maps, at, s), "attention"); }, 1,
                     kOpAttention, 4.0 * at.B * at.H * static_cast<double>(at.S) * static_cast<double>(at.S) * 128.0,
                     "attention"});
    };
    auto out_epi = [&](const float* g0, const float* g1, int64_t bstride) {
      EpilogueArgs e{};
      e.mode = tp ? (peer ? kEpiGatePeer : kEpiGateF32) : kEpiResidGate;
      e.out_f32 = tp ? part_ : h_;
      e.ld_out = D;
      e.gate[0] = g0;
      e.gate[1] = g1;
      e.gate_bstride = bstride;
      if (peer && tp_pull_) {
        // Pull form: the gated bf16 partial stays in this GPU's own memory
        // (one piece of R rows owned by slot 0 = this buffer); the owners
        // read it over NVLink in their LayerNorm.
        e.peer_bf16[0] = recv_peer_[rank_];
        e.chunk_rows = static_cast<int32_t>(R);
        e.piece_rows = static_cast<int32_t>(R);
        e.slot_rows = static_cast<int32_t>(R);
        e.peer_slot = 0;
      } else if (peer) {
        for (int j = 0; j < nranks_; ++j) e.peer_bf16[j] = recv_peer_[j];
        e.chunk_rows = static_cast<int32_t>(chunk_);
        e.piece_rows = static_cast<int32_t>(piece_rows_);
        e.slot_rows = static_cast<int32_t>(overlap_ ? own_max_ * kGranuleRows : tp_pieces_ * chunk_);
        e.peer_slot = rank_;
        e.gran_n = overlap_ ? nranks_ : 0;
      }
      return e;
    };
    // The exchange after a row-parallel GEMM, the LayerNorm that consumes it
    // and the GEMM that consumes the LayerNorm.  NCCL: all-reduce the
    // partials, every rank normalises every row.  Peer: a barrier (partials
    // landed); per row piece, the owner of each row sums its slots into the
    // residual and stores the normalised row into every rank's `a`; a
    // barrier (rows landed) before the GEMM reads that piece.  With two
    // pieces, piece 1's LayerNorm + all-gather runs on the side stream while
    // the GEMM works on piece 0.
    bool pending = false;
    auto site = [&]() {
      if (!tp) return;
      if (peer) add_tp_barrier(0, 0);
      else add_allreduce(part_, R * D);
      pending = true;
    };
    auto piece_range = [&](int p) {
      const int64_t lo = p * piece_rows_;
      return std::array<int64_t, 2>{lo, std::min<int64_t>(R, lo + piece_rows_)};
    };
    auto own_range = [&](int p) {
      const auto pr = piece_range(p);
      const int64_t lo = std::min<int64_t>(pr[1], pr[0] + rank_ * chunk_);
      return std::array<int64_t, 2>{lo, std::min<int64_t>(pr[1], lo + chunk_)};
    };
    // Granule form (overlap_): the segments stay whole; the kernel walks this
    // rank's 128-row granules.  push_rows: also store every row into the other
    // GPUs' buffers (for a LayerNorm whose GEMM is not overlapped).
    auto gran_norm = [&](NormArgs n, bool push_rows) {
      n.gran_rank = rank_;
      n.gran_n = nranks_;
      n.n_slots = nranks_;
      n.slots = recv_peer_[rank_];
      n.slot_stride = own_max_ * kGranuleRows * D;
      n.n_peer_out = 0;
      if (push_rows)
        for (int j = 0; j < nranks_; ++j)
          if (j != rank_) n.y_peer[n.n_peer_out++] = a_peer_[j] + (n.y - a_);
      return n;
    };
    int ag_site = 0;
    // The all-gather of this rank's rows of `a` (which the LayerNorm just
    // wrote) runs inside the next GEMM: its two push warps per CTA store the
    // rows into the other GPUs, its producer waits for their granules.
    auto ag_push = [&]() {
      AgWait w{};
      w.flags = ag_flags_peer_[rank_];
      w.step = step_dev_;
      w.site = ag_site;
      w.rank = rank_;
      w.n = nranks_;
      w.rows = static_cast<int32_t>(R);
      w.ld = D;
      w.a = a_;
      for (int j = 0; j < nranks_; ++j) {
        w.a_peer[j] = a_peer_[j];
        w.flags_peer[j] = ag_flags_peer_[j];
      }
      w.count = ag_count_ + static_cast<size_t>(ag_site) * own_max_;
      next_ag_ = w;
      ++ag_site;
    };
    auto peer_norm = [&](NormArgs n, int p) {
      const auto own = own_range(p);
      int k = 0;
      for (int i = 0; i < n.n_segments; ++i) {
        NormSegment sg = n.seg[i];
        const int64_t a0 = std::max<int64_t>(own[0], sg.src_row0), a1 = std::min<int64_t>(own[1], sg.src_row0 + sg.rows);
        if (a1 <= a0) continue;
        sg.dst_row0 += static_cast<int32_t>(a0 - sg.src_row0);
        sg.src_row0 = static_cast<int32_t>(a0);
        sg.rows = static_cast<int32_t>(a1 - a0);
        n.seg[k++] = sg;
      }
      n.n_segments = k;
      n.n_slots = nranks_;
      if (tp_pull_) {  // every rank's full-row partial, read from its memory
        for (int j = 0; j < nranks_; ++j) n.slot_ptr[j] = recv_peer_[j];
        n.slot_row0 = 0;
      } else {
        n.slots = recv_peer_[rank_];
        n.slot_stride = tp_pieces_ * chunk_ * D;
        n.slot_row0 = own[0] - p * chunk_;  // slot row of source row r: p * chunk + (r - own[0])
      }
      n.n_peer_out = 0;
      for (int j = 0; j < nranks_; ++j)
        if (j != rank_) n.y_peer[n.n_peer_out++] = a_peer_[j] + (n.y - a_);
      return n;
    };
    auto split_groups = [&](const std::vector<GemmGroup>& groups) {
      std::vector<std::vector<GemmGroup>> out(tp_pieces_);
      for (int p = 0; p < tp_pieces_; ++p) {
        const auto pr = piece_range(p);
        for (GemmGroup g : groups) {
          const int64_t a0 = std::max<int64_t>(pr[0], g.row0), a1 = std::min<int64_t>(pr[1], g.row0 + g.rows);
          if (a1 <= a0) continue;
          const int32_t d = static_cast<int32_t>(a0 - g.row0);
          g.row0 += d;
          g.orow0 += d;
          g.tok0 += d;
          g.rows = static_cast<int32_t>(a1 - a0);
          out[p].push_back(g);
        }
      }
      return out;
    };
    using Emit = std::function<void(const std::vector<std::vector<GemmGroup>>&, const std::function<void(int)>&)>;
    // joint_rows: the LayerNorm writes row r of `a` from row r of h (block
    // norms); norm_out drops the text rows, so its GEMM is not split.
    auto norm_gemm = [&](NormArgs n, bool joint_rows, const std::vector<GemmGroup>& groups, const Emit& emit) {
      if (!(pending && peer)) {
        if (pending) n.resid = part_;
        add_norm(n);
        pending = false;
        emit({groups}, nullptr);
        return;
      }
      pending = false;
      if (overlap_) {
        add_norm(gran_norm(n, !joint_rows));
        if (joint_rows) {
          ag_push();
        } else {
          add_tp_barrier(0, 0);
        }
        emit({groups}, nullptr);
        return;
      }
      if (!joint_rows || tp_pieces_ == 1) {
        for (int p = 0; p < tp_pieces_; ++p) {
          NormArgs q = peer_norm(n, p);
          if (q.n_segments) add_norm(q);
        }
        add_tp_barrier(0, 0);
        emit({groups}, nullptr);
        return;
      }
      cudaEvent_t ln0 = plan_event(), done1 = plan_event();
      emit(split_groups(groups), [&, n, ln0, done1](int p) {
        if (p == 0) {
          NormArgs q0 = peer_norm(n, 0);
          if (q0.n_segments) add_norm(q0);
          add_record(ln0, 0);
          add_tp_barrier(0, 0);
          add_wait(ln0, 1);
          NormArgs q1 = peer_norm(n, 1);
          if (q1.n_segments) add_norm(q1, 1);
          add_tp_barrier(1, 1);
          add_record(done1, 1);
        } else {
          add_wait(done1, 0);
        }
      });
    };
    const float* mods_dbl[2] = {mod_txt_v_, mod_img_v_};
    // 4. double-stream blocks (Flux2TransformerBlock.hpp:45-117).
    for (auto& blk : dbl_) {
      EpilogueArgs e{};
      e.mode = kEpiQkvMlp;
      e.qkv_cols = static_cast<int32_t>(3 * Dl);
      e.inner = static_cast<int32_t>(Dl);
      e.seq = static_cast<int32_t>(S);
      e.heads = static_cast<int32_t>(Hl);
      e.norm_q[0] = blk.norm_q[0].data;
      e.norm_q[1] = blk.norm_q[1].data;
      e.norm_k[0] = blk.norm_k[0].data;
      e.norm_k[1] = blk.norm_k[1].data;
      e.eps = eps;
      e.rope = rope_;
      e.q_out = q_;
      e.k_out = k_;
      e.v_out = v_;
      e.vt_stride = sp;
      e.mlp_out = cat_ + Dl;
      e.ld_mlp = ldc;
      norm_gemm(norm_args(mods_dbl, 6 * D, 0, D, false, a_, D, nullptr, Ni), true, stream_groups(true),
                [&](const std::vector<std::vector<GemmGroup>>& pcs, const std::function<void(int)>& hook) {
                  add_gemm_pieces("qkv", a_, D, D, &blk.qkv[0], &blk.qkv[1], pcs, e, 3 * Dl, hook);
                });
      prefetch_next();
      attn_op();
      add_gemm("attn_out", cat_, ldc, Dl, &blk.out[0], &blk.out[1], stream_groups(true),
               out_epi(mod_txt_v_ + 2 * D, mod_img_v_ + 2 * D, 6 * D), D);
      site();
      EpilogueArgs f = e;
      f.qkv_cols = 0;
      norm_gemm(norm_args(mods_dbl, 6 * D, 3 * D, 4 * D, false, a_, D, nullptr, Ni), true, stream_groups(true),
                [&](const std::vector<std::vector<GemmGroup>>& pcs, const std::function<void(int)>& hook) {
                  add_gemm_pieces("ff_in", a_, D, D, &blk.ff_in[0], &blk.ff_in[1], pcs, f, 2 * Fl, hook);
                });
      add_gemm("ff_out", cat_ + Dl, ldc, Fl, &blk.ff_out[0], &blk.ff_out[1], stream_groups(true),
               out_epi(mod_txt_v_ + 5 * D, mod_img_v_ + 5 * D, 6 * D), D);
      site();
    }
    // 5. single-stream blocks on the joint stream (Flux2SingleTransformerBlock.hpp:36-72).
    const float* mods_s[2] = {mod_s_v_, mod_s_v_};
    for (auto& blk : sgl_) {
      EpilogueArgs e{};
      e.mode = kEpiQkvMlp;
      e.qkv_cols = static_cast<int32_t>(3 * Dl);
      e.inner = static_cast<int32_t>(Dl);
      e.seq = static_cast<int32_t>(S);
      e.heads = static_cast<int32_t>(Hl);
      e.norm_q[0] = e.norm_q[1] = blk.norm_q.data;
      e.norm_k[0] = e.norm_k[1] = blk.norm_k.data;
      e.eps = eps;
      e.rope = rope_;
      e.q_out = q_;
      e.k_out = k_;
      e.v_out = v_;
      e.vt_stride = sp;
      e.mlp_out = cat_ + Dl;
      e.ld_mlp = ldc;
      norm_gemm(norm_args(mods_s, 3 * D, 0, D, false, a_, D, nullptr, Ni), true, stream_groups(false),
                [&](const std::vector<std::vector<GemmGroup>>& pcs, const std::function<void(int)>& hook) {
                  add_gemm_pieces("qkv_mlp", a_, D, D, &blk.qkv_mlp, nullptr, pcs, e, 3 * Dl + 2 * Fl, hook);
                });
      prefetch_next();
      attn_op();
      add_gemm("out", cat_, ldc, Dl + Fl, &blk.out, nullptr, stream_groups(false),
               out_epi(mod_s_v_ + 2 * D, mod_s_v_ + 2 * D, 3 * D), D);
      site();
    }
    // 6. drop text tokens, norm_out (scale first, then shift; AdaLayerNormContinuous.inl:26-43), proj_out.
    //    The denoise step also drops the reference tokens: only the Nl latent
    //    tokens of each batch element are integrated (Flux2KleinPipeline.cpp:531-536).
    const float* mods_o[2] = {mod_o_v_, mod_o_v_};
    {
      const int64_t out_rows = euler ? Nl : Ni;
      std::vector<GemmGroup> g;
      for (int64_t b = 0; b < B; ++b) {
        GemmGroup gg{};
        gg.row0 = gg.orow0 = static_cast<int32_t>(b * Ni);
        gg.rows = static_cast<int32_t>(out_rows);
        gg.batch = static_cast<int32_t>(b);
        g.push_back(gg);
      }
      EpilogueArgs e{};
      e.ld_out = out_ch;
      if (euler) {
        e.mode = kEpiEuler;
        e.out_f32 = lat_out;
        e.x_in = lat_in;
        e.dt = dt_dev_;
      } else {
        e.mode = kEpiF32;
        e.out_f32 = lat_out;
      }
      norm_gemm(norm_args(mods_o, 2 * D, D, 0, true, a_, D, nullptr, out_rows), false, g,
                [&](const std::vector<std::vector<GemmGroup>>& pcs, const std::function<void(int)>& hook) {
                  add_gemm_pieces("proj_out", a_, D, D, &proj_out_, nullptr, pcs, e, out_ch, hook);
                });
    }
    end_ops();
  };
  guidance_given_ = cfg_.guidance_embeds;
  build_ops(ops_fwd_, lat_[0], out_dev_, false);
  // The Euler step needs noise prediction and latents of the same shape.
  if (cfg_.out_ch() == cfg_.in_channels) {
    build_ops(step_ops_[0], lat_[0], lat_[1], true);
    build_ops(step_ops_[1], lat_[1], lat_[0], true);
  }
  launches_per_step_ = 0;
  for (auto& o : (step_ops_[0].empty() ? ops_fwd_ : step_ops_[0])) launches_per_step_ += o.launches;
}

}  // namespace dcpp

namespace dcpp {

// ----------------------------------------------------------------- execution

void Flux2Transformer2DModel::copy_inputs(const float* hidden, const float* encoder, const float* timestep,
                                          const int32_t* img_ids, const int32_t* txt_ids, const float* guidance) {
  cudaStream_t s = ctx_.stream;
  const size_t na = cfg_.axes_dims_rope.size();
  if (hidden)
    cuda_check(cudaMemcpyAsync(lat_[cur_], hidden, B_ * Ni_ * cfg_.in_channels * 4, cudaMemcpyDefault, s), "copy hidden");
  if (encoder)
    cuda_check(cudaMemcpyAsync(enc_in_, encoder, B_ * Nt_ * cfg_.joint_attention_dim * 4, cudaMemcpyDefault, s),
               "copy encoder");
  if (timestep) cuda_check(cudaMemcpyAsync(t_dev_, timestep, B_ * 4, cudaMemcpyDefault, s), "copy timestep");
  if (guidance) cuda_check(cudaMemcpyAsync(g_dev_, guidance, B_ * 4, cudaMemcpyDefault, s), "copy guidance");
  if (txt_ids) cuda_check(cudaMemcpyAsync(ids_dev_, txt_ids, Nt_ * na * 4, cudaMemcpyDefault, s), "copy txt_ids");
  if (img_ids)
    cuda_check(cudaMemcpyAsync(ids_dev_ + Nt_ * na, img_ids, Ni_ * na * 4, cudaMemcpyDefault, s), "copy img_ids");
}

void Flux2Transformer2DModel::forward(const float* hidden, const float* encoder, const float* timestep,
                                      const int32_t* img_ids, const int32_t* txt_ids, const float* guidance,
                                      float* out) {
  if (!planned_) fail(DCPP_ERR_STATE, "forward before prepare");
  if (!hidden || !encoder || !timestep || !img_ids || !txt_ids || !out) fail(DCPP_ERR_INVALID_ARG, "forward: null input");
  if (cfg_.guidance_embeds && !guidance) fail(DCPP_ERR_INVALID_ARG, "forward: guidance required (guidance_embeds)");
  cur_ = 0;
  copy_inputs(hidden, encoder, timestep, img_ids, txt_ids, guidance);
  run_ops(ops_fwd_, &graph_fwd_);
  cuda_check(cudaMemcpyAsync(out, out_dev_, B_ * Ni_ * cfg_.out_ch() * 4, cudaMemcpyDefault, ctx_.stream), "copy out");
  ctx_.check_device_error();
}

void Flux2Transformer2DModel::copy_latents(const float* latents, int buf) {
  const size_t C = static_cast<size_t>(cfg_.in_channels) * 4;
  cuda_check(cudaMemcpy2DAsync(lat_[buf], Ni_ * C, latents, Nl_ * C, Nl_ * C, B_, cudaMemcpyDefault, ctx_.stream),
             "copy latents");
}

void Flux2Transformer2DModel::copy_ref(const float* ref_latents, const int32_t* ref_ids) {
  if (Nr_ == 0) return;
  const size_t C = static_cast<size_t>(cfg_.in_channels) * 4;
  for (int k = 0; k < 2; ++k)
    cuda_check(cudaMemcpy2DAsync(reinterpret_cast<uint8_t*>(lat_[k]) + Nl_ * C, Ni_ * C, ref_latents, Nr_ * C, Nr_ * C,
                                 B_, cudaMemcpyDefault, ctx_.stream),
               "copy reference latents");
  const size_t na = cfg_.axes_dims_rope.size();
  cuda_check(cudaMemcpyAsync(ids_dev_ + (Nt_ + Nl_) * na, ref_ids, Nr_ * na * 4, cudaMemcpyDefault, ctx_.stream),
             "copy reference ids");
}

void Flux2Transformer2DModel::copy_latents_out(float* out, int buf) {
  const size_t C = static_cast<size_t>(cfg_.in_channels) * 4;
  cuda_check(cudaMemcpy2DAsync(out, Nl_ * C, lat_[buf], Ni_ * C, Nl_ * C, B_, cudaMemcpyDefault, ctx_.stream),
             "copy latents");
}

void Flux2Transformer2DModel::check_ref_args(const float* ref_latents, const int32_t* ref_ids, const char* what) const {
  if (Nr_ > 0 && (!ref_latents || !ref_ids))
    fail(DCPP_ERR_INVALID_ARG, std::string(what) + ": the plan has " + std::to_string(Nr_) +
                                   " reference tokens, so image_latents and image_latent_ids are required");
  if (Nr_ == 0 && (ref_latents || ref_ids))
    fail(DCPP_ERR_INVALID_ARG, std::string(what) + ": reference latents given but the plan has no reference tokens "
                                                   "(prepare with n_ref > 0)");
}

void Flux2Transformer2DModel::denoise(const float* latents, const float* ref_latents, const int32_t* ref_ids,
                                      const float* encoder, const float* timestep, float dt, const int32_t* img_ids,
                                      const int32_t* txt_ids, float* latents_out) {
  if (!planned_) fail(DCPP_ERR_STATE, "denoise before prepare");
  if (step_ops_[0].empty()) fail(DCPP_ERR_UNSUPPORTED, "denoise needs out_channels == in_channels");
  if (cfg_.guidance_embeds) fail(DCPP_ERR_UNSUPPORTED, "denoise passes no guidance (Flux2KleinPipeline.cpp:527)");
  if (!latents || !encoder || !timestep || !img_ids || !txt_ids || !latents_out)
    fail(DCPP_ERR_INVALID_ARG, "denoise: null input");
  check_ref_args(ref_latents, ref_ids, "denoise");
  cur_ = 0;
  copy_latents(latents, 0);
  copy_ref(ref_latents, ref_ids);
  const size_t na = cfg_.axes_dims_rope.size();
  copy_inputs(nullptr, encoder, timestep, nullptr, txt_ids, nullptr);
  cuda_check(cudaMemcpyAsync(ids_dev_ + Nt_ * na, img_ids, Nl_ * na * 4, cudaMemcpyDefault, ctx_.stream), "copy img_ids");
  cuda_check(cudaMemcpyAsync(dt_dev_, &dt, 4, cudaMemcpyHostToDevice, ctx_.stream), "copy dt");
  run_ops(step_ops_[0], &graph_step_[0]);
  copy_latents_out(latents_out, 1);
  ctx_.check_device_error();
}

void Flux2Transformer2DModel::load_inputs(const float* latents, const float* ref_latents, const int32_t* ref_ids,
                                          const float* encoder, const int32_t* img_ids, const int32_t* txt_ids) {
  if (!planned_) fail(DCPP_ERR_STATE, "load_inputs before prepare");
  check_ref_args(ref_latents, ref_ids, "load_inputs");
  cur_ = 0;
  if (latents) copy_latents(latents, 0);
  copy_ref(ref_latents, ref_ids);
  const size_t na = cfg_.axes_dims_rope.size();
  copy_inputs(nullptr, encoder, nullptr, nullptr, txt_ids, nullptr);
  if (img_ids)
    cuda_check(cudaMemcpyAsync(ids_dev_ + Nt_ * na, img_ids, Nl_ * na * 4, cudaMemcpyDefault, ctx_.stream),
               "copy img_ids");
}

void Flux2Transformer2DModel::set_timestep(float timestep, float dt) {
  if (!planned_) fail(DCPP_ERR_STATE, "set_timestep before prepare");
  float host[8];
  for (int64_t b = 0; b < B_; ++b) host[b] = timestep;
  cuda_check(cudaMemcpyAsync(t_dev_, host, B_ * 4, cudaMemcpyHostToDevice, ctx_.stream), "copy timestep");
  cuda_check(cudaMemcpyAsync(dt_dev_, &dt, 4, cudaMemcpyHostToDevice, ctx_.stream), "copy dt");
}

void Flux2Transformer2DModel::run_resident_step() {
  if (!planned_) fail(DCPP_ERR_STATE, "run before prepare");
  if (step_ops_[0].empty()) fail(DCPP_ERR_UNSUPPORTED, "denoise needs out_channels == in_channels");
  run_ops(step_ops_[cur_], &graph_step_[cur_]);
  cur_ ^= 1;
}

void Flux2Transformer2DModel::set_profiling(bool on) {
  require_device("set_profiling");
  if (on == profiling_) return;
  cudaStreamSynchronize(ctx_.stream);
  free_plan();
  profiling_ = on;
}


void Flux2Transformer2DModel::read_latents(float* out) {
  if (!planned_) fail(DCPP_ERR_STATE, "read_latents before prepare");
  copy_latents_out(out, cur_);
  ctx_.check_device_error();
}

}  // namespace dcpp

// ----------------------------------------------------------------- C ABI
namespace {

template <class F>
dcpp_status model_call(dcpp_flux2* m, const char* entry, F&& f) {
  if (!m || !m->ctx) return DCPP_ERR_INVALID_ARG;
  dcpp_ctx* ctx = m->ctx;
  try {
    ctx->maybe_inject(entry);
    if (ctx->device >= 0) cudaSetDevice(ctx->device);
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

void dcpp_flux2_config_default(dcpp_flux2_config* cfg) {
  if (cfg) dcpp::Flux2Config().to_c(*cfg);
}

dcpp_status dcpp_flux2_config_from_file(const char* path, dcpp_flux2_config* cfg) {
  if (!path || !cfg) return DCPP_ERR_INVALID_ARG;
  try {
    dcpp::Flux2Config::from_file(path).to_c(*cfg);
    return DCPP_OK;
  } catch (const dcpp::Error& e) {
    return e.status;
  } catch (const std::exception&) {
    return DCPP_ERR_INVALID_ARG;
  }
}

dcpp_status dcpp_flux2_create(dcpp_ctx* ctx, const dcpp_flux2_config* cfg, dcpp_flux2** out) {
  if (!ctx || !cfg || !out) return DCPP_ERR_INVALID_ARG;
  *out = nullptr;
  try {
    ctx->maybe_inject("dcpp_flux2_create");
    cudaSetDevice(ctx->device);
    auto* m = new dcpp_flux2();
    m->ctx = ctx;
    try {
      m->model.reset(new dcpp::Flux2Transformer2DModel(*ctx, dcpp::Flux2Config::from_c(*cfg)));
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

dcpp_status dcpp_flux2_create_host(const dcpp_flux2_config* cfg, dcpp_flux2** out) {
  if (!cfg || !out) return DCPP_ERR_INVALID_ARG;
  *out = nullptr;
  auto* m = new dcpp_flux2();
  m->own_ctx.reset(new dcpp_ctx());
  m->own_ctx->device = -1;
  m->ctx = m->own_ctx.get();
  try {
    m->model.reset(new dcpp::Flux2Transformer2DModel(*m->ctx, dcpp::Flux2Config::from_c(*cfg), true));
  } catch (const dcpp::Error& e) {
    delete m;
    return e.status;
  } catch (const std::exception&) {
    delete m;
    return DCPP_ERR_INVALID_ARG;
  }
  *out = m;
  return DCPP_OK;
}

const char* dcpp_flux2_last_error(dcpp_flux2* m) {
  if (!m || !m->ctx) return "invalid model handle";
  return m->ctx->last_error.c_str();
}

dcpp_status dcpp_flux2_read_param(dcpp_flux2* m, const char* name, int* type, int64_t* rows, int64_t* cols, void* dst,
                                  size_t cap, size_t* nbytes) {
  return model_call(m, "dcpp_flux2_read_param", [&](dcpp::Flux2Transformer2DModel& mm) {
    if (!name) dcpp::fail(DCPP_ERR_INVALID_ARG, "read_param: null name");
    mm.read_param(name, type, rows, cols, dst, cap, nbytes);
  });
}

dcpp_status dcpp_flux2_destroy(dcpp_flux2* m) {
  if (!m) return DCPP_ERR_INVALID_ARG;
  if (m->ctx && m->ctx->device >= 0) cudaSetDevice(m->ctx->device);
  delete m;
  return DCPP_OK;
}

dcpp_status dcpp_flux2_set_param(dcpp_flux2* m, const char* name, int type, int n_dims, const int64_t* shape,
                                 const void* data, size_t nbytes) {
  return model_call(m, "dcpp_flux2_set_param", [&](dcpp::Flux2Transformer2DModel& mm) {
    if (!name || !shape || n_dims < 1 || n_dims > 4) dcpp::fail(DCPP_ERR_INVALID_ARG, "set_param: bad name or shape");
    mm.set_param(name, type, std::vector<int64_t>(shape, shape + n_dims), data, nbytes);
  });
}

dcpp_status dcpp_flux2_missing(dcpp_flux2* m, int* count, char* first, size_t cap) {
  return model_call(m, "dcpp_flux2_missing", [&](dcpp::Flux2Transformer2DModel& mm) {
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

dcpp_status dcpp_flux2_prepare(dcpp_flux2* m, int64_t batch, int64_t n_img, int64_t n_txt, int use_graph) {
  return model_call(m, "dcpp_flux2_prepare",
                    [&](dcpp::Flux2Transformer2DModel& mm) { mm.prepare(batch, n_img, n_txt, use_graph != 0); });
}

dcpp_status dcpp_flux2_forward(dcpp_flux2* m, const float* hidden, const float* encoder, const float* timestep,
                               const int32_t* img_ids, const int32_t* txt_ids, const float* guidance, float* out) {
  return model_call(m, "dcpp_flux2_forward", [&](dcpp::Flux2Transformer2DModel& mm) {
    mm.forward(hidden, encoder, timestep, img_ids, txt_ids, guidance, out);
  });
}

dcpp_status dcpp_flux2_denoise_step(dcpp_flux2* m, const float* latents_in, const float* encoder,
                                    const float* timestep, float dt, const int32_t* img_ids, const int32_t* txt_ids,
                                    float* latents_out) {
  return model_call(m, "dcpp_flux2_denoise_step", [&](dcpp::Flux2Transformer2DModel& mm) {
    mm.denoise(latents_in, nullptr, nullptr, encoder, timestep, dt, img_ids, txt_ids, latents_out);
  });
}

dcpp_status dcpp_flux2_prepare_ref(dcpp_flux2* m, int64_t batch, int64_t n_img, int64_t n_ref, int64_t n_txt,
                                   int use_graph) {
  return model_call(m, "dcpp_flux2_prepare_ref", [&](dcpp::Flux2Transformer2DModel& mm) {
    mm.prepare(batch, n_img, n_txt, use_graph != 0, n_ref);
  });
}

dcpp_status dcpp_flux2_denoise_step_ref(dcpp_flux2* m, const float* latents_in, const float* image_latents,
                                        const int32_t* image_latent_ids, const float* encoder, const float* timestep,
                                        float dt, const int32_t* img_ids, const int32_t* txt_ids, float* latents_out) {
  return model_call(m, "dcpp_flux2_denoise_step_ref", [&](dcpp::Flux2Transformer2DModel& mm) {
    mm.denoise(latents_in, image_latents, image_latent_ids, encoder, timestep, dt, img_ids, txt_ids, latents_out);
  });
}

dcpp_status dcpp_flux2_load_inputs_ref(dcpp_flux2* m, const float* latents, const float* image_latents,
                                       const int32_t* image_latent_ids, const float* encoder, const int32_t* img_ids,
                                       const int32_t* txt_ids) {
  return model_call(m, "dcpp_flux2_load_inputs_ref", [&](dcpp::Flux2Transformer2DModel& mm) {
    mm.load_inputs(latents, image_latents, image_latent_ids, encoder, img_ids, txt_ids);
  });
}

dcpp_status dcpp_flux2_load_inputs(dcpp_flux2* m, const float* latents, const float* encoder, const int32_t* img_ids,
                                   const int32_t* txt_ids) {
  return model_call(m, "dcpp_flux2_load_inputs", [&](dcpp::Flux2Transformer2DModel& mm) {
    mm.load_inputs(latents, nullptr, nullptr, encoder, img_ids, txt_ids);
  });
}

dcpp_status dcpp_flux2_set_timestep(dcpp_flux2* m, float timestep, float dt) {
  return model_call(m, "dcpp_flux2_set_timestep",
                    [&](dcpp::Flux2Transformer2DModel& mm) { mm.set_timestep(timestep, dt); });
}

dcpp_status dcpp_flux2_run_resident(dcpp_flux2* m) {
  return model_call(m, "dcpp_flux2_run_resident", [&](dcpp::Flux2Transformer2DModel& mm) { mm.run_resident_step(); });
}

dcpp_status dcpp_flux2_read_latents(dcpp_flux2* m, float* out) {
  return model_call(m, "dcpp_flux2_read_latents", [&](dcpp::Flux2Transformer2DModel& mm) { mm.read_latents(out); });
}

dcpp_status dcpp_flux2_launches_per_step(dcpp_flux2* m, int64_t* out) {
  return model_call(m, "dcpp_flux2_launches_per_step", [&](dcpp::Flux2Transformer2DModel& mm) {
    if (!out) dcpp::fail(DCPP_ERR_INVALID_ARG, "null output");
    *out = mm.launches_per_step();
  });
}

dcpp_status dcpp_flux2_set_profiling(dcpp_flux2* m, int on) {
  return model_call(m, "dcpp_flux2_set_profiling", [&](dcpp::Flux2Transformer2DModel& mm) { mm.set_profiling(on != 0); });
}

dcpp_status dcpp_flux2_profile(dcpp_flux2* m, int kind, double* ms, double* flops, int64_t* launches) {
  return model_call(m, "dcpp_flux2_profile", [&](dcpp::Flux2Transformer2DModel& mm) {
    if (kind < 0 || kind >= dcpp::Flux2Transformer2DModel::kOpKinds) dcpp::fail(DCPP_ERR_INVALID_ARG, "bad kind");
    mm.profile(kind, ms, flops, launches);
  });
}

dcpp_status dcpp_flux2_set_tensor_parallel(dcpp_flux2* m, int rank, int nranks) {
  return model_call(m, "dcpp_flux2_set_tensor_parallel",
                    [&](dcpp::Flux2Transformer2DModel& mm) { mm.set_tensor_parallel(rank, nranks); });
}

dcpp_status dcpp_flux2_set_tensor_split(dcpp_flux2* m, int rank, int nranks, const float* ratios) {
  return model_call(m, "dcpp_flux2_set_tensor_split", [&](dcpp::Flux2Transformer2DModel& mm) {
    std::vector<double> f;
    if (ratios) f.assign(ratios, ratios + std::max(nranks, 0));
    mm.set_tensor_parallel(rank, nranks, f);
  });
}

dcpp_status dcpp_flux2_shard(dcpp_flux2* m, int64_t* head0, int64_t* heads, int64_t* mlp0, int64_t* mlp_features) {
  return model_call(m, "dcpp_flux2_shard", [&](dcpp::Flux2Transformer2DModel& mm) {
    int64_t a = 0, b = 0, c = 0, d = 0;
    mm.shard(&a, &b, &c, &d);
    if (head0) *head0 = a;
    if (heads) *heads = b;
    if (mlp0) *mlp0 = c;
    if (mlp_features) *mlp_features = d;
  });
}

dcpp_status dcpp_tp_plan_split(int64_t units, int nranks, const float* ratios, int64_t* out_units) {
  if (units < 0 || nranks < 1 || !out_units) return DCPP_ERR_INVALID_ARG;
  try {
    std::vector<double> f(static_cast<size_t>(nranks), 1.0);
    if (ratios) f.assign(ratios, ratios + nranks);
    const auto m = dcpp::plan_tensor_split(units, f);
    for (int j = 0; j < nranks; ++j) out_units[j] = m[j];
    return DCPP_OK;
  } catch (const dcpp::Error& e) {
    return e.status;
  }
}

dcpp_status dcpp_flow_match_schedule(int n, float shift, float* timesteps, float* sigmas) {
  if (n <= 0 || !timesteps || !sigmas) return DCPP_ERR_INVALID_ARG;
  try {
    dcpp::FlowMatchEulerDiscreteScheduler sch;
    sch.shift = shift;
    std::vector<float> t, s, base(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i) base[i] = static_cast<float>(1.0 - static_cast<double>(i) / n);
    sch.schedule(n, 0.0f, base, t, s);
    memcpy(timesteps, t.data(), n * sizeof(float));
    memcpy(sigmas, s.data(), (n + 1) * sizeof(float));
    return DCPP_OK;
  } catch (const dcpp::Error& e) {
    return e.status;
  }
}

void dcpp_flow_match_config_default(dcpp_flow_match_config* c) {
  if (!c) return;
  *c = dcpp_flow_match_config{};
  c->num_train_timesteps = 1000;
  c->shift = 1.0f;
  c->time_shift_type = DCPP_TIME_SHIFT_EXPONENTIAL;
}

dcpp_status dcpp_flow_match_schedule_ex(const dcpp_flow_match_config* c, int n, float mu, const float* sigmas_in,
                                        float* timesteps, float* sigmas) {
  if (!c || n <= 0 || !timesteps || !sigmas) return DCPP_ERR_INVALID_ARG;
  if (c->time_shift_type != DCPP_TIME_SHIFT_EXPONENTIAL && c->time_shift_type != DCPP_TIME_SHIFT_LINEAR)
    return DCPP_ERR_INVALID_ARG;
  try {
    dcpp::FlowMatchEulerDiscreteScheduler sch;
    sch.num_train_timesteps = c->num_train_timesteps;
    sch.shift = c->shift;
    sch.use_dynamic_shifting = c->use_dynamic_shifting != 0;
    sch.has_shift_terminal = c->has_shift_terminal != 0;
    sch.shift_terminal = c->shift_terminal;
    sch.invert_sigmas = c->invert_sigmas != 0;
    sch.linear_time_shift = c->time_shift_type == DCPP_TIME_SHIFT_LINEAR;
    std::vector<float> base, t, s;
    if (sigmas_in) base.assign(sigmas_in, sigmas_in + n);
    sch.schedule(n, mu, base, t, s);
    memcpy(timesteps, t.data(), n * sizeof(float));
    memcpy(sigmas, s.data(), (n + 1) * sizeof(float));
    return DCPP_OK;
  } catch (const dcpp::Error& e) {
    return e.status;
  }
}

dcpp_status dcpp_flux2_prepare_txt_ids(int64_t batch, int64_t seq_len, int32_t* out) {
  if (batch < 0 || seq_len < 0 || (!out && batch * seq_len > 0)) return DCPP_ERR_INVALID_ARG;
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t l = 0; l < seq_len; ++l) {
      int32_t* id = out + (b * seq_len + l) * 4;
      id[0] = id[1] = id[2] = 0;
      id[3] = static_cast<int32_t>(l);
    }
  return DCPP_OK;
}

dcpp_status dcpp_flux2_prepare_img_ids(int64_t batch, int64_t packed_h, int64_t packed_w, int32_t* out) {
  if (batch < 0 || packed_h < 0 || packed_w < 0 || (!out && batch * packed_h * packed_w > 0))
    return DCPP_ERR_INVALID_ARG;
  int32_t* id = out;
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t y = 0; y < packed_h; ++y)
      for (int64_t x = 0; x < packed_w; ++x, id += 4) {
        id[0] = 0;
        id[1] = static_cast<int32_t>(y);
        id[2] = static_cast<int32_t>(x);
        id[3] = 0;
      }
  return DCPP_OK;
}

dcpp_status dcpp_flux2_prepare_ref_image_ids(int64_t batch, int64_t n_images, const int64_t* packed_hw, int32_t* out) {
  if (batch < 0 || n_images < 0 || (n_images > 0 && !packed_hw)) return DCPP_ERR_INVALID_ARG;
  int64_t tokens = 0;
  for (int64_t i = 0; i < n_images; ++i) {
    if (packed_hw[2 * i] < 0 || packed_hw[2 * i + 1] < 0) return DCPP_ERR_INVALID_ARG;
    tokens += packed_hw[2 * i] * packed_hw[2 * i + 1];
  }
  if (!out && batch * tokens > 0) return DCPP_ERR_INVALID_ARG;
  int32_t* id = out;
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t i = 0; i < n_images; ++i)  // image i sits at time coordinate 10 (i + 1)
      for (int64_t y = 0; y < packed_hw[2 * i]; ++y)
        for (int64_t x = 0; x < packed_hw[2 * i + 1]; ++x, id += 4) {
          id[0] = static_cast<int32_t>(10 + 10 * i);
          id[1] = static_cast<int32_t>(y);
          id[2] = static_cast<int32_t>(x);
          id[3] = 0;
        }
  return DCPP_OK;
}

dcpp_status dcpp_flux2_empirical_mu(int64_t image_seq_len, int num_steps, float* mu) {
  if (!mu) return DCPP_ERR_INVALID_ARG;
  *mu = dcpp::flux2_empirical_mu(image_seq_len, num_steps);
  return DCPP_OK;
}

}  // extern "C"

// GGUF checkpoints.
extern "C" {

dcpp_status dcpp_flux2_load_gguf(dcpp_flux2* m, const dcpp_gguf* f, int64_t* n_bound, int64_t* n_unused) {
  return model_call(m, "dcpp_flux2_load_gguf", [&](dcpp::Flux2Transformer2DModel& mm) {
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

dcpp_status dcpp_flux2_from_pretrained(dcpp_ctx* ctx, const char* dir, dcpp_flux2** out) {
  if (!ctx || !dir || !out) return DCPP_ERR_INVALID_ARG;
  *out = nullptr;
  dcpp_flux2_config cfg;
  try {
    dcpp::Flux2Config::from_file(std::string(dir) + "/config.json").to_c(cfg);
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
  st = dcpp_flux2_create(ctx, &cfg, out);
  if (st == DCPP_OK) st = dcpp_flux2_load_gguf(*out, g, nullptr, nullptr);
  dcpp_gguf_close(g);
  if (st != DCPP_OK && *out) {
    dcpp_flux2_destroy(*out);
    *out = nullptr;
  }
  return st;
}

}  // extern "C"
