// Flux2 VAE decode: see vae.hpp.
#include "vae.hpp"

#include <cuda_fp16.h>
#include <string.h>

#include <algorithm>
#include <array>
#include <cmath>

#include "gguf.hpp"

namespace dcpp {

namespace {

std::vector<float> to_f32(int type, const void* data, size_t nbytes, int64_t n, const std::string& name) {
  std::vector<float> out(static_cast<size_t>(n));
  auto need = [&](size_t b) {
    if (nbytes != b) fail(DCPP_ERR_INVALID_ARG, "Tensor '" + name + "': byte size mismatch");
  };
  const auto* u16 = static_cast<const uint16_t*>(data);
  if (type == kTypeF32) {
    need(static_cast<size_t>(n) * 4);
    memcpy(out.data(), data, nbytes);
  } else if (type == kTypeF16 || type == kTypeBF16) {
    need(static_cast<size_t>(n) * 2);
    for (int64_t i = 0; i < n; ++i) {
      if (type == kTypeBF16) {
        const uint32_t b = static_cast<uint32_t>(u16[i]) << 16;
        memcpy(&out[i], &b, 4);
      } else {
        out[i] = __half2float(__ushort_as_half(u16[i]));
      }
    }
  } else if (type == kTypeQ8_0 || type == kTypeQ4_K) {
    need(row_bytes_of(type, n));
    host_dequant_row(type, static_cast<const uint8_t*>(data), n, out.data());
  } else {
    fail(DCPP_ERR_UNSUPPORTED, "Tensor '" + name + "': type " + std::to_string(type) + " is not supported");
  }
  return out;
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// Rows of the 2x-upsampled 3x3 conv tap k that phase a reads, as an offset
// into the two-tap (a - 1, a) window of the low-resolution image.
int phase_tap(int a, int k) {
  const int src = (a + k - 1) >= 0 ? (a + k - 1) / 2 : -1;  // floor((a + k - 1) / 2)
  return src - (a - 1);
}

}  // namespace

// ----------------------------------------------------------------- config
VAEConfig VAEConfig::from_file(const std::string& path) {
  auto m = read_json_object(path);
  VAEConfig c;
  auto num = [&](const char* k, auto& dst) {
    auto it = m.find(k);
    if (it == m.end() || it->second == "null") return;
    using T = std::decay_t<decltype(dst)>;
    dst = static_cast<T>(std::stod(it->second));
  };
  auto flag = [&](const char* k, bool& dst) {
    auto it = m.find(k);
    if (it != m.end() && it->second != "null") dst = it->second == "true";
  };
  num("in_channels", c.in_channels);
  num("out_channels", c.out_channels);
  {
    auto it = m.find("block_out_channels");
    if (it != m.end() && it->second != "null") c.block_out_channels = parse_int_list(it->second);
  }
  num("layers_per_block", c.layers_per_block);
  num("latent_channels", c.latent_channels);
  num("norm_num_groups", c.norm_num_groups);
  num("sample_size", c.sample_size);
  flag("force_upcast", c.force_upcast);
  flag("use_quant_conv", c.use_quant_conv);
  flag("use_post_quant_conv", c.use_post_quant_conv);
  flag("mid_block_add_attention", c.mid_block_add_attention);
  num("batch_norm_eps", c.batch_norm_eps);
  num("batch_norm_momentum", c.batch_norm_momentum);
  {
    auto it = m.find("patch_size");
    if (it != m.end() && it->second != "null") {
      auto p = parse_int_list(it->second);
      if (p.size() != 2) fail(DCPP_ERR_INVALID_ARG, "patch_size must be an array of length 2");
      c.patch_h = p[0];
      c.patch_w = p[1];
    }
  }
  return c;
}

VAEConfig VAEConfig::from_c(const dcpp_vae_config& s) {
  VAEConfig c;
  c.in_channels = s.in_channels;
  c.out_channels = s.out_channels;
  if (s.n_blocks < 1 || s.n_blocks > 8) fail(DCPP_ERR_INVALID_ARG, "n_blocks must be 1..8");
  c.block_out_channels.assign(s.block_out_channels, s.block_out_channels + s.n_blocks);
  c.layers_per_block = s.layers_per_block;
  c.latent_channels = s.latent_channels;
  c.norm_num_groups = s.norm_num_groups;
  c.sample_size = s.sample_size;
  c.force_upcast = s.force_upcast != 0;
  c.use_quant_conv = s.use_quant_conv != 0;
  c.use_post_quant_conv = s.use_post_quant_conv != 0;
  c.mid_block_add_attention = s.mid_block_add_attention != 0;
  c.batch_norm_eps = s.batch_norm_eps;
  c.batch_norm_momentum = s.batch_norm_momentum;
  c.patch_h = s.patch_size[0];
  c.patch_w = s.patch_size[1];
  return c;
}

void VAEConfig::to_c(dcpp_vae_config& s) const {
  memset(&s, 0, sizeof(s));
  s.in_channels = in_channels;
  s.out_channels = out_channels;
  s.n_blocks = static_cast<int32_t>(std::min<size_t>(block_out_channels.size(), 8));
  for (int i = 0; i < s.n_blocks; ++i) s.block_out_channels[i] = block_out_channels[i];
  s.layers_per_block = layers_per_block;
  s.latent_channels = latent_channels;
  s.norm_num_groups = norm_num_groups;
  s.sample_size = sample_size;
  s.force_upcast = force_upcast;
  s.use_quant_conv = use_quant_conv;
  s.use_post_quant_conv = use_post_quant_conv;
  s.mid_block_add_attention = mid_block_add_attention;
  s.batch_norm_eps = batch_norm_eps;
  s.batch_norm_momentum = batch_norm_momentum;
  s.patch_size[0] = patch_h;
  s.patch_size[1] = patch_w;
}

// ----------------------------------------------------------------- model
AutoencoderKLFlux2Decoder::AutoencoderKLFlux2Decoder(Ctx& ctx, const VAEConfig& cfg) : StepPlanner(ctx), cfg_(cfg) {
  const auto& c = cfg_;
  if (c.block_out_channels.empty()) fail(DCPP_ERR_INVALID_ARG, "block_out_channels is empty");
  for (int64_t ch : c.block_out_channels)
    if (ch < 64 || ch % 64 || c.norm_num_groups < 1 || ch % c.norm_num_groups || ch > 1024)
      fail(DCPP_ERR_UNSUPPORTED, "block_out_channels must be multiples of 64 (<= 1024) divisible by norm_num_groups");
  if (c.patch_h != 2 || c.patch_w != 2) fail(DCPP_ERR_UNSUPPORTED, "patch_size must be [2, 2]");
  if (c.out_channels != 1 && c.out_channels != 3 && c.out_channels != 4)
    fail(DCPP_ERR_UNSUPPORTED, "out_channels must be 1, 3 or 4");
  if (c.latent_channels < 1 || c.latent_channels > 256 || c.layers_per_block < 0)
    fail(DCPP_ERR_INVALID_ARG, "bad latent_channels / layers_per_block");
  if (c.mid_block_add_attention && c.block_out_channels.back() > 512)
    fail(DCPP_ERR_UNSUPPORTED, "mid-block attention width above 512");

  // Parameter registry (the decode path of diffusers' AutoencoderKLFlux2).
  const int64_t L = c.latent_channels;
  const auto& ch = c.block_out_channels;
  expect("bn.running_mean", {4 * L});
  expect("bn.running_var", {4 * L});
  if (c.use_post_quant_conv) {
    expect("post_quant_conv.weight", {L, L, 1, 1});
    expect("post_quant_conv.bias", {L});
  }
  auto conv = [&](const std::string& n, int64_t cin, int64_t cout, int64_t k) {
    expect(n + ".weight", {cout, cin, k, k});
    expect(n + ".bias", {cout});
  };
  auto norm = [&](const std::string& n, int64_t C) {
    expect(n + ".weight", {C});
    expect(n + ".bias", {C});
  };
  auto resnet = [&](const std::string& n, int64_t cin, int64_t cout) {
    norm(n + ".norm1", cin);
    conv(n + ".conv1", cin, cout, 3);
    norm(n + ".norm2", cout);
    conv(n + ".conv2", cout, cout, 3);
    if (cin != cout) conv(n + ".conv_shortcut", cin, cout, 1);
  };
  const int64_t top = ch.back();
  conv("decoder.conv_in", L, top, 3);
  resnet("decoder.mid_block.resnets.0", top, top);
  if (c.mid_block_add_attention) {
    const std::string p = "decoder.mid_block.attentions.0";
    norm(p + ".group_norm", top);
    for (const char* n : {"to_q", "to_k", "to_v", "to_out.0"}) {
      expect(p + "." + n + ".weight", {top, top});
      expect(p + "." + n + ".bias", {top});
    }
  }
  resnet("decoder.mid_block.resnets.1", top, top);
  const int n_up = static_cast<int>(ch.size());
  int64_t prev = top;
  for (int i = 0; i < n_up; ++i) {
    const int64_t out = ch[n_up - 1 - i];
    for (int j = 0; j <= c.layers_per_block; ++j)
      resnet("decoder.up_blocks." + std::to_string(i) + ".resnets." + std::to_string(j), j == 0 ? prev : out, out);
    if (i < n_up - 1) conv("decoder.up_blocks." + std::to_string(i) + ".upsamplers.0.conv", out, out, 3);
    prev = out;
  }
  norm("decoder.conv_norm_out", ch[0]);
  conv("decoder.conv_out", ch[0], c.out_channels, 3);
}

AutoencoderKLFlux2Decoder::~AutoencoderKLFlux2Decoder() {
  cudaSetDevice(ctx_.device);
  cudaStreamSynchronize(ctx_.stream);
  free_plan();
  free_weights();
}

void AutoencoderKLFlux2Decoder::expect(const std::string& name, std::vector<int64_t> shape) {
  params_[name].shape = std::move(shape);
}

void AutoencoderKLFlux2Decoder::set_param(const std::string& name, int type, const std::vector<int64_t>& shape,
                                          const void* data, size_t nbytes) {
  if (!data) fail(DCPP_ERR_INVALID_ARG, "Tensor '" + name + "': null data");
  if (name == "bn.num_batches_tracked") return;  // BatchNorm bookkeeping, unused by decode
  auto it = params_.find(name);
  if (it == params_.end()) fail(DCPP_ERR_NOT_FOUND, "Error while loading Tensor '" + name + "': Tensor not found");
  HostParam& p = it->second;
  if (shape != p.shape)
    fail(DCPP_ERR_INVALID_ARG, "Error while loading Tensor '" + name + "': Parameter shape mismatch: expected " +
                                   shape_str(p.shape) + ", got " + shape_str(shape));
  int64_t n = 1;
  for (int64_t d : shape) n *= d;
  p.data = to_f32(type, data, nbytes, n, name);
  p.set = true;
  if (weights_built_) {
    cudaStreamSynchronize(ctx_.stream);
    free_plan();
    free_weights();
  }
}

std::vector<std::string> AutoencoderKLFlux2Decoder::missing() const {
  std::vector<std::string> m;
  for (const auto& kv : params_)
    if (!kv.second.set) m.push_back(kv.first);
  return m;
}

const std::vector<float>& AutoencoderKLFlux2Decoder::host(const std::string& name) const {
  auto it = params_.find(name);
  if (it == params_.end() || !it->second.set) fail(DCPP_ERR_STATE, "internal: parameter '" + name + "' not set");
  return it->second.data;
}

void* AutoencoderKLFlux2Decoder::dev_alloc(size_t bytes, std::vector<void*>& list) {
  void* p = nullptr;
  if (cudaMalloc(&p, std::max<size_t>(bytes, 256)) != cudaSuccess) {
    cudaGetLastError();
    fail(DCPP_ERR_OOM, "VAE device allocation of " + std::to_string(bytes) + " bytes failed");
  }
  list.push_back(p);
  return p;
}

AutoencoderKLFlux2Decoder::Conv AutoencoderKLFlux2Decoder::make_conv(const std::string& prefix, int64_t cin_pad,
                                                                      bool upsampler) {
  const auto& sh = params_.at(prefix + ".weight").shape;
  const auto& w = host(prefix + ".weight");
  Conv c;
  c.cout = sh[0];
  c.cin = sh[1];
  c.k = sh[2];
  c.cin_pad = cin_pad;
  const int64_t taps = c.k * c.k;
  auto upload_bf16 = [&](const std::vector<uint16_t>& h) {
    auto* d = static_cast<uint16_t*>(dev_alloc(h.size() * 2, weight_allocs_));
    cuda_check(cudaMemcpy(d, h.data(), h.size() * 2, cudaMemcpyHostToDevice), "upload conv weight");
    return d;
  };
  // [cout, taps * cin_pad], K ordered (tap = 3 ky + kx, channel).
  std::vector<uint16_t> h(static_cast<size_t>(c.cout * taps * cin_pad), 0);
  for (int64_t co = 0; co < c.cout; ++co)
    for (int64_t ci = 0; ci < c.cin; ++ci)
      for (int64_t t = 0; t < taps; ++t)
        h[(co * taps + t) * cin_pad + ci] = host_f32_to_bf16(w[(co * c.cin + ci) * taps + t]);
  c.w = upload_bf16(h);
  if (upsampler) {
    // Nearest 2x upsample then 3x3 conv == per output phase (a, b) a 2x2
    // conv over the low-resolution image with taps summed (exactly, in
    // double, then rounded once).
    for (int a = 0; a < 2; ++a)
      for (int b = 0; b < 2; ++b) {
        std::vector<double> acc(static_cast<size_t>(c.cout * 4 * cin_pad), 0.0);
        for (int64_t co = 0; co < c.cout; ++co)
          for (int64_t ci = 0; ci < c.cin; ++ci)
            for (int ky = 0; ky < 3; ++ky)
              for (int kx = 0; kx < 3; ++kx) {
                const int t = phase_tap(a, ky) * 2 + phase_tap(b, kx);
                acc[(co * 4 + t) * cin_pad + ci] += w[((co * c.cin + ci) * 3 + ky) * 3 + kx];
              }
        std::vector<uint16_t> hp(acc.size());
        for (size_t i = 0; i < acc.size(); ++i) hp[i] = host_f32_to_bf16(static_cast<float>(acc[i]));
        c.phase[a * 2 + b] = upload_bf16(hp);
      }
  }
  const auto& bias = host(prefix + ".bias");
  c.bias = static_cast<float*>(dev_alloc(bias.size() * 4, weight_allocs_));
  cuda_check(cudaMemcpy(c.bias, bias.data(), bias.size() * 4, cudaMemcpyHostToDevice), "upload conv bias");
  return c;
}

AutoencoderKLFlux2Decoder::Norm AutoencoderKLFlux2Decoder::make_norm(const std::string& prefix) {
  Norm n;
  for (int k = 0; k < 2; ++k) {
    const auto& v = host(prefix + (k == 0 ? ".weight" : ".bias"));
    auto* d = static_cast<float*>(dev_alloc(v.size() * 4, weight_allocs_));
    cuda_check(cudaMemcpy(d, v.data(), v.size() * 4, cudaMemcpyHostToDevice), "upload norm");
    (k == 0 ? n.gamma : n.beta) = d;
  }
  return n;
}

void AutoencoderKLFlux2Decoder::build_weights() {
  const auto& c = cfg_;
  const auto& ch = c.block_out_channels;
  const int64_t Lpad = round_up(c.latent_channels, 64);
  auto f32_upload = [&](const std::vector<float>& v) {
    auto* d = static_cast<float*>(dev_alloc(v.size() * 4, weight_allocs_));
    cuda_check(cudaMemcpy(d, v.data(), v.size() * 4, cudaMemcpyHostToDevice), "upload");
    return d;
  };
  bn_mean_ = f32_upload(host("bn.running_mean"));
  bn_var_ = f32_upload(host("bn.running_var"));
  if (c.use_post_quant_conv) convs_["post_quant_conv"] = make_conv("post_quant_conv", Lpad, false);
  convs_["decoder.conv_in"] = make_conv("decoder.conv_in", Lpad, false);
  auto resnet = [&](const std::string& n, int64_t cin) {
    norms_[n + ".norm1"] = make_norm(n + ".norm1");
    convs_[n + ".conv1"] = make_conv(n + ".conv1", cin, false);
    norms_[n + ".norm2"] = make_norm(n + ".norm2");
    const int64_t cout = params_.at(n + ".conv1.weight").shape[0];
    convs_[n + ".conv2"] = make_conv(n + ".conv2", cout, false);
    if (params_.count(n + ".conv_shortcut.weight")) convs_[n + ".conv_shortcut"] = make_conv(n + ".conv_shortcut", cin, false);
  };
  const int64_t top = ch.back();
  resnet("decoder.mid_block.resnets.0", top);
  if (c.mid_block_add_attention) {
    const std::string p = "decoder.mid_block.attentions.0";
    norms_[p + ".group_norm"] = make_norm(p + ".group_norm");
    std::vector<uint16_t> qkv(static_cast<size_t>(3 * top * top));
    std::vector<float> qkv_b(static_cast<size_t>(3 * top));
    const char* names[3] = {"to_q", "to_k", "to_v"};
    for (int k = 0; k < 3; ++k) {
      const auto& w = host(p + "." + names[k] + ".weight");
      const auto& b = host(p + "." + names[k] + ".bias");
      for (int64_t i = 0; i < top * top; ++i) qkv[k * top * top + i] = host_f32_to_bf16(w[i]);
      for (int64_t i = 0; i < top; ++i) qkv_b[k * top + i] = b[i];
    }
    attn_qkv_w_ = static_cast<uint16_t*>(dev_alloc(qkv.size() * 2, weight_allocs_));
    cuda_check(cudaMemcpy(attn_qkv_w_, qkv.data(), qkv.size() * 2, cudaMemcpyHostToDevice), "upload qkv");
    attn_qkv_b_ = f32_upload(qkv_b);
    const auto& wo = host(p + ".to_out.0.weight");
    std::vector<uint16_t> o(wo.size());
    for (size_t i = 0; i < wo.size(); ++i) o[i] = host_f32_to_bf16(wo[i]);
    attn_out_w_ = static_cast<uint16_t*>(dev_alloc(o.size() * 2, weight_allocs_));
    cuda_check(cudaMemcpy(attn_out_w_, o.data(), o.size() * 2, cudaMemcpyHostToDevice), "upload out");
    attn_out_b_ = f32_upload(host(p + ".to_out.0.bias"));
  }
  resnet("decoder.mid_block.resnets.1", top);
  const int n_up = static_cast<int>(ch.size());
  int64_t prev = top;
  for (int i = 0; i < n_up; ++i) {
    const int64_t out = ch[n_up - 1 - i];
    const std::string b = "decoder.up_blocks." + std::to_string(i);
    for (int j = 0; j <= c.layers_per_block; ++j) resnet(b + ".resnets." + std::to_string(j), j == 0 ? prev : out);
    if (i < n_up - 1) convs_[b + ".upsamplers.0.conv"] = make_conv(b + ".upsamplers.0.conv", out, true);
    prev = out;
  }
  norms_["decoder.conv_norm_out"] = make_norm("decoder.conv_norm_out");
  convs_["decoder.conv_out"] = make_conv("decoder.conv_out", ch[0], false);
  weights_built_ = true;
}

void AutoencoderKLFlux2Decoder::free_weights() {
  for (void* p : weight_allocs_) cudaFree(p);
  weight_allocs_.clear();
  convs_.clear();
  norms_.clear();
  attn_qkv_w_ = attn_out_w_ = nullptr;
  attn_qkv_b_ = attn_out_b_ = bn_mean_ = bn_var_ = nullptr;
  weights_built_ = false;
}

void AutoencoderKLFlux2Decoder::free_plan() {
  if (graph_) cudaGraphExecDestroy(graph_);
  graph_ = nullptr;
  for (void* p : allocs_) cudaFree(p);
  allocs_.clear();
  ops_.clear();
  last_ops_ = nullptr;
  release_plan_events();
  planned_ = false;
}

void AutoencoderKLFlux2Decoder::prepare(int64_t batch, int64_t packed_h, int64_t packed_w, bool use_graph,
                                        int64_t tile_size) {
  auto miss = missing();
  if (!miss.empty())
    fail(DCPP_ERR_STATE, "parameters not set: " + miss.front() + " (+" + std::to_string(miss.size() - 1) + " more)");
  if (batch < 1 || packed_h < 1 || packed_w < 1 || batch * packed_h * packed_w * 256 > (int64_t(1) << 26))
    fail(DCPP_ERR_UNSUPPORTED, "batch x image size out of range");
  if (tile_size < 0) fail(DCPP_ERR_INVALID_ARG, "decode_tiled(): tile size must be positive");
  if (tile_size > 0) {
    const int64_t scale = cfg_.scale_factor();
    if (tile_size % scale != 0)
      fail(DCPP_ERR_INVALID_ARG, "decode_tiled(): tile size must be divisible by the VAE's scale factor");
    if (tile_size / scale * 3 / 4 < 1)
      fail(DCPP_ERR_INVALID_ARG, "tiled_forward(): tile size too small (3/4 of it must be >= 1)");
  }
  if (planned_ && batch == B_ && packed_h == ph_ && packed_w == pw_ && use_graph == use_graph_ && tile_size == tile_)
    return;
  cudaStreamSynchronize(ctx_.stream);
  free_plan();
  if (!weights_built_) build_weights();
  tile_ = tile_size;
  B_ = batch;
  ph_ = packed_h;
  pw_ = packed_w;
  use_graph_ = use_graph;
  build_plan();
  planned_ = true;
}

void AutoencoderKLFlux2Decoder::build_plan() {
  const auto& c = cfg_;
  const auto& ch = c.block_out_channels;
  const int64_t B = B_, L = c.latent_channels, Lpad = round_up(L, 64), G = c.norm_num_groups;
  const int n_up = static_cast<int>(ch.size());
  const int64_t top = ch.back();
  auto alloc = [&](size_t bytes) { return dev_alloc(bytes, allocs_); };

  lat_dev_ = static_cast<float*>(alloc(B * ph_ * pw_ * 4 * L * 4));
  const int64_t h0 = 2 * ph_, w0 = 2 * pw_;
  const int64_t Hout = h0 * c.scale_factor(), Wout = w0 * c.scale_factor();
  img_dev_ = static_cast<float*>(alloc(B * c.out_channels * Hout * Wout * 4));
  auto* zfull = static_cast<uint16_t*>(alloc(B * h0 * w0 * Lpad * 2));
  constexpr int kMaxNorms = 128;

  // Activation buffers of one decode of an h x w latent image (one set per
  // distinct size: the tiles of a tiled decode share them).
  struct Bufs {
    float* X[2] = {nullptr, nullptr};
    uint16_t* Xb[2] = {nullptr, nullptr};
    uint16_t *Hb = nullptr, *A = nullptr, *zq = nullptr, *qkv = nullptr, *vt = nullptr, *Pm = nullptr, *O = nullptr;
    float *Sc = nullptr, *S = nullptr, *part_x = nullptr, *part_h = nullptr;
    double* stats = nullptr;
    int64_t part_floats = 0;
  };
  std::map<std::pair<int64_t, int64_t>, Bufs> bufs;
  auto get_bufs = [&](int64_t h0, int64_t w0) -> Bufs& {
    auto key = std::make_pair(h0, w0);
    auto it = bufs.find(key);
    if (it != bufs.end()) return it->second;
    Bufs& d = bufs[key];
    const int64_t P0 = h0 * w0;
    // Largest pixels x channels of any activation.
    int64_t max_pc = P0 * std::max(top, Lpad);
    {
      int64_t P = P0, prev = top;
      for (int i = 0; i < n_up; ++i) {
        const int64_t out = ch[n_up - 1 - i];
        max_pc = std::max(max_pc, P * std::max(prev, out));
        if (i < n_up - 1) P *= 4;
        max_pc = std::max(max_pc, P * out);
        prev = out;
      }
    }
    const int64_t E = B * max_pc;
    d.zq = static_cast<uint16_t*>(alloc(B * P0 * Lpad * 2));
    cuda_check(cudaMemset(d.zq, 0, B * P0 * Lpad * 2), "memset zq");
    for (int k = 0; k < 2; ++k) {
      d.X[k] = static_cast<float*>(alloc(E * 4));
      d.Xb[k] = static_cast<uint16_t*>(alloc(E * 2));
    }
    d.Hb = static_cast<uint16_t*>(alloc(E * 2));  // conv1 outputs (bf16: only GroupNorm reads them)
    d.Sc = static_cast<float*>(alloc(E * 4));
    // GroupNorm partial sums written by the producing convolution's epilogue
    // (one buffer for the residual stream's producer, one for conv1).
    const int64_t Hf = h0 * c.scale_factor(), Wf = w0 * c.scale_factor();
    d.part_floats = B * 4 * (round_up(Wf, 128) * round_up(Hf, 8) / 128) * 2 * G + 64;
    d.part_x = static_cast<float*>(alloc(d.part_floats * 4));
    d.part_h = static_cast<float*>(alloc(d.part_floats * 4));
    d.A = static_cast<uint16_t*>(alloc(E * 2));
    d.stats = static_cast<double*>(alloc(kMaxNorms * B * G * 2 * sizeof(double)));
    const int64_t Pk = round_up(P0, 64);
    if (c.mid_block_add_attention) {
      d.qkv = static_cast<uint16_t*>(alloc(B * P0 * 3 * top * 2));
      d.vt = static_cast<uint16_t*>(alloc(top * Pk * 2));
      cuda_check(cudaMemset(d.vt, 0, top * Pk * 2), "memset vt");
      d.S = static_cast<float*>(alloc(P0 * Pk * 4));
      d.Pm = static_cast<uint16_t*>(alloc(P0 * Pk * 2));
      cuda_check(cudaMemset(d.Pm, 0, P0 * Pk * 2), "memset P");
      d.O = static_cast<uint16_t*>(alloc(B * P0 * top * 2));
    }

  return d;
  };

  Ctx* cx = &ctx_;
  int* err = ctx_.d_err;
  begin_ops(ops_);

  // 1. Packed tokens -> de-normalised, unpatchified z (Flux2KleinPipeline.cpp:538-551).
  {
    const float* lat = lat_dev_;
    const float *mean = bn_mean_, *var = bn_var_;
    const float eps = c.batch_norm_eps;
    const int ph = static_cast<int>(ph_), pw = static_cast<int>(pw_);
    building_->push_back({[=](cudaStream_t s) {
                            cuda_check(launch_latent_unpack(lat, mean, var, eps, static_cast<int>(B), ph, pw,
                                                            static_cast<int>(L), static_cast<int>(Lpad), zfull, s),
                                       "latent unpack");
                          },
                          1, kOpOther, 0.0, "latent unpack"});
  }

  // One AutoencoderKLFlux2::decode (AutoencoderKLFlux2.cpp:139-150) of the
  // NHWC latent z_in [B, h0, w0, Lpad] into the NCHW image img.
  auto emit_decode = [&](const uint16_t* z_in, int64_t h0, int64_t w0, float* img) {
      Bufs& d = get_bufs(h0, w0);
      const int64_t P0 = h0 * w0, Pk = round_up(P0, 64);
      float* X[2] = {d.X[0], d.X[1]};
      uint16_t* Xb[2] = {d.Xb[0], d.Xb[1]};
      uint16_t* const Hb = d.Hb;
      float* const Sc = d.Sc;
      uint16_t* const A = d.A;
      double* const stats = d.stats;
      float* const part_x = d.part_x;
      float* const part_h = d.part_h;
      const int64_t part_floats = d.part_floats;
      uint16_t *const zq = d.zq, *const qkv = d.qkv, *const vt = d.vt, *const Pm = d.Pm, *const O = d.O;
      float* const S = d.S;
      int n_norms = 0;

    // N tile: the narrowest of 32 / 64 / 128 / 256 columns holding N (32 and
    // 64 only on the one-SM kernel).
    auto tile_for = [](int64_t N) { return N <= 32 ? 32 : N <= 64 ? 64 : N <= 128 ? 128 : 256; };

    // Plain GEMM: Y[M, N] = A[M, K] . W[N, K]^T with the conv epilogue.
    auto add_mm = [&](const std::string& tag, const uint16_t* a, int64_t lda, int64_t M, int64_t K, const uint16_t* w,
                      int64_t ldw, int64_t N, EpilogueArgs ep, int mode = kEpiConv) {
      const int tn = tile_for(N);
      const bool pair = cx->use_pair(M) && tn >= 128;
      auto maps = std::make_shared<std::array<CUtensorMap, 2>>();
      cuda_check(make_tmap_bf16(&(*maps)[0], a, K, M, lda, kGemmBM), "tensor map A");
      cuda_check(make_tmap_bf16(&(*maps)[1], w, K, N, ldw, pair ? tn / 2 : tn), "tensor map W");
      GemmArgs g{};
      g.N = static_cast<int32_t>(N);
      g.K = static_cast<int32_t>(K);
      g.n_groups = 1;
      g.groups[0].rows = static_cast<int32_t>(M);
      ep.mode = mode;
      if (mode == kEpiConv) ep.up_phase = -1;
      g.ep = ep;
      g.err = err;
      gemm_finalize_groups(g, pair ? 256 : kGemmBM, tn);
      building_->push_back({[maps, g, cx, pair](cudaStream_t s) {
                              const auto& m = *maps;
                              if (pair) cuda_check(launch_gemm_pair(m[0], m[1], m[1], g, kBSrcBf16, cx->num_sms, s), "vae gemm (pair)");
                              else cuda_check(launch_gemm(m[0], m[1], m[1], g, kBSrcBf16, cx->num_sms, s), "vae gemm");
                            },
                            1, kOpGemm, 2.0 * M * N * K, tag});
    };

    // Implicit-GEMM convolution over x [B, H, W, C] bf16 with the given taps.
    // Where the GroupNorm of a tensor finds its statistics: partial sums from
    // the producing convolutions (n regions of `stride` floats, `slots` 32-row
    // slots per image), or none (a statistics pass over the tensor).
    struct StatSrc {
      float* part = nullptr;
      int n = 0;
      int64_t stride = 0, slots = 0;
    };
    auto add_conv = [&](const std::string& tag, const uint16_t* x, int64_t H, int64_t W, int64_t C,
                        const std::vector<std::pair<int, int>>& taps, const uint16_t* w, int64_t N, EpilogueArgs ep,
                        int up_phase, StatSrc* stats_out = nullptr, int region = 0) {
      int tw = 128;
      int64_t best = -1;
      for (int cand : {128, 64, 32, 16}) {
        const int th = 128 / cand;
        const int64_t cover = round_up(W, cand) * round_up(H, th);
        if (best < 0 || cover < best) {
          best = cover;
          tw = cand;
        }
      }
      const int th = 128 / tw;
      const int64_t tiles_x = (W + tw - 1) / tw, tiles_y = (H + th - 1) / th;
      const int64_t rows = B * tiles_x * tiles_y * 128;
      if (rows >= (int64_t(1) << 31)) fail(DCPP_ERR_UNSUPPORTED, "convolution too large");
      if (taps.empty() || taps.size() > 9 || C % 64) fail(DCPP_ERR_UNSUPPORTED, "internal: convolution taps / channels");
      const size_t n_taps = std::min<size_t>(taps.size(), 9);
      const int64_t K = static_cast<int64_t>(n_taps) * C;
      const int tn = tile_for(N);
      const bool pair = cx->use_pair(rows) && tn >= 128;
      // Rows of 128 pixels on CTA pairs: halo patches (one load per channel
      // block serves every tap).
      const bool halo = pair && tw == 128 && th == 1;
      auto maps = std::make_shared<std::array<CUtensorMap, 2>>();
      if (halo)
        cuda_check(make_tmap_conv_patch(&(*maps)[0], x, B, H, W, C), "tensor map conv patch");
      else
        cuda_check(make_tmap_conv(&(*maps)[0], x, B, H, W, C, tw, th), "tensor map conv");
      cuda_check(make_tmap_bf16(&(*maps)[1], w, K, N, K, pair ? tn / 2 : tn), "tensor map conv W");
      GemmArgs g{};
      g.N = static_cast<int32_t>(N);
      g.K = static_cast<int32_t>(K);
      g.n_groups = 1;
      g.groups[0].rows = static_cast<int32_t>(rows);
      ep.mode = kEpiConv;
      ep.up_phase = up_phase;
      if (stats_out) {
        const int64_t cpg = N / G;
        const int64_t slots = tiles_x * tiles_y * 4;
        const int64_t stride = B * slots * 2 * G;
        if (N % G == 0 && (cpg == 2 || cpg == 4 || cpg == 8 || cpg == 16 || cpg == 32) &&
            (region + 1) * stride <= part_floats && (region == 0 || stats_out->stride == stride)) {
          ep.gn_part = stats_out->part + region * stride;
          ep.gn_cpg = static_cast<int32_t>(cpg);
          ep.gn_groups = static_cast<int32_t>(G);
          stats_out->n = region + 1;
          stats_out->stride = stride;
          stats_out->slots = slots;
        } else {
          stats_out->part = nullptr;  // the GroupNorm computes its own statistics
        }
      }
      g.ep = ep;
      g.err = err;
      g.conv.taps = static_cast<int32_t>(n_taps);
      g.conv.cin_blocks = static_cast<int32_t>(C / 64);
      g.conv.H = static_cast<int32_t>(H);
      g.conv.W = static_cast<int32_t>(W);
      g.conv.tile_w = tw;
      g.conv.tile_h = th;
      g.conv.tiles_x = static_cast<int32_t>(tiles_x);
      g.conv.tiles_y = static_cast<int32_t>(tiles_y);
      g.conv.halo = halo ? 1 : 0;
      for (size_t t = 0; t < n_taps; ++t) {
        g.conv.dy[t] = static_cast<int8_t>(taps[t].first);
        g.conv.dx[t] = static_cast<int8_t>(taps[t].second);
      }
      gemm_finalize_groups(g, pair ? 256 : kGemmBM, tn);
      building_->push_back({[maps, g, cx, pair](cudaStream_t s) {
                              const auto& m = *maps;
                              if (pair) cuda_check(launch_gemm_pair(m[0], m[1], m[1], g, kBSrcBf16, cx->num_sms, s), "conv (pair)");
                              else cuda_check(launch_gemm(m[0], m[1], m[1], g, kBSrcBf16, cx->num_sms, s), "conv");
                            },
                            1, kOpGemm, 2.0 * B * H * W * N * K, tag});
    };
    std::vector<std::pair<int, int>> taps3;
    for (int ky = 0; ky < 3; ++ky)
      for (int kx = 0; kx < 3; ++kx) taps3.push_back({ky - 1, kx - 1});

    auto conv_ep = [](float* out_f32, uint16_t* out_bf16, int64_t ld, const float* bias, const float* resid) {
      EpilogueArgs e{};
      e.out_f32 = out_f32;
      e.out_bf16 = out_bf16;
      e.ld_out = ld;
      e.bias = bias;
      e.resid = resid;
      e.ld_resid = ld;
      return e;
    };

    // GroupNorm (+ SiLU) of x (bf16 [B, HW, C]) into the bf16 operand A, with
    // the statistics from the producer's partial sums when it left them.
    auto group_norm = [&](const std::string& tag, const uint16_t* x, int64_t HW, int64_t C, const Norm& n, bool silu,
                          const StatSrc& src) {
      if (n_norms >= kMaxNorms) fail(DCPP_ERR_UNSUPPORTED, "too many GroupNorms");
      double* st = stats + static_cast<int64_t>(n_norms++) * B * G * 2;
      const float eps = 1e-6f;
      if (src.part) {
        const StatSrc sc = src;
        building_->push_back({[=](cudaStream_t s) {
                                cuda_check(launch_gn_finalize(sc.part, sc.n, sc.stride, sc.slots, static_cast<int>(B),
                                                              static_cast<int>(G), st, s),
                                           "gn finalize");
                              },
                              1, kOpNorm, 0.0, tag + " stats"});
      } else {
        building_->push_back({[=](cudaStream_t s) {
                                cuda_check(launch_gn_stats(x, true, static_cast<int>(B), HW, static_cast<int>(C),
                                                           static_cast<int>(G), st, s),
                                           "gn stats");
                              },
                              1, kOpNorm, 0.0, tag + " stats"});
      }
      building_->push_back({[=](cudaStream_t s) {
                              cuda_check(launch_gn_apply(x, true, static_cast<int>(B), HW, static_cast<int>(C),
                                                         static_cast<int>(G), st, n.gamma, n.beta, eps, silu, A, s),
                                         "gn apply");
                            },
                            1, kOpNorm, 0.0, tag});
    };

    // Zero every GroupNorm statistics slot once per decode.
    building_->push_back({[=](cudaStream_t s) {
                            cuda_check(cudaMemsetAsync(stats, 0, kMaxNorms * B * G * 2 * sizeof(double), s), "memset stats");
                          },
                          0, kOpOther, 0.0, "zero stats"});

    // 2. post_quant_conv (1x1) and conv_in (AutoencoderKLFlux2.cpp:139-150, Decoder.hpp:110-115).
    const uint16_t* z = z_in;
    if (c.use_post_quant_conv) {
      const Conv& pq = convs_.at("post_quant_conv");
      add_mm("post_quant_conv", z_in, Lpad, B * P0, Lpad, pq.w, Lpad, L, conv_ep(nullptr, zq, Lpad, pq.bias, nullptr));
      z = zq;
    }
    int cur = 0;
    StatSrc x_src;  // statistics of the residual stream X[cur]
    {
      const Conv& ci = convs_.at("decoder.conv_in");
      x_src.part = part_x;
      add_conv("conv_in", z, h0, w0, Lpad, taps3, ci.w, top, conv_ep(X[0], Xb[0], top, ci.bias, nullptr), -1, &x_src);
    }

    // ResnetBlock2D (ResnetBlock2D.inl:108-190) at H x W: X[cur] (+ Xb[cur]) -> X[cur ^ 1] (+ Xb[cur ^ 1]).
    // f32_out: whether the f32 copy of the output is read (as the next
    // residual); GroupNorm, shortcuts and upsamplers read the bf16 copy.
    auto resnet = [&](const std::string& n, int64_t H, int64_t W, int64_t cin, bool f32_out) {
      const Conv& c1 = convs_.at(n + ".conv1");
      const Conv& c2 = convs_.at(n + ".conv2");
      const int64_t cout = c1.cout, HW = H * W;
      group_norm(n + ".norm1", Xb[cur], HW, cin, norms_.at(n + ".norm1"), true, x_src);
      StatSrc h_src;
      h_src.part = part_h;
      add_conv(n + ".conv1", A, H, W, cin, taps3, c1.w, cout, conv_ep(nullptr, Hb, cout, c1.bias, nullptr), -1, &h_src);
      group_norm(n + ".norm2", Hb, HW, cout, norms_.at(n + ".norm2"), true, h_src);
      const float* resid = X[cur];
      auto sc = convs_.find(n + ".conv_shortcut");
      if (sc != convs_.end()) {
        add_mm(n + ".conv_shortcut", Xb[cur], cin, B * HW, cin, sc->second.w, cin, cout,
               conv_ep(Sc, nullptr, cout, sc->second.bias, nullptr));
        resid = Sc;
      }
      x_src = StatSrc();
      x_src.part = part_x;
      add_conv(n + ".conv2", A, H, W, cout, taps3, c2.w, cout,
               conv_ep(f32_out ? X[cur ^ 1] : nullptr, Xb[cur ^ 1], cout, c2.bias, resid), -1,
               &x_src);
      cur ^= 1;
    };

    // 3. Mid block (UNetMidBlock2D.cpp): resnet, attention, resnet.
    resnet("decoder.mid_block.resnets.0", h0, w0, top, true);
    if (c.mid_block_add_attention) {
      const std::string p = "decoder.mid_block.attentions.0";
      const int64_t C = top;
      group_norm(p + ".group_norm", Xb[cur], P0, C, norms_.at(p + ".group_norm"), false, x_src);
      add_mm(p + ".to_qkv", A, C, B * P0, C, attn_qkv_w_, C, 3 * C, conv_ep(nullptr, qkv, 3 * C, attn_qkv_b_, nullptr));
      const float scale = 1.0f / std::sqrt(static_cast<float>(C));
      for (int64_t b = 0; b < B; ++b) {
        const uint16_t* q = qkv + b * P0 * 3 * C;
        EpilogueArgs se{};
        se.out_f32 = S;
        se.ld_out = Pk;
        add_mm(p + ".scores", q, 3 * C, P0, C, q + C, 3 * C, P0, se, kEpiF32);
        building_->push_back({[=](cudaStream_t s) {
                                cuda_check(launch_softmax_rows(S, P0, P0, Pk, scale, Pm, Pk, s), "softmax");
                              },
                              1, kOpAttention, 0.0, p + ".softmax"});
        building_->push_back({[=](cudaStream_t s) {
                                cuda_check(launch_transpose_bf16(q + 2 * C, P0, C, 3 * C, vt, Pk, s), "transpose v");
                              },
                              1, kOpOther, 0.0, p + ".v^T"});
        add_mm(p + ".pv", Pm, Pk, P0, P0, vt, Pk, C, conv_ep(nullptr, O + b * P0 * C, C, nullptr, nullptr));
      }
      add_mm(p + ".to_out", O, C, B * P0, C, attn_out_w_, C, C, conv_ep(X[cur ^ 1], Xb[cur ^ 1], C, attn_out_b_, X[cur]));
      cur ^= 1;
      x_src = StatSrc();  // the next GroupNorm runs its own statistics pass
    }
    // The first up-block resnet reads X as its residual unless it has a
    // shortcut (channel change).
    const int64_t top_next = ch[n_up - 1];
    resnet("decoder.mid_block.resnets.1", h0, w0, top, top_next == top);

    // 4. Up blocks (UpDecoderBlock2D.cpp): resnets, then Upsample2D as four
    //    phase convolutions over the low-resolution image.
    int64_t H = h0, W = w0, prev = top;
    for (int i = 0; i < n_up; ++i) {
      const int64_t out = ch[n_up - 1 - i];
      const std::string b = "decoder.up_blocks." + std::to_string(i);
      for (int j = 0; j <= c.layers_per_block; ++j) {
        // The last resnet of a block feeds an upsampler or the final norm.
        resnet(b + ".resnets." + std::to_string(j), H, W, j == 0 ? prev : out, j < c.layers_per_block);
      }
      if (i < n_up - 1) {
        const Conv& up = convs_.at(b + ".upsamplers.0.conv");
        x_src = StatSrc();
        x_src.part = part_x;
        for (int ph = 0; ph < 4; ++ph) {
          const int a = ph >> 1, bb = ph & 1;
          std::vector<std::pair<int, int>> taps;
          for (int ty = 0; ty < 2; ++ty)
            for (int tx = 0; tx < 2; ++tx) taps.push_back({a - 1 + ty, bb - 1 + tx});
          // The next block's first resnet reads X as its residual unless it
          // has a shortcut.
          const bool f32_out = ch[n_up - 2 - i] == out;
          add_conv(b + ".upsample phase " + std::to_string(ph), Xb[cur], H, W, out, taps, up.phase[ph], out,
                   conv_ep(f32_out ? X[cur ^ 1] : nullptr, Xb[cur ^ 1], out, up.bias, nullptr), ph,
                   x_src.part ? &x_src : nullptr, ph);
        }
        cur ^= 1;
        H *= 2;
        W *= 2;
      }
      prev = out;
    }

    // 5. conv_norm_out, SiLU, conv_out (Decoder.hpp:132-162) -> NCHW image.
    group_norm("decoder.conv_norm_out", Xb[cur], H * W, ch[0], norms_.at("decoder.conv_norm_out"), true, x_src);
    {
      // A few output channels: a 32-column tile on one SM, the epilogue
      // storing the f32 image planes (NCHW) directly.
      const Conv& co = convs_.at("decoder.conv_out");
      EpilogueArgs e = conv_ep(img, nullptr, c.out_channels, co.bias, nullptr);
      e.nchw_hw = static_cast<int32_t>(H * W);
      add_conv("decoder.conv_out", A, H, W, ch[0], taps3, co.w, c.out_channels, e, -1);
    }

  };

  if (tile_ <= 0) {
    emit_decode(zfull, h0, w0, img_dev_);
  } else {
    // AutoencoderKLFlux2::decode_tiled (AutoencoderKLFlux2.cpp:380-405) with
    // tiled_forward (:262-378): latent tiles at a 3/4 stride, each decoded
    // alone; each decoded tile is blended in place with the (blended) tile
    // above, then with the one to its left, over a quarter tile with the
    // linear ramp x / extent, and its top-left band goes to the image.
    const int64_t scale = c.scale_factor();
    const int64_t lt = tile_ / scale, stride = lt * 3 / 4;
    const int64_t blend = tile_ / 4, band = tile_ - blend;
    std::vector<int64_t> ys, xs;
    for (int64_t i = 0; i < h0; i += stride) ys.push_back(i);
    for (int64_t j = 0; j < w0; j += stride) xs.push_back(j);
    const int Co = static_cast<int>(c.out_channels);
    std::vector<std::vector<float*>> timg(ys.size(), std::vector<float*>(xs.size(), nullptr));
    std::map<std::pair<int64_t, int64_t>, uint16_t*> tz;  // contiguous latent tiles, one per size
    int64_t oy = 0;
    for (size_t a = 0; a < ys.size(); ++a) {
      const int64_t th = std::min(lt, h0 - ys[a]), hp = th * scale;
      int64_t ox = 0;
      for (size_t bx = 0; bx < xs.size(); ++bx) {
        const int64_t tw = std::min(lt, w0 - xs[bx]), wp = tw * scale;
        uint16_t*& zt = tz[std::make_pair(th, tw)];
        if (!zt) zt = static_cast<uint16_t*>(alloc(B * th * tw * Lpad * 2));
        {
          uint16_t* dst = zt;
          const uint16_t* src = zfull + (ys[a] * w0 + xs[bx]) * Lpad;
          building_->push_back({[=](cudaStream_t s) {
                                  for (int64_t bb = 0; bb < B; ++bb)
                                    cuda_check(cudaMemcpy2DAsync(dst + bb * th * tw * Lpad, tw * Lpad * 2,
                                                                 src + bb * h0 * w0 * Lpad, w0 * Lpad * 2,
                                                                 tw * Lpad * 2, th, cudaMemcpyDeviceToDevice, s),
                                               "latent tile");
                                },
                                0, kOpOther, 0.0, "latent tile"});
        }
        float* img = static_cast<float*>(alloc(B * Co * hp * wp * 4));
        timg[a][bx] = img;
        emit_decode(zt, th, tw, img);
        const float* above = a > 0 ? timg[a - 1][bx] : nullptr;
        const float* left = bx > 0 ? timg[a][bx - 1] : nullptr;
        const int64_t ha = a > 0 ? std::min(lt, h0 - ys[a - 1]) * scale : 0;
        const int64_t wl = bx > 0 ? std::min(lt, w0 - xs[bx - 1]) * scale : 0;
        const int64_t ev = above ? std::min({ha, hp, blend}) : 0;
        const int64_t eh = left ? std::min({wl, wp, blend}) : 0;
        const int64_t keep_h = std::min(hp, band), keep_w = std::min(wp, band);
        float* out = img_dev_;
        const int64_t y0 = oy, x0 = ox;
        building_->push_back({[=](cudaStream_t s) {
                                cuda_check(launch_tile_blend(img, above, ha, left, wl, static_cast<int>(B), Co, hp, wp,
                                                             ev, eh, keep_h, keep_w, out, Hout, Wout, y0, x0, s),
                                           "tile blend");
                              },
                              1, kOpOther, 0.0, "tile blend"});
        ox += keep_w;
        if (bx + 1 == xs.size() && ox != Wout) fail(DCPP_ERR_STATE, "internal: tiled decode width");
      }
      oy += std::min(hp, band);
    }
    if (oy != Hout) fail(DCPP_ERR_STATE, "internal: tiled decode height");
  }
  end_ops();
  launches_per_step_ = 0;
  for (auto& o : ops_) launches_per_step_ += o.launches;
}

void AutoencoderKLFlux2Decoder::decode(const float* latents, float* image) {
  if (!planned_) fail(DCPP_ERR_STATE, "decode before prepare");
  if (!latents || !image) fail(DCPP_ERR_INVALID_ARG, "decode: null pointer");
  const int64_t L = cfg_.latent_channels;
  const int64_t Hout = 2 * ph_ * cfg_.scale_factor(), Wout = 2 * pw_ * cfg_.scale_factor();
  cuda_check(cudaMemcpyAsync(lat_dev_, latents, B_ * ph_ * pw_ * 4 * L * 4, cudaMemcpyDefault, ctx_.stream),
             "copy latents");
  run_ops(ops_, &graph_);
  cuda_check(cudaMemcpyAsync(image, img_dev_, B_ * cfg_.out_channels * Hout * Wout * 4, cudaMemcpyDefault,
                             ctx_.stream),
             "copy image");
  ctx_.check_device_error();
}

void AutoencoderKLFlux2Decoder::set_profiling(bool on) {
  if (on == profiling_) return;
  cudaStreamSynchronize(ctx_.stream);
  free_plan();
  profiling_ = on;
}

}  // namespace dcpp

// ------------------------------------------------------------------ C ABI
namespace {

template <class F>
dcpp_status vae_call(dcpp_vae* m, const char* entry, F&& f) {
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

void dcpp_vae_config_default(dcpp_vae_config* cfg) {
  if (cfg) dcpp::VAEConfig().to_c(*cfg);
}

dcpp_status dcpp_vae_config_from_file(const char* path, dcpp_vae_config* cfg) {
  if (!path || !cfg) return DCPP_ERR_INVALID_ARG;
  try {
    dcpp::VAEConfig::from_file(path).to_c(*cfg);
    return DCPP_OK;
  } catch (const dcpp::Error& e) {
    return e.status;
  } catch (const std::exception&) {
    return DCPP_ERR_INVALID_ARG;
  }
}

dcpp_status dcpp_vae_create(dcpp_ctx* ctx, const dcpp_vae_config* cfg, dcpp_vae** out) {
  if (!ctx || !cfg || !out) return DCPP_ERR_INVALID_ARG;
  *out = nullptr;
  try {
    ctx->maybe_inject("dcpp_vae_create");
    cudaSetDevice(ctx->device);
    auto* m = new dcpp_vae();
    m->ctx = ctx;
    try {
      m->model.reset(new dcpp::AutoencoderKLFlux2Decoder(*ctx, dcpp::VAEConfig::from_c(*cfg)));
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

dcpp_status dcpp_vae_destroy(dcpp_vae* m) {
  if (!m) return DCPP_ERR_INVALID_ARG;
  if (m->ctx) cudaSetDevice(m->ctx->device);
  delete m;
  return DCPP_OK;
}

dcpp_status dcpp_vae_set_param(dcpp_vae* m, const char* name, int type, int n_dims, const int64_t* shape,
                               const void* data, size_t nbytes) {
  return vae_call(m, "dcpp_vae_set_param", [&](dcpp::AutoencoderKLFlux2Decoder& mm) {
    if (!name || !shape || n_dims < 1 || n_dims > 4) dcpp::fail(DCPP_ERR_INVALID_ARG, "set_param: bad name or shape");
    mm.set_param(name, type, std::vector<int64_t>(shape, shape + n_dims), data, nbytes);
  });
}

dcpp_status dcpp_vae_missing(dcpp_vae* m, int* count, char* first, size_t cap) {
  return vae_call(m, "dcpp_vae_missing", [&](dcpp::AutoencoderKLFlux2Decoder& mm) {
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

dcpp_status dcpp_vae_load_gguf(dcpp_vae* m, const dcpp_gguf* f, int64_t* n_bound, int64_t* n_unused) {
  return vae_call(m, "dcpp_vae_load_gguf", [&](dcpp::AutoencoderKLFlux2Decoder& mm) {
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

dcpp_status dcpp_vae_from_pretrained(dcpp_ctx* ctx, const char* dir, dcpp_vae** out) {
  if (!ctx || !dir || !out) return DCPP_ERR_INVALID_ARG;
  *out = nullptr;
  dcpp_vae_config cfg;
  try {
    dcpp::VAEConfig::from_file(std::string(dir) + "/config.json").to_c(cfg);
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
  st = dcpp_vae_create(ctx, &cfg, out);
  if (st == DCPP_OK) st = dcpp_vae_load_gguf(*out, g, nullptr, nullptr);
  dcpp_gguf_close(g);
  if (st != DCPP_OK && *out) {
    dcpp_vae_destroy(*out);
    *out = nullptr;
  }
  return st;
}

dcpp_status dcpp_vae_prepare(dcpp_vae* m, int64_t batch, int64_t packed_h, int64_t packed_w, int use_graph) {
  return vae_call(m, "dcpp_vae_prepare", [&](dcpp::AutoencoderKLFlux2Decoder& mm) {
    mm.prepare(batch, packed_h, packed_w, use_graph != 0, 0);
  });
}

dcpp_status dcpp_vae_prepare_tiled(dcpp_vae* m, int64_t batch, int64_t packed_h, int64_t packed_w, int64_t tile_size,
                                   int use_graph) {
  return vae_call(m, "dcpp_vae_prepare_tiled", [&](dcpp::AutoencoderKLFlux2Decoder& mm) {
    if (tile_size <= 0) dcpp::fail(DCPP_ERR_INVALID_ARG, "decode_tiled(): tile size must be positive");
    mm.prepare(batch, packed_h, packed_w, use_graph != 0, tile_size);
  });
}

dcpp_status dcpp_vae_decode(dcpp_vae* m, const float* latents, float* image) {
  return vae_call(m, "dcpp_vae_decode", [&](dcpp::AutoencoderKLFlux2Decoder& mm) { mm.decode(latents, image); });
}

dcpp_status dcpp_vae_set_profiling(dcpp_vae* m, int on) {
  return vae_call(m, "dcpp_vae_set_profiling", [&](dcpp::AutoencoderKLFlux2Decoder& mm) { mm.set_profiling(on != 0); });
}

dcpp_status dcpp_vae_profile(dcpp_vae* m, int kind, double* ms, double* flops, int64_t* launches) {
  return vae_call(m, "dcpp_vae_profile",
                  [&](dcpp::AutoencoderKLFlux2Decoder& mm) { mm.profile(kind, ms, flops, launches); });
}

dcpp_status dcpp_vae_launches_per_step(dcpp_vae* m, int64_t* out) {
  return vae_call(m, "dcpp_vae_launches_per_step", [&](dcpp::AutoencoderKLFlux2Decoder& mm) {
    if (out) *out = mm.launches_per_step();
  });
}

}  // extern "C"
