// C++ host API of the Flux2 VAE decode (the pipeline step after the
// denoise loop).  Mirrors the reference's module and pipeline surface:
//   AutoencoderKLFlux2::Config / from_file   (AutoencoderKLFlux2.hpp:10-33, .cpp:422-468)
//   AutoencoderKLFlux2::decode               (AutoencoderKLFlux2.cpp:139-150): post_quant_conv + Decoder
//   Decoder::forward                         (vae/Decoder.hpp:110-165)
//   Flux2KleinPipeline::decode               (Flux2KleinPipeline.cpp:538-556): unpack the packed
//                                            tokens, BatchNorm de-normalisation, unpatchify, decode
// Parameters bind by their GGUF names (diffusers state-dict paths,
// "decoder.up_blocks.1.resnets.0.conv1.weight"); encoder-side tensors of a
// full VAE checkpoint are not part of the decoder (DCPP_ERR_NOT_FOUND, which
// a GGUF load counts as unused).
//
// Execution: NHWC activations; every convolution with more than a few
// output channels is an implicit GEMM on the tcgen05 GEMM (ConvGeom: 4-D
// TMA loads of shifted pixel rectangles, zero fill as padding); the 2x
// nearest upsample + 3x3 conv runs as four 2x2 convolutions over the
// low-resolution image (one per output phase, taps pre-summed), so the
// upsampled image is never materialised; GroupNorm is a statistics pass and
// an apply (+ SiLU) pass producing the bf16 GEMM operand; the mid-block
// attention (one head of dim C over all pixels) is QK^T GEMM -> row softmax
// -> PV GEMM; conv_out (3 channels) runs on 32-column tiles of the one-SM
// GEMM with an epilogue that writes the NCHW image.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "plan.hpp"

namespace dcpp {

struct VAEConfig {
  int64_t in_channels = 3;
  int64_t out_channels = 3;
  std::vector<int64_t> block_out_channels = {128, 256, 512, 512};
  int64_t layers_per_block = 2;
  int64_t latent_channels = 32;
  int64_t norm_num_groups = 32;
  int64_t sample_size = 1024;
  bool force_upcast = true;
  bool use_quant_conv = true;
  bool use_post_quant_conv = true;
  bool mid_block_add_attention = true;
  float batch_norm_eps = 1e-4f;
  float batch_norm_momentum = 0.1f;
  int64_t patch_h = 2, patch_w = 2;

  static VAEConfig from_file(const std::string& path);
  static VAEConfig from_c(const dcpp_vae_config& c);
  void to_c(dcpp_vae_config& c) const;
  int64_t scale_factor() const { return int64_t(1) << (block_out_channels.size() - 1); }
};

class AutoencoderKLFlux2Decoder : public StepPlanner {
 public:
  AutoencoderKLFlux2Decoder(Ctx& ctx, const VAEConfig& cfg);
  ~AutoencoderKLFlux2Decoder() override;

  const VAEConfig& config() const { return cfg_; }
  void set_param(const std::string& name, int type, const std::vector<int64_t>& shape, const void* data,
                 size_t nbytes);
  std::vector<std::string> missing() const;

  // Plan a decode of `batch` packed latents of packed_h x packed_w tokens
  // (image 16 packed_h x 16 packed_w for the default config); tile_size > 0:
  // the tiled decode with tiles of tile_size pixels (decode_tiled).
  void prepare(int64_t batch, int64_t packed_h, int64_t packed_w, bool use_graph, int64_t tile_size = 0);
  // Flux2KleinPipeline::decode (untiled): latents [B, ph*pw, 4 latent_channels]
  // f32 -> image [B, out_channels, H, W] f32.  Host or device pointers.
  void decode(const float* latents, float* image);
  void set_profiling(bool on);

 private:
  struct HostParam {
    std::vector<int64_t> shape;
    std::vector<float> data;
    bool set = false;
  };
  struct Conv {  // implicit-GEMM convolution weights
    int64_t cin = 0, cin_pad = 0, cout = 0, k = 0;
    uint16_t* w = nullptr;            // [cout, taps * cin_pad] bf16, K = (tap, channel)
    uint16_t* phase[4] = {};          // upsamplers: [cout, 4 * cin_pad] per output phase
    float* bias = nullptr;
  };
  struct Norm {
    float* gamma = nullptr;
    float* beta = nullptr;
  };
  void expect(const std::string& name, std::vector<int64_t> shape);
  const std::vector<float>& host(const std::string& name) const;
  void build_weights();
  void free_weights();
  void free_plan();
  void build_plan();
  void* dev_alloc(size_t bytes, std::vector<void*>& list);
  Conv make_conv(const std::string& prefix, int64_t cin_pad, bool upsampler);
  Norm make_norm(const std::string& prefix);

  VAEConfig cfg_;
  std::map<std::string, HostParam> params_;
  bool weights_built_ = false;
  std::vector<void*> weight_allocs_;
  std::map<std::string, Conv> convs_;
  std::map<std::string, Norm> norms_;
  uint16_t* attn_qkv_w_ = nullptr;  // [3C, C]
  float* attn_qkv_b_ = nullptr;     // [3C]
  uint16_t* attn_out_w_ = nullptr;
  float* attn_out_b_ = nullptr;
  float* bn_mean_ = nullptr;
  float* bn_var_ = nullptr;

  int64_t B_ = 0, ph_ = 0, pw_ = 0, tile_ = 0;
  bool planned_ = false;
  std::vector<void*> allocs_;
  float* lat_dev_ = nullptr;
  float* img_dev_ = nullptr;
  std::vector<Op> ops_;
  cudaGraphExec_t graph_ = nullptr;
};

}  // namespace dcpp

struct dcpp_vae {
  std::unique_ptr<dcpp::AutoencoderKLFlux2Decoder> model;
  dcpp_ctx* ctx = nullptr;
};
