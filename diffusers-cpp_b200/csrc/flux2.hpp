// C++ host API of the Flux2 DiT denoise step.  Mirrors the reference's
// module and pipeline surface:
//   Flux2Transformer2DModel::Config / from_file  (Flux2Transformer2DModel.hpp:10-31, .cpp:253-284)
//   Flux2Transformer2DModel::forward             (Flux2Transformer2DModel.cpp:111-231)
//   Flux2KleinPipeline::denoise                  (Flux2KleinPipeline.cpp:496-537)
//   FlowMatchEulerDiscreteScheduler::schedule / integrate (FlowMatchEulerDiscreteScheduler.cpp:68-222)
// Parameters bind by their GGUF names (module paths, ModulePath.hpp) as the
// GGUFLoaderVisitor does, including the fused tensors it byte-slices.
// Execution is a fixed list of launches on the context's stream plus one
// side stream (weight expansion ahead of its GEMM), joined by events and
// optionally replayed from a CUDA graph; every kernel comes from this
// library.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <array>
#include <functional>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "gemm.cuh"
#include "kernels.cuh"
#include "plan.hpp"
#include "runtime.hpp"

namespace dcpp {

struct Flux2Config {
  int64_t patch_size = 1;
  int64_t in_channels = 128;
  int64_t out_channels = -1;  // <= 0: in_channels
  int64_t num_layers = 8;
  int64_t num_single_layers = 48;
  int64_t attention_head_dim = 128;
  int64_t num_attention_heads = 48;
  int64_t joint_attention_dim = 15360;
  int64_t timestep_guidance_channels = 256;
  float mlp_ratio = 3.0f;
  std::vector<int64_t> axes_dims_rope = {32, 32, 32, 32};
  int64_t rope_theta = 2000;
  float eps = 1e-6f;
  bool guidance_embeds = true;

  static Flux2Config from_file(const std::string& path);
  static Flux2Config from_c(const dcpp_flux2_config& c);
  void to_c(dcpp_flux2_config& c) const;
  int64_t inner_dim() const { return num_attention_heads * attention_head_dim; }
  int64_t mlp_hidden() const { return static_cast<int64_t>(inner_dim() * mlp_ratio); }
  int64_t out_ch() const { return patch_size * patch_size * (out_channels > 0 ? out_channels : in_channels); }
};

class Flux2Transformer2DModel : public StepPlanner {
 public:
  // host_only: parameters are assembled (and tensor-parallel sharded) on
  // the host and never uploaded; the model cannot execute.  Used to inspect
  // the exact shards a rank would load, without a GPU.
  Flux2Transformer2DModel(Ctx& ctx, const Flux2Config& cfg, bool host_only = false);
  ~Flux2Transformer2DModel();

  const Flux2Config& config() const { return cfg_; }
  // Shard over nranks GPUs: rank keeps a contiguous run of heads and of MLP
  // features, in proportion to `ratios` (one per rank; empty = even), split
  // by plan_tensor_split.
  void set_tensor_parallel(int rank, int nranks, const std::vector<double>& ratios = {});
  // This rank's shard: first head, heads, first MLP feature, MLP features.
  void shard(int64_t* h0, int64_t* hn, int64_t* f0, int64_t* fn) const {
    *h0 = h0_;
    *hn = hn_;
    *f0 = f0_;
    *fn = fn_;
  }
  void set_param(const std::string& name, int type, const std::vector<int64_t>& shape, const void* data,
                 size_t nbytes);
  std::vector<std::string> missing() const;
  // Copy an assembled parameter by its model name (weights: the fused name,
  // e.g. transformer_blocks.0.attn.to_qkv; vectors: the GGUF name).  With
  // dst == nullptr only the type, shape and byte size are returned.
  void read_param(const std::string& name, int* type, int64_t* rows, int64_t* cols, void* dst, size_t cap,
                  size_t* nbytes);

  // Plan buffers / tensor maps / graph for B x (n_img + n_ref + n_txt)
  // tokens.  n_ref reference-image tokens (img2img / edit) follow the n_img
  // latent tokens in the image stream (Flux2KleinPipeline.cpp:511-519); the
  // denoise step integrates only the latent tokens (:531-536).
  void prepare(int64_t batch, int64_t n_img, int64_t n_txt, bool use_graph, int64_t n_ref = 0);

  // forward(): output = noise prediction of every image token (hidden and
  // img_ids cover the n_img + n_ref image tokens, as the reference's forward
  // receives them).  denoise(): output = latents + dt * v over the n_img
  // latent tokens; ref_latents [B, n_ref, C] / ref_ids [n_ref, n_axes] are
  // the reference tokens (null when the plan has none).
  void forward(const float* hidden, const float* encoder, const float* timestep, const int32_t* img_ids,
               const int32_t* txt_ids, const float* guidance, float* out);
  void denoise(const float* latents, const float* ref_latents, const int32_t* ref_ids, const float* encoder,
               const float* timestep, float dt, const int32_t* img_ids, const int32_t* txt_ids, float* latents_out);

  // Resident execution (inputs already in the model's device buffers):
  // load the inputs once, then run steps; each run integrates the latent
  // in place (ping-pong) so repeated runs follow a schedule.  Reference
  // tokens are loaded into both latent buffers and never integrated.
  void load_inputs(const float* latents, const float* ref_latents, const int32_t* ref_ids, const float* encoder,
                   const int32_t* img_ids, const int32_t* txt_ids);
  void set_timestep(float timestep, float dt);
  void run_resident_step();
  void read_latents(float* out);

  // Profiling: when on (set before prepare), every kernel op of a step is
  // bracketed by CUDA event records; profile() (StepPlanner) sums the last
  // executed step's times per op kind.
  void set_profiling(bool on);

 private:
  struct DoubleBlock {
    DevWeight qkv[2], out[2], ff_in[2], ff_out[2];  // [0] txt stream, [1] img stream
    DevVector norm_q[2], norm_k[2];
  };
  struct SingleBlock {
    DevWeight qkv_mlp, out;
    DevVector norm_q, norm_k;
  };
  void build_registry();
  void place_rows(DevWeight& w, const std::string& part, int type, const std::vector<int64_t>& shape,
                  const uint8_t* src, const std::function<int64_t(int64_t)>& row_map,
                  const std::vector<std::array<int64_t, 3>>& col_ranges);
  void finish_weight(DevWeight& w);
  void expand_staging_bf16(DevWeight& w);
  void require_device(const char* what) const;
  void set_vector(DevVector& v, int type, const std::vector<int64_t>& shape, const void* data, size_t nbytes);
  void free_plan();
  void build_plan();
  void copy_inputs(const float* hidden, const float* encoder, const float* timestep, const int32_t* img_ids,
                   const int32_t* txt_ids, const float* guidance);
  // Latent tokens [B, Nl, C] into latent buffer `buf` (rows strided by the
  // Ni image tokens), reference tokens [B, Nr, C] into both buffers, their
  // ids after the latent tokens' ids.
  void copy_latents(const float* latents, int buf);
  void copy_ref(const float* ref_latents, const int32_t* ref_ids);
  void copy_latents_out(float* out, int buf);
  void check_ref_args(const float* ref_latents, const int32_t* ref_ids, const char* what) const;

  // Plan helpers (tensor parallelism).
  void add_allreduce(float* buf, int64_t count);
  void add_tp_barrier(int set, int stream);
  // The projection weights of block k (double blocks first, then single).
  std::vector<const DevWeight*> block_weights(size_t k) const;

  Flux2Config cfg_;
  bool host_only_ = false;
  int rank_ = 0, nranks_ = 1;
  int64_t h0_ = 0, hn_ = 0, f0_ = 0, fn_ = 0;  // this rank's heads [h0, h0 + hn), MLP features [f0, f0 + fn)
  int64_t D_ = 0, F_ = 0, H_ = 0, Dl_ = 0, Fl_ = 0, Hl_ = 0;

  // Parameters.
  DevWeight time1_, time2_, guid1_, guid2_, mod_img_, mod_txt_, mod_single_, x_embed_, ctx_embed_, norm_out_,
      proj_out_;
  std::vector<DoubleBlock> dbl_;
  std::vector<SingleBlock> sgl_;
  // name -> setter
  std::map<std::string, std::function<void(int, const std::vector<int64_t>&, const void*, size_t)>> setters_;
  std::vector<DevWeight*> weights_;
  std::vector<DevVector*> vectors_;

  // Plan state.
  // Ni_ image tokens per batch element = Nl_ latent tokens + Nr_ reference tokens.
  int64_t B_ = 0, Ni_ = 0, Nt_ = 0, S_ = 0, Nl_ = 0, Nr_ = 0;
  bool planned_ = false;
  bool guidance_given_ = false;
  std::vector<void*> allocs_;
  float *h_ = nullptr, *part_ = nullptr, *lat_[2] = {nullptr, nullptr}, *enc_in_ = nullptr, *t_dev_ = nullptr,
        *g_dev_ = nullptr, *dt_dev_ = nullptr, *out_dev_ = nullptr;
  float *tproj_ = nullptr, *th_ = nullptr, *temb_ = nullptr, *gproj_ = nullptr, *gh_ = nullptr, *gemb_ = nullptr;
  float *mod_img_v_ = nullptr, *mod_txt_v_ = nullptr, *mod_s_v_ = nullptr, *mod_o_v_ = nullptr;
  uint16_t *a_ = nullptr, *q_ = nullptr, *k_ = nullptr, *v_ = nullptr, *cat_ = nullptr, *xb_ = nullptr,
           *eb_ = nullptr;
  int32_t* ids_dev_ = nullptr;
  float2* rope_ = nullptr;
  // Tensor parallelism over peer memory (the default exchange): the
  // row-parallel GEMMs store their gated partials (bf16) straight into the
  // owning rank's receive slots (recv, [nranks][chunk_ rows][D] on each
  // GPU), the owner's LayerNorm sums the slots into its residual rows and
  // stores the normalised bf16 rows into every rank's activation buffer (a_).
  // DCPP_TP_COMM=nccl selects ncclAllReduce of the partials instead.
  // The token rows are cut into tp_pieces_ pieces (1 or 2), each split
  // evenly over the ranks; with two, the LayerNorm + all-gather of piece 1
  // (side stream) overlaps the column-parallel GEMM of piece 0.  Chosen per
  // plan from the exchange size unless DCPP_TP_PIECES sets it.
  bool tp_peer_ = true;
  // Pull form of the peer exchange (DCPP_TP_PULL=1): each
  // row-parallel GEMM keeps its gated bf16 partial in local memory and the
  // row owners read all ranks' partials over NVLink in the LayerNorm, so the
  // GEMM is not held up by NVLink stores and the reads (ingress) overlap the
  // all-gather stores (egress) of the same kernel.  Default (push form): the
  // GEMM epilogue stores each partial into its owner's receive slot, which
  // measured faster at 2 GPUs (the LayerNorm's remote reads cost more than
  // the GEMM saves there).
  bool tp_pull_ = false;
  // Overlapped all-gather (DCPP_TP_OVERLAP=1, with the push form and CTA-pair
  // GEMMs): rows are owned in 128-row granules round-robin over the ranks;
  // the owner's LayerNorm writes only its own rows, and the next
  // column-parallel GEMM starts at once: two extra warps per CTA copy this
  // rank's rows to the other GPUs in row order and raise a per-granule flag
  // there, while its TMA producer waits (bounded) for each tile's granules
  // from the others instead of a barrier for all rows.  Off by default: on
  // the 1024^2 step it measured slower at 2, 4 and 8 GPUs (the GEMM's first
  // wave already needs a third of the rows at 8 GPUs, so it mostly waits for
  // the transfer, and it runs slower beside the NVLink stores).
  bool tp_overlap_ = false;
  bool overlap_ = false;  // in effect for the current plan
  int64_t own_max_ = 0;   // granules per rank, at most
  uint32_t* ag_flags_peer_[8] = {};
  uint32_t* ag_count_ = nullptr;  // [kAgSitesPerStep][own_max_] rows pushed, cleared every step
  uint32_t* step_dev_ = nullptr;
  int tp_pieces_ = 1;
  int tp_pieces_env_ = 0;
  PeerBuffer sym_;
  int64_t piece_rows_ = 0, chunk_ = 0;
  uint16_t* recv_peer_[8] = {};  // bf16 receive slots
  uint16_t* a_peer_[8] = {};
  uint32_t* flags_peer_[2][8] = {};  // barrier flag sets: 0 main stream, 1 side stream
  uint32_t* epoch_[2] = {};
  float* host_scalars_ = nullptr;  // pinned: t[B], dt
  int cur_ = 0;                    // latent ping-pong index
  std::vector<Op> ops_fwd_;        // forward (noise prediction) plan
  std::vector<Op> step_ops_[2];    // denoise step plans (Euler fused), per latent parity
  cudaGraphExec_t graph_fwd_ = nullptr, graph_step_[2] = {nullptr, nullptr};
  // Dequantisation fused into the GEMM (weights packed at load) when
  // DCPP_FUSED_DEQUANT=1.  The default expands each quantised projection to
  // bf16 right before its GEMM, which measured faster for these 4608-row
  // GEMMs (the fused kernels are bound by shared-memory traffic).
  bool fused_dequant_ = false;
  // DCPP_BLOCK_PREFETCH=1: expand each block's quantised weights a whole
  // block ahead, under the previous block's attention, instead of each
  // projection right before its GEMM (overlapping the GEMM before it).
  // Measured equal within noise on config 2 (the step is power-capped), so
  // the default stays per projection.
  bool block_prefetch_ = false;
};

// Units per rank of a tensor-parallel split in proportion to `ratios`
// (floor, then the remainder by largest fractional part, ties to the later
// rank).
std::vector<int64_t> plan_tensor_split(int64_t units, const std::vector<double>& ratios);

// FlowMatchEulerDiscreteScheduler with the reference constructor's options
// and defaults (FlowMatchEulerDiscreteScheduler.hpp:11-18).
struct FlowMatchEulerDiscreteScheduler {
  int num_train_timesteps = 1000;
  float shift = 1.0f;
  bool use_dynamic_shifting = false;
  bool has_shift_terminal = false;
  float shift_terminal = 0.0f;
  bool invert_sigmas = false;
  bool linear_time_shift = false;  // time_shift_type "linear" (default "exponential")
  // schedule(n, mu, sigmas) (FlowMatchEulerDiscreteScheduler.cpp:68-208):
  // base sigmas (`sigmas_in`, n values, or, when empty, n points from
  // sigma_max = 1 down to sigma_min = 1 / num_train_timesteps), shifted
  // (dynamically by mu or statically by `shift`), stretched to
  // shift_terminal, n timesteps (sigma * num_train_timesteps), optionally
  // inverted; n + 1 sigmas (the endpoint 0, or 1 when inverted).
  void schedule(int n, float mu, const std::vector<float>& sigmas_in, std::vector<float>& timesteps,
                std::vector<float>& sigmas) const;
  // The pipeline's call (Flux2KleinPipeline.cpp:348-358): sigmas 1 - i/n,
  // mu = flux2_empirical_mu(image_seq_len, n).
  void pipeline_schedule(int n, int64_t image_seq_len, std::vector<float>& timesteps,
                         std::vector<float>& sigmas) const;
};

// compute_empirical_mu of the Flux2 Klein pipeline (Flux2KleinPipeline.cpp:130-141):
// the dynamic-shift mu for an image of image_seq_len tokens and num_steps steps.
float flux2_empirical_mu(int64_t image_seq_len, int num_steps);

}  // namespace dcpp

struct dcpp_flux2 {
  std::unique_ptr<dcpp::Flux2Transformer2DModel> model;
  dcpp_ctx* ctx = nullptr;
  std::unique_ptr<dcpp_ctx> own_ctx;  // host-only models: error text, no device
};
