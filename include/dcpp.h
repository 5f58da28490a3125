/*
 * dcpp.h -- C ABI of the B200 (sm_100a) Flux2 DiT denoise path.
 *
 * This is the drop-in boundary for the transformer step of diffusers-cpp.
 * In the reference every model module records ggml ops through the virtual
 * `Runtime` op set (src/ggml/Runtime.hpp:7-317), `ExecutionRuntime` executes
 * the graph (src/ggml/ExecutionRuntime.hpp:29-40, .cpp:42-313) and every
 * arithmetic kernel is a ggml op.  Here the same ops are hand-written CUDA
 * kernels behind plain `extern "C"` entry points: device or host pointers,
 * sizes, ggml type ids and an integer status.  No torch and no ggml types
 * appear in any signature.
 *
 * Conventions
 *   - Every call returns a dcpp_status; DCPP_OK == 0.  On error the context
 *     keeps a message, read with dcpp_last_error().  Nothing aborts or traps
 *     on the device: kernels that wait on barriers give up after a bounded
 *     time and report DCPP_ERR_TIMEOUT.
 *   - Tensor shapes are given in PyTorch order (outermost first), as in the
 *     reference's Tensor wrapper (src/ggml/Tensor.hpp:16-401).  A weight of a
 *     Linear is [out_features, in_features], rows contiguous, quantisation
 *     blocks running along in_features, exactly as a GGUF file stores it.
 *   - Pointers named d_* must be device pointers; pointers named p_* may be
 *     host (pageable or pinned) or device pointers (copied with UVA).
 *   - A context is bound to one GPU and one CUDA stream.  Calls on one
 *     context are not re-entrant; use one context per host thread.
 *   - bf16 values are passed as uint16_t bit patterns.
 */
#ifndef DCPP_H
#define DCPP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The reference throws std::runtime_error / invalid_argument
 * (e.g. src/ggml/ExecutionRuntime.cpp:227-228, GGUFLoaderVisitor.cpp:249-250);
 * the C++ host wrapper (dcpp::check) turns a non-zero status back into a
 * std::runtime_error carrying dcpp_last_error(). */
typedef enum dcpp_status {
    DCPP_OK = 0,
    DCPP_ERR_INVALID_ARG = 1,  /* bad pointer, size, shape or name          */
    DCPP_ERR_UNSUPPORTED = 2,  /* type / shape outside what the kernels do  */
    DCPP_ERR_CUDA = 3,         /* a CUDA runtime or driver call failed      */
    DCPP_ERR_NCCL = 4,         /* an NCCL call failed                       */
    DCPP_ERR_TIMEOUT = 5,      /* a bounded device or host wait ran out     */
    DCPP_ERR_OOM = 6,          /* device allocation failed                  */
    DCPP_ERR_STATE = 7,        /* call out of order (e.g. missing params)   */
    DCPP_ERR_NOT_FOUND = 8,    /* unknown parameter name                    */
    DCPP_ERR_INJECTED = 9      /* host-side fault injection (tests)         */
} dcpp_status;

/* ggml type ids, numerically identical to ggml's enum ggml_type
 * (gguf-py 0.19.0 constants.py GGMLQuantizationType). */
enum {
    DCPP_TYPE_F32 = 0,
    DCPP_TYPE_F16 = 1,
    DCPP_TYPE_Q8_0 = 8,
    DCPP_TYPE_Q4_K = 12,
    DCPP_TYPE_BF16 = 30
};

typedef struct dcpp_ctx dcpp_ctx;

/* ---------------------------------------------------------------------- */
/* Context, memory, streams                                                */
/* ---------------------------------------------------------------------- */

/* Library version string and the device architecture it was built for. */
const char* dcpp_version(void);

/* Create a context on CUDA device `device`.  Replaces the reference's
 * Backend/Device pair (src/ggml/Backend.hpp:5-31, Device.hpp:8-27). */
dcpp_status dcpp_init(int device, dcpp_ctx** out_ctx);
dcpp_status dcpp_destroy(dcpp_ctx* ctx);

/* Message of the last failed call on this context (never NULL). */
const char* dcpp_last_error(const dcpp_ctx* ctx);

/* Use an external cudaStream_t (NULL = the context's own stream). */
dcpp_status dcpp_set_stream(dcpp_ctx* ctx, void* cuda_stream);
dcpp_status dcpp_synchronize(dcpp_ctx* ctx);

dcpp_status dcpp_alloc(dcpp_ctx* ctx, size_t bytes, void** d_out);
dcpp_status dcpp_free(dcpp_ctx* ctx, void* d_ptr);
dcpp_status dcpp_memcpy(dcpp_ctx* ctx, void* p_dst, const void* p_src, size_t bytes);

/* Size in bytes of one row of `n` elements of ggml type `type`
 * (ggml_row_size semantics; n must be a multiple of the block size). */
dcpp_status dcpp_row_bytes(int type, int64_t n, size_t* out_bytes);

/* GEMM kernel used by this context's GEMM entry points and the models it
 * creates (read at dcpp_flux2_prepare): 0 = auto (CTA pairs for launches
 * with >= 256 rows), 1 = single-SM tcgen05 kernel (128 x 256 tiles),
 * 2 = CTA-pair kernel (tcgen05 cta_group::2, 256 x 256 tiles). */
dcpp_status dcpp_set_gemm_kernel(dcpp_ctx* ctx, int kind);

/* Attention kernel used by dcpp_attention and the models this context
 * creates (read at dcpp_flux2_prepare): 0 = auto (by the number of waves
 * each needs on 148 SMs), 1 = one 128-row query tile per CTA,
 * 2 = two query tiles per CTA (ping-pong of their softmax and MMAs); both
 * use 128-key tiles. */
dcpp_status dcpp_set_attention_kernel(dcpp_ctx* ctx, int kind);

/* Limit of the cross-GPU barrier waits (the tensor-parallel exchange's flag
 * barriers) in plans prepared after this call, in seconds: 0 restores the
 * default of 1 s, else 0.001 .. 60.  A wait that runs out makes the kernel
 * record an error and return; the call that ran it returns DCPP_ERR_TIMEOUT
 * ("a peer GPU did not arrive") and the context stays usable.  Plays the
 * role of the process-group timeout around the reference's AllReduce
 * (ExecutionRuntime.cpp:227-228 throws on a failed graph compute). */
dcpp_status dcpp_set_wait_timeout(dcpp_ctx* ctx, double seconds);

/* Failure-path self-test of the cross-GPU barrier on one GPU (no counterpart
 * in the reference): runs the tensor-parallel barrier kernel as rank 0 of a
 * group of `nranks` (1..8) whose other ranks are flag slots in local device
 * memory.  Ranks whose bit is set in `arrived_mask` have already arrived;
 * the others never do, so the wait runs out after the context's wait limit
 * (dcpp_set_wait_timeout) and the call returns DCPP_ERR_TIMEOUT.  With every
 * rank arrived it returns DCPP_OK.  Nothing faults or hangs: the kernel
 * gives up and returns. */
dcpp_status dcpp_tp_barrier_selftest(dcpp_ctx* ctx, int nranks, uint32_t arrived_mask);

/* Host-side fault injection for failure-path tests: the `nth` next call
 * (1 = the next one) of entry point `name` (e.g. "dcpp_gemm") returns
 * DCPP_ERR_INJECTED without touching the GPU.  name == NULL clears. */
dcpp_status dcpp_inject_fault(dcpp_ctx* ctx, const char* name, int nth);

/* ---------------------------------------------------------------------- */
/* Op-level entry points (device pointers)                                 */
/* ---------------------------------------------------------------------- */

/* Dequantise `n` weights of ggml type `type` (Q8_0, Q4_K, F16, BF16, F32)
 * to f32, bit-identical to gguf-py 0.19.0 dequantize (quants.py:396-401 for
 * Q8_0, :504-523 for Q4_K), which the reference's tests declare to be what
 * ggml computes (test/utils/__init__.py:198-228).  n % block size == 0.
 * Alignment: d_out 16 bytes; Q4_K blocks 16 bytes (144-byte blocks keep
 * every row of a cudaMalloc'd tensor aligned); Q8_0 blocks 2 bytes. */
dcpp_status dcpp_dequant(dcpp_ctx* ctx, int type, const void* d_blocks, int64_t n, float* d_out);

/* Same values rounded to bf16 (round-to-nearest-even); the GEMM operand. */
dcpp_status dcpp_dequant_bf16(dcpp_ctx* ctx, int type, const void* d_blocks, int64_t n, uint16_t* d_out);

/* Convert f32 -> bf16 (RNE). */
dcpp_status dcpp_f32_to_bf16(dcpp_ctx* ctx, const float* d_in, int64_t n, uint16_t* d_out);

/* y[M,N] (f32) = x[M,K] (bf16) . W[N,K]^T, W of ggml type wtype.
 * The ggml_mul_mat(W, x) of Linear::forward (src/nn/Linear.cpp:17-36,
 * Runtime.hpp:136 mul_mat).  Runs on the tcgen05/TMEM tensor-core GEMM; a
 * non-bf16 W is first expanded to bf16 (the exact dequantised values rounded
 * once) in a context scratch buffer.  When the output tiles fill the CTA pairs
 * poorly (few rows, long K) the product is computed in K slices into f32
 * partials in a second context buffer and summed in slice order into y
 * (deterministic).  K % 8 == 0; M, N arbitrary. */
dcpp_status dcpp_gemm(dcpp_ctx* ctx, int wtype, const void* d_w, int64_t N, int64_t K,
                      const uint16_t* d_x, int64_t M, float* d_y);

/* Dequantisation fused into the GEMM (the models use it when the environment
 * sets DCPP_FUSED_DEQUANT=1; by default they expand each quantised projection
 * to bf16 right before its GEMM, which measured faster).  A Q4_K / Q8_0
 * weight is first packed once (dcpp_pack_weight) from its GGUF rows into
 * stages of 256 rows x 64 K, each one contiguous block that a bulk TMA copy
 * brings into shared memory, holding the raw 4-bit / 8-bit codes and the
 * block scales (Q4_K: d*sc and dmin*m per 32 weights, Q8_0: d) as bf16.
 * dcpp_gemm_packed then dequantises each stage in shared memory with packed
 * bf16x2 arithmetic (w = q*s - m, or q*d, one rounding) straight into the
 * tensor-core operand layout.  Q4_K needs K % 256 == 0, Q8_0 K % 64 == 0.
 * dcpp_packed_bytes gives the packed size (N padded to 256 rows). */
dcpp_status dcpp_packed_bytes(int type, int64_t N, int64_t K, size_t* out_bytes);
dcpp_status dcpp_pack_weight(dcpp_ctx* ctx, int type, const void* d_raw, int64_t N, int64_t K, void* d_packed);
dcpp_status dcpp_gemm_packed(dcpp_ctx* ctx, int wtype, const void* d_packed, int64_t N, int64_t K,
                             const uint16_t* d_x, int64_t M, float* d_y);

/* dcpp_gemm for callers that cannot allocate device memory.  No counterpart
 * in the reference.  Same arguments, result and precision as dcpp_gemm, but
 * it allocates nothing: a quantised W is expanded to bf16 in a fixed 32 MiB
 * device array that is part of the loaded library (held on every GPU that
 * loads it until the process exits), in row chunks that fit it.  This serves
 * hosts that own all device memory through their own pool, code that must
 * not make a synchronising cudaMalloc / cudaFree call mid-sequence, and
 * deployments with a memory budget fixed in advance.
 * Limits: K <= 65536 (else DCPP_ERR_UNSUPPORTED with the reason).  The first
 * call in each CUDA context (per device; again after the host re-creates the
 * context) looks up the array's device address (cudaGetSymbolAddress); make
 * that first call before any stream capture.
 * The array is shared by every call on the device and keeps the last call's
 * contents: calls whose GPU work overlaps (other streams or contexts on the
 * same device) race on it and must be serialised by the caller. */
dcpp_status dcpp_gemm_noalloc(dcpp_ctx* ctx, int wtype, const void* d_w, int64_t N, int64_t K,
                              const uint16_t* d_x, int64_t M, float* d_y);

/* LayerNorm without affine (ggml_norm, eps) followed by adaLN modulation
 * y = norm(x) * (1 + scale) + shift  (Flux2TransformerBlock.hpp:65-66,
 * LayerNorm.cpp:16-32).  x f32 [rows, D]; shift/scale f32 [D]; y bf16. */
dcpp_status dcpp_layernorm_mod(dcpp_ctx* ctx, const float* d_x, int64_t rows, int64_t D,
                               const float* d_shift, const float* d_scale, float eps,
                               uint16_t* d_y);

/* Joint attention with the Flux2 prologue fused:
 *   q,k <- RMSNorm(q|k over head_dim, eps) * w_{q,k}   (RMSNorm.cpp:12-22)
 *   q,k <- RoPE NORMAL per axis section (Flux2PosEmbed.hpp:18-109) using
 *          ids[S,n_axes] (int32) and theta
 *   o    = softmax(q k^T / sqrt(head_dim)) v            (FlashAttentionOp.cpp)
 * qkv: bf16 [B, S, 3, H, head_dim] (the fused q|k|v projection output rows);
 * o: bf16 [B, S, H, head_dim].  head_dim == 128; axes_dims sum to 128. */
dcpp_status dcpp_attention(dcpp_ctx* ctx, const uint16_t* d_qkv, int64_t B, int64_t S, int64_t H,
                           int64_t head_dim, const float* d_norm_q, const float* d_norm_k, float eps,
                           const int32_t* d_ids, int n_axes, const int64_t* axes_dims, float theta,
                           uint16_t* d_out);

/* ---------------------------------------------------------------------- */
/* Model-level entry points: Flux2Transformer2DModel + Euler step          */
/* ---------------------------------------------------------------------- */

/* Mirrors Flux2Transformer2DModel::Config (Flux2Transformer2DModel.hpp:10-31). */
typedef struct dcpp_flux2_config {
    int64_t patch_size;                 /* 1                          */
    int64_t in_channels;                /* 128                        */
    int64_t out_channels;               /* <= 0: same as in_channels  */
    int64_t num_layers;                 /* double-stream blocks       */
    int64_t num_single_layers;          /* single-stream blocks       */
    int64_t attention_head_dim;         /* 128                        */
    int64_t num_attention_heads;
    int64_t joint_attention_dim;
    int64_t timestep_guidance_channels; /* 256                        */
    float mlp_ratio;                    /* 3.0                        */
    int64_t n_axes;                     /* entries used in axes_dims_rope */
    int64_t axes_dims_rope[8];          /* {32,32,32,32}              */
    int64_t rope_theta;                 /* 2000                       */
    float eps;                          /* 1e-6                       */
    int32_t guidance_embeds;            /* 0 / 1                      */
} dcpp_flux2_config;

typedef struct dcpp_flux2 dcpp_flux2;

/* Fill `cfg` with the reference's defaults (Flux2Transformer2DModel.hpp:13-30). */
void dcpp_flux2_config_default(dcpp_flux2_config* cfg);

/* Parse a diffusers transformer/config.json (Config::from_file,
 * Flux2Transformer2DModel.cpp:253-284) into `cfg` (defaults kept for
 * missing keys). */
dcpp_status dcpp_flux2_config_from_file(const char* path, dcpp_flux2_config* cfg);

/* Build the module tree (Flux2Transformer2DModel.cpp:35-109).  Device
 * memory for parameters is allocated as they are set. */
dcpp_status dcpp_flux2_create(dcpp_ctx* ctx, const dcpp_flux2_config* cfg, dcpp_flux2** out_model);
dcpp_status dcpp_flux2_destroy(dcpp_flux2* model);

/* Bind one parameter by its GGUF / module-path name (ModulePath.hpp:7-44),
 * e.g. "single_transformer_blocks.3.attn.to_qkv_mlp_proj.weight".  Accepts
 * the fused GGUF tensors (to_qkv_mlp_proj, to_out, ff.linear_in) that the
 * reference's loader byte-slices (GGUFLoaderVisitor.cpp:283-429) as well as
 * the split per-module names.  Shapes are checked like Parameter::set /
 * GGUFLoaderVisitor::visit (:244-250).  `p_data` holds the raw GGUF bytes. */
dcpp_status dcpp_flux2_set_param(dcpp_flux2* model, const char* name, int type, int n_dims,
                                 const int64_t* shape, const void* p_data, size_t nbytes);

/* Number of parameters still unbound; `first_missing` gets one name. */
dcpp_status dcpp_flux2_missing(dcpp_flux2* model, int* count, char* first_missing, size_t cap);

/* Plan the execution for a problem size: batch B, n_img image tokens and
 * n_txt text tokens.  Allocates the activation arena, encodes tensor maps
 * and (if use_graph) captures the per-step CUDA graph on first use. */
dcpp_status dcpp_flux2_prepare(dcpp_flux2* model, int64_t batch, int64_t n_img, int64_t n_txt,
                               int use_graph);

/* Flux2Transformer2DModel::forward (Flux2Transformer2DModel.cpp:111-231):
 *   hidden [B, n_img, in_channels] f32, encoder [B, n_txt, joint_dim] f32,
 *   timestep [B] f32 (in [0,1]; multiplied by 1000 inside, :199),
 *   img_ids [B?, n_img, n_axes] int32, txt_ids [B?, n_txt, n_axes] int32
 *   (one id set shared by the batch), guidance [B] f32 or NULL,
 *   out [B, n_img, out_channels] f32.  p_* are host or device pointers. */
dcpp_status dcpp_flux2_forward(dcpp_flux2* model, const float* p_hidden, const float* p_encoder,
                               const float* p_timestep, const int32_t* p_img_ids,
                               const int32_t* p_txt_ids, const float* p_guidance, float* p_out);

/* Flux2KleinPipeline::denoise (Flux2KleinPipeline.cpp:496-537) for one
 * schedule step: latents <- latents + dt * forward(latents, ...), with the
 * Euler update (FlowMatchEulerDiscreteScheduler.cpp:210-222) fused into the
 * final projection.  `timestep` is sigma in [0,1] per batch element. */
dcpp_status dcpp_flux2_denoise_step(dcpp_flux2* model, const float* p_latents_in,
                                    const float* p_encoder, const float* p_timestep, float dt,
                                    const int32_t* p_img_ids, const int32_t* p_txt_ids,
                                    float* p_latents_out);

/* Reference-image (img2img / edit) denoising, Flux2KleinPipeline::denoise
 * with image_latents (Flux2KleinPipeline.cpp:511-536): the n_ref reference
 * tokens and their ids join the image stream after the n_img latent tokens
 * (the transformer sees n_img + n_ref image tokens, num_ref_tokens = n_ref),
 * and only the n_img latent tokens' noise prediction is integrated.
 *   prepare_ref        plans B x (n_img + n_ref + n_txt) tokens; n_ref = 0
 *                      is dcpp_flux2_prepare.  forward() on such a plan takes
 *                      the concatenated [B, n_img + n_ref, C] input and ids
 *                      and returns every image token's prediction, as the
 *                      reference's forward does;
 *   denoise_step_ref   latents [B, n_img, C], image_latents [B, n_ref, C],
 *                      image_latent_ids [n_ref, n_axes], the rest as
 *                      dcpp_flux2_denoise_step; latents_out [B, n_img, C];
 *   load_inputs_ref    the resident form: the reference tokens are held
 *                      fixed across run_resident steps; read_latents returns
 *                      [B, n_img, C].
 * On a plan with reference tokens the calls without _ref return
 * DCPP_ERR_INVALID_ARG, and the _ref calls need non-NULL reference inputs. */
dcpp_status dcpp_flux2_prepare_ref(dcpp_flux2* model, int64_t batch, int64_t n_img, int64_t n_ref, int64_t n_txt,
                                   int use_graph);
dcpp_status dcpp_flux2_denoise_step_ref(dcpp_flux2* model, const float* p_latents_in, const float* p_image_latents,
                                        const int32_t* p_image_latent_ids, const float* p_encoder,
                                        const float* p_timestep, float dt, const int32_t* p_img_ids,
                                        const int32_t* p_txt_ids, float* p_latents_out);
dcpp_status dcpp_flux2_load_inputs_ref(dcpp_flux2* model, const float* p_latents, const float* p_image_latents,
                                       const int32_t* p_image_latent_ids, const float* p_encoder,
                                       const int32_t* p_img_ids, const int32_t* p_txt_ids);

/* Resident execution, for callers that keep the latent on the device across
 * the schedule (the reference instead copies the latent through host
 * memory every step, ExecutionRuntime.cpp:218-238,302-313):
 *   load_inputs  copies latents / encoder states / ids into the model's
 *                device buffers once;
 *   set_timestep sets the step's timestep (sigma) and dt;
 *   run_resident runs one denoise step on the resident latent in place;
 *   read_latents copies the current latent out (and synchronises). */
dcpp_status dcpp_flux2_load_inputs(dcpp_flux2* model, const float* p_latents, const float* p_encoder,
                                   const int32_t* p_img_ids, const int32_t* p_txt_ids);
dcpp_status dcpp_flux2_set_timestep(dcpp_flux2* model, float timestep, float dt);
dcpp_status dcpp_flux2_run_resident(dcpp_flux2* model);
dcpp_status dcpp_flux2_read_latents(dcpp_flux2* model, float* p_out);

/* Number of this library's kernel launches in one denoise step. */
dcpp_status dcpp_flux2_launches_per_step(dcpp_flux2* model, int64_t* out);

/* Per-kernel timing of the executed step (no counterpart in the reference,
 * which has only a progress bar).  With profiling on (set before prepare),
 * every kernel launch of a step is bracketed by CUDA event records, which
 * the step's CUDA graph replays; dcpp_flux2_profile sums, for one kind
 * (0 GEMM, 1 attention, 2 LayerNorm, 3 GEMV, 4 dequant, 5 other,
 * 6 all-reduce), the last executed step's milliseconds, algorithmic FLOPs
 * and launch count. */
dcpp_status dcpp_flux2_set_profiling(dcpp_flux2* model, int on);
dcpp_status dcpp_flux2_profile(dcpp_flux2* model, int kind, double* ms, double* flops, int64_t* launches);

/* FlowMatchEulerDiscreteScheduler::schedule (.cpp:68-208) with the
 * pipeline's sigmas 1 - i/n (Flux2KleinPipeline.cpp:348-356) and the
 * default (shift 1, no dynamic shift) scheduler: writes n timesteps
 * (1000*sigma) and n+1 sigmas. */
dcpp_status dcpp_flow_match_schedule(int n, float shift, float* timesteps, float* sigmas);

/* The scheduler's constructor options (FlowMatchEulerDiscreteScheduler.hpp:11-18);
 * dcpp_flow_match_config_default gives the reference's defaults
 * (1000 train timesteps, shift 1, no dynamic shifting, no shift_terminal,
 * not inverted, exponential time shift). */
#define DCPP_TIME_SHIFT_EXPONENTIAL 0
#define DCPP_TIME_SHIFT_LINEAR 1
typedef struct dcpp_flow_match_config {
  int32_t num_train_timesteps;
  float shift;
  int32_t use_dynamic_shifting;
  int32_t has_shift_terminal; /* shift_terminal is set (std::optional) */
  float shift_terminal;
  int32_t invert_sigmas;
  int32_t time_shift_type; /* DCPP_TIME_SHIFT_* */
} dcpp_flow_match_config;
void dcpp_flow_match_config_default(dcpp_flow_match_config* config);

/* FlowMatchEulerDiscreteScheduler::schedule(n, mu, sigmas)
 * (FlowMatchEulerDiscreteScheduler.cpp:68-208) for any configuration:
 * sigmas_in holds n base sigmas, or is NULL for n points from sigma_max = 1
 * down to sigma_min = 1 / num_train_timesteps; writes n timesteps and n + 1
 * sigmas (last 0, or 1 when inverted).  Same float arithmetic as the
 * reference.  DCPP_ERR_INVALID_ARG for n <= 0, num_train_timesteps <= 0, an
 * unknown time_shift_type, or a sigma <= 0 under dynamic shifting (the
 * reference throws std::invalid_argument for each). */
dcpp_status dcpp_flow_match_schedule_ex(const dcpp_flow_match_config* config, int n, float mu,
                                        const float* sigmas_in, float* timesteps, float* sigmas);

/* The pipeline's compute_empirical_mu (Flux2KleinPipeline.cpp:130-141): mu
 * for dynamic shifting from the packed image token count and step count. */
dcpp_status dcpp_flux2_empirical_mu(int64_t image_seq_len, int num_steps, float* mu);

/* The pipeline's RoPE position ids (host memory, int32, 4 axes (t, h, w, l)
 * per token, batch-major):
 *   txt_ids [batch, seq_len, 4] = (0, 0, 0, l)           (prepare_txt_ids, Flux2KleinPipeline.cpp:26-46)
 *   img_ids [batch, packed_h * packed_w, 4] = (0, y, x, 0) (prepare_img_ids, :48-72)
 *   image_latent_ids [batch, sum_i h_i * w_i, 4] = (10 + 10 i, y, x, 0) for
 *     reference image i of packed size packed_hw[2 i] x packed_hw[2 i + 1]
 *     (the image size / (VAE scale factor * 2))      (prepare_ref_image_ids, :75-127)
 * The token counts are batch * ... ; out must hold 4 int32 per token. */
dcpp_status dcpp_flux2_prepare_txt_ids(int64_t batch, int64_t seq_len, int32_t* out);
dcpp_status dcpp_flux2_prepare_img_ids(int64_t batch, int64_t packed_h, int64_t packed_w, int32_t* out);
dcpp_status dcpp_flux2_prepare_ref_image_ids(int64_t batch, int64_t n_images, const int64_t* packed_hw, int32_t* out);

/* ---------------------------------------------------------------------- */
/* Tensor parallelism (the sharding planner's column/row layout)           */
/* ---------------------------------------------------------------------- */

/* Size of the opaque NCCL unique id blob (ncclUniqueId). */
#define DCPP_NCCL_ID_BYTES 128

/* Rank 0 creates the id; all ranks pass it to dcpp_tp_init.  NCCL is
 * loaded at run time (dlopen of libnccl.so.2). */
dcpp_status dcpp_tp_get_unique_id(void* id_out /* DCPP_NCCL_ID_BYTES */);

/* Join a tensor-parallel group of `nranks` GPUs (one process per GPU).
 * Replaces the reference's meta-backend device mesh (MetaDevice.hpp:24-111)
 * and its AllReduce at every P->R bridge (ShardingRuntime.hpp:1082-1091). */
dcpp_status dcpp_tp_init(dcpp_ctx* ctx, int rank, int nranks, const void* nccl_id);

/* In-place sum all-reduce over the TP group (ncclAllReduce); dtype is a
 * DCPP_TYPE_* (F32 or BF16). */
dcpp_status dcpp_allreduce(dcpp_ctx* ctx, void* d_buf, int64_t count, int dtype);

/* Shard a model created on this context over nranks GPUs with equal ratios
 * (heads and MLP features split as evenly as whole heads and 64-feature
 * units allow; see dcpp_flux2_set_tensor_split).  Must be called before
 * set_param.  The layout follows ShardingRuntime.cpp:47-57 (column-parallel
 * q/k/v/gate/up, row-parallel out projections, one all-reduce per
 * row-parallel site). */
dcpp_status dcpp_flux2_set_tensor_parallel(dcpp_flux2* model, int rank, int nranks);

/* The sharding planner's uneven split (tensor_split ratios,
 * ShardingRuntime.cpp:280-296 and :296-528): rank keeps a contiguous run of
 * heads and of MLP features (in units of 64) in proportion to
 * ratios[0..nranks) (NULL = equal ratios, i.e. dcpp_flux2_set_tensor_parallel,
 * which now also accepts head counts that do not divide by nranks).  Each
 * ratio group is rounded like the reference planner: floor of the
 * proportional share, then the remaining units one by one to the ranks with
 * the largest fractional parts, ties to the later rank.  A rank left without
 * a head or without 64 features gives DCPP_ERR_UNSUPPORTED.  Before
 * set_param. */
dcpp_status dcpp_flux2_set_tensor_split(dcpp_flux2* model, int rank, int nranks, const float* ratios);
/* This rank's shard: heads [head0, head0 + heads), MLP features
 * [mlp0, mlp0 + mlp_features) (outputs may be NULL). */
dcpp_status dcpp_flux2_shard(dcpp_flux2* model, int64_t* head0, int64_t* heads, int64_t* mlp0,
                             int64_t* mlp_features);
/* The planner's rounding alone: `units` split over nranks in proportion to
 * ratios (NULL = equal) into out_units[nranks]. */
dcpp_status dcpp_tp_plan_split(int64_t units, int nranks, const float* ratios, int64_t* out_units);

/* A model that assembles parameters on the host only: set_param and
 * set_tensor_parallel work as on a device model (same checks, same shard
 * layout, same load-time conversions), nothing is uploaded and the model
 * cannot execute (prepare returns DCPP_ERR_STATE).  No counterpart in the
 * reference; it lets a loader, or a test without a GPU, inspect the exact
 * shard each rank would hold.  Errors: dcpp_flux2_last_error. */
dcpp_status dcpp_flux2_create_host(const dcpp_flux2_config* cfg, dcpp_flux2** out_model);

/* Text of the last error raised by a call on `model` (also the context's
 * dcpp_last_error for device models). */
const char* dcpp_flux2_last_error(dcpp_flux2* model);

/* Copy an assembled parameter out (host memory), by model name: weights
 * under their fused name (e.g. "transformer_blocks.0.attn.to_qkv",
 * "single_transformer_blocks.0.attn.to_out.weight"; rows and columns are
 * this rank's shard), RMSNorm vectors under their GGUF name (returned as
 * F32, rows 1).  A tensor-parallel column shard that does not fall on the
 * quantisation blocks is held as BF16.  With dst NULL only type, shape and
 * byte size are returned.  Weights held only in the fused-dequant packed
 * layout return DCPP_ERR_UNSUPPORTED. */
dcpp_status dcpp_flux2_read_param(dcpp_flux2* model, const char* name, int* type, int64_t* rows,
                                  int64_t* cols, void* dst, size_t cap, size_t* nbytes);

/* ---------------------------------------------------------------------- */
/* Qwen3 text-encoder prefill (the Flux2 Klein pipeline's prompt encoder)  */
/* ---------------------------------------------------------------------- */

/* Qwen3Config (src/transformers/models/qwen3/Qwen3Config.hpp) fields used
 * by the prefill. */
typedef struct dcpp_qwen3_config {
    int64_t vocab_size;             /* 151936 */
    int64_t hidden_size;            /* 2560   */
    int64_t intermediate_size;      /* 9728   */
    int64_t num_hidden_layers;      /* 36     */
    int64_t num_attention_heads;    /* 32     */
    int64_t num_key_value_heads;    /* 8      */
    int64_t head_dim;               /* 128 (the only value supported) */
    float rms_norm_eps;             /* 1e-6   */
    float rope_theta;               /* 1e6    */
} dcpp_qwen3_config;

typedef struct dcpp_qwen3 dcpp_qwen3;

/* Defaults of the text encoder the Flux2 Klein pipeline loads (the
 * reference benchmark's Qwen3 prefill configuration). */
void dcpp_qwen3_config_default(dcpp_qwen3_config* cfg);
/* Parse a transformers config.json (Qwen3Config::from_file,
 * Qwen3Config.cpp:26-68); defaults kept for missing keys. */
dcpp_status dcpp_qwen3_config_from_file(const char* path, dcpp_qwen3_config* cfg);

/* Build the module tree (Qwen3Model.cpp:11-34). */
dcpp_status dcpp_qwen3_create(dcpp_ctx* ctx, const dcpp_qwen3_config* cfg, dcpp_qwen3** out_model);
dcpp_status dcpp_qwen3_destroy(dcpp_qwen3* model);

/* Bind one parameter by its GGUF / module-path name, with or without the
 * "model." prefix of Qwen3ForCausalLM (e.g. "model.layers.3.mlp.up_proj.weight",
 * "model.embed_tokens.weight", "model.norm.weight"); "lm_head.weight" is
 * accepted and ignored (the prefill returns hidden states).  Linear and
 * embedding weights: Q8_0, Q4_K, F16, BF16 or F32; norm weights F32 / F16 /
 * BF16. */
dcpp_status dcpp_qwen3_set_param(dcpp_qwen3* model, const char* name, int type, int n_dims, const int64_t* shape,
                                 const void* p_data, size_t nbytes);
dcpp_status dcpp_qwen3_missing(dcpp_qwen3* model, int* count, char* first_missing, size_t cap);

/* Plan a prefill of `batch` prompts of `seq` tokens.  tap_layers[n_taps]:
 * layer indices t in [0, num_hidden_layers] whose input hidden states
 * (t = num_hidden_layers: the final normed output) the forward returns,
 * stacked along the feature axis (the pipeline taps 9, 18, 27,
 * Flux2KleinPipeline.cpp:481-491). */
dcpp_status dcpp_qwen3_prepare(dcpp_qwen3* model, int64_t batch, int64_t seq, int n_taps, const int* tap_layers,
                               int use_graph);

/* Qwen3Model::forward (Qwen3Model.cpp:99-208) over input_ids [B, S]
 * (int32, positions 0..S-1, causal attention): attention_mask [B, S] f32
 * (the tokenizer's mask: nonzero = attend, zero = padding key; NULL = all
 * attend), last_hidden [B, S, hidden] f32 after the final RMSNorm (may be
 * NULL), taps [B, S, n_taps * hidden] f32 (may be NULL).  Host or device
 * pointers.  Ids outside the vocabulary give DCPP_ERR_INVALID_ARG. */
dcpp_status dcpp_qwen3_forward(dcpp_qwen3* model, const int32_t* p_input_ids, const float* p_attention_mask,
                               float* p_last_hidden, float* p_taps);

/* Profiling of the prefill plan, as dcpp_flux2_set_profiling / _profile. */
dcpp_status dcpp_qwen3_set_profiling(dcpp_qwen3* model, int on);
dcpp_status dcpp_qwen3_profile(dcpp_qwen3* model, int kind, double* ms, double* flops, int64_t* launches);
dcpp_status dcpp_qwen3_launches_per_step(dcpp_qwen3* model, int64_t* out);

/* ---------------------------------------------------------------------- */
/* GGUF checkpoints (GGUFLoaderVisitor, src/ggml/GGUFLoaderVisitor.cpp)    */
/* ---------------------------------------------------------------------- */

/* A memory-mapped GGUF file (v2 / v3, little-endian).  Replaces the
 * metadata parse of GGUFLoaderVisitor::GGUFLoaderVisitor
 * (GGUFLoaderVisitor.cpp:131-173) and its per-tensor file reads (:15-97,
 * :235-266): tensors are bound straight from the mapping. */
typedef struct dcpp_gguf dcpp_gguf;

/* Open a .gguf file, or the first *.gguf (in name order) of a directory.
 * On failure *out is NULL and err (if err_cap > 0) holds the message
 * ("No such GGUF file in path: ...", "Failed to initialize GGUF file: ...
 * truncated while reading ...", ...). */
dcpp_status dcpp_gguf_open(const char* path, dcpp_gguf** out, char* err, size_t err_cap);
void dcpp_gguf_close(dcpp_gguf* file);
dcpp_status dcpp_gguf_info(const dcpp_gguf* file, uint32_t* version, uint64_t* alignment, uint64_t* data_offset,
                           int64_t* n_tensors, int64_t* n_kv);
/* Tensor i (file order): name (valid while open), ggml type, dimensions in
 * ggml order (ne[0] = row length; unused entries 1), the absolute file
 * offset and byte size of its data, and its bytes in the mapping.  Any
 * output may be NULL. */
dcpp_status dcpp_gguf_tensor(const dcpp_gguf* file, int64_t i, const char** name, int* type, int* n_dims,
                             int64_t ne[4], uint64_t* offset, uint64_t* nbytes, const void** data);
/* Index of the named tensor, -1 if absent. */
int64_t dcpp_gguf_find_tensor(const dcpp_gguf* file, const char* name);
/* Metadata entry i: key (valid while open), GGUF value type (0 u8, 1 i8,
 * 2 u16, 3 i16, 4 u32, 5 i32, 6 f32, 7 bool, 8 string, 9 array, 10 u64,
 * 11 i64, 12 f64), array element type and length (0 for scalars). */
dcpp_status dcpp_gguf_kv(const dcpp_gguf* file, int64_t i, const char** key, uint32_t* type, uint32_t* elem_type,
                         uint64_t* count);
/* Metadata values by key; index -1 reads a scalar, index k >= 0 element k
 * of an array.  Integers and bools through get_int, floats through
 * get_float, strings copied NUL-terminated through get_string.  Unknown
 * key: DCPP_ERR_NOT_FOUND; wrong type, index or too small a buffer:
 * DCPP_ERR_INVALID_ARG. */
dcpp_status dcpp_gguf_get_int(const dcpp_gguf* file, const char* key, int64_t index, int64_t* out);
dcpp_status dcpp_gguf_get_float(const dcpp_gguf* file, const char* key, int64_t index, double* out);
dcpp_status dcpp_gguf_get_string(const dcpp_gguf* file, const char* key, int64_t index, char* buf, size_t cap);

/* Bind every tensor of the file that the model knows, with set_param's
 * name / shape / type rules (the shape is the file's dimensions with
 * trailing unit dimensions dropped, in row-major order, as
 * GGUFLoaderVisitor::visit builds it, :244-258).  Tensors the model does
 * not know are skipped and counted in *n_unused (the reference's validate()
 * only reports them, :175-189).  Afterwards a parameter the file did not
 * provide fails with DCPP_ERR_NOT_FOUND: "Error while loading Tensor
 * '<name>': Tensor not found".  Tensor-parallel models
 * (dcpp_flux2_set_tensor_parallel first) slice their shards from the
 * mapping. */
dcpp_status dcpp_flux2_load_gguf(dcpp_flux2* model, const dcpp_gguf* file, int64_t* n_bound, int64_t* n_unused);
dcpp_status dcpp_qwen3_load_gguf(dcpp_qwen3* model, const dcpp_gguf* file, int64_t* n_bound, int64_t* n_unused);
/* config.json + the GGUF file of one pipeline component folder
 * (Flux2KleinPipeline::from_pretrained, Flux2KleinPipeline.cpp:559-590:
 * "<model>/transformer", "<model>/text_encoder").  Errors: the context's
 * dcpp_last_error. */
dcpp_status dcpp_flux2_from_pretrained(dcpp_ctx* ctx, const char* dir, dcpp_flux2** out_model);
dcpp_status dcpp_qwen3_from_pretrained(dcpp_ctx* ctx, const char* dir, dcpp_qwen3** out_model);

/* ---------------------------------------------------------------------- */
/* Flux2 VAE decode (the pipeline step after the denoise loop)             */
/* ---------------------------------------------------------------------- */

/* AutoencoderKLFlux2::Config (AutoencoderKLFlux2.hpp:10-33). */
typedef struct dcpp_vae_config {
    int64_t in_channels;              /* 3 */
    int64_t out_channels;             /* 3 (1, 3 or 4 supported) */
    int64_t block_out_channels[8];    /* 128, 256, 512, 512 (multiples of 64) */
    int32_t n_blocks;                 /* 4 */
    int64_t layers_per_block;         /* 2 */
    int64_t latent_channels;          /* 32 */
    int64_t norm_num_groups;          /* 32 */
    int64_t sample_size;              /* 1024 */
    int32_t force_upcast;             /* 1 */
    int32_t use_quant_conv;           /* 1 (encoder side, unused by decode) */
    int32_t use_post_quant_conv;      /* 1 */
    int32_t mid_block_add_attention;  /* 1 */
    float batch_norm_eps;             /* 1e-4 */
    float batch_norm_momentum;        /* 0.1 */
    int64_t patch_size[2];            /* 2, 2 (the only value supported) */
} dcpp_vae_config;

typedef struct dcpp_vae dcpp_vae;

void dcpp_vae_config_default(dcpp_vae_config* cfg);
/* AutoencoderKLFlux2::Config::from_file (AutoencoderKLFlux2.cpp:422-468). */
dcpp_status dcpp_vae_config_from_file(const char* path, dcpp_vae_config* cfg);
/* The decoder of AutoencoderKLFlux2 (post_quant_conv, Decoder, the
 * BatchNorm running statistics the pipeline de-normalises with). */
dcpp_status dcpp_vae_create(dcpp_ctx* ctx, const dcpp_vae_config* cfg, dcpp_vae** out_model);
dcpp_status dcpp_vae_destroy(dcpp_vae* model);
/* Bind one parameter by its GGUF name ("decoder.conv_in.weight",
 * "decoder.up_blocks.0.resnets.1.norm2.bias", "bn.running_var", ...).
 * F32, F16, BF16, Q8_0 or Q4_K; shapes as PyTorch's (conv weights
 * [Cout, Cin, k, k]).  Encoder-side names give DCPP_ERR_NOT_FOUND;
 * "bn.num_batches_tracked" is accepted and ignored. */
dcpp_status dcpp_vae_set_param(dcpp_vae* model, const char* name, int type, int n_dims, const int64_t* shape,
                               const void* p_data, size_t nbytes);
dcpp_status dcpp_vae_missing(dcpp_vae* model, int* count, char* first_missing, size_t cap);
/* As dcpp_flux2_load_gguf (a full VAE checkpoint's encoder tensors count
 * as unused). */
dcpp_status dcpp_vae_load_gguf(dcpp_vae* model, const dcpp_gguf* file, int64_t* n_bound, int64_t* n_unused);
/* config.json + the GGUF file of the pipeline's "<model>/vae" folder. */
dcpp_status dcpp_vae_from_pretrained(dcpp_ctx* ctx, const char* dir, dcpp_vae** out_model);
/* Plan the decode of `batch` packed latents of packed_h x packed_w tokens
 * (the DiT's image tokens; image = 2 * scale_factor * packed_h pixels high). */
dcpp_status dcpp_vae_prepare(dcpp_vae* model, int64_t batch, int64_t packed_h, int64_t packed_w, int use_graph);
/* The same with decode_tiled (AutoencoderKLFlux2.cpp:380-405; the
 * pipeline's tile_size argument): tiles of tile_size x tile_size pixels
 * (divisible by the VAE's scale factor) at a 3/4 stride, each decoded on
 * its own and blended with its upper and left neighbours over a quarter
 * tile, so that the activation memory follows the tile size.  Invalid
 * sizes: DCPP_ERR_INVALID_ARG with the reference's message. */
dcpp_status dcpp_vae_prepare_tiled(dcpp_vae* model, int64_t batch, int64_t packed_h, int64_t packed_w,
                                   int64_t tile_size, int use_graph);
/* Flux2KleinPipeline::decode (Flux2KleinPipeline.cpp:538-556), untiled or
 * tiled as prepared: latents [B, packed_h * packed_w, 4 * latent_channels] f32 (the denoised
 * tokens) -> image [B, out_channels, H, W] f32.  Host or device pointers. */
dcpp_status dcpp_vae_decode(dcpp_vae* model, const float* p_latents, float* p_image);
dcpp_status dcpp_vae_set_profiling(dcpp_vae* model, int on);
dcpp_status dcpp_vae_profile(dcpp_vae* model, int kind, double* ms, double* flops, int64_t* launches);
dcpp_status dcpp_vae_launches_per_step(dcpp_vae* model, int64_t* out);

#ifdef __cplusplus
}
#endif

#endif /* DCPP_H */
