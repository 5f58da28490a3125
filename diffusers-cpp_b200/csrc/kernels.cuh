// Launch entry points of the non-GEMM kernels (host-callable, C++ linkage).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace dcpp {

// ggml type ids (ggml enum ggml_type).
constexpr int kTypeF32 = 0;
constexpr int kTypeF16 = 1;
constexpr int kTypeQ8_0 = 8;
constexpr int kTypeQ4_K = 12;
constexpr int kTypeBF16 = 30;

// ---- dequant.cu
cudaError_t launch_dequant_f32(int type, const void* blocks, int64_t n, float* out, cudaStream_t s);
cudaError_t launch_dequant_bf16(int type, const void* blocks, int64_t n, uint16_t* out, cudaStream_t s);
// Raw GGUF rows [N, K] (Q4_K / Q8_0) -> the packed stage layout read by the
// fused-dequant GEMM (gemm.cuh QuantB; packed_bytes(type, N, K) bytes).
cudaError_t launch_pack_weight(int type, const void* raw, int64_t N, int64_t K, void* out, cudaStream_t s);

// ---- rowops.cu
constexpr int kMaxNormSegments = 8;
constexpr int kGranuleRows = 128;  // row granule of the tensor-parallel exchange's ownership
constexpr uint32_t kAgSitesPerStep = 256;  // epochs of the all-gather flags: step * 256 + site + 1

// One contiguous run of rows normalised with one (shift, scale) pair.
struct NormSegment {
  int32_t src_row0;     // first row in x
  int32_t dst_row0;     // first row in y
  int32_t rows;
  const float* shift;   // [D] (may be null -> 0)
  const float* scale;   // [D] (may be null -> 0, i.e. factor 1)
};

struct NormArgs {
  const float* x;       // f32 [*, D] (the residual stream)
  float* x_out;         // if resid: x_out = x + resid (may alias x)
  const float* resid;   // optional addend (TP partials), same layout as x, or n_slots slots (below)
  uint16_t* y;          // bf16 [*, ld_y]
  int64_t ld_x;
  int64_t ld_y;
  int32_t D;
  float eps;
  int32_t n_segments;
  NormSegment seg[kMaxNormSegments];
  // Tensor-parallel reduce + all-gather form (n_slots > 0): the addend of
  // row r is the sum over s < n_slots of the bf16 partials
  // slots[s * slot_stride + (r - slot_row0) * ld_x], added in slot order;
  // the bf16 output row is also stored to y_peer[k] (k < n_peer_out, other
  // GPUs' buffers mapped into this process).
  // With slot_ptr[0] set, slot s is instead slot_ptr[s] + (r - slot_row0) * ld_x
  // (the pull form: each rank's full-row partials in its own memory, read
  // over NVLink by the row's owner).
  const uint16_t* slots;
  int32_t n_slots;
  int64_t slot_stride;
  int64_t slot_row0;
  const uint16_t* slot_ptr[8];
  int32_t n_peer_out;
  uint16_t* y_peer[7];
  // RMSNorm form (rms != 0): no mean subtraction, y = weight * x / rms(x)
  // (weight may be null); the segments' shift / scale are not used.
  int32_t rms;
  const float* weight;
  float* y_f32;         // optional f32 copy of the output (row stride ld_y)
  // Granule form (gran_n > 0): this kernel normalises the rows of the
  // 128-row granules g with g % gran_n == gran_rank, in granule order (block
  // b: granule k = b / 128 of this rank, g = k gran_n + gran_rank, row
  // 128 g + b % 128); each row takes the segment that contains it as src
  // (dst = dst_row0 + row - src_row0), and its slot row is 128 k + b % 128.
  int32_t gran_rank;
  int32_t gran_n;
};

// *step += 1 (one thread): the per-step base of the granule flags' epochs.
cudaError_t launch_step_counter(uint32_t* step, cudaStream_t s);

// out[i, :] = dequantised row ids[i] of table [n_rows, dim] (ggml_get_rows,
// Embedding::forward).  An id outside [0, n_rows) gives a zero row and
// records kDevBadIndex in err.
cudaError_t launch_get_rows(int type, const void* table, int64_t n_rows, int64_t dim, const int32_t* ids,
                            int64_t n_ids, float* out, int* err, cudaStream_t s);

// Attention mask [B, S] (nonzero = attend, as the reference's float mask)
// -> bits [B, words] (bit k % 32 of word k / 32); words >= ceil(S / 32),
// the tail bits are clear.
cudaError_t launch_mask_bits(const float* mask, int64_t B, int64_t S, int64_t words, uint32_t* bits, cudaStream_t s);

// Cross-GPU barrier of a tensor-parallel group.  flags[j] is rank j's flag
// array (mapped from its GPU), one uint32 per source rank; each barrier
// bumps the local epoch, writes it into every rank's flags[.][rank] and waits
// (bounded: kDevTimeoutPeer into err after 1 s) until all of this rank's
// flags reach it.  All writes issued before the barrier on this stream are
// visible to the peers after it.
struct TpBarrierArgs {
  uint32_t* flags[8];
  uint32_t* epoch;   // local device counter
  int* err;
  int32_t rank;
  int32_t nranks;
  uint64_t timeout_ns;  // wait limit; 0 = the library default (1 s)
};
cudaError_t launch_tp_barrier(const TpBarrierArgs& a, cudaStream_t s);

// y = LayerNorm(x) * (1 + scale) + shift, one warp per row.
cudaError_t launch_layernorm_mod(const NormArgs& a, cudaStream_t s);

cudaError_t launch_f32_to_bf16(const float* in, int64_t n, uint16_t* out, cudaStream_t s);

// Rotary table [S, 64] of (cos, sin) for head_dim 128 split into axis
// sections of axes_dims (ggml rope NORMAL, theta_scale = base^(-2/n_dims)).
cudaError_t launch_rope_table(const int32_t* ids, int64_t S, int n_axes, const int32_t* axes_dims_dev,
                              float theta, float2* table, cudaStream_t s);

// Sinusoidal timestep features (Timesteps.cpp:17-46, flip_sin_to_cos):
// out[b, :half] = cos(t_b * mult * f_i), out[b, half:] = sin(...),
// f_i = exp(-ln(10000) * i / half).
cudaError_t launch_timestep_proj(const float* t, int B, int channels, float mult, float* out, cudaStream_t s);

// y[b, n] = act_out( sum_k act_in(x[b, k]) * W[n, k] ), W of ggml type wtype
// in raw GGUF layout; B <= 4 rows.  act: 0 none, 1 SiLU.
cudaError_t launch_gemv(int wtype, const void* W, int64_t N, int64_t K, const float* x, int B, int act_in,
                        int act_out, float* y, cudaStream_t s);

// In-place y += a (f32).
cudaError_t launch_add_f32(float* y, const float* a, int64_t n, cudaStream_t s);

// ---- attention.cu
// Standalone q/k RMSNorm + RoPE + relayout from the fused qkv projection
// rows [B*S, 3*H*128] into q/k [B, H, S, 128] and transposed v
// [B, H, 128, vt_stride] (the tcgen05 attention's operand layouts).
cudaError_t launch_qk_norm_rope(const uint16_t* qkv, int64_t B, int64_t S, int64_t H, const float* norm_q,
                                const float* norm_k, float eps, const float2* rope, uint16_t* q, uint16_t* k,
                                uint16_t* vt, int64_t vt_stride, cudaStream_t s);

// Flux2 VAE decode (vae_ops.cu).  Images are NHWC (row (b H + y) W + x).
// Packed latent tokens [B, ph*pw, 4C] f32 -> BatchNorm de-normalised,
// unpatchified z [B, 2ph, 2pw, Cpad] bf16 (channels >= C zero).
cudaError_t launch_latent_unpack(const float* lat, const float* mean, const float* var, float eps, int B, int ph,
                                 int pw, int C, int Cpad, uint16_t* out, cudaStream_t s);
// GroupNorm statistics: stats[b, g] += (sum, sum of squares) in double over
// x [B, HW, C] (f32, or bf16 when bf16); stats must be zeroed first.
cudaError_t launch_gn_stats(const void* x, bool bf16, int B, int64_t HW, int C, int G, double* stats,
                            cudaStream_t s);
// y = GroupNorm(x) * gamma + beta (then SiLU when silu), bf16 [B, HW, C].
cudaError_t launch_gn_apply(const void* x, bool bf16, int B, int64_t HW, int C, int G, const double* stats,
                            const float* gamma, const float* beta, float eps, bool silu, uint16_t* y,
                            cudaStream_t s);
// P = softmax(scale * S) over each row of n columns (bf16 out); row strides
// multiples of 4 elements.
cudaError_t launch_softmax_rows(const float* S, int64_t rows, int64_t n, int64_t ld_s, float scale, uint16_t* P,
                                int64_t ld_p, cudaStream_t s);
cudaError_t launch_transpose_bf16(const uint16_t* in, int64_t rows, int64_t cols, int64_t ld_in, uint16_t* out,
                                  int64_t ld_out, cudaStream_t s);
// GroupNorm statistics from convolution-epilogue partial sums (gn_part of
// EpilogueArgs): n_regions launches, each region_stride floats, of
// B x slots_per_img slots of 2 G floats -> stats [B, G, 2] (double,
// accumulated: zero it first).
cudaError_t launch_gn_finalize(const float* part, int n_regions, int64_t region_stride, int64_t slots_per_img, int B,
                               int G, double* stats, cudaStream_t s);

// Tiled VAE decode: blend tile T [B, C, h, w] (f32 NCHW) in place with the
// tile above (ha rows high; its last ev rows, may be null) and then the tile
// to the left (wl columns wide; its last eh columns, may be null) with the
// linear ramps of diffusers' blend_v / blend_h, and copy its top-left
// keep_h x keep_w band into out [B, C, H, W] at (oy, ox).
cudaError_t launch_tile_blend(float* T, const float* above, int64_t ha, const float* left, int64_t wl, int B, int C,
                              int64_t h, int64_t w, int64_t ev, int64_t eh, int64_t keep_h, int64_t keep_w, float* out,
                              int64_t H, int64_t W, int64_t oy, int64_t ox, cudaStream_t s);

// K-split GEMM reduction: out[r, c] (+)= sum_{s < S} ws[s * stride + r * ld_ws + c]
// (slices summed in order, then added to out when `add`: deterministic),
// rows x N f32.
cudaError_t launch_split_reduce(const float* ws, int S, int64_t stride, int64_t rows, int64_t N, int64_t ld_ws,
                                float* out, int64_t ld_out, cudaStream_t s, bool add);

}  // namespace dcpp
