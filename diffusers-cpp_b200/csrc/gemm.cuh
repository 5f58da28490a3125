// Grouped tcgen05 GEMM: Y[rows, N] = X[rows, K] . W_g[N, K]^T with fused
// epilogues.  Host-visible parameter structs and launch entry points.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dcpp {

constexpr int kGemmBM = 128;      // rows per tile (TMEM lanes)
constexpr int kGemmBN = 256;      // columns per tile (TMEM columns per accumulator)
constexpr int kGemmBK = 64;       // K per smem stage (one 128-byte swizzle atom of bf16)
constexpr int kGemmStages = 4;    // smem pipeline depth
constexpr int kGemmMaxGroups = 8; // row groups (txt/img stream x batch)

// B operand source of a GEMM launch.
enum GemmBSource : int {
  kBSrcBf16 = 0,   // bf16 weight [N, K] loaded by TMA (128B swizzle)
  kBSrcQ8_0 = 1,   // Q8_0 weight in the packed stage layout, dequantised in smem inside the GEMM
  kBSrcQ4_K = 2,   // Q4_K weight in the packed stage layout, dequantised in smem inside the GEMM
};

// Epilogue of a GEMM launch.  The accumulator is f32 in TMEM; each
// epilogue thread owns one output row of the 128-row tile.
enum GemmEpilogue : int {
  kEpiF32 = 0,        // out_f32[r, c] = acc
  kEpiBf16 = 1,       // out_bf16[r, c] = bf16(acc)
  kEpiResidGate = 2,  // out_f32[r, c] += gate_g[c] * acc   (gated residual, Flux2TransformerBlock.hpp:86-87)
  kEpiQkvMlp = 3,     // q/k: RMSNorm + RoPE -> [B,H,S,d]; v -> [B,H,S,d]; mlp gate/up -> SwiGLU
  kEpiEuler = 4,      // out_f32[r, c] = x_in[r, c] + dt * acc  (FlowMatchEuler integrate)
  kEpiGateF32 = 5,    // out_f32[r, c] = gate_g[c] * acc   (TP partial before the all-reduce)
  kEpiGatePeer = 6,   // bf16(gate_g[c] * acc) stored into the owning rank's receive slot (TP reduce-scatter)
  kEpiConv = 7,       // v = acc + bias[c] (+ resid[r', c]) -> out_f32 and / or out_bf16 at row r' (convolutions)
};

struct GemmGroup {
  int32_t row0;     // first row of this group in A
  int32_t orow0;    // first row of this group in Y (the epilogue's output)
  int32_t rows;     // number of rows
  int32_t wsel;     // which weight (0 or 1)
  int32_t batch;    // batch index of these rows
  int32_t tile0;    // first linear tile index of the group
  int32_t m_tiles;  // ceil(rows / 128)
  int32_t sel;      // per-group parameter selector (0 = txt stream, 1 = img stream)
  int32_t tok0;     // token index (within its batch) of row0
};

struct EpilogueArgs {
  int mode;
  float* out_f32;
  uint16_t* out_bf16;
  int64_t ld_out;            // row stride of out (elements)
  const float* x_in;         // Euler: previous latents (same layout as out_f32)
  const float* dt;           // Euler: device scalar
  const float* gate[2];      // per selector: gate vector [N] (batch stride gate_bstride)
  int64_t gate_bstride;
  // kEpiQkvMlp
  int32_t qkv_cols;          // columns holding q|k|v (inner + 2 * kv_inner); 0 = mlp only
  int32_t inner;             // local q dim (heads_local * 128)
  int32_t kv_inner;          // local k / v dim (heads_kv * 128); 0: = inner
  int32_t seq;               // tokens per batch element (S)
  int32_t heads;             // local q heads
  int32_t heads_kv;          // local k / v heads (grouped-query attention); 0: = heads
  int32_t rope_neox;         // 0: rotate adjacent pairs (2i, 2i+1); 1: rotate (i, i + 64)
  const float* norm_q[2];    // per selector RMSNorm weights [128]
  const float* norm_k[2];
  float eps;
  const float2* rope;        // [S, 64] (cos, sin) per token and rotary pair
  uint16_t* q_out;           // [B, H, S, 128]
  uint16_t* k_out;           // [B, H_kv, S, 128]
  uint16_t* v_out;           // transposed: [B, H_kv, 128, vt_stride]
  int64_t vt_stride;         // keys per V^T row (S rounded up to 64)
  uint16_t* mlp_out;         // SwiGLU output, row stride ld_mlp
  int64_t ld_mlp;
  // kEpiGatePeer: the rows are cut into pieces of piece_rows rows, each
  // piece into chunks of chunk_rows rows owned by ranks 0, 1, ...: row r of
  // piece p = r / piece_rows belongs to rank o = (r - p piece_rows) / chunk_rows
  // and is row l = p chunk_rows + (r - p piece_rows - o chunk_rows) of that
  // rank's receive slots (peer_bf16[o], mapped from its GPU; slot_rows rows
  // per source rank).  This rank writes slot peer_slot:
  //   peer_bf16[o] + (peer_slot * slot_rows + l) * ld_out.
  // gran_n > 0 (granule ownership): row r belongs to rank (r / 128) % gran_n
  // and is row ((r / 128) / gran_n) 128 + r % 128 of its receive slots
  // (chunk_rows / piece_rows unused).
  uint16_t* peer_bf16[8];
  int32_t chunk_rows;
  int32_t piece_rows;
  int32_t slot_rows;
  int32_t peer_slot;
  int32_t gran_n;
  // kEpiConv: output row r' of accumulator row r is r itself for a plain
  //   GEMM, and for an implicit convolution (ConvGeom) the row-major index
  //   (b H + y) W + x of the pixel the row computes (rows outside the image
  //   are dropped).  bias [N] (may be null); resid: f32 [rows', ld_resid]
  //   added (may be null); up_phase >= 0: the output grid is the 2x
  //   nearest-upsampled one and this launch computes its phase
  //   (a, b) = (up_phase / 2, up_phase % 2): pixel (y, x) goes to
  //   (2y + a, 2x + b) of the [2H, 2W] grid; nchw_hw > 0: out_f32 is NCHW,
  //   element (r', c) at ((b N + c) nchw_hw + r' % nchw_hw).
  const float* bias;
  const float* resid;
  int64_t ld_resid;
  int32_t up_phase;
  int32_t nchw_hw;
  // GroupNorm statistics of the stored values (implicit convolutions only):
  // each warp's 32 accumulator rows write, per group g of gn_cpg channels
  // in its columns, (sum, sum of squares) to
  // gn_part[(row / 32) * 2 gn_groups + 2 g + {0, 1}] (rows outside the image
  // count as zeros).  gn_cpg in {2, 4, 8, 16, 32}; null: none.
  float* gn_part;
  int32_t gn_cpg;
  int32_t gn_groups;
};

// Implicit-GEMM convolution A operand over an NHWC bf16 image [B, H, W, C]
// (C a multiple of 64).  K runs over (tap, channel); every 128 rows of A are
// one tile_h x tile_w pixel rectangle (tile_w * tile_h = 128), rectangles
// ordered (b, ty, tx) over a tiles_y x tiles_x cover of the image, so row
// r of block k is pixel (ty tile_h + r / tile_w, tx tile_w + r % tile_w):
// A[row, t C + c] = X[b, y + dy_t, x + dx_t, c], zero outside the image.
// Each (tap, 64-channel block) of a rectangle is one 4-D TMA load at the
// tap's shifted coordinates; TMA's zero fill is the padding.
struct ConvGeom {
  int32_t taps;        // 0: plain 2-D A
  int32_t cin_blocks;  // C / 64
  int32_t H, W;
  int32_t tile_w, tile_h;
  int32_t tiles_x, tiles_y;
  int8_t dy[9], dx[9];  // tap offsets, each in [-1, 1]
  // 1 (CTA-pair kernel, bf16 weights, 128 x 1 rectangles): the A map is a
  // halo patch map (make_tmap_conv_patch) and every 64-channel block of a
  // rectangle is loaded once as a 3 x 130-pixel patch, each tap reading its
  // shifted 128-row view of it, instead of one box per tap.
  int32_t halo;
};

// A quantised weight packed per (256-row tile, 64-K stage) by
// launch_pack_weight (dequant.cu); stage (n_tile, kb) starts at
// packed + (n_tile * K/64 + kb) * packed_stage_bytes(type).
struct QuantB {
  const void* packed;
};

struct GemmArgs {
  int32_t N, K;
  int32_t n_tiles_n;
  int32_t total_tiles;
  // Tile order (set by gemm_finalize_groups).  The M tiles of all groups form
  // one sequence of m_tiles_all tiles (group g's start at groups[g].tile0).
  // raster 0: bands of `band` M tiles; within a band, N tiles outer and the
  // band's M tiles inner, so the band's A rows stay in L2 while each B tile
  // is read once per band.  raster 1: bands of `band` N tiles; within a band,
  // M tiles outer and the band's N tiles inner (B stays in L2, A is read once
  // per band).  The persistent CTAs walk this order.
  int32_t m_tiles_all;
  int32_t raster;
  int32_t band;
  int32_t n_groups;
  GemmGroup groups[kGemmMaxGroups];
  EpilogueArgs ep;
  QuantB qb[2];
  ConvGeom conv;
  int32_t tile_n;  // columns per tile (set by gemm_finalize_groups)
  // K split (CTA-pair kernel, bf16 B, kEpiF32 only): work unit t covers tile
  // t % tiles_per_split over the K-blocks of slice t / tiles_per_split, and
  // slice s stores its f32 partial at out_f32 + s * split_stride (a reduce
  // kernel sums the slices).  k_splits 0 / 1: none.
  int32_t k_splits;
  int32_t tiles_per_split;
  int64_t split_stride;
  int* err;
  // The tensor-parallel all-gather of A, overlapped with this GEMM (CTA-pair
  // kernel only).  A's rows are cut into 128-row granules; granule g belongs
  // to rank g % ag_n.  epoch = *ag_step * kAgSitesPerStep + ag_site + 1.
  //  * push: two extra warps per CTA (the gemm_pair_ag_kernel variant) copy
  //    this rank's granules of A (ag_rows rows of ag_ld bf16 at ag_a, in
  //    pieces of up to 2 KB, in row order) into every other rank's copy
  //    ag_a_peer[j]; when all pieces of granule g are out, the warp that
  //    stored the last one sets ag_flags_peer[j][g] = epoch (release, system
  //    scope).  ag_count[k] counts the pieces of this rank's k-th granule
  //    stored so far (zero at launch).
  //  * wait: before loading an A tile, the producer waits (bounded) until
  //    ag_flags[g] (this rank's flags, which the others set) reached the epoch
  //    for every granule g of the tile's rows that another rank owns.
  const uint32_t* ag_flags;
  const uint32_t* ag_step;
  int32_t ag_site;
  int32_t ag_rank;
  int32_t ag_n;
  int32_t ag_rows;
  int64_t ag_ld;
  const uint16_t* ag_a;
  uint16_t* ag_a_peer[8];
  uint32_t* ag_flags_peer[8];
  uint32_t* ag_count;
};

// Host-side: build a 2-D bf16 tensor map with 128-byte swizzle for a
// K-major operand [outer rows, inner K] with row stride `ld` elements.
cudaError_t make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                           uint64_t ld_elems, uint32_t box_outer);

// Host-side: 4-D tensor map over an NHWC bf16 image [B, H, W, C] with a
// (64 channel, tile_w, tile_h, 1) box and 128-byte swizzle: the A operand
// of an implicit-GEMM convolution (ConvGeom).
cudaError_t make_tmap_conv(CUtensorMap* map, const void* base, int64_t B, int64_t H, int64_t W, int64_t C,
                           int tile_w, int tile_h);

// The halo patch map of the same image: (64 channel, 130, 3, 1) boxes.
cudaError_t make_tmap_conv_patch(CUtensorMap* map, const void* base, int64_t B, int64_t H, int64_t W, int64_t C);

// Launch the grouped GEMM.  `a` maps X (box 64 x 128), b0/b1 map the two
// bf16 weights (box 64 x 256) when bsrc == kBSrcBf16.
cudaError_t launch_gemm(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                        const GemmArgs& args, int bsrc, int num_sms, cudaStream_t stream);

// Bytes of one packed (256-row, 64-K) stage: Q4_K 10240, Q8_0 17408.
int packed_stage_bytes(int ggml_type);
// Total bytes of a packed [N, K] weight (N padded to 256 rows).
size_t packed_bytes(int ggml_type, int64_t N, int64_t K);

// The 2-SM variant (CTA pairs, 256 x 256 tiles, tcgen05 cta_group::2).  `args`
// must be finalised with tile_m = 256; bf16 B maps use a 128-row box (each
// CTA of the pair loads half of the 256-row B tile).
cudaError_t launch_gemm_pair(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                             const GemmArgs& args, int bsrc, int num_sms, cudaStream_t stream);

// Fill the tile prefix sums of `args` from its groups (M tile of tile_m rows:
// 128 for launch_gemm, 256 for launch_gemm_pair; N tile of tile_n columns:
// 256, or for bf16 weights 128 (both kernels) and 64 / 32 (launch_gemm) --
// the B tensor map's box is tile_n rows, tile_n / 2 for the pair).
void gemm_finalize_groups(GemmArgs& args, int tile_m = kGemmBM, int tile_n = kGemmBN);
// K slices for a CTA-pair bf16 GEMM of `tiles` output tiles whose waves of
// num_sms / 2 pairs are poorly filled: a time model of the tensor work at
// ~1.3 PFLOP/s scaled by the wave fill, plus the reduce's HBM traffic at
// ~5 TB/s (S partials read, the output written, and read as well when the
// reduce adds to it).  Splits only when the model's time drops below
// (1 - min_gain) of the unsplit one, up to max_splits slices of at least
// min_kb K blocks; returns 1 otherwise.
int gemm_choose_k_splits(int64_t tiles, int num_sms, int64_t rows, int64_t N, int64_t K, int max_splits, int min_kb,
                         bool reduce_adds, double min_gain);

// Turn a finalised kEpiF32 launch into k_splits K slices (see GemmArgs).
void gemm_set_k_splits(GemmArgs& args, int k_splits, int64_t split_stride);

}  // namespace dcpp
