// Grouped, persistent tcgen05 GEMM for sm_100a.
//
//   Y[rows, N] = X[rows, K] (bf16) . W_g[N, K]^T (bf16)   f32 accumulate in TMEM
//
// This is the ggml_mul_mat of every Linear on the Flux2 hot path
// (src/nn/Linear.cpp:17-36).  Rows are split into groups that use
// different weights: the double-stream block runs its text-stream
// projections (add_q/k/v, to_add_out, ff_context) and image-stream
// projections (to_q/k/v, to_out, ff) in one launch over the joint
// [txt | img] token buffer (Flux2Attention.hpp:76-89, Flux2TransformerBlock.hpp).
//
// Warp roles (192 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer: A tile 128x64 and B tile 256x64 per stage
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..5  epilogue: TMEM -> registers -> fused epilogue -> global
// Two 128x256 f32 accumulators (512 TMEM columns) let the epilogue of
// tile i overlap the main loop of tile i+1.
#include "common.cuh"
#include "gemm.cuh"
#include "kernels.cuh"

#include <algorithm>

namespace dcpp {

namespace {

constexpr int kAStageBytes = kGemmBM * kGemmBK * 2;  // 16 KB
constexpr int kTmemCols = 512;

struct TileCoord {
  int g;       // group
  int m_tile;  // within group
  int n_tile;
  int split;   // K slice (0 without a K split)
};

__device__ __forceinline__ TileCoord decode_tile(const GemmArgs& p, int t) {
  int split = 0;
  if (p.k_splits > 1) {
    split = t / p.tiles_per_split;
    t -= split * p.tiles_per_split;
  }
  // (outer, inner) extents: raster 0 bands M tiles, raster 1 bands N tiles.
  const int n_out = p.raster ? p.n_tiles_n : p.m_tiles_all;  // the banded dimension
  const int n_in = p.raster ? p.m_tiles_all : p.n_tiles_n;   // walked whole inside a band
  const int band = p.band;
  const int full = n_out / band;
  int b0, bw, u;
  if (t < full * band * n_in) {
    const int b = t / (band * n_in);
    b0 = b * band;
    bw = band;
    u = t - b * band * n_in;
  } else {
    b0 = full * band;
    bw = n_out - b0;
    u = t - full * band * n_in;
  }
  const int across = u / bw;            // index in the unbanded dimension
  const int within = b0 + (u - across * bw);  // index in the banded dimension
  const int m_all = p.raster ? across : within;
  const int n_tile = p.raster ? within : across;
  int g = 0;
#pragma unroll 1
  for (int i = 1; i < p.n_groups; ++i)
    if (m_all >= p.groups[i].tile0) g = i;
  TileCoord c;
  c.g = g;
  c.n_tile = n_tile;
  c.m_tile = m_all - p.groups[g].tile0;
  c.split = split;
  return c;
}

// Wait (bounded) until the rows [r0, r1) of A that other GPUs store have
// arrived: every 128-row granule they touch that another rank owns must show
// the epoch in its flag.  Then the generic-proxy stores that brought them
// are made visible to the async proxy (TMA) of this thread.
__device__ __forceinline__ bool wait_rows_arrived(const GemmArgs& p, int r0, int r1, uint32_t epoch) {
  if (r1 <= r0) return true;
  bool waited = false;
  for (int g = r0 / kGranuleRows; g <= (r1 - 1) / kGranuleRows; ++g) {
    if (g % p.ag_n == p.ag_rank) continue;  // this rank's own rows: written before the launch
    const uint32_t* f = p.ag_flags + g;
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if (static_cast<int32_t>(v - epoch) >= 0) {
      waited = true;
      continue;
    }
    const unsigned long long t0 = globaltimer();
    for (;;) {
      __nanosleep(200);
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if (static_cast<int32_t>(v - epoch) >= 0) break;
      if (error_raised(p.err)) return false;
      if (globaltimer() - t0 > kWaitTimeoutNs) {
        record_error(p.err, kDevTimeoutPeer);
        return false;
      }
    }
    waited = true;
  }
  if (waited) asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// The push half of the overlapped all-gather (GemmArgs::ag_a), run by two
// extra warps per CTA beside the GEMM's roles.  This rank's rows are
// numbered i = 0.. granule by granule (its k-th granule is
// g = k * ag_n + ag_rank; all but the globally last granule are full) and
// cut into pieces of at most 128 16-byte vectors (ppr per row); piece
// q = i * ppr + c.  Warp w of the grid's W push warps takes pieces w,
// w + W, ... in rounds of kAgRound (all loads of a round in flight, then
// the stores to every other rank), so the first rows complete first, which
// is the order the M-outer tile walk consumes them.  After a round, one lane
// per piece makes the stores visible system-wide (fence), counts the piece on
// its granule and, if it was the granule's last, publishes the granule
// (flag = epoch, release) on every other rank.
constexpr int kAgRound = 8;

__device__ __forceinline__ void ag_push_all(const GemmArgs& p, int64_t w, int64_t W, int lane) {
  const int n = p.ag_n, me = p.ag_rank;
  const int64_t ngr = (static_cast<int64_t>(p.ag_rows) + kGranuleRows - 1) / kGranuleRows;
  const int64_t own = ngr > me ? (ngr - me + n - 1) / n : 0;
  if (own == 0) return;
  const int64_t last_g = (own - 1) * n + me;
  const int64_t own_rows =
      (own - 1) * kGranuleRows + min(static_cast<int64_t>(kGranuleRows), p.ag_rows - last_g * kGranuleRows);
  const int vpr = static_cast<int>(p.ag_ld / 8);  // 16-byte vectors per row
  const int ppr = (vpr + 127) / 128;
  const int pv = (vpr + ppr - 1) / ppr;
  const int64_t pieces = own_rows * ppr;
  const uint32_t epoch = *p.ag_step * kAgSitesPerStep + static_cast<uint32_t>(p.ag_site) + 1u;
  for (int64_t q0 = w; q0 < pieces; q0 += kAgRound * W) {
    int64_t off[kAgRound];
    int cnt[kAgRound];
    uint4 v[kAgRound][4];
#pragma unroll
    for (int b = 0; b < kAgRound; ++b) {
      const int64_t q = q0 + b * W;
      cnt[b] = 0;
      off[b] = 0;
      if (q < pieces) {
        const int64_t i = q / ppr;
        const int c0 = static_cast<int>(q - i * ppr) * pv;
        const int64_t k = i / kGranuleRows;
        cnt[b] = min(pv, vpr - c0);
        off[b] = ((k * n + me) * kGranuleRows + (i - k * kGranuleRows)) * p.ag_ld + static_cast<int64_t>(c0) * 8;
        const uint4* src = reinterpret_cast<const uint4*>(p.ag_a + off[b]);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (u * 32 + lane < cnt[b]) v[b][u] = src[u * 32 + lane];
      }
    }
#pragma unroll 1
    for (int j = 0; j < n; ++j) {
      if (j == me) continue;
#pragma unroll
      for (int b = 0; b < kAgRound; ++b) {
        uint4* dst = reinterpret_cast<uint4*>(p.ag_a_peer[j] + off[b]);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (u * 32 + lane < cnt[b]) dst[u * 32 + lane] = v[b][u];
      }
    }
    __syncwarp();
    const int64_t q = q0 + lane * W;
    if (lane < kAgRound && q < pieces) {
      __threadfence_system();
      const int64_t k = q / ppr / kGranuleRows;
      const int64_t g = k * n + me;
      const int64_t rows_g = min(static_cast<int64_t>(kGranuleRows), p.ag_rows - g * kGranuleRows);
      if (atomicAdd(p.ag_count + k, 1u) + 1u == static_cast<uint32_t>(rows_g * ppr)) {
        __threadfence_system();
        for (int j = 0; j < n; ++j)
          if (j != me)
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p.ag_flags_peer[j] + g), "r"(epoch) : "memory");
      }
    }
    __syncwarp();
  }
}

// K blocks [kb0, kb1) of a work unit.
__device__ __forceinline__ void k_range(const GemmArgs& p, const TileCoord& tc, int nk, int& kb0, int& kb1) {
  if (p.k_splits > 1) {
    kb0 = tc.split * nk / p.k_splits;
    kb1 = (tc.split + 1) * nk / p.k_splits;
  } else {
    kb0 = 0;
    kb1 = nk;
  }
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// ------------------------------------------------------------------ epilogue
// One thread = one row of the tile; `taddr` addresses this warp's 32 TMEM
// lanes at the accumulator's column 0.
// `row_base` is the first row (within the group) of the 128 accumulator rows
// this CTA holds: m_tile * 128 for 1-SM tiles, m_tile * 256 + rank * 128 for
// the 2-SM pair.
// Per-warp staging for the peer-store epilogue: 32 rows x 64 columns bf16,
// row stride 144 bytes (16-byte aligned rows; conflict-free 16-byte access
// both row-wise and column-wise).
constexpr int kEpiStageRowBytes = 144;
constexpr int kEpiStageStride = kEpiStageRowBytes / 4;  // in floats
constexpr int kEpiStageBytes = 4 * 32 * kEpiStageRowBytes;

// Warp transpose-reduce: afterwards lane l holds the sum over the warp's
// lanes of a[l] (recursive halving, 31 shuffles for 32 values).
__device__ __forceinline__ float warp_reduce_32(float a[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? a[i] : a[i + off];
      const float keep = upper ? a[i + off] : a[i];
      a[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return a[0];
}

// GroupNorm partial sums of one 32-column chunk (groups of CPG channels);
// warp-collective.  slot_ok: the warp's 32 rows lie inside the launch.
template <int CPG>
__device__ __forceinline__ void gn_chunk_stats(const EpilogueArgs& e, const float v[32], bool valid, bool slot_ok,
                                               int nv, int cb, int64_t row) {
  constexpr int NG = 32 / CPG;
  float a[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) a[i] = 0.f;
  if (valid) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < nv) {
        a[2 * (j / CPG)] += v[j];
        a[2 * (j / CPG) + 1] += v[j] * v[j];
      }
    }
  }
  const float t = warp_reduce_32(a);
  const int lane = threadIdx.x & 31;
  if (slot_ok && lane < 2 * NG) e.gn_part[(row >> 5) * (2 * e.gn_groups) + (cb / CPG) * 2 + lane] = t;
}

// kConv: whether the kernel carries the convolution epilogue (bf16-weight
// kernels; the fused-dequant kernels leave it out for their registers).
template <int BN, bool kConv>
__device__ __forceinline__ void epilogue_row(const GemmArgs& p, const TileCoord& tc, int row_base, int row_in_tile,
                                             uint32_t taddr, float* stage) {
  const GemmGroup& G = p.groups[tc.g];
  const EpilogueArgs& e = p.ep;
  const int local_row = row_base + row_in_tile;
  const bool row_ok = local_row < G.rows;
  const int64_t row = static_cast<int64_t>(G.orow0) + local_row;
  const int col0 = tc.n_tile * BN;
  const int sel = G.sel;

  if (e.mode == kEpiQkvMlp) {
    const int tok = G.tok0 + local_row;
    // 128-column halves (two per 256-column tile); each is one head of q, k or v, or 64 SwiGLU
    // outputs (gate/up interleaved in 64-column blocks by the loader).
#pragma unroll 1
    for (int half = 0; half < BN / 128; ++half) {
      const int c0 = col0 + half * 128;
      if (c0 >= p.N) break;
      const uint32_t hbase = taddr + half * 128;
      if (c0 < e.qkv_cols) {
        const int kvi = e.kv_inner ? e.kv_inner : e.inner;
        const int hkv = e.heads_kv ? e.heads_kv : e.heads;
        const int region = c0 < e.inner ? 0 : (c0 < e.inner + kvi ? 1 : 2);  // q, k, v
        const int head = (c0 - (region == 0 ? 0 : (region == 1 ? e.inner : e.inner + kvi))) >> 7;
        const int nh = region == 0 ? e.heads : hkv;
        uint16_t* dst_base = region == 0 ? e.q_out : (region == 1 ? e.k_out : e.v_out);
        const int64_t dst_row = ((static_cast<int64_t>(G.batch) * nh + head) * e.seq + tok) * 128;
        if (region == 2) {
          // V is stored transposed, [B, H_kv, 128, vt_stride]: the attention's
          // P.V MMA then reads a K-major operand.  Lanes hold consecutive
          // tokens, so each 2-byte store of the warp covers 64 contiguous bytes.
          uint16_t* vt = e.v_out + (static_cast<int64_t>(G.batch) * nh + head) * 128 * e.vt_stride + tok;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld32(hbase + c * 32, r);
            tmem_ld_wait();
            if (row_ok) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                __nv_bfloat16 b = __float2bfloat16_rn(__uint_as_float(r[j]));
                vt[static_cast<int64_t>(c * 32 + j) * e.vt_stride] = *reinterpret_cast<uint16_t*>(&b);
              }
            }
          }
        } else {
          // RMSNorm over the head (RMSNorm.cpp:12-22, ggml_rms_norm) then
          // RoPE NORMAL on adjacent pairs (Flux2PosEmbed.hpp:18-109).
          float ss = 0.f;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld32(hbase + c * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float v = __uint_as_float(r[j]);
              ss = fmaf(v, v, ss);
            }
          }
          const float rs = 1.0f / sqrtf(ss * (1.0f / 128.0f) + e.eps);
          const float* w = region == 0 ? e.norm_q[sel] : e.norm_k[sel];
          const float2* rp = e.rope + static_cast<int64_t>(tok) * 64;
          if (e.rope_neox) {
            // RoPE NEOX (ggml GGML_ROPE_TYPE_NEOX, Qwen3RotaryEmbedding.cpp:15-33):
            // channel d rotates with d + 64 by the angle of pair d.
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
              uint32_t a[32], b[32];
              tmem_ld32(hbase + c * 32, a);
              tmem_ld32(hbase + (c + 2) * 32, b);
              tmem_ld_wait();
              if (row_ok) {
                uint32_t olo[16], ohi[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  float ylo[2], yhi[2];
#pragma unroll
                  for (int t = 0; t < 2; ++t) {
                    const int d = c * 32 + 2 * j + t;
                    const float xa = __uint_as_float(a[2 * j + t]) * rs * __ldg(w + d);
                    const float xb = __uint_as_float(b[2 * j + t]) * rs * __ldg(w + d + 64);
                    const float2 cs = __ldg(rp + d);
                    ylo[t] = xa * cs.x - xb * cs.y;
                    yhi[t] = xb * cs.x + xa * cs.y;
                  }
                  olo[j] = pack_bf16x2(ylo[0], ylo[1]);
                  ohi[j] = pack_bf16x2(yhi[0], yhi[1]);
                }
                uint4* dlo = reinterpret_cast<uint4*>(dst_base + dst_row + c * 32);
                uint4* dhi = reinterpret_cast<uint4*>(dst_base + dst_row + (c + 2) * 32);
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                  dlo[v] = make_uint4(olo[4 * v], olo[4 * v + 1], olo[4 * v + 2], olo[4 * v + 3]);
                  dhi[v] = make_uint4(ohi[4 * v], ohi[4 * v + 1], ohi[4 * v + 2], ohi[4 * v + 3]);
                }
              }
            }
            continue;
          }
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld32(hbase + c * 32, r);
            tmem_ld_wait();
            if (row_ok) {
              uint32_t o[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int d0 = c * 32 + 2 * j;
                float x0 = __uint_as_float(r[2 * j]) * rs * __ldg(w + d0);
                float x1 = __uint_as_float(r[2 * j + 1]) * rs * __ldg(w + d0 + 1);
                float2 cs = __ldg(rp + (d0 >> 1));
                float y0 = x0 * cs.x - x1 * cs.y;
                float y1 = x0 * cs.y + x1 * cs.x;
                o[j] = pack_bf16x2(y0, y1);
              }
              uint4* dst = reinterpret_cast<uint4*>(dst_base + dst_row + c * 32);
#pragma unroll
              for (int v = 0; v < 4; ++v) dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
            }
          }
        }
      } else {
        // SwiGLU: silu(gate) * up (Flux2SwiGLU.hpp:17-21, SiLU.hpp:9-13).
        const int64_t mcol = (c0 - e.qkv_cols) >> 1;  // first of 64 outputs
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t g[32], u[32];
          tmem_ld32(hbase + c * 32, g);
          tmem_ld32(hbase + 64 + c * 32, u);
          tmem_ld_wait();
          if (row_ok) {
            uint4* dst = reinterpret_cast<uint4*>(e.mlp_out + row * e.ld_mlp + mcol + c * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t o[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int i = 8 * v + 2 * j;
                float a0 = silu(__uint_as_float(g[i])) * __uint_as_float(u[i]);
                float a1 = silu(__uint_as_float(g[i + 1])) * __uint_as_float(u[i + 1]);
                o[j] = pack_bf16x2(a0, a1);
              }
              dst[v] = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
        }
      }
    }
    return;
  }

  if (kConv && e.mode == kEpiConv) {
    // Convolution output: pixel row -> output row (2x upsample phase), bias,
    // residual, f32 and / or bf16 NHWC stores or an f32 NCHW store.
    int64_t orow = row;
    bool pix_ok = true;
    if (p.conv.taps) {
      const ConvGeom& g = p.conv;
      const int64_t blk = row >> 7;
      const int r = static_cast<int>(row & 127);
      const int64_t per_img = static_cast<int64_t>(g.tiles_x) * g.tiles_y;
      const int64_t bb = blk / per_img;
      const int rem = static_cast<int>(blk - bb * per_img);
      const int ty = rem / g.tiles_x, tx = rem - ty * g.tiles_x;
      const int y = ty * g.tile_h + r / g.tile_w, x = tx * g.tile_w + r % g.tile_w;
      pix_ok = y < g.H && x < g.W;
      if (e.up_phase >= 0)
        orow = (bb * 2 * g.H + 2 * y + (e.up_phase >> 1)) * (2 * static_cast<int64_t>(g.W)) + 2 * x +
               (e.up_phase & 1);
      else
        orow = (bb * g.H + y) * static_cast<int64_t>(g.W) + x;
    }
    const bool valid = row_ok && pix_ok;
    // Coalesced path: each 32-row x 32-column chunk is staged in shared
    // memory and handled transposed -- lane t owns column quad t & 7 of
    // rows (t >> 3) + 4 i -- so every global load and store of the warp
    // covers whole 128-byte (f32) or 64-byte (bf16) row segments, the
    // residual of the next chunk is loaded while this one is stored, and the
    // GroupNorm partial sums reduce over a few lanes.
    if (e.nchw_hw == 0 && (p.N & 3) == 0 && (e.ld_out & 3) == 0 && (!e.resid || (e.ld_resid & 3) == 0)) {
      const int lane = row_in_tile & 31;
      const int q = lane & 7, rsub = lane >> 3;
      int64_t orows[8];
      bool oks[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        orows[i] = __shfl_sync(0xffffffffu, static_cast<long long>(orow), rsub + 4 * i);
        oks[i] = __shfl_sync(0xffffffffu, valid ? 1 : 0, rsub + 4 * i) != 0;
      }
      const bool slot_ok = __shfl_sync(0xffffffffu, row_ok ? 1 : 0, 0) != 0;
      const int nch = BN / 32;
      float4 rc[8], rn[8];
      auto load_resid = [&](int cbx, float4* dst) {
        const int col = cbx + 4 * q;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          dst[i] = (oks[i] && col < p.N) ? __ldg(reinterpret_cast<const float4*>(e.resid + orows[i] * e.ld_resid + col))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
      };
      if (e.resid) load_resid(col0, rc);
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        const int cb = col0 + c * 32;
        uint32_t r[32];
        tmem_ld32(taddr + c * 32, r);
        tmem_ld_wait();
        if (cb >= p.N) continue;  // warp-uniform
        float4* srow = reinterpret_cast<float4*>(stage + lane * kEpiStageStride);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          srow[k] = make_float4(__uint_as_float(r[4 * k]), __uint_as_float(r[4 * k + 1]),
                                __uint_as_float(r[4 * k + 2]), __uint_as_float(r[4 * k + 3]));
        __syncwarp();
        if (e.resid && c + 1 < nch && cb + 32 < p.N) load_resid(cb + 32, rn);
        const int col = cb + 4 * q;
        const bool col_ok = col < p.N;
        const float4 bia = (e.bias && col_ok) ? __ldg(reinterpret_cast<const float4*>(e.bias + col))
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
        float gs0 = 0.f, gs1 = 0.f, gq0 = 0.f, gq1 = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float4 v = *reinterpret_cast<const float4*>(stage + (rsub + 4 * i) * kEpiStageStride + 4 * q);
          v.x += bia.x; v.y += bia.y; v.z += bia.z; v.w += bia.w;
          if (e.resid) {
            v.x += rc[i].x; v.y += rc[i].y; v.z += rc[i].z; v.w += rc[i].w;
          }
          if (oks[i] && col_ok) {
            if (e.out_f32) *reinterpret_cast<float4*>(e.out_f32 + orows[i] * e.ld_out + col) = v;
            if (e.out_bf16)
              *reinterpret_cast<uint2*>(e.out_bf16 + orows[i] * e.ld_out + col) =
                  make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
            gs0 += v.x + v.y;
            gq0 += v.x * v.x + v.y * v.y;
            gs1 += v.z + v.w;
            gq1 += v.z * v.z + v.w * v.w;
          }
        }
        __syncwarp();  // the stage is rewritten by the next chunk
        if (e.gn_part) {
          float* part = e.gn_part + (row >> 5) * (2 * e.gn_groups);
          const int cpg = e.gn_cpg;
          if (cpg == 2) {  // channel pairs (col, col + 1) and (col + 2, col + 3) are two groups
#pragma unroll
            for (int o = 8; o <= 16; o <<= 1) {
              gs0 += __shfl_xor_sync(0xffffffffu, gs0, o);
              gq0 += __shfl_xor_sync(0xffffffffu, gq0, o);
              gs1 += __shfl_xor_sync(0xffffffffu, gs1, o);
              gq1 += __shfl_xor_sync(0xffffffffu, gq1, o);
            }
            if (slot_ok && rsub == 0 && col_ok) {
              *reinterpret_cast<float4*>(part + col) = make_float4(gs0, gq0, gs1, gq1);
            }
          } else {
            float gs = gs0 + gs1, gq = gq0 + gq1;
#pragma unroll
            for (int o = 8; o <= 16; o <<= 1) {
              gs += __shfl_xor_sync(0xffffffffu, gs, o);
              gq += __shfl_xor_sync(0xffffffffu, gq, o);
            }
            for (int o = 1; o < cpg / 4; o <<= 1) {
              gs += __shfl_xor_sync(0xffffffffu, gs, o);
              gq += __shfl_xor_sync(0xffffffffu, gq, o);
            }
            if (slot_ok && rsub == 0 && col_ok && (q & (cpg / 4 - 1)) == 0) {
              const int g = col / cpg;
              part[2 * g] = gs;
              part[2 * g + 1] = gq;
            }
          }
        }
        if (e.resid) {
#pragma unroll
          for (int i = 0; i < 8; ++i) rc[i] = rn[i];
        }
      }
      return;
    }
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      const int cb = col0 + c * 32;
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_ld_wait();
      if (cb >= p.N) continue;  // warp-uniform
      const int nv = min(32, p.N - cb);
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      if (e.bias) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < nv) v[j] += __ldg(e.bias + cb + j);
      }
      if (valid && e.resid) {
        const float* rs = e.resid + orow * e.ld_resid + cb;
        if (nv == 32 && (reinterpret_cast<uintptr_t>(rs) & 15) == 0) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(rs) + q);
            v[4 * q] += t.x; v[4 * q + 1] += t.y; v[4 * q + 2] += t.z; v[4 * q + 3] += t.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nv) v[j] += rs[j];
        }
      }
      if (e.gn_part) {
        switch (e.gn_cpg) {
          case 2: gn_chunk_stats<2>(e, v, valid, row_ok, nv, cb, row); break;
          case 4: gn_chunk_stats<4>(e, v, valid, row_ok, nv, cb, row); break;
          case 8: gn_chunk_stats<8>(e, v, valid, row_ok, nv, cb, row); break;
          case 16: gn_chunk_stats<16>(e, v, valid, row_ok, nv, cb, row); break;
          default: gn_chunk_stats<32>(e, v, valid, row_ok, nv, cb, row); break;
        }
      }
      if (!valid) continue;
      if (e.nchw_hw > 0) {
        const int64_t bb = orow / e.nchw_hw, hw = orow - bb * e.nchw_hw;
        float* base = e.out_f32 + (bb * p.N + cb) * e.nchw_hw + hw;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < nv) base[static_cast<int64_t>(j) * e.nchw_hw] = v[j];
        continue;
      }
      if (e.out_f32) {
        float* dst = e.out_f32 + orow * e.ld_out + cb;
        if (nv == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            reinterpret_cast<float4*>(dst)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nv) dst[j] = v[j];
        }
      }
      if (e.out_bf16) {
        uint16_t* dst = e.out_bf16 + orow * e.ld_out + cb;
        if (nv == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            reinterpret_cast<uint4*>(dst)[q] =
                make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                           pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j < nv) {
              __nv_bfloat16 b = __float2bfloat16_rn(v[j]);
              dst[j] = *reinterpret_cast<uint16_t*>(&b);
            }
          }
        }
      }
    }
    return;
  }

  // Column-wise epilogues: 8 chunks of 32 columns.
  const float* gate = nullptr;
  const bool gate_only = e.mode == kEpiGateF32 || e.mode == kEpiGatePeer;
  if (e.mode == kEpiResidGate || gate_only) {
    gate = e.gate[sel];
    if (gate) gate += static_cast<int64_t>(G.batch) * e.gate_bstride;
  }
  if (e.mode == kEpiGatePeer) {
    // Rows go to other GPUs over NVLink as bf16: gate and round 64 columns
    // of the warp's 32 rows into shared memory, then store them transposed
    // so that every store instruction writes 4 rows x 128 contiguous bytes
    // (whole lines) instead of 32 scattered pieces.
    const int lane = row_in_tile & 31;
    uintptr_t rdst = 0;
    if (row_ok) {
      int64_t owner, l;
      if (e.gran_n > 0) {
        const int64_t g = row / kGranuleRows;
        owner = g % e.gran_n;
        l = (g / e.gran_n) * kGranuleRows + (row - g * kGranuleRows);
      } else {
        const int64_t pc = row / e.piece_rows;
        const int64_t rp = row - pc * e.piece_rows;
        owner = rp / e.chunk_rows;
        l = pc * e.chunk_rows + (rp - owner * e.chunk_rows);
      }
      rdst = reinterpret_cast<uintptr_t>(e.peer_bf16[owner] +
                                         (static_cast<int64_t>(e.peer_slot) * e.slot_rows + l) * e.ld_out);
    }
    const int sub = lane >> 3, q = lane & 7;
    uint8_t* srow = reinterpret_cast<uint8_t*>(stage) + lane * kEpiStageRowBytes;
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      const int cb = col0 + c * 64;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t r[32];
        tmem_ld32(taddr + c * 64 + h * 32, r);
        tmem_ld_wait();
        const int gc = cb + h * 32;
        const bool g_ok = gate && gc + 32 <= p.N;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          float gv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) gv[i] = 1.f;
          if (g_ok) {
            const float4 g0 = __ldg(reinterpret_cast<const float4*>(gate + gc) + 2 * v);
            const float4 g1 = __ldg(reinterpret_cast<const float4*>(gate + gc) + 2 * v + 1);
            gv[0] = g0.x; gv[1] = g0.y; gv[2] = g0.z; gv[3] = g0.w;
            gv[4] = g1.x; gv[5] = g1.y; gv[6] = g1.z; gv[7] = g1.w;
          } else if (gate) {
#pragma unroll
            for (int i = 0; i < 8; ++i) gv[i] = (gc + 8 * v + i < p.N) ? gate[gc + 8 * v + i] : 0.f;
          }
          uint4 o;
          o.x = pack_bf16x2(gv[0] * __uint_as_float(r[8 * v + 0]), gv[1] * __uint_as_float(r[8 * v + 1]));
          o.y = pack_bf16x2(gv[2] * __uint_as_float(r[8 * v + 2]), gv[3] * __uint_as_float(r[8 * v + 3]));
          o.z = pack_bf16x2(gv[4] * __uint_as_float(r[8 * v + 4]), gv[5] * __uint_as_float(r[8 * v + 5]));
          o.w = pack_bf16x2(gv[6] * __uint_as_float(r[8 * v + 6]), gv[7] * __uint_as_float(r[8 * v + 7]));
          *reinterpret_cast<uint4*>(srow + h * 64 + v * 16) = o;
        }
      }
      __syncwarp();
      const int col = cb + 8 * q;
      const bool col_ok = col + 8 <= p.N;
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int rr = it * 4 + sub;
        const uintptr_t d = __shfl_sync(0xffffffffu, static_cast<unsigned long long>(rdst), rr);
        const uint4 a = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(stage) +
                                                         rr * kEpiStageRowBytes + q * 16);
        if (d && col_ok) *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(d) + col) = a;
      }
      __syncwarp();
    }
    return;
  }
  const float dt = (e.mode == kEpiEuler) ? __ldg(e.dt) : 0.f;
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    const int cb = col0 + c * 32;
    uint32_t r[32];
    tmem_ld32(taddr + c * 32, r);
    tmem_ld_wait();
    if (!row_ok || cb >= p.N) continue;
    // Vector stores need 16-byte aligned rows (ld_out % 4 floats / % 8 bf16).
    bool full = cb + 32 <= p.N;
    if (e.mode == kEpiBf16) {
      uint16_t* dst = e.out_bf16 + row * e.ld_out + cb;
      full = full && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0);
      if (full) {
        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 o;
          o.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1]));
          o.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
          o.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
          o.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
          d4[v] = o;
        }
      } else {
        for (int j = 0; j < 32 && cb + j < p.N; ++j) {
          __nv_bfloat16 b = __float2bfloat16_rn(__uint_as_float(r[j]));
          dst[j] = *reinterpret_cast<uint16_t*>(&b);
        }
      }
      continue;
    }
    float* dst = e.out_f32 + static_cast<int64_t>(tc.split) * p.split_stride + row * e.ld_out + cb;
    full = full && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) &&
           (!gate || (reinterpret_cast<uintptr_t>(gate + cb) & 15) == 0) &&
           (e.mode != kEpiEuler || (reinterpret_cast<uintptr_t>(e.x_in + row * e.ld_out + cb) & 15) == 0);
    if (full) {
      float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        float4 a = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                               __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
        if (e.mode == kEpiF32) {
          d4[v] = a;
        } else if (e.mode == kEpiResidGate || gate_only) {
          float4 gg = gate ? __ldg(reinterpret_cast<const float4*>(gate + cb) + v)
                           : make_float4(1.f, 1.f, 1.f, 1.f);
          if (e.mode == kEpiResidGate) {
            float4 h = d4[v];
            h.x += gg.x * a.x; h.y += gg.y * a.y; h.z += gg.z * a.z; h.w += gg.w * a.w;
            d4[v] = h;
          } else {
            d4[v] = make_float4(gg.x * a.x, gg.y * a.y, gg.z * a.z, gg.w * a.w);
          }
        } else {  // Euler
          const float4 x = __ldg(reinterpret_cast<const float4*>(e.x_in + row * e.ld_out + cb) + v);
          d4[v] = make_float4(x.x + dt * a.x, x.y + dt * a.y, x.z + dt * a.z, x.w + dt * a.w);
        }
      }
    } else {
      for (int j = 0; j < 32 && cb + j < p.N; ++j) {
        float a = __uint_as_float(r[j]);
        if (e.mode == kEpiF32) dst[j] = a;
        else if (e.mode == kEpiResidGate) dst[j] += (gate ? gate[cb + j] : 1.f) * a;
        else if (gate_only) dst[j] = (gate ? gate[cb + j] : 1.f) * a;
        else dst[j] = e.x_in[row * e.ld_out + cb + j] + dt * a;
      }
    }
  }
}

// ------------------------------------------------------------------ implicit conv
// TMA coordinates (channel, x, y, batch) of the A box of rows [m, m + 128)
// for K block kb (ConvGeom).
struct ConvCoord {
  int32_t c, x, y, b;
};
__device__ __forceinline__ ConvCoord conv_coord(const ConvGeom& g, int m, int kb) {
  const int blk = m >> 7;
  const int per_img = g.tiles_x * g.tiles_y;
  ConvCoord o;
  o.b = blk / per_img;
  const int rem = blk - o.b * per_img;
  const int ty = rem / g.tiles_x;
  const int tx = rem - ty * g.tiles_x;
  const int tap = kb / g.cin_blocks;
  o.c = (kb - tap * g.cin_blocks) * 64;
  o.x = tx * g.tile_w + g.dx[tap];
  o.y = ty * g.tile_h + g.dy[tap];
  return o;
}

// ------------------------------------------------------------------ fused dequant
// Quantised B tiles arrive packed per (256-row, 64-K) stage (see
// pack_weight in dequant.cu):
//   Q4_K: [256 rows x 32 B nibbles][256 rows x (s0, m0, s1, m1) bf16]
//   Q8_0: [256 rows x 64 B int8  ][256 rows x (d0, d1) bf16]
// Dequant warps turn one row of a stage into the 64 bf16 values of the B
// tile row, in the 128-byte swizzled K-major layout TMA would have written
// (16-byte chunk c of row r at r*128 + ((c ^ (r & 7)) << 4)).  Arithmetic is
// packed bf16x2: q is built exactly from a 0x4300 magic exponent, then
// w = q * s - m (Q4_K) or w = q * d (Q8_0) with one rounding.
template <int BSRC>
struct BCfg;
template <>
struct BCfg<kBSrcBf16> {
  static constexpr int kStages = 4;
  static constexpr int kRawBytes = 0;
  static constexpr int kDequantWarps = 0;
};
template <>
struct BCfg<kBSrcQ4_K> {
  static constexpr int kStages = 3;
  static constexpr int kRawBytes = kGemmBN * 32 + kGemmBN * 8;  // 10 KB
  static constexpr int kDequantWarps = 8;
};
template <>
struct BCfg<kBSrcQ8_0> {
  static constexpr int kStages = 3;
  static constexpr int kRawBytes = kGemmBN * 64 + kGemmBN * 4;  // 17 KB
  static constexpr int kDequantWarps = 8;
};

template <int BSRC>
constexpr int gemm_threads() { return (6 + BCfg<BSRC>::kDequantWarps) * 32; }
// Narrower N tiles (bf16 weights only) buy deeper pipelines.
template <int BSRC, int BN>
__host__ __device__ constexpr int gemm_stages() {
  return BSRC != kBSrcBf16 || BN >= 256 ? BCfg<BSRC>::kStages : (BN >= 128 ? 6 : 8);
}
template <int BSRC, int BN>
__host__ __device__ constexpr int gemm_stage_bytes() { return kAStageBytes + BN * kGemmBK * 2 + BCfg<BSRC>::kRawBytes; }
template <int BSRC, int BN = kGemmBN>
__host__ __device__ constexpr int gemm_smem_bytes() {
  return gemm_stages<BSRC, BN>() * gemm_stage_bytes<BSRC, BN>() + kEpiStageBytes + 1024 + 256;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

constexpr uint32_t kBf16x2_128 = 0x43004300u;  // (128.0, 128.0)
constexpr uint32_t kHi43 = 0x43434343u;        // byte source for the bf16 high bytes

// prmt selectors: result bytes {a.b0, 0x43, a.b1, 0x43} and {a.b2, 0x43, a.b3, 0x43},
// i.e. the bf16 pair (128 + byte, 128 + byte') for bytes below 128.
constexpr uint32_t kSelLo = 0x5140u;
constexpr uint32_t kSelHi = 0x7362u;

// 8 nibbles (bytes b0..b7 of w0, w1, already masked to 0x0F) -> 4 bf16x2 of
// q * s - m (s2 = (s, s), nm2 = (-m, -m)).
__device__ __forceinline__ uint4 q4_chunk(uint32_t w0, uint32_t w1, uint32_t s2, uint32_t nm2) {
  uint4 o;
  o.x = bf2_fma(bf2_sub(prmt(w0, kHi43, kSelLo), kBf16x2_128), s2, nm2);
  o.y = bf2_fma(bf2_sub(prmt(w0, kHi43, kSelHi), kBf16x2_128), s2, nm2);
  o.z = bf2_fma(bf2_sub(prmt(w1, kHi43, kSelLo), kBf16x2_128), s2, nm2);
  o.w = bf2_fma(bf2_sub(prmt(w1, kHi43, kSelHi), kBf16x2_128), s2, nm2);
  return o;
}

// 8 int8 (bytes of w0, w1) -> 4 bf16x2 of q * d.  q is rebuilt exactly as
// (128 + (b & 127)) - (128 or 256 by the sign bit).
__device__ __forceinline__ uint32_t q8_pair(uint32_t lo7, uint32_t sgn, uint32_t sel, uint32_t d2) {
  const uint32_t v = prmt(lo7, kHi43, sel);
  const uint32_t sub = prmt(sgn, kHi43, sel);  // bytes {0x00|0x80, 0x43}: 128.0 or 256.0
  return bf2_mul(bf2_sub(v, sub), d2);
}
__device__ __forceinline__ uint4 q8_chunk(uint32_t w0, uint32_t w1, uint32_t d2) {
  const uint32_t l0 = w0 & 0x7F7F7F7Fu, s0 = w0 & 0x80808080u;
  const uint32_t l1 = w1 & 0x7F7F7F7Fu, s1 = w1 & 0x80808080u;
  uint4 o;
  o.x = q8_pair(l0, s0, kSelLo, d2);
  o.y = q8_pair(l0, s0, kSelHi, d2);
  o.z = q8_pair(l1, s1, kSelLo, d2);
  o.w = q8_pair(l1, s1, kSelHi, d2);
  return o;
}

// Half a row: 32 of the 64 K values (16-byte chunks 4h .. 4h + 3).  Q4_K:
// h = 0 are the low nibbles (sub-block 2g), h = 1 the high nibbles
// (sub-block 2g + 1); Q8_0: h selects the 32-weight block.
template <int BSRC, int kRows>
__device__ __forceinline__ void dequant_half_row(const uint8_t* raw, uint8_t* btile, int r, int h) {
  uint8_t* dst = btile + r * 128;
  const int sw = r & 7;
  if (BSRC == kBSrcQ4_K) {
    const uint4 qa = *reinterpret_cast<const uint4*>(raw + r * 32);
    const uint4 qb = *reinterpret_cast<const uint4*>(raw + r * 32 + 16);
    const uint32_t sc = *reinterpret_cast<const uint32_t*>(raw + kRows * 32 + r * 8 + h * 4);  // (s, m)
    const uint32_t s2 = prmt(sc, 0, 0x1010), nm2 = prmt(sc, 0, 0x3232) ^ 0x80008000u;
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const int sh = 4 * h;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 o = q4_chunk((w[2 * c] >> sh) & 0x0F0F0F0Fu, (w[2 * c + 1] >> sh) & 0x0F0F0F0Fu, s2, nm2);
      *reinterpret_cast<uint4*>(dst + (((c + 4 * h) ^ sw) << 4)) = o;
    }
  } else {
    const uint4* q = reinterpret_cast<const uint4*>(raw + r * 64 + h * 32);
    const uint32_t ds = *reinterpret_cast<const uint32_t*>(raw + kRows * 64 + r * 4);
    const uint32_t d2 = h ? prmt(ds, 0, 0x3232) : prmt(ds, 0, 0x1010);
#pragma unroll
    for (int i = 0; i < 2; ++i) {  // 16 bytes = K 32h + 16i .. + 15
      const uint4 v = q[i];
      *reinterpret_cast<uint4*>(dst + (((4 * h + 2 * i) ^ sw) << 4)) = q8_chunk(v.x, v.y, d2);
      *reinterpret_cast<uint4*>(dst + (((4 * h + 2 * i + 1) ^ sw) << 4)) = q8_chunk(v.z, v.w, d2);
    }
  }
}

// kRows: rows in the raw stage (256 for the 1-SM tile, 128 per CTA of a pair):
// [kRows x nibbles / int8][kRows x scales].
template <int BSRC, int kRows = kGemmBN>
__device__ __forceinline__ void dequant_row(const uint8_t* raw, uint8_t* btile, int r) {
  uint8_t* dst = btile + r * 128;
  const int sw = r & 7;
  if (BSRC == kBSrcQ4_K) {
    const uint4 qa = *reinterpret_cast<const uint4*>(raw + r * 32);
    const uint4 qb = *reinterpret_cast<const uint4*>(raw + r * 32 + 16);
    const uint2 sc = *reinterpret_cast<const uint2*>(raw + kRows * 32 + r * 8);
    // sc.x = (s0, m0), sc.y = (s1, m1) as bf16 (low half first)
    const uint32_t s0 = prmt(sc.x, 0, 0x1010), nm0 = prmt(sc.x, 0, 0x3232) ^ 0x80008000u;
    const uint32_t s1 = prmt(sc.y, 0, 0x1010), nm1 = prmt(sc.y, 0, 0x3232) ^ 0x80008000u;
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {  // low nibbles: K 8c .. 8c+7 (sub-block 2g)
      const uint4 o = q4_chunk(w[2 * c] & 0x0F0F0F0Fu, w[2 * c + 1] & 0x0F0F0F0Fu, s0, nm0);
      *reinterpret_cast<uint4*>(dst + ((c ^ sw) << 4)) = o;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {  // high nibbles: K 32 + 8c .. (sub-block 2g+1)
      const uint4 o = q4_chunk((w[2 * c] >> 4) & 0x0F0F0F0Fu, (w[2 * c + 1] >> 4) & 0x0F0F0F0Fu, s1, nm1);
      *reinterpret_cast<uint4*>(dst + (((c + 4) ^ sw) << 4)) = o;
    }
  } else {
    const uint4* q = reinterpret_cast<const uint4*>(raw + r * 64);
    const uint32_t ds = *reinterpret_cast<const uint32_t*>(raw + kRows * 64 + r * 4);
    const uint32_t d0 = prmt(ds, 0, 0x1010), d1 = prmt(ds, 0, 0x3232);
#pragma unroll
    for (int h = 0; h < 4; ++h) {  // 16 bytes = K 16h .. 16h+15
      const uint4 v = q[h];
      const uint32_t d2 = h < 2 ? d0 : d1;
      *reinterpret_cast<uint4*>(dst + (((2 * h) ^ sw) << 4)) = q8_chunk(v.x, v.y, d2);
      *reinterpret_cast<uint4*>(dst + (((2 * h + 1) ^ sw) << 4)) = q8_chunk(v.z, v.w, d2);
    }
  }
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------------ kernel
template <int BSRC, int BN>
__global__ void __launch_bounds__(gemm_threads<BSRC>(), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ GemmArgs p) {
  constexpr int kStages = gemm_stages<BSRC, BN>();
  constexpr int kRaw = BCfg<BSRC>::kRawBytes;
  constexpr bool kQuant = BSRC != kBSrcBf16;
  constexpr int kDqThreads = BCfg<BSRC>::kDequantWarps * 32;
  constexpr int kBSt = BN * kGemmBK * 2;  // B stage bytes
  static_assert(!kQuant || BN == kGemmBN, "fused dequantisation uses 256-column tiles");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + kStages * kAStageBytes;
  uint8_t* smR = smB + kStages * kBSt;  // raw quantised stages (kQuant)
  float* epi_stage = reinterpret_cast<float*>(smR + kStages * kRaw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smR + kStages * kRaw + kEpiStageBytes);
  uint64_t* full = bars;                        // [stages] TMA A (+ raw B) landed
  uint64_t* empty = bars + kStages;             // [stages] MMA done with the stage
  uint64_t* bready = bars + 2 * kStages;        // [stages] dequantised B written (kQuant)
  uint64_t* acc_full = bars + 3 * kStages;      // [2]
  uint64_t* acc_empty = acc_full + 2;           // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nk = (p.K + kGemmBK - 1) / kGemmBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&bready[s], kQuant ? BCfg<BSRC>::kDequantWarps : 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    if (!kQuant) {
      tma_prefetch_desc(&tmB0);
      tma_prefetch_desc(&tmB1);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
        const TileCoord tc = decode_tile(p, t);
        const GemmGroup& G = p.groups[tc.g];
        const int ya = G.row0 + tc.m_tile * kGemmBM;
        const int yb = tc.n_tile * BN;
        const void* tmB = G.wsel ? static_cast<const void*>(&tmB1) : static_cast<const void*>(&tmB0);
        const uint8_t* packed = kQuant ? static_cast<const uint8_t*>(p.qb[G.wsel].packed) : nullptr;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait_sleep(&empty[stage], phase ^ 1, p.err, kDevTimeoutEmpty)) { ok = false; break; }
          if (kQuant) {
            mbar_arrive_expect_tx(&full[stage], kAStageBytes + kRaw);
            tma_load_2d(smA + stage * kAStageBytes, &tmA, &full[stage], kb * kGemmBK, ya);
            bulk_load(smR + stage * kRaw, packed + (static_cast<int64_t>(tc.n_tile) * nk + kb) * kRaw, kRaw,
                      &full[stage]);
          } else {
            mbar_arrive_expect_tx(&full[stage], kAStageBytes + kBSt);
            if (p.conv.taps) {
              const ConvCoord cc = conv_coord(p.conv, ya, kb);
              tma_load_4d(smA + stage * kAStageBytes, &tmA, &full[stage], cc.c, cc.x, cc.y, cc.b);
            } else {
              tma_load_2d(smA + stage * kAStageBytes, &tmA, &full[stage], kb * kGemmBK, ya);
            }
            tma_load_2d(smB + stage * kBSt, tmB, &full[stage], kb * kGemmBK, yb);
          }
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // Converged warp, descriptors built once, one elected lane issuing (as in
    // the pair kernel).
    constexpr uint32_t idesc = make_idesc_bf16(kGemmBM, BN);
    const bool leader = elect_one_sync();
    const uint64_t dA = make_sdesc_sw128(smem_u32(smA)), dB = make_sdesc_sw128(smem_u32(smB));
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
      if (!__all_sync(0xffffffffu, mbar_wait_sleep(&acc_empty[acc], acc_phase ^ 1, p.err, kDevTimeoutAccumFree))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < nk; ++kb) {
        uint64_t* ready = kQuant ? &bready[stage] : &full[stage];
        if (!__all_sync(0xffffffffu, mbar_wait_sleep(ready, phase, p.err, kDevTimeoutFull))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t a = dA + static_cast<uint64_t>(stage * (kAStageBytes >> 4));
        const uint64_t b = dB + static_cast<uint64_t>(stage * (kBSt >> 4));
        if (leader) {
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) umma_bf16(d_tmem, a + 2 * k, b + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (leader) umma_commit(&acc_full[acc]);
      __syncwarp();
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  } else if (warp < 6) {
    // Epilogue warps 2..5 -> TMEM lane quarter (warp % 4).
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
      bool ok = mbar_wait(&acc_full[acc], acc_phase, p.err, kDevTimeoutAccum);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const TileCoord tc = decode_tile(p, t);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      epilogue_row<BN, !kQuant>(p, tc, tc.m_tile * kGemmBM, row_in_tile, taddr, epi_stage + quarter * 32 * kEpiStageStride);
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  } else if (kQuant) {
    // Dequant warps 6.. : thread = one B tile row per stage.
    const int r = threadIdx.x - 6 * 32;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < nk; ++kb) {
        ok = __all_sync(0xffffffffu, mbar_wait(&full[stage], phase, p.err, kDevTimeoutDequant));
        if (!ok) break;
        for (int rr = r; rr < kGemmBN; rr += kDqThreads)
          dequant_row<BSRC>(smR + stage * kRaw, smB + stage * kBSt, rr);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bready[stage]);
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------------ 2-SM kernel
// A cluster of two CTAs (two SMs) computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2: CTA rank r holds A rows [128 r, 128 r + 128) and
// B rows (output columns) [128 r, 128 r + 128) of the tile in its own shared
// memory and receives accumulator rows [128 r, 128 r + 128) x 256 in its own
// TMEM.  Rank 0 issues the MMAs; every shared-memory stage holds half the
// bytes of the 1-SM kernel per SM, and with quantised weights each SM
// dequantises only its 128 B rows.  Barriers: full / bready / acc_empty live
// in rank 0 (the MMA waits on them; rank 1 signals them through shared::cluster
// addresses), empty / acc_full in both (the MMA's commit arrives in both).
template <int BSRC>
struct PairCfg;
template <>
struct PairCfg<kBSrcBf16> {
  static constexpr int kStages = 6;
  static constexpr int kQs = 0, kSc = 0;
  static constexpr int kDequantWarps = 0;
};
// Eight dequant warps per CTA: thread t dequantises half of B row t % 128
// (two warps per SM sub-partition, so their instruction latencies overlap).
template <>
struct PairCfg<kBSrcQ4_K> {
  static constexpr int kStages = 5;
  static constexpr int kQs = 32, kSc = 8;
  static constexpr int kDequantWarps = 8;
};
template <>
struct PairCfg<kBSrcQ8_0> {
  static constexpr int kStages = 5;
  static constexpr int kQs = 64, kSc = 4;
  static constexpr int kDequantWarps = 8;
};
constexpr int kPairA = 128 * kGemmBK * 2;  // 16 KB per CTA

template <int BSRC>
__host__ __device__ constexpr int pair_raw_bytes() { return 128 * (PairCfg<BSRC>::kQs + PairCfg<BSRC>::kSc); }
// kPush: two more warps for the overlapped all-gather push (GemmArgs::ag_a;
// bf16 B only).  Only the GEMMs that carry one use this variant: the extra
// warps' registers would keep weight-expansion CTAs off the GEMM's SMs.
// That variant is its own kernel, gemm_pair_ag_kernel<BN>.
template <int BSRC, bool kPush = false>
__host__ __device__ constexpr int pair_threads() {
  return (6 + PairCfg<BSRC>::kDequantWarps + (kPush ? 2 : 0)) * 32;
}
template <int BSRC, int BN>
__host__ __device__ constexpr int pair_stages() {
  return BSRC != kBSrcBf16 || BN >= 256 ? PairCfg<BSRC>::kStages : 8;
}
template <int BSRC, int BN = kGemmBN>
__host__ __device__ constexpr int pair_smem_bytes() {
  return pair_stages<BSRC, BN>() * (kPairA + (BN / 2) * kGemmBK * 2 + pair_raw_bytes<BSRC>()) + kEpiStageBytes +
         1024 + 256;
}

static_assert(gemm_smem_bytes<kBSrcBf16>() <= 232448 && gemm_smem_bytes<kBSrcQ4_K>() <= 232448 &&
                  gemm_smem_bytes<kBSrcQ8_0>() <= 232448 && gemm_smem_bytes<kBSrcBf16, 128>() <= 232448 &&
                  gemm_smem_bytes<kBSrcBf16, 64>() <= 232448 && gemm_smem_bytes<kBSrcBf16, 32>() <= 232448,
              "GEMM shared memory above the 227 KB per-CTA limit");
static_assert(pair_smem_bytes<kBSrcBf16>() <= 232448 && pair_smem_bytes<kBSrcQ4_K>() <= 232448 &&
                  pair_smem_bytes<kBSrcQ8_0>() <= 232448 && pair_smem_bytes<kBSrcBf16, 128>() <= 232448,
              "pair GEMM shared memory above the 227 KB per-CTA limit");

template <int BSRC, int BN, bool kPush>
__device__ __forceinline__ void gemm_pair_body(const CUtensorMap& tmA, const CUtensorMap& tmB0, const CUtensorMap& tmB1,
                                               const GemmArgs& p) {
  constexpr int kStages = pair_stages<BSRC, BN>();
  constexpr int kPB = (BN / 2) * kGemmBK * 2;  // this CTA's half of the B stage
  constexpr bool kQuant = BSRC != kBSrcBf16;
  static_assert(!kQuant || BN == kGemmBN, "fused dequantisation uses 256-column tiles");
  constexpr int kQs = PairCfg<BSRC>::kQs, kSc = PairCfg<BSRC>::kSc;
  constexpr int kRaw = pair_raw_bytes<BSRC>();
  constexpr int kDqWarps = PairCfg<BSRC>::kDequantWarps;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smA + kStages * kPairA;
  uint8_t* smR = smB + kStages * kPB;
  float* epi_stage = reinterpret_cast<float*>(smR + kStages * kRaw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smR + kStages * kRaw + kEpiStageBytes);
  uint64_t* full = bars;                     // [stages] rank 0: A (+ B) bytes of both CTAs
  uint64_t* empty = bars + kStages;          // [stages] both: the MMA released the stage
  uint64_t* rfull = bars + 2 * kStages;      // [stages] both: this CTA's raw quantised rows landed
  uint64_t* bready = bars + 3 * kStages;     // [stages] both: this CTA's dequant warps wrote its B half
  uint64_t* bpeer = bars + 4 * kStages;      // [stages] rank 0: rank 1's B half is ready
  uint64_t* acc_full = bars + 5 * kStages;   // [2] both
  uint64_t* acc_empty = acc_full + 2;        // [2] rank 0: epilogue threads of both CTAs
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int nk = (p.K + kGemmBK - 1) / kGemmBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&rfull[s], 1);
      mbar_init(&bready[s], kQuant ? kDqWarps : 1);
      mbar_init(&bpeer[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 256);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    if (!kQuant) {
      tma_prefetch_desc(&tmB0);
      tma_prefetch_desc(&tmB1);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised before any remote arrive / TMA
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint32_t ag_epoch = p.ag_flags ? *p.ag_step * kAgSitesPerStep + static_cast<uint32_t>(p.ag_site) + 1u : 0u;
      for (int t = pair; t < p.total_tiles && ok; t += npairs) {
        const TileCoord tc = decode_tile(p, t);
        const GemmGroup& G = p.groups[tc.g];
        const int ya = G.row0 + tc.m_tile * 256 + static_cast<int>(rank) * 128;
        const int yb = tc.n_tile * BN + static_cast<int>(rank) * (BN / 2);
        if (p.ag_flags && !wait_rows_arrived(p, ya, min(ya + 128, G.row0 + G.rows), ag_epoch)) {
          ok = false;
          break;
        }
        const void* tmB = G.wsel ? static_cast<const void*>(&tmB1) : static_cast<const void*>(&tmB0);
        const uint8_t* packed = kQuant ? static_cast<const uint8_t*>(p.qb[G.wsel].packed) : nullptr;
        int kb0, kb1;
        k_range(p, tc, nk, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_sleep(&empty[stage], phase ^ 1, p.err, kDevTimeoutEmpty)) { ok = false; break; }
          const uint32_t full0 = mapa_shared(smem_u32(&full[stage]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], kQuant ? 2 * kPairA : 2 * (kPairA + kPB));
          if (!kQuant && p.conv.taps) {
            const ConvCoord cc = conv_coord(p.conv, ya, kb);
            tma_load_4d_pair(smA + stage * kPairA, &tmA, full0, cc.c, cc.x, cc.y, cc.b);
          } else {
            tma_load_2d_pair(smA + stage * kPairA, &tmA, full0, kb * kGemmBK, ya);
          }
          if (kQuant) {
            const uint8_t* st = packed + (static_cast<int64_t>(tc.n_tile) * nk + kb) * (256 * (kQs + kSc));
            mbar_arrive_expect_tx(&rfull[stage], kRaw);
            bulk_load(smR + stage * kRaw, st + rank * 128 * kQs, 128 * kQs, &rfull[stage]);
            bulk_load(smR + stage * kRaw + 128 * kQs, st + 256 * kQs + rank * 128 * kSc, 128 * kSc, &rfull[stage]);
          } else {
            tma_load_2d_pair(smB + stage * kPB, tmB, full0, kb * kGemmBK, yb);
          }
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // The whole warp runs the loop (waits and descriptors are warp-uniform,
      // the descriptors built once); one elected lane issues the MMAs and
      // their commits.  A k step or a stage only moves the descriptor's
      // start-address field (16-byte units, no carry out of its 14 bits).
      constexpr uint32_t idesc = make_idesc_bf16(256, BN);
      const bool leader = elect_one_sync();
      const uint64_t dA = make_sdesc_sw128(smem_u32(smA)), dB = make_sdesc_sw128(smem_u32(smB));
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < p.total_tiles && ok; t += npairs) {
        if (!__all_sync(0xffffffffu, mbar_wait_sleep(&acc_empty[acc], acc_phase ^ 1, p.err, kDevTimeoutAccumFree))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        int kb0, kb1;
        k_range(p, decode_tile(p, t), nk, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          bool w = mbar_wait_sleep(&full[stage], phase, p.err, kDevTimeoutFull);
          if (kQuant)
            w = w && mbar_wait(&bready[stage], phase, p.err, kDevTimeoutDequant) &&
                mbar_wait_cluster(&bpeer[stage], phase, p.err, kDevTimeoutDequant);
          if (!__all_sync(0xffffffffu, w)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a = dA + static_cast<uint64_t>(stage * (kPairA >> 4));
          const uint64_t b = dB + static_cast<uint64_t>(stage * (kPB >> 4));
          if (leader) {
#pragma unroll
            for (int k = 0; k < kGemmBK / 16; ++k)
              umma_bf16_pair(d_tmem, a + 2 * k, b + 2 * k, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
            umma_commit_pair(&empty[stage], 0x3);
          }
          __syncwarp();
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (leader) umma_commit_pair(&acc_full[acc], 0x3);
        __syncwarp();
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    } else if (lane == 0 && kQuant) {
      // Rank 1: forward "my B half is dequantised" to rank 0 with one
      // cluster-scope arrive per stage, so the dequant warps themselves only
      // arrive on a local barrier.
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < p.total_tiles && ok; t += npairs) {
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&bready[stage], phase, p.err, kDevTimeoutDequant)) { ok = false; break; }
          mbar_arrive_cluster(mapa_shared(smem_u32(&bpeer[stage]), 0));
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp < 6) {
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair; t < p.total_tiles; t += npairs) {
      bool ok = mbar_wait(&acc_full[acc], acc_phase, p.err, kDevTimeoutAccum);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const TileCoord tc = decode_tile(p, t);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      epilogue_row<BN, !kQuant>(p, tc, tc.m_tile * 256 + static_cast<int>(rank) * 128, row_in_tile, taddr,
                   epi_stage + quarter * 32 * kEpiStageStride);
      tc_fence_before();
      mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[acc]), 0));
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  } else if (kQuant) {
    const int t_dq = threadIdx.x - 6 * 32;
    const int r = t_dq & 127;  // B row within this CTA's half
    const int h = t_dq >> 7;   // which 32 of the row's 64 K values
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = pair; t < p.total_tiles && ok; t += npairs) {
      for (int kb = 0; kb < nk; ++kb) {
        ok = __all_sync(0xffffffffu, mbar_wait(&rfull[stage], phase, p.err, kDevTimeoutDequant));
        if (!ok) break;
        dequant_half_row<BSRC, 128>(smR + stage * kRaw, smB + stage * kPB, r, h);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bready[stage]);
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
    }
  } else {
    // The all-gather push warps (kPush).
    if constexpr (kPush && !kQuant) {
      if (p.ag_a) ag_push_all(p, static_cast<int64_t>(blockIdx.x) * 2 + (warp - 6), static_cast<int64_t>(gridDim.x) * 2, lane);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no remote arrive may target a CTA that has exited
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <int BSRC, int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair_threads<BSRC>(), 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                     const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ GemmArgs p) {
  gemm_pair_body<BSRC, BN, false>(tmA, tmB0, tmB1, p);
}

template <int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair_threads<kBSrcBf16, true>(), 1)
    gemm_pair_ag_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                        const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ GemmArgs p) {
  gemm_pair_body<kBSrcBf16, BN, true>(tmA, tmB0, tmB1, p);
}

// ------------------------------------------------------------------ conv halo
// Implicit 3x3 / phase convolution on CTA pairs with halo reuse (ConvGeom.halo):
// each CTA's 128-row A block is one image row segment of 128 pixels; per
// 64-channel block the producer loads the 3 x 130-pixel patch around it
// once (one 4-D TMA box, zero fill outside the image), and the MMA of tap
// (dy, dx) reads the 128 rows of the patch starting at row
// (dy + 1) * 130 + dx + 1 -- a shifted view of the 128-byte-swizzled patch
// (the swizzle follows the shared-memory address bits, which TMA and the
// MMA both use, so a view may start at any 128-byte row with a plain
// descriptor; checked against the float64 oracle).  B (bf16 weights) streams one
// (tap, channel block) stage at a time as in gemm_pair_kernel; the
// epilogue is the same.
constexpr int kPatchW = 130, kPatchH = 3;
constexpr int kPatchTxBytes = kPatchW * kPatchH * 128;      // 49920
constexpr int kPatchBytes = (kPatchTxBytes + 1023) / 1024 * 1024;
template <int BN>
__host__ __device__ constexpr int halo_stages() { return BN >= 256 ? 6 : 8; }
template <int BN>
__host__ __device__ constexpr int halo_smem_bytes() {
  return 2 * kPatchBytes + halo_stages<BN>() * (BN / 2) * kGemmBK * 2 + kEpiStageBytes + 1024 + 256;
}
static_assert(halo_smem_bytes<256>() <= 232448 && halo_smem_bytes<128>() <= 232448,
              "halo conv shared memory above the 227 KB per-CTA limit");

template <int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    conv_halo_pair_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ GemmArgs p) {
  constexpr int kStages = halo_stages<BN>();
  constexpr int kPB = (BN / 2) * kGemmBK * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smP = smem;                      // [2] patches
  uint8_t* smB = smP + 2 * kPatchBytes;     // [kStages] this CTA's half of the B stage
  float* epi_stage = reinterpret_cast<float*>(smB + kStages * kPB);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smB + kStages * kPB + kEpiStageBytes);
  uint64_t* bfull = bars;                   // [stages] rank 0: B bytes of both CTAs
  uint64_t* bempty = bars + kStages;        // [stages] both
  uint64_t* pfull = bars + 2 * kStages;     // [2] rank 0: patch bytes of both CTAs
  uint64_t* pempty = pfull + 2;             // [2] both
  uint64_t* acc_full = pempty + 2;          // [2] both
  uint64_t* acc_empty = acc_full + 2;       // [2] rank 0
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const ConvGeom& cg = p.conv;
  const int ncb = cg.cin_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bfull[s], 1);
      mbar_init(&bempty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&pfull[a], 1);
      mbar_init(&pempty[a], 1);
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 256);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmP);
    tma_prefetch_desc(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int bs = 0, ps = 0;
      uint32_t bph = 0, pph = 0;
      bool ok = true;
      for (int t = pair; t < p.total_tiles && ok; t += npairs) {
        const TileCoord tc = decode_tile(p, t);
        const GemmGroup& G = p.groups[tc.g];
        const int blk = (G.row0 + tc.m_tile * 256 + static_cast<int>(rank) * 128) >> 7;
        const int per_img = cg.tiles_x * cg.tiles_y;
        const int b = blk / per_img;
        const int rem = blk - b * per_img;
        const int y0 = rem / cg.tiles_x;
        const int x0 = (rem - y0 * cg.tiles_x) * 128;
        const int yb = tc.n_tile * BN + static_cast<int>(rank) * (BN / 2);
        for (int cb = 0; cb < ncb && ok; ++cb) {
          if (!mbar_wait_sleep(&pempty[ps], pph ^ 1, p.err, kDevTimeoutEmpty)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(&pfull[ps], 2 * kPatchTxBytes);
          tma_load_4d_pair(smP + ps * kPatchBytes, &tmP, mapa_shared(smem_u32(&pfull[ps]), 0), cb * 64, x0 - 1,
                           y0 - 1, b);
          for (int tap = 0; tap < cg.taps; ++tap) {
            if (!mbar_wait_sleep(&bempty[bs], bph ^ 1, p.err, kDevTimeoutEmpty)) { ok = false; break; }
            if (rank == 0) mbar_arrive_expect_tx(&bfull[bs], 2 * kPB);
            tma_load_2d_pair(smB + bs * kPB, &tmB, mapa_shared(smem_u32(&bfull[bs]), 0),
                             (tap * ncb + cb) * kGemmBK, yb);
            if (++bs == kStages) { bs = 0; bph ^= 1; }
          }
          if (++ps == 2) { ps = 0; pph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // Converged warp, descriptors built once, one elected lane issuing (as
      // in the pair GEMM); a tap's view of the patch moves the start field
      // by its row offset.
      constexpr uint32_t idesc = make_idesc_bf16(256, BN);
      const bool leader = elect_one_sync();
      const uint64_t dP = make_sdesc_sw128(smem_u32(smP)), dB = make_sdesc_sw128(smem_u32(smB));
      int bs = 0, ps = 0, acc = 0;
      uint32_t bph = 0, pph = 0, acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < p.total_tiles && ok; t += npairs) {
        if (!__all_sync(0xffffffffu, mbar_wait_sleep(&acc_empty[acc], acc_phase ^ 1, p.err, kDevTimeoutAccumFree))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool first = true;
        for (int cb = 0; cb < ncb && ok; ++cb) {
          if (!__all_sync(0xffffffffu, mbar_wait_sleep(&pfull[ps], pph, p.err, kDevTimeoutFull))) {
            ok = false;
            break;
          }
          const uint64_t patch = dP + static_cast<uint64_t>(ps * (kPatchBytes >> 4));
          for (int tap = 0; tap < cg.taps; ++tap) {
            if (!__all_sync(0xffffffffu, mbar_wait_sleep(&bfull[bs], bph, p.err, kDevTimeoutFull))) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t a = patch + static_cast<uint64_t>(((cg.dy[tap] + 1) * kPatchW + cg.dx[tap] + 1) * 8);
            const uint64_t b = dB + static_cast<uint64_t>(bs * (kPB >> 4));
            if (leader) {
#pragma unroll
              for (int k = 0; k < kGemmBK / 16; ++k)
                umma_bf16_pair(d_tmem, a + 2 * k, b + 2 * k, idesc, (first && k == 0) ? 0u : 1u);
              umma_commit_pair(&bempty[bs], 0x3);
            }
            __syncwarp();
            first = false;
            if (++bs == kStages) { bs = 0; bph ^= 1; }
          }
          if (leader) umma_commit_pair(&pempty[ps], 0x3);
          __syncwarp();
          if (++ps == 2) { ps = 0; pph ^= 1; }
        }
        if (!ok) break;
        if (leader) umma_commit_pair(&acc_full[acc], 0x3);
        __syncwarp();
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  } else {
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair; t < p.total_tiles; t += npairs) {
      bool ok = mbar_wait(&acc_full[acc], acc_phase, p.err, kDevTimeoutAccum);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const TileCoord tc = decode_tile(p, t);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      epilogue_row<BN, true>(p, tc, tc.m_tile * 256 + static_cast<int>(rank) * 128, row_in_tile, taddr,
                             epi_stage + quarter * 32 * kEpiStageStride);
      tc_fence_before();
      mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[acc]), 0));
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

template <int BSRC, int BN = kGemmBN>
cudaError_t launch_gemm_t(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1, const GemmArgs& args,
                          int num_sms, cudaStream_t stream) {
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<BSRC, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         gemm_smem_bytes<BSRC, BN>());
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const int grid = std::min(args.total_tiles, num_sms);
  gemm_kernel<BSRC, BN><<<grid, gemm_threads<BSRC>(), gemm_smem_bytes<BSRC, BN>(), stream>>>(a, b0, b1, args);
  return cudaGetLastError();
}

template <int BSRC, int BN = kGemmBN, bool kPush = false>
cudaError_t launch_gemm_pair_t(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1,
                               const GemmArgs& args, int num_sms, cudaStream_t stream) {
  void (*kern)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const GemmArgs) = nullptr;
  if constexpr (kPush)
    kern = gemm_pair_ag_kernel<BN>;
  else
    kern = gemm_pair_kernel<BSRC, BN>;
  static int max_clusters = 0;
  if (max_clusters == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         pair_smem_bytes<BSRC, BN>());
    if (e != cudaSuccess) return e;
    // Persistent grid: only as many pairs as can be resident at once (a GPC
    // with an odd SM count leaves one SM out of the pairs).
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * (num_sms / 2), 1, 1);
    cfg.blockDim = dim3(pair_threads<BSRC, kPush>(), 1, 1);
    cfg.dynamicSmemBytes = pair_smem_bytes<BSRC, BN>();
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess) return e;
    if (n <= 0) return cudaErrorInvalidConfiguration;
    max_clusters = n;
  }
  const int pairs = std::min(args.total_tiles, max_clusters);
  kern<<<2 * pairs, pair_threads<BSRC, kPush>(), pair_smem_bytes<BSRC, BN>(), stream>>>(a, b0, b1, args);
  return cudaGetLastError();
}

template <int BN>
cudaError_t launch_conv_halo_t(const CUtensorMap& a, const CUtensorMap& b, const GemmArgs& args, int num_sms,
                               cudaStream_t stream) {
  static int max_clusters = 0;
  if (max_clusters == 0) {
    cudaError_t e = cudaFuncSetAttribute(conv_halo_pair_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         halo_smem_bytes<BN>());
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * (num_sms / 2), 1, 1);
    cfg.blockDim = dim3(192, 1, 1);
    cfg.dynamicSmemBytes = halo_smem_bytes<BN>();
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, conv_halo_pair_kernel<BN>, &cfg);
    if (e != cudaSuccess) return e;
    if (n <= 0) return cudaErrorInvalidConfiguration;
    max_clusters = n;
  }
  const int pairs = std::min(args.total_tiles, max_clusters);
  conv_halo_pair_kernel<BN><<<2 * pairs, 192, halo_smem_bytes<BN>(), stream>>>(a, b, args);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_pair(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1, const GemmArgs& args,
                             int bsrc, int num_sms, cudaStream_t stream) {
  if (args.total_tiles <= 0) return cudaSuccess;
  if (args.tile_n != kGemmBN && (bsrc != kBSrcBf16 || args.tile_n != 128)) return cudaErrorInvalidValue;
  if (args.ag_flags && (args.conv.taps || args.ag_n < 2 || args.ag_n > 8 || args.ag_rank < 0 ||
                        args.ag_rank >= args.ag_n || !args.ag_step))
    return cudaErrorInvalidValue;
  if (args.ag_a) {
    if (!args.ag_flags || bsrc != kBSrcBf16 || !args.ag_count || args.ag_rows <= 0 || args.ag_ld <= 0 ||
        args.ag_ld % 8 || (reinterpret_cast<uintptr_t>(args.ag_a) & 15))
      return cudaErrorInvalidValue;
    for (int j = 0; j < args.ag_n; ++j)
      if (j != args.ag_rank && (!args.ag_a_peer[j] || !args.ag_flags_peer[j] ||
                                (reinterpret_cast<uintptr_t>(args.ag_a_peer[j]) & 15)))
        return cudaErrorInvalidValue;
  }
  if (args.k_splits > 1 && (bsrc != kBSrcBf16 || args.ep.mode != kEpiF32 || args.conv.taps ||
                            args.tiles_per_split * args.k_splits != args.total_tiles ||
                            args.k_splits > (args.K + kGemmBK - 1) / kGemmBK))
    return cudaErrorInvalidValue;
  if (args.conv.halo) {
    if (bsrc != kBSrcBf16 || args.conv.taps < 1 || args.conv.taps > 9 || args.conv.tile_w != 128 ||
        args.conv.tile_h != 1)
      return cudaErrorInvalidValue;
    for (int t = 0; t < args.conv.taps; ++t)
      if (args.conv.dy[t] < -1 || args.conv.dy[t] > 1 || args.conv.dx[t] < -1 || args.conv.dx[t] > 1)
        return cudaErrorInvalidValue;
    return args.tile_n == 128 ? launch_conv_halo_t<128>(a, b0, args, num_sms, stream)
                              : launch_conv_halo_t<256>(a, b0, args, num_sms, stream);
  }
  switch (bsrc) {
    case kBSrcBf16:
      if (args.ag_a)
        return args.tile_n == 128 ? launch_gemm_pair_t<kBSrcBf16, 128, true>(a, b0, b1, args, num_sms, stream)
                                  : launch_gemm_pair_t<kBSrcBf16, kGemmBN, true>(a, b0, b1, args, num_sms, stream);
      return args.tile_n == 128 ? launch_gemm_pair_t<kBSrcBf16, 128>(a, b0, b1, args, num_sms, stream)
                                : launch_gemm_pair_t<kBSrcBf16>(a, b0, b1, args, num_sms, stream);
    case kBSrcQ4_K:
    case kBSrcQ8_0: {
      if (args.K % kGemmBK) return cudaErrorInvalidValue;
      for (int i = 0; i < args.n_groups; ++i)
        if (!args.qb[args.groups[i].wsel].packed ||
            (reinterpret_cast<uintptr_t>(args.qb[args.groups[i].wsel].packed) & 15))
          return cudaErrorInvalidValue;
      return bsrc == kBSrcQ4_K ? launch_gemm_pair_t<kBSrcQ4_K>(a, b0, b1, args, num_sms, stream)
                               : launch_gemm_pair_t<kBSrcQ8_0>(a, b0, b1, args, num_sms, stream);
    }
    default: return cudaErrorNotSupported;
  }
}

cudaError_t make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                           uint64_t ld_elems, uint32_t box_outer) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld_elems * 2) & 15)) return cudaErrorMisalignedAddress;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kGemmBK), box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_tmap_conv(CUtensorMap* map, const void* base, int64_t B, int64_t H, int64_t W, int64_t C,
                           int tile_w, int tile_h) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return cudaErrorNotSupported;
  if (reinterpret_cast<uintptr_t>(base) & 15) return cudaErrorMisalignedAddress;
  if (C % 64 != 0 || tile_w < 1 || tile_h < 1 || tile_w > 256 || tile_h > 256 || tile_w * tile_h != kGemmBM)
    return cudaErrorInvalidValue;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(C * 2), static_cast<cuuint64_t>(W * C * 2),
                           static_cast<cuuint64_t>(H * W * C * 2)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(tile_w), static_cast<cuuint32_t>(tile_h), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_tmap_conv_patch(CUtensorMap* map, const void* base, int64_t B, int64_t H, int64_t W, int64_t C) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return cudaErrorNotSupported;
  if (reinterpret_cast<uintptr_t>(base) & 15) return cudaErrorMisalignedAddress;
  if (C % 64 != 0) return cudaErrorInvalidValue;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(C * 2), static_cast<cuuint64_t>(W * C * 2),
                           static_cast<cuuint64_t>(H * W * C * 2)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(kPatchW), static_cast<cuuint32_t>(kPatchH), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

int gemm_choose_k_splits(int64_t tiles, int num_sms, int64_t rows, int64_t N, int64_t K, int max_splits, int min_kb,
                         bool reduce_adds, double min_gain) {
  const int64_t units = std::max(num_sms / 2, 1), nk = (K + kGemmBK - 1) / kGemmBK;
  auto fill = [&](int64_t u) { return static_cast<double>(u) / (static_cast<double>((u + units - 1) / units) * units); };
  const double flops = 2.0 * static_cast<double>(rows) * static_cast<double>(N) * static_cast<double>(K);
  const double out_bytes = static_cast<double>(rows) * static_cast<double>(N) * 4.0;
  auto cost = [&](int sp) {
    const double t = flops / (1.3e15 * fill(tiles * sp));
    return sp == 1 ? t : t + (sp + (reduce_adds ? 2.0 : 1.0)) * out_bytes / 5e12;
  };
  const double base = cost(1);
  double best = base;
  int splits = 1;
  for (int sp = 2; sp <= max_splits; ++sp) {
    if (nk / sp < min_kb) break;
    const double c = cost(sp);
    if (c < best && c < (1.0 - min_gain) * base) {
      best = c;
      splits = sp;
    }
  }
  return splits;
}

void gemm_set_k_splits(GemmArgs& a, int k_splits, int64_t split_stride) {
  a.k_splits = k_splits;
  a.tiles_per_split = a.total_tiles;
  a.total_tiles *= k_splits;
  a.split_stride = split_stride;
}

void gemm_finalize_groups(GemmArgs& a, int tile_m, int tile_n) {
  a.tile_n = tile_n;
  a.n_tiles_n = (a.N + tile_n - 1) / tile_n;
  int mt = 0;
  bool w_used[2] = {false, false};
  for (int g = 0; g < a.n_groups; ++g) {
    a.groups[g].m_tiles = (a.groups[g].rows + tile_m - 1) / tile_m;
    a.groups[g].tile0 = mt;
    mt += a.groups[g].m_tiles;
    w_used[a.groups[g].wsel & 1] = true;
  }
  a.m_tiles_all = mt;
  a.total_tiles = mt * a.n_tiles_n;
  // Tile order: keep one operand's band in L2 and stream the other once per
  // band, picking the order and band width with the fewest modelled DRAM
  // bytes (bf16 operands; a band's resident bytes at most the L2 budget).
  // Convolutions keep M-inner order with one band (their A is an image).
  a.raster = 0;
  a.band = std::max(mt, 1);
  if (a.conv.taps == 0 && mt > 0) {
    double budget = 64.0 * (1 << 20);
    if (const char* f = getenv("DCPP_GEMM_L2_MB")) budget = std::max(1.0, atof(f)) * (1 << 20);
    const double a_row = static_cast<double>(tile_m) * a.K * 2.0;                              // one M tile of A
    const double b_col = static_cast<double>(tile_n) * a.K * 2.0 * (w_used[0] + w_used[1]);  // one N tile of B
    const double a_all = a_row * mt, b_all = b_col * a.n_tiles_n;
    const int bm = std::max(1, std::min(mt, static_cast<int>(budget / a_row)));
    const int bn = std::max(1, std::min(a.n_tiles_n, static_cast<int>(budget / b_col)));
    const double cost_m = a_all + b_all * ((mt + bm - 1) / bm);
    const double cost_n = b_all + a_all * ((a.n_tiles_n + bn - 1) / bn);
    if (cost_n < cost_m) {
      a.raster = 1;
      a.band = bn;
    } else {
      a.band = bm;
    }
    if (const char* f = getenv("DCPP_GEMM_RASTER")) {  // 0 / 1 force the order with one band (measurements)
      a.raster = atoi(f) ? 1 : 0;
      a.band = a.raster ? a.n_tiles_n : mt;
    }
  }
}

cudaError_t launch_gemm(const CUtensorMap& a, const CUtensorMap& b0, const CUtensorMap& b1, const GemmArgs& args,
                        int bsrc, int num_sms, cudaStream_t stream) {
  if (args.total_tiles <= 0) return cudaSuccess;
  if (args.k_splits > 1) return cudaErrorInvalidValue;  // the one-SM kernel has no K split
  if (args.ag_flags || args.ag_a) return cudaErrorInvalidValue;  // nor the overlapped all-gather
  if (args.tile_n != kGemmBN && bsrc != kBSrcBf16) return cudaErrorInvalidValue;
  switch (bsrc) {
    case kBSrcBf16:
      switch (args.tile_n) {
        case 256: return launch_gemm_t<kBSrcBf16>(a, b0, b1, args, num_sms, stream);
        case 128: return launch_gemm_t<kBSrcBf16, 128>(a, b0, b1, args, num_sms, stream);
        case 64: return launch_gemm_t<kBSrcBf16, 64>(a, b0, b1, args, num_sms, stream);
        case 32: return launch_gemm_t<kBSrcBf16, 32>(a, b0, b1, args, num_sms, stream);
        default: return cudaErrorInvalidValue;
      }
    case kBSrcQ4_K:
    case kBSrcQ8_0: {
      if (args.K % kGemmBK) return cudaErrorInvalidValue;
      for (int i = 0; i < args.n_groups; ++i)
        if (!args.qb[args.groups[i].wsel].packed || (reinterpret_cast<uintptr_t>(args.qb[args.groups[i].wsel].packed) & 15))
          return cudaErrorInvalidValue;
      return bsrc == kBSrcQ4_K ? launch_gemm_t<kBSrcQ4_K>(a, b0, b1, args, num_sms, stream)
                               : launch_gemm_t<kBSrcQ8_0>(a, b0, b1, args, num_sms, stream);
    }
    default: return cudaErrorNotSupported;
  }
}

}  // namespace dcpp
