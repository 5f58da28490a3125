// Row-wise and small kernels of the Flux2 step: adaLN LayerNorm +
// modulation, f32 -> bf16 conversion, the RoPE table, sinusoidal timestep
// features and the batch-1 conditioning GEMVs.  All HBM-bound: coalesced
// 16-byte accesses, warp-shuffle reductions.
#include "common.cuh"
#include <algorithm>

#include "kernels.cuh"

#include <math.h>

namespace dcpp {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------ LayerNorm + mod
// One CTA per destination row; each thread keeps up to kVec float4 of the
// row in registers.  Two-pass mean / variance like ggml_norm
// (LayerNorm.cpp:16-32 with elementwise_affine = false), then the adaLN
// modulation (1 + scale) * n + shift (Flux2TransformerBlock.hpp:66,72,92,106;
// Flux2SingleTransformerBlock.hpp:53-54; AdaLayerNormContinuous.inl:43).
template <int kW>
struct PackOut;
template <>
struct PackOut<4> { using T = uint2; };
template <>
struct PackOut<8> { using T = uint4; };

__device__ __forceinline__ void add_bf16x4(float4& t, uint2 u) {
  t.x += __uint_as_float(u.x << 16); t.y += __uint_as_float(u.x & 0xFFFF0000u);
  t.z += __uint_as_float(u.y << 16); t.w += __uint_as_float(u.y & 0xFFFF0000u);
}

// Four bf16 of a slot load: the load itself (4-wide) or its half f (8-wide).
__device__ __forceinline__ uint2 slot_half(uint2 u, int) { return u; }
__device__ __forceinline__ uint2 slot_half(uint4 u, int f) { return f ? make_uint2(u.z, u.w) : make_uint2(u.x, u.y); }

// kW elements (4 or 8) per thread and step: one or two float4 loads of x,
// one 8- or 16-byte bf16 store per output buffer.
template <int kThreads, int kVec, int kW>
__global__ void __launch_bounds__(kThreads) layernorm_mod_kernel(const __grid_constant__ NormArgs a) {
  constexpr int kF4 = kW / 4;
  using OutT = typename PackOut<kW>::T;
  __shared__ float red[kThreads / 32];
  __shared__ float stat;
  int blk = blockIdx.x;
  int sidx = 0;
  int64_t src, dst, slot_row;
  if (a.gran_n > 0) {  // this rank's granules, in order
    const int64_t k = blk / kGranuleRows, off = blk % kGranuleRows;
    src = (k * a.gran_n + a.gran_rank) * kGranuleRows + off;
    slot_row = k * kGranuleRows + off;
#pragma unroll 1
    for (; sidx < a.n_segments; ++sidx)
      if (src >= a.seg[sidx].src_row0 && src < a.seg[sidx].src_row0 + a.seg[sidx].rows) break;
    if (sidx >= a.n_segments) return;
    dst = a.seg[sidx].dst_row0 + (src - a.seg[sidx].src_row0);
  } else {
#pragma unroll 1
    for (; sidx < a.n_segments; ++sidx) {
      if (blk < a.seg[sidx].rows) break;
      blk -= a.seg[sidx].rows;
    }
    if (sidx >= a.n_segments) return;
    src = a.seg[sidx].src_row0 + blk;
    dst = a.seg[sidx].dst_row0 + blk;
    slot_row = src - a.slot_row0;
  }
  const NormSegment& sg = a.seg[sidx];
  const int D = a.D;
  const int ng = D / kW;
  const float4* x4 = reinterpret_cast<const float4*>(a.x + src * a.ld_x);
  const float4* r4 = a.resid ? reinterpret_cast<const float4*>(a.resid + src * a.ld_x) : nullptr;
  const bool slotted = a.n_slots > 0;
  const int64_t srow = slot_row * a.ld_x;
  float4* xo4 = (a.resid || slotted) ? reinterpret_cast<float4*>(a.x_out + src * a.ld_x) : nullptr;

  float4 v[kVec][kF4];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    if (idx < ng) {
      // The slot loads first (over NVLink in the pull form, so they must be
      // in flight together): one kW-element (8- or 16-byte) load per slot.
      OutT pv[8];
      if (slotted) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (k < a.n_slots) {
            const uint16_t* base = a.slot_ptr[0] ? a.slot_ptr[k] : a.slots + k * a.slot_stride;
            pv[k] = reinterpret_cast<const OutT*>(base + srow)[idx];
          }
        }
      }
#pragma unroll
      for (int f = 0; f < kF4; ++f) {
        float4 t = x4[idx * kF4 + f];
        if (r4) {
          const float4 r = r4[idx * kF4 + f];
          t.x += r.x; t.y += r.y; t.z += r.z; t.w += r.w;
        }
        if (slotted) {  // the sums in slot order
#pragma unroll
          for (int k = 0; k < 8; ++k)
            if (k < a.n_slots) add_bf16x4(t, slot_half(pv[k], f));
        }
        if (xo4) xo4[idx * kF4 + f] = t;
        v[i][f] = t;
        sum += (t.x + t.y) + (t.z + t.w);
      }
    } else {
#pragma unroll
      for (int f = 0; f < kF4; ++f) v[i][f] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  sum = warp_sum(sum);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x < 32) {
    float s = threadIdx.x < kThreads / 32 ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) stat = s / static_cast<float>(D);
  }
  __syncthreads();
  const float mean = a.rms ? 0.f : stat;  // RMSNorm: no centring
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    if (idx < ng) {
#pragma unroll
      for (int f = 0; f < kF4; ++f) {
        float4& t = v[i][f];
        t.x -= mean; t.y -= mean; t.z -= mean; t.w -= mean;
        sq += (t.x * t.x + t.y * t.y) + (t.z * t.z + t.w * t.w);
      }
    }
  }
  __syncthreads();
  sq = warp_sum(sq);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x < 32) {
    float s = threadIdx.x < kThreads / 32 ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) stat = 1.0f / sqrtf(s / static_cast<float>(D) + a.eps);
  }
  __syncthreads();
  const float rstd = stat;
  const float4* sh4 = reinterpret_cast<const float4*>(sg.shift);
  const float4* sc4 = reinterpret_cast<const float4*>(sg.scale);
  OutT* yo = reinterpret_cast<OutT*>(a.y + dst * a.ld_y);
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    if (idx < ng) {
      uint32_t pk[2 * kF4];
#pragma unroll
      for (int f = 0; f < kF4; ++f) {
        const float4 t = v[i][f];
        float4 o;
        if (a.rms) {  // Qwen3RMSNorm.cpp:11-19: weight * (x * rsqrt(mean(x^2) + eps))
          const float4 w = a.weight ? __ldg(reinterpret_cast<const float4*>(a.weight) + idx * kF4 + f)
                                    : make_float4(1.f, 1.f, 1.f, 1.f);
          o = make_float4(w.x * (t.x * rstd), w.y * (t.y * rstd), w.z * (t.z * rstd), w.w * (t.w * rstd));
        } else {
          const float4 sh = sh4 ? __ldg(sh4 + idx * kF4 + f) : make_float4(0.f, 0.f, 0.f, 0.f);
          const float4 sc = sc4 ? __ldg(sc4 + idx * kF4 + f) : make_float4(0.f, 0.f, 0.f, 0.f);
          o = make_float4((1.0f + sc.x) * (t.x * rstd) + sh.x, (1.0f + sc.y) * (t.y * rstd) + sh.y,
                          (1.0f + sc.z) * (t.z * rstd) + sh.z, (1.0f + sc.w) * (t.w * rstd) + sh.w);
        }
        if (a.y_f32) reinterpret_cast<float4*>(a.y_f32 + dst * a.ld_y)[idx * kF4 + f] = o;
        pk[2 * f] = pack_bf16x2(o.x, o.y);
        pk[2 * f + 1] = pack_bf16x2(o.z, o.w);
      }
      OutT o;
      if constexpr (kW == 8) o = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      else o = make_uint2(pk[0], pk[1]);
      yo[idx] = o;
      for (int k = 0; k < a.n_peer_out; ++k) reinterpret_cast<OutT*>(a.y_peer[k] + dst * a.ld_y)[idx] = o;
    }
  }
}

// One CTA of up to 32 threads; thread j exchanges arrivals with rank j.
__global__ void tp_barrier_kernel(const __grid_constant__ TpBarrierArgs a) {
  __shared__ uint32_t ep_s;
  if (threadIdx.x == 0) ep_s = *a.epoch + 1u;
  __syncthreads();
  const uint32_t ep = ep_s;
  const int j = threadIdx.x;
  if (j < a.nranks) {
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.flags[j] + a.rank), "r"(ep) : "memory");
    const uint32_t* mine = a.flags[a.rank] + j;
    const unsigned long long limit = a.timeout_ns ? a.timeout_ns : kWaitTimeoutNs;
    const unsigned long long t0 = globaltimer();
    while (true) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if (static_cast<int32_t>(v - ep) >= 0) break;
      if (globaltimer() - t0 > limit) {
        atomicCAS(a.err, 0, kDevTimeoutPeer);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *a.epoch = ep;
}

__global__ void f32_to_bf16_kernel(const float4* __restrict__ in, int64_t n4, uint2* __restrict__ out) {
  int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (; i < n4; i += stride) {
    const float4 v = in[i];
    out[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

__global__ void f32_to_bf16_tail_kernel(const float* __restrict__ in, int64_t start, int64_t n, uint16_t* out) {
  int64_t i = start + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n) {
    __nv_bfloat16 b = __float2bfloat16_rn(in[i]);
    out[i] = *reinterpret_cast<uint16_t*>(&b);
  }
}

struct AxesDims {
  int n;
  int dims[8];
};

// ggml rope NORMAL cache (ggml_rope_cache_init with freq_scale 1,
// ext_factor 0, attn_factor 1): theta starts at the position and is
// multiplied by theta_scale = base^(-2/n_dims) once per rotary pair.
__global__ void rope_table_kernel(const int32_t* __restrict__ ids, int64_t S, AxesDims ax, float base,
                                  float2* __restrict__ table) {
  int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (s >= S) return;
  int pair = 0;
#pragma unroll 1
  for (int a = 0; a < ax.n; ++a) {
    const int nd = ax.dims[a];
    const float theta_scale = powf(base, -2.0f / static_cast<float>(nd));
    float theta = static_cast<float>(ids[s * ax.n + a]);
#pragma unroll 1
    for (int p = 0; p < nd / 2; ++p) {
      float sn, cs;
      sincosf(theta, &sn, &cs);
      table[s * 64 + pair] = make_float2(cs, sn);
      ++pair;
      theta *= theta_scale;
    }
  }
}

__global__ void timestep_proj_kernel(const float* __restrict__ t, int channels, float mult, float* __restrict__ out) {
  const int b = blockIdx.x;
  const int half = channels / 2;
  const float c = -logf(10000.0f) / static_cast<float>(half);
  const float tb = t[b] * mult;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float f = expf(static_cast<float>(i) * c);
    const float arg = tb * f;
    out[b * channels + i] = cosf(arg);
    out[b * channels + half + i] = sinf(arg);
  }
  if ((channels & 1) && threadIdx.x == 0) out[b * channels + channels - 1] = 0.f;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// Batch-1..4 GEMV y[b] = W x[b] for the conditioning path (timestep /
// guidance embedders, the three modulation projections, norm_out), reading
// the raw GGUF rows.  One warp per row, kGemvRowsPerWarp rows per warp so a
// CTA's fill of x into shared memory (with the optional SiLU of the input)
// serves 32 rows.  Lanes walk a row so that each quarter-warp reads 128
// contiguous bytes of x (conflict-free float4 shared loads) and the warp
// reads contiguous weight bytes:
//   Q4_K: lane L = 8m + t takes nibble bytes [4t, 4t+4) of 32-byte group m of
//         each 256-weight block: weights 4t..4t+3 of sub-blocks 2m (low
//         nibbles) and 2m+1 (high nibbles);
//   Q8_0: 8 lanes per 32-weight block, 4 weights each, 4 blocks per step;
//   BF16 / F16: 8 consecutive weights per lane (one 16-byte load).
// Weights are dequantised exactly as dequant.cu does (d*sc*q - dmin*m with
// separate roundings), then accumulated with FMAs in f32.
constexpr int kGemvRowsPerWarp = 4;
constexpr int kGemvRowsPerCta = 8 * kGemvRowsPerWarp;

__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t* s, int& sc, int& m) {
  if (j < 4) {
    sc = s[j] & 0x3F;
    m = s[j + 4] & 0x3F;
  } else {
    sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 2) & 0x30);
    m = (s[j + 4] >> 4) | ((s[j] >> 2) & 0x30);
  }
}

template <int kType>
__global__ void __launch_bounds__(256) gemv_kernel(const uint8_t* __restrict__ W, int64_t N, int64_t K,
                                                   const float* __restrict__ x, int B, int act_in, int act_out,
                                                   float* __restrict__ y) {
  extern __shared__ float4 xs4[];  // [B, K]
  float* xs = reinterpret_cast<float*>(xs4);
  for (int64_t i = threadIdx.x; i < static_cast<int64_t>(B) * K; i += blockDim.x) {
    float v = x[i];
    xs[i] = act_in ? silu_f(v) : v;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t row0 = (static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5)) * kGemvRowsPerWarp;
#pragma unroll 1
  for (int rr = 0; rr < kGemvRowsPerWarp; ++rr) {
    const int64_t n = row0 + rr;
    if (n >= N) break;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (kType == kTypeQ4_K) {
      const int m = lane >> 3, t = lane & 7;
      const int64_t nblk = K / 256;
      const uint8_t* row = W + n * nblk * 144;
#pragma unroll 4
      for (int64_t bk = 0; bk < nblk; ++bk) {
        const uint8_t* bp = row + bk * 144;
        const uint32_t dd = __ldg(reinterpret_cast<const uint32_t*>(bp));
        const uint32_t q = __ldg(reinterpret_cast<const uint32_t*>(bp + 16 + m * 32 + 4 * t));
        const float d = __half2float(__ushort_as_half(static_cast<uint16_t>(dd & 0xFFFF)));
        const float dmin = __half2float(__ushort_as_half(static_cast<uint16_t>(dd >> 16)));
        int sc0, m0, sc1, m1;
        q4k_scale_min(2 * m, bp + 4, sc0, m0);
        q4k_scale_min(2 * m + 1, bp + 4, sc1, m1);
        const float ds0 = __fmul_rn(d, static_cast<float>(sc0)), dm0 = __fmul_rn(dmin, static_cast<float>(m0));
        const float ds1 = __fmul_rn(d, static_cast<float>(sc1)), dm1 = __fmul_rn(dmin, static_cast<float>(m1));
        float w0[4], w1[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          w0[i] = __fsub_rn(__fmul_rn(ds0, static_cast<float>((q >> (8 * i)) & 0xF)), dm0);
          w1[i] = __fsub_rn(__fmul_rn(ds1, static_cast<float>((q >> (8 * i + 4)) & 0xF)), dm1);
        }
        for (int b = 0; b < B; ++b) {
          const float* xb = xs + b * K + bk * 256 + 4 * t;
          const float4 x0 = *reinterpret_cast<const float4*>(xb + (2 * m) * 32);
          const float4 x1 = *reinterpret_cast<const float4*>(xb + (2 * m + 1) * 32);
          float a = acc[b];
          a = fmaf(w0[0], x0.x, a); a = fmaf(w0[1], x0.y, a); a = fmaf(w0[2], x0.z, a); a = fmaf(w0[3], x0.w, a);
          a = fmaf(w1[0], x1.x, a); a = fmaf(w1[1], x1.y, a); a = fmaf(w1[2], x1.z, a); a = fmaf(w1[3], x1.w, a);
          acc[b] = a;
        }
      }
    } else if (kType == kTypeQ8_0) {
      const int t = lane & 7;
      const int64_t nblk = K / 32;
      const uint8_t* row = W + n * nblk * 34;
#pragma unroll 2
      for (int64_t bk = lane >> 3; bk < nblk; bk += 4) {
        const uint16_t* bp = reinterpret_cast<const uint16_t*>(row + bk * 34);
        const float d = __half2float(__ushort_as_half(__ldg(bp)));
        const uint32_t lo = __ldg(bp + 1 + 2 * t), hi = __ldg(bp + 2 + 2 * t);
        const uint32_t q = lo | (hi << 16);
        float w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = __fmul_rn(d, static_cast<float>(static_cast<int8_t>((q >> (8 * i)) & 0xFF)));
        for (int b = 0; b < B; ++b) {
          const float4 xv = *reinterpret_cast<const float4*>(xs + b * K + bk * 32 + 4 * t);
          float a = acc[b];
          a = fmaf(w[0], xv.x, a); a = fmaf(w[1], xv.y, a); a = fmaf(w[2], xv.z, a); a = fmaf(w[3], xv.w, a);
          acc[b] = a;
        }
      }
    } else if (kType == kTypeBF16 || kType == kTypeF16) {
      const uint16_t* row = reinterpret_cast<const uint16_t*>(W) + n * K;
#pragma unroll 2
      for (int64_t c = lane; c < K / 8; c += 32) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(row) + c);
        const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
        float wf[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (kType == kTypeBF16) {
            wf[2 * i] = __uint_as_float(wv[i] << 16);
            wf[2 * i + 1] = __uint_as_float(wv[i] & 0xFFFF0000u);
          } else {
            wf[2 * i] = __half2float(__ushort_as_half(static_cast<uint16_t>(wv[i] & 0xFFFF)));
            wf[2 * i + 1] = __half2float(__ushort_as_half(static_cast<uint16_t>(wv[i] >> 16)));
          }
        }
        for (int b = 0; b < B; ++b) {
          const float4 xa = *reinterpret_cast<const float4*>(xs + b * K + c * 8);
          const float4 xb = *reinterpret_cast<const float4*>(xs + b * K + c * 8 + 4);
          float a = acc[b];
          a = fmaf(wf[0], xa.x, a); a = fmaf(wf[1], xa.y, a); a = fmaf(wf[2], xa.z, a); a = fmaf(wf[3], xa.w, a);
          a = fmaf(wf[4], xb.x, a); a = fmaf(wf[5], xb.y, a); a = fmaf(wf[6], xb.z, a); a = fmaf(wf[7], xb.w, a);
          acc[b] = a;
        }
      }
    } else {  // F32
      const float* row = reinterpret_cast<const float*>(W) + n * K;
      for (int64_t c = lane; c < K; c += 32)
        for (int b = 0; b < B; ++b) acc[b] = fmaf(row[c], xs[b * K + c], acc[b]);
    }
    for (int b = 0; b < B; ++b) {
      float v = warp_sum(acc[b]);
      if (lane == 0) y[b * N + n] = act_out ? silu_f(v) : v;
    }
  }
}

// GEMV for K % 256 == 0: one thread per 256-weight unit of a row (a Q4_K
// super-block, eight Q8_0 blocks or 256 bf16 / f16 weights), read with
// independent 16-byte loads (9 / 17 / 32 per unit), so a warp keeps 4.5-16 KB
// of weights in flight.  A CTA covers whole rows (kGemvUnitsPerCta / U rows);
// each thread's partial dot products go to shared memory and one thread per
// row adds its U partials in order (deterministic, no atomics).  x sits in
// shared memory with 4 floats of padding per 256, so the 8 lanes of a
// quarter-warp reading the same offset of 8 consecutive units hit distinct
// banks.
constexpr int kGemvUnitsPerCta = 256;
constexpr int kGemvUnitStride = 260;  // floats per 256-weight unit of x in smem

template <int kType>
__global__ void __launch_bounds__(256) gemv_unit_kernel(const uint8_t* __restrict__ W, int64_t N, int64_t K,
                                                        const float* __restrict__ x, int B, int act_in, int act_out,
                                                        float* __restrict__ y) {
  extern __shared__ float4 sm4[];
  float* xs = reinterpret_cast<float*>(sm4);            // [B][U * 260]
  const int U = static_cast<int>(K >> 8);
  float* part = xs + static_cast<int64_t>(B) * U * kGemvUnitStride;  // [256][B]
  for (int64_t i = threadIdx.x; i < static_cast<int64_t>(B) * K; i += blockDim.x) {
    const int b = static_cast<int>(i / K);
    const int k = static_cast<int>(i - static_cast<int64_t>(b) * K);
    const float v = x[i];
    xs[static_cast<int64_t>(b) * U * kGemvUnitStride + (k >> 8) * kGemvUnitStride + (k & 255)] = act_in ? silu_f(v) : v;
  }
  __syncthreads();
  const int rows_per_cta = kGemvUnitsPerCta / U;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * rows_per_cta;
  const int t = threadIdx.x;
  const int r_local = t / U;
  const int u = t - r_local * U;
  const int64_t row = row0 + r_local;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (r_local < rows_per_cta && row < N) {
    const float* xu = xs + u * kGemvUnitStride;
    const int64_t xb = static_cast<int64_t>(U) * kGemvUnitStride;
    if (kType == kTypeQ4_K) {
      const uint4* p = reinterpret_cast<const uint4*>(W + (row * U + u) * 144);
      uint4 w[9];
#pragma unroll
      for (int i = 0; i < 9; ++i) w[i] = __ldg(p + i);
      const float d = __half2float(__ushort_as_half(static_cast<uint16_t>(w[0].x & 0xFFFF)));
      const float dmin = __half2float(__ushort_as_half(static_cast<uint16_t>(w[0].x >> 16)));
      uint8_t sb[12];
      const uint32_t hw[3] = {w[0].y, w[0].z, w[0].w};
#pragma unroll
      for (int i = 0; i < 12; ++i) sb[i] = static_cast<uint8_t>(hw[i >> 2] >> (8 * (i & 3)));
#pragma unroll
      for (int g = 0; g < 4; ++g) {  // 32-byte nibble group g: sub-blocks 2g (low), 2g+1 (high)
        int sc0, m0, sc1, m1;
        q4k_scale_min(2 * g, sb, sc0, m0);
        q4k_scale_min(2 * g + 1, sb, sc1, m1);
        const float ds0 = __fmul_rn(d, static_cast<float>(sc0)), dm0 = __fmul_rn(dmin, static_cast<float>(m0));
        const float ds1 = __fmul_rn(d, static_cast<float>(sc1)), dm1 = __fmul_rn(dmin, static_cast<float>(m1));
        const uint32_t q[8] = {w[1 + 2 * g].x, w[1 + 2 * g].y, w[1 + 2 * g].z, w[1 + 2 * g].w,
                               w[2 + 2 * g].x, w[2 + 2 * g].y, w[2 + 2 * g].z, w[2 + 2 * g].w};
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float lo[4], hi[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            lo[i] = __fsub_rn(__fmul_rn(ds0, static_cast<float>((q[c] >> (8 * i)) & 0xF)), dm0);
            hi[i] = __fsub_rn(__fmul_rn(ds1, static_cast<float>((q[c] >> (8 * i + 4)) & 0xF)), dm1);
          }
          #pragma unroll
          for (int b = 0; b < 4; ++b) {
            if (b >= B) break;
            const float4 x0 = *reinterpret_cast<const float4*>(xu + b * xb + (2 * g) * 32 + 4 * c);
            const float4 x1 = *reinterpret_cast<const float4*>(xu + b * xb + (2 * g + 1) * 32 + 4 * c);
            float a = acc[b];
            a = fmaf(lo[0], x0.x, a); a = fmaf(lo[1], x0.y, a); a = fmaf(lo[2], x0.z, a); a = fmaf(lo[3], x0.w, a);
            a = fmaf(hi[0], x1.x, a); a = fmaf(hi[1], x1.y, a); a = fmaf(hi[2], x1.z, a); a = fmaf(hi[3], x1.w, a);
            acc[b] = a;
          }
        }
      }
    } else if (kType == kTypeQ8_0) {
      // Eight 34-byte blocks = 272 bytes = 17 aligned uint4 (rows are K/32*34
      // bytes, a multiple of 272 since K % 256 == 0).
      const uint4* p = reinterpret_cast<const uint4*>(W + (row * U + u) * 272);
      uint32_t w[68];
#pragma unroll
      for (int i = 0; i < 17; ++i) {
        const uint4 v = __ldg(p + i);
        w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
      }
      auto byte_at = [&](int off) -> uint32_t { return (w[off >> 2] >> (8 * (off & 3))) & 0xFF; };
#pragma unroll
      for (int blk = 0; blk < 8; ++blk) {
        const int o = blk * 34;
        const float d = __half2float(__ushort_as_half(static_cast<uint16_t>(byte_at(o) | (byte_at(o + 1) << 8))));
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float wv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            wv[i] = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(byte_at(o + 2 + 4 * c + i))));
          #pragma unroll
          for (int b = 0; b < 4; ++b) {
            if (b >= B) break;
            const float4 xv = *reinterpret_cast<const float4*>(xu + b * xb + blk * 32 + 4 * c);
            float a = acc[b];
            a = fmaf(wv[0], xv.x, a); a = fmaf(wv[1], xv.y, a); a = fmaf(wv[2], xv.z, a); a = fmaf(wv[3], xv.w, a);
            acc[b] = a;
          }
        }
      }
    } else {  // BF16 / F16: 256 weights = 32 uint4, in 4 batches of 8
      const uint4* p = reinterpret_cast<const uint4*>(W + (row * U + u) * 512);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        uint4 w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = __ldg(p + 8 * h + i);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t wv[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
          float wf[8];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (kType == kTypeBF16) {
              wf[2 * k] = __uint_as_float(wv[k] << 16);
              wf[2 * k + 1] = __uint_as_float(wv[k] & 0xFFFF0000u);
            } else {
              wf[2 * k] = __half2float(__ushort_as_half(static_cast<uint16_t>(wv[k] & 0xFFFF)));
              wf[2 * k + 1] = __half2float(__ushort_as_half(static_cast<uint16_t>(wv[k] >> 16)));
            }
          }
          const int e = (8 * h + i) * 8;
          #pragma unroll
          for (int b = 0; b < 4; ++b) {
            if (b >= B) break;
            const float4 xa = *reinterpret_cast<const float4*>(xu + b * xb + e);
            const float4 xc = *reinterpret_cast<const float4*>(xu + b * xb + e + 4);
            float a = acc[b];
            a = fmaf(wf[0], xa.x, a); a = fmaf(wf[1], xa.y, a); a = fmaf(wf[2], xa.z, a); a = fmaf(wf[3], xa.w, a);
            a = fmaf(wf[4], xc.x, a); a = fmaf(wf[5], xc.y, a); a = fmaf(wf[6], xc.z, a); a = fmaf(wf[7], xc.w, a);
            acc[b] = a;
          }
        }
      }
    }
  }
#pragma unroll
  for (int b = 0; b < 4; ++b) part[t * 4 + b] = acc[b];
  __syncthreads();
  if (t < rows_per_cta && row0 + t < N) {
    #pragma unroll
          for (int b = 0; b < 4; ++b) {
            if (b >= B) break;
      float v = 0.f;
      for (int i = 0; i < U; ++i) v += part[(t * U + i) * 4 + b];
      y[b * N + row0 + t] = act_out ? silu_f(v) : v;
    }
  }
}

// Embedding row gather with dequantisation (ggml_get_rows on Q8_0 / Q4_K /
// F16 / BF16 / F32 tables; Embedding::forward).  One CTA per id.
__global__ void __launch_bounds__(256) get_rows_kernel(int type, const uint8_t* __restrict__ table, int64_t n_rows,
                                                       int64_t dim, const int32_t* __restrict__ ids,
                                                       float* __restrict__ out, int* err) {
  const int64_t i = blockIdx.x;
  const int32_t id = ids[i];
  float* o = out + i * dim;
  if (id < 0 || id >= n_rows) {
    for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) o[c] = 0.f;
    if (threadIdx.x == 0 && err) atomicCAS(err, 0, kDevBadIndex);
    return;
  }
  if (type == kTypeQ8_0) {
    const uint8_t* row = table + static_cast<int64_t>(id) * (dim / 32) * 34;
    for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) {
      const uint8_t* blk = row + (c / 32) * 34;
      const float d = __half2float(__ushort_as_half(static_cast<uint16_t>(blk[0] | (blk[1] << 8))));
      o[c] = __fmul_rn(static_cast<float>(static_cast<int8_t>(blk[2 + (c & 31)])), d);
    }
  } else if (type == kTypeQ4_K) {
    const uint8_t* row = table + static_cast<int64_t>(id) * (dim / 256) * 144;
    for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) {
      const uint8_t* blk = row + (c / 256) * 144;
      const int e = static_cast<int>(c & 255), j = e / 32, l = e & 31;
      const float d = __half2float(__ushort_as_half(static_cast<uint16_t>(blk[0] | (blk[1] << 8))));
      const float dmin = __half2float(__ushort_as_half(static_cast<uint16_t>(blk[2] | (blk[3] << 8))));
      int sc, m;
      q4k_scale_min(j, blk + 4, sc, m);
      const float q = static_cast<float>((blk[16 + (j >> 1) * 32 + l] >> ((j & 1) * 4)) & 0xF);
      o[c] = __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), q), __fmul_rn(dmin, static_cast<float>(m)));
    }
  } else if (type == kTypeF32) {
    const float* row = reinterpret_cast<const float*>(table) + static_cast<int64_t>(id) * dim;
    for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) o[c] = row[c];
  } else {
    const uint16_t* row = reinterpret_cast<const uint16_t*>(table) + static_cast<int64_t>(id) * dim;
    for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) {
      const uint16_t h = row[c];
      o[c] = type == kTypeBF16 ? __uint_as_float(static_cast<uint32_t>(h) << 16) : __half2float(__ushort_as_half(h));
    }
  }
}

__global__ void mask_bits_kernel(const float* __restrict__ mask, int64_t S, int64_t words, uint32_t* __restrict__ bits) {
  const int64_t b = blockIdx.y;
  const int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (w >= words) return;
  uint32_t v = 0;
  for (int i = 0; i < 32; ++i) {
    const int64_t k = w * 32 + i;
    if (k < S && mask[b * S + k] != 0.f) v |= 1u << i;
  }
  bits[b * words + w] = v;
}

__global__ void step_counter_kernel(uint32_t* step) { *step += 1u; }

__global__ void add_f32_kernel(float* __restrict__ y, const float* __restrict__ a, int64_t n) {
  int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (; i < n; i += stride) y[i] += a[i];
}

}  // namespace

cudaError_t launch_layernorm_mod(const NormArgs& a, cudaStream_t s) {
  if (a.D % 4 != 0 || a.D > 8192 || (a.ld_x % 4) || (a.ld_y % 4)) return cudaErrorInvalidValue;
  if (a.n_slots < 0 || a.n_slots > 8 || (a.slot_stride % 8) || a.n_peer_out < 0 || a.n_peer_out > 7)
    return cudaErrorInvalidValue;
  if (a.n_slots > 0 && !a.slot_ptr[0] && (!a.slots || (reinterpret_cast<uintptr_t>(a.slots) & 15)))
    return cudaErrorInvalidValue;
  if (a.n_slots > 0 && a.slot_ptr[0])
    for (int k = 0; k < a.n_slots; ++k)
      if (!a.slot_ptr[k] || (reinterpret_cast<uintptr_t>(a.slot_ptr[k]) & 15)) return cudaErrorInvalidValue;
  int64_t rows = 0;
  for (int i = 0; i < a.n_segments; ++i) rows += a.seg[i].rows;
  if (rows == 0) return cudaSuccess;
  if (a.gran_n > 0) {  // blocks over this rank's granules of the rows the segments cover
    if (a.gran_rank < 0 || a.gran_rank >= a.gran_n) return cudaErrorInvalidValue;
    int64_t end = 0;
    for (int i = 0; i < a.n_segments; ++i) end = std::max<int64_t>(end, a.seg[i].src_row0 + a.seg[i].rows);
    const int64_t ngr = (end + kGranuleRows - 1) / kGranuleRows;
    const int64_t own = ngr > a.gran_rank ? (ngr - a.gran_rank + a.gran_n - 1) / a.gran_n : 0;
    rows = own * kGranuleRows;
    if (rows == 0) return cudaSuccess;
  }
  const bool w8 = a.D % 8 == 0 && a.ld_y % 8 == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0;
  for (int k = 0; k < a.n_peer_out; ++k)
    if (reinterpret_cast<uintptr_t>(a.y_peer[k]) & (w8 ? 15 : 7)) return cudaErrorInvalidValue;
  const unsigned grid = static_cast<unsigned>(rows);
  if (w8) {
    if (a.D <= 128 * 8 * 4)
      layernorm_mod_kernel<128, 4, 8><<<grid, 128, 0, s>>>(a);
    else
      layernorm_mod_kernel<256, 4, 8><<<grid, 256, 0, s>>>(a);
  } else {
    if (a.D <= 128 * 4 * 8)
      layernorm_mod_kernel<128, 8, 4><<<grid, 128, 0, s>>>(a);
    else
      layernorm_mod_kernel<256, 8, 4><<<grid, 256, 0, s>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launch_step_counter(uint32_t* step, cudaStream_t s) {
  step_counter_kernel<<<1, 1, 0, s>>>(step);
  return cudaGetLastError();
}

cudaError_t launch_get_rows(int type, const void* table, int64_t n_rows, int64_t dim, const int32_t* ids,
                            int64_t n_ids, float* out, int* err, cudaStream_t s) {
  if (n_ids <= 0) return cudaSuccess;
  if (!table || !ids || !out || n_rows <= 0 || dim <= 0) return cudaErrorInvalidValue;
  if ((type == kTypeQ8_0 && dim % 32) || (type == kTypeQ4_K && dim % 256)) return cudaErrorInvalidValue;
  if (type != kTypeQ8_0 && type != kTypeQ4_K && type != kTypeF32 && type != kTypeF16 && type != kTypeBF16)
    return cudaErrorNotSupported;
  get_rows_kernel<<<static_cast<unsigned>(n_ids), 256, 0, s>>>(type, static_cast<const uint8_t*>(table), n_rows, dim,
                                                                ids, out, err);
  return cudaGetLastError();
}

cudaError_t launch_mask_bits(const float* mask, int64_t B, int64_t S, int64_t words, uint32_t* bits, cudaStream_t s) {
  if (B <= 0 || S <= 0) return cudaSuccess;
  if (!mask || !bits || words * 32 < S) return cudaErrorInvalidValue;
  dim3 grid(static_cast<unsigned>((words + 127) / 128), static_cast<unsigned>(B));
  mask_bits_kernel<<<grid, 128, 0, s>>>(mask, S, words, bits);
  return cudaGetLastError();
}

cudaError_t launch_tp_barrier(const TpBarrierArgs& a, cudaStream_t s) {
  if (a.nranks < 1 || a.nranks > 8 || a.rank < 0 || a.rank >= a.nranks || !a.epoch || !a.err)
    return cudaErrorInvalidValue;
  for (int j = 0; j < a.nranks; ++j)
    if (!a.flags[j]) return cudaErrorInvalidValue;
  tp_barrier_kernel<<<1, 32, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_f32_to_bf16(const float* in, int64_t n, uint16_t* out, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const int64_t n4 = ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) ? 0 : n / 4;
  if (n4) {
    int64_t blocks = (n4 + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    f32_to_bf16_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(reinterpret_cast<const float4*>(in), n4,
                                                                       reinterpret_cast<uint2*>(out));
  }
  const int64_t rest = n - n4 * 4;
  if (rest) f32_to_bf16_tail_kernel<<<static_cast<unsigned>((rest + 255) / 256), 256, 0, s>>>(in, n4 * 4, n, out);
  return cudaGetLastError();
}

cudaError_t launch_rope_table(const int32_t* ids, int64_t S, int n_axes, const int32_t* axes_dims, float theta,
                              float2* table, cudaStream_t s) {
  AxesDims ax;
  if (n_axes < 1 || n_axes > 8) return cudaErrorInvalidValue;
  ax.n = n_axes;
  int total = 0;
  for (int i = 0; i < n_axes; ++i) {
    ax.dims[i] = axes_dims[i];
    if (axes_dims[i] <= 0 || (axes_dims[i] & 1)) return cudaErrorInvalidValue;
    total += axes_dims[i];
  }
  if (total != 128) return cudaErrorInvalidValue;
  if (S <= 0) return cudaSuccess;
  rope_table_kernel<<<static_cast<unsigned>((S + 127) / 128), 128, 0, s>>>(ids, S, ax, theta, table);
  return cudaGetLastError();
}

cudaError_t launch_timestep_proj(const float* t, int B, int channels, float mult, float* out, cudaStream_t s) {
  if (B <= 0) return cudaSuccess;
  timestep_proj_kernel<<<B, 128, 0, s>>>(t, channels, mult, out);
  return cudaGetLastError();
}

cudaError_t launch_gemv(int wtype, const void* W, int64_t N, int64_t K, const float* x, int B, int act_in,
                        int act_out, float* y, cudaStream_t s) {
  if (B < 1 || B > 4) return cudaErrorInvalidValue;
  const uint8_t* wb = static_cast<const uint8_t*>(W);
  if (K % 256 == 0 && K / 256 <= kGemvUnitsPerCta && (reinterpret_cast<uintptr_t>(W) & 15) == 0 &&
      (wtype == kTypeQ4_K || wtype == kTypeQ8_0 || wtype == kTypeBF16 || wtype == kTypeF16)) {
    const int U = static_cast<int>(K / 256);
    const size_t usmem = (static_cast<size_t>(B) * U * kGemvUnitStride + kGemvUnitsPerCta * 4) * sizeof(float);
    if (usmem <= 200 * 1024) {
      const int rows_per_cta = kGemvUnitsPerCta / U;
      const unsigned ugrid = static_cast<unsigned>((N + rows_per_cta - 1) / rows_per_cta);
#define DCPP_GEMV_U(T)                                                                                   \
  do {                                                                                                   \
    static bool attr = false;                                                                            \
    if (!attr) {                                                                                         \
      cudaFuncSetAttribute(gemv_unit_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); \
      attr = true;                                                                                       \
    }                                                                                                    \
    gemv_unit_kernel<T><<<ugrid, 256, usmem, s>>>(wb, N, K, x, B, act_in, act_out, y);                   \
  } while (0)
      switch (wtype) {
        case kTypeQ4_K: DCPP_GEMV_U(kTypeQ4_K); break;
        case kTypeQ8_0: DCPP_GEMV_U(kTypeQ8_0); break;
        case kTypeBF16: DCPP_GEMV_U(kTypeBF16); break;
        default: DCPP_GEMV_U(kTypeF16); break;
      }
#undef DCPP_GEMV_U
      return cudaGetLastError();
    }
  }
  const size_t smem = static_cast<size_t>(B) * K * sizeof(float);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  const unsigned grid = static_cast<unsigned>((N + kGemvRowsPerCta - 1) / kGemvRowsPerCta);
  const uint8_t* w = static_cast<const uint8_t*>(W);
#define DCPP_GEMV(T)                                                                                   \
  do {                                                                                                 \
    static bool attr = false;                                                                          \
    if (!attr) {                                                                                       \
      cudaFuncSetAttribute(gemv_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);   \
      attr = true;                                                                                     \
    }                                                                                                  \
    gemv_kernel<T><<<grid, 256, smem, s>>>(w, N, K, x, B, act_in, act_out, y);                         \
  } while (0)
  switch (wtype) {
    case kTypeQ4_K: if (K % 256) return cudaErrorInvalidValue; DCPP_GEMV(kTypeQ4_K); break;
    case kTypeQ8_0: if (K % 32) return cudaErrorInvalidValue; DCPP_GEMV(kTypeQ8_0); break;
    case kTypeBF16: if (K % 8) return cudaErrorInvalidValue; DCPP_GEMV(kTypeBF16); break;
    case kTypeF16: if (K % 8) return cudaErrorInvalidValue; DCPP_GEMV(kTypeF16); break;
    case kTypeF32: DCPP_GEMV(kTypeF32); break;
    default: return cudaErrorNotSupported;
  }
#undef DCPP_GEMV
  return cudaGetLastError();
}

cudaError_t launch_add_f32(float* y, const float* a, int64_t n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  add_f32_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(y, a, n);
  return cudaGetLastError();
}

namespace {
// out[r, c] += sum over s (in order) of ws[s * stride + r * ld_ws + c].
__global__ void split_reduce_kernel(const float* __restrict__ ws, int S, int64_t stride, int64_t rows, int64_t n4,
                                    int64_t ld_ws, float* __restrict__ out, int64_t ld_out, bool add) {
  const int64_t total = rows * n4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / n4, c = (i - r * n4) * 4;
    float4 acc = __ldg(reinterpret_cast<const float4*>(ws + r * ld_ws + c));
    for (int k = 1; k < S; ++k) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(ws + k * stride + r * ld_ws + c));
      acc.x += t.x; acc.y += t.y; acc.z += t.z; acc.w += t.w;
    }
    float4* o = reinterpret_cast<float4*>(out + r * ld_out + c);
    if (add) {
      const float4 h = *o;
      acc.x += h.x; acc.y += h.y; acc.z += h.z; acc.w += h.w;
    }
    *o = acc;
  }
}
}  // namespace

cudaError_t launch_split_reduce(const float* ws, int S, int64_t stride, int64_t rows, int64_t N, int64_t ld_ws,
                                float* out, int64_t ld_out, cudaStream_t s, bool add) {
  if (N % 4 || ld_ws % 4 || ld_out % 4 || stride % 4 || S < 1) return cudaErrorInvalidValue;
  const int64_t total = rows * (N / 4);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 8);
  split_reduce_kernel<<<static_cast<unsigned>(std::max<int64_t>(blocks, 1)), 256, 0, s>>>(ws, S, stride, rows, N / 4,
                                                                                          ld_ws, out, ld_out, add);
  return cudaGetLastError();
}

}  // namespace dcpp
