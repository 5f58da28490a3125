// Row / pixel kernels of the Flux2 VAE decode (the convolutions themselves
// are implicit GEMMs on the tcgen05 GEMM, gemm.cu):
//   latent unpack + BatchNorm de-normalisation + unpatchify
//       (Flux2KleinPipeline.cpp:538-556, :606-630)
//   GroupNorm statistics and GroupNorm (+ SiLU) application
//       (GroupNorm.cpp: ggml_norm over (C/G) x H x W per group, eps 1e-6, affine)
//   row softmax of the mid-block attention scores (SoftmaxAttentionOp.cpp)
//   bf16 transpose
// Images are NHWC: pixel (b, y, x) is row (b H + y) W + x, channels contiguous.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace dcpp {

namespace {

__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  __nv_bfloat16 b = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&b);
}

// ----------------------------------------------------------------- latents
__global__ void latent_unpack_kernel(const float* __restrict__ lat, const float* __restrict__ mean,
                                     const float* __restrict__ var, float eps, int B, int ph, int pw, int C,
                                     int Cpad, uint16_t* __restrict__ out) {
  const int64_t total = static_cast<int64_t>(B) * 4 * ph * pw * Cpad;
  const int W = 2 * pw, H = 2 * ph;
  for (int64_t o = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; o < total;
       o += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(o % Cpad);
    const int64_t pix = o / Cpad;
    const int X = static_cast<int>(pix % W);
    const int64_t t = pix / W;
    const int Y = static_cast<int>(t % H);
    const int b = static_cast<int>(t / H);
    float v = 0.f;
    if (c < C) {
      const int ch = 4 * c + 2 * (Y & 1) + (X & 1);
      const int64_t tok = static_cast<int64_t>(b) * ph * pw + (Y >> 1) * pw + (X >> 1);
      v = lat[tok * 4 * C + ch] * sqrtf(var[ch] + eps) + mean[ch];
    }
    out[o] = f32_to_bf16(v);
  }
}

// --------------------------------------------------------------- GroupNorm
// Per (batch, group) sum and sum of squares in double.  Block (x, b) covers
// rows [x * rows_per_block, ...) of image b; thread t owns channel quad
// t % (C/4) and every (blockDim / (C/4))-th row.
template <typename T>
__device__ __forceinline__ void load4(const T* p, float v[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float v[4]) {
  const float4 t = __ldg(reinterpret_cast<const float4*>(p));
  v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
template <>
__device__ __forceinline__ void load4<uint16_t>(const uint16_t* p, float v[4]) {
  const uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
  v[0] = __uint_as_float(t.x << 16); v[1] = __uint_as_float(t.x & 0xFFFF0000u);
  v[2] = __uint_as_float(t.y << 16); v[3] = __uint_as_float(t.y & 0xFFFF0000u);
}

template <typename T>
__global__ void __launch_bounds__(256) gn_stats_kernel(const T* __restrict__ x, int64_t HW, int C, int G,
                                                        int64_t rows_per_block, double* __restrict__ stats) {
  extern __shared__ double sh[];  // [2 G]
  const int b = blockIdx.y;
  for (int i = threadIdx.x; i < 2 * G; i += blockDim.x) sh[i] = 0.0;
  __syncthreads();
  const int cq = C / 4;
  const int q = threadIdx.x % cq;
  const int r0 = threadIdx.x / cq;
  const int rstep = blockDim.x / cq;
  if (r0 < rstep) {
    double s[4] = {0, 0, 0, 0}, ss[4] = {0, 0, 0, 0};
    const int64_t begin = blockIdx.x * rows_per_block;
    const int64_t end = min(HW, begin + rows_per_block);
    const T* base = x + static_cast<int64_t>(b) * HW * C + 4 * q;
    for (int64_t r = begin + r0; r < end; r += rstep) {
      float v[4];
      load4<T>(base + r * C, v);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        s[k] += v[k];
        ss[k] += static_cast<double>(v[k]) * v[k];
      }
    }
    const int cpg = C / G;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int g = (4 * q + k) / cpg;
      atomicAdd(&sh[2 * g], s[k]);
      atomicAdd(&sh[2 * g + 1], ss[k]);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * G; i += blockDim.x) atomicAdd(&stats[static_cast<int64_t>(b) * 2 * G + i], sh[i]);
}

// y = (x - mean_g) * rstd_g * gamma + beta (optionally SiLU), bf16 out;
// grid (x, b).  Every thread owns one 8-channel column block for the whole
// launch (the grid stride is a multiple of C / 8), so its scale / shift
// coefficients stay in registers and the loop is 16-byte loads and stores.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float v[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float v[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<uint16_t>(const uint16_t* p, float v[8]) {
  const uint4 t = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[2 * k] = __uint_as_float(w[k] << 16);
    v[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) gn_apply_kernel(const T* __restrict__ x, int64_t HW, int C, int G,
                                                        const double* __restrict__ stats,
                                                        const float* __restrict__ gamma,
                                                        const float* __restrict__ beta, float eps, int silu,
                                                        uint16_t* __restrict__ y) {
  const int b = blockIdx.y;
  const int cpg = C / G;
  const int cu = C / 8;  // 8-channel blocks per pixel; divides 256
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  const int c0 = (tid % cu) * 8;
  float a[8], sh[8];
  const double inv_n = 1.0 / (static_cast<double>(HW) * cpg);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int c = c0 + k, g = c / cpg;
    // Mean and variance in double (the sums are large), rstd in float.
    const double mean = stats[(static_cast<int64_t>(b) * G + g) * 2] * inv_n;
    const double var = fmax(stats[(static_cast<int64_t>(b) * G + g) * 2 + 1] * inv_n - mean * mean, 0.0);
    const float rstd = rsqrtf(static_cast<float>(var) + eps);
    a[k] = rstd * __ldg(gamma + c);
    sh[k] = __ldg(beta + c) - static_cast<float>(mean) * a[k];
  }
  const int64_t units = HW * cu;
  const T* xb = x + static_cast<int64_t>(b) * HW * C;
  uint16_t* yb = y + static_cast<int64_t>(b) * HW * C;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
#pragma unroll 4
  for (int64_t u = tid; u < units; u += stride) {
    const int64_t e = u * 8;
    float v[8];
    load8<T>(xb + e, v);
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
      float a0 = fmaf(v[k], a[k], sh[k]);
      float a1 = fmaf(v[k + 1], a[k + 1], sh[k + 1]);
      if (silu) {  // the result is rounded to bf16: fast division suffices
        a0 = __fdividef(a0, 1.f + __expf(-a0));
        a1 = __fdividef(a1, 1.f + __expf(-a1));
      }
      o[k / 2] = pack_bf16x2(a0, a1);
    }
    *reinterpret_cast<uint4*>(yb + e) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ----------------------------------------------------------------- softmax
// P[r, :] = softmax(scale * S[r, :]) in bf16; one block per row, an online
// max / sum pass then a write pass.
__global__ void __launch_bounds__(256) softmax_rows_kernel(const float* __restrict__ S, int64_t n, int64_t ld_s,
                                                           float scale, uint16_t* __restrict__ P, int64_t ld_p) {
  const float* row = S + blockIdx.x * ld_s;
  uint16_t* out = P + blockIdx.x * ld_p;
  const float c = scale * 1.4426950408889634f;
  float m = -INFINITY, l = 0.f;
  const int64_t n4 = n & ~int64_t(3);  // float4 part; the n % 4 tail one element per thread
  for (int64_t i = threadIdx.x * 4; i < n4; i += 4 * blockDim.x) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(row + i));
    const float mx = fmaxf(fmaxf(t.x, t.y), fmaxf(t.z, t.w)) * c;
    const float mn = fmaxf(m, mx);
    l = l * exp2f(m - mn) + exp2f(t.x * c - mn) + exp2f(t.y * c - mn) + exp2f(t.z * c - mn) + exp2f(t.w * c - mn);
    m = mn;
  }
  if (n4 + threadIdx.x < n) {
    const float v = row[n4 + threadIdx.x] * c;
    const float mn = fmaxf(m, v);
    l = (m == -INFINITY ? 0.f : l * exp2f(m - mn)) + exp2f(v - mn);
    m = mn;
  }
  __shared__ float sm[32], sl[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float l2 = __shfl_xor_sync(0xffffffffu, l, o);
    const float mn = fmaxf(m, m2);
    l = (m == -INFINITY ? 0.f : l * exp2f(m - mn)) + (m2 == -INFINITY ? 0.f : l2 * exp2f(m2 - mn));
    m = mn;
  }
  if (lane == 0) {
    sm[warp] = m;
    sl[warp] = l;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? sm[lane] : -INFINITY;
    l = lane < nw ? sl[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float l2 = __shfl_xor_sync(0xffffffffu, l, o);
      const float mn = fmaxf(m, m2);
      l = (m == -INFINITY ? 0.f : l * exp2f(m - mn)) + (m2 == -INFINITY ? 0.f : l2 * exp2f(m2 - mn));
      m = mn;
    }
    if (lane == 0) {
      sm[0] = m;
      sl[0] = 1.f / l;
    }
  }
  __syncthreads();
  m = sm[0];
  const float inv = sl[0];
  for (int64_t i = threadIdx.x * 4; i < n4; i += 4 * blockDim.x) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(row + i));
    const uint32_t lo = pack_bf16x2(exp2f(t.x * c - m) * inv, exp2f(t.y * c - m) * inv);
    const uint32_t hi = pack_bf16x2(exp2f(t.z * c - m) * inv, exp2f(t.w * c - m) * inv);
    *reinterpret_cast<uint2*>(out + i) = make_uint2(lo, hi);
  }
  if (n4 + threadIdx.x < n) out[n4 + threadIdx.x] = f32_to_bf16(exp2f(row[n4 + threadIdx.x] * c - m) * inv);
}

// --------------------------------------------------------------- transpose
__global__ void transpose_bf16_kernel(const uint16_t* __restrict__ in, int64_t rows, int64_t cols, int64_t ld_in,
                                      uint16_t* __restrict__ out, int64_t ld_out) {
  __shared__ uint16_t t[32][33];
  const int64_t r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int64_t r = r0 + k, c = c0 + threadIdx.x;
    if (r < rows && c < cols) t[k][threadIdx.x] = in[r * ld_in + c];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int64_t c = c0 + k, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[c * ld_out + r] = t[threadIdx.x][k];
  }
}

// GroupNorm statistics from the partial sums a convolution epilogue wrote
// (gn_part, EpilogueArgs): stats[b, g] += sums over regions and slots (stats
// zeroed first).  Block (x, b, region) reads kSlots consecutive slots as
// whole coalesced rows of 2 G floats; thread t keeps element t % 2G.
constexpr int kFinalizeSlots = 64;
__global__ void __launch_bounds__(256) gn_finalize_kernel(const float* __restrict__ part, int64_t region_stride,
                                                          int64_t slots_per_img, int G,
                                                          double* __restrict__ stats) {
  const int b = blockIdx.y;
  const int e2 = 2 * G;
  const int el = threadIdx.x % e2;
  const int sub = threadIdx.x / e2, nsub = blockDim.x / e2;
  const float* base = part + blockIdx.z * region_stride + static_cast<int64_t>(b) * slots_per_img * e2;
  const int64_t s0 = static_cast<int64_t>(blockIdx.x) * kFinalizeSlots;
  const int64_t s1 = min(slots_per_img, s0 + kFinalizeSlots);
  double acc = 0.0;
  if (sub < nsub)
    for (int64_t sl = s0 + sub; sl < s1; sl += nsub) acc += base[sl * e2 + el];
  __shared__ double red[256];
  red[threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.x < e2) {
    double t = 0.0;
    for (int k = 0; k < nsub; ++k) t += red[k * e2 + threadIdx.x];
    atomicAdd(&stats[static_cast<int64_t>(b) * e2 + threadIdx.x], t);
  }
}

// Tiled decode: blend the decoded tile T [B, C, h, w] in place with the
// tile above (its last ev rows) and then the tile to the left (its last eh
// columns), weights y / ev and x / eh on T, and copy the top-left
// keep_h x keep_w band to out [B, C, H, W] at (oy, ox).
__global__ void tile_blend_kernel(float* __restrict__ T, const float* __restrict__ above, int64_t ha,
                                  const float* __restrict__ left, int64_t wl, int64_t BC, int64_t h, int64_t w,
                                  int64_t ev, int64_t eh, int64_t keep_h, int64_t keep_w, float* __restrict__ out,
                                  int64_t H, int64_t W, int64_t oy, int64_t ox) {
  const int64_t total = BC * h * w;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t x = i % w;
    const int64_t y = (i / w) % h;
    const int64_t bc = i / (h * w);
    float t = T[i];
    if (y < ev) {
      const float wv = static_cast<float>(y) / static_cast<float>(ev);
      t = above[(bc * ha + (ha - ev + y)) * w + x] * (1.0f - wv) + t * wv;
    }
    if (x < eh) {
      const float wh = static_cast<float>(x) / static_cast<float>(eh);
      t = left[(bc * h + y) * wl + (wl - eh + x)] * (1.0f - wh) + t * wh;
    }
    T[i] = t;
    if (y < keep_h && x < keep_w) out[(bc * H + oy + y) * W + ox + x] = t;
  }
}

int grid_for(int64_t units, int threads) {
  const int64_t g = (units + threads - 1) / threads;
  return static_cast<int>(g < 1 ? 1 : (g > 148 * 32 ? 148 * 32 : g));
}

}  // namespace

cudaError_t launch_latent_unpack(const float* lat, const float* mean, const float* var, float eps, int B, int ph,
                                 int pw, int C, int Cpad, uint16_t* out, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(B) * 4 * ph * pw * Cpad;
  latent_unpack_kernel<<<grid_for(total, 256), 256, 0, s>>>(lat, mean, var, eps, B, ph, pw, C, Cpad, out);
  return cudaGetLastError();
}

cudaError_t launch_gn_stats(const void* x, bool bf16, int B, int64_t HW, int C, int G, double* stats,
                            cudaStream_t s) {
  if (C % 4 != 0 || C % G != 0 || C / 4 > 256) return cudaErrorInvalidValue;
  const int rstep = 256 / (C / 4);
  int64_t rpb = (HW + 295) / 296;
  rpb = (rpb + rstep - 1) / rstep * rstep;
  dim3 grid(static_cast<unsigned>((HW + rpb - 1) / rpb), static_cast<unsigned>(B));
  const size_t sh = sizeof(double) * 2 * G;
  if (bf16)
    gn_stats_kernel<uint16_t><<<grid, 256, sh, s>>>(static_cast<const uint16_t*>(x), HW, C, G, rpb, stats);
  else
    gn_stats_kernel<float><<<grid, 256, sh, s>>>(static_cast<const float*>(x), HW, C, G, rpb, stats);
  return cudaGetLastError();
}

cudaError_t launch_gn_apply(const void* x, bool bf16, int B, int64_t HW, int C, int G, const double* stats,
                            const float* gamma, const float* beta, float eps, bool silu, uint16_t* y,
                            cudaStream_t s) {
  if (C % 8 != 0 || C % G != 0 || 256 % (C / 8) != 0) return cudaErrorInvalidValue;
  const int64_t units = HW * (C / 8);
  // Eight resident blocks per SM over the whole launch.
  int64_t blocks = std::min<int64_t>((units + 255) / 256, std::max<int64_t>(1, 148 * 8 / B));
  dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(B));
  if (bf16)
    gn_apply_kernel<uint16_t><<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(x), HW, C, G, stats, gamma, beta,
                                                   eps, silu ? 1 : 0, y);
  else
    gn_apply_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(x), HW, C, G, stats, gamma, beta, eps,
                                                silu ? 1 : 0, y);
  return cudaGetLastError();
}

cudaError_t launch_softmax_rows(const float* S, int64_t rows, int64_t n, int64_t ld_s, float scale, uint16_t* P,
                                int64_t ld_p, cudaStream_t s) {
  if (ld_s % 4 != 0 || ld_p % 4 != 0) return cudaErrorInvalidValue;
  softmax_rows_kernel<<<static_cast<unsigned>(rows), 256, 0, s>>>(S, n, ld_s, scale, P, ld_p);
  return cudaGetLastError();
}

cudaError_t launch_transpose_bf16(const uint16_t* in, int64_t rows, int64_t cols, int64_t ld_in, uint16_t* out,
                                  int64_t ld_out, cudaStream_t s) {
  dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((rows + 31) / 32));
  transpose_bf16_kernel<<<grid, dim3(32, 8), 0, s>>>(in, rows, cols, ld_in, out, ld_out);
  return cudaGetLastError();
}

cudaError_t launch_gn_finalize(const float* part, int n_regions, int64_t region_stride, int64_t slots_per_img, int B,
                               int G, double* stats, cudaStream_t s) {
  if (2 * G > 256) return cudaErrorInvalidValue;
  dim3 grid(static_cast<unsigned>((slots_per_img + kFinalizeSlots - 1) / kFinalizeSlots), static_cast<unsigned>(B),
            static_cast<unsigned>(n_regions));
  gn_finalize_kernel<<<grid, 256, 0, s>>>(part, region_stride, slots_per_img, G, stats);
  return cudaGetLastError();
}

cudaError_t launch_tile_blend(float* T, const float* above, int64_t ha, const float* left, int64_t wl, int B, int C,
                              int64_t h, int64_t w, int64_t ev, int64_t eh, int64_t keep_h, int64_t keep_w, float* out,
                              int64_t H, int64_t W, int64_t oy, int64_t ox, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(B) * C * h * w;
  tile_blend_kernel<<<grid_for(total, 256), 256, 0, s>>>(T, above, ha, left, wl, static_cast<int64_t>(B) * C, h, w, ev,
                                                          eh, keep_h, keep_w, out, H, W, oy, ox);
  return cudaGetLastError();
}

}  // namespace dcpp
