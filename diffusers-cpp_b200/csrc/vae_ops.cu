// Row / pixel kernels of the Flux2 VAE decode (the convolutions themselves
// are implicit GEMMs on the tcgen05 GEMM, gemm.cu):
//   latent unpack + BatchNorm de-normalisation + unpatchify
//       (Flux2KleinPipeline.cpp:538-556, :606-630)
//   GroupNorm statistics and GroupNorm (+ SiLU) application
//       (GroupNorm.cpp: ggml_norm over (C/G) x H x W per group, eps 1e-6, affine)
//   row softmax of the mid-block attention scores (SoftmaxAttentionOp.cpp)
//   bf16 transpose, 3x3 convolution with few output channels (conv_out)
// Images are NHWC: pixel (b, y, x) is row (b H + y) W + x, channels contiguous.
#include <cuda_bf16.h>

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
// grid (x, b): 8 channels per thread and step.
template <typename T>
__global__ void __launch_bounds__(256) gn_apply_kernel(const T* __restrict__ x, int64_t HW, int C, int G,
                                                        const double* __restrict__ stats,
                                                        const float* __restrict__ gamma,
                                                        const float* __restrict__ beta, float eps, int silu,
                                                        uint16_t* __restrict__ y) {
  extern __shared__ float coef[];  // [2 C]: scale, shift
  const int b = blockIdx.y;
  const int cpg = C / G;
  const double n = static_cast<double>(HW) * cpg;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const int g = c / cpg;
    const double mean = stats[(static_cast<int64_t>(b) * G + g) * 2] / n;
    const double var = fmax(stats[(static_cast<int64_t>(b) * G + g) * 2 + 1] / n - mean * mean, 0.0);
    const float rstd = static_cast<float>(1.0 / sqrt(var + static_cast<double>(eps)));
    const float a = rstd * gamma[c];
    coef[c] = a;
    coef[C + c] = beta[c] - static_cast<float>(mean) * a;
  }
  __syncthreads();
  const int64_t units = HW * (C / 8);
  const T* xb = x + static_cast<int64_t>(b) * HW * C;
  uint16_t* yb = y + static_cast<int64_t>(b) * HW * C;
  for (int64_t u = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; u < units;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = u * 8;
    const int c0 = static_cast<int>(e % C);
    float v[8];
    load4<T>(xb + e, v);
    load4<T>(xb + e + 4, v + 4);
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
      float a0 = v[k] * coef[c0 + k] + coef[C + c0 + k];
      float a1 = v[k + 1] * coef[c0 + k + 1] + coef[C + c0 + k + 1];
      if (silu) {
        a0 = a0 / (1.f + __expf(-a0));
        a1 = a1 / (1.f + __expf(-a1));
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
  for (int64_t i = threadIdx.x * 4; i < n; i += 4 * blockDim.x) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(row + i));
    const float mx = fmaxf(fmaxf(t.x, t.y), fmaxf(t.z, t.w)) * c;
    const float mn = fmaxf(m, mx);
    l = l * exp2f(m - mn) + exp2f(t.x * c - mn) + exp2f(t.y * c - mn) + exp2f(t.z * c - mn) + exp2f(t.w * c - mn);
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
  for (int64_t i = threadIdx.x * 4; i < n; i += 4 * blockDim.x) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(row + i));
    const uint32_t lo = pack_bf16x2(exp2f(t.x * c - m) * inv, exp2f(t.y * c - m) * inv);
    const uint32_t hi = pack_bf16x2(exp2f(t.z * c - m) * inv, exp2f(t.w * c - m) * inv);
    *reinterpret_cast<uint2*>(out + i) = make_uint2(lo, hi);
  }
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

// ------------------------------------------------------- small-Cout conv3x3
// out[b, co, y, x] = bias[co] + sum_{tap, c} w[co][tap][c] * X[b, y+dy, x+dx, c]
// (pad 1), X bf16 NHWC, out f32 NCHW; one thread per pixel, weights in smem.
template <int kCout>
__global__ void __launch_bounds__(128) conv3x3_small_kernel(const uint16_t* __restrict__ X, int B, int H, int W,
                                                            int C, const float* __restrict__ w,
                                                            const float* __restrict__ bias, float* __restrict__ out) {
  extern __shared__ float ws[];  // [kCout][9][C]
  for (int i = threadIdx.x; i < kCout * 9 * C; i += blockDim.x) ws[i] = w[i];
  __syncthreads();
  const int64_t HW = static_cast<int64_t>(H) * W;
  const int64_t pix = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (pix >= B * HW) return;
  const int b = static_cast<int>(pix / HW);
  const int64_t hw = pix - b * HW;
  const int y = static_cast<int>(hw / W), x = static_cast<int>(hw % W);
  float acc[kCout];
#pragma unroll
  for (int co = 0; co < kCout; ++co) acc[co] = bias[co];
  for (int tap = 0; tap < 9; ++tap) {
    const int yy = y + tap / 3 - 1, xx = x + tap % 3 - 1;
    if (yy < 0 || yy >= H || xx < 0 || xx >= W) continue;
    const uint16_t* src = X + ((static_cast<int64_t>(b) * H + yy) * W + xx) * C;
    for (int c = 0; c < C; c += 8) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(src + c));
      const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
      float v[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[2 * k] = __uint_as_float(wd[k] << 16);
        v[2 * k + 1] = __uint_as_float(wd[k] & 0xFFFF0000u);
      }
#pragma unroll
      for (int co = 0; co < kCout; ++co) {
        const float* wr = ws + (co * 9 + tap) * C + c;
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[co] = fmaf(wr[k], v[k], acc[co]);
      }
    }
  }
#pragma unroll
  for (int co = 0; co < kCout; ++co) out[(static_cast<int64_t>(b) * kCout + co) * HW + hw] = acc[co];
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
  if (C % 8 != 0 || C % G != 0) return cudaErrorInvalidValue;
  const int64_t units = HW * (C / 8);
  dim3 grid(static_cast<unsigned>(grid_for(units, 256) / B + 1), static_cast<unsigned>(B));
  const size_t sh = sizeof(float) * 2 * C;
  if (bf16)
    gn_apply_kernel<uint16_t><<<grid, 256, sh, s>>>(static_cast<const uint16_t*>(x), HW, C, G, stats, gamma, beta,
                                                    eps, silu ? 1 : 0, y);
  else
    gn_apply_kernel<float><<<grid, 256, sh, s>>>(static_cast<const float*>(x), HW, C, G, stats, gamma, beta, eps,
                                                 silu ? 1 : 0, y);
  return cudaGetLastError();
}

cudaError_t launch_softmax_rows(const float* S, int64_t rows, int64_t n, int64_t ld_s, float scale, uint16_t* P,
                                int64_t ld_p, cudaStream_t s) {
  if (n % 4 != 0 || ld_s % 4 != 0 || ld_p % 4 != 0) return cudaErrorInvalidValue;
  softmax_rows_kernel<<<static_cast<unsigned>(rows), 256, 0, s>>>(S, n, ld_s, scale, P, ld_p);
  return cudaGetLastError();
}

cudaError_t launch_transpose_bf16(const uint16_t* in, int64_t rows, int64_t cols, int64_t ld_in, uint16_t* out,
                                  int64_t ld_out, cudaStream_t s) {
  dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((rows + 31) / 32));
  transpose_bf16_kernel<<<grid, dim3(32, 8), 0, s>>>(in, rows, cols, ld_in, out, ld_out);
  return cudaGetLastError();
}

cudaError_t launch_conv3x3_small(const uint16_t* X, int B, int H, int W, int C, int Cout, const float* w,
                                 const float* bias, float* out, cudaStream_t s) {
  if (C % 8 != 0) return cudaErrorInvalidValue;
  const int64_t pixels = static_cast<int64_t>(B) * H * W;
  const unsigned grid = static_cast<unsigned>((pixels + 127) / 128);
  const size_t sh = sizeof(float) * Cout * 9 * C;
  if (sh > 200 * 1024) return cudaErrorInvalidValue;
  switch (Cout) {
    case 1:
      cudaFuncSetAttribute(conv3x3_small_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sh));
      conv3x3_small_kernel<1><<<grid, 128, sh, s>>>(X, B, H, W, C, w, bias, out);
      break;
    case 3:
      cudaFuncSetAttribute(conv3x3_small_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sh));
      conv3x3_small_kernel<3><<<grid, 128, sh, s>>>(X, B, H, W, C, w, bias, out);
      break;
    case 4:
      cudaFuncSetAttribute(conv3x3_small_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sh));
      conv3x3_small_kernel<4><<<grid, 128, sh, s>>>(X, B, H, W, C, w, bias, out);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace dcpp
