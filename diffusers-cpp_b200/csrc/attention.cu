// Attention prologue for the op-level entry point: RMSNorm + RoPE of q and
// k and the relayout of the fused q|k|v projection rows into the attention
// kernel's operands (Flux2Attention.hpp:93-122, Flux2ParallelSelfAttention.hpp:
// 236-249).  Inside the model this work is fused into the QKV GEMM epilogue.
#include "common.cuh"
#include "kernels.cuh"

namespace dcpp {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per (token row, head, region in {q, k, v}); lane l owns dims
// 4l..4l+3 (rotary pairs 2l and 2l+1).  q, k -> [B, H, S, 128];
// v -> transposed [B, H, 128, vt_stride].
__global__ void qk_norm_rope_kernel(const uint16_t* __restrict__ qkv, int64_t B, int64_t S, int64_t H,
                                    const float* __restrict__ wq, const float* __restrict__ wk, float eps,
                                    const float2* __restrict__ rope, uint16_t* q, uint16_t* k, uint16_t* vt,
                                    int64_t vt_stride) {
  const int64_t wid = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total = B * S * H * 3;
  if (wid >= total) return;
  const int region = static_cast<int>(wid % 3);
  const int64_t hh = (wid / 3) % H;
  const int64_t row = wid / (3 * H);  // b*S + s
  const int64_t bb = row / S;
  const int64_t s = row - bb * S;
  const uint16_t* src = qkv + row * (3 * H * 128) + region * H * 128 + hh * 128 + lane * 4;
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  float x[4] = {__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xFFFF0000u), __uint_as_float(raw.y << 16),
                __uint_as_float(raw.y & 0xFFFF0000u)};
  if (region == 2) {
    uint16_t* dst = vt + ((bb * H + hh) * 128 + lane * 4) * vt_stride + s;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat16 b = __float2bfloat16_rn(x[i]);
      dst[i * vt_stride] = *reinterpret_cast<uint16_t*>(&b);
    }
    return;
  }
  const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
  const float rs = 1.0f / sqrtf(ss * (1.0f / 128.0f) + eps);
  const float* w = region == 0 ? wq : wk;
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = x[i] * rs * w[lane * 4 + i];
#pragma unroll
  for (int pr = 0; pr < 2; ++pr) {
    const float2 cs = rope[s * 64 + lane * 2 + pr];
    const float x0 = x[2 * pr], x1 = x[2 * pr + 1];
    x[2 * pr] = x0 * cs.x - x1 * cs.y;
    x[2 * pr + 1] = x0 * cs.y + x1 * cs.x;
  }
  uint16_t* dst = (region == 0 ? q : k) + ((bb * H + hh) * S + s) * 128 + lane * 4;
  *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
}

}  // namespace

cudaError_t launch_qk_norm_rope(const uint16_t* qkv, int64_t B, int64_t S, int64_t H, const float* norm_q,
                                const float* norm_k, float eps, const float2* rope, uint16_t* q, uint16_t* k,
                                uint16_t* vt, int64_t vt_stride, cudaStream_t s) {
  const int64_t warps = B * S * H * 3;
  if (warps <= 0) return cudaSuccess;
  const int64_t blocks = (warps * 32 + 255) / 256;
  qk_norm_rope_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(qkv, B, S, H, norm_q, norm_k, eps, rope, q, k,
                                                                      vt, vt_stride);
  return cudaGetLastError();
}

}  // namespace dcpp
