// Joint image+text attention of the Flux2 blocks:
//   O = softmax(Q K^T * scale) V,  no mask  (FlashAttentionOp.cpp:6-105,
//   ggml_flash_attn_ext(q, k, v, nullptr, 1/sqrt(d)))
// Q/K arrive already RMS-normalised and rotated (the QKV GEMM epilogue or
// qk_norm_rope_kernel below does that), laid out [B, H, S, 128] bf16.
//
// Flash-attention forward with online softmax in the exp2 domain.  CTA =
// 8 warps x 16 query rows = 128 rows of one (batch, head); K/V tiles of 64
// keys are double-buffered in shared memory with cp.async (16-byte rows
// XOR-swizzled by row to avoid bank conflicts).  The Q tile stays in
// shared memory for the whole key loop.
#include "common.cuh"
#include "kernels.cuh"

namespace dcpp {

namespace {

constexpr int kAttnWarps = 8;
constexpr int kAttnBQ = kAttnWarps * 16;  // 128 query rows
constexpr int kAttnBK = 64;               // keys per tile
constexpr int kHeadDim = 128;
constexpr int kRowBytes = kHeadDim * 2;   // 256 bytes
constexpr int kTileBytes = kAttnBK * kRowBytes;  // 16 KB
constexpr int kAttnSmem = kAttnBQ * kRowBytes + 4 * kTileBytes;  // Q + 2x(K,V) = 96 KB

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * kRowBytes + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Load rows [row0, row0 + nrows) of a [S, 128] bf16 matrix into a swizzled
// smem tile (rows beyond S are zero-filled).
__device__ __forceinline__ void load_tile(uint32_t sbase, const uint16_t* g, int row0, int nrows, int S) {
  for (int i = threadIdx.x; i < nrows * 16; i += kAttnWarps * 32) {
    const int r = i >> 4;
    const int c = i & 15;
    const int gr = row0 + r;
    const bool valid = gr < S;
    const uint16_t* src = g + static_cast<int64_t>(valid ? gr : 0) * kHeadDim + c * 8;
    cp_async16(sbase + swz(r, c), src, valid);
  }
}

__global__ void __launch_bounds__(kAttnWarps * 32, 2) flash_attn_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int qt = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int S = a.S;
  const int64_t bh = (static_cast<int64_t>(b) * a.H + h) * S;
  const uint16_t* Qg = a.q + bh * kHeadDim;
  const uint16_t* Kg = a.k + bh * kHeadDim;
  const uint16_t* Vg = a.v + bh * kHeadDim;

  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK[2] = {sQ + kAttnBQ * kRowBytes, sQ + kAttnBQ * kRowBytes + 2 * kTileBytes};
  const uint32_t sV[2] = {sK[0] + kTileBytes, sK[1] + kTileBytes};

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;  // row within 8
  const int t = lane & 3;   // column pair

  load_tile(sQ, Qg, qt * kAttnBQ, kAttnBQ, S);
  load_tile(sK[0], Kg, 0, kAttnBK, S);
  load_tile(sV[0], Vg, 0, kAttnBK, S);
  cp_async_commit();

  const float sl2 = a.scale * 1.4426950408889634f;
  const int nkt = (S + kAttnBK - 1) / kAttnBK;

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int j = 0; j < nkt; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkt) {
      load_tile(sK[buf ^ 1], Kg, (j + 1) * kAttnBK, kAttnBK, S);
      load_tile(sV[buf ^ 1], Vg, (j + 1) * kAttnBK, kAttnBK, S);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();

    // S = Q K^T for 16 rows x 64 keys.
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    {
      const int mi = lane >> 3;
      const int qr = warp * 16 + (mi & 1) * 8 + (lane & 7);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t qf[4];
        ldsm_x4(sQ + swz(qr, ks * 2 + (mi >> 1)), qf[0], qf[1], qf[2], qf[3]);
#pragma unroll
        for (int nt = 0; nt < 8; nt += 2) {
          const int key = (nt + (mi >> 1)) * 8 + (lane & 7);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(sK[buf] + swz(key, ks * 2 + (mi & 1)), b0, b1, b2, b3);
          mma_bf16(s[nt], qf, b0, b1);
          mma_bf16(s[nt + 1], qf, b2, b3);
        }
      }
    }
    // Mask keys beyond S (last tile only).
    const int kbase = j * kAttnBK;
    if (kbase + kAttnBK > S) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int c = kbase + nt * 8 + 2 * t;
        if (c >= S) { s[nt][0] = -INFINITY; s[nt][2] = -INFINITY; }
        if (c + 1 >= S) { s[nt][1] = -INFINITY; s[nt][3] = -INFINITY; }
      }
    }
    // Online softmax (rows g and g+8 of this warp).
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]) * sl2);
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]) * sl2);
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float c0 = fast_exp2(m0 - mx0);
    const float c1 = fast_exp2(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pf[8][2];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = fast_exp2(s[nt][0] * sl2 - mx0);
      const float p1 = fast_exp2(s[nt][1] * sl2 - mx0);
      const float p2 = fast_exp2(s[nt][2] * sl2 - mx1);
      const float p3 = fast_exp2(s[nt][3] * sl2 - mx1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      pf[nt][0] = pack_bf16x2(p0, p1);
      pf[nt][1] = pack_bf16x2(p2, p3);
    }
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      o[dt][0] *= c0; o[dt][1] *= c0;
      o[dt][2] *= c1; o[dt][3] *= c1;
    }
    // O += P V.
    {
      const int mi = lane >> 3;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint32_t af[4] = {pf[2 * ks][0], pf[2 * ks][1], pf[2 * ks + 1][0], pf[2 * ks + 1][1]};
        const int key = ks * 16 + (mi & 1) * 8 + (lane & 7);
#pragma unroll
        for (int dt = 0; dt < 16; dt += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(sV[buf] + swz(key, dt + (mi >> 1)), b0, b1, b2, b3);
          mma_bf16(o[dt], af, b0, b1);
          mma_bf16(o[dt + 1], af, b2, b3);
        }
      }
    }
    __syncthreads();
  }

  // Row sums across the quad, normalise, store bf16.
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.0f / l0;
  const float inv1 = 1.0f / l1;
  const int r0 = qt * kAttnBQ + warp * 16 + g;
  const int r1 = r0 + 8;
  uint16_t* out0 = a.o + (static_cast<int64_t>(b) * S + r0) * a.ld_o + h * kHeadDim;
  uint16_t* out1 = a.o + (static_cast<int64_t>(b) * S + r1) * a.ld_o + h * kHeadDim;
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    const int d = dt * 8 + 2 * t;
    if (r0 < S) *reinterpret_cast<uint32_t*>(out0 + d) = pack_bf16x2(o[dt][0] * inv0, o[dt][1] * inv0);
    if (r1 < S) *reinterpret_cast<uint32_t*>(out1 + d) = pack_bf16x2(o[dt][2] * inv1, o[dt][3] * inv1);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per (token row, head, region in {q, k, v}); lane l owns dims
// 4l..4l+3 (rotary pairs 2l and 2l+1).
__global__ void qk_norm_rope_kernel(const uint16_t* __restrict__ qkv, int64_t B, int64_t S, int64_t H,
                                    const float* __restrict__ wq, const float* __restrict__ wk, float eps,
                                    const float2* __restrict__ rope, uint16_t* q, uint16_t* k, uint16_t* v) {
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
  uint16_t* dst = (region == 0 ? q : (region == 1 ? k : v)) + ((bb * H + hh) * S + s) * 128 + lane * 4;
  if (region < 2) {
    const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
    const float rs = 1.0f / sqrtf(ss * (1.0f / 128.0f) + eps);
    const float* w = region == 0 ? wq : wk;
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = x[i] * rs * w[lane * 4 + i];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float2 cs = rope[s * 64 + lane * 2 + p];
      const float x0 = x[2 * p], x1 = x[2 * p + 1];
      x[2 * p] = x0 * cs.x - x1 * cs.y;
      x[2 * p + 1] = x0 * cs.y + x1 * cs.x;
    }
  }
  *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
}

}  // namespace

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s) {
  if (a.S <= 0 || a.H <= 0 || a.B <= 0) return cudaSuccess;
  if (a.ld_o % 8) return cudaErrorInvalidValue;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(flash_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  dim3 grid((a.S + kAttnBQ - 1) / kAttnBQ, a.H, a.B);
  flash_attn_kernel<<<grid, kAttnWarps * 32, kAttnSmem, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_qk_norm_rope(const uint16_t* qkv, int64_t B, int64_t S, int64_t H, const float* norm_q,
                                const float* norm_k, float eps, const float2* rope, uint16_t* q, uint16_t* k,
                                uint16_t* v, cudaStream_t s) {
  const int64_t warps = B * S * H * 3;
  if (warps <= 0) return cudaSuccess;
  const int64_t blocks = (warps * 32 + 255) / 256;
  qk_norm_rope_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(qkv, B, S, H, norm_q, norm_k, eps, rope, q, k, v);
  return cudaGetLastError();
}

}  // namespace dcpp
