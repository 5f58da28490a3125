// ggml block-quantised weight formats on the device.
//
// Q8_0 (34 bytes / 32 weights): f16 d, int8 q[32];          w = d * q
// Q4_K (144 bytes / 256 weights): f16 d, f16 dmin, 12 bytes of packed
//   6-bit (scale, min) pairs for 8 sub-blocks of 32, 128 bytes of nibbles;
//   sub-block j: w = (d * sc_j) * q - (dmin * m_j).  Nibbles: byte l of
//   the 32-byte group g holds element l of sub-block 2g (low nibble) and of
//   sub-block 2g+1 (high nibble).
// The arithmetic follows gguf-py 0.19.0 quants.py (Q8_0 :396-401, Q4_K
// :475-523) operation by operation in f32 with round-to-nearest and no
// contraction (__fmul_rn / __fsub_rn), so the f32 output is bit-identical.
#include "common.cuh"
#include "kernels.cuh"

namespace dcpp {

namespace {

__device__ __forceinline__ float half_bits_to_f32(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

// Unpack the 6-bit scale and min of sub-block j (0..7) from the 12 packed
// bytes (gguf-py Q4_K.get_scale_min: bytes 0-3 low scales, 4-7 low mins,
// 8-11 high bits).
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, int j, int& sc, int& m) {
  if (j < 4) {
    sc = s[j] & 0x3F;
    m = s[j + 4] & 0x3F;
  } else {
    sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 2) & 0x30);
    m = (s[j + 4] >> 4) | ((s[j] >> 2) & 0x30);
  }
}

template <bool kBf16>
__device__ __forceinline__ void store_val(void* out, int64_t i, float v) {
  if (kBf16) {
    __nv_bfloat16 b = __float2bfloat16_rn(v);
    reinterpret_cast<__nv_bfloat16*>(out)[i] = b;
  } else {
    reinterpret_cast<float*>(out)[i] = v;
  }
}

// Eight consecutive outputs per thread, written as one 16-byte (bf16) or
// two 16-byte (f32) stores, so a warp writes 512 / 1024 contiguous bytes.
template <bool kBf16>
__device__ __forceinline__ void store8(void* out, int64_t i0, const float (&v)[8]) {
  if (kBf16) {
    uint4 o = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                         pack_bf16x2(v[6], v[7]));
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out) + i0) = o;
  } else {
    float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + i0);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// One thread per 8 weights of a Q8_0 block (4 threads per block), grid-stride
// over blocks; the 8 quants are read as four 2-byte loads (blocks are only
// 2-byte aligned).
template <bool kBf16>
__global__ void __launch_bounds__(256) dequant_q8_0_kernel(const uint8_t* __restrict__ blocks, int64_t nblocks,
                                                           void* out) {
  const int64_t n = nblocks * 4;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = t >> 2;
    const int part = static_cast<int>(t & 3);
    const uint16_t* blk = reinterpret_cast<const uint16_t*>(blocks + b * 34);
    const float d = half_bits_to_f32(__ldg(blk));
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint16_t q2 = __ldg(blk + 1 + part * 4 + i);
      v[2 * i] = __fmul_rn(static_cast<float>(static_cast<int8_t>(q2 & 0xFF)), d);
      v[2 * i + 1] = __fmul_rn(static_cast<float>(static_cast<int8_t>(q2 >> 8)), d);
    }
    store8<kBf16>(out, b * 32 + part * 8, v);
  }
}

// One thread per 8 weights of a Q4_K super-block (32 threads per block),
// grid-stride over blocks; the 16-byte header (d, dmin, 12 scale bytes) is
// one vector load (blocks are 16-byte aligned: 144 = 9 x 16).
template <bool kBf16>
__global__ void __launch_bounds__(256) dequant_q4_k_kernel(const uint8_t* __restrict__ blocks, int64_t nblocks,
                                                           void* out) {
  const int64_t n = nblocks * 32;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = t >> 5;
    const int j = static_cast<int>((t >> 2) & 7);  // sub-block
    const int l0 = static_cast<int>(t & 3) * 8;    // first element within the sub-block
    const uint8_t* blk = blocks + b * 144;
    const uint4 h = __ldg(reinterpret_cast<const uint4*>(blk));
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(blk + 16 + (j >> 1) * 32 + l0));
    const float d = half_bits_to_f32(static_cast<uint16_t>(h.x & 0xFFFF));
    const float dmin = half_bits_to_f32(static_cast<uint16_t>(h.x >> 16));
    uint8_t sb[12];
    const uint32_t hw[3] = {h.y, h.z, h.w};
#pragma unroll
    for (int i = 0; i < 12; ++i) sb[i] = static_cast<uint8_t>(hw[i >> 2] >> (8 * (i & 3)));
    int sc, m;
    q4k_scale_min(sb, j, sc, m);
    const float ds = __fmul_rn(d, static_cast<float>(sc));
    const float dm = __fmul_rn(dmin, static_cast<float>(m));
    const int shift = (j & 1) * 4;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t w = i < 4 ? raw.x : raw.y;
      const float q = static_cast<float>((w >> (8 * (i & 3) + shift)) & 0x0F);
      v[i] = __fsub_rn(__fmul_rn(ds, q), dm);
    }
    store8<kBf16>(out, b * 256 + j * 32 + l0, v);
  }
}

template <bool kBf16>
__global__ void dequant_f16_kernel(const uint16_t* __restrict__ in, int64_t n, void* out) {
  int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n) store_val<kBf16>(out, i, half_bits_to_f32(in[i]));
}

template <bool kBf16>
__global__ void dequant_bf16_kernel(const uint16_t* __restrict__ in, int64_t n, void* out) {
  int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n) {
    if (kBf16) reinterpret_cast<uint16_t*>(out)[i] = in[i];
    else reinterpret_cast<float*>(out)[i] = bf16_bits_to_f32(in[i]);
  }
}

template <bool kBf16>
__global__ void dequant_f32_kernel(const float* __restrict__ in, int64_t n, void* out) {
  int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n) store_val<kBf16>(out, i, in[i]);
}

// Eight elements per thread (16-byte loads of f16 / bf16, two of f32;
// 16-byte bf16 or two 16-byte f32 stores) when n % 8 == 0 and the input is
// 16-byte aligned.
template <int kType, bool kBf16>
__global__ void convert8_kernel(const void* __restrict__ in, int64_t n8, void* out) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= n8) return;
  float v[8];
  if (kType == kTypeF32) {
    const float4* p = reinterpret_cast<const float4*>(in) + 2 * i;
    const float4 a = __ldg(p), b = __ldg(p + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(in) + i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (kType == kTypeBF16) {
        v[2 * k] = __uint_as_float(w[k] << 16);
        v[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
      } else {
        v[2 * k] = half_bits_to_f32(static_cast<uint16_t>(w[k] & 0xFFFF));
        v[2 * k + 1] = half_bits_to_f32(static_cast<uint16_t>(w[k] >> 16));
      }
    }
  }
  store8<kBf16>(out, i * 8, v);
}

// Grid-stride kernels: at most 16 CTAs of 256 threads per SM (148 SMs).
inline unsigned grid_cap(int64_t n, int threads) {
  const int64_t g = (n + threads - 1) / threads;
  return static_cast<unsigned>(g < 148 * 16 ? g : 148 * 16);
}

inline unsigned grid_for(int64_t n, int threads) {
  return static_cast<unsigned>((n + threads - 1) / threads);
}

template <bool kBf16>
cudaError_t dequant_impl(int type, const void* blocks, int64_t n, void* out, cudaStream_t s) {
  constexpr int T = 256;
  // 16-byte vector stores; Q4_K reads its nibbles 8 bytes at a time.
  if (reinterpret_cast<uintptr_t>(out) & 15) return cudaErrorMisalignedAddress;
  if (type == kTypeQ4_K && (reinterpret_cast<uintptr_t>(blocks) & 15)) return cudaErrorMisalignedAddress;
  if (type == kTypeQ8_0 && (reinterpret_cast<uintptr_t>(blocks) & 1)) return cudaErrorMisalignedAddress;
  const bool vec8 = n > 0 && n % 8 == 0 && (reinterpret_cast<uintptr_t>(blocks) & 15) == 0;
  switch (type) {
    case kTypeQ8_0: {
      if (n % 32) return cudaErrorInvalidValue;
      int64_t nb = n / 32;
      if (nb) dequant_q8_0_kernel<kBf16><<<grid_cap(nb * 4, T), T, 0, s>>>(static_cast<const uint8_t*>(blocks), nb, out);
      break;
    }
    case kTypeQ4_K: {
      if (n % 256) return cudaErrorInvalidValue;
      int64_t nb = n / 256;
      if (nb) dequant_q4_k_kernel<kBf16><<<grid_cap(nb * 32, T), T, 0, s>>>(static_cast<const uint8_t*>(blocks), nb, out);
      break;
    }
    case kTypeF16:
      if (vec8) convert8_kernel<kTypeF16, kBf16><<<grid_for(n / 8, T), T, 0, s>>>(blocks, n / 8, out);
      else if (n) dequant_f16_kernel<kBf16><<<grid_for(n, T), T, 0, s>>>(static_cast<const uint16_t*>(blocks), n, out);
      break;
    case kTypeBF16:
      if (vec8) convert8_kernel<kTypeBF16, kBf16><<<grid_for(n / 8, T), T, 0, s>>>(blocks, n / 8, out);
      else if (n) dequant_bf16_kernel<kBf16><<<grid_for(n, T), T, 0, s>>>(static_cast<const uint16_t*>(blocks), n, out);
      break;
    case kTypeF32:
      if (vec8) convert8_kernel<kTypeF32, kBf16><<<grid_for(n / 8, T), T, 0, s>>>(blocks, n / 8, out);
      else if (n) dequant_f32_kernel<kBf16><<<grid_for(n, T), T, 0, s>>>(static_cast<const float*>(blocks), n, out);
      break;
    default:
      return cudaErrorNotSupported;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_dequant_f32(int type, const void* blocks, int64_t n, float* out, cudaStream_t s) {
  return dequant_impl<false>(type, blocks, n, out, s);
}

cudaError_t launch_dequant_bf16(int type, const void* blocks, int64_t n, uint16_t* out, cudaStream_t s) {
  return dequant_impl<true>(type, blocks, n, out, s);
}

// ------------------------------------------------------------------ packing
// The fused-dequant GEMM reads a quantised weight [N, K] as stages of 256
// rows x 64 K, each one contiguous block so that one bulk TMA copy brings it:
//   Q4_K stage (10240 B): [256 x 32 B nibbles][256 x (s0, m0, s1, m1) bf16]
//       the 32 nibble bytes are the GGUF block's qs[32 g .. 32 g + 31] for
//       the stage's 64-wide group g (low nibble: sub-block 2g, high: 2g+1);
//       s_j = d * sc_j and m_j = dmin * m_j are exact in f32, rounded once
//       to bf16.
//   Q8_0 stage (17408 B): [256 x 64 int8][256 x (d0, d1) bf16] for the
//       stage's two 32-weight blocks.
// Stage (n_tile, kb) starts at (n_tile * K/64 + kb) * stage bytes; rows
// beyond N are zero.

namespace {

__device__ __forceinline__ uint16_t bf16_bits(float v) {
  __nv_bfloat16 b = __float2bfloat16_rn(v);
  return *reinterpret_cast<uint16_t*>(&b);
}

template <int kType>
__global__ void pack_weight_kernel(const uint8_t* __restrict__ raw, int64_t N, int64_t K, uint8_t* __restrict__ out,
                                   int64_t total) {
  const int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (t >= total) return;
  constexpr int kQs = kType == kTypeQ4_K ? 32 : 64;
  constexpr int kSc = kType == kTypeQ4_K ? 8 : 4;
  constexpr int kStage = 256 * (kQs + kSc);
  const int64_t nkb = K / 64;
  const int r = static_cast<int>(t & 255);
  const int64_t stage = t >> 8;  // n_tile * nkb + kb
  const int64_t kb = stage % nkb;
  const int64_t n = (stage / nkb) * 256 + r;
  uint8_t* qs_out = out + stage * kStage + r * kQs;
  uint8_t* sc_out = out + stage * kStage + 256 * kQs + r * kSc;
  if (n >= N) {
    for (int i = 0; i < kQs; i += 16) *reinterpret_cast<uint4*>(qs_out + i) = make_uint4(0, 0, 0, 0);
    if (kSc == 8) *reinterpret_cast<uint2*>(sc_out) = make_uint2(0, 0);
    else *reinterpret_cast<uint32_t*>(sc_out) = 0;
    return;
  }
  if (kType == kTypeQ4_K) {
    const uint8_t* blk = raw + n * (K / 256) * 144 + (kb >> 2) * 144;
    const int g = static_cast<int>(kb & 3);
    const float d = half_bits_to_f32(static_cast<uint16_t>(blk[0] | (blk[1] << 8)));
    const float dmin = half_bits_to_f32(static_cast<uint16_t>(blk[2] | (blk[3] << 8)));
    int sc0, m0, sc1, m1;
    q4k_scale_min(blk + 4, 2 * g, sc0, m0);
    q4k_scale_min(blk + 4, 2 * g + 1, sc1, m1);
    const uint16_t v[4] = {bf16_bits(__fmul_rn(d, static_cast<float>(sc0))),
                           bf16_bits(__fmul_rn(dmin, static_cast<float>(m0))),
                           bf16_bits(__fmul_rn(d, static_cast<float>(sc1))),
                           bf16_bits(__fmul_rn(dmin, static_cast<float>(m1)))};
    *reinterpret_cast<uint2*>(sc_out) =
        make_uint2(v[0] | (static_cast<uint32_t>(v[1]) << 16), v[2] | (static_cast<uint32_t>(v[3]) << 16));
    const uint4* q = reinterpret_cast<const uint4*>(blk + 16 + g * 32);
    reinterpret_cast<uint4*>(qs_out)[0] = q[0];
    reinterpret_cast<uint4*>(qs_out)[1] = q[1];
  } else {
    const uint8_t* b0 = raw + n * (K / 32) * 34 + (2 * kb) * 34;
    const uint8_t* b1 = b0 + 34;
    const float d0 = half_bits_to_f32(static_cast<uint16_t>(b0[0] | (b0[1] << 8)));
    const float d1 = half_bits_to_f32(static_cast<uint16_t>(b1[0] | (b1[1] << 8)));
    *reinterpret_cast<uint32_t*>(sc_out) = bf16_bits(d0) | (static_cast<uint32_t>(bf16_bits(d1)) << 16);
    // 2 blocks x 32 int8 = 16 words (the blocks are only 2-byte aligned).
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint8_t* s = i < 8 ? b0 + 2 + 4 * i : b1 + 2 + 4 * (i - 8);
      w[i] = s[0] | (s[1] << 8) | (s[2] << 16) | (static_cast<uint32_t>(s[3]) << 24);
    }
    uint4* o = reinterpret_cast<uint4*>(qs_out);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  }
}

}  // namespace

int packed_stage_bytes(int type) {
  if (type == kTypeQ4_K) return 256 * (32 + 8);
  if (type == kTypeQ8_0) return 256 * (64 + 4);
  return 0;
}

size_t packed_bytes(int type, int64_t N, int64_t K) {
  const int sb = packed_stage_bytes(type);
  if (!sb || K % 64) return 0;
  return static_cast<size_t>((N + 255) / 256) * static_cast<size_t>(K / 64) * static_cast<size_t>(sb);
}

cudaError_t launch_pack_weight(int type, const void* raw, int64_t N, int64_t K, void* out, cudaStream_t s) {
  if (N <= 0 || K <= 0) return cudaSuccess;
  if ((type == kTypeQ4_K && K % 256) || (type == kTypeQ8_0 && K % 64)) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(out) & 15) return cudaErrorMisalignedAddress;
  if (type == kTypeQ4_K && (reinterpret_cast<uintptr_t>(raw) & 15)) return cudaErrorMisalignedAddress;
  const int64_t total = (N + 255) / 256 * 256 * (K / 64);
  const unsigned grid = static_cast<unsigned>((total + 255) / 256);
  if (type == kTypeQ4_K)
    pack_weight_kernel<kTypeQ4_K><<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(raw), N, K,
                                                       static_cast<uint8_t*>(out), total);
  else if (type == kTypeQ8_0)
    pack_weight_kernel<kTypeQ8_0><<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(raw), N, K,
                                                       static_cast<uint8_t*>(out), total);
  else
    return cudaErrorNotSupported;
  return cudaGetLastError();
}

}  // namespace dcpp
