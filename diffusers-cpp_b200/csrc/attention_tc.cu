// Joint attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
//   O = softmax(Q K^T * scale) V, no mask (FlashAttentionOp.cpp:6-105,
//   ggml_flash_attn_ext(q, k, v, nullptr, 1/sqrt(128)))
//
// Layouts (bf16): Q, K [B*H, S, 128] (row per token), V^T [B*H, 128, Sp]
// (row per head-dim channel, Sp = S rounded up to 64, zero padded), so every
// shared-memory operand is K-major and arrives through TMA with the 128-byte
// swizzle.
//
// Two kernels share the softmax code: the one-tile kernel below and a
// two-tile kernel (further down) whose two query tiles ping-pong between the
// tensor core and the softmax warps; launch_attention_tc picks by how many
// waves of 148 SMs each needs.
//
// One-tile kernel: one CTA = one 128-row query tile of one (batch, head); 192 threads:
//   warp 0     TMA: Q once, then K_j / V_j^T tiles of 128 keys (3 stages)
//   warp 1     TMEM allocation and the single MMA-issuing thread:
//                S_j = Q K_j^T   (M 128, N 128 keys, K 128) -> TMEM buffer j % 3
//                O  += P_j V_j   (A = P_j read from TMEM, B = V_j^T from smem)
//              Order S_0, S_1, PV_0, S_2, PV_1, ...: the scores of the next
//              tiles are computed while the softmax runs.
//   warps 2-5  softmax, one thread per query row (its TMEM lane): online
//              softmax in the exp2 domain; P_j (bf16) is written back over
//              its own S_j in TMEM (no shared memory, no proxy fence); O is
//              rescaled in TMEM only when a row maximum grows by more than
//              2^8 (otherwise the stale maximum is kept, which is exact
//              because l uses the same one).  At the end they normalise O
//              by l and store bf16 rows.
// TMEM: S/P buffers at columns 0, 128, 256 and O at 384 (512 allocated).
#include "attention_tc.cuh"
#include "common.cuh"

namespace dcpp {

namespace {

constexpr int kBQ = 128;                    // query rows per CTA
constexpr int kBKV = 128;                   // keys per tile
constexpr int kKVStages = 3;
constexpr int kSBufs = 3;
constexpr int kHalfBytes = 128 * 128;       // one 64-wide swizzle-atom column block of 128 rows: 16 KB
constexpr int kTileBytes = 2 * kHalfBytes;  // 128 x 128 bf16 = 32 KB
constexpr int kThreads = 192;
constexpr int kTmemCols = 512;
constexpr int kOCol = 384;
constexpr int kSmemBytes = (1 + 2 * kKVStages) * kTileBytes + 1024 + 256;  // Q, (K, V) x 3 + barriers
constexpr float kRescaleThreshold = 8.0f;   // log2 units

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// O (+)= A[tmem] * B[smem desc]^T, A (M x K bf16) read from TMEM.
__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed f32x2 arithmetic (two lanes of a 64-bit register per instruction).
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f2lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x of a pair on the FMA / integer pipes, for a share of the softmax exponentials
// (the MUFU unit alone would limit the softmax: one ex2 per 512 tensor
// FLOPs is exactly its throughput).  Range reduction x = n + f with
// n = round(x) (the 1.5 * 2^23 rounding trick), f in [-1/2, 1/2]; 2^f by a
// degree-3 polynomial fitted here to minimise the maximum relative error on
// that interval (7.5e-5, far below the bf16 rounding P gets next); 2^n is
// added to the exponent field.  x is clamped to -126 (masked keys give
// ~2^-126 instead of 0, which vanishes in bf16 sums of O(1) terms).
__device__ __forceinline__ uint64_t ex2_poly2(uint64_t x) {
  x = f2(fmaxf(f2lo(x), -126.0f), fmaxf(f2hi(x), -126.0f));
  const uint64_t magic = f2(12582912.0f, 12582912.0f), neg_magic = f2(-12582912.0f, -12582912.0f);
  const uint64_t t = add2(x, magic);
  const uint64_t n = add2(t, neg_magic);
  const uint64_t f = fma2(n, f2(-1.0f, -1.0f), x);
  uint64_t p = fma2(f2(0.0551716648f, 0.0551716648f), f, f2(0.24261114f, 0.24261114f));
  p = fma2(p, f, f2(0.693260968f, 0.693260968f));
  p = fma2(p, f, f2(0.999928057f, 0.999928057f));
  const uint32_t lo = static_cast<uint32_t>(p) + ((static_cast<uint32_t>(t) - 0x4B400000u) << 23);
  const uint32_t hi = static_cast<uint32_t>(p >> 32) + ((static_cast<uint32_t>(t >> 32) - 0x4B400000u) << 23);
  return (static_cast<uint64_t>(hi) << 32) | lo;
}

// Key padding mask of a 128-key tile: four 32-bit words per batch row.
__device__ __forceinline__ void apply_key_bits(const AttnTcArgs& p, int b, int kbase, float (&s)[128]) {
  const uint32_t* w = p.key_bits + static_cast<int64_t>(b) * p.key_words + (kbase >> 5);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t bits = ((kbase >> 5) + q < p.key_words) ? __ldg(w + q) : 0u;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (!((bits >> i) & 1u)) s[q * 32 + i] = -INFINITY;
  }
}

// Softmax numerators of one row's n scores (n % 8 == 0) against the running
// maximum: row max with three-input max in 8 chains, then for each pair
// x = s * c - m (packed FMA), 2^x on MUFU (three pairs in four) or the FMA
// pipe (the fourth), packed partial sums, bf16x2 packing of P.  Returns the
// new maximum in m_use (lazy: kept unless the tile's maximum exceeds it by
// more than the threshold), the row sum of the numerators in *sum.
template <int n>
__device__ __forceinline__ void softmax_tile(const float (&s)[n], float c, float m, float& m_use, float& alpha,
                                             bool& grow, float& sum, uint32_t (&pk)[n / 2]) {
  float mp[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) mp[k] = s[k];
#pragma unroll
  for (int i = 8; i < n; i += 2) mp[(i >> 1) & 7] = max3(mp[(i >> 1) & 7], s[i], s[i + 1]);
  const float mx = c * max3(max3(mp[0], mp[1], mp[2]), max3(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
  grow = mx > m + kRescaleThreshold;
  m_use = grow ? mx : m;
  alpha = grow ? ex2(m - m_use) : 1.0f;
  const uint64_t c2 = f2(c, c), nm2 = f2(-m_use, -m_use);
  uint64_t sp[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < n / 2; ++i) {
    const uint64_t x = fma2(f2(s[2 * i], s[2 * i + 1]), c2, nm2);
    const uint64_t e = (i & 3) == 3 ? ex2_poly2(x) : f2(ex2(f2lo(x)), ex2(f2hi(x)));
    sp[i & 3] = add2(sp[i & 3], e);
    pk[i] = pack_bf16x2(f2lo(e), f2hi(e));
  }
  const uint64_t t = add2(add2(sp[0], sp[1]), add2(sp[2], sp[3]));
  sum = f2lo(t) + f2hi(t);
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ AttnTcArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kTileBytes;                      // kKVStages stages
  uint8_t* sV = smem + (1 + kKVStages) * kTileBytes;    // kKVStages stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (1 + 2 * kKVStages) * kTileBytes);
  uint64_t* q_full = bars;                     // Q landed
  uint64_t* kv_full = bars + 1;                // [3] K_j, V_j landed
  uint64_t* kv_empty = kv_full + kKVStages;    // [3] PV_j done with the stage
  uint64_t* s_full = kv_empty + kKVStages;     // [3] S_j computed in buffer j % 3
  uint64_t* s_free = s_full + kSBufs;          // [3] PV_j read P_j: buffer free
  uint64_t* p_full = s_free + kSBufs;          // P_j written, O rescaled (128 arrivals)
  uint64_t* o_done = p_full + 1;               // PV_j done: O current
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = blockIdx.x;
  const int bh = blockIdx.y;  // b * H + h
  const int S = p.S;
  const int hkv = p.H_kv > 0 ? p.H_kv : p.H;
  const int bhkv = (bh / p.H) * hkv + (bh % p.H) / (p.H / hkv);  // K / V head of this query head
  // Causal: query tile qt sees key tiles 0..qt (kBQ == kBKV).
  const int nkv = p.causal ? min((S + kBKV - 1) / kBKV, qt + 1) : (S + kBKV - 1) / kBKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kKVStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < kSBufs; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 1);
    }
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_3d(sQ, &tmQ, q_full, 0, qt * kBQ, bh);
      tma_load_3d(sQ + kHalfBytes, &tmQ, q_full, 64, qt * kBQ, bh);
      for (int j = 0; j < nkv; ++j) {
        const int st = j % kKVStages;
        if (!mbar_wait(&kv_empty[st], ((j / kKVStages) & 1) ^ 1, p.err, kDevTimeoutAttn)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kTileBytes);
        uint8_t* k = sK + st * kTileBytes;
        uint8_t* v = sV + st * kTileBytes;
        tma_load_3d(k, &tmK, &kv_full[st], 0, j * kBKV, bhkv);
        tma_load_3d(k + kHalfBytes, &tmK, &kv_full[st], 64, j * kBKV, bhkv);
        tma_load_3d(v, &tmV, &kv_full[st], j * kBKV, 0, bhkv);
        tma_load_3d(v + kHalfBytes, &tmV, &kv_full[st], j * kBKV + 64, 0, bhkv);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(128, 128);
      const uint32_t tO = tmem_base + kOCol;
      const uint32_t aQ = smem_u32(sQ);
      // S_j = Q K_j^T into buffer j % 3.
      auto issue_s = [&](int j) -> bool {
        const int st = j % kKVStages;
        const int b = j % kSBufs;
        if (!mbar_wait(&kv_full[st], (j / kKVStages) & 1, p.err, kDevTimeoutAttn)) return false;
        if (!mbar_wait(&s_free[b], ((j / kSBufs) & 1) ^ 1, p.err, kDevTimeoutAttn)) return false;
        tc_fence_after();
        const uint32_t aK = smem_u32(sK + st * kTileBytes);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * kHalfBytes + (k & 3) * 32;
          umma_bf16(tmem_base + b * 128, make_sdesc_sw128(aQ + off), make_sdesc_sw128(aK + off), idesc,
                    k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[b]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, p.err, kDevTimeoutAttn);
      if (ok) ok = issue_s(0);
      if (ok && nkv > 1) ok = issue_s(1);
      for (int j = 0; j < nkv && ok; ++j) {
        if (!mbar_wait(p_full, j & 1, p.err, kDevTimeoutAttn)) break;
        tc_fence_after();
        const int st = j % kKVStages;
        const int b = j % kSBufs;
        const uint32_t aV = smem_u32(sV + st * kTileBytes);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          // A = P_j: 16 keys = 8 packed bf16x2 TMEM columns per MMA.
          const uint32_t off = (k >> 2) * kHalfBytes + (k & 3) * 32;
          umma_bf16_ts(tO, tmem_base + b * 128 + k * 8, make_sdesc_sw128(aV + off), idesc,
                       (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&s_free[b]);
        umma_commit(&kv_empty[st]);
        umma_commit(o_done);
        if (j + 2 < nkv) ok = issue_s(j + 2);
      }
    }
  } else {
    // Softmax warps 2..5 -> TMEM lane quarter (warp % 4); thread = query row.
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tO = tmem_base + lane_off + kOCol;
    const float c = p.scale * 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int b = j % kSBufs;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[b], (j / kSBufs) & 1, p.err, kDevTimeoutAttn));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tS = tmem_base + lane_off + b * 128;
      uint32_t r0[32], r1[32], r2[32], r3[32];
      tmem_ld32(tS, r0);
      tmem_ld32(tS + 32, r1);
      tmem_ld32(tS + 64, r2);
      tmem_ld32(tS + 96, r3);
      tmem_ld_wait();
      float s[128];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        s[i] = __uint_as_float(r0[i]);
        s[32 + i] = __uint_as_float(r1[i]);
        s[64 + i] = __uint_as_float(r2[i]);
        s[96 + i] = __uint_as_float(r3[i]);
      }
      const int kbase = j * kBKV;
      if (kbase + kBKV > S) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (kbase + i >= S) s[i] = -INFINITY;
      }
      if (p.causal && j == nkv - 1) {  // the diagonal tile
        const int qrow = qt * kBQ + row;
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (kbase + i > qrow) s[i] = -INFINITY;
      }
      if (p.key_bits) apply_key_bits(p, bh / p.H, kbase, s);
      float m_use, alpha, sum;
      bool grow;
      uint32_t pk[64];
      softmax_tile<128>(s, c, m, m_use, alpha, grow, sum, pk);
      l = l * alpha + sum;
      m = m_use;
      if (j > 0) {
        // PV_{j-1} done: O is current (and buffer (j-1) % 3 is being recycled).
        ok = __all_sync(0xffffffffu, mbar_wait(o_done, (j - 1) & 1, p.err, kDevTimeoutAttn));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll 1
          for (int ch = 0; ch < 4; ++ch) {
            uint32_t r[32];
            tmem_ld32(tO + ch * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(tO + ch * 32, r);
          }
        }
      }
      // P_j (bf16, two keys per column) over the first 64 columns of S_j.
      tmem_st32(tS, pk);
      tmem_st32(tS + 32, pk + 32);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(o_done, (nkv - 1) & 1, p.err, kDevTimeoutAttn));
    if (ok) {
      tc_fence_after();
      const int q = qt * kBQ + row;
      const float inv = 1.0f / l;
      uint16_t* dst = p.o + (static_cast<int64_t>(bh / p.H) * S + q) * p.ld_o + (bh % p.H) * 128;
      uint32_t r0[32], r1[32], r2[32], r3[32];
      tmem_ld32(tO, r0);
      tmem_ld32(tO + 32, r1);
      tmem_ld32(tO + 64, r2);
      tmem_ld32(tO + 96, r3);
      tmem_ld_wait();
      if (q < S) {
        const uint32_t* rs[4] = {r0, r1, r2, r3};
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + ch * 32);
          const uint32_t* r = rs[ch];
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            d4[v] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * v]) * inv, __uint_as_float(r[8 * v + 1]) * inv),
                               pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv),
                               pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv),
                               pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv));
          }
        }
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

// ---------------------------------------------------------------------------
// Two-tile variant: one CTA = two 128-row query tiles (A, B) of one (batch,
// head), 128-key K / V tiles, 320 threads:
//   warp 0      TMA: Q_A, Q_B once, then K_j and V_j^T into a 2-stage ring
//   warp 1      TMEM allocation and the MMAs (the warp runs the loop with
//               descriptors built once; one elected lane issues); order
//                 S_A0 S_B0 | PV_A0 S_A1 PV_B0 S_B1 | PV_A1 S_A2 PV_B1 S_B2 ...
//               so that while one tile's softmax runs, the tensor core
//               computes the other tile's P.V and next scores
//   warps 2-5   softmax of tile A, warps 6-9 softmax of tile B (one thread
//               per query row), as in the one-tile kernel; two softmax warps
//               per SM sub-partition hide each other's latencies.
// TMEM (512 columns): S_A / P_A at 0, S_B / P_B at 128, O_A at 256, O_B at
// 384.  S_X(j+1) overwrites S_X only after PV_X(j) (which reads P_X(j) from
// it) has completed.  The warps that mostly wait (TMA, MMA) sleep in their
// barrier waits, leaving issue slots to the softmax warps beside them.
constexpr int k2Tiles = 2;
constexpr int k2Stages = 2;
constexpr int k2Threads = 320;
constexpr int k2SmemBytes = (k2Tiles + 2 * k2Stages) * kTileBytes + 1024 + 256;

__global__ void __launch_bounds__(k2Threads, 1)
    attn_tc2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ AttnTcArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                    // Q_A | Q_B
  uint8_t* sK = smem + k2Tiles * kTileBytes;             // k2Stages x 32 KB
  uint8_t* sV = sK + k2Stages * kTileBytes;              // k2Stages x 32 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + k2Stages * kTileBytes);
  uint64_t* q_full = bars;                               // Q_A and Q_B landed
  uint64_t* kv_full = q_full + 1;                        // [2]
  uint64_t* kv_empty = kv_full + k2Stages;               // [2]
  uint64_t* s_full = kv_empty + k2Stages;                // [tile]
  uint64_t* p_full = s_full + 2;                         // [tile], 128 arrivals
  uint64_t* pv_done = p_full + 2;                        // [tile]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * (k2Tiles * kBQ);
  const int bh = blockIdx.y;
  const int S = p.S;
  const int hkv = p.H_kv > 0 ? p.H_kv : p.H;
  const int bhkv = (bh / p.H) * hkv + (bh % p.H) / (p.H / hkv);
  // Causal: the CTA's query tiles 2 qt2 and 2 qt2 + 1 see key tiles up to 2 qt2 + 1.
  const int nkv = p.causal ? min((S + kBKV - 1) / kBKV, static_cast<int>(blockIdx.x) * 2 + 2) : (S + kBKV - 1) / kBKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < k2Stages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 128);
      mbar_init(&pv_done[x], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, k2Tiles * kTileBytes);
      for (int x = 0; x < k2Tiles; ++x) {
        tma_load_3d(sQ + x * kTileBytes, &tmQ, q_full, 0, q0 + x * kBQ, bh);
        tma_load_3d(sQ + x * kTileBytes + kHalfBytes, &tmQ, q_full, 64, q0 + x * kBQ, bh);
      }
      for (int j = 0; j < nkv; ++j) {
        const int st = j % k2Stages;
        if (!mbar_wait_sleep(&kv_empty[st], ((j / k2Stages) & 1) ^ 1, p.err, kDevTimeoutAttn)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kTileBytes);
        uint8_t* k = sK + st * kTileBytes;
        uint8_t* v = sV + st * kTileBytes;
        tma_load_3d(k, &tmK, &kv_full[st], 0, j * kBKV, bhkv);
        tma_load_3d(k + kHalfBytes, &tmK, &kv_full[st], 64, j * kBKV, bhkv);
        tma_load_3d(v, &tmV, &kv_full[st], j * kBKV, 0, bhkv);
        tma_load_3d(v + kHalfBytes, &tmV, &kv_full[st], j * kBKV + 64, 0, bhkv);
      }
    }
  } else if (warp == 1) {
    // The whole warp runs the loop (waits, descriptors: warp-uniform); one
    // elected lane issues the MMAs and their commits.
    constexpr uint32_t idesc = make_idesc_bf16(128, 128);
    const uint64_t dQ = make_sdesc_sw128(smem_u32(sQ));
    const uint64_t dK = make_sdesc_sw128(smem_u32(sK));
    const uint64_t dV = make_sdesc_sw128(smem_u32(sV));
    auto koff = [](int k) -> uint64_t { return static_cast<uint64_t>(((k >> 2) * kHalfBytes + (k & 3) * 32) >> 4); };
    constexpr uint64_t kTileD = kTileBytes >> 4;
    const bool leader = elect_one_sync();
    auto issue_s = [&](int x, int j) -> bool {
      const int st = j % k2Stages;
      if (!__all_sync(0xffffffffu, mbar_wait_sleep(&kv_full[st], (j / k2Stages) & 1, p.err, kDevTimeoutAttn))) return false;
      tc_fence_after();
      const uint64_t q = dQ + x * kTileD, kd = dK + st * kTileD;
      const uint32_t tS = tmem_base + x * 128;
      if (leader) {
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16(tS, q + koff(k), kd + koff(k), idesc, k > 0 ? 1u : 0u);
        umma_commit(&s_full[x]);
      }
      __syncwarp();
      return true;
    };
    bool ok = __all_sync(0xffffffffu, mbar_wait_sleep(q_full, 0, p.err, kDevTimeoutAttn));
    for (int x = 0; x < k2Tiles && ok; ++x) ok = issue_s(x, 0);
    for (int j = 0; j < nkv && ok; ++j) {
      const int st = j % k2Stages;
      const uint64_t vd = dV + st * kTileD;
      for (int x = 0; x < k2Tiles && ok; ++x) {
        if (!__all_sync(0xffffffffu, mbar_wait_sleep(&p_full[x], j & 1, p.err, kDevTimeoutAttn))) { ok = false; break; }
        tc_fence_after();
        const uint32_t tO = tmem_base + 256 + x * 128, tP = tmem_base + x * 128;
        if (leader) {
          umma_bf16_ts(tO, tP, vd, idesc, j > 0 ? 1u : 0u);
#pragma unroll
          for (int k = 1; k < 8; ++k) umma_bf16_ts(tO, tP + k * 8, vd + koff(k), idesc, 1u);
          umma_commit(&pv_done[x]);
          if (x == k2Tiles - 1) umma_commit(&kv_empty[st]);
        }
        __syncwarp();
        if (j + 1 < nkv) {
          if (!__all_sync(0xffffffffu, mbar_wait_sleep(&pv_done[x], j & 1, p.err, kDevTimeoutAttn))) { ok = false; break; }
          ok = issue_s(x, j + 1);
        }
      }
    }
  } else {
    // Softmax: warps 2-5 tile A, 6-9 tile B; TMEM lane quarter = warp % 4.
    const int x = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + x * 128;
    const uint32_t tO = tmem_base + lane_off + 256 + x * 128;
    const float c = p.scale * 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait_sleep(&s_full[x], j & 1, p.err, kDevTimeoutAttn));
      if (!ok) break;
      tc_fence_after();
      uint32_t r0[32], r1[32], r2[32], r3[32];
      tmem_ld32(tS, r0);
      tmem_ld32(tS + 32, r1);
      tmem_ld32(tS + 64, r2);
      tmem_ld32(tS + 96, r3);
      tmem_ld_wait();
      float sv[128];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        sv[i] = __uint_as_float(r0[i]);
        sv[32 + i] = __uint_as_float(r1[i]);
        sv[64 + i] = __uint_as_float(r2[i]);
        sv[96 + i] = __uint_as_float(r3[i]);
      }
      const int kbase = j * kBKV;
      if (kbase + kBKV > S) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (kbase + i >= S) sv[i] = -INFINITY;
      }
      if (p.causal && kbase + kBKV - 1 > q0 + x * kBQ) {  // tiles reaching past this tile's first query
        const int qrow = q0 + x * kBQ + row;
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (kbase + i > qrow) sv[i] = -INFINITY;
      }
      if (p.key_bits) apply_key_bits(p, bh / p.H, kbase, sv);
      float m_use, alpha, sum;
      bool grow;
      uint32_t pk[64];
      softmax_tile<128>(sv, c, m, m_use, alpha, grow, sum, pk);
      l = l * alpha + sum;
      m = m_use;
      if (j > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait_sleep(&pv_done[x], (j - 1) & 1, p.err, kDevTimeoutAttn));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll 1
          for (int ch = 0; ch < 4; ++ch) {
            uint32_t r[32];
            tmem_ld32(tO + ch * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(tO + ch * 32, r);
          }
        }
      }
      tmem_st32(tS, pk);
      tmem_st32(tS + 32, pk + 32);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[x]);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait_sleep(&pv_done[x], (nkv - 1) & 1, p.err, kDevTimeoutAttn));
    if (ok) {
      tc_fence_after();
      const int q = q0 + x * kBQ + row;
      const float inv = 1.0f / l;
      uint32_t r0[32], r1[32], r2[32], r3[32];
      tmem_ld32(tO, r0);
      tmem_ld32(tO + 32, r1);
      tmem_ld32(tO + 64, r2);
      tmem_ld32(tO + 96, r3);
      tmem_ld_wait();
      if (q < S) {
        uint16_t* dst = p.o + (static_cast<int64_t>(bh / p.H) * S + q) * p.ld_o + (bh % p.H) * 128;
        const uint32_t* rs[4] = {r0, r1, r2, r3};
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + ch * 32);
          const uint32_t* r = rs[ch];
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            d4[v] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * v]) * inv, __uint_as_float(r[8 * v + 1]) * inv),
                               pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv),
                               pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv),
                               pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv));
          }
        }
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

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) == cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(q);
  }
  return fn;
}

// 3-D bf16 map {inner, mid, outer} with box {64, box_mid, 1}, 128-byte swizzle.
cudaError_t make_map3(CUtensorMap* m, const void* base, uint64_t inner, uint64_t mid, uint64_t outer,
                      uint32_t box_mid = 128) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (inner * 2) % 16) return cudaErrorMisalignedAddress;
  cuuint64_t dims[3] = {inner, mid, outer};
  cuuint64_t strides[2] = {inner * 2, inner * mid * 2};
  cuuint32_t box[3] = {64, box_mid, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

int64_t attn_vt_stride(int64_t S) { return (S + 63) / 64 * 64; }

cudaError_t make_attn_maps(AttnTcMaps* maps, const uint16_t* q, const uint16_t* k, const uint16_t* vt, int B, int H,
                           int S, int H_kv) {
  const uint64_t bh = static_cast<uint64_t>(B) * H;
  const uint64_t bhkv = static_cast<uint64_t>(B) * (H_kv > 0 ? H_kv : H);
  cudaError_t e = make_map3(&maps->q, q, 128, S, bh);
  if (e == cudaSuccess) e = make_map3(&maps->k, k, 128, S, bhkv);
  if (e == cudaSuccess) e = make_map3(&maps->v, vt, attn_vt_stride(S), 128, bhkv);
  if (e == cudaSuccess) e = make_map3(&maps->k64, k, 128, S, bhkv, 64);
  return e;
}

int attention_kernel_for(int B, int H, int S, int requested) {
  if (requested == 1 || requested == 2) return requested;
  // The two-tile kernel does a CTA's two tiles in ~1.55x the time the
  // one-tile kernel takes for one (measured per SM clock at S 4608, 24
  // heads: 29% more work per clock).  Compare whole waves of 148 SMs.
  const int64_t bh = static_cast<int64_t>(B) * H;
  const int64_t c1 = (S + 127) / 128 * bh, c2 = (S + 255) / 256 * bh;
  const double t1 = static_cast<double>((c1 + 147) / 148), t2 = 1.55 * static_cast<double>((c2 + 147) / 148);
  return t2 < t1 ? 2 : 1;
}

cudaError_t launch_attention_tc(const AttnTcMaps& maps, const AttnTcArgs& a, cudaStream_t s) {
  if (a.S <= 0 || a.H <= 0 || a.B <= 0) return cudaSuccess;
  if (a.ld_o % 8 || (reinterpret_cast<uintptr_t>(a.o) & 15)) return cudaErrorInvalidValue;
  if (a.H_kv < 0 || (a.H_kv > 0 && a.H % a.H_kv)) return cudaErrorInvalidValue;
  if (attention_kernel_for(a.B, a.H, a.S, a.kernel) == 2) {
    static bool attr2 = false;
    if (!attr2) {
      cudaError_t e = cudaFuncSetAttribute(attn_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, k2SmemBytes);
      if (e != cudaSuccess) return e;
      attr2 = true;
    }
    dim3 grid2((a.S + 255) / 256, a.B * a.H);
    attn_tc2_kernel<<<grid2, k2Threads, k2SmemBytes, s>>>(maps.q, maps.k, maps.v, a);
    return cudaGetLastError();
  }
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  dim3 grid((a.S + kBQ - 1) / kBQ, a.B * a.H);
  attn_tc_kernel<<<grid, kThreads, kSmemBytes, s>>>(maps.q, maps.k, maps.v, a);
  return cudaGetLastError();
}

}  // namespace dcpp
