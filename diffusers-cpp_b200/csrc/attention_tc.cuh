// tcgen05 joint attention: host-side types and launch entry points.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dcpp {

struct AttnTcArgs {
  uint16_t* o;     // output row (b * S + s), column h * 128 + d
  int64_t ld_o;    // row stride of o (elements, multiple of 8)
  int32_t B, H, S;
  float scale;     // softmax scale
  int* err;        // device error word for bounded waits
  int32_t kernel;  // 0 auto, 1 one query tile per CTA, 2 two query tiles per CTA
  int32_t causal;  // 1: key j attends to query i only if j <= i
  int32_t H_kv;    // key / value heads (grouped-query attention: H % H_kv == 0); 0: = H
  // Optional key padding mask: bit (k % 32) of key_bits[b * key_words + k / 32]
  // set = key k of batch element b is attended; clear = masked (-inf).
  const uint32_t* key_bits;
  int32_t key_words;
};

struct AttnTcMaps {
  CUtensorMap q, k, v;  // boxes of 128 rows
  CUtensorMap k64;      // K with 64-row boxes (two-tile kernel)
};

// Which kernel a launch uses for (B, H, S): 1 or 2 (requested 0 = auto).
int attention_kernel_for(int B, int H, int S, int requested);

// Row stride (keys) of the transposed V buffer [B*H, 128, Sp]: S rounded up to 64.
int64_t attn_vt_stride(int64_t S);

// Tensor maps over q [B*H, S, 128], k [B*H_kv, S, 128] and vt
// [B*H_kv, 128, Sp] (bf16); H_kv = 0 means H.
cudaError_t make_attn_maps(AttnTcMaps* maps, const uint16_t* q, const uint16_t* k, const uint16_t* vt, int B, int H,
                           int S, int H_kv = 0);

cudaError_t launch_attention_tc(const AttnTcMaps& maps, const AttnTcArgs& a, cudaStream_t s);

}  // namespace dcpp
