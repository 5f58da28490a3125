"""TEST INFRASTRUCTURE ONLY -- CPU oracle of the Qwen3 text-encoder prefill.

Only tests/ and bench.py may import this module; the product path
(``diffusers-cpp_b200``) never does.

A PyTorch-CPU restatement (float64 by default) of the reference's Qwen3
prefill, op by op, with ggml op semantics:

* ``Qwen3Model::forward``          src/transformers/models/qwen3/Qwen3Model.cpp:99-208
  (embedding lookup, causal mask ``j <= i`` (:35-97), layers, final norm, the
  hidden states taken before chosen layers (:176-181, :200-205))
* ``Qwen3DecoderLayer::forward``   Qwen3DecoderLayer.cpp:16-49
* ``Qwen3Attention::forward``      Qwen3Attention.inl:36-87 (q/k/v projections,
  per-head RMSNorm on q and k, RoPE, SDPA with scale head_dim^-1/2, o_proj)
* ``Qwen3RotaryEmbedding``         Qwen3RotaryEmbedding.cpp:11-36 (ggml rope NEOX:
  channel d rotates with d + head_dim/2, angle pos * theta^(-2d/head_dim))
* ``Qwen3RMSNorm``                 Qwen3RMSNorm.cpp:8-18 (weight * x * rsqrt(mean(x^2) + eps))
* ``Qwen3MLP``                     Qwen3MLP.cpp:13-25 (down(silu(gate(x)) * up(x)))
* grouped-query attention: query head h uses key / value head h // (H / H_kv)
  (ggml_flash_attn_ext broadcasting the kv heads)

Weights are dequantised with the C oracle (``oracle/dequant.c``, pinned to
gguf-py).  Parity: the restatement is pinned against HF transformers'
Qwen3Model (the library the reference's own Qwen3 tests compare with,
test/src/transformers/models/qwen3/Qwen3Model.py) by the committed fixture
tests/golden/qwen3_golden.npz (tests/golden/make_qwen3_golden.py).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional, Sequence

import numpy as np
import torch

from flux2_oracle import Weights, linear, silu


@dataclass
class Qwen3Config:
    vocab_size: int = 151936
    hidden_size: int = 2560
    intermediate_size: int = 9728
    num_hidden_layers: int = 36
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return w * (x * torch.rsqrt((x * x).mean(dim=-1, keepdim=True) + eps))


def rope_neox(x: torch.Tensor, pos: torch.Tensor, theta: float) -> torch.Tensor:
    """x [B, S, H, d]; rotate (x_i, x_{i + d/2}) by pos * theta^(-2i/d)."""
    d = x.shape[-1]
    half = d // 2
    inv = float(theta) ** (-2.0 * torch.arange(half, dtype=x.dtype) / d)
    ang = pos.to(x.dtype)[:, None] * inv[None, :]
    c, s = torch.cos(ang)[None, :, None, :], torch.sin(ang)[None, :, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def causal_sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                key_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """q [B, S, H, d], k / v [B, S, Hkv, d] -> [B, S, H, d]; key j <= query i,
    and (key_mask [B, S], zero = padding) padding keys masked with -inf (the
    reference's (1 - mask) * -1e9 in an f16 mask, Qwen3Model.cpp:78-94)."""
    B, S, H, d = q.shape
    g = H // k.shape[2]
    mask = torch.triu(torch.ones(S, S, dtype=torch.bool), diagonal=1)[None]
    if key_mask is not None:
        mask = mask | (key_mask == 0)[:, None, :]
    out = torch.empty_like(q)
    for h in range(H):
        qh = q[:, :, h]
        kh, vh = k[:, :, h // g], v[:, :, h // g]
        sc = (qh @ kh.transpose(-1, -2)) * (1.0 / math.sqrt(d))
        sc = sc.masked_fill(mask, float("-inf"))
        out[:, :, h] = torch.softmax(sc, dim=-1) @ vh
    return out


class Qwen3Oracle:
    def __init__(self, cfg: Qwen3Config, params, dtype=torch.float64):
        self.cfg = cfg
        self.w = Weights(params, dtype)
        self.dtype = dtype

    def layer(self, i: int, h: torch.Tensor, pos: torch.Tensor, key_mask=None) -> torch.Tensor:
        c, w = self.cfg, self.w
        p = f"model.layers.{i}."
        B, S, _ = h.shape
        x = rms_norm(h, w.get(p + "input_layernorm.weight"), c.rms_norm_eps)
        q = linear(x, w.get(p + "self_attn.q_proj.weight")).unflatten(-1, (c.num_attention_heads, c.head_dim))
        k = linear(x, w.get(p + "self_attn.k_proj.weight")).unflatten(-1, (c.num_key_value_heads, c.head_dim))
        v = linear(x, w.get(p + "self_attn.v_proj.weight")).unflatten(-1, (c.num_key_value_heads, c.head_dim))
        q = rope_neox(rms_norm(q, w.get(p + "self_attn.q_norm.weight"), c.rms_norm_eps), pos, c.rope_theta)
        k = rope_neox(rms_norm(k, w.get(p + "self_attn.k_norm.weight"), c.rms_norm_eps), pos, c.rope_theta)
        o = causal_sdpa(q, k, v, key_mask).flatten(2)
        h = h + linear(o, w.get(p + "self_attn.o_proj.weight"))
        x = rms_norm(h, w.get(p + "post_attention_layernorm.weight"), c.rms_norm_eps)
        m = silu(linear(x, w.get(p + "mlp.gate_proj.weight"))) * linear(x, w.get(p + "mlp.up_proj.weight"))
        return h + linear(m, w.get(p + "mlp.down_proj.weight"))

    def forward(self, input_ids: torch.Tensor, taps: Sequence[int] = (), n_layers: Optional[int] = None,
                attention_mask: Optional[torch.Tensor] = None):
        """input_ids [B, S] -> (last_hidden [B, S, D], {tap: hidden before layer tap});
        attention_mask [B, S] (zero = padding key) optional.
        n_layers limits the layers run (bounded CPU samples); the final norm
        is then applied to that layer's output."""
        c, w = self.cfg, self.w
        emb = w.get("model.embed_tokens.weight")
        h = emb[input_ids.long()]
        S = input_ids.shape[1]
        pos = torch.arange(S)
        nl = c.num_hidden_layers if n_layers is None else n_layers
        got: Dict[int, torch.Tensor] = {}
        for i in range(nl):
            if i in taps:
                got[i] = h.clone()
            h = self.layer(i, h, pos, attention_mask)
        h = rms_norm(h, w.get("model.norm.weight"), c.rms_norm_eps)
        if nl in taps:
            got[nl] = h.clone()
        return h, got
