"""TEST INFRASTRUCTURE ONLY -- CPU oracle of the Flux2 DiT denoise step.

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py`` (its cpu_baseline
and ``--impl reference`` legs) may import this module; the product path
(``diffusers-cpp_b200``) never does.

A PyTorch-CPU restatement (float64 by default, float32 for the timed CPU
baseline) of the reference's forward, op by op, with ggml op semantics:

* ``Flux2Transformer2DModel::forward``  src/diffusers/models/transformers/flux2/Flux2Transformer2DModel.cpp:111-231
* ``Flux2TransformerBlock::forward``    Flux2TransformerBlock.hpp:45-117
* ``Flux2Attention::forward``           Flux2Attention.hpp:64-159
* ``Flux2SingleTransformerBlock``       Flux2SingleTransformerBlock.hpp:36-72
* ``Flux2ParallelSelfAttention``        Flux2ParallelSelfAttention.hpp:52-101
* ``Flux2FeedForward`` / ``Flux2SwiGLU``  Flux2FeedForward.hpp:52-65, Flux2SwiGLU.hpp:17-21
* ``Flux2Modulation``                   Flux2Modulation.hpp:14-41
* ``Flux2PosEmbed`` (ggml rope NORMAL)  Flux2PosEmbed.hpp:18-109
* ``Timesteps`` / ``TimestepEmbedding``  src/diffusers/models/embeddings/Timesteps.cpp:17-46, TimestepEmbedding.inl:26-44
* ``AdaLayerNormContinuous``            src/diffusers/models/normalization/AdaLayerNormContinuous.inl:26-43
* ``LayerNorm`` / ``RMSNorm`` (ggml_norm / ggml_rms_norm, eps)  src/nn/modules/normalization/*.cpp
* ``FlashAttentionOp`` (softmax(q k^T / sqrt(d)) v, no mask)  src/nn/attention/FlashAttentionOp.cpp:6-105
* Euler ``x + dt * v``                  src/diffusers/schedulers/FlowMatchEulerDiscreteScheduler.cpp:210-222
* fused GGUF tensors split like GGUFLoaderVisitor.cpp:283-429

Weights are dequantised with the C oracle (``oracle/dequant.c``), which is
pinned bit-for-bit against gguf-py 0.19.0 ``gguf.dequantize``.

Parity status: weight dequantisation is pinned (golden fixtures).  The
forward itself is *parity unpinned*: the reference's Flux2 tests compare
against HF diffusers at run time (no golden vectors), diffusers is not
installed here and ggml (the reference's arithmetic) is not vendored, so this
restatement is checked only against the reference's source, line by line.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from dataclasses import dataclass, field
from typing import Dict, Optional, Tuple

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_BF16 = 0, 1, 8, 12, 30
BLOCK = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_BF16: (1, 2), GGML_Q8_0: (32, 34), GGML_Q4_K: (256, 144)}


def _lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            subprocess.check_call(["make", "-s", "-C", _HERE])
        lib = ctypes.CDLL(path)
        lib.oracle_dequant.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        lib.oracle_dequant.restype = ctypes.c_int
        _LIB = lib
    return _LIB


def row_bytes(gtype: int, n: int) -> int:
    bs, bb = BLOCK[gtype]
    assert n % bs == 0
    return n // bs * bb


def dequant(gtype: int, data: np.ndarray, n: int) -> np.ndarray:
    """Dequantise ``n`` weights of ggml type ``gtype`` to float32 (bit-exact)."""
    if hasattr(data, "numpy"):
        data = data.contiguous().cpu().numpy()
    buf = np.ascontiguousarray(np.frombuffer(memoryview(np.ascontiguousarray(data)).cast("B"), dtype=np.uint8))
    assert buf.size == row_bytes(gtype, n), (buf.size, gtype, n)
    out = np.empty(n, dtype=np.float32)
    rc = _lib().oracle_dequant(gtype, buf.ctypes.data, n, out.ctypes.data)
    if rc != 0:
        raise ValueError(f"oracle_dequant failed for type {gtype}")
    return out


@dataclass
class Config:
    """Flux2Transformer2DModel::Config (Flux2Transformer2DModel.hpp:10-31)."""
    patch_size: int = 1
    in_channels: int = 128
    out_channels: Optional[int] = None
    num_layers: int = 8
    num_single_layers: int = 48
    attention_head_dim: int = 128
    num_attention_heads: int = 48
    joint_attention_dim: int = 15360
    timestep_guidance_channels: int = 256
    mlp_ratio: float = 3.0
    axes_dims_rope: Tuple[int, ...] = (32, 32, 32, 32)
    rope_theta: int = 2000
    eps: float = 1e-6
    guidance_embeds: bool = True

    @property
    def inner_dim(self) -> int:
        return self.num_attention_heads * self.attention_head_dim

    @property
    def mlp_hidden(self) -> int:
        return int(self.inner_dim * self.mlp_ratio)

    @property
    def out_ch(self) -> int:
        return self.patch_size * self.patch_size * (self.out_channels or self.in_channels)


class Weights:
    """Resolves GGUF-named raw parameters into float matrices on demand."""

    def __init__(self, params: Dict[str, Tuple[int, Tuple[int, ...], np.ndarray]], dtype=torch.float64,
                 device: str = "cpu"):
        self.params = params
        self.dtype = dtype
        self.device = torch.device(device)
        self.cache: Dict[str, torch.Tensor] = {}

    def get(self, name: str) -> torch.Tensor:
        if name not in self.cache:
            gtype, shape, data = self.params[name]
            n = int(np.prod(shape))
            w = torch.from_numpy(dequant(gtype, data, n).reshape(shape))
            self.cache[name] = w.to(self.device).to(self.dtype)
        return self.cache[name]

    def has(self, name: str) -> bool:
        return name in self.params

    def rows(self, name: str, fused: str, r0: int, r1: int) -> torch.Tensor:
        """`name` if given split, else rows [r0, r1) of the fused tensor (read_rows)."""
        if self.has(name):
            return self.get(name)
        return self.get(fused)[r0:r1]

    def cols(self, name: str, fused: str, c0: int, c1: int) -> torch.Tensor:
        """`name` if given split, else columns [c0, c1) of the fused tensor (read_cols)."""
        if self.has(name):
            return self.get(name)
        return self.get(fused)[:, c0:c1]

    def drop(self, prefix: str):
        for k in [k for k in self.cache if k.startswith(prefix)]:
            del self.cache[k]


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    # ggml_mul_mat(W, x): y = x W^T (Linear.cpp:17-36), no bias in Flux2.
    return x @ w.t()


def silu(x: torch.Tensor) -> torch.Tensor:
    # SiLU.hpp: x * sigmoid(x)
    return x * torch.sigmoid(x)


def layer_norm(x: torch.Tensor, eps: float) -> torch.Tensor:
    # ggml_norm: (x - mean) / sqrt(var + eps), biased variance, no affine.
    mean = x.mean(dim=-1, keepdim=True)
    xc = x - mean
    var = (xc * xc).mean(dim=-1, keepdim=True)
    return xc / torch.sqrt(var + eps)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    # ggml_rms_norm then * weight (RMSNorm.cpp:12-22).
    ms = (x * x).mean(dim=-1, keepdim=True)
    return x / torch.sqrt(ms + eps) * w


def timestep_proj(t: torch.Tensor, channels: int) -> torch.Tensor:
    # Timesteps(channels, flip_sin_to_cos=True, shift=0, scale=1) (Timesteps.cpp:17-46).
    half = channels // 2
    exponent = torch.arange(half, dtype=t.dtype, device=t.device) * (-math.log(10000.0) / half)
    emb = torch.exp(exponent)
    emb = t[:, None] * emb[None, :]
    out = torch.cat([torch.cos(emb), torch.sin(emb)], dim=-1)
    if channels % 2 == 1:
        out = torch.cat([out, torch.zeros(out.shape[0], 1, dtype=out.dtype, device=out.device)], dim=-1)
    return out


def rope_cos_sin(ids: torch.Tensor, axes_dims, theta: float, dtype) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-token cos/sin of every rotary pair: section a (axes_dims[a] dims)
    rotates pair p by pos_a * theta^(-2p/axes_dims[a]) (ggml rope NORMAL,
    Flux2PosEmbed.hpp:18-109)."""
    cs, sn = [], []
    for a, nd in enumerate(axes_dims):
        p = torch.arange(nd // 2, dtype=dtype, device=ids.device)
        freq = float(theta) ** (-2.0 * p / nd)
        ang = ids[:, a].to(dtype)[:, None] * freq[None, :]
        cs.append(torch.cos(ang))
        sn.append(torch.sin(ang))
    return torch.cat(cs, dim=-1), torch.cat(sn, dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, S, H, d]; rotate adjacent pairs (x_2i, x_2i+1)."""
    x0 = x[..., 0::2]
    x1 = x[..., 1::2]
    c = cos[None, :, None, :]
    s = sin[None, :, None, :]
    y0 = x0 * c - x1 * s
    y1 = x0 * s + x1 * c
    return torch.stack([y0, y1], dim=-1).flatten(-2)


def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """q, k, v [B, S, H, d] -> [B, S, H, d]; softmax(q k^T / sqrt(d)) v."""
    d = q.shape[-1]
    qh, kh, vh = (t.transpose(1, 2) for t in (q, k, v))
    out = []
    for h in range(qh.shape[1]):  # per head keeps peak memory at S^2
        s = (qh[:, h] @ kh[:, h].transpose(-1, -2)) * (1.0 / math.sqrt(d))
        p = torch.softmax(s, dim=-1)
        out.append(p @ vh[:, h])
    return torch.stack(out, dim=1).transpose(1, 2)


def _heads(x: torch.Tensor, H: int) -> torch.Tensor:
    return x.unflatten(-1, (H, -1))


class Flux2Oracle:
    """``device``: where the float arithmetic runs.  The default is the CPU;
    the real-width parity tests run the same float64 restatement on a GPU
    (torch's float64 kernels) only to finish in seconds.  The weights are
    always dequantised by the C oracle on the host first."""

    def __init__(self, cfg: Config, params, dtype=torch.float64, keep_weights: bool = True, device: str = "cpu"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.w = Weights(params, dtype, device)
        self.dtype = dtype
        self.keep = keep_weights

    # -- conditioning --------------------------------------------------------
    def temb(self, timestep: torch.Tensor, guidance: Optional[torch.Tensor]) -> torch.Tensor:
        c, w = self.cfg, self.w
        t = timestep.to(self.device, self.dtype) * 1000.0
        p = "time_guidance_embed."
        e = linear(silu(linear(timestep_proj(t, c.timestep_guidance_channels), w.get(p + "timestep_embedder.linear_1.weight"))),
                   w.get(p + "timestep_embedder.linear_2.weight"))
        if c.guidance_embeds:
            g = guidance.to(self.device, self.dtype) * 1000.0
            e = e + linear(silu(linear(timestep_proj(g, c.timestep_guidance_channels), w.get(p + "guidance_embedder.linear_1.weight"))),
                           w.get(p + "guidance_embedder.linear_2.weight"))
        return e

    # -- blocks --------------------------------------------------------------
    def double_block(self, i: int, hs: torch.Tensor, ehs: torch.Tensor, mod_img, mod_txt, cos, sin):
        c, w = self.cfg, self.w
        D, F, H, eps = c.inner_dim, c.mlp_hidden, c.num_attention_heads, c.eps
        p = f"transformer_blocks.{i}."
        sh, sc, g, sh2, sc2, g2 = mod_img[:, None, :].chunk(6, dim=-1)
        csh, csc, cg, csh2, csc2, cg2 = mod_txt[:, None, :].chunk(6, dim=-1)
        n = (1.0 + sc) * layer_norm(hs, eps) + sh
        ne = (1.0 + csc) * layer_norm(ehs, eps) + csh
        q = rms_norm(_heads(linear(n, w.get(p + "attn.to_q.weight")), H), w.get(p + "attn.norm_q.weight"), eps)
        k = rms_norm(_heads(linear(n, w.get(p + "attn.to_k.weight")), H), w.get(p + "attn.norm_k.weight"), eps)
        v = _heads(linear(n, w.get(p + "attn.to_v.weight")), H)
        eq = rms_norm(_heads(linear(ne, w.get(p + "attn.add_q_proj.weight")), H), w.get(p + "attn.norm_added_q.weight"), eps)
        ek = rms_norm(_heads(linear(ne, w.get(p + "attn.add_k_proj.weight")), H), w.get(p + "attn.norm_added_k.weight"), eps)
        ev = _heads(linear(ne, w.get(p + "attn.add_v_proj.weight")), H)
        q = apply_rope(torch.cat([eq, q], dim=1), cos, sin)
        k = apply_rope(torch.cat([ek, k], dim=1), cos, sin)
        vv = torch.cat([ev, v], dim=1)
        o = sdpa(q, k, vv).flatten(2)
        nt = ehs.shape[1]
        o_txt, o_img = o[:, :nt], o[:, nt:]
        o_txt = linear(o_txt, w.get(p + "attn.to_add_out.weight"))
        o_img = linear(o_img, w.get(p + "attn.to_out.0.weight"))
        hs = hs + g * o_img
        n2 = layer_norm(hs, eps) * (1.0 + sc2) + sh2
        hs = hs + g2 * self.ff(p + "ff", n2, F)
        ehs = ehs + cg * o_txt
        ne2 = layer_norm(ehs, eps) * (1.0 + csc2) + csh2
        ehs = ehs + cg2 * self.ff(p + "ff_context", ne2, F)
        if not self.keep:
            w.drop(p)
        return hs, ehs

    def ff(self, prefix: str, x: torch.Tensor, F: int) -> torch.Tensor:
        w = self.w
        gate = linear(x, w.rows(prefix + ".linear_in_gate.weight", prefix + ".linear_in.weight", 0, F))
        up = linear(x, w.rows(prefix + ".linear_in_up.weight", prefix + ".linear_in.weight", F, 2 * F))
        return linear(silu(gate) * up, w.get(prefix + ".linear_out.weight"))

    def single_block(self, i: int, hs: torch.Tensor, mod, cos, sin):
        c, w = self.cfg, self.w
        D, F, H, eps = c.inner_dim, c.mlp_hidden, c.num_attention_heads, c.eps
        p = f"single_transformer_blocks.{i}.attn."
        sh, sc, g = mod[:, None, :].chunk(3, dim=-1)
        n = (1.0 + sc) * layer_norm(hs, eps) + sh
        fq = p + "to_qkv_mlp_proj.weight"
        q = linear(n, w.rows(p + "to_qkv_mlp_proj.q.weight", fq, 0, D))
        k = linear(n, w.rows(p + "to_qkv_mlp_proj.k.weight", fq, D, 2 * D))
        v = linear(n, w.rows(p + "to_qkv_mlp_proj.v.weight", fq, 2 * D, 3 * D))
        gate = linear(n, w.rows(p + "to_qkv_mlp_proj.mlp_in_gate.weight", fq, 3 * D, 3 * D + F))
        up = linear(n, w.rows(p + "to_qkv_mlp_proj.mlp_in_up.weight", fq, 3 * D + F, 3 * D + 2 * F))
        q = apply_rope(rms_norm(_heads(q, H), w.get(p + "norm_q.weight"), eps), cos, sin)
        k = apply_rope(rms_norm(_heads(k, H), w.get(p + "norm_k.weight"), eps), cos, sin)
        o = sdpa(q, k, _heads(v, H)).flatten(2)
        m = silu(gate) * up
        fo = p + "to_out.weight"
        out = linear(o, w.cols(p + "to_out.attn.weight", fo, 0, D)) + linear(m, w.cols(p + "to_out.mlp.weight", fo, D, D + F))
        if not self.keep:
            w.drop(f"single_transformer_blocks.{i}.")
        return hs + g * out

    # -- model ---------------------------------------------------------------
    def forward(self, hidden, encoder, timestep, img_ids, txt_ids, guidance=None,
                n_double: Optional[int] = None, n_single: Optional[int] = None) -> torch.Tensor:
        """Flux2Transformer2DModel::forward.  hidden [B, Ni, in], encoder
        [B, Nt, jd], timestep [B], img_ids [Ni, n_axes], txt_ids [Nt, n_axes].
        n_double / n_single limit the blocks run (bounded CPU samples)."""
        c, w = self.cfg, self.w
        dt = self.dtype
        hidden, encoder = hidden.to(self.device, dt), encoder.to(self.device, dt)
        temb = self.temb(timestep, guidance)
        st = silu(temb)
        mod_img = linear(st, w.get("double_stream_modulation_img.linear.weight"))
        mod_txt = linear(st, w.get("double_stream_modulation_txt.linear.weight"))
        mod_s = linear(st, w.get("single_stream_modulation.linear.weight"))
        hs = linear(hidden, w.get("x_embedder.weight"))
        ehs = linear(encoder, w.get("context_embedder.weight"))
        if img_ids.dim() == 3:
            img_ids = img_ids[0]
        if txt_ids.dim() == 3:
            txt_ids = txt_ids[0]
        ids = torch.cat([txt_ids, img_ids], dim=0).to(self.device)
        cos, sin = rope_cos_sin(ids, c.axes_dims_rope, c.rope_theta, dt)
        nd = c.num_layers if n_double is None else n_double
        ns = c.num_single_layers if n_single is None else n_single
        for i in range(nd):
            hs, ehs = self.double_block(i, hs, ehs, mod_img, mod_txt, cos, sin)
        nt = ehs.shape[1]
        hs = torch.cat([ehs, hs], dim=1)
        for i in range(ns):
            hs = self.single_block(i, hs, mod_s, cos, sin)
        hs = hs[:, nt:]
        emb = linear(st, w.get("norm_out.linear.weight"))
        scale, shift = emb.chunk(2, dim=1)
        hs = layer_norm(hs, c.eps) * (1.0 + scale)[:, None, :] + shift[:, None, :]
        return linear(hs, w.get("proj_out.weight"))

    def denoise(self, latents, encoder, timestep, dt, img_ids, txt_ids,
                image_latents=None, image_latent_ids=None) -> torch.Tensor:
        """Flux2KleinPipeline::denoise (Flux2KleinPipeline.cpp:496-537) +
        FlowMatchEulerDiscreteScheduler::integrate.  With image_latents the
        reference tokens and their ids are appended to the image tokens
        (:511-519), the forward runs on both, and the noise prediction is
        sliced back to the latent tokens before the Euler update (:531-536)."""
        x, ids = latents, img_ids
        if image_latents is not None:
            if image_latent_ids is None:
                raise ValueError("denoise(): image_latent_ids is required when image_latents is provided")
            if img_ids.dim() == 3:
                img_ids = img_ids[0]
            if image_latent_ids.dim() == 3:
                image_latent_ids = image_latent_ids[0]
            x = torch.cat([latents.to(image_latents.dtype), image_latents], dim=1)
            ids = torch.cat([img_ids, image_latent_ids], dim=0)
        v = self.forward(x, encoder, timestep, ids, txt_ids, None)
        v = v[:, : latents.shape[1]]
        return latents.to(self.device, self.dtype) + dt * v


def flow_match_schedule(n: int, shift: float = 1.0):
    """FlowMatchEulerDiscreteScheduler::schedule (default ctor) with the
    pipeline's sigmas 1 - i/n (Flux2KleinPipeline.cpp:348-356)."""
    sig = [np.float32(1.0 - i / n) for i in range(n)]
    sig = [np.float32(shift * s / (1.0 + (shift - 1.0) * s)) for s in sig]
    ts = [np.float32(s * 1000.0) for s in sig]
    return ts, sig + [np.float32(0.0)]


def flow_match_schedule_full(n: int, mu: float = 0.0, sigmas=None, num_train_timesteps: int = 1000,
                             shift: float = 1.0, use_dynamic_shifting: bool = False, shift_terminal=None,
                             invert_sigmas: bool = False, time_shift_type: str = "exponential"):
    """FlowMatchEulerDiscreteScheduler::schedule(n, mu, sigmas) for every
    constructor option, one float32 operation at a time
    (FlowMatchEulerDiscreteScheduler.cpp:8-37 options, :43-66 time_shift,
    :68-208 schedule).  Returns (timesteps[n], sigmas[n + 1]) as float32."""
    f = np.float32
    if num_train_timesteps <= 0 or n <= 0 or time_shift_type not in ("exponential", "linear"):
        raise ValueError("invalid scheduler arguments")
    T = f(num_train_timesteps)
    if sigmas is not None:
        if len(sigmas) != n:
            raise ValueError("sigmas must have n entries")
        base = [f(s) for s in sigmas]
    else:
        t_max = f(1.0) * T
        t_min = (f(1.0) / T) * T
        if n == 1:
            base = [t_max / T]
        else:
            base = [(t_max - f(i) * (t_max - t_min) / f(n - 1)) / T for i in range(n)]
    out = []
    for s in base:
        if use_dynamic_shifting:
            if s <= 0:
                raise ValueError("t must be positive")
            odds = np.power(f(1.0) / s - f(1.0), f(1.0))
            e = f(mu) if time_shift_type == "linear" else f(np.exp(np.float64(mu)))
            out.append(e / (e + odds))
        else:
            sh = f(shift)
            out.append(sh * s / (f(1.0) + (sh - f(1.0)) * s))
    if shift_terminal is not None:
        scale = (f(1.0) - out[-1]) / (f(1.0) - f(shift_terminal))
        out = [f(1.0) - (f(1.0) - s) / scale for s in out]
    if invert_sigmas:
        out = [f(1.0) - s for s in out]
    ts = np.array([s * T for s in out], dtype=np.float32)
    return ts, np.array(out + [f(1.0) if invert_sigmas else f(0.0)], dtype=np.float32)


def prepare_txt_ids(batch: int, seq_len: int) -> np.ndarray:
    """txt_ids [B, L, 4] = (0, 0, 0, l) (Flux2KleinPipeline.cpp:26-46)."""
    ids = np.zeros((batch, seq_len, 4), dtype=np.int32)
    ids[:, :, 3] = np.arange(seq_len, dtype=np.int32)
    return ids


def prepare_img_ids(batch: int, packed_h: int, packed_w: int) -> np.ndarray:
    """img_ids [B, h*w, 4] = (0, y, x, 0), row-major over (y, x)
    (Flux2KleinPipeline.cpp:48-72)."""
    ids = np.zeros((batch, packed_h * packed_w, 4), dtype=np.int32)
    for y in range(packed_h):
        for x in range(packed_w):
            ids[:, y * packed_w + x, 1] = y
            ids[:, y * packed_w + x, 2] = x
    return ids


def prepare_ref_image_ids(batch: int, packed_sizes) -> np.ndarray:
    """image_latent_ids [B, sum h_i*w_i, 4] = (10 + 10 i, y, x, 0) per
    reference image i (Flux2KleinPipeline.cpp:75-127)."""
    rows = []
    for i, (h, w) in enumerate(packed_sizes):
        for y in range(h):
            for x in range(w):
                rows.append((10 + 10 * i, y, x, 0))
    one = np.array(rows, dtype=np.int32).reshape(-1, 4)
    return np.repeat(one[None], batch, axis=0)


def compute_empirical_mu(image_seq_len: int, num_steps: int) -> np.float32:
    """The Flux2 Klein pipeline's dynamic-shift mu (Flux2KleinPipeline.cpp:130-141),
    in float32."""
    f = np.float32
    a1, b1, a2, b2 = f(8.73809524e-05), f(1.89833333), f(0.00016927), f(0.45666666)
    length = f(image_seq_len)
    if image_seq_len > 4300:
        return a2 * length + b2
    m_200 = a2 * length + b2
    m_10 = a1 * length + b1
    a = (m_200 - m_10) / f(190.0)
    b = m_200 - f(200.0) * a
    return a * f(num_steps) + b
