"""Seeded synthetic Flux2 parameters and inputs in GGUF layout.

Weights are N(0, 1/fan_in) from a per-tensor seeded torch generator (seed,
tensor name), quantised with ``quant.py`` following the reference's per-tensor
type map (utils/convert-model/flux2-klein-9b-q8.json): every projection in the
blocks and the modulations in the chosen quantised type, the input / output
projections and the time embedding in BF16, the RMSNorm weights in F32.
Tensor names are the GGUF names, with the fused tensors the reference's
loader byte-slices (GGUFLoaderVisitor.cpp:283-429) unless ``split=True``.
"""
from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch

from . import TYPE_BF16, TYPE_F32, TYPE_Q4_K, TYPE_Q8_0
from .quant import quantize

BF16_NAMES = (
    "x_embedder.weight",
    "context_embedder.weight",
    "time_guidance_embed.timestep_embedder.linear_1.weight",
    "time_guidance_embed.timestep_embedder.linear_2.weight",
    "time_guidance_embed.guidance_embedder.linear_1.weight",
    "time_guidance_embed.guidance_embedder.linear_2.weight",
    "norm_out.linear.weight",
    "proj_out.weight",
)


@dataclass
class Flux2Cfg:
    """Same fields as Flux2Transformer2DModel::Config."""
    patch_size: int = 1
    in_channels: int = 128
    out_channels: Optional[int] = None
    num_layers: int = 5
    num_single_layers: int = 20
    attention_head_dim: int = 128
    num_attention_heads: int = 24
    joint_attention_dim: int = 7680
    timestep_guidance_channels: int = 256
    mlp_ratio: float = 3.0
    axes_dims_rope: Tuple[int, ...] = (32, 32, 32, 32)
    rope_theta: int = 2000
    eps: float = 1e-6
    guidance_embeds: bool = False

    @property
    def inner_dim(self) -> int:
        return self.num_attention_heads * self.attention_head_dim

    @property
    def mlp_hidden(self) -> int:
        return int(self.inner_dim * self.mlp_ratio)


def tensor_seed(seed: int, name: str) -> int:
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


def param_shapes(cfg: Flux2Cfg, split: bool = False) -> Dict[str, Tuple[int, ...]]:
    D, F, tg = cfg.inner_dim, cfg.mlp_hidden, cfg.timestep_guidance_channels
    out_ch = cfg.patch_size ** 2 * (cfg.out_channels or cfg.in_channels)
    s: Dict[str, Tuple[int, ...]] = {
        "time_guidance_embed.timestep_embedder.linear_1.weight": (D, tg),
        "time_guidance_embed.timestep_embedder.linear_2.weight": (D, D),
        "double_stream_modulation_img.linear.weight": (6 * D, D),
        "double_stream_modulation_txt.linear.weight": (6 * D, D),
        "single_stream_modulation.linear.weight": (3 * D, D),
        "x_embedder.weight": (D, cfg.in_channels),
        "context_embedder.weight": (D, cfg.joint_attention_dim),
        "norm_out.linear.weight": (2 * D, D),
        "proj_out.weight": (out_ch, D),
    }
    if cfg.guidance_embeds:
        s["time_guidance_embed.guidance_embedder.linear_1.weight"] = (D, tg)
        s["time_guidance_embed.guidance_embedder.linear_2.weight"] = (D, D)
    hd = cfg.attention_head_dim
    for i in range(cfg.num_layers):
        p = f"transformer_blocks.{i}."
        for n in ("to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj", "to_add_out", "to_out.0"):
            s[p + "attn." + n + ".weight"] = (D, D)
        for n in ("norm_q", "norm_k", "norm_added_q", "norm_added_k"):
            s[p + "attn." + n + ".weight"] = (hd,)
        for ff in ("ff", "ff_context"):
            if split:
                s[p + ff + ".linear_in_gate.weight"] = (F, D)
                s[p + ff + ".linear_in_up.weight"] = (F, D)
            else:
                s[p + ff + ".linear_in.weight"] = (2 * F, D)
            s[p + ff + ".linear_out.weight"] = (D, F)
    for i in range(cfg.num_single_layers):
        p = f"single_transformer_blocks.{i}.attn."
        if split:
            for n in ("q", "k", "v"):
                s[p + "to_qkv_mlp_proj." + n + ".weight"] = (D, D)
            s[p + "to_qkv_mlp_proj.mlp_in_gate.weight"] = (F, D)
            s[p + "to_qkv_mlp_proj.mlp_in_up.weight"] = (F, D)
            s[p + "to_out.attn.weight"] = (D, D)
            s[p + "to_out.mlp.weight"] = (D, F)
        else:
            s[p + "to_qkv_mlp_proj.weight"] = (3 * D + 2 * F, D)
            s[p + "to_out.weight"] = (D, D + F)
        s[p + "norm_q.weight"] = (hd,)
        s[p + "norm_k.weight"] = (hd,)
    return s


def type_for(name: str, shape, wtype: int) -> int:
    if len(shape) == 1:
        return TYPE_F32
    if name in BF16_NAMES:
        return TYPE_BF16
    return wtype


def make_params(cfg: Flux2Cfg, wtype: int = TYPE_Q4_K, seed: int = 0, device: str = "cpu", split: bool = False,
                to_cpu: bool = True):
    """Dict name -> (ggml type, shape, uint8 tensor of raw GGUF bytes)."""
    out = {}
    for name, shape in param_shapes(cfg, split).items():
        g = torch.Generator(device=device)
        g.manual_seed(tensor_seed(seed, name))
        if len(shape) == 1:
            w = 1.0 + 0.1 * torch.randn(shape, generator=g, device=device, dtype=torch.float32)
        else:
            w = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * (1.0 / math.sqrt(shape[1]))
        t = type_for(name, shape, wtype)
        q = quantize(w, t).contiguous()
        if to_cpu:
            q = q.cpu()
        out[name] = (t, tuple(shape), q)
        del w
    return out


def make_inputs(cfg: Flux2Cfg, batch: int, grid_h: int, grid_w: int, n_txt: int, seed: int = 1, device: str = "cpu"):
    """hidden [B, h*w, in] N(0,1) (seed), encoder [B, n_txt, jd] N(0,1) (seed+1),
    img_ids [h*w, 4] = [0, y, x, 0], txt_ids [n_txt, 4] = [0, 0, 0, l]
    (prepare_img_ids / prepare_txt_ids, Flux2KleinPipeline.cpp:26-72)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    n_img = grid_h * grid_w
    hidden = torch.randn(batch, n_img, cfg.in_channels, generator=g, device=device)
    g.manual_seed(seed + 1)
    encoder = torch.randn(batch, n_txt, cfg.joint_attention_dim, generator=g, device=device)
    ys, xs = torch.meshgrid(torch.arange(grid_h), torch.arange(grid_w), indexing="ij")
    n_axes = len(cfg.axes_dims_rope)
    img_ids = torch.zeros(n_img, n_axes, dtype=torch.int32)
    txt_ids = torch.zeros(n_txt, n_axes, dtype=torch.int32)
    if n_axes >= 3:
        img_ids[:, 1] = ys.reshape(-1).int()
        img_ids[:, 2] = xs.reshape(-1).int()
    txt_ids[:, n_axes - 1] = torch.arange(n_txt, dtype=torch.int32)
    return hidden, encoder, img_ids.to(device), txt_ids.to(device)


# --------------------------------------------------------------------------- Qwen3 text encoder
@dataclass
class Qwen3Cfg:
    """Same fields as Qwen3Config (the prefill's subset); defaults: the text
    encoder of the reference benchmark's Qwen3 prefill configuration."""
    vocab_size: int = 151936
    hidden_size: int = 2560
    intermediate_size: int = 9728
    num_hidden_layers: int = 36
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0


def qwen3_param_shapes(cfg: Qwen3Cfg):
    D, I = cfg.hidden_size, cfg.intermediate_size
    Dq, Dkv = cfg.num_attention_heads * cfg.head_dim, cfg.num_key_value_heads * cfg.head_dim
    s = {"model.embed_tokens.weight": (cfg.vocab_size, D), "model.norm.weight": (D,)}
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        s[p + "self_attn.q_proj.weight"] = (Dq, D)
        s[p + "self_attn.k_proj.weight"] = (Dkv, D)
        s[p + "self_attn.v_proj.weight"] = (Dkv, D)
        s[p + "self_attn.o_proj.weight"] = (D, Dq)
        s[p + "self_attn.q_norm.weight"] = (cfg.head_dim,)
        s[p + "self_attn.k_norm.weight"] = (cfg.head_dim,)
        s[p + "mlp.gate_proj.weight"] = (I, D)
        s[p + "mlp.up_proj.weight"] = (I, D)
        s[p + "mlp.down_proj.weight"] = (D, I)
        s[p + "input_layernorm.weight"] = (D,)
        s[p + "post_attention_layernorm.weight"] = (D,)
    return s


# The reference converter's per-tensor types for the Klein text encoder
# (utils/convert-model/flux2-klein-9b-q8.json, "text_encoder": attention
# projections BF16, norms F32, everything else Q8_0).
QWEN3_KLEIN_TYPES = {"self_attn.q_proj.weight": TYPE_BF16, "self_attn.k_proj.weight": TYPE_BF16,
                     "self_attn.v_proj.weight": TYPE_BF16, "self_attn.o_proj.weight": TYPE_BF16}


def make_qwen3_params(cfg: Qwen3Cfg, wtype: int = TYPE_Q8_0, seed: int = 0, device: str = "cpu",
                      to_cpu: bool = True, types: Optional[Dict[str, int]] = None):
    """Dict name -> (ggml type, shape, uint8 tensor): matrices N(0, 0.02)
    quantised to `wtype` (or to types[suffix] for names ending in a key of
    `types`), norm weights 1 + 0.1 N(0, 1) in F32."""
    out = {}
    for name, shape in qwen3_param_shapes(cfg).items():
        g = torch.Generator(device=device)
        g.manual_seed(tensor_seed(seed, name))
        if len(shape) == 1:
            w = 1.0 + 0.1 * torch.randn(shape, generator=g, device=device, dtype=torch.float32)
            t = TYPE_F32
        else:
            w = 0.02 * torch.randn(shape, generator=g, device=device, dtype=torch.float32)
            t = next((v for k, v in (types or {}).items() if name.endswith(k)), wtype)
        q = quantize(w, t).contiguous()
        out[name] = (t, tuple(shape), q.cpu() if to_cpu else q)
    return out


def make_qwen3_ids(cfg: Qwen3Cfg, batch: int, seq: int, seed: int = 1):
    """Token ids [batch, seq] int32, uniform in [0, vocab_size)."""
    g = torch.Generator()
    g.manual_seed(seed)
    return torch.randint(0, cfg.vocab_size, (batch, seq), generator=g, dtype=torch.int64).to(torch.int32)


# --------------------------------------------------------------------------- Flux2 VAE decoder
@dataclass
class VAECfg:
    """Same fields as AutoencoderKLFlux2::Config (decode subset); defaults:
    the Flux2 VAE (1024-pixel images from 64 x 64 packed tokens)."""
    in_channels: int = 3
    out_channels: int = 3
    block_out_channels: Tuple[int, ...] = (128, 256, 512, 512)
    layers_per_block: int = 2
    latent_channels: int = 32
    norm_num_groups: int = 32
    batch_norm_eps: float = 1e-4
    use_post_quant_conv: bool = True
    mid_block_add_attention: bool = True


def vae_param_shapes(cfg: VAECfg) -> Dict[str, Tuple[int, ...]]:
    """Decode-path parameter names (diffusers AutoencoderKLFlux2 state dict)
    and PyTorch shapes."""
    s: Dict[str, Tuple[int, ...]] = {}
    L, ch = cfg.latent_channels, list(cfg.block_out_channels)
    s["bn.running_mean"] = (4 * L,)
    s["bn.running_var"] = (4 * L,)
    if cfg.use_post_quant_conv:
        s["post_quant_conv.weight"] = (L, L, 1, 1)
        s["post_quant_conv.bias"] = (L,)

    def conv(n, cin, cout, k):
        s[n + ".weight"] = (cout, cin, k, k)
        s[n + ".bias"] = (cout,)

    def norm(n, c):
        s[n + ".weight"] = (c,)
        s[n + ".bias"] = (c,)

    def resnet(n, cin, cout):
        norm(n + ".norm1", cin)
        conv(n + ".conv1", cin, cout, 3)
        norm(n + ".norm2", cout)
        conv(n + ".conv2", cout, cout, 3)
        if cin != cout:
            conv(n + ".conv_shortcut", cin, cout, 1)

    top = ch[-1]
    conv("decoder.conv_in", L, top, 3)
    resnet("decoder.mid_block.resnets.0", top, top)
    if cfg.mid_block_add_attention:
        p = "decoder.mid_block.attentions.0"
        norm(p + ".group_norm", top)
        for n in ("to_q", "to_k", "to_v", "to_out.0"):
            s[f"{p}.{n}.weight"] = (top, top)
            s[f"{p}.{n}.bias"] = (top,)
    resnet("decoder.mid_block.resnets.1", top, top)
    rev = ch[::-1]
    prev = rev[0]
    for i, out in enumerate(rev):
        for j in range(cfg.layers_per_block + 1):
            resnet(f"decoder.up_blocks.{i}.resnets.{j}", prev if j == 0 else out, out)
        if i < len(rev) - 1:
            conv(f"decoder.up_blocks.{i}.upsamplers.0.conv", out, out, 3)
        prev = out
    norm("decoder.conv_norm_out", ch[0])
    conv("decoder.conv_out", ch[0], cfg.out_channels, 3)
    return s


def make_vae_params(cfg: VAECfg, seed: int = 0, device: str = "cpu", to_cpu: bool = True):
    """Dict name -> (ggml type, shape, uint8 tensor), all F32 (the reference
    converter's type map stores the VAE in F32): conv / linear weights
    N(0, 1/fan_in), biases N(0, 0.02^2), GroupNorm scale 1 + 0.1 N and shift
    0.1 N, BatchNorm running mean 0.1 N and variance 1 + 0.5 U."""
    out = {}
    for name, shape in vae_param_shapes(cfg).items():
        g = torch.Generator(device=device)
        g.manual_seed(tensor_seed(seed, name))
        r = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
        if name == "bn.running_var":
            w = 1.0 + 0.5 * torch.rand(shape, generator=g, device=device, dtype=torch.float32)
        elif name == "bn.running_mean":
            w = 0.1 * r
        elif len(shape) >= 2:
            fan_in = math.prod(shape[1:])
            w = r / math.sqrt(fan_in)
        elif ".norm" in name or "group_norm" in name or "conv_norm_out" in name:
            w = (1.0 + 0.1 * r) if name.endswith(".weight") else 0.1 * r
        else:
            w = 0.02 * r
        q = w.contiguous().view(torch.uint8).reshape(-1)
        out[name] = (TYPE_F32, tuple(shape), q.cpu() if to_cpu else q)
    return out


def make_vae_latents(cfg: VAECfg, batch: int, packed_h: int, packed_w: int, seed: int = 3, device: str = "cpu"):
    """Packed denoised tokens [batch, packed_h * packed_w, 4 * latent_channels] f32, N(0, 1)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn(batch, packed_h * packed_w, 4 * cfg.latent_channels, generator=g, device=device,
                       dtype=torch.float32)
