"""TEST INFRASTRUCTURE ONLY -- CPU oracle of the Flux2 VAE decode.

Only tests/ and bench.py may import this module; the product path
(``diffusers-cpp_b200``) never does.

A PyTorch-CPU restatement (float64 by default) of the pipeline's latent
decode, op by op:

* ``Flux2KleinPipeline::decode``        src/diffusers/pipelines/flux2/Flux2KleinPipeline.cpp:538-556
  (unpack the packed tokens :606-612, BatchNorm de-normalisation with the
  running statistics, unpatchify :614-630, VAE decode or decode_tiled)
* ``AutoencoderKLFlux2::decode``        src/diffusers/models/autoencoders/AutoencoderKLFlux2.cpp:139-150
  (post_quant_conv, then the decoder)
* ``Decoder::forward``                  src/diffusers/models/autoencoders/vae/Decoder.hpp:110-165
  (conv_in, mid block, up blocks, GroupNorm, SiLU, conv_out)
* ``UNetMidBlock2D``                    src/diffusers/models/unets/unet2d/UNetMidBlock2D.cpp (resnet,
  attention, resnet)
* ``UpDecoderBlock2D``                  src/diffusers/models/unets/unet2d/UpDecoderBlock2D.cpp
  (layers_per_block + 1 resnets, then Upsample2D: nearest 2x + 3x3 conv,
  src/diffusers/models/resnet/Upsample2D.cpp)
* ``ResnetBlock2D::forward``            src/diffusers/models/resnet/ResnetBlock2D.inl:108-190
  (GroupNorm, SiLU, conv1, GroupNorm, SiLU, conv2, 1x1 conv_shortcut when
  the channel count changes, residual add; eps 1e-6)
* ``Attention::forward``                src/diffusers/models/attention_processor/Attention.inl
  (GroupNorm, single head of dim C over the H*W tokens, biased q/k/v/out
  projections, residual) with ``SoftmaxAttentionOp`` (scale d^-1/2, softmax
  over keys; the reference omits the max subtraction, which is the same
  function)
* ``AutoencoderKLFlux2::decode_tiled``  AutoencoderKLFlux2.cpp:258-380 (3/4-stride tiles, linear
  blending over a quarter tile, top-left bands kept)

Parity: unpinned.  The reference's VAE tests compare against HF diffusers,
which is not installed here; the restatement is checked against the
reference source only.  The operators are torch's own conv2d / group_norm /
softmax in float64.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

from flux2_oracle import Weights


@dataclass
class VAEConfig:
    in_channels: int = 3
    out_channels: int = 3
    block_out_channels: Tuple[int, ...] = (128, 256, 512, 512)
    layers_per_block: int = 2
    latent_channels: int = 32
    norm_num_groups: int = 32
    batch_norm_eps: float = 1e-4
    patch_size: Tuple[int, int] = (2, 2)
    use_post_quant_conv: bool = True
    mid_block_add_attention: bool = True


def unpack_unpatchify(latents: torch.Tensor, mean: torch.Tensor, var: torch.Tensor, eps: float, ph: int, pw: int,
                      C: int) -> torch.Tensor:
    """[B, ph*pw, 4C] packed tokens -> z [B, C, 2ph, 2pw] with
    z[b, c, 2i+r, 2j+s] = packed[b, i*pw+j, 4c+2r+s] * sqrt(var + eps) + mean."""
    B = latents.shape[0]
    zp = latents.permute(0, 2, 1).reshape(B, 4 * C, ph, pw)
    zp = zp * torch.sqrt(var.reshape(1, -1, 1, 1) + eps) + mean.reshape(1, -1, 1, 1)
    z = zp.reshape(B, C, 2, 2, ph, pw).permute(0, 1, 4, 2, 5, 3)
    return z.reshape(B, C, 2 * ph, 2 * pw)


class VAEDecoderOracle:
    def __init__(self, cfg: VAEConfig, params, dtype=torch.float64):
        self.cfg = cfg
        self.w = Weights(params, dtype)
        self.dtype = dtype

    def _p(self, name):
        return self.w.get(name)

    def conv(self, x, prefix, padding):
        return F.conv2d(x, self._p(prefix + ".weight"), self._p(prefix + ".bias"), padding=padding)

    def gn(self, x, prefix, eps=1e-6):
        return F.group_norm(x, self.cfg.norm_num_groups, self._p(prefix + ".weight"), self._p(prefix + ".bias"), eps)

    def resnet(self, x, prefix):
        h = self.conv(F.silu(self.gn(x, prefix + ".norm1")), prefix + ".conv1", 1)
        h = self.conv(F.silu(self.gn(h, prefix + ".norm2")), prefix + ".conv2", 1)
        if self.w.has(prefix + ".conv_shortcut.weight"):
            x = self.conv(x, prefix + ".conv_shortcut", 0)
        return x + h

    def attention(self, x, prefix):
        B, C, H, W = x.shape
        h = self.gn(x, prefix + ".group_norm").permute(0, 2, 3, 1).reshape(B, H * W, C)
        q = F.linear(h, self._p(prefix + ".to_q.weight"), self._p(prefix + ".to_q.bias"))
        k = F.linear(h, self._p(prefix + ".to_k.weight"), self._p(prefix + ".to_k.bias"))
        v = F.linear(h, self._p(prefix + ".to_v.weight"), self._p(prefix + ".to_v.bias"))
        a = torch.softmax((q @ k.transpose(1, 2)) / math.sqrt(C), dim=-1) @ v
        o = F.linear(a, self._p(prefix + ".to_out.0.weight"), self._p(prefix + ".to_out.0.bias"))
        return o.reshape(B, H, W, C).permute(0, 3, 1, 2) + x

    def decode(self, z: torch.Tensor) -> torch.Tensor:
        """z [B, latent_channels, h, w] -> image [B, out_channels, 8h, 8w] (AutoencoderKLFlux2::decode)."""
        c = self.cfg
        x = z.to(self.dtype)
        if c.use_post_quant_conv:
            x = self.conv(x, "post_quant_conv", 0)
        x = self.conv(x, "decoder.conv_in", 1)
        x = self.resnet(x, "decoder.mid_block.resnets.0")
        if c.mid_block_add_attention:
            x = self.attention(x, "decoder.mid_block.attentions.0")
        x = self.resnet(x, "decoder.mid_block.resnets.1")
        n_up = len(c.block_out_channels)
        for i in range(n_up):
            for j in range(c.layers_per_block + 1):
                x = self.resnet(x, f"decoder.up_blocks.{i}.resnets.{j}")
            if i < n_up - 1:
                x = F.interpolate(x, scale_factor=2.0, mode="nearest")
                x = self.conv(x, f"decoder.up_blocks.{i}.upsamplers.0.conv", 1)
        x = F.silu(self.gn(x, "decoder.conv_norm_out"))
        return self.conv(x, "decoder.conv_out", 1)

    def decode_packed(self, latents: torch.Tensor, ph: int, pw: int, tile: int = 0) -> torch.Tensor:
        """Flux2KleinPipeline::decode: packed tokens [B, ph*pw, 4C] -> image [B, 3, 16ph, 16pw]."""
        c = self.cfg
        z = unpack_unpatchify(latents.to(self.dtype), self._p("bn.running_mean"), self._p("bn.running_var"),
                              c.batch_norm_eps, ph, pw, c.latent_channels)
        if tile > 0:
            return self.decode_tiled(z, tile, tile)
        return self.decode(z)

    def decode_tiled(self, z: torch.Tensor, tile_h: int, tile_w: int) -> torch.Tensor:
        """AutoencoderKLFlux2::decode_tiled with pixel tile sizes."""
        scale = 1 << (len(self.cfg.block_out_channels) - 1)
        lt_h, lt_w = tile_h // scale, tile_w // scale
        blend_h, blend_w = tile_h // 4, tile_w // 4
        band_h, band_w = tile_h - blend_h, tile_w - blend_w
        stride_h, stride_w = lt_h * 3 // 4, lt_w * 3 // 4
        H, W = z.shape[2], z.shape[3]
        rows: List[List[torch.Tensor]] = []
        for i in range(0, H, stride_h):
            rows.append([self.decode(z[:, :, i:i + lt_h, j:j + lt_w]) for j in range(0, W, stride_w)])
        out_rows = []
        for i, row in enumerate(rows):
            bands = []
            for j, tile in enumerate(row):
                if i > 0:
                    tile = _blend_v(rows[i - 1][j], tile, blend_h)
                if j > 0:
                    tile = _blend_h(row[j - 1], tile, blend_w)
                row[j] = tile
                bands.append(tile[:, :, :band_h, :band_w])
            out_rows.append(torch.cat(bands, dim=-1))
        return torch.cat(out_rows, dim=-2)


def _blend_v(a, b, extent):
    extent = min(a.shape[2], b.shape[2], extent)
    if extent <= 0:
        return b
    w = (torch.arange(extent, dtype=b.dtype) / extent).reshape(1, 1, extent, 1)
    head = a[:, :, a.shape[2] - extent:, :] * (1 - w) + b[:, :, :extent, :] * w
    return head if extent >= b.shape[2] else torch.cat([head, b[:, :, extent:, :]], dim=2)


def _blend_h(a, b, extent):
    extent = min(a.shape[3], b.shape[3], extent)
    if extent <= 0:
        return b
    w = (torch.arange(extent, dtype=b.dtype) / extent).reshape(1, 1, 1, extent)
    head = a[:, :, :, a.shape[3] - extent:] * (1 - w) + b[:, :, :, :extent] * w
    return head if extent >= b.shape[3] else torch.cat([head, b[:, :, :, extent:]], dim=3)


def decoder_param_shapes(cfg: VAEConfig) -> Dict[str, Tuple[int, ...]]:
    """Names and shapes of the decode path's parameters (diffusers
    AutoencoderKLFlux2 state-dict names, as the reference's modules path them)."""
    s: Dict[str, Tuple[int, ...]] = {}
    L, ch = cfg.latent_channels, list(cfg.block_out_channels)
    s["bn.running_mean"] = (4 * L,)
    s["bn.running_var"] = (4 * L,)
    if cfg.use_post_quant_conv:
        s["post_quant_conv.weight"] = (L, L, 1, 1)
        s["post_quant_conv.bias"] = (L,)

    def conv(name, cin, cout, k):
        s[name + ".weight"] = (cout, cin, k, k)
        s[name + ".bias"] = (cout,)

    def norm(name, c):
        s[name + ".weight"] = (c,)
        s[name + ".bias"] = (c,)

    def resnet(name, cin, cout):
        norm(name + ".norm1", cin)
        conv(name + ".conv1", cin, cout, 3)
        norm(name + ".norm2", cout)
        conv(name + ".conv2", cout, cout, 3)
        if cin != cout:
            conv(name + ".conv_shortcut", cin, cout, 1)

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
