"""Tensor-parallel restatement of the Flux2 forward, for tests only.

Runs one rank's share of ``Flux2Transformer2DModel::forward`` in float64 on
the CPU from the exact shards the library assembled for that rank (read back
from a host-only model, ``dcpp_flux2_read_param``), summing the partial
outputs of the row-parallel projections with a caller-supplied all-reduce
(``torch.distributed`` over gloo in the tests).  The sharding it checks is the
reference planner's (ShardingRuntime.cpp:47-57): q/k/v/gate/up column
parallel (whole heads, ``mlp_hidden / n`` features), the attention and MLP
output projections row parallel, one all-reduce per row-parallel site.

Shard layouts (model names, as ``read_param`` takes them):
  transformer_blocks.i.attn.to_qkv / attn.add_qkv   [3 Dl, D]  q | k | v rows of this rank's heads
  transformer_blocks.i.attn.to_out.0.weight / attn.to_add_out.weight   [D, Dl]
  transformer_blocks.i.ff(_context).linear_in.weight [2 Fl, D]  gate/up interleaved in 64-row blocks
  transformer_blocks.i.ff(_context).linear_out.weight [D, Fl]
  single_transformer_blocks.i.attn.to_qkv_mlp_proj.weight [3 Dl + 2 Fl, D]
  single_transformer_blocks.i.attn.to_out.weight     [D, Dl + Fl]  attention columns | MLP columns
Everything else is replicated.
"""
from __future__ import annotations

from typing import Callable, Dict, List

import numpy as np
import torch

import flux2_oracle as fo


def weight_names(c) -> List[str]:
    """Model names of every weight matrix (fused names for the block projections)."""
    n = ["time_guidance_embed.timestep_embedder.linear_1.weight", "time_guidance_embed.timestep_embedder.linear_2.weight"]
    if c.guidance_embeds:
        n += ["time_guidance_embed.guidance_embedder.linear_1.weight",
              "time_guidance_embed.guidance_embedder.linear_2.weight"]
    n += ["double_stream_modulation_img.linear.weight", "double_stream_modulation_txt.linear.weight",
          "single_stream_modulation.linear.weight", "x_embedder.weight", "context_embedder.weight",
          "norm_out.linear.weight", "proj_out.weight"]
    for i in range(c.num_layers):
        p = f"transformer_blocks.{i}."
        n += [p + "attn.add_qkv", p + "attn.to_qkv", p + "attn.to_add_out.weight", p + "attn.to_out.0.weight",
              p + "ff_context.linear_in.weight", p + "ff.linear_in.weight", p + "ff_context.linear_out.weight",
              p + "ff.linear_out.weight"]
    for i in range(c.num_single_layers):
        p = f"single_transformer_blocks.{i}.attn."
        n += [p + "to_qkv_mlp_proj.weight", p + "to_out.weight"]
    return n


def vector_names(c) -> List[str]:
    n = []
    for i in range(c.num_layers):
        p = f"transformer_blocks.{i}.attn."
        n += [p + s + ".weight" for s in ("norm_q", "norm_k", "norm_added_q", "norm_added_k")]
    for i in range(c.num_single_layers):
        p = f"single_transformer_blocks.{i}.attn."
        n += [p + "norm_q.weight", p + "norm_k.weight"]
    return n


def decode(gtype: int, shape, buf: np.ndarray) -> torch.Tensor:
    """A read_param result as a float64 matrix (bit-exact dequantisation)."""
    rows, cols = shape
    return torch.from_numpy(fo.dequant(gtype, buf, rows * cols).reshape(rows, cols)).double()


def interleave64(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """Rows gate block 0, up block 0, gate block 1, ... (64-row blocks)."""
    g = gate.unflatten(0, (-1, 64))
    u = up.unflatten(0, (-1, 64))
    return torch.stack([g, u], dim=1).flatten(0, 2)


def deinterleave64(y: torch.Tensor):
    z = y.unflatten(-1, (-1, 2, 64))
    return z[..., 0, :].flatten(-2), z[..., 1, :].flatten(-2)


def plan_split(units: int, ratios) -> List[int]:
    """The sharding planner's rounding (ShardingRuntime.cpp:280-296), restated:
    floor(units * f_j / sum f), then the remaining units one by one to the
    ranks with the largest fractional parts (ties: the later rank)."""
    s = sum(ratios)
    c = [units * f / s for f in ratios]
    m = [int(x // 1) for x in c]
    frac = [x - mi for x, mi in zip(c, m)]
    for _ in range(units - sum(m)):
        best = 0
        for j in range(1, len(ratios)):
            if frac[j] >= frac[best]:
                best = j
        m[best] += 1
        frac[best] = -1.0
    return m


def shard_of(c, rank: int, n: int, ratios=None):
    """(first head, heads, first MLP feature, MLP features) of `rank`."""
    ratios = ratios or [1.0] * n
    heads = plan_split(c.num_attention_heads, ratios)
    units = plan_split(c.mlp_hidden // 64, ratios)
    return sum(heads[:rank]), heads[rank], 64 * sum(units[:rank]), 64 * units[rank]


def expected_shards(c, w: fo.Weights, rank: int, n: int, ratios=None) -> Dict[str, torch.Tensor]:
    """Float weights each shard must hold, sliced from the full (unsharded) weights."""
    D, F = c.inner_dim, c.mlp_hidden
    h0, hn, f0, fn = shard_of(c, rank, n, ratios)
    hs, fs = slice(h0 * 128, (h0 + hn) * 128), slice(f0, f0 + fn)
    out = {}
    for name in weight_names(c):
        if not (name.startswith("transformer_blocks.") or name.startswith("single_transformer_blocks.")):
            out[name] = w.get(name)
    for i in range(c.num_layers):
        p = f"transformer_blocks.{i}."
        for fused, names in (("attn.to_qkv", ("attn.to_q", "attn.to_k", "attn.to_v")),
                             ("attn.add_qkv", ("attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj"))):
            out[p + fused] = torch.cat([w.get(p + s + ".weight")[hs] for s in names])
        for o in ("attn.to_out.0.weight", "attn.to_add_out.weight"):
            out[p + o] = w.get(p + o)[:, hs]
        for ff in ("ff", "ff_context"):
            q = p + ff
            gate = w.rows(q + ".linear_in_gate.weight", q + ".linear_in.weight", 0, F)[fs]
            up = w.rows(q + ".linear_in_up.weight", q + ".linear_in.weight", F, 2 * F)[fs]
            out[q + ".linear_in.weight"] = interleave64(gate, up)
            out[q + ".linear_out.weight"] = w.get(q + ".linear_out.weight")[:, fs]
    for i in range(c.num_single_layers):
        p = f"single_transformer_blocks.{i}.attn."
        fq = p + "to_qkv_mlp_proj.weight"
        qkv = [w.rows(p + f"to_qkv_mlp_proj.{s}.weight", fq, g * D, (g + 1) * D)[hs] for g, s in enumerate("qkv")]
        gate = w.rows(p + "to_qkv_mlp_proj.mlp_in_gate.weight", fq, 3 * D, 3 * D + F)[fs]
        up = w.rows(p + "to_qkv_mlp_proj.mlp_in_up.weight", fq, 3 * D + F, 3 * D + 2 * F)[fs]
        out[fq] = torch.cat(qkv + [interleave64(gate, up)])
        fo_ = p + "to_out.weight"
        attn = w.cols(p + "to_out.attn.weight", fo_, 0, D)[:, hs]
        mlp = w.cols(p + "to_out.mlp.weight", fo_, D, D + F)[:, fs]
        out[fo_] = torch.cat([attn, mlp], dim=1)
    return out


class TPOracle(fo.Flux2Oracle):
    """One rank of the tensor-parallel forward, on its own shards.

    ``shards``: model name -> float64 matrix (weights) or vector (norms), as
    read from a host-only model of this rank; ``allreduce`` sums a tensor over
    the ranks and returns it."""

    def __init__(self, cfg: fo.Config, shards: Dict[str, torch.Tensor], n: int,
                 allreduce: Callable[[torch.Tensor], torch.Tensor], heads: int = 0):
        super().__init__(cfg, {}, dtype=torch.float64)
        self.s = shards
        self.n = n
        self.hl = heads or cfg.num_attention_heads // n  # this rank's heads
        self.allreduce = allreduce
        # Replicated weights resolve through the base class's Weights cache.
        self.w.cache.update({k: v for k, v in shards.items()
                             if not k.startswith(("transformer_blocks.", "single_transformer_blocks."))})

    def double_block(self, i, hs, ehs, mod_img, mod_txt, cos, sin):
        c, S = self.cfg, self.s
        eps, Hl = c.eps, self.hl
        Dl = Hl * c.attention_head_dim
        p = f"transformer_blocks.{i}."
        sh, sc, g, sh2, sc2, g2 = mod_img[:, None, :].chunk(6, dim=-1)
        csh, csc, cg, csh2, csc2, cg2 = mod_txt[:, None, :].chunk(6, dim=-1)
        n = (1.0 + sc) * fo.layer_norm(hs, eps) + sh
        ne = (1.0 + csc) * fo.layer_norm(ehs, eps) + csh
        qkv = fo.linear(n, S[p + "attn.to_qkv"])
        eqkv = fo.linear(ne, S[p + "attn.add_qkv"])
        heads = lambda x: fo._heads(x, Hl)
        q = fo.rms_norm(heads(qkv[..., :Dl]), S[p + "attn.norm_q.weight"], eps)
        k = fo.rms_norm(heads(qkv[..., Dl:2 * Dl]), S[p + "attn.norm_k.weight"], eps)
        v = heads(qkv[..., 2 * Dl:])
        eq = fo.rms_norm(heads(eqkv[..., :Dl]), S[p + "attn.norm_added_q.weight"], eps)
        ek = fo.rms_norm(heads(eqkv[..., Dl:2 * Dl]), S[p + "attn.norm_added_k.weight"], eps)
        ev = heads(eqkv[..., 2 * Dl:])
        q = fo.apply_rope(torch.cat([eq, q], dim=1), cos, sin)
        k = fo.apply_rope(torch.cat([ek, k], dim=1), cos, sin)
        o = fo.sdpa(q, k, torch.cat([ev, v], dim=1)).flatten(2)
        nt = ehs.shape[1]
        o_txt = self.allreduce(fo.linear(o[:, :nt], S[p + "attn.to_add_out.weight"]))
        o_img = self.allreduce(fo.linear(o[:, nt:], S[p + "attn.to_out.0.weight"]))
        hs = hs + g * o_img
        n2 = fo.layer_norm(hs, eps) * (1.0 + sc2) + sh2
        hs = hs + g2 * self.ff_tp(p + "ff", n2)
        ehs = ehs + cg * o_txt
        ne2 = fo.layer_norm(ehs, eps) * (1.0 + csc2) + csh2
        ehs = ehs + cg2 * self.ff_tp(p + "ff_context", ne2)
        return hs, ehs

    def ff_tp(self, prefix, x):
        gate, up = deinterleave64(fo.linear(x, self.s[prefix + ".linear_in.weight"]))
        return self.allreduce(fo.linear(fo.silu(gate) * up, self.s[prefix + ".linear_out.weight"]))

    def single_block(self, i, hs, mod, cos, sin):
        c, S = self.cfg, self.s
        eps, Hl = c.eps, self.hl
        Dl = Hl * c.attention_head_dim
        p = f"single_transformer_blocks.{i}.attn."
        sh, sc, g = mod[:, None, :].chunk(3, dim=-1)
        n = (1.0 + sc) * fo.layer_norm(hs, eps) + sh
        y = fo.linear(n, S[p + "to_qkv_mlp_proj.weight"])
        heads = lambda x: fo._heads(x, Hl)
        q = fo.apply_rope(fo.rms_norm(heads(y[..., :Dl]), S[p + "norm_q.weight"], eps), cos, sin)
        k = fo.apply_rope(fo.rms_norm(heads(y[..., Dl:2 * Dl]), S[p + "norm_k.weight"], eps), cos, sin)
        o = fo.sdpa(q, k, heads(y[..., 2 * Dl:3 * Dl])).flatten(2)
        gate, up = deinterleave64(y[..., 3 * Dl:])
        out = self.allreduce(fo.linear(torch.cat([o, fo.silu(gate) * up], dim=-1), S[p + "to_out.weight"]))
        return hs + g * out


def read_shards(model, c) -> Dict[str, tuple]:
    """name -> (ggml type, (rows, cols), raw bytes) of every weight and norm vector."""
    return {name: model.read_param(name) for name in weight_names(c) + vector_names(c)}


def decode_shards(raw: Dict[str, tuple]) -> Dict[str, torch.Tensor]:
    out = {}
    for name, (gt, shape, buf) in raw.items():
        t = decode(gt, shape, buf)
        out[name] = t[0] if shape[0] == 1 and name.endswith(("norm_q.weight", "norm_k.weight", "norm_added_q.weight",
                                                              "norm_added_k.weight")) else t
    return out
