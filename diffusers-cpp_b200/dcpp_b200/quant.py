"""ggml block quantisers in torch (run on CPU or on the GPU).

Used to produce synthetic GGUF-layout weights (the reference's converter does
the same with gguf-py, utils/convert-model/src/convert_hf_safetensors_to_gguf.py:340-358).

* ``quantize_q8_0``: bit-identical to gguf-py 0.19.0 ``Q8_0.quantize_blocks``
  (quants.py:380-394), which is bit-identical to ggml's quantize_row_q8_0:
  d = max|x| / 127, q = round_half_away(x / d), d stored as f16.
* ``quantize_q4_k``: our own Q4_K quantiser (gguf-py has none): per
  32-weight sub-block a (scale, min) pair from its range, 6-bit scale and
  min codes relative to the super-block's f16 d / dmin, then 4-bit codes.
  The byte layout is exactly ggml's block_q4_K (f16 d, f16 dmin, 12 bytes of
  packed 6-bit scales / mins, 128 bytes of nibbles).
* ``to_bf16_bytes``: round-to-nearest-even f32 -> bf16.
"""
from __future__ import annotations

import torch


def _round_half_away(v: torch.Tensor) -> torch.Tensor:
    a = v.abs()
    fl = torch.floor(a)
    return torch.sign(v) * (fl + torch.floor(2 * (a - fl)))


def quantize_q8_0(x: torch.Tensor) -> torch.Tensor:
    """x f32 [..., K] (K % 32 == 0) -> uint8 [..., K // 32 * 34]."""
    assert x.dtype == torch.float32 and x.shape[-1] % 32 == 0
    lead = x.shape[:-1]
    b = x.reshape(-1, 32)
    d = b.abs().amax(dim=1, keepdim=True) / 127
    inv = torch.where(d == 0, torch.zeros_like(d), 1 / d)
    q = _round_half_away(b * inv).to(torch.int8)
    dh = d.to(torch.float16).view(torch.uint8).reshape(-1, 2)
    out = torch.cat([dh, q.view(torch.uint8)], dim=1)
    return out.reshape(*lead, -1)


def quantize_q4_k(x: torch.Tensor) -> torch.Tensor:
    """x f32 [..., K] (K % 256 == 0) -> uint8 [..., K // 256 * 144]."""
    assert x.dtype == torch.float32 and x.shape[-1] % 256 == 0
    lead = x.shape[:-1]
    b = x.reshape(-1, 8, 32)
    nb = b.shape[0]
    mn = torch.clamp(b.amin(dim=2), max=0.0)          # [nb, 8]
    mx = b.amax(dim=2)
    scale = (mx - mn) / 15.0
    mins = -mn
    d = scale.amax(dim=1, keepdim=True) / 63.0         # [nb, 1]
    dmin = mins.amax(dim=1, keepdim=True) / 63.0
    d16 = d.to(torch.float16)
    dmin16 = dmin.to(torch.float16)
    df, dmf = d16.float(), dmin16.float()
    isc = torch.where(df > 0, torch.floor(scale / torch.where(df > 0, df, torch.ones_like(df)) + 0.5), torch.zeros_like(scale))
    im = torch.where(dmf > 0, torch.floor(mins / torch.where(dmf > 0, dmf, torch.ones_like(dmf)) + 0.5), torch.zeros_like(mins))
    isc = isc.clamp(0, 63).to(torch.int32)
    im = im.clamp(0, 63).to(torch.int32)
    eff_s = df * isc.float()                          # [nb, 8]
    eff_m = dmf * im.float()
    safe = torch.where(eff_s > 0, eff_s, torch.ones_like(eff_s))
    q = torch.floor((b + eff_m[..., None]) / safe[..., None] + 0.5)
    q = torch.where(eff_s[..., None] > 0, q, torch.zeros_like(q)).clamp(0, 15).to(torch.int32)  # [nb, 8, 32]
    # 12 packed scale bytes (inverse of gguf-py Q4_K.get_scale_min).
    sc_lo, sc_hi = isc[:, :4], isc[:, 4:]
    m_lo, m_hi = im[:, :4], im[:, 4:]
    s0 = (sc_lo & 63) | ((sc_hi >> 4) << 6)
    s1 = (m_lo & 63) | ((m_hi >> 4) << 6)
    s2 = (sc_hi & 15) | ((m_hi & 15) << 4)
    scales = torch.cat([s0, s1, s2], dim=1).to(torch.uint8)  # [nb, 12]
    # nibbles: byte 32*g + l = q[2g][l] | q[2g+1][l] << 4
    qq = q.reshape(nb, 4, 2, 32)
    qs = (qq[:, :, 0, :] | (qq[:, :, 1, :] << 4)).to(torch.uint8).reshape(nb, 128)
    hdr = torch.cat([d16.view(torch.uint8).reshape(nb, 2), dmin16.view(torch.uint8).reshape(nb, 2)], dim=1)
    out = torch.cat([hdr, scales, qs], dim=1)
    return out.reshape(*lead, -1)


def to_bf16_bytes(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).view(torch.uint8).reshape(*x.shape[:-1], -1)


def quantize(x: torch.Tensor, gtype: int) -> torch.Tensor:
    from . import TYPE_BF16, TYPE_F16, TYPE_F32, TYPE_Q4_K, TYPE_Q8_0
    if gtype == TYPE_Q8_0:
        return quantize_q8_0(x)
    if gtype == TYPE_Q4_K:
        return quantize_q4_k(x)
    if gtype == TYPE_BF16:
        return to_bf16_bytes(x)
    if gtype == TYPE_F16:
        return x.to(torch.float16).view(torch.uint8).reshape(*x.shape[:-1], -1)
    if gtype == TYPE_F32:
        return x.contiguous().view(torch.uint8).reshape(*x.shape[:-1], -1)
    raise ValueError(f"unsupported ggml type {gtype}")
