"""The Flux2 oracle's hand-written primitives (oracle/flux2_oracle.py)
checked against PyTorch's own implementations, which the reference's Python
tests reach through HF diffusers: LayerNorm without affine (ggml_norm),
RMSNorm with weight, SiLU, scaled-dot-product attention, and the rotary
embedding against a complex-number rotation of the same (cos, sin) table.
CPU only, float64."""
import math

import pytest
import torch
import torch.nn.functional as F

import flux2_oracle as fo


def rnd(*shape, seed=0, scale=1.0, shift=0.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g, dtype=torch.float64) * scale + shift


@pytest.mark.parametrize("D,eps", [(3072, 1e-6), (128, 1e-5), (7, 1e-6)])
def test_layer_norm_matches_torch(D, eps):
    x = rnd(5, D, seed=D, scale=3.0, shift=1.5)
    ref = F.layer_norm(x, (D,), eps=eps)
    assert torch.allclose(fo.layer_norm(x, eps), ref, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("D", [128, 2560])
def test_rms_norm_matches_torch(D):
    x = rnd(4, 3, D, seed=1, scale=2.0)
    w = rnd(D, seed=2, scale=0.1, shift=1.0)
    ref = F.rms_norm(x, (D,), w, eps=1e-6)
    assert torch.allclose(fo.rms_norm(x, w, 1e-6), ref, rtol=1e-12, atol=1e-12)


def test_silu_matches_torch():
    x = rnd(1000, seed=3, scale=6.0)
    assert torch.allclose(fo.silu(x), F.silu(x), rtol=1e-14, atol=1e-14)


@pytest.mark.parametrize("B,S,H,d", [(1, 33, 2, 128), (2, 200, 3, 64)])
def test_sdpa_matches_torch(B, S, H, d):
    q, k, v = (rnd(B, S, H, d, seed=s) for s in (4, 5, 6))
    ref = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
    assert torch.allclose(fo.sdpa(q, k, v), ref, rtol=1e-10, atol=1e-12)


def test_rope_matches_complex_rotation():
    """Pair (x_2i, x_2i+1) as the complex number x_2i + i x_2i+1, multiplied
    by exp(i * pos_a * theta^(-2p / axes_dims[a])) per axis section."""
    S, H, axes, theta = 37, 2, (32, 32, 32, 32), 2000.0
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, 64, (S, 4), generator=g, dtype=torch.int32)
    x = rnd(1, S, H, sum(axes), seed=8)
    cos, sin = fo.rope_cos_sin(ids, axes, theta, torch.float64)
    got = fo.apply_rope(x, cos, sin)
    ang = []
    for a, nd in enumerate(axes):
        p = torch.arange(nd // 2, dtype=torch.float64)
        ang.append(ids[:, a].double()[:, None] * theta ** (-2.0 * p / nd)[None, :])
    rot = torch.polar(torch.ones(S, sum(axes) // 2, dtype=torch.float64), torch.cat(ang, dim=-1))
    xc = torch.view_as_complex(x.reshape(1, S, H, -1, 2).contiguous())
    ref = torch.view_as_real(xc * rot[None, :, None, :]).flatten(-2)
    assert torch.allclose(got, ref, rtol=1e-12, atol=1e-12)


def test_timestep_features_match_sinusoidal_formula():
    """flip_sin_to_cos = True, downscale_freq_shift = 0, max period 10^4:
    [cos(t w_j), sin(t w_j)] with w_j = exp(-ln(10^4) j / half)."""
    t = torch.tensor([0.0, 1.0, 500.0, 999.0], dtype=torch.float64)
    C = 256
    half = C // 2
    w = torch.tensor([math.exp(-math.log(10000.0) * j / half) for j in range(half)], dtype=torch.float64)
    ref = torch.cat([torch.cos(t[:, None] * w), torch.sin(t[:, None] * w)], dim=-1)
    assert torch.allclose(fo.timestep_proj(t, C), ref, rtol=1e-12, atol=1e-12)
