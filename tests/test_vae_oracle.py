"""The VAE-decode oracle on CPU (no GPU): its latent unpack / unpatchify
against a literal transcription of the reference's reshape / permute
sequence, the nearest-2x-upsample + 3x3-conv identity the GPU path relies on
(four 2x2 phase convolutions with summed taps), and the tiled decode's
blending against the untiled decode where they must agree."""
import math

import pytest
import torch
import torch.nn.functional as F

import vae_oracle as vo
from dcpp_b200 import synth


def reference_unpatchify(packed, ph, pw, C):
    """Flux2KleinPipeline::unpack_latents + unpatchify_latents
    (Flux2KleinPipeline.cpp:606-630), step by step."""
    B = packed.shape[0]
    t = packed.permute(0, 2, 1).contiguous().reshape(B, 4 * C, ph, pw)
    N = ph * pw
    t = t.reshape(B, 4 * C, N).reshape(B, 2 * C, 2, N).permute(0, 1, 3, 2).contiguous()
    t = t.reshape(B, 2 * C, ph, 2 * pw).reshape(B * C, 2, ph, 2 * pw).permute(0, 2, 1, 3).contiguous()
    return t.reshape(B, C, 2 * ph, 2 * pw)


@pytest.mark.parametrize("ph,pw", [(2, 3), (4, 4)])
def test_unpatchify_matches_reference_sequence(ph, pw):
    C = 32
    g = torch.Generator().manual_seed(0)
    lat = torch.randn(2, ph * pw, 4 * C, generator=g, dtype=torch.float64)
    mean = torch.zeros(4 * C, dtype=torch.float64)
    var = torch.ones(4 * C, dtype=torch.float64) - 1e-4
    got = vo.unpack_unpatchify(lat, mean, var, 1e-4, ph, pw, C)
    assert torch.allclose(got, reference_unpatchify(lat, ph, pw, C), rtol=0, atol=1e-12)


def phase_tap(a, k):
    """Offset, within the (a - 1, a) window of the low-resolution image, of the
    row that tap k of the 3x3 conv reads at output phase a (the rule the
    library applies when it builds the phase weights)."""
    return math.floor((a + k - 1) / 2) - (a - 1)


def test_upsample_conv_equals_four_phase_convs():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 5, 6, 7, generator=g, dtype=torch.float64)
    w = torch.randn(4, 5, 3, 3, generator=g, dtype=torch.float64)
    ref = F.conv2d(F.interpolate(x, scale_factor=2.0, mode="nearest"), w, padding=1)
    out = torch.zeros_like(ref)
    for a in range(2):
        for b in range(2):
            wp = torch.zeros(4, 5, 2, 2, dtype=torch.float64)
            for ky in range(3):
                for kx in range(3):
                    wp[:, :, phase_tap(a, ky), phase_tap(b, kx)] += w[:, :, ky, kx]
            # taps at row offsets (a - 1, a), column offsets (b - 1, b)
            xp = F.pad(x, (1 - b, b, 1 - a, a))
            out[:, :, a::2, b::2] = F.conv2d(xp, wp)
    assert torch.allclose(out, ref, rtol=0, atol=1e-10)


def small_cfg(**kw):
    base = dict(block_out_channels=(64, 128, 128), layers_per_block=1, norm_num_groups=32)
    base.update(kw)
    return synth.VAECfg(**base)


def oracle(c, params):
    return vo.VAEDecoderOracle(vo.VAEConfig(**{k: getattr(c, k) for k in (
        "in_channels", "out_channels", "block_out_channels", "layers_per_block", "latent_channels",
        "norm_num_groups", "batch_norm_eps", "use_post_quant_conv", "mid_block_add_attention")}), params)


def test_oracle_decode_shapes_and_tiling():
    c = small_cfg()
    params = synth.make_vae_params(c, seed=5)
    o = oracle(c, params)
    lat = synth.make_vae_latents(c, 1, 4, 6, seed=6)
    img = o.decode_packed(lat, 4, 6)
    assert img.shape == (1, 3, 4 * 2 * 4, 6 * 2 * 4)
    assert torch.isfinite(img).all()
    # A tile covering the whole image reproduces the untiled decode.
    big = o.decode_packed(lat, 4, 6, tile=64)
    assert torch.allclose(big, img, rtol=0, atol=1e-12)
    # Overlapping tiles: same shape, blended seams, close to the untiled decode
    # away from the borders the tiles cut.
    tiled = o.decode_packed(lat, 4, 6, tile=16)
    assert tiled.shape == img.shape and torch.isfinite(tiled).all()
