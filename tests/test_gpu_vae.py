"""GPU parity tests of the Flux2 VAE decode (dcpp_vae_*) against the float64
oracle (oracle/vae_oracle.py): implicit-GEMM 3x3 / 1x1 convolutions,
GroupNorm (+ SiLU), the mid-block attention, the phase-decomposed 2x
upsample, latent unpack / BatchNorm / unpatchify, on reduced configs and
ragged image sizes (partial pixel rectangles), batch 1 and 2; graph vs
eager; GGUF loading of a full VAE checkpoint; error paths."""
import json
from dataclasses import asdict

import pytest
import torch

import dcpp_b200
import vae_oracle as vo
from dcpp_b200 import synth
from gguf_util import write_gguf

pytestmark = pytest.mark.gpu

# Image tolerance (relative L2 vs the float64 oracle): bf16 conv / attention
# operands with f32 accumulation, f32 residual stream.
IMG_TOL = 1e-2


def rel(a, b):
    a, b = torch.as_tensor(a).double().cpu(), torch.as_tensor(b).double().cpu()
    return ((a - b).norm() / b.norm()).item()


def oracle(c, params):
    return vo.VAEDecoderOracle(vo.VAEConfig(**{k: getattr(c, k) for k in (
        "in_channels", "out_channels", "block_out_channels", "layers_per_block", "latent_channels",
        "norm_num_groups", "batch_norm_eps", "use_post_quant_conv", "mid_block_add_attention")}), params)


def run(ctx, c, params, B, ph, pw, graph=True, seed=3):
    m = dcpp_b200.VAEModel(ctx, c)
    m.load_params(params)
    m.prepare(B, ph, pw, use_graph=graph)
    lat = synth.make_vae_latents(c, B, ph, pw, seed=seed)
    s = 2 ** (len(c.block_out_channels) - 1)
    img = torch.empty(B, c.out_channels, 2 * ph * s, 2 * pw * s, dtype=torch.float32)
    m.decode(lat, img)
    return m, lat, img


CASES = [
    # (block_out_channels, layers_per_block, B, ph, pw)
    ((64, 128, 128), 1, 1, 4, 4),
    ((64, 128, 128), 1, 2, 3, 5),      # ragged: widths 10, 20, 40 -> partial rectangles
    ((128, 128, 256, 256), 1, 1, 4, 8),
    ((64, 64), 2, 1, 9, 16),           # wide rows (W = 32, 64), shortcut-free
    ((64, 128, 128), 1, 1, 6, 40),     # W = 160, 320: halo patches with a partial last patch per row
]


@pytest.mark.parametrize("ch,lpb,B,ph,pw", CASES)
def test_decode_matches_oracle(ctx, ch, lpb, B, ph, pw):
    c = synth.VAECfg(block_out_channels=ch, layers_per_block=lpb)
    params = synth.make_vae_params(c, seed=11)
    m, lat, img = run(ctx, c, params, B, ph, pw)
    m.close()
    ref = oracle(c, params).decode_packed(lat, ph, pw)
    r = rel(img, ref)
    err = (img.double() - ref).abs().max().item()
    assert r < IMG_TOL, (r, err)


@pytest.mark.parametrize("ph,pw,tile", [(8, 12, 32), (9, 6, 48), (4, 4, 64)])
def test_tiled_decode_matches_oracle(ctx, ph, pw, tile):
    """decode_tiled: ragged tile rows / columns (tiles clipped at the image
    border, a non-last clipped row), blending with the upper and left
    neighbours; a tile covering the image equals the untiled decode."""
    c = synth.VAECfg(block_out_channels=(64, 128, 128), layers_per_block=1)
    params = synth.make_vae_params(c, seed=17)
    m = dcpp_b200.VAEModel(ctx, c)
    m.load_params(params)
    m.prepare(1, ph, pw, tile_size=tile)
    lat = synth.make_vae_latents(c, 1, ph, pw, seed=18)
    img = torch.empty(1, 3, 8 * ph, 8 * pw, dtype=torch.float32)
    m.decode(lat, img)
    o = oracle(c, params)
    ref = o.decode_packed(lat, ph, pw, tile=tile)
    assert ref.shape == img.shape
    r = rel(img, ref)
    assert r < IMG_TOL, r
    if tile >= 8 * max(ph, pw) * 2:
        m.prepare(1, ph, pw)
        whole = torch.empty_like(img)
        m.decode(lat, whole)
        assert torch.equal(whole, img)
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.prepare(1, ph, pw, tile_size=30)
    assert "divisible by the VAE's scale factor" in str(e.value)
    m.close()


def test_decode_without_attention_and_post_quant(ctx):
    c = synth.VAECfg(block_out_channels=(64, 128), layers_per_block=1, use_post_quant_conv=False,
                     mid_block_add_attention=False)
    params = synth.make_vae_params(c, seed=12)
    m, lat, img = run(ctx, c, params, 1, 6, 6)
    m.close()
    assert rel(img, oracle(c, params).decode_packed(lat, 6, 6)) < IMG_TOL


def test_graph_and_eager_agree_bitwise(ctx):
    c = synth.VAECfg(block_out_channels=(64, 128, 128), layers_per_block=1)
    params = synth.make_vae_params(c, seed=13)
    a, _, img_a = run(ctx, c, params, 1, 4, 6, graph=True)
    b, _, img_b = run(ctx, c, params, 1, 4, 6, graph=False)
    a.close()
    b.close()
    assert torch.equal(img_a, img_b)


def test_from_pretrained_full_checkpoint(ctx, tmp_path):
    """A VAE folder (config.json + GGUF) holding encoder tensors too: they
    are skipped, the decode matches set_param bitwise."""
    c = synth.VAECfg(block_out_channels=(64, 128, 128), layers_per_block=1)
    params = synth.make_vae_params(c, seed=14)
    file_params = dict(params)
    file_params["encoder.conv_in.weight"] = (0, (64, 3, 3, 3), torch.zeros(64 * 27 * 4, dtype=torch.uint8))
    file_params["quant_conv.bias"] = (0, (64,), torch.zeros(64 * 4, dtype=torch.uint8))
    d = tmp_path / "vae"
    d.mkdir()
    cfg = asdict(c)
    cfg["block_out_channels"] = list(c.block_out_channels)
    cfg["patch_size"] = [2, 2]
    (d / "config.json").write_text(json.dumps(cfg))
    write_gguf(d / "diffusion_pytorch_model.gguf", file_params, arch="vae")
    m = dcpp_b200.VAEModel.from_pretrained(ctx, d)
    m.prepare(1, 4, 4)
    lat = synth.make_vae_latents(c, 1, 4, 4, seed=15)
    img = torch.empty(1, 3, 32, 32, dtype=torch.float32)
    m.decode(lat, img)
    m.close()
    ref_m, _, ref_img = run(ctx, c, params, 1, 4, 4, seed=15)
    ref_m.close()
    assert torch.equal(img, ref_img)
    g = dcpp_b200.VAEModel(ctx, c)
    assert g.load_gguf(d) == (len(params), 2)
    g.close()


def test_errors(ctx):
    c = synth.VAECfg(block_out_channels=(64, 128), layers_per_block=1)
    params = synth.make_vae_params(c, seed=16)
    m = dcpp_b200.VAEModel(ctx, c)
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.prepare(1, 4, 4)
    assert e.value.status == 7  # parameters missing
    name = "decoder.conv_in.weight"
    gt, shape, data = params[name]
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.set_param(name, gt, (shape[0], shape[1], 1, 9), data)
    assert "shape mismatch" in str(e.value)
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.set_param("encoder.conv_in.weight", gt, shape, data)
    assert e.value.status == 8
    m.close()
