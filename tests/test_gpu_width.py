"""GPU parity tests at the benchmarked widths (hidden 3072, 24 heads x 128).

* BASELINE config 1 (the configuration the north star pins parity on):
  2 double-stream + 4 single-stream blocks, 1024 image tokens (32 x 32 grid)
  + 256 text tokens of 3072 features, Q8_0 weights from seed 0, one
  denoising step at sigma = 0.5 with dt = -0.25, in the shape of the
  reference's test_multiple_blocks
  (test/src/diffusers/models/transformers/flux2/Flux2Transformer2DModel.py:149).
* A full-width slice of config 2: 1 double + 1 single block over 4096 image
  + 512 text tokens (7680 text features), Q4_K weights.

The GPU path (C ABI, bf16 operands, f32 accumulation) is compared with the
float64 restatement in oracle/flux2_oracle.py.  The oracle runs its float64
arithmetic on the GPU (torch's float64 kernels) only to finish in seconds;
its weights come from the C dequantisation oracle.  Bars: per-step latent
relative L2 <= 1e-2 (the north star's), noise prediction <= 1e-2 (measured
2.4-2.7e-3 on a B200); max-abs errors are printed."""
import pytest
import torch

import dcpp_b200
import flux2_oracle as fo
from dcpp_b200 import synth

pytestmark = pytest.mark.gpu

LAT_TOL = 1e-2
V_TOL = 1e-2


def oracle_cfg(c):
    return fo.Config(**{k: getattr(c, k) for k in fo.Config.__dataclass_fields__})


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm()).item()


def maxabs(a, b):
    return (a.double().cpu() - b.double().cpu()).abs().max().item()


def run_case(ctx, c, wtype, gh, gw, nt, sigma, dt, seed=0):
    params = synth.make_params(c, wtype, seed=seed, device="cuda")
    torch.cuda.empty_cache()
    hid, enc, iid, tid = synth.make_inputs(c, 1, gh, gw, nt, seed=1)
    ni = gh * gw
    m = dcpp_b200.Flux2Model(ctx, c)
    m.load_params(params)
    m.prepare(1, ni, nt, use_graph=True)
    t = torch.tensor([sigma], dtype=torch.float32)
    v = torch.empty(1, ni, c.in_channels)
    lat = torch.empty(1, ni, c.in_channels)
    m.forward(hid, enc, t, iid, tid, v)
    m.denoise_step(hid, enc, t, dt, iid, tid, lat)
    m.close()
    torch.cuda.empty_cache()
    orc = fo.Flux2Oracle(oracle_cfg(c), params, keep_weights=False, device="cuda")
    v_ref = orc.forward(hid, enc, t, iid, tid).cpu()
    lat_ref = hid.double() + dt * v_ref
    del orc
    torch.cuda.empty_cache()
    return v, lat, v_ref, lat_ref


def test_config1_denoise_step_matches_oracle(ctx):
    """D 3072, 24 x 128 heads, 2 double + 4 single blocks,
    1024 + 256 tokens, jd 3072, Q8_0, one step at sigma 0.5, dt -0.25."""
    c = synth.Flux2Cfg(num_layers=2, num_single_layers=4, num_attention_heads=24, joint_attention_dim=3072,
                       in_channels=128, guidance_embeds=False)
    v, lat, v_ref, lat_ref = run_case(ctx, c, fo.GGML_Q8_0, 32, 32, 256, 0.5, -0.25)
    rv, rl = rel(v, v_ref), rel(lat, lat_ref)
    print(f"config 1: noise prediction rel-L2 {rv:.3e} max-abs {maxabs(v, v_ref):.3e}; "
          f"latent rel-L2 {rl:.3e} max-abs {maxabs(lat, lat_ref):.3e}")
    assert rl <= LAT_TOL, (rl, maxabs(lat, lat_ref))
    assert rv <= V_TOL, (rv, maxabs(v, v_ref))


def test_config2_slice_denoise_step_matches_oracle(ctx):
    """Full-width config-2 slice: D 3072, 1 double + 1 single block, 4096 +
    512 tokens, jd 7680, Q4_K, a step at sigma 0.75 (dt -0.25)."""
    c = synth.Flux2Cfg(num_layers=1, num_single_layers=1, num_attention_heads=24, joint_attention_dim=7680,
                       in_channels=128, guidance_embeds=False)
    v, lat, v_ref, lat_ref = run_case(ctx, c, fo.GGML_Q4_K, 64, 64, 512, 0.75, -0.25, seed=3)
    rv, rl = rel(v, v_ref), rel(lat, lat_ref)
    print(f"config 2 slice: noise prediction rel-L2 {rv:.3e} max-abs {maxabs(v, v_ref):.3e}; "
          f"latent rel-L2 {rl:.3e} max-abs {maxabs(lat, lat_ref):.3e}")
    assert rl <= LAT_TOL, (rl, maxabs(lat, lat_ref))
    assert rv <= V_TOL, (rv, maxabs(v, v_ref))
