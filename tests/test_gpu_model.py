"""GPU parity tests of the model-level C ABI (Flux2Transformer2DModel::forward
and the denoise step) against the float64 CPU oracle, on reduced configs in
the shape of the reference's own tests (1-2 double / single blocks, small
token counts, ragged text lengths) plus error paths."""
import numpy as np
import pytest
import torch

import dcpp_b200
import flux2_oracle as fo
from dcpp_b200 import synth

pytestmark = pytest.mark.gpu

# Noise-prediction tolerance (relative L2 vs the float64 oracle): the GPU path
# rounds GEMM operands to bf16 and accumulates in f32.
V_TOL = 3e-2
# Latent tolerance after one Euler step (the north star's 1e-2 bar).
LAT_TOL = 1e-2


def cfg_small(**kw):
    base = dict(num_layers=1, num_single_layers=1, num_attention_heads=2, attention_head_dim=128,
                joint_attention_dim=64, in_channels=32, timestep_guidance_channels=256, guidance_embeds=False)
    base.update(kw)
    return synth.Flux2Cfg(**base)


def oracle_cfg(c):
    return fo.Config(**{k: getattr(c, k) for k in fo.Config.__dataclass_fields__})


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm()).item()


def build(ctx, c, wtype, seed=0, split=False, graph=True, B=1, gh=4, gw=4, nt=8):
    params = synth.make_params(c, wtype, seed=seed, split=split)
    m = dcpp_b200.Flux2Model(ctx, c)
    m.load_params(params)
    m.prepare(B, gh * gw, nt, use_graph=graph)
    return m, params


@pytest.mark.parametrize("wtype", [fo.GGML_Q8_0, fo.GGML_Q4_K])
def test_forward_matches_oracle(ctx, wtype):
    c = cfg_small()
    m, params = build(ctx, c, wtype)
    hid, enc, iid, tid = synth.make_inputs(c, 1, 4, 4, 8, seed=3)
    t = torch.tensor([0.5], dtype=torch.float32)
    out = torch.empty(1, 16, c.in_channels, dtype=torch.float32)
    m.forward(hid, enc, t, iid, tid, out)
    ref = fo.Flux2Oracle(oracle_cfg(c), params).forward(hid, enc, t, iid, tid)
    r = rel(out, ref)
    assert r < V_TOL, r


@pytest.mark.parametrize("wtype", [fo.GGML_Q8_0, fo.GGML_Q4_K])
def test_forward_fused_dequant_matches_oracle(ctx, monkeypatch, wtype):
    """The block projections run on the fused-dequant GEMM (weights packed at load)."""
    monkeypatch.setenv("DCPP_FUSED_DEQUANT", "1")
    c = cfg_small(num_layers=2, num_single_layers=2)
    m, params = build(ctx, c, wtype, seed=21, gh=16, gw=16, nt=40)
    hid, enc, iid, tid = synth.make_inputs(c, 1, 16, 16, 40, seed=22)
    t = torch.tensor([0.6], dtype=torch.float32)
    out = torch.empty(1, 256, c.in_channels, dtype=torch.float32)
    m.forward(hid, enc, t, iid, tid, out)
    ref = fo.Flux2Oracle(oracle_cfg(c), params).forward(hid, enc, t, iid, tid)
    r = rel(out, ref)
    assert r < V_TOL, r


@pytest.mark.parametrize("attn", [1, 2], ids=["one_tile", "two_tiles"])
def test_forward_each_attention_kernel(ctx, attn):
    """The model with each attention kernel forced (auto picks by grid size)."""
    c = cfg_small(num_layers=1, num_single_layers=2)
    ctx.set_attention_kernel(attn)
    try:
        m, params = build(ctx, c, fo.GGML_Q8_0, seed=23, gh=12, gw=20, nt=37)
        hid, enc, iid, tid = synth.make_inputs(c, 1, 12, 20, 37, seed=24)
        t = torch.tensor([0.45], dtype=torch.float32)
        out = torch.empty(1, 240, c.in_channels, dtype=torch.float32)
        m.forward(hid, enc, t, iid, tid, out)
        m.close()
    finally:
        ctx.set_attention_kernel(0)
    ref = fo.Flux2Oracle(oracle_cfg(c), params).forward(hid, enc, t, iid, tid)
    r = rel(out, ref)
    assert r < V_TOL, r


def test_forward_batch2_ragged_text_guidance(ctx):
    c = cfg_small(num_layers=2, num_single_layers=2, guidance_embeds=True)
    m, params = build(ctx, c, fo.GGML_Q8_0, seed=4, B=2, gh=10, gw=13, nt=131)
    hid, enc, iid, tid = synth.make_inputs(c, 2, 10, 13, 131, seed=5)
    t = torch.tensor([0.8, 0.3], dtype=torch.float32)
    guid = torch.tensor([2.0, 3.5], dtype=torch.float32)
    out = torch.empty(2, 130, c.in_channels, dtype=torch.float32)
    m.forward(hid, enc, t, iid, tid, out, guidance=guid)
    ref = fo.Flux2Oracle(oracle_cfg(c), params).forward(hid, enc, t, iid, tid, guidance=guid)
    for b in range(2):
        r = rel(out[b], ref[b])
        assert r < V_TOL, (b, r)


def test_split_and_fused_names_give_identical_results(ctx):
    c = cfg_small()
    fused = synth.make_params(c, fo.GGML_Q8_0, seed=9)
    D, F = c.inner_dim, c.mlp_hidden
    split = {}
    for name, (gt, shp, data) in fused.items():
        raw = data.numpy()
        if name.endswith("to_qkv_mlp_proj.weight"):
            rb = fo.row_bytes(gt, shp[1])
            r = raw.reshape(shp[0], rb)
            p = name[: -len("weight")]
            for sub, (a, b) in {"q": (0, D), "k": (D, 2 * D), "v": (2 * D, 3 * D),
                                "mlp_in_gate": (3 * D, 3 * D + F), "mlp_in_up": (3 * D + F, 3 * D + 2 * F)}.items():
                split[p + sub + ".weight"] = (gt, (b - a, shp[1]), r[a:b].copy())
        elif name.endswith("attn.to_out.weight"):
            rb = fo.row_bytes(gt, shp[1])
            r = raw.reshape(shp[0], rb)
            ca = fo.row_bytes(gt, D)
            p = name[: -len("weight")]
            split[p + "attn.weight"] = (gt, (D, D), r[:, :ca].copy())
            split[p + "mlp.weight"] = (gt, (D, F), r[:, ca:].copy())
        elif name.endswith("linear_in.weight"):
            rb = fo.row_bytes(gt, shp[1])
            r = raw.reshape(shp[0], rb)
            p = name[: -len("linear_in.weight")]
            split[p + "linear_in_gate.weight"] = (gt, (F, D), r[:F].copy())
            split[p + "linear_in_up.weight"] = (gt, (F, D), r[F:].copy())
        else:
            split[name] = (gt, shp, raw)
    hid, enc, iid, tid = synth.make_inputs(c, 1, 3, 5, 9, seed=2)
    t = torch.tensor([0.25])
    outs = []
    for params in (fused, split):
        m = dcpp_b200.Flux2Model(ctx, c)
        m.load_params(params)
        m.prepare(1, 15, 9)
        o = torch.empty(1, 15, c.in_channels)
        m.forward(hid, enc, t, iid, tid, o)
        outs.append(o)
        m.close()
    assert torch.equal(outs[0], outs[1])


def test_graph_and_eager_agree_bitwise(ctx):
    c = cfg_small()
    hid, enc, iid, tid = synth.make_inputs(c, 1, 4, 4, 8, seed=3)
    t = torch.tensor([0.5])
    outs = []
    for graph in (True, False):
        m, _ = build(ctx, c, fo.GGML_Q4_K, graph=graph)
        o = torch.empty(1, 16, c.in_channels)
        m.forward(hid, enc, t, iid, tid, o)
        m.forward(hid, enc, t, iid, tid, o)  # second call replays the graph
        outs.append(o)
        m.close()
    assert torch.equal(outs[0], outs[1])


def test_denoise_step_latent_within_1e2(ctx):
    c = cfg_small(num_layers=2, num_single_layers=2)
    m, params = build(ctx, c, fo.GGML_Q4_K, seed=11, gh=8, gw=8, nt=40)
    hid, enc, iid, tid = synth.make_inputs(c, 1, 8, 8, 40, seed=12)
    t = torch.tensor([0.75])
    out = torch.empty_like(hid)
    m.denoise_step(hid, enc, t, -0.25, iid, tid, out)
    ref = fo.Flux2Oracle(oracle_cfg(c), params).denoise(hid, enc, t, -0.25, iid, tid)
    r = rel(out, ref)
    maxabs = (out.double() - ref).abs().max().item()
    assert r < LAT_TOL, (r, maxabs)


def test_resident_schedule_matches_oracle(ctx):
    c = cfg_small()
    m, params = build(ctx, c, fo.GGML_Q8_0, seed=13, gh=4, gw=6, nt=16)
    hid, enc, iid, tid = synth.make_inputs(c, 1, 4, 6, 16, seed=14)
    ts, sg = dcpp_b200.flow_match_schedule(4)
    m.load_inputs(hid, enc, iid, tid)
    for i in range(4):
        m.set_timestep(float(ts[i]) / 1000.0, float(sg[i + 1] - sg[i]))
        m.run_resident()
    out = torch.empty_like(hid)
    m.read_latents(out)
    o = fo.Flux2Oracle(oracle_cfg(c), params)
    x = hid.double()
    for i in range(4):
        x = o.denoise(x, enc, torch.tensor([float(ts[i]) / 1000.0]), float(sg[i + 1] - sg[i]), iid, tid)
    r = rel(out, x)
    assert r < LAT_TOL, r


def test_missing_parameter_is_a_state_error(ctx):
    c = cfg_small()
    params = synth.make_params(c, fo.GGML_Q8_0)
    m = dcpp_b200.Flux2Model(ctx, c)
    for name, (gt, shp, data) in params.items():
        if name != "proj_out.weight":
            m.set_param(name, gt, shp, data)
    n, first = m.missing()
    assert n == 1 and first == "proj_out.weight"
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.prepare(1, 4, 4)
    assert e.value.status == 7 and "proj_out.weight" in str(e.value)


def test_bad_shape_and_unknown_name(ctx):
    c = cfg_small()
    m = dcpp_b200.Flux2Model(ctx, c)
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.set_param("x_embedder.weight", fo.GGML_BF16, (256, 31), np.zeros(256 * 31 * 2, np.uint8))
    assert e.value.status == 1 and "shape mismatch" in str(e.value)
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.set_param("x_embedder.bias", fo.GGML_F32, (256,), np.zeros(1024, np.uint8))
    assert e.value.status == 8


def test_injected_fault_surfaces_as_error_then_recovers(ctx):
    c = cfg_small()
    m, params = build(ctx, c, fo.GGML_Q8_0)
    hid, enc, iid, tid = synth.make_inputs(c, 1, 4, 4, 8, seed=3)
    t = torch.tensor([0.5])
    out = torch.empty(1, 16, c.in_channels)
    ctx.inject_fault("dcpp_flux2_forward", 1)
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.forward(hid, enc, t, iid, tid, out)
    assert e.value.status == 9
    m.forward(hid, enc, t, iid, tid, out)
    assert torch.isfinite(out).all()


def make_ref_tokens(c, B, n_ref, seed):
    """Reference-image latents [B, n_ref, C] and ids [n_ref, 4] on a second
    time coordinate (T = 10), as the pipeline's prepare_image_latents gives
    its first reference image."""
    g = torch.Generator().manual_seed(seed)
    lat = torch.randn(B, n_ref, c.in_channels, generator=g)
    ids = torch.zeros(n_ref, len(c.axes_dims_rope), dtype=torch.int32)
    ids[:, 0] = 10
    ids[:, 1] = torch.arange(n_ref, dtype=torch.int32) // 4
    ids[:, 2] = torch.arange(n_ref, dtype=torch.int32) % 4
    return lat, ids


@pytest.mark.parametrize("B", [1, 2])
def test_denoise_with_ref_images_matches_oracle(ctx, B):
    """Flux2KleinPipeline::denoise with image_latents (Flux2KleinPipeline.cpp:511-536),
    in the shape of test_denoise_with_ref_images
    (test/src/diffusers/pipelines/flux2/Flux2KleinPipeline.py:500-734): a 2 x 3
    packed latent grid, 12 reference tokens, one step."""
    c = cfg_small()
    params = synth.make_params(c, fo.GGML_Q8_0, seed=31)
    hid, enc, iid, tid = synth.make_inputs(c, B, 2, 3, 16, seed=32)
    ref_lat, ref_ids = make_ref_tokens(c, B, 12, seed=33)
    m = dcpp_b200.Flux2Model(ctx, c)
    m.load_params(params)
    m.prepare(B, 6, 16, n_ref=12)
    t = torch.full((B,), 1.0)
    out = torch.full_like(hid, float("nan"))
    m.denoise_step(hid, enc, t, -1.0, iid, tid, out, image_latents=ref_lat, image_latent_ids=ref_ids)
    o = fo.Flux2Oracle(oracle_cfg(c), params)
    ref = o.denoise(hid, enc, t, -1.0, iid, tid, image_latents=ref_lat, image_latent_ids=ref_ids)
    r = rel(out, ref)
    assert r < LAT_TOL, (r, (out.double() - ref).abs().max().item())
    # The reference tokens change the result (they are attended to), by far
    # more than the GPU path's error.
    plain = o.denoise(hid, enc, t, -1.0, iid, tid)
    assert rel(plain, ref) > 2 * LAT_TOL and r < rel(plain, ref) / 5, (rel(plain, ref), r)
    m.close()


def test_forward_on_ref_plan_returns_every_image_token(ctx):
    """forward() on a plan with reference tokens takes the concatenated
    image tokens and returns all of their predictions, as the reference's
    forward does (it slices nothing, Flux2Transformer2DModel.cpp:217-230)."""
    c = cfg_small()
    params = synth.make_params(c, fo.GGML_Q8_0, seed=34)
    hid, enc, iid, tid = synth.make_inputs(c, 1, 2, 3, 16, seed=35)
    ref_lat, ref_ids = make_ref_tokens(c, 1, 12, seed=36)
    x = torch.cat([hid, ref_lat], dim=1).contiguous()
    ids = torch.cat([iid, ref_ids], dim=0).contiguous()
    m = dcpp_b200.Flux2Model(ctx, c)
    m.load_params(params)
    m.prepare(1, 6, 16, n_ref=12)
    t = torch.tensor([0.5])
    out = torch.empty(1, 18, c.in_channels)
    m.forward(x, enc, t, ids, tid, out)
    ref = fo.Flux2Oracle(oracle_cfg(c), params).forward(x, enc, t, ids, tid)
    assert rel(out, ref) < V_TOL
    m.close()


def test_resident_schedule_with_ref_images(ctx):
    """Two resident steps with reference tokens: the reference latents stay
    fixed while the latent tokens follow the schedule."""
    c = cfg_small()
    params = synth.make_params(c, fo.GGML_Q4_K, seed=37)
    hid, enc, iid, tid = synth.make_inputs(c, 1, 4, 4, 8, seed=38)
    ref_lat, ref_ids = make_ref_tokens(c, 1, 8, seed=39)
    m = dcpp_b200.Flux2Model(ctx, c)
    m.load_params(params)
    m.prepare(1, 16, 8, n_ref=8)
    ts, sg = dcpp_b200.flow_match_schedule(2)
    m.load_inputs(hid, enc, iid, tid, image_latents=ref_lat, image_latent_ids=ref_ids)
    for i in range(2):
        m.set_timestep(float(ts[i]) / 1000.0, float(sg[i + 1] - sg[i]))
        m.run_resident()
    out = torch.empty_like(hid)
    m.read_latents(out)
    o = fo.Flux2Oracle(oracle_cfg(c), params)
    x = hid.double()
    for i in range(2):
        x = o.denoise(x, enc, torch.tensor([float(ts[i]) / 1000.0]), float(sg[i + 1] - sg[i]), iid, tid,
                      image_latents=ref_lat.double(), image_latent_ids=ref_ids)
    r = rel(out, x)
    assert r < LAT_TOL, r
    m.close()


def test_ref_plan_rejects_calls_without_ref_inputs(ctx):
    c = cfg_small()
    m, _ = build(ctx, c, fo.GGML_Q8_0)
    hid, enc, iid, tid = synth.make_inputs(c, 1, 4, 4, 8, seed=3)
    ref_lat, ref_ids = make_ref_tokens(c, 1, 4, seed=40)
    out = torch.empty_like(hid)
    t = torch.tensor([0.5])
    # a plan without reference tokens refuses reference inputs
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.denoise_step(hid, enc, t, -0.25, iid, tid, out, image_latents=ref_lat, image_latent_ids=ref_ids)
    assert e.value.status == 1
    m.prepare(1, 16, 8, n_ref=4)
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.denoise_step(hid, enc, t, -0.25, iid, tid, out)
    assert e.value.status == 1 and "reference tokens" in str(e.value)
    m.denoise_step(hid, enc, t, -0.25, iid, tid, out, image_latents=ref_lat, image_latent_ids=ref_ids)
    assert torch.isfinite(out).all()
    m.close()
