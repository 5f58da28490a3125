"""GPU parity tests of the Qwen3 text-encoder prefill (dcpp_qwen3_*) against
the float64 oracle (oracle/qwen3_oracle.py, itself pinned to HF transformers):
grouped-query causal attention over ragged prompt lengths, NEOX RoPE with
per-head q/k RMSNorm, SwiGLU MLP, hidden-state taps, error paths."""
import numpy as np
import pytest
import torch

import dcpp_b200
import qwen3_oracle as qo
from dcpp_b200 import synth

pytestmark = pytest.mark.gpu

# Hidden states are carried in f32 between layers; the GEMM / attention
# operands are bf16 with f32 accumulation.
H_TOL = 2e-2


def rel(a, b):
    a, b = torch.as_tensor(a).double().cpu(), torch.as_tensor(b).double().cpu()
    return ((a - b).norm() / b.norm()).item()


def build(ctx, c, seed, B, S, taps, wtype=dcpp_b200.TYPE_Q8_0, graph=True):
    params = synth.make_qwen3_params(c, wtype, seed=seed)
    m = dcpp_b200.Qwen3Model(ctx, c)
    m.load_params(params)
    m.prepare(B, S, taps, use_graph=graph)
    return m, params


def run(m, c, ids, n_taps):
    B, S = ids.shape
    last = torch.empty(B, S, c.hidden_size, dtype=torch.float32)
    taps = torch.empty(B, S, max(n_taps, 1) * c.hidden_size, dtype=torch.float32)
    m.forward(ids.contiguous(), last, taps if n_taps else None)
    return last, taps


@pytest.mark.parametrize("attn", [0, 1, 2], ids=["auto", "one_tile", "two_tiles"])
def test_prefill_matches_oracle(ctx, attn):
    c = synth.Qwen3Cfg(vocab_size=1000, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                       num_attention_heads=8, num_key_value_heads=2)
    B, S, taps = 3, 300, (0, 1, 2)
    ctx.set_attention_kernel(attn)
    try:
        m, params = build(ctx, c, seed=11, B=B, S=S, taps=taps)
        ids = synth.make_qwen3_ids(c, B, S, seed=12)
        last, tp = run(m, c, ids, len(taps))
        m.close()
    finally:
        ctx.set_attention_kernel(0)
    o = qo.Qwen3Oracle(qo.Qwen3Config(**c.__dict__), params)
    ref_last, ref_taps = o.forward(ids, taps=taps)
    assert rel(last, ref_last) < H_TOL, rel(last, ref_last)
    D = c.hidden_size
    for k, t in enumerate(taps):
        r = rel(tp[..., k * D:(k + 1) * D], ref_taps[t])
        assert r < H_TOL, (t, r)
    # the embedding tap is an exact copy of the dequantised rows
    assert rel(tp[..., :D], ref_taps[0]) < 1e-7


def test_prefill_right_padded_prompts_match_oracle(ctx):
    """Prompts padded on the right (the tokenizer's mask): padding keys are
    masked for every query."""
    c = synth.Qwen3Cfg(vocab_size=500, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2)
    B, S = 3, 200
    lengths = (200, 131, 7)
    m, params = build(ctx, c, seed=31, B=B, S=S, taps=(1,))
    ids = synth.make_qwen3_ids(c, B, S, seed=32)
    mask = torch.zeros(B, S)
    for b, n in enumerate(lengths):
        mask[b, :n] = 1
    last = torch.empty(B, S, c.hidden_size)
    tp = torch.empty(B, S, c.hidden_size)
    m.forward(ids, last, tp, attention_mask=mask)
    o = qo.Qwen3Oracle(qo.Qwen3Config(**c.__dict__), params)
    ref, ref_t = o.forward(ids, taps=(1,), attention_mask=mask)
    assert rel(last, ref) < H_TOL, rel(last, ref)
    assert rel(tp, ref_t[1]) < H_TOL
    # Without the mask the real tokens of a right-padded prompt are unchanged
    # (causal: they never see the later padding).
    m.forward(ids, last)
    assert rel(last[1, :131], ref[1, :131]) < H_TOL
    m.close()


def test_prefill_golden_config_and_graph_eager_bitwise(ctx):
    g = np.load(__file__.replace("test_gpu_qwen3.py", "golden/qwen3_golden.npz"))
    keys = ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
            "num_key_value_heads", "head_dim")
    c = synth.Qwen3Cfg(**dict(zip(keys, (int(v) for v in g["config"]))))
    ids = torch.from_numpy(g["ids"])
    B, S = ids.shape
    outs = []
    for graph in (True, False):
        m, _ = build(ctx, c, seed=int(g["seed"][0]), B=B, S=S, taps=(), graph=graph)
        last, _ = run(m, c, ids, 0)
        m.forward(ids.contiguous(), last)  # second call replays the graph
        outs.append(last)
        m.close()
    assert torch.equal(outs[0], outs[1])
    assert rel(outs[0], g["final"]) < H_TOL, rel(outs[0], g["final"])


def test_bad_token_id_and_missing_parameter(ctx):
    c = synth.Qwen3Cfg(vocab_size=64, hidden_size=256, intermediate_size=256, num_hidden_layers=1,
                       num_attention_heads=2, num_key_value_heads=1)
    m, _ = build(ctx, c, seed=1, B=1, S=8, taps=())
    ids = torch.zeros(1, 8, dtype=torch.int32)
    ids[0, 3] = 64  # one past the vocabulary
    out = torch.empty(1, 8, c.hidden_size)
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.forward(ids, out)
    assert e.value.status == 1 and "embedding" in str(e.value)
    ids[0, 3] = 5
    m.forward(ids, out)  # the context recovers
    assert torch.isfinite(out).all()
    m.close()
    m2 = dcpp_b200.Qwen3Model(ctx, c)
    params = synth.make_qwen3_params(c, dcpp_b200.TYPE_Q8_0, seed=1)
    for name, (gt, shp, data) in params.items():
        if name != "model.layers.0.mlp.up_proj.weight":
            m2.set_param(name[len("model."):] if name.startswith("model.layers") else name, gt, shp, data)
    n, first = m2.missing()
    assert n == 1 and "gate_up" in first
    with pytest.raises(dcpp_b200.DcppError) as e:
        m2.prepare(1, 8)
    assert e.value.status == 7
    m2.close()


def test_prefill_k_split_projections(ctx, monkeypatch):
    """The config-4 projection shapes (M = 4 x 512, N = 2560, K = 4096 / 9728)
    run as K-split GEMMs (f32 partials, ordered reduce): against the oracle,
    against the unsplit GEMMs, and deterministic from run to run."""
    c = synth.Qwen3Cfg(vocab_size=1000, num_hidden_layers=1)
    B, S, taps = 4, 512, (1,)
    params = synth.make_qwen3_params(c, seed=21)
    ids = synth.make_qwen3_ids(c, B, S, seed=22)
    outs = []
    for ksplit in ("1", "1", "0"):
        monkeypatch.setenv("DCPP_GEMM_KSPLIT", ksplit)
        m = dcpp_b200.Qwen3Model(ctx, c)
        m.load_params(params)
        m.prepare(B, S, taps)
        outs.append(run(m, c, ids, len(taps)))
        m.close()
    assert torch.equal(outs[0][0], outs[1][0])
    ref_last, _ = qo.Qwen3Oracle(qo.Qwen3Config(**c.__dict__), params).forward(ids, taps=taps)
    for last, _ in (outs[0], outs[2]):
        assert rel(last, ref_last) < H_TOL, rel(last, ref_last)
    assert rel(outs[0][0], outs[2][0]) < 2e-3
