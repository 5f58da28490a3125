"""Models loaded from GGUF checkpoints on the GPU: from_pretrained over a
component folder (config.json + *.gguf, the layout
Flux2KleinPipeline::from_pretrained reads) must give bit-identical outputs to
the same parameters bound with set_param, and match the oracle.  The text
encoder uses the reference converter's type map (BF16 attention projections,
F32 norms, Q8_0 elsewhere) and carries the lm_head.weight a Qwen3ForCausalLM
checkpoint holds."""
import json
from dataclasses import asdict

import pytest
import torch

import dcpp_b200
import flux2_oracle as fo
import qwen3_oracle as qo
from dcpp_b200 import synth
from gguf_util import write_gguf

pytestmark = pytest.mark.gpu

V_TOL = 3e-2
H_TOL = 2e-2


def rel(a, b):
    a, b = torch.as_tensor(a).double().cpu(), torch.as_tensor(b).double().cpu()
    return ((a - b).norm() / b.norm()).item()


def test_flux2_from_pretrained_equals_set_param(ctx, tmp_path):
    c = synth.Flux2Cfg(num_layers=1, num_single_layers=2, num_attention_heads=2, attention_head_dim=128,
                       joint_attention_dim=64, in_channels=32, timestep_guidance_channels=256, guidance_embeds=False)
    params = synth.make_params(c, fo.GGML_Q4_K, seed=31, split=True)
    d = tmp_path / "transformer"
    d.mkdir()
    cfg = asdict(c)
    cfg["axes_dims_rope"] = list(c.axes_dims_rope)
    (d / "config.json").write_text(json.dumps(cfg))
    write_gguf(d / "diffusion_pytorch_model.gguf", params)

    a = dcpp_b200.Flux2Model.from_pretrained(ctx, d)
    b = dcpp_b200.Flux2Model(ctx, c)
    b.load_params(params)
    hid, enc, iid, tid = synth.make_inputs(c, 1, 6, 8, 11, seed=32)
    t = torch.tensor([0.4], dtype=torch.float32)
    outs = []
    for m in (a, b):
        m.prepare(1, 48, 11)
        out = torch.empty(1, 48, c.in_channels, dtype=torch.float32)
        m.forward(hid, enc, t, iid, tid, out)
        outs.append(out)
        m.close()
    assert torch.equal(outs[0], outs[1])
    oc = fo.Config(**{k: getattr(c, k) for k in fo.Config.__dataclass_fields__})
    r = rel(outs[0], fo.Flux2Oracle(oc, params).forward(hid, enc, t, iid, tid))
    assert r < V_TOL, r


def test_qwen3_from_pretrained_reference_types(ctx, tmp_path):
    c = synth.Qwen3Cfg(vocab_size=1000, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                       num_attention_heads=8, num_key_value_heads=2)
    params = synth.make_qwen3_params(c, seed=41, types=synth.QWEN3_KLEIN_TYPES)
    assert params["model.layers.0.self_attn.q_proj.weight"][0] == dcpp_b200.TYPE_BF16
    file_params = dict(params)
    file_params["lm_head.weight"] = params["model.embed_tokens.weight"]
    d = tmp_path / "text_encoder"
    d.mkdir()
    (d / "config.json").write_text(json.dumps({**asdict(c), "architectures": ["Qwen3ForCausalLM"],
                                               "tie_word_embeddings": False}))
    write_gguf(d / "model.gguf", file_params, arch="qwen3")

    B, S, taps = 2, 200, (1, 2)
    ids = synth.make_qwen3_ids(c, B, S, seed=42)
    a = dcpp_b200.Qwen3Model.from_pretrained(ctx, d)
    b = dcpp_b200.Qwen3Model(ctx, c)
    b.load_params(params)
    outs = []
    for m in (a, b):
        m.prepare(B, S, taps)
        last = torch.empty(B, S, c.hidden_size, dtype=torch.float32)
        tp = torch.empty(B, S, len(taps) * c.hidden_size, dtype=torch.float32)
        m.forward(ids, last, tp)
        outs.append((last, tp))
        m.close()
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    ref_last, ref_taps = qo.Qwen3Oracle(qo.Qwen3Config(**asdict(c)), params).forward(ids, taps=taps)
    assert rel(outs[0][0], ref_last) < H_TOL
    D = c.hidden_size
    for k, t in enumerate(taps):
        assert rel(outs[0][1][..., k * D:(k + 1) * D], ref_taps[t]) < H_TOL


def test_from_pretrained_errors(ctx, tmp_path):
    d = tmp_path / "transformer"
    d.mkdir()
    with pytest.raises(dcpp_b200.DcppError):  # no config.json
        dcpp_b200.Flux2Model.from_pretrained(ctx, d)
    (d / "config.json").write_text(json.dumps({"num_layers": 1, "num_single_layers": 1}))
    with pytest.raises(dcpp_b200.DcppError) as e:  # no GGUF file
        dcpp_b200.Flux2Model.from_pretrained(ctx, d)
    assert "No such GGUF file" in str(e.value)
