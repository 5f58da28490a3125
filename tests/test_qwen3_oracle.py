"""The Qwen3 prefill oracle pinned against HF transformers' Qwen3Model
(tests/golden/qwen3_golden.npz, made by tests/golden/make_qwen3_golden.py)."""
import os

import numpy as np
import torch

import qwen3_oracle as qo
from dcpp_b200 import TYPE_Q8_0, synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "qwen3_golden.npz")


def test_oracle_matches_hf_transformers_golden():
    g = np.load(GOLDEN)
    keys = ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
            "num_key_value_heads", "head_dim")
    cfg = dict(zip(keys, (int(v) for v in g["config"])))
    c = synth.Qwen3Cfg(**cfg)
    params = synth.make_qwen3_params(c, TYPE_Q8_0, seed=int(g["seed"][0]))
    ids = torch.from_numpy(g["ids"])
    taps = tuple(int(t) for t in g["taps"])
    o = qo.Qwen3Oracle(qo.Qwen3Config(**cfg), params)
    last, got = o.forward(ids, taps=taps)
    # HF keeps its RMSNorms and rotary tables in float32 even in a float64
    # model, so agreement is to ~1e-6 relative, not to float64 rounding.
    def rel(a, b):
        return float(np.linalg.norm(a - b) / np.linalg.norm(b))
    assert rel(last.numpy(), g["final"]) < 1e-5
    for t in taps[:-1]:
        assert rel(got[t].numpy(), g[f"hidden_{t}"]) < 1e-5, t
    assert torch.equal(got[taps[-1]], last)


def test_causal_mask_and_gqa_restatement():
    """Changing a later token must not change earlier positions; with one kv
    head shared by all query heads the result equals repeating that head."""
    c = qo.Qwen3Config(vocab_size=64, hidden_size=256, intermediate_size=256, num_hidden_layers=1,
                       num_attention_heads=4, num_key_value_heads=1)
    params = synth.make_qwen3_params(synth.Qwen3Cfg(**c.__dict__), TYPE_Q8_0, seed=3)
    o = qo.Qwen3Oracle(c, params)
    ids = torch.randint(0, 64, (1, 12), generator=torch.Generator().manual_seed(0)).to(torch.int32)
    a, _ = o.forward(ids)
    ids2 = ids.clone()
    ids2[0, 9] = (ids2[0, 9] + 1) % 64
    b, _ = o.forward(ids2)
    assert torch.equal(a[:, :9], b[:, :9])
    assert not torch.equal(a[:, 9:], b[:, 9:])
