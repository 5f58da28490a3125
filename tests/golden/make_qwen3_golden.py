"""Generate the Qwen3 prefill fixture (tests/golden/qwen3_golden.npz).

HF transformers' Qwen3Model -- the implementation the reference's own Qwen3
tests compare the C++ modules with (test/src/transformers/models/qwen3/
Qwen3Model.py) -- runs in float64 on the CPU with the dequantised weights of
a small seeded Qwen3 (Q8_0 matrices, F32 norms, dcpp_b200.synth), on seeded
token ids.  Stored: the config, the ids, the hidden states before layers
0, 1 and 3 (hidden_states[i]) and the final normed output.  The oracle
(oracle/qwen3_oracle.py) is pinned against these; the params are regenerated
from the same seed by the tests.

Run:  python tests/golden/make_qwen3_golden.py
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "diffusers-cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import flux2_oracle as fo  # noqa: E402
from dcpp_b200 import TYPE_Q8_0, synth  # noqa: E402

CFG = dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=3, num_attention_heads=4,
           num_key_value_heads=2, head_dim=128, rms_norm_eps=1e-6, rope_theta=1000000.0)
SEED = 7
B, S = 2, 37
TAPS = (0, 1, 3)


def main():
    from transformers import Qwen3Config, Qwen3Model

    c = synth.Qwen3Cfg(**CFG)
    params = synth.make_qwen3_params(c, TYPE_Q8_0, seed=SEED)
    ids = synth.make_qwen3_ids(c, B, S, seed=SEED + 1)
    hf_cfg = Qwen3Config(vocab_size=c.vocab_size, hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
                         num_hidden_layers=c.num_hidden_layers, num_attention_heads=c.num_attention_heads,
                         num_key_value_heads=c.num_key_value_heads, head_dim=c.head_dim, rms_norm_eps=c.rms_norm_eps,
                         rope_theta=c.rope_theta, max_position_embeddings=4096, attention_bias=False,
                         tie_word_embeddings=False)
    hf_cfg._attn_implementation = "eager"
    model = Qwen3Model(hf_cfg).to(torch.float64).eval()
    w = fo.Weights(params)
    state = {}
    for name in params:
        state[name[len("model."):]] = w.get(name)
    model.load_state_dict(state, strict=True)
    with torch.no_grad():
        out = model(input_ids=ids.long(), output_hidden_states=True)
    hs = out.hidden_states
    np.savez_compressed(
        os.path.join(HERE, "qwen3_golden.npz"),
        config=np.array([CFG[k] for k in ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
                                          "num_attention_heads", "num_key_value_heads", "head_dim")], dtype=np.int64),
        seed=np.array([SEED]),
        ids=ids.numpy(),
        taps=np.array(TAPS),
        **{f"hidden_{t}": hs[t].numpy() for t in TAPS[:-1]},
        final=out.last_hidden_state.numpy(),
    )
    print("wrote", os.path.join(HERE, "qwen3_golden.npz"))


if __name__ == "__main__":
    main()
