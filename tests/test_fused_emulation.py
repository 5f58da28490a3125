"""CPU checks of the fused-dequant emulation used by the GPU tests: exact
bf16 rounding, and closeness to the exact (gguf-py) dequantised weights."""
import numpy as np
import torch

import flux2_oracle as fo
from dcpp_b200 import quant
from fused_emulation import fused_weights, round_bf16


def test_round_bf16_matches_torch_on_f32_values():
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32)
    ref = torch.from_numpy(x).to(torch.bfloat16).double().numpy()
    assert np.array_equal(round_bf16(x.astype(np.float64)), ref)


def test_round_bf16_ties_to_even():
    assert round_bf16(np.array([1.00390625, 1.01171875]))[0] == 1.0
    assert round_bf16(np.array([1.01171875]))[0] == 1.015625


def test_fused_weights_close_to_exact_dequant():
    g = torch.Generator().manual_seed(4)
    for gtype in (fo.GGML_Q4_K, fo.GGML_Q8_0):
        w = torch.randn(64, 512, generator=g) / 512 ** 0.5
        raw = quant.quantize(w, gtype).numpy()
        exact = fo.dequant(gtype, raw, w.numel()).reshape(64, 512).astype(np.float64)
        emu = fused_weights(gtype, raw, 64, 512)
        rel = np.linalg.norm(emu - exact) / np.linalg.norm(exact)
        assert rel < 8e-3, (gtype, rel)
        # every emulated value is a bf16 number
        assert np.array_equal(round_bf16(emu), emu)
