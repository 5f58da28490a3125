"""CPU tests of the C ABI boundary: the library loads, exports every symbol
include/dcpp.h declares, and its host-only entry points behave (no GPU
compute is launched here)."""
import ctypes
import json
import os
import re

import numpy as np
import pytest

import dcpp_b200
import flux2_oracle as fo

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dcpp.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dcpp_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("dcpp_init", "dcpp_gemm", "dcpp_dequant", "dcpp_attention", "dcpp_flux2_forward",
                 "dcpp_flux2_denoise_step", "dcpp_tp_init", "dcpp_allreduce"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = dcpp_b200.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert set(declared_functions()) <= set(dcpp_b200.exported_symbols())


@pytest.mark.parametrize("gtype,n,expect", [
    (dcpp_b200.TYPE_F32, 10, 40), (dcpp_b200.TYPE_BF16, 10, 20), (dcpp_b200.TYPE_F16, 3, 6),
    (dcpp_b200.TYPE_Q8_0, 64, 68), (dcpp_b200.TYPE_Q4_K, 512, 288)])
def test_row_bytes(gtype, n, expect):
    assert dcpp_b200.row_bytes(gtype, n) == expect


def test_row_bytes_rejects_ragged_blocks():
    with pytest.raises(dcpp_b200.DcppError) as e:
        dcpp_b200.row_bytes(dcpp_b200.TYPE_Q4_K, 100)
    assert e.value.status == 1


def test_schedule_matches_oracle():
    ts, sg = dcpp_b200.flow_match_schedule(4)
    ots, osg = fo.flow_match_schedule(4)
    assert np.array_equal(ts, np.array(ots, np.float32))
    assert np.array_equal(sg, np.array(osg, np.float32))


def test_config_from_file(tmp_path):
    p = tmp_path / "config.json"
    p.write_text(json.dumps({"_class_name": "Flux2Transformer2DModel", "num_layers": 5, "num_single_layers": 20,
                             "num_attention_heads": 24, "joint_attention_dim": 7680, "axes_dims_rope": [32, 32, 32, 32],
                             "guidance_embeds": False, "out_channels": None, "mlp_ratio": 3.0, "eps": 1e-6}))
    c = dcpp_b200.Flux2ConfigC()
    st = dcpp_b200.lib().dcpp_flux2_config_from_file(str(p).encode(), ctypes.byref(c))
    assert st == 0
    assert (c.num_layers, c.num_single_layers, c.num_attention_heads, c.joint_attention_dim) == (5, 20, 24, 7680)
    assert c.guidance_embeds == 0 and c.out_channels == -1 and c.n_axes == 4
    assert c.attention_head_dim == 128 and c.rope_theta == 2000  # defaults kept


def test_config_from_missing_file_is_not_found():
    c = dcpp_b200.Flux2ConfigC()
    assert dcpp_b200.lib().dcpp_flux2_config_from_file(b"/nonexistent/config.json", ctypes.byref(c)) == 8


def test_init_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    h = ctypes.c_void_p()
    assert dcpp_b200.lib().dcpp_init(0, ctypes.byref(h)) == 3  # DCPP_ERR_CUDA
    assert not h.value


def test_null_context_is_invalid_arg():
    L = dcpp_b200.lib()
    assert L.dcpp_synchronize(None) == 1
    assert L.dcpp_gemm(None, 8, None, 1, 1, None, 1, None) == 1
    assert L.dcpp_flux2_forward(None, None, None, None, None, None, None, None) == 1
