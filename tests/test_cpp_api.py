"""The C++ surface (include/dcpp.hpp: CudaRuntime, ShardingPlan,
Flux2Transformer2DModel, FlowMatchEulerDiscreteScheduler, Flux2KleinPipeline)
compiled into a small program (tests/cpp/api_test.cpp) the way a
diffusers-cpp caller would build against the library: config parsing, the
planner's split, the scheduler and the host-only loader on the CPU, and one
reference-image denoise step on the GPU checked against the float64 oracle."""
import json
import os
import shutil
import struct
import subprocess

import numpy as np
import pytest
import torch

import dcpp_b200
import flux2_oracle as fo
from dcpp_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.dirname(dcpp_b200.LIB_PATH)


@pytest.fixture(scope="module")
def api_test(tmp_path_factory):
    gxx = shutil.which("g++")
    if not gxx:
        pytest.skip("no g++")
    dcpp_b200.lib()  # the library must be built
    exe = str(tmp_path_factory.mktemp("cpp") / "api_test")
    subprocess.check_call([gxx, "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                           os.path.join(ROOT, "tests", "cpp", "api_test.cpp"), "-L", LIBDIR, "-ldcpp_b200",
                           f"-Wl,-rpath,{LIBDIR}", "-o", exe])
    return exe


def test_cpp_api_host_side(api_test, tmp_path):
    cfg = tmp_path / "config.json"
    cfg.write_text(json.dumps({"num_layers": 1, "num_single_layers": 1, "num_attention_heads": 6,
                               "joint_attention_dim": 64, "guidance_embeds": False}))
    r = subprocess.run([api_test, "cpu", str(cfg)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr


@pytest.mark.gpu
def test_cpp_api_denoise_with_ref_images(api_test, tmp_path):
    c = synth.Flux2Cfg(num_layers=1, num_single_layers=1, num_attention_heads=2, joint_attention_dim=64,
                       in_channels=32, guidance_embeds=False)
    params = synth.make_params(c, fo.GGML_Q4_K, seed=61)
    hid, enc, iid, tid = synth.make_inputs(c, 1, 4, 4, 12, seed=62)
    g = torch.Generator().manual_seed(63)
    n_ref = 8
    ref = torch.randn(1, n_ref, c.in_channels, generator=g)
    ref_ids = torch.zeros(n_ref, 4, dtype=torch.int32)
    ref_ids[:, 0] = 10
    ref_ids[:, 2] = torch.arange(n_ref, dtype=torch.int32)
    sigma, dt = 0.75, -0.25
    with open(tmp_path / "params.bin", "wb") as f:
        f.write(struct.pack("<q", len(params)))
        for name, (gt, shp, data) in params.items():
            raw = np.ascontiguousarray(data.numpy() if hasattr(data, "numpy") else data).tobytes()
            f.write(struct.pack("<q", len(name)) + name.encode() + struct.pack("<qq", gt, len(shp)))
            f.write(struct.pack(f"<{len(shp)}q", *shp) + struct.pack("<q", len(raw)) + raw)
    with open(tmp_path / "inputs.bin", "wb") as f:
        f.write(struct.pack("<8q", c.num_layers, c.num_single_layers, c.num_attention_heads, c.joint_attention_dim,
                            c.in_channels, 16, n_ref, 12))
        f.write(struct.pack("<ff", sigma, dt))
        for t in (hid, ref, enc, iid, ref_ids, tid):
            f.write(t.contiguous().numpy().tobytes())
    out = tmp_path / "out.bin"
    r = subprocess.run([api_test, "gpu", str(tmp_path / "params.bin"), str(tmp_path / "inputs.bin"), str(out)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    got = torch.from_numpy(np.fromfile(out, dtype=np.float32).reshape(1, 16, c.in_channels))
    o = fo.Flux2Oracle(fo.Config(**{k: getattr(c, k) for k in fo.Config.__dataclass_fields__}), params)
    want = o.denoise(hid, enc, torch.tensor([sigma]), dt, iid, tid, image_latents=ref, image_latent_ids=ref_ids)
    rel = ((got.double() - want).norm() / want.norm()).item()
    assert rel < 1e-2, rel
