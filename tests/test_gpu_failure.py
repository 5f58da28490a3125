"""Failure detection on the GPU without a fault: a bounded device-side wait
runs out on a flag that nothing sets, the kernel records an error and
returns, the host reads DCPP_ERR_TIMEOUT, and the same context then runs a
forward that matches the oracle.

The wait is the tensor-parallel flag barrier (rank 0 of an emulated group
whose other ranks are flag slots in local memory), with the context's wait
limit shortened to 20 ms."""
import time

import pytest
import torch

import dcpp_b200
import flux2_oracle as fo
from dcpp_b200 import synth

pytestmark = pytest.mark.gpu

DCPP_ERR_TIMEOUT = 5


def test_barrier_wait_runs_out_then_context_recovers(ctx):
    ctx.set_wait_timeout(0.02)
    try:
        assert ctx.tp_barrier_selftest(4, 0b1110) == 0  # every rank arrived
        t0 = time.perf_counter()
        st = ctx.tp_barrier_selftest(2, 0)  # rank 1 never arrives
        took = time.perf_counter() - t0
        assert st == DCPP_ERR_TIMEOUT, st
        msg = dcpp_b200.lib().dcpp_last_error(ctx.h).decode()
        assert "peer GPU" in msg, msg
        assert took < 0.9, took  # the 20 ms limit, not the 1 s default
        assert ctx.tp_barrier_selftest(4, 0b0110) == DCPP_ERR_TIMEOUT  # rank 3 missing
        assert ctx.tp_barrier_selftest(1, 0) == 0  # a group of one never waits
    finally:
        ctx.set_wait_timeout(0)
    # The error word was cleared and the context still computes correctly.
    c = synth.Flux2Cfg(num_layers=1, num_single_layers=1, num_attention_heads=2, joint_attention_dim=64,
                       in_channels=32, guidance_embeds=False)
    params = synth.make_params(c, fo.GGML_Q8_0, seed=41)
    m = dcpp_b200.Flux2Model(ctx, c)
    m.load_params(params)
    m.prepare(1, 16, 8)
    hid, enc, iid, tid = synth.make_inputs(c, 1, 4, 4, 8, seed=42)
    t = torch.tensor([0.5])
    out = torch.empty_like(hid)
    m.forward(hid, enc, t, iid, tid, out)
    m.close()
    ref = fo.Flux2Oracle(fo.Config(**{k: getattr(c, k) for k in fo.Config.__dataclass_fields__}), params).forward(
        hid, enc, t, iid, tid)
    r = ((out.double() - ref).norm() / ref.norm()).item()
    assert r < 3e-2, r


def test_wait_timeout_rejects_bad_values(ctx):
    for bad in (-1.0, 1e-5, 1000.0):
        with pytest.raises(dcpp_b200.DcppError) as e:
            ctx.set_wait_timeout(bad)
        assert e.value.status == 1
