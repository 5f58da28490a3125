"""FlowMatchEulerDiscreteScheduler through the C ABI (dcpp_flow_match_schedule_ex)
against the float32 restatement in the oracle, for every constructor option
the reference scheduler has (FlowMatchEulerDiscreteScheduler.cpp:8-208) and
the pipeline's dynamic-shift mu (Flux2KleinPipeline.cpp:130-141).  The
reference's own tests (test/src/diffusers/schedulers/
FlowMatchEulerDiscreteScheduler.py) cover the default, dynamic-shifting and
single-step schedules; those cases are here too.  CPU only."""
import numpy as np
import pytest

import dcpp_b200
import flux2_oracle as fo

STEPS = [1, 2, 4, 28, 50]


def run(n, mu=0.0, sigmas=None, **cfg):
    got = dcpp_b200.FlowMatchEulerDiscreteScheduler(**cfg).schedule(n, mu, sigmas)
    want = fo.flow_match_schedule_full(n, mu, sigmas, **cfg)
    return got, want


def pipeline_sigmas(n):
    return [np.float32(1.0 - i / n) for i in range(n)]


@pytest.mark.parametrize("n", STEPS)
def test_default_linspace_bit_exact(n):
    (ts, sg), (wts, wsg) = run(n)
    assert np.array_equal(ts, wts) and np.array_equal(sg, wsg)
    assert sg[0] == 1.0 and sg[-1] == 0.0
    if n > 1:
        assert sg[n - 1] == np.float32(1.0) / np.float32(1000.0)  # sigma_min


@pytest.mark.parametrize("shift", [1.0, 3.0, 0.5])
@pytest.mark.parametrize("n", STEPS)
def test_static_shift_with_pipeline_sigmas_bit_exact(n, shift):
    (ts, sg), (wts, wsg) = run(n, 0.0, pipeline_sigmas(n), shift=shift)
    assert np.array_equal(ts, wts) and np.array_equal(sg, wsg)
    # the pipeline-form entry point agrees
    pts, psg = dcpp_b200.flow_match_schedule(n, shift)
    assert np.array_equal(ts, pts) and np.array_equal(sg, psg)


@pytest.mark.parametrize("seq_len", [256, 1024, 4096, 4300, 4301, 16384])
@pytest.mark.parametrize("n", STEPS)
def test_empirical_mu_bit_exact(seq_len, n):
    assert np.float32(dcpp_b200.flux2_empirical_mu(seq_len, n)) == fo.compute_empirical_mu(seq_len, n)


@pytest.mark.parametrize("n", STEPS)
def test_dynamic_exponential(n):
    # the reference test's dynamic-shifting case: mu from the image length
    mu = fo.compute_empirical_mu(4096, n)
    (ts, sg), (wts, wsg) = run(n, float(mu), pipeline_sigmas(n), use_dynamic_shifting=True)
    # exp(mu) may round differently (libm expf vs a float64 exp rounded): 2 ulp
    np.testing.assert_allclose(sg, wsg, rtol=2.5e-7, atol=0)
    np.testing.assert_allclose(ts, wts, rtol=2.5e-7, atol=0)
    assert np.all(np.diff(sg) < 0)  # still decreasing to 0


@pytest.mark.parametrize("n", STEPS)
def test_dynamic_exponential_default_sigmas(n):
    (ts, sg), (wts, wsg) = run(n, 1.15, None, use_dynamic_shifting=True)
    np.testing.assert_allclose(sg, wsg, rtol=2.5e-7, atol=0)


def test_dynamic_mu_zero_is_the_identity():
    base = pipeline_sigmas(8)
    _, sg = dcpp_b200.FlowMatchEulerDiscreteScheduler(use_dynamic_shifting=True).schedule(8, 0.0, base)
    np.testing.assert_allclose(sg[:-1], np.array(base, np.float32), rtol=1e-6)
    _, sg = dcpp_b200.FlowMatchEulerDiscreteScheduler(use_dynamic_shifting=True,
                                                      time_shift_type="linear").schedule(8, 1.0, base)
    np.testing.assert_allclose(sg[:-1], np.array(base, np.float32), rtol=1e-6)


@pytest.mark.parametrize("mu", [0.5, 1.15, 3.0])
def test_dynamic_linear_bit_exact(mu):
    (ts, sg), (wts, wsg) = run(10, mu, pipeline_sigmas(10), use_dynamic_shifting=True, time_shift_type="linear")
    assert np.array_equal(ts, wts) and np.array_equal(sg, wsg)


@pytest.mark.parametrize("terminal", [0.02, 0.1])
def test_shift_terminal_bit_exact(terminal):
    (ts, sg), (wts, wsg) = run(12, 0.0, None, shift=3.0, shift_terminal=terminal)
    assert np.array_equal(ts, wts) and np.array_equal(sg, wsg)
    np.testing.assert_allclose(sg[-2], terminal, rtol=1e-5)  # the last sigma is stretched to it


def test_invert_sigmas_bit_exact():
    (ts, sg), (wts, wsg) = run(6, 0.0, pipeline_sigmas(6), shift=2.0, invert_sigmas=True)
    assert np.array_equal(ts, wts) and np.array_equal(sg, wsg)
    assert sg[-1] == 1.0 and sg[0] == 0.0


def test_num_train_timesteps():
    (ts, sg), (wts, wsg) = run(5, 0.0, None, num_train_timesteps=500)
    assert np.array_equal(ts, wts) and np.array_equal(sg, wsg)
    assert ts[0] == 500.0


@pytest.mark.parametrize("bad", [dict(n=0), dict(n=3, cfg=dict(num_train_timesteps=0)),
                                 dict(n=2, sigmas=[1.0, 0.0], cfg=dict(use_dynamic_shifting=True)),
                                 dict(n=3, sigmas=[1.0, 0.5])])
def test_invalid_arguments_fail(bad):
    with pytest.raises(dcpp_b200.DcppError) as e:
        dcpp_b200.FlowMatchEulerDiscreteScheduler(**bad.get("cfg", {})).schedule(bad["n"], 0.0, bad.get("sigmas"))
    assert e.value.status == 1


def test_unknown_time_shift_type_fails():
    with pytest.raises(dcpp_b200.DcppError):
        dcpp_b200.FlowMatchEulerDiscreteScheduler(time_shift_type="cubic")


# ----------------------------------------------------------------- position ids
@pytest.mark.parametrize("batch,seq_len", [(1, 512), (2, 77), (3, 0)])
def test_txt_ids_match_oracle(batch, seq_len):
    assert np.array_equal(dcpp_b200.prepare_txt_ids(batch, seq_len), fo.prepare_txt_ids(batch, seq_len))


@pytest.mark.parametrize("batch,h,w", [(1, 64, 64), (2, 9, 14), (1, 1, 7)])
def test_img_ids_match_oracle(batch, h, w):
    got = dcpp_b200.prepare_img_ids(batch, h, w)
    assert np.array_equal(got, fo.prepare_img_ids(batch, h, w))
    # the synthetic inputs the model tests use carry the same ids
    from dcpp_b200 import synth
    c = synth.Flux2Cfg(num_layers=1, num_single_layers=1, num_attention_heads=2, joint_attention_dim=64,
                       in_channels=32)
    _, _, iid, tid = synth.make_inputs(c, 1, h, w, 5)
    assert np.array_equal(got[0], iid.numpy()) and np.array_equal(dcpp_b200.prepare_txt_ids(1, 5)[0], tid.numpy())


@pytest.mark.parametrize("batch,sizes", [(1, [(32, 32)]), (2, [(4, 6), (3, 5)]), (1, [])])
def test_ref_image_ids_match_oracle(batch, sizes):
    got = dcpp_b200.prepare_ref_image_ids(batch, sizes)
    want = fo.prepare_ref_image_ids(batch, sizes) if sizes else np.zeros((batch, 0, 4), np.int32)
    assert np.array_equal(got, want)
    if sizes:
        assert got[0, 0, 0] == 10 and (len(sizes) < 2 or got[0, -1, 0] == 10 + 10 * (len(sizes) - 1))


def test_ids_reject_negative_sizes():
    assert dcpp_b200.lib().dcpp_flux2_prepare_img_ids(1, -1, 4, None) == 1
    assert dcpp_b200.lib().dcpp_flux2_prepare_txt_ids(-1, 4, None) == 1
