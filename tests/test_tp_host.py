"""Tensor-parallel sharding of the C++ loader, checked without a GPU.

Host-only models (dcpp_flux2_create_host) assemble each rank's shards with the
same code a device model uses; these tests read the shards back and check
(1) their exact layout against slices of the full weights, for a config whose
shards fall on the quantisation blocks (kept in Q8_0 / Q4_K) and one whose
Q4_K shards do not (expanded to bf16 at load), and (2) that world-size-2 gloo
ranks running the forward on their own shards, with an all-reduce after every
row-parallel projection, reproduce the unsharded oracle.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import dcpp_b200
import flux2_oracle as fo
import tp_oracle as tpo
from dcpp_b200 import synth


def cfg(heads, **kw):
    base = dict(num_layers=1, num_single_layers=1, num_attention_heads=heads, attention_head_dim=128,
                joint_attention_dim=64, in_channels=32, timestep_guidance_channels=256, guidance_embeds=True)
    base.update(kw)
    return synth.Flux2Cfg(**base)


def oracle_cfg(c):
    return fo.Config(**{k: getattr(c, k) for k in fo.Config.__dataclass_fields__})


def host_model(c, params, rank, n, ratios=None):
    m = dcpp_b200.Flux2Model(None, c, tp_rank=rank, tp_size=n, tp_split=ratios)
    m.load_params(params)
    assert m.missing() == (0, "")
    return m


# heads=4, n=2: Dl = 256, Fl = 768 -> Q4_K shards stay Q4_K.
# heads=6, n=2: Dl = 384, Fl = 1152 -> Q4_K row-parallel shards become bf16.
# Uneven (tensor_split ratios): 6 heads at 2:1 -> 4 / 2 heads, 36 MLP units
# -> 24 / 12; 6 heads over 4 equal ranks -> 1, 1, 2, 2 heads (ties to the
# later rank); 6 heads at 1:1:3 with Q4_K (bf16 shards).
LAYOUTS = [(4, 2, fo.GGML_Q8_0, False, None), (4, 2, fo.GGML_Q4_K, False, None), (6, 2, fo.GGML_Q4_K, False, None),
           (6, 2, fo.GGML_Q4_K, True, None), (4, 4, fo.GGML_Q8_0, True, None), (6, 2, fo.GGML_Q8_0, False, [2.0, 1.0]),
           (6, 4, fo.GGML_Q8_0, False, [1.0, 1.0, 1.0, 1.0]), (6, 3, fo.GGML_Q4_K, True, [1.0, 1.0, 3.0])]


@pytest.mark.parametrize("heads,n,wtype,split,ratios", LAYOUTS)
def test_shard_layout_exact(heads, n, wtype, split, ratios):
    c = cfg(heads)
    params = synth.make_params(c, wtype, seed=5, split=split)
    full = fo.Weights(params)
    D, F = c.inner_dim, c.mlp_hidden
    for rank in range(n):
        m = host_model(c, params, rank, n, ratios)
        h0, hn, f0, fn = tpo.shard_of(c, rank, n, ratios)
        assert m.shard() == (h0, hn, f0, fn)
        exp = tpo.expected_shards(c, full, rank, n, ratios)
        for name, want in exp.items():
            gt, shape, buf = m.read_param(name)
            assert shape == tuple(want.shape), (name, shape, want.shape)
            got = tpo.decode(gt, shape, buf)
            if gt == fo.GGML_BF16 and wtype != fo.GGML_BF16:
                # expanded at load: the dequantised value rounded once to bf16
                want = want.float().to(torch.bfloat16).double()
            assert torch.equal(got, want), name
            unaligned = any(x % 256 for x in (h0 * 128, hn * 128, f0, fn))
            block = name.startswith(("transformer_blocks.", "single_transformer_blocks."))
            if block and (wtype == fo.GGML_Q8_0 or not unaligned):
                assert gt == wtype, (name, gt)
        for name in tpo.vector_names(c):
            gt, shape, buf = m.read_param(name)
            assert gt == fo.GGML_F32 and shape == (1, 128)
            want = torch.from_numpy(fo.dequant(params[name][0], params[name][2], 128)).double()
            assert torch.equal(tpo.decode(gt, shape, buf)[0], want)
        m.close()


def test_host_model_cannot_execute_and_reports_errors():
    c = cfg(4)
    m = dcpp_b200.Flux2Model(None, c)
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.read_param("proj_out.weight")
    assert e.value.status == 7 and "not fully set" in str(e.value)
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.read_param("no.such.weight")
    assert e.value.status == 8
    m.load_params(synth.make_params(c, fo.GGML_Q8_0, seed=1))
    with pytest.raises(dcpp_b200.DcppError) as e:
        m.prepare(1, 16, 8)
    assert e.value.status == 7 and "host-only" in str(e.value)
    m.close()


def test_bad_tp_sizes_rejected():
    c = cfg(2)
    with pytest.raises(dcpp_b200.DcppError) as e:
        dcpp_b200.Flux2Model(None, c, tp_rank=0, tp_size=4)  # 2 heads over 4 ranks: two ranks get none
    assert e.value.status == 2 and "without a head" in str(e.value)
    with pytest.raises(dcpp_b200.DcppError) as e:
        dcpp_b200.Flux2Model(None, cfg(6), tp_rank=0, tp_size=2, tp_split=[1.0, -1.0])
    assert e.value.status == 1
    c = cfg(6)
    with pytest.raises(dcpp_b200.DcppError) as e:
        dcpp_b200.Flux2Model(None, c, tp_rank=2, tp_size=2)
    assert e.value.status == 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_split_planner_matches_restatement():
    """dcpp_tp_plan_split against the restated rounding, including ties and
    remainders that several ranks compete for."""
    g = np.random.default_rng(3)
    cases = [(24, [1] * 8), (24, [1] * 5), (144, [2, 1, 1]), (24, [1.5, 1.0]), (7, [1, 1, 1]), (100, [0.3, 0.3, 0.4])]
    for _ in range(200):
        n = int(g.integers(1, 9))
        cases.append((int(g.integers(n, 400)), list(g.uniform(0.1, 3.0, n))))
    for units, ratios in cases:
        r32 = [float(np.float32(f)) for f in ratios]  # the C ABI takes float ratios
        assert dcpp_b200.tp_plan_split(units, len(ratios), ratios) == tpo.plan_split(units, r32), (units, ratios)
        assert sum(dcpp_b200.tp_plan_split(units, len(ratios), ratios)) == units


def _tp_rank(rank, n, port, heads, wtype, tol, result_dir, ratios=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=n)
    try:
        c = cfg(heads, num_layers=2, num_single_layers=2)
        params = synth.make_params(c, wtype, seed=31)
        hid, enc, iid, tid = synth.make_inputs(c, 2, 3, 5, 11, seed=32)
        t = torch.tensor([0.7, 0.2])
        guid = torch.tensor([1.5, 4.0])
        m = host_model(c, params, rank, n, ratios)
        hl = m.shard()[1]
        shards = tpo.decode_shards(tpo.read_shards(m, c))
        m.close()

        def allreduce(x):
            x = x.clone()
            dist.all_reduce(x)
            return x

        out = tpo.TPOracle(oracle_cfg(c), shards, n, allreduce, heads=hl).forward(hid, enc, t, iid, tid,
                                                                                  guidance=guid)
        if rank == 0:
            ref = fo.Flux2Oracle(oracle_cfg(c), params).forward(hid, enc, t, iid, tid, guidance=guid)
            r = ((out - ref).norm() / ref.norm()).item()
            np.save(os.path.join(result_dir, "rel.npy"), np.array([r]))
            assert r < tol, r
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("heads,wtype,tol,ratios", [(4, fo.GGML_Q8_0, 1e-12, None), (6, fo.GGML_Q4_K, 2e-2, None),
                                                    (6, fo.GGML_Q8_0, 1e-12, [2.0, 1.0]),
                                                    (5, fo.GGML_Q8_0, 1e-12, [1.0, 1.0])])
def test_tp_forward_gloo_world2_matches_oracle(tmp_path, heads, wtype, tol, ratios):
    """Two gloo ranks, each on its own shards, summed after every row-parallel
    projection.  Q8_0 shards are exact slices (float64 sums differ only in
    rounding); the 6-head Q4_K shards are bf16 expansions (one bf16 rounding
    of the weights).  Uneven splits: 4 + 2 heads (ratios 2:1) and 2 + 3 heads
    (5 heads, equal ratios)."""
    mp.spawn(_tp_rank, args=(2, _free_port(), heads, wtype, tol, str(tmp_path), ratios), nprocs=2, join=True)
    r = float(np.load(tmp_path / "rel.npy")[0])
    assert r < tol
