"""Tensor parallelism on 2 GPUs over NCCL: the sharded model (column-parallel
q/k/v/gate/up, row-parallel output projections, an all-reduce after each) must
match the float64 oracle like the single-GPU model does.  Runs the ranks as
child processes under torch.distributed.run, bounded by a timeout that kills
the whole process group; skipped with fewer than 2 GPUs."""
import json
import os
import signal
import socket
import subprocess
import sys

import pytest
import torch

import flux2_oracle as fo

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
V_TOL = 3e-2
LAT_TOL = 1e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(tmp_path, heads, wtype, comm, pieces=2, n=2, timeout=600, ratios="even"):
    out = tmp_path / "tp.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "tp_gpu_worker.py"), str(out), str(heads), str(wtype), comm, str(pieces), ratios]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    p = subprocess.Popen(cmd, env=env, start_new_session=True, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    try:
        log, _ = p.communicate(timeout=timeout)
    except subprocess.TimeoutExpired:
        os.killpg(p.pid, signal.SIGKILL)
        log, _ = p.communicate()
        pytest.fail("TP ranks timed out:\n" + log.decode(errors="replace")[-4000:])
    assert p.returncode == 0, log.decode(errors="replace")[-4000:]
    return json.loads(out.read_text())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("heads,wtype,comm,pieces", [(4, fo.GGML_Q8_0, "peer", 2), (6, fo.GGML_Q4_K, "peer", 2),
                                                     (4, fo.GGML_Q8_0, "peer", 1), (4, fo.GGML_Q8_0, "nccl", 1),
                                                     (6, fo.GGML_Q4_K, "nccl", 1), (4, fo.GGML_Q8_0, "pull", 2),
                                                     (6, fo.GGML_Q4_K, "pull", 1), (4, fo.GGML_Q8_0, "overlap", 1),
                                                     (6, fo.GGML_Q4_K, "overlap", 1)],
                         ids=["q8_0_peer", "q4_k_bf16_shards_peer", "q8_0_peer_one_piece", "q8_0_nccl",
                              "q4_k_bf16_shards_nccl", "q8_0_pull", "q4_k_bf16_shards_pull_one_piece", "q8_0_overlap",
                              "q4_k_bf16_shards_overlap"])
def test_tp2_matches_oracle(tmp_path, heads, wtype, comm, pieces):
    """peer: the GEMM epilogue stores each partial into the owning GPU's
    receive slot, the owner's LayerNorm sums its slots and stores the
    normalised rows into every GPU, and a barrier precedes the next GEMM, in
    one or two row pieces (the second overlapping the first piece's GEMM);
    overlap: rows owned in 128-row granules, the owner's LayerNorm writes only
    its own rows, and the next GEMM pushes them to the other GPU from two
    extra warps while its producer waits per granule; pull: each GPU keeps
    its bf16 partial and the owners read them in their LayerNorm; nccl:
    ncclAllReduce of the partials."""
    r = run_ranks(tmp_path, heads, wtype, comm, pieces)
    assert r["ranks_identical"], r
    assert r["replay_identical"], r
    assert r["forward_rel"] < V_TOL, r
    assert r["denoise_rel"] < LAT_TOL, r
    assert r["resident_rel"] < LAT_TOL, r


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("heads,ratios,comm", [(6, "2,1", "peer"), (5, "even", "peer"), (6, "1,2", "nccl")],
                         ids=["6_heads_2_to_1_peer", "5_heads_even_peer", "6_heads_1_to_2_nccl"])
def test_tp2_uneven_split_matches_oracle(tmp_path, heads, ratios, comm):
    """The planner's uneven tensor_split (ratio-rounded heads and MLP units,
    dcpp_flux2_set_tensor_split): each rank computes a different number of
    heads, the exchange still sums full rows."""
    r = run_ranks(tmp_path, heads, fo.GGML_Q8_0, comm, 1, ratios=ratios)
    assert r["ranks_identical"], r
    assert r["forward_rel"] < V_TOL, r
    assert r["denoise_rel"] < LAT_TOL, r
    assert r["resident_rel"] < LAT_TOL, r
