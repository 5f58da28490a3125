"""One rank of the 2-GPU tensor-parallel parity test (launched by
tests/test_gpu_tp.py under torch.distributed.run, one process per GPU).

Each rank joins a gloo group (only to hand out the NCCL id), joins the
library's NCCL group, loads the full synthetic parameters into a sharded
model (the loader keeps this rank's heads / MLP features), and runs the
forward (CUDA graph with the NCCL all-reduces captured), a denoise step and
two resident steps.  Rank 0 compares every result with the float64 oracle and
writes the relative errors to the JSON file named on the command line.
"""
import datetime
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (os.path.join(ROOT, "diffusers-cpp_b200"), os.path.join(ROOT, "oracle")):
    sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import dcpp_b200  # noqa: E402
import flux2_oracle as fo  # noqa: E402
from dcpp_b200 import synth  # noqa: E402


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm()).item()


def main():
    out_path, heads, wtype, comm = sys.argv[1], int(sys.argv[2]), int(sys.argv[3]), sys.argv[4]
    # "peer": the peer exchange (default push form: partials stored into the
    # owners' slots, the owners' LayerNorm stores the rows into every GPU, a
    # barrier before the next GEMM); "overlap": the same with the all-gather
    # overlapped with the next GEMM (DCPP_TP_OVERLAP=1); "pull": its pull form
    # (DCPP_TP_PULL=1, partials read by their owners); "nccl": ncclAllReduce.
    # Read when a model is created.
    os.environ["DCPP_TP_COMM"] = "peer" if comm in ("pull", "overlap") else comm
    os.environ["DCPP_TP_PULL"] = "1" if comm == "pull" else "0"
    os.environ["DCPP_TP_OVERLAP"] = "1" if comm == "overlap" else "0"
    if len(sys.argv) > 5:
        os.environ["DCPP_TP_PIECES"] = sys.argv[5]  # row pieces of the peer exchange (1 or 2)
    # tensor_split ratios ("2,1"), or "even"
    ratios = None if len(sys.argv) <= 6 or sys.argv[6] == "even" else [float(x) for x in sys.argv[6].split(",")]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    ctx = dcpp_b200.Context(local)
    uid = [dcpp_b200.Context.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    ctx.tp_init(rank, world, uid[0])

    c = synth.Flux2Cfg(num_layers=2, num_single_layers=2, num_attention_heads=heads, attention_head_dim=128,
                       joint_attention_dim=64, in_channels=32, timestep_guidance_channels=256, guidance_embeds=True)
    params = synth.make_params(c, wtype, seed=41)
    B, gh, gw, nt = 2, 9, 14, 77
    hid, enc, iid, tid = synth.make_inputs(c, B, gh, gw, nt, seed=42)
    t = torch.tensor([0.8, 0.35], dtype=torch.float32)
    guid = torch.tensor([2.5, 1.0], dtype=torch.float32)
    ni = gh * gw
    res = {}

    m = dcpp_b200.Flux2Model(ctx, c, tp_rank=rank, tp_size=world, tp_split=ratios)
    m.load_params(params)
    m.prepare(B, ni, nt, use_graph=True)
    out = torch.empty(B, ni, c.in_channels, dtype=torch.float32)
    m.forward(hid, enc, t, iid, tid, out, guidance=guid)
    out2 = torch.empty_like(out)
    m.forward(hid, enc, t, iid, tid, out2, guidance=guid)  # graph replay
    m.close()
    # The denoise step passes no guidance (as the Klein pipeline does): a
    # model without the guidance embedder, same other weights.
    c_ng = synth.Flux2Cfg(**{**c.__dict__, "guidance_embeds": False})
    params_ng = {k: v for k, v in params.items() if "guidance_embedder" not in k}
    m = dcpp_b200.Flux2Model(ctx, c_ng, tp_rank=rank, tp_size=world, tp_split=ratios)
    m.load_params(params_ng)
    m.prepare(B, ni, nt, use_graph=True)
    lat = torch.empty_like(hid)
    m.denoise_step(hid, enc, t, -0.25, iid, tid, lat)
    # resident schedule: two steps on the latent kept on the device
    m.load_inputs(hid, enc, iid, tid)
    ts, sg = dcpp_b200.flow_match_schedule(4)
    for i in range(2):
        m.set_timestep(float(ts[i]) / 1000.0, float(sg[i + 1] - sg[i]))
        m.run_resident()
    res_lat = torch.empty_like(hid)
    m.read_latents(res_lat)
    m.close()

    # every rank holds the same replicated result
    peer = out.clone()
    dist.broadcast(peer, src=0)
    res["ranks_identical"] = bool(torch.equal(peer, out))
    if rank == 0:
        o = fo.Flux2Oracle(fo.Config(**{k: getattr(c, k) for k in fo.Config.__dataclass_fields__}), params)
        ref = o.forward(hid, enc, t, iid, tid, guidance=guid)
        res["forward_rel"] = rel(out, ref)
        res["replay_identical"] = bool(torch.equal(out, out2))
        o_ng = fo.Flux2Oracle(fo.Config(**{k: getattr(c_ng, k) for k in fo.Config.__dataclass_fields__}), params_ng)
        ref_nog = o_ng.forward(hid, enc, t, iid, tid)
        res["denoise_rel"] = rel(lat, hid.double() + (-0.25) * ref_nog)
        x = hid.double()
        for i in range(2):
            tt = torch.full((B,), float(ts[i]) / 1000.0)
            x = x + float(sg[i + 1] - sg[i]) * o_ng.forward(x, enc, tt, iid, tid)
        res["resident_rel"] = rel(res_lat, x)
        res["max_abs_latent"] = (lat.double() - (hid.double() - 0.25 * ref_nog)).abs().max().item()
        with open(out_path, "w") as f:
            json.dump(res, f)
    ctx.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
