"""Benchmark of the Flux2 DiT denoise step (BASELINE.json metric: DiT denoise
steps/s at 1024^2, Q4_K, on 1/2/4/8 B200, plus tensor-pipe fraction of peak).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 2|3|4|5|vae]

One step = one Flux2Transformer2DModel::forward + Euler update on the
resident latent (hidden 3072, 24 heads x 128, 5 double +
20 single blocks, Q4_K weights, 4096 image + 512 text tokens, batch 1).
For N > 1 it is launched under torchrun, one process per GPU, and the model
runs tensor-parallel over the N GPUs (column / row-parallel projections with
an NCCL all-reduce after each row-parallel site); the total work per step is
fixed, so scaling is "strong".

--impl reference times the reference's CPU path on this box's host cores.
The reference's ggml CPU backend cannot be built here (its ggml submodule is
not vendored), so this leg runs the CPU restatement of the same forward
(oracle/flux2_oracle.py, float32, all host threads) on a bounded sample of
the step: one double-stream and one single-stream block at full size, plus
the embeddings and output layers, extrapolated to the 5 + 20 blocks.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "diffusers-cpp_b200")
ORACLE = os.path.join(ROOT, "oracle")
for _p in (PKG, ORACLE):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "DiT denoise steps/s at 1024^2 (Q4_K)"

CONFIGS = {
    # the reduced DiT the reference runs on its CPU
    # path, one denoising step at sigma 0.5 (dt -0.25); the CPU arms time the
    # whole step (no extrapolation).
    "1": dict(model=dict(num_layers=2, num_single_layers=4, num_attention_heads=24, joint_attention_dim=3072,
                         in_channels=128, guidance_embeds=False),
              wtype="Q8_0", batch=1, grid=(32, 32), n_txt=256, single_step=(0.5, -0.25), cpu_full=True,
              metric="DiT denoise steps/s at 512^2 (config 1: Q8_0, 2 double + 4 single blocks)",
              workload="config1: reduced Flux2 DiT (D 3072, 24x128 heads, 2 double + 4 single), Q8_0, "
                       "B=1, 1024 img + 256 txt tokens (3072 features), one denoising step at sigma 0.5"),
    # full-depth Flux2-style DiT on 1 B200.
    "2": dict(model=dict(num_layers=5, num_single_layers=20, num_attention_heads=24, joint_attention_dim=7680,
                         in_channels=128, guidance_embeds=False),
              wtype="Q4_K", batch=1, grid=(64, 64), n_txt=512,
              workload="config2: full-depth Flux2 DiT (D 3072, 24x128 heads, 5 double + 20 single), Q4_K, "
                       "B=1, 4096 img + 512 txt tokens, 4-step flow-match Euler schedule"),
    # larger DiT, tensor-parallel.
    "3": dict(model=dict(num_layers=8, num_single_layers=24, num_attention_heads=32, joint_attention_dim=12288,
                         in_channels=128, guidance_embeds=False),
              wtype="Q8_0", batch=2, grid=(64, 64), n_txt=512,
              workload="config3: Flux2 DiT (D 4096, 32x128 heads, 8 double + 24 single), Q8_0, "
                       "B=2, 4096 img + 512 txt tokens, 4-step flow-match Euler schedule"),
}


# DRAM traffic of the step's dominant kernel (gemm_pair_kernel), per launch,
# averaged over one step's GEMM launches: dram__bytes_read.sum +
# dram__bytes_write.sum from one ncu capture of this bench's own command
# (its summary and command are kept under profiles/).  Keyed by (config, n_gpus).
GEMM_TRAFFIC = {
    ("2", 1): {"dram_bytes_per_launch": 356.4e6, "algorithmic_bytes_per_launch": 298.9e6,
               "source": "ncu dram__bytes_read.sum + dram__bytes_write.sum over the 63 gemm_pair_kernel launches "
                         "of one step of this bench (cold cache), per launch; summary under profiles/"},
}


def weight_bytes(cfg, wtype, world):
    """Weight bytes one GPU moves per step for the block projections
    (the conditioning GEMVs and embedders are excluded): the algorithmic
    quantised bytes, and what the default path moves through memory: the
    quantised read + the bf16 expansion written + the bf16 read back by the
    GEMM (at least once).  Row-parallel shards that are not on the
    quantisation blocks are held as bf16 from load and expanded per step by
    nobody (TP 8 with Q4_K)."""
    D, F = cfg.inner_dim, cfg.mlp_hidden
    bpw = {"Q4_K": 144 / 256, "Q8_0": 34 / 32}[wtype]
    bs = {"Q4_K": 256, "Q8_0": 32}[wtype]
    Dl, Fl = D // world, F // world
    col_par = 3 * Dl * D + 2 * Fl * D            # qkv + gate/up rows of this rank, K = D
    row_dbl = D * Dl + D * Fl                    # to_out (K = Dl) + ff.linear_out (K = Fl)
    row_sgl = D * (Dl + Fl)                      # single-block fused to_out
    aligned = Dl % bs == 0 and Fl % bs == 0
    q_w = cfg.num_layers * 2 * col_par + cfg.num_single_layers * col_par
    r_w = cfg.num_layers * 2 * row_dbl + cfg.num_single_layers * row_sgl
    if aligned:
        q_w += r_w
        bf16_w = 0
    else:
        bf16_w = r_w
    return {"quantised_weights": q_w, "bf16_weights_held_from_load": bf16_w,
            "algorithmic_bytes": q_w * bpw + bf16_w * 2,
            "quantised_read": q_w * bpw, "bf16_expansion_written": q_w * 2, "bf16_gemm_read_min": (q_w + bf16_w) * 2,
            "moved_bytes_min": q_w * bpw + q_w * 2 + (q_w + bf16_w) * 2}


def algorithmic_flops(cfg, batch, n_img, n_txt):
    """FLOPs of one DiT forward: per block 2*S*13*D^2 + 4*S^2*D, embedders,
    batch-1 GEMVs; per batch element."""
    D = cfg.inner_dim
    S = n_img + n_txt
    blocks = cfg.num_layers + cfg.num_single_layers
    per = blocks * (2 * S * 13 * D * D + 4 * S * S * D)
    per += 2 * n_img * cfg.in_channels * D * 2 + 2 * n_txt * cfg.joint_attention_dim * D
    per += 2 * (15 * D * D + 2 * D * D + 256 * D + D * D)
    return batch * per


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled every 5 ms through
    NVML during the timed region (nvidia-smi at its 200 ms minimum period
    would see no sample of a sub-second region); nvidia-smi when NVML is
    unavailable.  Reasons reported: hw_slowdown, hw_thermal_slowdown,
    sw_thermal_slowdown, sw_power_cap."""

    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, cuda_index):
        self.cuda_index = cuda_index
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self.stop_evt = threading.Event()
        self.t = None
        self.h = None
        self.src = "nvml"
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self.nv = pynvml
            try:
                pr = torch.cuda.get_device_properties(cuda_index)
                bus = "%08x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
        except Exception:
            self.h = None
            self.src = "nvidia-smi"

    def _poll(self):
        nv = self.nv
        while not self.stop_evt.is_set():
            try:
                self.samples.append(float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h) if hasattr(
                    nv, "nvmlDeviceGetCurrentClocksEventReasons") else nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                for name, bit in self.BITS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.005)

    def start(self):
        if self.h is not None:
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return
        try:
            q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.cuda_index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.lines = []
            self.t = threading.Thread(target=lambda: [self.lines.append(x.strip()) for x in self.proc.stdout],
                                      daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def stop(self):
        if self.h is not None:
            self.stop_evt.set()
            self.t.join(timeout=2)
        elif getattr(self, "proc", None):
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for ln in self.lines:
                parts = [p.strip() for p in ln.split(",")]
                try:
                    self.samples.append(float(parts[0]))
                    self.max_mhz = float(parts[1])
                except (ValueError, IndexError):
                    continue
                for n, v in zip(names, parts[2:6]):
                    if v.lower().startswith("active"):
                        self.reasons.add(n)
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": self.src}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


# --------------------------------------------------------------------------- reference arm
def cpu_sample(cfg_name, steps, warmup, threads):
    """Time the CPU restatement on a bounded sample of one step; returns
    (seconds per step, sample description)."""
    import torch

    import flux2_oracle as fo
    from dcpp_b200 import synth

    spec = CONFIGS[cfg_name]
    torch.set_num_threads(threads)
    full = synth.Flux2Cfg(**spec["model"])
    if spec.get("cpu_full"):
        return cpu_full_step(spec, full, steps, warmup, threads)
    sample_cfg = synth.Flux2Cfg(**{**spec["model"], "num_layers": 1, "num_single_layers": 1})
    wt = {"Q4_K": 12, "Q8_0": 8}[spec["wtype"]]
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    params = synth.make_params(sample_cfg, wt, seed=0, device=dev)
    gh, gw = spec["grid"]
    hid, enc, iid, tid = synth.make_inputs(sample_cfg, spec["batch"], gh, gw, spec["n_txt"], seed=1)
    ocfg = fo.Config(**{k: getattr(sample_cfg, k) for k in fo.Config.__dataclass_fields__})
    orc = fo.Flux2Oracle(ocfg, params, dtype=torch.float32)
    t = torch.full((spec["batch"],), 0.75)
    # Pre-dequantise the sample's weights (the ggml path keeps quantised
    # weights; dequantisation is not part of the timed sample).
    orc.forward(hid[:, :64], enc[:, :16], t, iid[:64], tid[:16], n_double=1, n_single=1)

    sample_s = []

    def one():
        t0 = time.perf_counter()
        orc.forward(hid, enc, t, iid, tid, n_double=0, n_single=0)
        t1 = time.perf_counter()
        orc.forward(hid, enc, t, iid, tid, n_double=1, n_single=0)
        t2 = time.perf_counter()
        orc.forward(hid, enc, t, iid, tid, n_double=0, n_single=1)
        t3 = time.perf_counter()
        sample_s.append(t3 - t0)
        base = t1 - t0
        dbl = (t2 - t1) - base
        sgl = (t3 - t2) - base
        return base + full.num_layers * dbl + full.num_single_layers * sgl

    for _ in range(warmup):
        one()
    times = [one() for _ in range(steps)]
    desc = (f"CPU restatement (oracle/flux2_oracle.py, torch float32, {threads} threads) of {spec['workload']}; "
            f"each step = 1 double + 1 single block at full size plus embeddings/output, extrapolated to "
            f"{full.num_layers} + {full.num_single_layers} blocks; ggml CPU path unavailable (submodule not vendored)")
    return statistics.median(times), desc, statistics.median(sample_s[warmup:] or sample_s)


def cpu_full_step(spec, cfg, steps, warmup, threads):
    """The whole step of a CPU-sized config through the CPU restatement
    (float32, all host threads), weights dequantised beforehand."""
    import torch

    import flux2_oracle as fo
    from dcpp_b200 import synth

    wt = {"Q4_K": 12, "Q8_0": 8}[spec["wtype"]]
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    params = synth.make_params(cfg, wt, seed=0, device=dev)
    gh, gw = spec["grid"]
    hid, enc, iid, tid = synth.make_inputs(cfg, spec["batch"], gh, gw, spec["n_txt"], seed=1)
    ocfg = fo.Config(**{k: getattr(cfg, k) for k in fo.Config.__dataclass_fields__})
    orc = fo.Flux2Oracle(ocfg, params, dtype=torch.float32)
    sigma, dt = spec["single_step"]
    t = torch.full((spec["batch"],), sigma)
    orc.forward(hid[:, :64], enc[:, :16], t, iid[:64], tid[:16])  # dequantise every weight once
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        orc.denoise(hid, enc, t, dt, iid, tid)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    desc = (f"CPU restatement (oracle/flux2_oracle.py, torch float32, {threads} threads) of {spec['workload']}; "
            f"the whole step timed (no extrapolation); ggml CPU path unavailable (submodule not vendored)")
    return statistics.median(times), desc, statistics.median(times)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    # Each sample is a few seconds of CPU work: at most 3 timed samples after
    # at most 1 warm-up keeps the arm within minutes whatever --steps says.
    steps, warmup = max(1, min(args.steps, 3)), min(args.warmup, 1)
    sec, desc, sample_sec = cpu_sample(args.config, steps, warmup, threads)
    value = 1.0 / sec
    line = {
        "impl": "reference", "metric": CONFIGS[args.config].get("metric", METRIC), "value": value, "unit": "steps/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "extrapolated": not CONFIGS[args.config].get("cpu_full", False), "sample_seconds": sample_sec,
        "extrapolation": ("none: the whole step is timed" if CONFIGS[args.config].get("cpu_full") else
                          "ms_per_step is the full step extrapolated from the timed sample (1 double + 1 single "
                          "block + embeddings/output); each timed sample took sample_seconds of wall time"),
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": CONFIGS[args.config]["workload"], "global_batch": CONFIGS[args.config]["batch"],
                   "seq_len": CONFIGS[args.config]["grid"][0] * CONFIGS[args.config]["grid"][1] + CONFIGS[args.config]["n_txt"],
                   # the GPU arm's job description (the same workload); this
                   # arm runs it on rank 0's host cores (cpu_baseline)
                   "parallelism": f"tp{args.gpus}", "weights": CONFIGS[args.config]["wtype"]},
        "cpu_baseline": {"value": value, "unit": "steps/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------- our arm
def run_ours(args):
    import torch
    import torch.distributed as dist

    import dcpp_b200
    from dcpp_b200 import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))

    spec = CONFIGS[args.config]
    cfg = synth.Flux2Cfg(**spec["model"])
    wt = {"Q4_K": dcpp_b200.TYPE_Q4_K, "Q8_0": dcpp_b200.TYPE_Q8_0}[spec["wtype"]]
    B, (gh, gw), nt = spec["batch"], spec["grid"], spec["n_txt"]
    ni = gh * gw

    ctx = dcpp_b200.Context(local)
    # A dedicated (non-default) stream shared by the library and the timing
    # events: the legacy default stream has handle 0, which the library
    # would read as "use your own stream".
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    assert stream.cuda_stream != 0
    ctx.set_stream(stream.cuda_stream)
    if args.attn_kernel:
        ctx.set_attention_kernel(args.attn_kernel)
    if world > 1:
        uid = [dcpp_b200.Context.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ctx.tp_init(rank, world, uid[0])
    model = dcpp_b200.Flux2Model(ctx, cfg, tp_rank=rank, tp_size=world)
    t0 = time.time()
    params = synth.make_params(cfg, wt, seed=0, device="cuda", to_cpu=False)
    for name, (gt, shp, data) in params.items():
        model.set_param(name, gt, shp, data.cpu())
    del params
    torch.cuda.empty_cache()
    load_s = time.time() - t0
    model.prepare(B, ni, nt, use_graph=not args.no_graph)

    hid, enc, iid, tid = synth.make_inputs(cfg, B, gh, gw, nt, seed=1)
    hid_p, enc_p = hid.pin_memory(), enc.pin_memory()
    out_p = torch.empty_like(hid).pin_memory()
    ts, sg = dcpp_b200.flow_match_schedule(4)
    sched = [(float(ts[i]) / 1000.0, float(sg[i + 1] - sg[i])) for i in range(4)]
    if spec.get("single_step"):  # one denoising step at a fixed sigma, repeated from the same latents
        sched = [tuple(spec["single_step"])] * 4

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident timing (value)
    model.load_inputs(hid_p, enc_p, iid, tid)
    for i in range(args.warmup):
        model.set_timestep(*sched[i % 4])
        model.run_resident()
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    # One untimed step queued right before the start event: its in-step
    # cross-GPU exchanges line the ranks' streams up, so the host-side skew
    # of leaving the barrier above is not timed as device work.
    model.set_timestep(*sched[0])
    model.run_resident()
    ev0.record(stream)
    for i in range(args.steps):
        model.set_timestep(*sched[i % 4])
        model.run_resident()
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    barrier()
    model.read_latents(out_p)
    assert torch.isfinite(out_p).all(), "non-finite latents"

    # ---- end-to-end through the public C ABI with host buffers (e2e)
    for i in range(min(args.warmup, 2)):
        model.denoise_step(hid_p, enc_p, torch.tensor([sched[0][0]]), sched[0][1], iid, tid, out_p)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tsteps = [torch.tensor([s[0]], dtype=torch.float32) for s in sched]
    model.denoise_step(hid_p, enc_p, tsteps[0], sched[0][1], iid, tid, out_p)  # aligns the ranks (untimed)
    e0.record(stream)
    for i in range(args.steps):
        model.denoise_step(hid_p, enc_p, tsteps[i % 4], sched[i % 4][1], iid, tid, out_p)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    barrier()

    # ---- multi-GPU parity: one denoise step of the N-GPU model on fixed inputs
    # against the same step of an unsharded model on rank 0's GPU (all ranks
    # run the sharded step; rank 0 then builds the 1-GPU model from the same
    # seeded weights).
    tp_parity = None
    if world > 1:
        t_par = torch.tensor([sched[1][0]], dtype=torch.float32)
        tp_out = torch.empty_like(hid).pin_memory()
        model.denoise_step(hid_p, enc_p, t_par, sched[1][1], iid, tid, tp_out)
        torch.cuda.synchronize()
        if rank == 0:
            solo = dcpp_b200.Flux2Model(ctx, cfg)
            sp = synth.make_params(cfg, wt, seed=0, device="cuda", to_cpu=False)
            for name, (gt, shp, data) in sp.items():
                solo.set_param(name, gt, shp, data.cpu())
            del sp
            torch.cuda.empty_cache()
            solo.prepare(B, ni, nt, use_graph=False)
            solo_out = torch.empty_like(hid)
            solo.denoise_step(hid_p, enc_p, t_par, sched[1][1], iid, tid, solo_out)
            torch.cuda.synchronize()
            solo.close()
            torch.cuda.empty_cache()
            d = tp_out.double() - solo_out.double()
            tp_parity = {"rel_l2": (d.norm() / solo_out.double().norm()).item(), "max_abs": d.abs().max().item(),
                         "against": "the same denoise step (sigma %.2f) on an unsharded 1-GPU model, same seeded "
                                    "weights and inputs" % sched[1][0]}
        barrier()

    # ---- per-kernel-kind device times: the same step replayed eagerly with a
    # CUDA event pair around every launch (not inside the graph, whose event
    # nodes would perturb the timing).
    model.set_profiling(True)
    model.prepare(B, ni, nt, use_graph=False)
    model.load_inputs(hid_p, enc_p, iid, tid)
    for i in range(3):
        model.set_timestep(*sched[i % 4])
        model.run_resident()
    torch.cuda.synchronize()
    if args.ops_csv and rank == 0:
        os.environ["DCPP_PROFILE_OPS"] = os.path.join(args.ops_csv, f"ops_config{args.config}_tp{world}.csv")
    prof = {k: model.profile(k) for k in dcpp_b200.Flux2Model.PROFILE_KINDS}
    os.environ.pop("DCPP_PROFILE_OPS", None)
    prof_step_ms = sum(v[0] for v in prof.values())

    # max over ranks
    vals = torch.tensor([ms, e2e_ms], dtype=torch.float64)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, e2e_ms = float(vals[0]), float(vals[1])
    launches = model.launches_per_step()

    if rank == 0:
        peak_b, peak_s, hbm, peak_src = measured_peaks()
        traffic = GEMM_TRAFFIC.get((args.config, world), {})
        g_ms, g_fl, g_n = prof["gemm"]
        achieved = g_fl / (g_ms * 1e-3) / 1e12 if g_ms > 0 else 0.0
        step_flops = algorithmic_flops(cfg, B, ni, nt)
        h2d = hid.numel() * 4 + enc.numel() * 4 + iid.numel() * 4 + tid.numel() * 4 + 4 * B + 4
        d2h = hid.numel() * 4
        line = {
            "metric": spec.get("metric", METRIC),
            "value": 1000.0 / ms,
            "unit": "steps/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1/fan_in) weights quantised to %s; N(0,1) inputs)" % spec["wtype"],
            "config": {
                "workload": spec["workload"],
                "global_batch": B,
                "seq_len": ni + nt,
                "parallelism": f"tp{world}",
                "weights": spec["wtype"],
                "l2": "no flush: each step streams %.1f GB of quantised block weights (read, expanded to bf16, "
                      "read again), far above the 126 MB L2" % (weight_bytes(cfg, spec["wtype"], world)["moved_bytes_min"] / 1e9),
                "cuda_graph": not args.no_graph,
                "dequant": ("fused into the GEMM" if os.environ.get("DCPP_FUSED_DEQUANT") == "1"
                            else "per-projection expansion to bf16 before each GEMM"),
                "row_parallel_weights": (None if world == 1 else
                                         "bf16, expanded once at load (row-parallel shards of %d / %d columns are "
                                         "not on the %s blocks), not expanded per step" % (
                                             cfg.inner_dim // world, cfg.mlp_hidden // world, spec["wtype"])
                                         if weight_bytes(cfg, spec["wtype"], world)["bf16_weights_held_from_load"]
                                         else "%s, expanded to bf16 per step like the column-parallel ones"
                                         % spec["wtype"]),
                "tp_exchange": (None if world == 1 else
                                "ncclAllReduce of the row-parallel partials" if os.environ.get("DCPP_TP_COMM") == "nccl"
                                else "GEMM epilogue stores partials into the owner GPU (NVLink peer memory); "
                                     "owner LayerNorm; the next GEMM pushes the rows to the other GPUs and waits "
                                     "per 128-row granule (all-gather overlapped); cross-GPU flag barrier"
                                if os.environ.get("DCPP_TP_OVERLAP") == "1"
                                else "GEMM epilogue stores partials into the owner GPU (NVLink peer memory); "
                                     "owner LayerNorm + all-gather stores; cross-GPU flag barriers"),
            },
            "e2e": {"value": 1000.0 / e2e_ms, "unit": "steps/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "dcpp_flux2_denoise_step with pinned host latents/encoder/ids in, latents out"},
            "gpu_launches": launches * args.steps,
            "tp_parity_rel": tp_parity["rel_l2"] if tp_parity else None,
            "tp_parity": tp_parity,
            "roofline": {
                "bound": "tensor",
                "kernel": "gemm_pair_kernel<0, 256> (bf16 B operand, 256 x 256 tiles; persistent tcgen05 "
                          "cta_group::2 grouped GEMM)",
                "achieved": achieved,
                "peak": peak_s,
                "unit": "TFLOP/s",
                "frac": achieved / peak_s if peak_s else None,
                "peak_kind": f"bf16 sustained ({peak_src})",
                "traffic": traffic.get("dram_bytes_per_launch"),
                "traffic_source": traffic.get("source"),
                "algorithmic_bytes_per_launch": traffic.get("algorithmic_bytes_per_launch"),
                "gemm_ms_per_step": g_ms,
                "gemm_launches_per_step": g_n,
                "step_tflops": step_flops / 1e12,
                "step_frac_of_peak": step_flops / (ms * 1e-3) / 1e12 / (world * peak_s),
                "step_frac_of_peak_note": "whole-job FLOP/s over n_gpus x the per-GPU peak",
            },
            "weight_bytes_per_step": weight_bytes(cfg, spec["wtype"], world),
            "kernel_ms_per_step": {k: round(v[0], 4) for k, v in prof.items()},
            "kernel_ms_sum": prof_step_ms,
            "kernel_timing": "eager replay of one step, CUDA events around each launch on the launching stream",
            "attention_tflops": (prof["attention"][1] / (prof["attention"][0] * 1e-3) / 1e12
                                 if prof["attention"][0] > 0 else None),
            "clocks": clk,
            "load_seconds": load_s,
        }
        if world == 1 and not args.no_cpu_baseline:
            try:
                threads = os.cpu_count() or 1
                sec, desc, sample_sec = cpu_sample(args.config, 1, 0, threads)
                line["cpu_baseline"] = {"value": 1.0 / sec, "unit": "steps/s", "cores": threads, "kind": "port",
                                        "sample": desc, "extrapolated": not spec.get("cpu_full", False),
                                        "sample_seconds": sample_sec}
            except Exception as e:  # the baseline is reported, never the target
                line["cpu_baseline"] = {"value": None, "unit": "steps/s", "cores": os.cpu_count(), "kind": "port",
                                        "sample": f"failed: {e}"}
        print(json.dumps(line), flush=True)
    model.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# --------------------------------------------------------------------------- config 4: Qwen3 prefill
QWEN3_METRIC = "Qwen3 text-encoder prefill tokens/s"


def qwen3_flops(c, B, S):
    D, I, Dq, Dkv = c.hidden_size, c.intermediate_size, c.num_attention_heads * 128, c.num_key_value_heads * 128
    lin = 2 * B * S * (D * (Dq + 2 * Dkv) + Dq * D + 3 * D * I)
    attn = 2 * B * c.num_attention_heads * S * (S + 1) * 128  # causal: half of 4 S^2 d
    return c.num_hidden_layers * (lin + attn)


def qwen3_cpu_sample(steps, warmup, threads):
    """Time the Qwen3 CPU restatement (oracle/qwen3_oracle.py, float32) on a
    bounded sample of one config-4 prefill: the full batch (4 x 512 tokens)
    through one and through two full-width layers, the difference being one
    layer, extrapolated to 36 layers.  The embedding table is cut to 4096
    rows (the gather's cost does not depend on its size).  Returns (seconds
    per prefill, sample description)."""
    import torch

    import qwen3_oracle as qo
    from dcpp_b200 import TYPE_Q8_0, synth

    torch.set_num_threads(threads)
    full = synth.Qwen3Cfg()
    sample = synth.Qwen3Cfg(vocab_size=4096, num_hidden_layers=2)
    params = synth.make_qwen3_params(sample, TYPE_Q8_0, seed=0)
    o = qo.Qwen3Oracle(qo.Qwen3Config(**{k: getattr(sample, k) for k in qo.Qwen3Config.__dataclass_fields__}),
                       params, dtype=torch.float32)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, sample.vocab_size, (4, 512), generator=g)
    o.forward(ids[:, :16], n_layers=2)  # dequantise the weights once (ggml keeps them quantised)

    def one():
        t0 = time.perf_counter()
        o.forward(ids, n_layers=1)
        t1 = time.perf_counter()
        o.forward(ids, n_layers=2)
        t2 = time.perf_counter()
        layer = (t2 - t1) - (t1 - t0)
        return (t1 - t0) - layer + full.num_hidden_layers * layer

    for _ in range(warmup):
        one()
    times = [one() for _ in range(steps)]
    desc = (f"CPU restatement (oracle/qwen3_oracle.py, torch float32, {threads} threads) of config 4 "
            f"(4 x 512 tokens): one and two full-width layers timed, extrapolated to "
            f"{full.num_hidden_layers} layers; ggml CPU path unavailable (submodule not vendored)")
    return statistics.median(times), desc


def run_qwen3_reference(args):
    """--impl reference --config 4: the CPU restatement's bounded sample of a
    prefill (qwen3_cpu_sample), at most 3 timed samples after at most 1
    warm-up (each sample is ~10-20 s of CPU work); rank 0 only."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    threads = os.cpu_count() or 1
    steps, warmup = max(1, min(args.steps, 3)), min(args.warmup, 1)
    sec, desc = qwen3_cpu_sample(steps, warmup, threads)
    tokens = 4 * 512
    value = tokens / sec
    line = {
        "impl": "reference", "metric": QWEN3_METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config4: Qwen3 text-encoder prefill, Q8_0, batch 4 x 512 tokens",
                   "global_batch": 4, "seq_len": 512, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_qwen3(args):
    """36 layers, hidden 2560, 32 / 8 heads x 128, SwiGLU
    9728, Q8_0 weights N(0, 0.02); batch 4 x 512 token ids uniform in the
    151936-token vocabulary; taps 9 / 18 / 27 (what the Flux2 pipeline reads).
    One GPU (the reference has no multi-GPU text encoder path)."""
    import torch

    import dcpp_b200
    from dcpp_b200 import synth

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("--config 4 runs on one GPU")
    c = synth.Qwen3Cfg()
    B, S, taps = 4, 512, (9, 18, 27)
    ctx = dcpp_b200.Context(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    if args.attn_kernel:
        ctx.set_attention_kernel(args.attn_kernel)
    m = dcpp_b200.Qwen3Model(ctx, c)
    t0 = time.time()
    params = synth.make_qwen3_params(c, dcpp_b200.TYPE_Q8_0, seed=0, device="cuda", to_cpu=False)
    for name, (gt, shp, data) in params.items():
        m.set_param(name, gt, shp, data.cpu())
    del params
    torch.cuda.empty_cache()
    load_s = time.time() - t0
    m.prepare(B, S, taps, use_graph=not args.no_graph)
    ids = synth.make_qwen3_ids(c, B, S, seed=1)
    ids_dev = ids.cuda()
    ids_p = ids.pin_memory()
    last = torch.empty(B, S, c.hidden_size, device="cuda")
    tap_dev = torch.empty(B, S, len(taps) * c.hidden_size, device="cuda")
    tap_p = torch.empty(B, S, len(taps) * c.hidden_size).pin_memory()
    for _ in range(args.warmup):
        m.forward(ids_dev, last, tap_dev)
    torch.cuda.synchronize()
    clocks = ClockSampler(0)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        m.forward(ids_dev, last, tap_dev)
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        m.forward(ids_p, None, tap_p)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    assert torch.isfinite(tap_p).all(), "non-finite hidden states"
    m.set_profiling(True)
    m.prepare(B, S, taps, use_graph=False)
    for _ in range(2):
        m.forward(ids_dev, last, tap_dev)
    torch.cuda.synchronize()
    prof = {k: m.profile(k) for k in dcpp_b200.Flux2Model.PROFILE_KINDS}
    launches = m.launches_per_step()
    peak_b, peak_s, hbm, peak_src = measured_peaks()
    g_ms, g_fl, _ = prof["gemm"]
    achieved = g_fl / (g_ms * 1e-3) / 1e12 if g_ms > 0 else 0.0
    tokens = B * S
    line = {
        "metric": QWEN3_METRIC,
        "value": tokens / (ms * 1e-3),
        "unit": "tokens/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights quantised to Q8_0, F32 norms; uniform token ids)",
        "config": {"workload": "config4: Qwen3 text-encoder prefill (36 layers, hidden 2560, 32 q / 8 kv heads x 128, "
                               "SwiGLU 9728, RoPE theta 1e6), Q8_0, batch 4 x 512 tokens, taps 9/18/27",
                   "global_batch": B, "seq_len": S, "parallelism": "tp1",
                   "l2": "no flush: each step streams > 3 GB of weights, far above the 126 MB L2",
                   "cuda_graph": not args.no_graph},
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": ids.numel() * 4,
                "d2h_bytes_per_step": tap_p.numel() * 4,
                "path": "dcpp_qwen3_forward with pinned host ids in, the three tapped hidden states out"},
        "gpu_launches": launches * args.steps,
        "roofline": {"bound": "tensor", "kernel": "gemm_pair_kernel (tcgen05 grouped GEMM)", "achieved": achieved,
                     "peak": peak_s, "unit": "TFLOP/s", "frac": achieved / peak_s if peak_s else None,
                     "peak_kind": f"bf16 sustained ({peak_src})", "traffic": None,
                     "step_tflops": qwen3_flops(c, B, S) / 1e12,
                     "step_frac_of_peak": qwen3_flops(c, B, S) / (ms * 1e-3) / 1e12 / peak_s},
        "kernel_ms_per_step": {k: round(v[0], 4) for k, v in prof.items()},
        "attention_tflops": prof["attention"][1] / (prof["attention"][0] * 1e-3) / 1e12 if prof["attention"][0] else None,
        "clocks": clk,
        "load_seconds": load_s,
    }
    if not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        sec, desc = qwen3_cpu_sample(1, 0, threads)
        line["cpu_baseline"] = {"value": tokens / sec, "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": desc}
    print(json.dumps(line), flush=True)
    m.close()
    ctx.close()
    return 0


VAE_METRIC = "Flux2 VAE decode images/s (1024x1024 by default)"


def vae_cpu_sample(packed, threads, steps=1, warmup=0):
    """The whole VAE decode of one image through the CPU restatement
    (oracle/vae_oracle.py, float32, all host threads); returns (seconds per
    image, description)."""
    import torch

    import vae_oracle as vo
    from dcpp_b200 import synth

    torch.set_num_threads(threads)
    c = synth.VAECfg()
    params = synth.make_vae_params(c, seed=0)
    ocfg = vo.VAEConfig(**{k: getattr(c, k) for k in vo.VAEConfig.__dataclass_fields__ if hasattr(c, k)})
    o = vo.VAEDecoderOracle(ocfg, params, dtype=torch.float32)
    lat = synth.make_vae_latents(c, 1, packed, packed, seed=1)
    o.decode_packed(lat[:, :4], 2, 2)  # dequantise / convert every weight once
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        o.decode_packed(lat, packed, packed)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    px = 16 * packed
    desc = (f"CPU restatement (oracle/vae_oracle.py, torch float32, {threads} threads) of the Flux2 VAE decode of one "
            f"{px} x {px} image, the whole decode timed; ggml CPU path unavailable (submodule not vendored)")
    return statistics.median(times), desc


def run_vae_reference(args):
    """--impl reference --config vae: one timed decode (after none or one
    warm-up) through the CPU restatement; rank 0 only."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    threads = os.cpu_count() or 1
    steps, warmup = 1, min(args.warmup, 1)
    sec, desc = vae_cpu_sample(args.vae_packed, threads, steps, warmup)
    value = 1.0 / sec
    line = {
        "impl": "reference", "metric": VAE_METRIC, "value": value, "unit": "images/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "extrapolated": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"vae: Flux2 VAE decode, {args.vae_packed} x {args.vae_packed} packed tokens",
                   "global_batch": 1, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "images/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_vae(args):
    """The pipeline's VAE decode (Flux2KleinPipeline::decode, untiled) of one
    1024 x 1024 image from 64 x 64 packed tokens, the Flux2 VAE config
    (block_out_channels 128/256/512/512, 2 layers per block, 32 latent
    channels), F32 weights as the reference's converter stores them.  Not a
    BASELINE config: the measurement of the widening row after the denoise
    step.  One GPU."""
    import torch

    import dcpp_b200
    from dcpp_b200 import synth

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("--config vae runs on one GPU")
    c = synth.VAECfg()
    B, ph, pw = 1, args.vae_packed, args.vae_packed
    ctx = dcpp_b200.Context(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    m = dcpp_b200.VAEModel(ctx, c)
    t0 = time.time()
    params = synth.make_vae_params(c, seed=0, device="cuda", to_cpu=False)
    for name, (gt, shp, data) in params.items():
        m.set_param(name, gt, shp, data.cpu())
    del params
    load_s = time.time() - t0
    m.prepare(B, ph, pw, use_graph=not args.no_graph, tile_size=args.vae_tile)
    lat = synth.make_vae_latents(c, B, ph, pw, seed=1)
    lat_dev = lat.cuda()
    lat_p = lat.pin_memory()
    H, W = 2 * ph * 8, 2 * pw * 8
    img = torch.empty(B, c.out_channels, H, W, device="cuda")
    img_p = torch.empty(B, c.out_channels, H, W).pin_memory()
    for _ in range(args.warmup):
        m.decode(lat_dev, img)
    torch.cuda.synchronize()
    clocks = ClockSampler(0)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        m.decode(lat_dev, img)
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        m.decode(lat_p, img_p)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    assert torch.isfinite(img_p).all(), "non-finite image"
    if args.ops_csv:
        os.makedirs(args.ops_csv, exist_ok=True)
        os.environ["DCPP_PROFILE_OPS"] = os.path.join(args.ops_csv, f"ops_vae_{H}.csv")
    m.set_profiling(True)
    m.prepare(B, ph, pw, use_graph=False, tile_size=args.vae_tile)
    for _ in range(2):
        m.decode(lat_dev, img)
    torch.cuda.synchronize()
    prof = {k: m.profile(k) for k in dcpp_b200.Flux2Model.PROFILE_KINDS}
    launches = m.launches_per_step()
    peak_b, peak_s, hbm, peak_src = measured_peaks()
    g_ms, g_fl, _ = prof["gemm"]
    achieved = g_fl / (g_ms * 1e-3) / 1e12 if g_ms > 0 else 0.0
    total_fl = sum(v[1] for v in prof.values())
    line = {
        "metric": VAE_METRIC,
        "value": B / (ms * 1e-3),
        "unit": "images/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1/fan_in) F32 weights; N(0,1) packed latents)",
        "config": {"workload": f"vae: Flux2 VAE decode (128/256/512/512 channels, 2 layers per block, 32 latent "
                               f"channels), {ph} x {pw} packed tokens -> {H} x {W} image, "
                               + (f"tiled ({args.vae_tile}-pixel tiles)" if args.vae_tile else "untiled"),
                   "global_batch": B, "parallelism": "tp1",
                   "l2": "no flush: every decode streams > 10 GB of activations through the 126 MB L2",
                   "cuda_graph": not args.no_graph},
        "e2e": {"value": B / (e2e_ms * 1e-3), "unit": "images/s", "h2d_bytes_per_step": lat.numel() * 4,
                "d2h_bytes_per_step": img_p.numel() * 4,
                "path": "dcpp_vae_decode with pinned host latents in, the f32 image out"},
        "gpu_launches": launches * args.steps,
        "roofline": {"bound": "tensor", "kernel": "gemm_pair_kernel (implicit-GEMM convolutions)",
                     "achieved": achieved, "peak": peak_s, "unit": "TFLOP/s",
                     "frac": achieved / peak_s if peak_s else None, "peak_kind": f"bf16 sustained ({peak_src})",
                     "traffic": None, "step_tflops": total_fl / 1e12,
                     "step_frac_of_peak": total_fl / (ms * 1e-3) / 1e12 / peak_s},
        "kernel_ms_per_step": {k: round(v[0], 4) for k, v in prof.items()},
        "clocks": clk,
        "load_seconds": load_s,
    }
    if not args.no_cpu_baseline and not args.vae_tile:
        threads = os.cpu_count() or 1
        sec, desc = vae_cpu_sample(args.vae_packed, threads)
        line["cpu_baseline"] = {"value": 1.0 / sec, "unit": "images/s", "cores": threads, "kind": "port",
                                "sample": desc}
    print(json.dumps(line), flush=True)
    m.close()
    ctx.close()
    return 0


GEMM_METRIC = "quantized GEMM TFLOP/s (config-5 sweep)"
GEMM_TYPES = {"Q4_K": 12, "Q8_0": 8, "F16": 1, "BF16": 30}
GEMM_SWEEP_M = (256, 1024, 4096, 8192)
GEMM_SWEEP_NK = ((3072, 3072), (9216, 3072), (3072, 9216), (12288, 4096))


def run_gemm_reference(args):
    """--impl reference --config 5: the CPU restatement of the quantised GEMM
    (dequantisation by oracle/dequant.c, then a torch float32 matmul on all
    host threads) over the Q4_K rows of the sweep (every M, every (N, K));
    value = total FLOP / total time, as the GPU arm reports it.  Rank 0 only."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    import torch

    import flux2_oracle as fo
    from dcpp_b200 import quant

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    tot_fl = tot_s = 0.0
    for (N, K) in GEMM_SWEEP_NK:
        w = torch.randn(N, K, generator=g) / K ** 0.5
        wq = quant.quantize(w, GEMM_TYPES["Q4_K"]).numpy()
        for M in GEMM_SWEEP_M:
            x = torch.randn(M, K, generator=g).to(torch.bfloat16).float()
            t0 = time.perf_counter()
            wd = torch.from_numpy(fo.dequant(GEMM_TYPES["Q4_K"], wq, N * K).reshape(N, K))
            y = x @ wd.t()
            tot_s += time.perf_counter() - t0
            tot_fl += 2.0 * M * N * K
            del y, wd
    value = tot_fl / tot_s / 1e12
    desc = (f"CPU restatement (oracle/dequant.c dequantisation + torch float32 matmul, {threads} threads) of the "
            f"config-5 sweep's Q4_K shapes (M in {list(GEMM_SWEEP_M)}, (N, K) in {list(GEMM_SWEEP_NK)}); ggml CPU "
            f"path unavailable (submodule not vendored)")
    line = {
        "impl": "reference", "metric": GEMM_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": 1, "warmup": 0, "ms_per_step": tot_s * 1e3, "higher_is_better": True, "extrapolated": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config5: quantized GEMM sweep, Q4_K shapes", "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_gemm_sweep(args):
    """dcpp_gemm (weight expansion to bf16 + tcgen05 GEMM,
    f32 output) for Q4_K / Q8_0 / F16 weights N(0, 1/K) and bf16 activations
    N(0, 1), M x (N, K) over the sweep grid (or --gemm-shapes
    TYPE:M:N:K,...).  Each timed call runs after a 256 MB write that flushes
    L2 and behind a device-side sleep that hides the host's launch time;
    CUDA events bracket the call alone.  One GPU."""
    import torch

    import dcpp_b200
    from dcpp_b200 import quant

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("--config 5 runs on one GPU")
    if args.gemm_shapes:
        shapes = []
        for item in args.gemm_shapes.split(","):
            t, m, n, k = item.split(":")
            shapes.append((t, int(m), int(n), int(k)))
    else:
        shapes = [(t, m, n, k) for t in ("Q4_K", "Q8_0", "F16") for (n, k) in GEMM_SWEEP_NK for m in GEMM_SWEEP_M]
    ctx = dcpp_b200.Context(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    peak_b, peak_s, hbm, peak_src = measured_peaks()
    g = torch.Generator().manual_seed(0)
    weights = {}
    results = []
    clocks = ClockSampler(0)
    clocks.start()
    tot_fl = tot_ms = 0.0
    for t, M, N, K in shapes:
        key = (t, N, K)
        if key not in weights:
            weights.clear()
            w = torch.randn(N, K, generator=g) / K ** 0.5
            weights[key] = (quant.quantize(w, GEMM_TYPES[t]) if t != "BF16" else w.to(torch.bfloat16).view(torch.uint8)).cuda()
        wq = weights[key]
        x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
        y = torch.empty(M, N, dtype=torch.float32, device="cuda")
        for _ in range(args.warmup):
            ctx.gemm(GEMM_TYPES[t], wq, N, K, x, M, y)
        ms = 0.0
        for _ in range(args.steps):
            flush.zero_()
            torch.cuda._sleep(2_000_000)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            ctx.gemm(GEMM_TYPES[t], wq, N, K, x, M, y)
            e1.record(stream)
            e1.synchronize()
            ms += e0.elapsed_time(e1)
        ms /= args.steps
        assert torch.isfinite(y).all(), "non-finite GEMM output"
        fl = 2.0 * M * N * K
        tf = fl / (ms * 1e-3) / 1e12
        tot_fl += fl
        tot_ms += ms
        results.append({"wtype": t, "M": M, "N": N, "K": K, "ms": round(ms, 4), "tflops": round(tf, 1),
                        "frac_of_peak": round(tf / peak_b, 3)})
    clk = clocks.stop()
    agg = tot_fl / (tot_ms * 1e-3) / 1e12
    line = {
        "metric": GEMM_METRIC,
        "value": agg,
        "unit": "TFLOP/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": tot_ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (weights N(0,1/K) quantised on the host; activations N(0,1) bf16)",
        "config": {"workload": "config5: dcpp_gemm sweep, weight expansion + tcgen05 GEMM, f32 output; value = "
                               "total FLOP / total time over the shapes",
                   "l2": "flushed (256 MB write) before every timed call", "parallelism": "tp1"},
        "roofline": {"bound": "tensor", "kernel": "gemm_pair_kernel (after the bf16 expansion)", "achieved": agg,
                     "peak": peak_b, "unit": "TFLOP/s", "frac": agg / peak_b, "peak_kind": f"bf16 burst ({peak_src})",
                     "traffic": None},
        "shapes": results,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    ctx.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS) + ["4", "5", "vae"], default="2")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ops-csv", default=None, help="directory for a per-op time CSV of the profiled step (rank 0)")
    ap.add_argument("--attn-kernel", type=int, default=0, help="0 auto, 1 one query tile per CTA, 2 two tiles")
    ap.add_argument("--vae-packed", type=int, default=64, help="--config vae: packed tokens per side (64: 1024^2)")
    ap.add_argument("--vae-tile", type=int, default=0, help="--config vae: decode_tiled tile size in pixels (0: untiled)")
    ap.add_argument("--gemm-shapes", default=None, help="--config 5: TYPE:M:N:K[,...] instead of the sweep grid")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.config == "4":
        if args.impl == "reference":
            return run_qwen3_reference(args)
        return run_qwen3(args)
    if args.config == "5":
        if args.impl == "reference":
            return run_gemm_reference(args)
        return run_gemm_sweep(args)
    if args.config == "vae":
        if args.impl == "reference":
            return run_vae_reference(args)
        return run_vae(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
