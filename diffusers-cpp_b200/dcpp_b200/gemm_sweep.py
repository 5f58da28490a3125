"""Quantised GEMM sweep on one B200 (the reference benchmark's GEMM sweep
configuration): Q4_K, Q8_0 and F16 weights W [N, K] (seeded N(0, 1/K)) times
bf16 activations X [M, K] (N(0, 1)), M in {256, 1024, 4096, 8192},
(N, K) in {(3072, 3072), (9216, 3072), (3072, 9216), (12288, 4096)}.

For every shape it times, with CUDA events on the launching stream after
warm-up, three library paths:
  * ``expand+gemm``: dcpp_gemm (weight expanded to bf16 in scratch, then the
    tcgen05 GEMM) -- what the model runs per projection by default;
  * ``gemm_bf16``: the GEMM alone on a pre-expanded bf16 weight;
  * ``fused``: dcpp_gemm_packed, dequantisation fused into the GEMM (Q4_K /
    Q8_0 only).
and prints one JSON line per (type, shape, path) with TFLOP/s (2 M N K per
call) and the fraction of the measured dense bf16 peak.

    python -m dcpp_b200.gemm_sweep [--iters 20] [--out sweep.jsonl]
"""
from __future__ import annotations

import argparse
import json
import os

import torch

import dcpp_b200
from dcpp_b200 import quant

TYPES = {"Q4_K": dcpp_b200.TYPE_Q4_K, "Q8_0": dcpp_b200.TYPE_Q8_0, "F16": dcpp_b200.TYPE_F16}
MS = (256, 1024, 4096, 8192)
NKS = ((3072, 3072), (9216, 3072), (3072, 9216), (12288, 4096))


def peak_tflops():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f).get("bf16_tflops", 1590.0)), "measured"
    return 1590.0, "fallback"


def time_call(fn, stream, iters):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--types", default="Q4_K,Q8_0,F16")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    peak, src = peak_tflops()
    ctx = dcpp_b200.Context(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    out = open(args.out, "w") if args.out else None
    g = torch.Generator(device="cuda")
    for tname in args.types.split(","):
        gt = TYPES[tname]
        for (N, K) in NKS:
            g.manual_seed(N * 131 + K)
            w = torch.randn(N, K, device="cuda", generator=g) / K ** 0.5
            wq = quant.quantize(w, gt).contiguous()
            wb = torch.empty(N, K, dtype=torch.bfloat16, device="cuda")
            ctx.dequant_bf16(gt, wq, N * K, wb)
            packed = None
            if gt in (dcpp_b200.TYPE_Q4_K, dcpp_b200.TYPE_Q8_0):
                packed = torch.empty(dcpp_b200.packed_bytes(gt, N, K), dtype=torch.uint8, device="cuda")
                ctx.pack_weight(gt, wq, N, K, packed)
            for M in MS:
                x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
                y = torch.empty(M, N, dtype=torch.float32, device="cuda")
                paths = {
                    "expand+gemm": lambda: ctx.gemm(gt, wq, N, K, x, M, y),
                    "gemm_bf16": lambda: ctx.gemm(dcpp_b200.TYPE_BF16, wb, N, K, x, M, y),
                }
                if packed is not None:
                    paths["fused"] = lambda: ctx.gemm_packed(gt, packed, N, K, x, M, y)
                for path, fn in paths.items():
                    ms = time_call(fn, stream, args.iters)
                    tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
                    line = {"weights": tname, "M": M, "N": N, "K": K, "path": path, "ms": round(ms, 5),
                            "tflops": round(tf, 1), "frac_of_peak": round(tf / peak, 3),
                            "peak": peak, "peak_kind": f"bf16 burst ({src})"}
                    print(json.dumps(line), flush=True)
                    if out:
                        out.write(json.dumps(line) + "\n")
                del x, y
            del w, wq, wb, packed
            torch.cuda.empty_cache()
    if out:
        out.close()
    ctx.close()


if __name__ == "__main__":
    main()
