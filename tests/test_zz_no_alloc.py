"""GPU test of dcpp_gemm_noalloc, the GEMM entry point for callers that
cannot allocate device memory (their device memory is owned by a host
framework's pool, or must not change while they record work).

It goes through the C ABI and must give the same result as dcpp_gemm (the
allocating entry point) within the GEMM tolerance of the other tests, on two
calls in a row (the second call reuses the shared fixed scratch that the first
one filled).  This file is named to be collected last, and it creates its own
context so that it passes alone in a fresh process as well as after the
other tests.
"""
import pytest
import torch

import dcpp_b200
import flux2_oracle as fo
from dcpp_b200 import quant

pytestmark = pytest.mark.gpu


def case(gtype, M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) / K ** 0.5
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    return quant.quantize(w, gtype).cuda(), x.cuda()


def test_noalloc_gemm_matches_gemm_on_two_calls():
    ctx = dcpp_b200.Context(0)
    try:
        # Call 1: Q4_K, 6144 x 3072 expands to 36 MiB of bf16 -> two row chunks.
        # Call 2: Q8_0 with another shape, reusing the same scratch.
        for gtype, M, N, K, seed in ((fo.GGML_Q4_K, 777, 6144, 3072, 1), (fo.GGML_Q8_0, 300, 520, 512, 2)):
            w, x = case(gtype, M, N, K, seed)
            ref = torch.empty(M, N, dtype=torch.float32, device="cuda")
            out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
            ctx.gemm(gtype, w, N, K, x, M, ref)
            ctx.gemm_noalloc(gtype, w, N, K, x, M, out)
            ctx.synchronize()
            err = (out - ref).abs().max().item()
            scale = ref.abs().max().item()
            assert err <= 1e-4 * max(scale, 1.0) + 1e-5, (gtype, err, scale)
    finally:
        ctx.close()


def test_noalloc_gemm_rejects_k_beyond_its_scratch():
    ctx = dcpp_b200.Context(0)
    try:
        K = 65536 + 256
        w = torch.zeros(K // 256 * 144, dtype=torch.uint8, device="cuda")
        x = torch.zeros(1, K, dtype=torch.bfloat16, device="cuda")
        y = torch.zeros(1, 1, dtype=torch.float32, device="cuda")
        with pytest.raises(dcpp_b200.DcppError) as e:
            ctx.gemm_noalloc(fo.GGML_Q4_K, w, 1, K, x, 1, y)
        assert e.value.status == 2 and "65536" in str(e.value)
    finally:
        ctx.close()
