"""GPU tests of the fused-dequant GEMM (dcpp_pack_weight + dcpp_gemm_packed)
through the C ABI: against a float64 product of the same bf16 operands the
kernel computes (tight), and against the exact dequantised weights (loose)."""
import numpy as np
import pytest
import torch

import dcpp_b200
import flux2_oracle as fo
from dcpp_b200 import quant
from fused_emulation import fused_weights

pytestmark = pytest.mark.gpu


def run_fused(ctx, gtype, M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) / K ** 0.5
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    raw = quant.quantize(w, gtype)
    packed = torch.empty(dcpp_b200.packed_bytes(gtype, N, K), dtype=torch.uint8, device="cuda")
    ctx.pack_weight(gtype, raw.cuda(), N, K, packed)
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    ctx.gemm_packed(gtype, packed, N, K, x.cuda(), M, y)
    ctx.synchronize()
    xd = x.double().numpy()
    emu = fused_weights(gtype, raw.numpy(), N, K)
    exact = fo.dequant(gtype, raw.numpy(), N * K).reshape(N, K).astype(np.float64)
    return y.cpu().double().numpy(), xd @ emu.T, xd @ exact.T


@pytest.mark.parametrize("gtype", [fo.GGML_Q4_K, fo.GGML_Q8_0])
@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (300, 520, 512), (7, 33, 768), (1024, 768, 3072)])
def test_fused_gemm_matches_emulated_operands(ctx, gemm_kind, gtype, M, N, K):
    y, ref, ref_exact = run_fused(ctx, gtype, M, N, K, seed=M + N)
    scale = np.abs(ref).max()
    assert np.abs(y - ref).max() <= 1e-4 * max(scale, 1.0) + 1e-5
    rel = np.linalg.norm(y - ref_exact) / np.linalg.norm(ref_exact)
    assert rel < 1e-2, rel


def test_fused_gemm_many_tiles_large_k(ctx, gemm_kind):
    y, ref, _ = run_fused(ctx, fo.GGML_Q4_K, 4608, 2304, 9216, seed=3)
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert rel < 3e-5, rel


def test_pack_weight_rejects_bad_k(ctx):
    raw = torch.zeros(144, dtype=torch.uint8, device="cuda")
    out = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    with pytest.raises(dcpp_b200.DcppError) as e:
        ctx.pack_weight(fo.GGML_Q8_0, raw, 1, 96, out)
    assert e.value.status == 2
