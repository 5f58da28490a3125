"""GPU parity tests of the op-level C ABI entry points against the oracle
(dequant: bit-exact) and against torch fp32 references of the same op
(GEMM, LayerNorm+modulation, attention)."""
import os

import numpy as np
import pytest
import torch

import dcpp_b200
import flux2_oracle as fo
from dcpp_b200 import quant

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "dequant_golden.npz")


def dev_bytes(arr) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(arr, dtype=np.uint8)).cuda()


@pytest.mark.parametrize("kind", ["q8_0", "q4_k"])
def test_dequant_golden_bit_exact(ctx, kind):
    g = np.load(GOLDEN)
    blocks, ref = g[f"{kind}_blocks"], g[f"{kind}_deq"]
    gtype = fo.GGML_Q8_0 if kind == "q8_0" else fo.GGML_Q4_K
    out = torch.empty(ref.size, dtype=torch.float32, device="cuda")
    ctx.dequant(gtype, dev_bytes(blocks), ref.size, out)
    ctx.synchronize()
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("gtype,n", [(fo.GGML_Q8_0, 256 * 37), (fo.GGML_Q4_K, 256 * 37), (fo.GGML_F16, 256 * 37),
                                     (fo.GGML_BF16, 256 * 37), (fo.GGML_F32, 256 * 37), (fo.GGML_F16, 1001),
                                     (fo.GGML_BF16, 999), (fo.GGML_F32, 13)])
def test_dequant_random_bit_exact_vs_oracle(ctx, gtype, n):
    """Block formats, and the element formats on both the 8-wide and the ragged path."""
    g = torch.Generator().manual_seed(gtype)
    x = torch.randn(n, generator=g) * 0.1
    blocks = quant.quantize(x.reshape(1, -1), gtype).reshape(-1).numpy()
    ref = fo.dequant(gtype, blocks, n)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    ctx.dequant(gtype, dev_bytes(blocks), n, out)
    outb = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    ctx.dequant_bf16(gtype, dev_bytes(blocks), n, outb)
    ctx.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    assert torch.equal(outb.cpu(), torch.from_numpy(ref).to(torch.bfloat16))


def test_dequant_rejects_ragged(ctx):
    blk = torch.zeros(144, dtype=torch.uint8, device="cuda")
    out = torch.empty(256, dtype=torch.float32, device="cuda")
    with pytest.raises(dcpp_b200.DcppError) as e:
        ctx.dequant(fo.GGML_Q4_K, blk, 100, out)
    assert e.value.status == 1


def gemm_case(ctx, gtype, M, N, K, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) / K ** 0.5
    x = torch.randn(M, K, generator=g)
    wq = quant.quantize(w, gtype)
    wdeq = torch.from_numpy(fo.dequant(gtype, wq.numpy(), N * K).reshape(N, K))
    xb = x.to(torch.bfloat16)
    ref = xb.float().double() @ wdeq.to(torch.bfloat16).double().t()
    y = torch.empty(M, N, dtype=torch.float32, device="cuda")
    ctx.gemm(gtype, wq.cuda(), N, K, xb.cuda(), M, y)
    ctx.synchronize()
    return y.cpu().double(), ref


@pytest.mark.parametrize("gtype", [fo.GGML_BF16, fo.GGML_Q8_0, fo.GGML_Q4_K, fo.GGML_F16])
@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (300, 520, 512), (7, 33, 256), (1024, 768, 3072)])
def test_gemm_matches_fp32_reference(ctx, gemm_kind, gtype, M, N, K):
    y, ref = gemm_case(ctx, gtype, M, N, K)
    err = (y - ref).abs().max().item()
    scale = ref.abs().max().item()
    # bf16 operands, f32 accumulation: only summation order differs.
    assert err <= 1e-4 * max(scale, 1.0) + 1e-5, (err, scale)


def test_gemm_large_k_and_many_tiles(ctx, gemm_kind):
    y, ref = gemm_case(ctx, fo.GGML_Q4_K, 4608, 2304, 9216, seed=7)
    rel = ((y - ref).norm() / ref.norm()).item()
    # f32 accumulation over K = 9216 in the tensor-core order vs float64
    assert rel < 3e-5, rel


def test_layernorm_mod_matches_reference(ctx):
    g = torch.Generator().manual_seed(1)
    R, D = 333, 3072
    x = torch.randn(R, D, generator=g) * 3 + 1
    shift = torch.randn(D, generator=g)
    scale = torch.randn(D, generator=g) * 0.1
    y = torch.empty(R, D, dtype=torch.bfloat16, device="cuda")
    ctx.layernorm_mod(x.cuda(), R, D, shift.cuda(), scale.cuda(), 1e-6, y)
    ctx.synchronize()
    ref = fo.layer_norm(x.double(), 1e-6) * (1 + scale.double()) + shift.double()
    err = (y.cpu().double() - ref).abs().max().item()
    assert err < 0.02 * ref.abs().max().item()
    assert ((y.cpu().double() - ref).norm() / ref.norm()).item() < 4e-3


def test_attention_full_size_all_heads(ctx, attn_kind):
    """The config-2 attention shape (S = 4608, 24 heads), every head checked
    against the float64 restatement (run on the GPU in float64 only to
    finish in seconds)."""
    B, S, H = 1, 4608, 24
    g = torch.Generator().manual_seed(11)
    D = H * 128
    qkv = torch.randn(B, S, 3 * D, generator=g).to(torch.bfloat16)
    wq = 1 + 0.1 * torch.randn(128, generator=g)
    wk = 1 + 0.1 * torch.randn(128, generator=g)
    ids = torch.zeros(S, 4, dtype=torch.int32)
    ids[512:, 1] = (torch.arange(S - 512, dtype=torch.int32) // 64)
    ids[512:, 2] = (torch.arange(S - 512, dtype=torch.int32) % 64)
    ids[:512, 3] = torch.arange(512, dtype=torch.int32)
    out = torch.empty(B, S, D, dtype=torch.bfloat16, device="cuda")
    ctx.attention(qkv.cuda(), B, S, H, wq.cuda(), wk.cuda(), 1e-6, ids.cuda(), (32, 32, 32, 32), 2000.0, out)
    ctx.synchronize()
    cos, sin = fo.rope_cos_sin(ids.cuda(), (32, 32, 32, 32), 2000, torch.float64)
    x = qkv.cuda().double()
    q = x[..., :D].unflatten(-1, (H, 128))
    k = x[..., D:2 * D].unflatten(-1, (H, 128))
    v = x[..., 2 * D:].unflatten(-1, (H, 128))
    q = fo.apply_rope(fo.rms_norm(q, wq.cuda().double(), 1e-6), cos, sin)
    k = fo.apply_rope(fo.rms_norm(k, wk.cuda().double(), 1e-6), cos, sin)
    ref = fo.sdpa(q, k, v)
    got = out.double().unflatten(-1, (H, 128))
    worst = 0.0
    for h in range(H):
        rel = ((got[:, :, h] - ref[:, :, h]).norm() / ref[:, :, h].norm()).item()
        worst = max(worst, rel)
        assert rel < 1e-2, (h, rel)
    print(f"attention S={S} H={H}: worst per-head rel-L2 {worst:.2e}")


@pytest.mark.parametrize("B,S,H", [(1, 200, 2), (2, 333, 3), (1, 1024, 4), (1, 64, 1), (1, 300, 1)])
def test_attention_matches_oracle(ctx, attn_kind, B, S, H):
    g = torch.Generator().manual_seed(S)
    D = H * 128
    qkv = torch.randn(B, S, 3 * D, generator=g).to(torch.bfloat16)
    wq = 1 + 0.1 * torch.randn(128, generator=g)
    wk = 1 + 0.1 * torch.randn(128, generator=g)
    ids = torch.zeros(S, 4, dtype=torch.int32)
    ids[:, 1] = torch.arange(S, dtype=torch.int32) // 16
    ids[:, 2] = torch.arange(S, dtype=torch.int32) % 16
    ids[:, 3] = torch.arange(S, dtype=torch.int32) % 7
    out = torch.empty(B, S, D, dtype=torch.bfloat16, device="cuda")
    ctx.attention(qkv.cuda(), B, S, H, wq.cuda(), wk.cuda(), 1e-6, ids.cuda(), (32, 32, 32, 32), 2000.0, out)
    ctx.synchronize()
    x = qkv.double()
    q, k, v = x[..., :D].unflatten(-1, (H, 128)), x[..., D:2 * D].unflatten(-1, (H, 128)), x[..., 2 * D:].unflatten(-1, (H, 128))
    cos, sin = fo.rope_cos_sin(ids, (32, 32, 32, 32), 2000, torch.float64)
    q = fo.apply_rope(fo.rms_norm(q, wq.double(), 1e-6), cos, sin)
    k = fo.apply_rope(fo.rms_norm(k, wk.double(), 1e-6), cos, sin)
    ref = fo.sdpa(q, k, v).flatten(2)
    rel = ((out.cpu().double() - ref).norm() / ref.norm()).item()
    assert rel < 1e-2, rel


@pytest.mark.parametrize("S", [1024, 333])
def test_attention_growing_scores(ctx, attn_kind, S):
    """Keys turn from anti-aligned to aligned with every query along the
    sequence, the score rising linearly with the key index (no rotary
    rotation: all position ids 0), so each key tile's row maximum exceeds the
    running one by more than the lazy-rescale threshold (2^8): every tile
    takes the rescale path."""
    H, D = 2, 256
    g = torch.Generator().manual_seed(5)
    u = torch.randn(128, generator=g)
    v = torch.randn(128, generator=g)
    v -= (v @ u) / (u @ u) * u
    u, v = u / u.norm(), v / v.norm()
    cs = torch.linspace(-1.0, 1.0, S)
    keys = cs[:, None] * u + torch.sqrt(1 - cs * cs)[:, None] * v
    qkv = torch.zeros(1, S, 3 * D)
    for h in range(H):
        qkv[0, :, h * 128:(h + 1) * 128] = u + 0.05 * torch.randn(S, 128, generator=g)
        qkv[0, :, D + h * 128:D + (h + 1) * 128] = keys
        qkv[0, :, 2 * D + h * 128:2 * D + (h + 1) * 128] = torch.randn(S, 128, generator=g)
    qkv = qkv.to(torch.bfloat16)
    w = torch.full((128,), 2.0)
    ids = torch.zeros(S, 4, dtype=torch.int32)
    out = torch.empty(1, S, D, dtype=torch.bfloat16, device="cuda")
    ctx.attention(qkv.cuda(), 1, S, H, w.cuda(), w.cuda(), 1e-6, ids.cuda(), (32, 32, 32, 32), 2000.0, out)
    ctx.synchronize()
    x = qkv.double()
    q, k, vv = x[..., :D].unflatten(-1, (H, 128)), x[..., D:2 * D].unflatten(-1, (H, 128)), x[..., 2 * D:].unflatten(-1, (H, 128))
    q = fo.rms_norm(q, w.double(), 1e-6)
    k = fo.rms_norm(k, w.double(), 1e-6)
    ref = fo.sdpa(q, k, vv).flatten(2)
    rel = ((out.cpu().double() - ref).norm() / ref.norm()).item()
    assert rel < 1e-2, rel
