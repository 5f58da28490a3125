"""Test helper: numpy emulation of the weights the fused-dequant GEMM feeds to
the tensor cores (dcpp_pack_weight + dcpp_gemm_packed).

Per 32-weight block the kernel uses bf16 scales (Q4_K: s = d*sc and
m = dmin*m_code, exact in f32, rounded once to bf16; Q8_0: d rounded to
bf16) and computes one rounding of the exact q*s - m (or q*d) to bf16.
"""
import numpy as np

import flux2_oracle as fo


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float64 values to the nearest bf16 (ties to even), exactly."""
    x = np.asarray(x, dtype=np.float64)
    m, e = np.frexp(x)
    return np.ldexp(np.rint(m * 256.0) / 256.0, e)


def _f16(b0, b1):
    v = np.frombuffer(np.stack([b0, b1], -1).astype(np.uint8).tobytes(), dtype=np.float16).astype(np.float64)
    return v.reshape(np.shape(b0))


def fused_weights(gtype: int, raw: np.ndarray, N: int, K: int) -> np.ndarray:
    raw = np.ascontiguousarray(np.asarray(raw, dtype=np.uint8)).reshape(N, -1)
    if gtype == fo.GGML_Q8_0:
        blk = raw.reshape(N, K // 32, 34)
        d = _f16(blk[..., 0], blk[..., 1]).reshape(N, K // 32, 1)
        q = blk[..., 2:].view(np.int8).astype(np.float64)
        return round_bf16(q * round_bf16(d)).reshape(N, K)
    if gtype == fo.GGML_Q4_K:
        blk = raw.reshape(N, K // 256, 144)
        d = _f16(blk[..., 0], blk[..., 1])[..., None]
        dmin = _f16(blk[..., 2], blk[..., 3])[..., None]
        s = blk[..., 4:16].astype(np.int32)
        sc = np.concatenate([s[..., 0:4] & 63, (s[..., 8:12] & 15) | ((s[..., 0:4] >> 2) & 48)], -1)
        mn = np.concatenate([s[..., 4:8] & 63, (s[..., 8:12] >> 4) | ((s[..., 4:8] >> 2) & 48)], -1)
        sb = round_bf16((d.astype(np.float32) * sc.astype(np.float32)).astype(np.float64))   # [N, nb, 8]
        mb = round_bf16((dmin.astype(np.float32) * mn.astype(np.float32)).astype(np.float64))
        qs = blk[..., 16:].reshape(N, K // 256, 4, 32)
        q = np.stack([qs & 15, qs >> 4], axis=3).reshape(N, K // 256, 8, 32).astype(np.float64)
        return round_bf16(q * sb[..., None] - mb[..., None]).reshape(N, K)
    raise ValueError(gtype)
