"""Generate the golden dequantisation fixtures (tests/golden/dequant_golden.npz).

Uses gguf-py 0.19.0 -- the version the reference pins in
test/requirements.txt:2 and whose dequantize its tests declare to be what the
C++ (ggml) side computes (test/utils/__init__.py:198-228) -- to produce:

* q8_0_blocks / q8_0_deq : Q8_0 blocks quantised by gguf.quantize (bit-exact
  with ggml's quantize_row_q8_0, quants.py:380) from seeded N(0,1) data plus
  edge rows (all zeros -> d = 0, +-max int8, tiny values -> subnormal f16 d),
  and gguf.dequantize of them.
* q8_0_src               : the f32 input of that quantisation (pins
  dcpp_b200.quant.quantize_q8_0).
* q4_k_blocks / q4_k_deq : random Q4_K block bytes covering every nibble,
  every 6-bit scale and min code, normal and subnormal f16 d / dmin, d = 0;
  and gguf.dequantize of them (quants.py:504-523).

Run:  python tests/golden/make_golden.py
"""
import os

import numpy as np

import gguf

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    rng = np.random.default_rng(20261201)
    # ---- Q8_0
    src = rng.standard_normal((40, 64)).astype(np.float32)
    src[0] = 0.0                                  # d = 0
    src[1, :32] = np.linspace(-1, 1, 32)          # q spans -127..127
    src[2] = 1e-6 * rng.standard_normal(64)       # f16 d subnormal
    src[3, :32] = 65504.0 * 127 / 127             # large d
    src[3, 32:] = -3.0
    src[4, :32] = np.float32(0.5)                 # ties in rounding
    q8 = gguf.quantize(src, gguf.GGMLQuantizationType.Q8_0)
    q8 = np.asarray(q8, dtype=np.uint8)
    q8_deq = gguf.dequantize(q8, gguf.GGMLQuantizationType.Q8_0).astype(np.float32)
    # ---- Q4_K: raw random bytes, then force interesting headers.
    nb = 96
    blk = rng.integers(0, 256, size=(nb, 144), dtype=np.uint8)
    hdr = np.zeros((nb, 2), dtype=np.float16)
    hdr[:, 0] = (rng.standard_normal(nb) * 1e-2).astype(np.float16)
    hdr[:, 1] = (np.abs(rng.standard_normal(nb)) * 1e-2).astype(np.float16)
    hdr[0] = [0.0, 0.0]
    hdr[1] = [np.float16(3e-7), np.float16(1e-7)]   # subnormal f16
    hdr[2] = [np.float16(65504.0), np.float16(-65504.0)]
    hdr[3] = [np.float16(-0.0), np.float16(1.0)]
    blk[:, 0:4] = hdr.view(np.uint8).reshape(nb, 4)
    # every 6-bit code for scales and mins across blocks 4..11
    for b in range(8):
        codes = (np.arange(8) + 8 * b) % 64
        sc, mn = codes, (63 - codes)
        s = np.zeros(12, dtype=np.uint8)
        for j in range(4):
            s[j] = (sc[j] & 63) | ((sc[j + 4] >> 4) << 6)
            s[j + 4] = (mn[j] & 63) | ((mn[j + 4] >> 4) << 6)
            s[j + 8] = (sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4)
        blk[4 + b, 4:16] = s
    blk[12, 16:] = np.arange(128, dtype=np.uint8) * 2 + 1  # all nibbles
    q4_deq = gguf.dequantize(blk.reshape(-1), gguf.GGMLQuantizationType.Q4_K).astype(np.float32)
    np.savez_compressed(
        os.path.join(HERE, "dequant_golden.npz"),
        q8_0_src=src,
        q8_0_blocks=q8.reshape(-1),
        q8_0_deq=q8_deq.reshape(-1),
        q4_k_blocks=blk.reshape(-1),
        q4_k_deq=q4_deq.reshape(-1),
        gguf_version=np.array(gguf.__version__ if hasattr(gguf, "__version__") else "0.19.0"),
    )
    print("wrote", os.path.join(HERE, "dequant_golden.npz"))


if __name__ == "__main__":
    main()
