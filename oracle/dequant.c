/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for ggml weight-block
 * dequantisation.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference leg may load this; the product path never does.
 *
 * Plain C restatement of gguf-py 0.19.0 (the version pinned by the
 * reference's test/requirements.txt:2), which the reference's tests declare
 * to compute what ggml computes (test/utils/__init__.py:198-228):
 *   Q8_0  quants.py:396-401   w = float(int8 q) * float(f16 d)
 *   Q4_K  quants.py:475-523   w = (float(d) * sc_j) * q - (float(dmin) * m_j)
 *         scale / min unpack  quants.py:478-501 (get_scale_min)
 *   F16 / BF16 / F32          widening conversions
 * Every product and difference is one f32 operation with round-to-nearest
 * (compile without FMA contraction: -ffp-contract=off), as numpy does.
 * Pinned against gguf.dequantize by tests/golden/make_golden.py fixtures.
 */
#include <stdint.h>
#include <string.h>

static float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t exp = (h >> 10) & 0x1F;
    uint32_t mant = h & 0x3FF;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do {
                ++e;
                mant <<= 1;
            } while ((mant & 0x400) == 0);
            mant &= 0x3FF;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float bf16_to_f32(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Q8_0: 34-byte blocks of 32 weights. */
void oracle_dequant_q8_0(const uint8_t* blocks, int64_t nblocks, float* out) {
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t* blk = blocks + b * 34;
        const float d = f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        for (int i = 0; i < 32; ++i) {
            const float q = (float)(int8_t)blk[2 + i];
            out[b * 32 + i] = q * d;
        }
    }
}

/* 6-bit scale / min of sub-block j from the 12 packed bytes. */
static void q4k_scale_min(const uint8_t* s, int j, int* sc, int* m) {
    if (j < 4) {
        *sc = s[j] & 0x3F;
        *m = s[j + 4] & 0x3F;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 2) & 0x30);
        *m = (s[j + 4] >> 4) | ((s[j] >> 2) & 0x30);
    }
}

/* Q4_K: 144-byte super-blocks of 256 weights. */
void oracle_dequant_q4_k(const uint8_t* blocks, int64_t nblocks, float* out) {
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t* blk = blocks + b * 144;
        const float d = f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        const float dmin = f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
        for (int j = 0; j < 8; ++j) {
            int sc, m;
            q4k_scale_min(blk + 4, j, &sc, &m);
            const float ds = d * (float)sc;
            const float dm = dmin * (float)m;
            const uint8_t* qs = blk + 16 + (j / 2) * 32;
            const int shift = (j & 1) * 4;
            for (int l = 0; l < 32; ++l) {
                const float q = (float)((qs[l] >> shift) & 0x0F);
                const float p = ds * q;
                out[b * 256 + j * 32 + l] = p - dm;
            }
        }
    }
}

void oracle_dequant_f16(const uint16_t* in, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = f16_to_f32(in[i]);
}

void oracle_dequant_bf16(const uint16_t* in, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = bf16_to_f32(in[i]);
}

/* Dispatch on the ggml type id; returns 0 on success, -1 on a bad type or
 * a length that is not a whole number of blocks. */
int oracle_dequant(int type, const void* data, int64_t n, float* out) {
    switch (type) {
        case 0: memcpy(out, data, (size_t)n * 4); return 0;
        case 1: oracle_dequant_f16((const uint16_t*)data, n, out); return 0;
        case 30: oracle_dequant_bf16((const uint16_t*)data, n, out); return 0;
        case 8:
            if (n % 32) return -1;
            oracle_dequant_q8_0((const uint8_t*)data, n / 32, out);
            return 0;
        case 12:
            if (n % 256) return -1;
            oracle_dequant_q4_k((const uint8_t*)data, n / 256, out);
            return 0;
        default: return -1;
    }
}
