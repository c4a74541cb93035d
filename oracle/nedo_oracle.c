/*
 * nedo_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference CPU matrix-vector path of nedo.cpp,
 * used as the checker for the CUDA kernels.  Only tests/, the smoke check in
 * __graft_entry__.py and the CPU-baseline leg of bench.py may load it; the
 * product never does.
 *
 * What it restates (file:line in the reference project):
 *   fp16 decode ............ src/kernels.cpp:24-33   (exact IEEE half -> single)
 *   fp16 encode (RNE) ...... src/kernels.cpp:34-36   (F16C _cvtss_sh(f, 0) = round-to-nearest-even)
 *   block sizes ............ src/gguf.cpp:106-114    (Q4_0 18 B / 32, Q8_0 34 B / 32, F16 2 B)
 *   dot_f16 ................ src/kernels.cpp:109-123
 *   dot_q8 ................. src/kernels.cpp:124-138
 *   dot_q4 ................. src/kernels.cpp:139-160
 *   matvec row loop ........ src/kernels.cpp:162-169 (row r = bytes [r*rowbytes, (r+1)*rowbytes))
 *   embedding_row .......... src/kernels.cpp:170-176 (the dequantisation oracle)
 *   argmax (first maximum) . src/model.cpp:36        (std::max_element)
 *
 * The reference has two summation orders, selected at compile time:
 *   NATIVE   (AVX2 + FMA): eight fp32 lane accumulators, lane j sums elements
 *            i+j for i = 0, 8, 16, ... with fused multiply-add, then the eight
 *            lanes are added left to right; the per-block `sum += d*s` is
 *            contracted to an FMA by GCC (-ffp-contract=fast is the GNU default).
 *   PORTABLE (scalar): one accumulator, unfused multiply and add.
 * Both are restated; flavour 0 = native, 1 = portable.  This file must be
 * compiled with -ffp-contract=off so that the only fused operations are the
 * explicit fmaf() calls.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "nedo_oracle.h"

float oracle_fp16_to_fp32(uint16_t h) {
    /* src/kernels.cpp:28-31: exact expansion including subnormals, inf, NaN. */
    uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu, bits;
    if (e == 0) {
        if (m == 0) {
            bits = s;
        } else {
            /* subnormal: normalise the mantissa */
            int ee = 1;
            while ((m & 0x400u) == 0) {
                m <<= 1;
                --ee;
            }
            m &= 0x3ffu;
            bits = s | ((uint32_t)(ee + 112) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = s | 0x7f800000u | (m << 13);
    } else {
        bits = s | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t oracle_fp32_to_fp16_rne(float f) {
    /* Round-to-nearest-even, the rounding of F16C _cvtss_sh(f, 0) (src/kernels.cpp:35-36). */
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf or NaN */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u | ((ax >> 13) & 0x3ffu) : 0u));
    }
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520: overflow to inf */
    if (ax < 0x38800000u) {                                   /* result is subnormal or zero */
        if (ax < 0x33000000u) return (uint16_t)sign;          /* < 2^-25: rounds to zero */
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126u - e; /* 14..24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 112u; /* rebias 127 -> 15 */
    uint32_t m = ax & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q; /* carry into the exponent is correct */
    return (uint16_t)(sign | q);
}

int oracle_row_bytes(uint32_t type, uint64_t cols, uint64_t* out) {
    /* src/gguf.cpp:106-114 */
    switch (type) {
        case ORACLE_F16: *out = cols * 2u; return 0;
        case ORACLE_Q4_0: if (cols % 32u) return ORACLE_E_ALIGN; *out = cols / 32u * 18u; return 0;
        case ORACLE_Q8_0: if (cols % 32u) return ORACLE_E_ALIGN; *out = cols / 32u * 34u; return 0;
        default: return ORACLE_E_TYPE;
    }
}

static uint16_t load_u16(const uint8_t* p) {
    uint16_t v;
    memcpy(&v, p, 2);
    return v;
}

/* src/kernels.cpp:109-123 */
static float dot_f16(const uint8_t* w, const float* x, uint64_t n, int flavour) {
    float s = 0.f;
    uint64_t i = 0;
    if (flavour == ORACLE_NATIVE) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (; i + 8 <= n; i += 8)
            for (int j = 0; j < 8; ++j) acc[j] = fmaf(oracle_fp16_to_fp32(load_u16(w + 2 * (i + j))), x[i + j], acc[j]);
        for (int j = 0; j < 8; ++j) s += acc[j];
        for (; i < n; ++i) s = fmaf(oracle_fp16_to_fp32(load_u16(w + 2 * i)), x[i], s);
        return s;
    }
    for (; i < n; ++i) s += oracle_fp16_to_fp32(load_u16(w + 2 * i)) * x[i];
    return s;
}

/* src/kernels.cpp:124-138 */
static float dot_q8(const uint8_t* p, const float* x, uint64_t n, int flavour) {
    float sum = 0.f;
    uint64_t nb = n / 32u;
    for (uint64_t b = 0; b < nb; ++b, p += 34) {
        float d = oracle_fp16_to_fp32(load_u16(p));
        const int8_t* q = (const int8_t*)(p + 2);
        const float* xb = x + b * 32u;
        float s = 0.f;
        if (flavour == ORACLE_NATIVE) {
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int i = 0; i < 32; i += 8)
                for (int j = 0; j < 8; ++j) acc[j] = fmaf((float)q[i + j], xb[i + j], acc[j]);
            for (int j = 0; j < 8; ++j) s += acc[j];
            sum = fmaf(d, s, sum);
        } else {
            for (int i = 0; i < 32; ++i) s += (float)q[i] * xb[i];
            sum += d * s;
        }
    }
    return sum;
}

/* src/kernels.cpp:139-160.  Element k < 16 is the low nibble of quant byte k,
 * element k >= 16 the high nibble of byte k-16; both are offset by -8. */
static float dot_q4(const uint8_t* p, const float* x, uint64_t n, int flavour) {
    float sum = 0.f;
    uint64_t nb = n / 32u;
    for (uint64_t b = 0; b < nb; ++b, p += 18) {
        float d = oracle_fp16_to_fp32(load_u16(p));
        const uint8_t* q = p + 2;
        const float* xb = x + b * 32u;
        float s = 0.f;
        if (flavour == ORACLE_NATIVE) {
            float v[32];
            for (int i = 0; i < 16; ++i) {
                v[i] = (float)((int)(q[i] & 15) - 8);
                v[i + 16] = (float)((int)(q[i] >> 4) - 8);
            }
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int i = 0; i < 32; i += 8)
                for (int j = 0; j < 8; ++j) acc[j] = fmaf(v[i + j], xb[i + j], acc[j]);
            for (int j = 0; j < 8; ++j) s += acc[j];
            sum = fmaf(d, s, sum);
        } else {
            for (int i = 0; i < 16; ++i) {
                int lo = (q[i] & 15) - 8, hi = (q[i] >> 4) - 8;
                float t = (float)lo * xb[i] + (float)hi * xb[i + 16];
                s += t;
            }
            sum += d * s;
        }
    }
    return sum;
}

int oracle_matvec(int flavour, uint32_t type, uint64_t rows, uint64_t cols, const void* w, const float* x,
                  float* y) {
    uint64_t rb;
    int rc = oracle_row_bytes(type, cols, &rb);
    if (rc) return rc;
    const uint8_t* base = (const uint8_t*)w;
    for (uint64_t r = 0; r < rows; ++r) {
        const uint8_t* p = base + r * rb;
        switch (type) {
            case ORACLE_F16: y[r] = dot_f16(p, x, cols, flavour); break;
            case ORACLE_Q8_0: y[r] = dot_q8(p, x, cols, flavour); break;
            case ORACLE_Q4_0: y[r] = dot_q4(p, x, cols, flavour); break;
            default: return ORACLE_E_TYPE;
        }
    }
    return 0;
}

int oracle_matvec_batch(int flavour, uint32_t type, uint64_t rows, uint64_t cols, uint64_t batch, const void* w,
                        const float* x, float* y) {
    /* `batch` independent matvecs over the same weight: the reference's serial
     * prompt loop (src/model.cpp:262-266).  x is [batch][cols], y is [batch][rows]. */
    for (uint64_t b = 0; b < batch; ++b) {
        int rc = oracle_matvec(flavour, type, rows, cols, w, x + b * cols, y + b * rows);
        if (rc) return rc;
    }
    return 0;
}

int oracle_embedding_row(uint32_t type, uint64_t rows, uint64_t cols, const void* w, uint64_t row, float* out) {
    /* src/kernels.cpp:170-176: one fp32 multiply per element. */
    if (row >= rows) return ORACLE_E_ROW;
    uint64_t rb;
    int rc = oracle_row_bytes(type, cols, &rb);
    if (rc) return rc;
    const uint8_t* p = (const uint8_t*)w + row * rb;
    if (type == ORACLE_F16) {
        for (uint64_t i = 0; i < cols; ++i) out[i] = oracle_fp16_to_fp32(load_u16(p + 2 * i));
    } else if (type == ORACLE_Q8_0) {
        for (uint64_t b = 0; b < cols / 32u; ++b, p += 34) {
            float d = oracle_fp16_to_fp32(load_u16(p));
            const int8_t* q = (const int8_t*)(p + 2);
            for (int i = 0; i < 32; ++i) out[b * 32u + i] = d * (float)q[i];
        }
    } else {
        for (uint64_t b = 0; b < cols / 32u; ++b, p += 18) {
            float d = oracle_fp16_to_fp32(load_u16(p));
            const uint8_t* q = p + 2;
            for (int i = 0; i < 16; ++i) {
                out[b * 32u + i] = d * (float)((int)(q[i] & 15) - 8);
                out[b * 32u + i + 16] = d * (float)((int)(q[i] >> 4) - 8);
            }
        }
    }
    return 0;
}

int oracle_abs_dot(uint32_t type, uint64_t rows, uint64_t cols, const void* w, const float* x, double* out) {
    /* Tolerance scale per output: sum_i |w_i * x_i| with w_i from embedding_row. */
    uint64_t rb;
    int rc = oracle_row_bytes(type, cols, &rb);
    if (rc) return rc;
    const uint8_t* base = (const uint8_t*)w;
    for (uint64_t r = 0; r < rows; ++r) {
        const uint8_t* p = base + r * rb;
        double acc = 0.0;
        if (type == ORACLE_F16) {
            for (uint64_t i = 0; i < cols; ++i) acc += fabs((double)oracle_fp16_to_fp32(load_u16(p + 2 * i)) * x[i]);
        } else if (type == ORACLE_Q8_0) {
            for (uint64_t b = 0; b < cols / 32u; ++b, p += 34) {
                double d = fabs((double)oracle_fp16_to_fp32(load_u16(p)));
                const int8_t* q = (const int8_t*)(p + 2);
                double s = 0.0;
                for (int i = 0; i < 32; ++i) s += fabs((double)q[i] * x[b * 32u + i]);
                acc += d * s;
            }
        } else {
            for (uint64_t b = 0; b < cols / 32u; ++b, p += 18) {
                double d = fabs((double)oracle_fp16_to_fp32(load_u16(p)));
                const uint8_t* q = p + 2;
                double s = 0.0;
                for (int i = 0; i < 16; ++i) {
                    s += fabs((double)((int)(q[i] & 15) - 8) * x[b * 32u + i]);
                    s += fabs((double)((int)(q[i] >> 4) - 8) * x[b * 32u + i + 16]);
                }
                acc += d * s;
            }
        }
        out[r] = acc;
    }
    return 0;
}

int64_t oracle_argmax(const float* v, uint64_t n) {
    /* std::max_element: the first element not less than every other
     * (src/model.cpp:36); NaN inputs are outside the contract. */
    if (n == 0) return -1;
    uint64_t best = 0;
    for (uint64_t i = 1; i < n; ++i)
        if (v[best] < v[i]) best = i;
    return (int64_t)best;
}
