/*
 * oracle_quant.c -- CPU restatement of the reference's quantised weight
 * formats and projection arithmetic (src/kernels.rs, src/model/matmul.rs).
 * TEST INFRASTRUCTURE ONLY: the checker of the GPU dequantisers and linear
 * layer; the product never links it.
 *
 * Block layouts are GGML's (as the reference's BlockQ4K / BlockQ6K /
 * BlockQ8K, src/kernels.rs:10-41): Q4_K 144 bytes per 256 weights, Q6_K 210,
 * Q4_0 18 per 32, Q8_0 34 per 32, F16 2 per weight. Built with
 * -ffp-contract=off so that every f32 expression rounds as Rust's does.
 */
#include "oracle_attn.h"

#include <math.h>
#include <string.h>

#define QK_K 256

/* f16_to_f32: src/kernels.rs:46-70 (exact IEEE half -> single). */
float or_f16_to_f32(uint16_t h) {
    const uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign << 31;
        } else {
            uint32_t e = 0, m = mant;
            while ((m & 0x400u) == 0) {
                m <<= 1;
                ++e;
            }
            bits = (sign << 31) | ((113u - e) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (exp == 31) {
        bits = (sign << 31) | (0xFFu << 23) | (mant == 0 ? 0u : 0x7FFFFFu);
    } else {
        bits = (sign << 31) | ((exp + 127u - 15u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* The 8 six-bit scales and 8 mins of a Q4_K block (the utmp unpacking of
 * src/kernels.rs:194-203). */
static void q4k_scales(const uint8_t* s12, uint8_t sc[8], uint8_t mn[8]) {
    const uint32_t KMASK1 = 0x3f3f3f3fu, KMASK2 = 0x0f0f0f0fu, KMASK3 = 0x03030303u;
    uint32_t utmp[4] = {0, 0, 0, 0};
    memcpy(utmp, s12, 12);
    utmp[3] = ((utmp[2] >> 4) & KMASK2) | (((utmp[1] >> 6) & KMASK3) << 4);
    const uint32_t uaux = utmp[1] & KMASK1;
    utmp[1] = (utmp[2] & KMASK2) | (((utmp[0] >> 6) & KMASK3) << 4);
    utmp[2] = uaux;
    utmp[0] &= KMASK1;
    uint8_t b[16];
    memcpy(b, utmp, 16);
    memcpy(sc, b, 8);
    memcpy(mn, b + 8, 8);
}

/* dequantize_q4k_row: src/kernels.rs:189-217. */
void or_dequant_q4k_row(const uint8_t* blocks, int64_t n_blocks, float* out) {
    for (int64_t i = 0; i < n_blocks; ++i) {
        const uint8_t* b = blocks + i * 144;
        const float d = or_f16_to_f32(rd16(b)), dmin = or_f16_to_f32(rd16(b + 2));
        uint8_t sc[8], mn[8];
        q4k_scales(b + 4, sc, mn);
        const uint8_t* qs = b + 16;
        float* o = out + i * QK_K;
        for (int j = 0; j < QK_K / 64; ++j) {
            /* scales[2j], scales[2j+8] are sc[2j], mn[2j] of the unpacked 16 bytes */
            const float s1 = (float)sc[2 * j], m1 = (float)mn[2 * j];
            const float s2 = (float)sc[2 * j + 1], m2 = (float)mn[2 * j + 1];
            for (int k = 0; k < 32; ++k) {
                const uint8_t q = qs[j * 32 + k];
                o[j * 64 + k] = d * s1 * (float)(q & 0x0F) - dmin * m1;
                o[j * 64 + 32 + k] = d * s2 * (float)((q >> 4) & 0x0F) - dmin * m2;
            }
        }
    }
}

/* The 256 signed 6-bit values of a Q6_K block (src/kernels.rs:134-151). */
static void q6k_values(const uint8_t* b, int8_t aux[QK_K]) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    for (int l = 0; l < 32; ++l) {
        aux[l] = (int8_t)((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
        aux[l + 32] = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
        aux[l + 64] = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
        aux[l + 96] = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
    }
    for (int l = 0; l < 32; ++l) {
        aux[l + 128] = (int8_t)((ql[l + 64] & 0xF) | ((qh[l + 32] & 3) << 4)) - 32;
        aux[l + 160] = (int8_t)((ql[l + 96] & 0xF) | (((qh[l + 32] >> 2) & 3) << 4)) - 32;
        aux[l + 192] = (int8_t)((ql[l + 64] >> 4) | (((qh[l + 32] >> 4) & 3) << 4)) - 32;
        aux[l + 224] = (int8_t)((ql[l + 96] >> 4) | (((qh[l + 32] >> 6) & 3) << 4)) - 32;
    }
}

/* dequantize_q6k_row: src/kernels.rs:128-160. */
void or_dequant_q6k_row(const uint8_t* blocks, int64_t n_blocks, float* out) {
    for (int64_t i = 0; i < n_blocks; ++i) {
        const uint8_t* b = blocks + i * 210;
        const float d = or_f16_to_f32(rd16(b + 208));
        int8_t aux[QK_K];
        q6k_values(b, aux);
        const int8_t* scales = (const int8_t*)(b + 192);
        for (int j = 0; j < QK_K / 16; ++j) {
            const float sc = d * (float)scales[j];
            for (int k = 0; k < 16; ++k) out[i * QK_K + j * 16 + k] = sc * (float)aux[j * 16 + k];
        }
    }
}

/* dequantize_q4_0_row: src/kernels.rs:164-174. */
void or_dequant_q4_0_row(const uint8_t* bytes, int64_t n_blocks, float* out) {
    for (int64_t i = 0; i < n_blocks; ++i) {
        const uint8_t* b = bytes + i * 18;
        const float d = or_f16_to_f32(rd16(b));
        for (int k = 0; k < 16; ++k) {
            const uint8_t q = b[2 + k];
            out[i * 32 + k] = d * ((float)(q & 0x0F) - 8.0f);
            out[i * 32 + k + 16] = d * ((float)(q >> 4) - 8.0f);
        }
    }
}

/* dequantize_q8_0_row: src/kernels.rs:177-185. */
void or_dequant_q8_0_row(const uint8_t* bytes, int64_t n_blocks, float* out) {
    for (int64_t i = 0; i < n_blocks; ++i) {
        const uint8_t* b = bytes + i * 34;
        const float d = or_f16_to_f32(rd16(b));
        for (int k = 0; k < 32; ++k) out[i * 32 + k] = d * (float)(int8_t)b[2 + k];
    }
}

/* One row of `cols` weights of type qtype (GGML ids: 1 F16, 2 Q4_0, 8 Q8_0,
 * 12 Q4_K, 14 Q6_K) to f32. Returns 0, or -1 for an unknown type. */
int or_dequant_row(int32_t qtype, const uint8_t* row, int64_t cols, float* out) {
    switch (qtype) {
        case 1:
            for (int64_t i = 0; i < cols; ++i) out[i] = or_f16_to_f32(rd16(row + 2 * i));
            return 0;
        case 2: or_dequant_q4_0_row(row, cols / 32, out); return 0;
        case 8: or_dequant_q8_0_row(row, cols / 32, out); return 0;
        case 12: or_dequant_q4k_row(row, cols / QK_K, out); return 0;
        case 14: or_dequant_q6k_row(row, cols / QK_K, out); return 0;
        default: return -1;
    }
}

/* Bytes of one row of `cols` weights of type qtype (0 for unknown types). */
int64_t or_row_bytes(int32_t qtype, int64_t cols) {
    switch (qtype) {
        case 1: return 2 * cols;
        case 2: return cols / 32 * 18;
        case 8: return cols / 32 * 34;
        case 12: return cols / QK_K * 144;
        case 14: return cols / QK_K * 210;
        default: return 0;
    }
}

/* BlockQ8K::from_float as the reference uses it, src/kernels.rs:84-125:
 * per 256 values, the value of largest magnitude sets iscale = -128 / max;
 * q = min(round(iscale * x), 127); bsums of 16; d = 1 / iscale. Writes
 * n_blocks (d, qs[256], bsums[16]). */
void or_quantize_row_q8k(const float* x, int64_t n_blocks, float* d, int8_t* qs,
                         int16_t* bsums) {
    for (int64_t i = 0; i < n_blocks; ++i) {
        const float* xs = x + i * QK_K;
        float max = 0.0f, amax = 0.0f;
        for (int j = 0; j < QK_K; ++j)
            if (amax < fabsf(xs[j])) {
                amax = fabsf(xs[j]);
                max = xs[j];
            }
        int8_t* q = qs + i * QK_K;
        if (amax == 0.0f) {
            d[i] = 0.0f;
            memset(q, 0, QK_K);
            memset(bsums + i * 16, 0, 16 * sizeof(int16_t));
            continue;
        }
        const float iscale = -128.0f / max;
        for (int j = 0; j < QK_K; ++j) {
            float v = roundf(iscale * xs[j]);
            if (v > 127.0f) v = 127.0f;
            q[j] = (int8_t)v; /* `as i8` after min(127): v >= -128 by construction */
        }
        for (int j = 0; j < 16; ++j) {
            int32_t s = 0;
            for (int k = 0; k < 16; ++k) s += q[j * 16 + k];
            bsums[i * 16 + j] = (int16_t)s;
        }
        d[i] = 1.0f / iscale;
    }
}

/* Q4_K x Q8_K dot product (candle's scalar vec_dot, as the reference's test
 * copy src/kernels.rs:226-311): integer sums per 8 lanes, scaled per block. */
float or_vec_dot_q4k_q8k(const uint8_t* xb, const float* yd, const int8_t* yq,
                         const int16_t* ybs, int64_t n_blocks) {
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float sumf = 0.0f;
    for (int64_t i = 0; i < n_blocks; ++i) {
        const uint8_t* x = xb + i * 144;
        const int8_t* q8 = yq + i * QK_K;
        int8_t aux8[QK_K];
        for (int j = 0; j < QK_K / 64; ++j)
            for (int l = 0; l < 32; ++l) {
                aux8[j * 64 + l] = (int8_t)(x[16 + j * 32 + l] & 0xF);
                aux8[j * 64 + 32 + l] = (int8_t)(x[16 + j * 32 + l] >> 4);
            }
        uint8_t sc[8], mn[8];
        q4k_scales(x + 4, sc, mn);
        int32_t sumi = 0;
        for (int j = 0; j < 16; ++j) sumi += (int32_t)ybs[i * 16 + j] * (int32_t)mn[j / 2];
        int32_t aux32[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int off = 0;
        for (int s = 0; s < 8; ++s)
            for (int r = 0; r < 4; ++r) {
                for (int l = 0; l < 8; ++l)
                    aux32[l] += (int32_t)sc[s] * (int16_t)(q8[off + l] * aux8[off + l]);
                off += 8;
            }
        const float d = or_f16_to_f32(rd16(x)) * yd[i];
        for (int l = 0; l < 8; ++l) sums[l] += d * (float)aux32[l];
        const float dmin = or_f16_to_f32(rd16(x + 2)) * yd[i];
        sumf -= dmin * (float)sumi;
    }
    float t = 0.0f;
    for (int l = 0; l < 8; ++l) t += sums[l];
    return sumf + t;
}

/* Q6_K x Q8_K dot product (GGML's generic form, as the reference's test copy
 * src/kernels.rs:315-345). */
float or_vec_dot_q6k_q8k(const uint8_t* xb, const float* yd, const int8_t* yq,
                         int64_t n_blocks) {
    float sumf = 0.0f;
    for (int64_t i = 0; i < n_blocks; ++i) {
        const uint8_t* x = xb + i * 210;
        const float d = or_f16_to_f32(rd16(x + 208)) * yd[i];
        int8_t aux8[QK_K];
        q6k_values(x, aux8);
        const int8_t* scales = (const int8_t*)(x + 192);
        int32_t sumi = 0;
        for (int j = 0; j < 16; ++j)
            for (int k = 0; k < 16; ++k)
                sumi += (int32_t)scales[j] * aux8[j * 16 + k] * yq[i * QK_K + j * 16 + k];
        sumf += d * (float)sumi;
    }
    return sumf;
}

/* The reference's projection out[t * rows + r] = act row t . weight row r
 * (MatWeight::forward, src/model/matmul.rs:90-151) for Q4_K / Q6_K weights:
 * activations quantised to Q8_K once per row, then the quantised dot product.
 * Returns 0, or -1 for other weight types. */
int or_linear_q8k(int32_t qtype, const uint8_t* w, int64_t rows, int64_t cols,
                  const float* act, int64_t n, float* out) {
    if ((qtype != 12 && qtype != 14) || cols % QK_K) return -1;
    const int64_t nb = cols / QK_K, rb = or_row_bytes(qtype, cols);
    for (int64_t t = 0; t < n; ++t) {
        float yd[64];
        int8_t yq[64 * QK_K];
        int16_t ybs[64 * 16];
        if (nb > 64) return -1;
        or_quantize_row_q8k(act + t * cols, nb, yd, yq, ybs);
        for (int64_t r = 0; r < rows; ++r)
            out[t * rows + r] = qtype == 12 ? or_vec_dot_q4k_q8k(w + r * rb, yd, yq, ybs, nb)
                                            : or_vec_dot_q6k_q8k(w + r * rb, yd, yq, nb);
    }
    return 0;
}
