/*
 * oracle.c -- CPU restatement of the Qwen3 quantised decode path of
 * uya-lang/minicpm-o-uya.  TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Compiled with -ffp-contract=off so that every a*b+c below is a rounded
 * multiply followed by a rounded add, the same arithmetic the reference's
 * GPU shim requests with --fmad=false (gpu_shim.c:1089-1093).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* conversions                                                         */
/* ------------------------------------------------------------------ */

/* kernels.uya:48-78 / gpu_shim.c:2124-2149: exact f16 -> f32 widening. */
float orc_f16_to_f32(uint16_t bits) {
    uint32_t sign = ((uint32_t) bits & 0x8000u) << 16;
    uint32_t e = ((uint32_t) bits >> 10) & 31u;
    uint32_t m = (uint32_t) bits & 1023u;
    uint32_t out;
    float f;
    if (e == 0) {
        if (m == 0) {
            out = sign;
        } else {
            int ex = -14;
            while ((m & 1024u) == 0) { m <<= 1; ex -= 1; }
            m &= 1023u;
            out = sign | ((uint32_t) (ex + 127) << 23) | (m << 13);
        }
    } else if (e == 31) {
        out = sign | 0x7f800000u | (m << 13);
    } else {
        out = sign | ((e + 112u) << 23) | (m << 13);
    }
    memcpy(&f, &out, 4);
    return f;
}

/* gpu_shim.c:2151-2155 */
float orc_bf16_to_f32(uint16_t bits) {
    uint32_t u = (uint32_t) bits << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* kernels.uya:79-108 / gpu_shim.c:2157-2192.  Truncates the mantissa and adds
 * one unit when the first dropped bit is set (ties round away from zero). */
uint16_t orc_f32_to_f16(float value) {
    uint32_t u, sign, e, frac;
    uint16_t out;
    memcpy(&u, &value, 4);
    sign = (u >> 16) & 0x8000u;
    e = (u >> 23) & 0xffu;
    frac = u & 0x7fffffu;
    if (e == 255u) return (uint16_t) (sign | (frac != 0 ? 0x7e00u : 0x7c00u));
    if (e > 142u) return (uint16_t) (sign | 0x7c00u);
    if (e < 113u) {
        if (e < 103u) return (uint16_t) sign;
        frac |= 0x800000u;
        out = (uint16_t) (sign | (frac >> (126u - e)));
        if ((frac >> (125u - e)) & 1u) out = (uint16_t) (out + 1u);
        return out;
    }
    out = (uint16_t) (sign | ((e - 112u) << 10) | (frac >> 13));
    if (frac & 0x1000u) out = (uint16_t) (out + 1u);
    return out;
}

static uint16_t rd16(const uint8_t *p) { return (uint16_t) (p[0] | (p[1] << 8)); }

static float weight_at(const void *w, int dtype, size_t i) {
    if (dtype == ORC_F32) return ((const float *) w)[i];
    if (dtype == ORC_F16) return orc_f16_to_f32(((const uint16_t *) w)[i]);
    if (dtype == ORC_BF16) return orc_bf16_to_f32(((const uint16_t *) w)[i]);
    return NAN;
}

/* ------------------------------------------------------------------ */
/* block formats                                                       */
/* ------------------------------------------------------------------ */

size_t orc_row_bytes(int dtype, size_t cols) {
    switch (dtype) {
    case ORC_F32: return cols * 4;
    case ORC_F16: case ORC_BF16: return cols * 2;
    case ORC_Q8_0: return cols % 32 ? 0 : cols / 32 * 34;
    case ORC_Q4_K: return cols % 256 ? 0 : cols / 256 * 144;
    case ORC_Q6_K: return cols % 256 ? 0 : cols / 256 * 210;
    default: return 0;
    }
}

/* qwen3.uya:859-867, cpu_kernels.c:305-313: 6-bit scale/min unpacking. */
static void q4k_scale_min(int j, const uint8_t *s, uint8_t *sc, uint8_t *mn) {
    if (j < 4) {
        *sc = s[j] & 63u;
        *mn = s[j + 4] & 63u;
    } else {
        *sc = (uint8_t) ((s[j + 4] & 15u) | ((s[j - 4] >> 6) << 4));
        *mn = (uint8_t) ((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* Q6_K element e of a 256-block as a signed value in [-32, 31]
 * (qwen3.uya:966-1000 index pattern written per element). */
static int q6k_value(const uint8_t *b, int e, int *scale_index) {
    const uint8_t *ql = b, *qh = b + 128;
    int n = e / 128 * 128, r = e - n, quarter = r / 32, l = r % 32;
    int lo, hi;
    if (quarter == 0) { lo = ql[n / 2 + l] & 15; hi = (qh[n / 4 + l] >> 0) & 3; }
    else if (quarter == 1) { lo = ql[n / 2 + l + 32] & 15; hi = (qh[n / 4 + l] >> 2) & 3; }
    else if (quarter == 2) { lo = ql[n / 2 + l] >> 4; hi = (qh[n / 4 + l] >> 4) & 3; }
    else { lo = ql[n / 2 + l + 32] >> 4; hi = (qh[n / 4 + l] >> 6) & 3; }
    if (scale_index) *scale_index = n / 16 + l / 16 + 2 * quarter;
    return (lo | (hi << 4)) - 32;
}

/* Dequantise one row: Q4_K qwen3.uya:1105-1149, Q6_K 1069-1103,
 * Q8_0 / dense qwen3.uya:836-856.  Each value is computed with exactly the
 * reference's operation sequence. */
int orc_dequant_row(int dtype, const uint8_t *row, size_t cols, float *out) {
    size_t i;
    if (orc_row_bytes(dtype, cols) == 0) return 0;
    if (dtype == ORC_F32 || dtype == ORC_F16 || dtype == ORC_BF16) {
        for (i = 0; i < cols; ++i) out[i] = weight_at(row, dtype, i);
        return 1;
    }
    if (dtype == ORC_Q8_0) {
        for (i = 0; i < cols / 32; ++i) {
            const uint8_t *b = row + i * 34;
            float d = orc_f16_to_f32(rd16(b));
            int l;
            for (l = 0; l < 32; ++l) out[i * 32 + l] = d * (float) (int8_t) b[2 + l];
        }
        return 1;
    }
    if (dtype == ORC_Q4_K) {
        for (i = 0; i < cols / 256; ++i) {
            const uint8_t *b = row + i * 144;
            float d = orc_f16_to_f32(rd16(b)), dmin = orc_f16_to_f32(rd16(b + 2));
            const uint8_t *sc = b + 4, *qs = b + 16;
            int g, l;
            for (g = 0; g < 4; ++g) {
                uint8_t s0, m0, s1, m1;
                float d1, mm1, d2, mm2;
                q4k_scale_min(2 * g, sc, &s0, &m0);
                q4k_scale_min(2 * g + 1, sc, &s1, &m1);
                d1 = d * (float) s0; mm1 = dmin * (float) m0;
                d2 = d * (float) s1; mm2 = dmin * (float) m1;
                for (l = 0; l < 32; ++l) out[i * 256 + g * 64 + l] = d1 * (float) (qs[g * 32 + l] & 15) - mm1;
                for (l = 0; l < 32; ++l) out[i * 256 + g * 64 + 32 + l] = d2 * (float) (qs[g * 32 + l] >> 4) - mm2;
            }
        }
        return 1;
    }
    if (dtype == ORC_Q6_K) {
        for (i = 0; i < cols / 256; ++i) {
            const uint8_t *b = row + i * 210;
            const int8_t *sc = (const int8_t *) (b + 192);
            float d = orc_f16_to_f32(rd16(b + 208));
            int e;
            for (e = 0; e < 256; ++e) {
                int si, q = q6k_value(b, e, &si);
                out[i * 256 + e] = d * (float) sc[si] * (float) q;
            }
        }
        return 1;
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* Q8_1 activations                                                    */
/* ------------------------------------------------------------------ */

/* gpu_shim.c:336-378: per 32 values, sequential amax and sum, d = amax/127,
 * q = trunc(x/d +- 0.5) clamped to [-128, 127]; d and s stored as f16. */
int orc_q8_1_quantize(const float *x, size_t n, uint8_t *dst) {
    size_t b;
    if (x == NULL || dst == NULL || n == 0 || n % 32) return 0;
    for (b = 0; b < n / 32; ++b) {
        const float *xb = x + b * 32;
        uint8_t *o = dst + b * 36;
        float amax = 0.0f, sum = 0.0f;
        int i;
        for (i = 0; i < 32; ++i) {
            float ax = xb[i] < 0.0f ? -xb[i] : xb[i];
            if (ax > amax) amax = ax;
            sum += xb[i];
        }
        if (amax == 0.0f) {
            memset(o, 0, 36);
            continue;
        }
        {
            float d = amax / 127.0f;
            uint16_t db = orc_f32_to_f16(d), sb = orc_f32_to_f16(sum);
            o[0] = (uint8_t) db; o[1] = (uint8_t) (db >> 8);
            o[2] = (uint8_t) sb; o[3] = (uint8_t) (sb >> 8);
            for (i = 0; i < 32; ++i) {
                float v = xb[i] / d;
                int q = (int) (v >= 0.0f ? v + 0.5f : v - 0.5f);
                if (q > 127) q = 127;
                if (q < -128) q = -128;
                o[4 + i] = (uint8_t) (int8_t) q;
            }
        }
    }
    return 1;
}

int orc_q8_1_block_sums(const uint8_t *xq, size_t nblocks, int32_t *sums) {
    size_t b;
    for (b = 0; b < nblocks; ++b) {
        int32_t s = 0;
        int i;
        for (i = 0; i < 32; ++i) s += (int8_t) xq[b * 36 + 4 + i];
        sums[b] = s;
    }
    return 1;
}

static float q8_1_d(const uint8_t *xq, size_t block) { return orc_f16_to_f32(rd16(xq + block * 36)); }
static int8_t q8_1_q(const uint8_t *xq, size_t block, int i) { return (int8_t) xq[block * 36 + 4 + i]; }

int orc_q4_k_block_dots(const uint8_t *row, const uint8_t *xq, size_t cols, int32_t *dot_d, int32_t *dot_m) {
    size_t sb;
    if (cols % 256) return 0;
    for (sb = 0; sb < cols / 256; ++sb) {
        const uint8_t *qs = row + sb * 144 + 16;
        int j, l;
        for (j = 0; j < 8; ++j) {
            size_t blk = sb * 8 + j;
            int32_t d = 0, m = 0;
            for (l = 0; l < 32; ++l) {
                int q4 = (j & 1) ? (qs[(j / 2) * 32 + l] >> 4) : (qs[(j / 2) * 32 + l] & 15);
                int q8 = q8_1_q(xq, blk, l);
                d += q4 * q8;
                m += q8;
            }
            dot_d[blk] = d;
            dot_m[blk] = m;
        }
    }
    return 1;
}

int orc_q6_k_block_dots(const uint8_t *row, const uint8_t *xq, size_t cols, int32_t *dots) {
    size_t sb;
    if (cols % 256) return 0;
    for (sb = 0; sb < cols / 256; ++sb) {
        const uint8_t *b = row + sb * 210;
        int g, l;
        for (g = 0; g < 16; ++g) {
            int32_t acc = 0;
            for (l = 0; l < 16; ++l) {
                int e = g * 16 + l;
                acc += q6k_value(b, e, NULL) * q8_1_q(xq, sb * 8 + e / 32, e % 32);
            }
            dots[sb * 16 + g] = acc;
        }
    }
    return 1;
}

int orc_q8_0_block_dots(const uint8_t *row, const uint8_t *xq, size_t cols, int32_t *dots) {
    size_t b;
    if (cols % 32) return 0;
    for (b = 0; b < cols / 32; ++b) {
        int32_t acc = 0;
        int l;
        for (l = 0; l < 32; ++l) acc += (int8_t) row[b * 34 + 2 + l] * q8_1_q(xq, b, l);
        dots[b] = acc;
    }
    return 1;
}

/* Q6_K scale group g -> element e of its first value: e = g*16; the scale
 * index for that element (q6k_value) is the group's scale byte. */
static int q6k_group_scale(const uint8_t *b, int g) {
    int si;
    (void) q6k_value(b, g * 16, &si);
    return ((const int8_t *) (b + 192))[si];
}

/* Row dot with Q8_1 activations, the per-block formulas of
 * gpu_shim.c:746-808 (Q4_K: d*sum(d8*sc*dot) - dmin*sum(d8*m*sum q8)),
 * gpu_shim.c:856-878 (Q6_K: d*sum(d8*(dot*sc))) and d_w*d8*dot for Q8_0,
 * accumulated in natural block order. */
static float row_dot_q8_1(int dtype, const uint8_t *row, size_t cols, const uint8_t *xq) {
    float acc = 0.0f;
    size_t sb;
    if (dtype == ORC_Q4_K) {
        for (sb = 0; sb < cols / 256; ++sb) {
            const uint8_t *b = row + sb * 144;
            float d = orc_f16_to_f32(rd16(b)), dmin = orc_f16_to_f32(rd16(b + 2));
            float sum_d = 0.0f, sum_m = 0.0f;
            int j, l;
            for (j = 0; j < 8; ++j) {
                uint8_t sc, mn;
                int32_t dd = 0, mm = 0;
                float d8 = q8_1_d(xq, sb * 8 + j);
                q4k_scale_min(j, b + 4, &sc, &mn);
                for (l = 0; l < 32; ++l) {
                    int q4 = (j & 1) ? (b[16 + (j / 2) * 32 + l] >> 4) : (b[16 + (j / 2) * 32 + l] & 15);
                    int q8 = q8_1_q(xq, sb * 8 + j, l);
                    dd += q4 * q8;
                    mm += q8;
                }
                sum_d += d8 * (float) dd * (float) sc;
                sum_m += d8 * (float) mm * (float) mn;
            }
            acc += d * sum_d - dmin * sum_m;
        }
        return acc;
    }
    if (dtype == ORC_Q6_K) {
        for (sb = 0; sb < cols / 256; ++sb) {
            const uint8_t *b = row + sb * 210;
            float d = orc_f16_to_f32(rd16(b + 208)), sum = 0.0f;
            int g, l;
            for (g = 0; g < 16; ++g) {
                int32_t dd = 0;
                float d8 = q8_1_d(xq, sb * 8 + g / 2);
                for (l = 0; l < 16; ++l) {
                    int e = g * 16 + l;
                    dd += q6k_value(b, e, NULL) * q8_1_q(xq, sb * 8 + e / 32, e % 32);
                }
                sum += d8 * ((float) dd * (float) q6k_group_scale(b, g));
            }
            acc += d * sum;
        }
        return acc;
    }
    if (dtype == ORC_Q8_0) {
        size_t blk;
        for (blk = 0; blk < cols / 32; ++blk) {
            const uint8_t *b = row + blk * 34;
            int32_t dd = 0;
            int l;
            for (l = 0; l < 32; ++l) dd += (int8_t) b[2 + l] * q8_1_q(xq, blk, l);
            acc += orc_f16_to_f32(rd16(b)) * q8_1_d(xq, blk) * (float) dd;
        }
        return acc;
    }
    return NAN;
}

int orc_matvec_q8_1(int dtype, const uint8_t *w, size_t rows, size_t cols, const uint8_t *xq, float *y) {
    size_t rb = orc_row_bytes(dtype, cols), r;
    if (rb == 0 || (dtype != ORC_Q4_K && dtype != ORC_Q6_K && dtype != ORC_Q8_0)) return 0;
    if (dtype == ORC_Q8_0 && cols % 256) return 0; /* the device path works on 256-value groups */
    for (r = 0; r < rows; ++r) y[r] = row_dot_q8_1(dtype, w + r * rb, cols, xq);
    return 1;
}

/* f32-activation row dots: Q8_0 cpu_kernels.c:315-330 (x*d*q), Q4_K
 * cpu_kernels.c:332-365 (x*(d1*q-m1)), Q6_K cpu_kernels.c:367-395
 * (x*d*sc*q), dense qwen3.uya:1200-1245 (w*x). */
int orc_matvec_f32(int dtype, const uint8_t *w, size_t rows, size_t cols, const float *x, float *y) {
    size_t rb = orc_row_bytes(dtype, cols), r, i;
    float *tmp;
    if (rb == 0) return 0;
    tmp = (float *) malloc(cols * sizeof(float));
    if (!tmp) return 0;
    for (r = 0; r < rows; ++r) {
        float acc = 0.0f;
        const uint8_t *row = w + r * rb;
        if (dtype == ORC_Q8_0) {
            for (i = 0; i < cols / 32; ++i) {
                float d = orc_f16_to_f32(rd16(row + i * 34));
                int l;
                for (l = 0; l < 32; ++l) acc += x[i * 32 + l] * d * (float) (int8_t) row[i * 34 + 2 + l];
            }
        } else if (dtype == ORC_Q6_K) {
            for (i = 0; i < cols / 256; ++i) {
                const uint8_t *b = row + i * 210;
                float d = orc_f16_to_f32(rd16(b + 208));
                int e;
                /* element order of cpu_kernels.c:379-391: l-major across the 4 quarters */
                int n, l, qq;
                for (n = 0; n < 256; n += 128)
                    for (l = 0; l < 32; ++l)
                        for (qq = 0; qq < 4; ++qq) {
                            int si, q;
                            e = n + qq * 32 + l;
                            q = q6k_value(b, e, &si);
                            acc += x[i * 256 + e] * d * (float) ((const int8_t *) (b + 192))[si] * (float) q;
                        }
            }
        } else if (dtype == ORC_Q4_K) {
            (void) orc_dequant_row(dtype, row, cols, tmp);
            for (i = 0; i < cols; ++i) acc += x[i] * tmp[i];
        } else {
            for (i = 0; i < cols; ++i) acc += weight_at(row, dtype, i) * x[i];
        }
        y[r] = acc;
    }
    free(tmp);
    return 1;
}

/* ------------------------------------------------------------------ */
/* norms, rope, attention, sampler                                      */
/* ------------------------------------------------------------------ */

/* The reduction of gpu_shim.c:694-718 with blockDim 256: lane t sums
 * v[t], v[t+256], ... in order, then a halving tree (stride 128 .. 1). */
static float tree_sum_sq(const float *x, size_t n) {
    float part[256];
    size_t t, i;
    int stride;
    for (t = 0; t < 256; ++t) {
        float s = 0.0f;
        for (i = t; i < n; i += 256) s += x[i] * x[i];
        part[t] = s;
    }
    for (stride = 128; stride > 0; stride >>= 1)
        for (t = 0; t < (size_t) stride; ++t) part[t] += part[t + stride];
    return part[0];
}

int orc_rms_norm(const float *x, const void *w, int w_dtype, size_t n, float eps, int order, float *out) {
    float sum = 0.0f, inv;
    size_t i;
    if (n == 0) return 0;
    if (order == 0) {
        for (i = 0; i < n; ++i) sum += x[i] * x[i];
    } else {
        sum = tree_sum_sq(x, n);
    }
    inv = 1.0f / sqrtf(sum / (float) n + eps);
    for (i = 0; i < n; ++i) out[i] = x[i] * inv * weight_at(w, w_dtype, i);
    return 1;
}

int orc_head_norm(float *vec, const void *w, int w_dtype, size_t head_count, size_t head_dim, int order) {
    size_t h;
    float *tmp = (float *) malloc(head_dim * sizeof(float));
    if (!tmp) return 0;
    for (h = 0; h < head_count; ++h) {
        (void) orc_rms_norm(vec + h * head_dim, w, w_dtype, head_dim, 1e-6f, order, tmp);
        memcpy(vec + h * head_dim, tmp, head_dim * sizeof(float));
    }
    free(tmp);
    return 1;
}

int orc_rope_table(size_t context, size_t head_dim, float freq_base, float freq_scale, float *cos_out, float *sin_out) {
    size_t half = head_dim / 2, pos, d;
    if (half == 0) return 0;
    for (pos = 0; pos < context; ++pos)
        for (d = 0; d < half; ++d) {
            float theta = ((float) pos * freq_scale) / powf(freq_base, (float) (2 * d) / (float) head_dim);
            cos_out[pos * half + d] = cosf(theta);
            sin_out[pos * half + d] = sinf(theta);
        }
    return 1;
}

int orc_rope_apply(float *vec, size_t head_count, size_t head_dim, size_t pos, const float *cos_t, const float *sin_t) {
    size_t half = head_dim / 2, h, d;
    for (h = 0; h < head_count; ++h)
        for (d = 0; d < half; ++d) {
            float c = cos_t[pos * half + d], s = sin_t[pos * half + d];
            float x0 = vec[h * head_dim + d], x1 = vec[h * head_dim + half + d];
            vec[h * head_dim + d] = x0 * c - x1 * s;
            vec[h * head_dim + half + d] = x1 * c + x0 * s;
        }
    return 1;
}

static void softmax_ref(float *dst, const float *src, size_t n) {
    float maxv = src[0], sum = 0.0f;
    size_t i;
    for (i = 1; i < n; ++i) if (src[i] > maxv) maxv = src[i];
    for (i = 0; i < n; ++i) { float e = expf(src[i] - maxv); dst[i] = e; sum += e; }
    if (sum == 0.0f) return;
    for (i = 0; i < n; ++i) dst[i] = dst[i] / sum;
}

int orc_attention(float *out, const float *q, const float *k_cache, const float *v_cache, size_t layer, size_t pos,
                  size_t head_count, size_t kv_head_count, size_t head_dim, size_t context) {
    size_t kv_dim = kv_head_count * head_dim, h, t, d;
    float scale = 1.0f / sqrtf((float) head_dim);
    float *scores = (float *) malloc((pos + 1) * sizeof(float));
    float *probs = (float *) malloc((pos + 1) * sizeof(float));
    if (!scores || !probs) { free(scores); free(probs); return 0; }
    for (h = 0; h < head_count; ++h) {
        size_t kvh = (h * kv_head_count) / head_count;
        for (t = 0; t <= pos; ++t) {
            const float *krow = k_cache + (layer * context + t) * kv_dim + kvh * head_dim;
            float dot = 0.0f;
            for (d = 0; d < head_dim; ++d) dot += q[h * head_dim + d] * krow[d];
            scores[t] = dot * scale;
        }
        softmax_ref(probs, scores, pos + 1);
        for (d = 0; d < head_dim; ++d) {
            float sum = 0.0f;
            for (t = 0; t <= pos; ++t) sum += probs[t] * v_cache[(layer * context + t) * kv_dim + kvh * head_dim + d];
            out[h * head_dim + d] = sum;
        }
    }
    free(scores);
    free(probs);
    return 1;
}

void orc_silu_mul(float *dst, const float *gate, const float *up, size_t n) {
    size_t i;
    for (i = 0; i < n; ++i) dst[i] = (gate[i] / (1.0f + expf(0.0f - gate[i]))) * up[i];
}

static int seen_token(const uint32_t *seen, size_t n, uint32_t tok) {
    size_t i;
    for (i = 0; i < n; ++i) if (seen[i] == tok) return 1;
    return 0;
}

uint32_t orc_argmax_penalized(const float *values, size_t n, const uint32_t *seen, size_t seen_count, float penalty,
                              float *top2_gap) {
    size_t best = 0, i;
    float best_v, second = -INFINITY;
    if (n == 0) { if (top2_gap) *top2_gap = INFINITY; return 0; }
    best_v = values[0];
    if (penalty > 1.0f && seen_token(seen, seen_count, 0)) {
        if (best_v > 0.0f) best_v = best_v / penalty;
        if (best_v < 0.0f) best_v = best_v * penalty;
    }
    for (i = 1; i < n; ++i) {
        float v = values[i];
        if (penalty > 1.0f && seen_token(seen, seen_count, (uint32_t) i)) {
            if (v > 0.0f) v = v / penalty;
            if (v < 0.0f) v = v * penalty;
        }
        if (v > best_v) { second = best_v; best = i; best_v = v; }
        else if (v > second) second = v;
    }
    if (top2_gap) *top2_gap = n > 1 ? best_v - second : INFINITY;
    return (uint32_t) best;
}


/* qwen3.uya:2046-2057: xorshift32, and its unit draw value / 4294967295 */
static uint32_t xorshift32(uint32_t *state) {
    uint32_t x = *state;
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    *state = x;
    return x;
}

/* qwen3_sample (qwen3.uya:2073-2138): greedy (argmax with the penalty once
 * per seen token) unless temperature > 1e-6, top_k > 1 and vocab <= 256;
 * then the penalty per seen-list entry, logits / temperature, softmax
 * (kernels.uya:149-160), the reference's swap selection sort (descending,
 * not stable), top-k, top-p, min-p, renormalisation and one xorshift32
 * draw.  *margin (may be NULL): the smallest |r - running sum| met while
 * choosing (0 on the greedy path), so callers can tell draws that sit on a
 * cumulative boundary. */
uint32_t orc_sample(const float *logits, size_t vocab, const uint32_t *seen, size_t seen_count, float temp,
                    uint32_t top_k, float top_p, float min_p, float penalty, uint32_t *seed, float *margin) {
    float local[256], probs[256], maxv, sum, cumulative, max_prob, norm, r, acc, mg = INFINITY;
    uint32_t order[256];
    size_t i, a, b, limit, kept;
    if (margin) *margin = 0.0f;
    if (temp <= 0.000001f || top_k <= 1 || vocab > 256 || vocab == 0)
        return orc_argmax_penalized(logits, vocab, seen, seen_count, penalty, NULL);
    for (i = 0; i < vocab; ++i) { local[i] = logits[i]; order[i] = (uint32_t) i; }
    if (penalty > 1.0f)
        for (i = 0; i < seen_count; ++i) {
            size_t t = seen[i];
            if (t < vocab) {
                if (local[t] > 0.0f) local[t] = local[t] / penalty;
                if (local[t] < 0.0f) local[t] = local[t] * penalty;
            }
        }
    for (i = 0; i < vocab; ++i) local[i] = local[i] / temp;
    maxv = local[0];
    for (i = 1; i < vocab; ++i) if (local[i] > maxv) maxv = local[i];
    sum = 0.0f;
    for (i = 0; i < vocab; ++i) { probs[i] = expf(local[i] - maxv); sum = sum + probs[i]; }
    if (sum != 0.0f) for (i = 0; i < vocab; ++i) probs[i] = probs[i] / sum;
    for (a = 0; a < vocab; ++a)
        for (b = a + 1; b < vocab; ++b)
            if (probs[b] > probs[a]) {
                float tp = probs[a]; uint32_t ti = order[a];
                probs[a] = probs[b]; probs[b] = tp;
                order[a] = order[b]; order[b] = ti;
            }
    limit = vocab;
    if (top_k > 0 && top_k < limit) limit = top_k;
    cumulative = 0.0f;
    kept = 0;
    while (kept < limit) {
        if (kept >= vocab || kept >= 256) break;
        cumulative = cumulative + probs[kept];
        kept = kept + 1;
        if (cumulative >= top_p && top_p < 0.999999f) break;
    }
    max_prob = probs[0];
    if (min_p > 0.0f)
        while (kept > 1) {
            size_t tail = kept - 1;
            if (tail >= 256 || probs[tail] >= max_prob * min_p) break;
            kept = kept - 1;
        }
    norm = 0.0f;
    for (i = 0; i < kept; ++i) norm = norm + probs[i];
    r = (float) xorshift32(seed) / 4294967295.0f;
    acc = 0.0f;
    for (i = 0; i < kept; ++i) {
        acc = acc + probs[i] / norm;
        if (fabsf(r - acc) < mg) mg = fabsf(r - acc);
        if (r <= acc || i + 1 == kept) {
            if (margin) *margin = mg;
            return order[i];
        }
    }
    if (margin) *margin = mg;
    return order[0];
}

/* ------------------------------------------------------------------ */
/* device evaluation order (bit-exact contract with the B200 kernels)  */
/* ------------------------------------------------------------------ */

/* Cody-Waite reduction + degree-7 Taylor polynomial (Horner, fmaf), exact
 * scaling by 2^k; every step correctly rounded, so the CUDA build of the
 * same steps returns the same bits. */
float orc_expf_det(float x) {
    float k, r, p, sc;
    int ki;
    uint32_t bits;
    if (x != x) return x;
    if (x >= 88.72283935546875f) return INFINITY;
    if (x <= -103.97208404541015625f) return 0.0f;
    k = rintf(x * 1.44269502162933349609375f);
    r = fmaf(-k, 0.693145751953125f, x);
    r = fmaf(-k, 1.428606765330187045e-06f, r);
    p = 1.98412698412698e-4f;
    p = fmaf(p, r, 1.38888888888889e-3f);
    p = fmaf(p, r, 8.33333333333333e-3f);
    p = fmaf(p, r, 4.16666666666667e-2f);
    p = fmaf(p, r, 1.66666666666667e-1f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    ki = (int) k;
    if (ki > 127) { p = p * 2.0f; ki = 127; }
    if (ki < -126) { p = p * 5.42101086242752217e-20f; ki += 64; }
    bits = (uint32_t) (ki + 127) << 23;
    memcpy(&sc, &bits, 4);
    return p * sc;
}

int orc_attn_n_split(int n_kv) {
    int s = (256 + n_kv - 1) / n_kv;
    return s < 1 ? 1 : (s > 16 ? 16 : s);
}

uint16_t orc_f32_to_f16_rne(float v) {
    uint32_t u, sign, e, m, out, rem, half;
    int ex;
    memcpy(&u, &v, 4);
    sign = (u >> 16) & 0x8000u;
    e = (u >> 23) & 0xffu;
    m = u & 0x7fffffu;
    if (e == 255u) return (uint16_t) (sign | 0x7c00u | (m ? 0x200u : 0u));
    ex = (int) e - 127 + 15;
    if (ex >= 31) return (uint16_t) (sign | 0x7c00u);
    if (ex <= 0) {
        int shift;
        if (ex < -10) return (uint16_t) sign;
        m |= 0x800000u;
        shift = 14 - ex;
        out = m >> shift;
        rem = m & ((1u << shift) - 1u);
        half = 1u << (shift - 1);
        if (rem > half || (rem == half && (out & 1u))) out += 1u;
        return (uint16_t) (sign | out);
    }
    out = ((uint32_t) ex << 10) | (m >> 13);
    rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (out & 1u))) out += 1u;
    return (uint16_t) (sign | out);
}

static int lanes_per_row(size_t cols) {
    size_t nb = cols / 256;
    int lpr = 32;
    while (lpr > 1 && (nb % (size_t) lpr) != 0) lpr >>= 1;
    return lpr;
}

static float butterfly(float *v, int n) {
    float nv[32];
    int o, i;
    for (o = n >> 1; o > 0; o >>= 1) {
        for (i = 0; i < n; ++i) nv[i] = v[i] + v[i ^ o];
        for (i = 0; i < n; ++i) v[i] = nv[i];
    }
    return v[0];
}

/* one super-block (256 values) in the kernel's operation order:
 *  Q4_K: sum_d = fma(d8_j, float(sc_j*dot_j), sum_d), sum_m = fma(d8_j*sumq_j,
 *        float(m_j), sum_m) over j = 0..7; value = fma(d, sum_d, -(dmin*sum_m))
 *  Q6_K: per Q8_1 block b (groups 2b, 2b+1): sum = fma(d8_b,
 *        float(sc_2b*dot_2b + sc_2b+1*dot_2b+1), sum); value = d*sum
 *  Q8_0: sum = fma(d_w*d8_b, float(dot_b), sum) over b */
static float sb_dev(int dtype, const uint8_t *row, size_t sb, const uint8_t *xq) {
    float xd[8], xds[8];
    int j;
    for (j = 0; j < 8; ++j) {
        int i;
        int32_t s = 0;
        for (i = 0; i < 32; ++i) s += q8_1_q(xq, sb * 8 + j, i);
        xd[j] = q8_1_d(xq, sb * 8 + j);
        xds[j] = xd[j] * (float) s;
    }
    if (dtype == ORC_Q4_K) {
        const uint8_t *b = row + sb * 144;
        float d = orc_f16_to_f32(rd16(b)), dmin = orc_f16_to_f32(rd16(b + 2));
        float sum_d = 0.0f, sum_m = 0.0f;
        int g;
        for (g = 0; g < 4; ++g) {
            uint8_t s0, m0, s1, m1;
            int32_t dlo = 0, dhi = 0;
            int l;
            q4k_scale_min(2 * g, b + 4, &s0, &m0);
            q4k_scale_min(2 * g + 1, b + 4, &s1, &m1);
            for (l = 0; l < 32; ++l) {
                dlo += (b[16 + g * 32 + l] & 15) * q8_1_q(xq, sb * 8 + 2 * g, l);
                dhi += (b[16 + g * 32 + l] >> 4) * q8_1_q(xq, sb * 8 + 2 * g + 1, l);
            }
            sum_d = fmaf(xd[2 * g], (float) ((int32_t) s0 * dlo), sum_d);
            sum_d = fmaf(xd[2 * g + 1], (float) ((int32_t) s1 * dhi), sum_d);
            sum_m = fmaf(xds[2 * g], (float) m0, sum_m);
            sum_m = fmaf(xds[2 * g + 1], (float) m1, sum_m);
        }
        return fmaf(d, sum_d, -(dmin * sum_m));
    }
    if (dtype == ORC_Q6_K) {
        const uint8_t *b = row + sb * 210;
        float d = orc_f16_to_f32(rd16(b + 208)), sum = 0.0f;
        int blk;
        for (blk = 0; blk < 8; ++blk) {
            int32_t dd[2], h;
            for (h = 0; h < 2; ++h) {
                int g = 2 * blk + h, l;
                int32_t acc = 0;
                for (l = 0; l < 16; ++l) {
                    int e = g * 16 + l;
                    acc += q6k_value(b, e, NULL) * q8_1_q(xq, sb * 8 + e / 32, e % 32);
                }
                dd[h] = acc;
            }
            sum = fmaf(xd[blk], (float) (q6k_group_scale(b, 2 * blk) * dd[0] + q6k_group_scale(b, 2 * blk + 1) * dd[1]),
                       sum);
        }
        return d * sum;
    }
    {
        float sum = 0.0f;
        int blk;
        for (blk = 0; blk < 8; ++blk) {
            const uint8_t *b = row + (sb * 8 + blk) * 34;
            int32_t dd = 0;
            int l;
            for (l = 0; l < 32; ++l) dd += (int8_t) b[2 + l] * q8_1_q(xq, sb * 8 + blk, l);
            sum = fmaf(orc_f16_to_f32(rd16(b)) * xd[blk], (float) dd, sum);
        }
        return sum;
    }
}

int orc_matvec_q8_1_dev(int dtype, const uint8_t *w, size_t rows, size_t cols, const uint8_t *xq, float *y) {
    size_t rb = orc_row_bytes(dtype, cols), r;
    int lpr, li;
    size_t nb, ks, k;
    if (rb == 0 || cols % 256 || (dtype != ORC_Q4_K && dtype != ORC_Q6_K && dtype != ORC_Q8_0)) return 0;
    lpr = lanes_per_row(cols);
    nb = cols / 256;
    ks = nb / (size_t) lpr;
    for (r = 0; r < rows; ++r) {
        float v[32];
        for (li = 0; li < lpr; ++li) {
            float acc = 0.0f;
            for (k = 0; k < ks; ++k) acc = acc + sb_dev(dtype, w + r * rb, k * (size_t) lpr + (size_t) li, xq);
            v[li] = acc;
        }
        y[r] = butterfly(v, lpr);
    }
    return 1;
}

/* warp per row, lane l sums w[i]*x[i] for i = l, l+32, ... with fmaf, then
 * the 32-lane butterfly. */
int orc_matvec_dense_dev(int dtype, const uint8_t *w, size_t rows, size_t cols, const float *x, float *y) {
    size_t rb = orc_row_bytes(dtype, cols), r, i;
    if (rb == 0 || (dtype != ORC_F32 && dtype != ORC_F16 && dtype != ORC_BF16)) return 0;
    for (r = 0; r < rows; ++r) {
        float v[32];
        int l;
        for (l = 0; l < 32; ++l) {
            float acc = 0.0f;
            for (i = (size_t) l; i < cols; i += 32) acc = fmaf(weight_at(w + r * rb, dtype, i), x[i], acc);
            v[l] = acc;
        }
        y[r] = butterfly(v, 32);
    }
    return 1;
}

void orc_silu_mul_dev(float *dst, const float *gate, const float *up, size_t n) {
    size_t i;
    for (i = 0; i < n; ++i) dst[i] = (gate[i] / (1.0f + orc_expf_det(-gate[i]))) * up[i];
}

/* Flash-decode order of the attention kernel: per q head, per KV chunk of
 * max(32, ceil((pos+1)/splits)) positions, sub-chunks of 32 positions: scores
 * by sequential fma over d; m' = max(m, max s); alpha = exp(m - m'); p_t =
 * exp(s_t - m'); l = l*alpha + butterfly(p); acc_d = acc_d*alpha then fma(p_t,
 * v_td, acc_d) in t order.  Chunks merged as (sum_s w_s acc_s) * (1 / sum_s
 * w_s l_s), w_s = exp(m_s - max m), fma in split order. */
int orc_attention_dev(float *out, const float *q, const float *k_cache, const float *v_cache, const float *cur_k,
                      const float *cur_v, size_t layer, size_t pos, size_t head_count, size_t kv_head_count,
                      size_t head_dim, size_t context) {
    const size_t hd = head_dim, kv_dim = kv_head_count * hd;
    const float scale = 1.0f / sqrtf((float) hd);
    const size_t n_pos = pos + 1;
    /* blocks of 32 positions, each a partial (m, l, acc) of its own, merged
     * in block order */
    const size_t chunk = 32;
    size_t n_active, kvh;
    float *pm, *pl, *pacc, *acc;
    if (!(hd == 64 || hd == 128 || hd == 256 || hd <= 32)) return 0;
    n_active = (n_pos + chunk - 1) / chunk;
    pm = (float *) malloc(n_active * sizeof(float));
    pl = (float *) malloc(2 * n_active * sizeof(float)); /* l, then the merge weights */
    pacc = (float *) malloc(n_active * hd * sizeof(float));
    acc = (float *) malloc(hd * sizeof(float));
    if (!pm || !pl || !pacc || !acc) { free(pm); free(pl); free(pacc); free(acc); return 0; }
    for (kvh = 0; kvh < kv_head_count; ++kvh) {
        size_t hb = (kvh * head_count + kv_head_count - 1) / kv_head_count;
        size_t he = ((kvh + 1) * head_count + kv_head_count - 1) / kv_head_count, h;
        for (h = hb; h < he; ++h) {
            const float *qh = q + h * hd;
            size_t s, d;
            for (s = 0; s < n_active; ++s) {
                const size_t t0 = s * chunk, t1 = t0 + chunk < n_pos ? t0 + chunk : n_pos;
                float m = -INFINITY, l = 0.0f;
                size_t c0;
                for (d = 0; d < hd; ++d) acc[d] = 0.0f;
                for (c0 = t0; c0 < t1; c0 += 32) {
                    float sc[32], p[32], tmp[32], mx = -INFINITY, mn, alpha, psum;
                    const float *vrow[32];
                    int ln;
                    for (ln = 0; ln < 32; ++ln) {
                        const size_t t = c0 + (size_t) ln;
                        vrow[ln] = NULL;
                        if (t < t1) {
                            const int cur = t == pos;
                            const float *krow = cur ? cur_k + kvh * hd : k_cache + (layer * context + t) * kv_dim + kvh * hd;
                            float dot = 0.0f;
                            vrow[ln] = cur ? cur_v + kvh * hd : v_cache + (layer * context + t) * kv_dim + kvh * hd;
                            for (d = 0; d < hd; ++d) dot = fmaf(qh[d], krow[d], dot);
                            sc[ln] = dot * scale;
                        } else {
                            sc[ln] = -INFINITY;
                        }
                        mx = fmaxf(mx, sc[ln]);
                    }
                    mn = fmaxf(m, mx);
                    alpha = orc_expf_det(m - mn);
                    for (ln = 0; ln < 32; ++ln) {
                        p[ln] = vrow[ln] ? orc_expf_det(sc[ln] - mn) : 0.0f;
                        tmp[ln] = p[ln];
                    }
                    psum = butterfly(tmp, 32);
                    l = l * alpha + psum;
                    for (d = 0; d < hd; ++d) {
                        float a = acc[d] * alpha;
                        for (ln = 0; ln < 32; ++ln) a = fmaf(p[ln], vrow[ln] ? vrow[ln][d] : 0.0f, a);
                        acc[d] = a;
                    }
                    m = mn;
                }
                pm[s] = m;
                pl[s] = l;
                memcpy(pacc + s * hd, acc, hd * sizeof(float));
            }
            {
                float M = -INFINITY, L = 0.0f, inv, *w = pl + n_active;
                for (s = 0; s < n_active; ++s) M = fmaxf(M, pm[s]);
                for (s = 0; s < n_active; ++s) w[s] = orc_expf_det(pm[s] - M);
                for (s = 0; s < n_active; ++s) L = fmaf(w[s], pl[s], L);
                inv = L > 0.0f ? 1.0f / L : 0.0f;
                for (d = 0; d < hd; ++d) {
                    float o = 0.0f;
                    for (s = 0; s < n_active; ++s) o = fmaf(w[s], pacc[s * hd + d], o);
                    out[h * hd + d] = o * inv;
                }
            }
        }
    }
    free(pm);
    free(pl);
    free(pacc);
    free(acc);
    return 1;
}

/* ------------------------------------------------------------------ */
/* forward                                                             */
/* ------------------------------------------------------------------ */

size_t orc_state_kv_floats(const orc_model *m) {
    return (size_t) m->layers * m->context * m->kv_heads * m->head_dim;
}

static int mv(const orc_state *st, int dtype, const uint8_t *w, size_t rows, size_t cols, const float *x, float *y,
              uint8_t *xq_scratch) {
    if (st->q8_1_activations && (dtype == ORC_Q4_K || dtype == ORC_Q6_K || dtype == ORC_Q8_0)) {
        if (!orc_q8_1_quantize(x, cols, xq_scratch)) return 0;
        if (st->matvec_user) /* threaded over rows; the same bits */
            return orc_pool_matvec_q8_1(st->matvec_user, st->norm_order == 1, dtype, w, rows, cols, xq_scratch, y);
        if (st->norm_order == 1) return orc_matvec_q8_1_dev(dtype, w, rows, cols, xq_scratch, y);
        return orc_matvec_q8_1(dtype, w, rows, cols, xq_scratch, y);
    }
    if (st->norm_order == 1 && (dtype == ORC_F32 || dtype == ORC_F16 || dtype == ORC_BF16))
        return orc_matvec_dense_dev(dtype, w, rows, cols, x, y);
    if (!st->q8_1_activations && st->matvec) return st->matvec(st->matvec_user, dtype, w, rows, cols, x, y);
    return orc_matvec_f32(dtype, w, rows, cols, x, y);
}

static int forward_impl(const orc_model *m, orc_state *st, uint32_t token, const float *emb, size_t pos, float *logits,
                        float *hidden_out);

int orc_forward_token(const orc_model *m, orc_state *st, uint32_t token, size_t pos, float *logits, float *hidden_out) {
    return forward_impl(m, st, token, NULL, pos, logits, hidden_out);
}

/* qwen3.uya:2534-2557 (qwen3_append_prompt_embeddings -> qwen3_forward_embedding_runtime):
 * the layer stack on a caller-given f32 input row instead of a token's embedding row. */
int orc_forward_embedding(const orc_model *m, orc_state *st, const float *emb, size_t pos, float *logits,
                          float *hidden_out) {
    if (!emb) return 0;
    return forward_impl(m, st, 0u, emb, pos, logits, hidden_out);
}

static int forward_impl(const orc_model *m, orc_state *st, uint32_t token, const float *emb, size_t pos, float *logits,
                        float *hidden_out) {
    size_t h = m->hidden, qd = (size_t) m->heads * m->head_dim, kvd = (size_t) m->kv_heads * m->head_dim;
    size_t f = m->ffn, maxd = h, L;
    size_t emb_rb = orc_row_bytes(m->token_embd_dtype, h);
    float *hid, *nrm, *q, *k, *v, *ctx, *ao, *g, *u, *fu, *dn;
    uint8_t *xq;
    int ok = 1;
    if (pos >= m->context || token >= m->vocab || emb_rb == 0) return 0;
    if (qd > maxd) maxd = qd;
    if (f > maxd) maxd = f;
    hid = (float *) calloc(h, 4); nrm = (float *) calloc(h, 4);
    q = (float *) calloc(qd, 4); k = (float *) calloc(kvd, 4); v = (float *) calloc(kvd, 4);
    ctx = (float *) calloc(qd, 4); ao = (float *) calloc(h, 4);
    g = (float *) calloc(f, 4); u = (float *) calloc(f, 4); fu = (float *) calloc(f, 4); dn = (float *) calloc(h, 4);
    xq = (uint8_t *) calloc(maxd / 32 + 1, 36);
    if (!hid || !nrm || !q || !k || !v || !ctx || !ao || !g || !u || !fu || !dn || !xq) { ok = 0; goto done; }

    /* qwen3.uya:1164-1174: token embedding row (or the given input row) */
    if (emb) memcpy(hid, emb, h * sizeof(float));
    else if (!orc_dequant_row(m->token_embd_dtype, m->token_embd + (size_t) token * emb_rb, h, hid)) { ok = 0; goto done; }

    for (L = 0; L < m->layers && ok; ++L) {
        const orc_layer *lw = &m->layer[L];
        size_t i;
        ok = ok && orc_rms_norm(hid, lw->attn_norm, lw->attn_norm_dtype, h, m->eps, st->norm_order, nrm);
        ok = ok && mv(st, lw->q_dtype, lw->q, qd, h, nrm, q, xq);
        ok = ok && mv(st, lw->k_dtype, lw->k, kvd, h, nrm, k, xq);
        ok = ok && mv(st, lw->v_dtype, lw->v, kvd, h, nrm, v, xq);
        if (!ok) break;
        if (lw->q_norm) orc_head_norm(q, lw->q_norm, lw->q_norm_dtype, m->heads, m->head_dim, st->norm_order);
        if (lw->k_norm) orc_head_norm(k, lw->k_norm, lw->k_norm_dtype, m->kv_heads, m->head_dim, st->norm_order);
        orc_rope_apply(q, m->heads, m->head_dim, pos, m->rope_cos, m->rope_sin);
        orc_rope_apply(k, m->kv_heads, m->head_dim, pos, m->rope_cos, m->rope_sin);
        /* qwen3.uya:1668-1675 */
        memcpy(st->k_cache + ((size_t) L * m->context + pos) * kvd, k, kvd * 4);
        memcpy(st->v_cache + ((size_t) L * m->context + pos) * kvd, v, kvd * 4);
        if (st->norm_order == 1) {
            /* f16 cache: every position, the current one included, is read
             * back as stored (rounded to nearest even) */
            const float *cur_k = k, *cur_v = v;
            if (st->kv_f16) {
                float *kc = st->k_cache + ((size_t) L * m->context + pos) * kvd;
                float *vc = st->v_cache + ((size_t) L * m->context + pos) * kvd;
                for (i = 0; i < kvd; ++i) {
                    kc[i] = orc_f16_to_f32(orc_f32_to_f16_rne(kc[i]));
                    vc[i] = orc_f16_to_f32(orc_f32_to_f16_rne(vc[i]));
                }
                cur_k = kc;
                cur_v = vc;
            }
            ok = ok && orc_attention_dev(ctx, q, st->k_cache, st->v_cache, cur_k, cur_v, L, pos, m->heads,
                                         m->kv_heads, m->head_dim, m->context);
        } else {
            ok = ok && orc_attention(ctx, q, st->k_cache, st->v_cache, L, pos, m->heads, m->kv_heads, m->head_dim,
                                     m->context);
        }
        ok = ok && mv(st, lw->o_dtype, lw->o, h, qd, ctx, ao, xq);
        for (i = 0; i < h; ++i) hid[i] = hid[i] + ao[i];
        ok = ok && orc_rms_norm(hid, lw->ffn_norm, lw->ffn_norm_dtype, h, m->eps, st->norm_order, nrm);
        ok = ok && mv(st, lw->gate_dtype, lw->gate, f, h, nrm, g, xq);
        ok = ok && mv(st, lw->up_dtype, lw->up, f, h, nrm, u, xq);
        if (st->norm_order == 1)
            orc_silu_mul_dev(fu, g, u, f);
        else
            orc_silu_mul(fu, g, u, f);
        ok = ok && mv(st, lw->down_dtype, lw->down, h, f, fu, dn, xq);
        for (i = 0; i < h; ++i) hid[i] = hid[i] + dn[i];
    }
    if (ok && hidden_out) memcpy(hidden_out, hid, h * 4);
    if (ok && logits) {
        const uint8_t *out_w = m->output ? m->output : m->token_embd;
        int out_dt = m->output ? m->output_dtype : m->token_embd_dtype;
        ok = orc_rms_norm(hid, m->output_norm, m->output_norm_dtype, h, m->eps, st->norm_order, nrm);
        ok = ok && mv(st, out_dt, out_w, m->vocab, h, nrm, logits, xq);
    }
done:
    free(hid); free(nrm); free(q); free(k); free(v); free(ctx); free(ao);
    free(g); free(u); free(fu); free(dn); free(xq);
    return ok;
}
