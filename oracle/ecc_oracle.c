/*
 * ecc_oracle.c -- CPU oracle for the ECC-INT4 KV-cache hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the CUDA library, the
 * Python packages) links, loads or calls this file.  It is used by tests/,
 * by __graft_entry__.smoke() and by bench.py's CPU-baseline leg, always as
 * the reference results the CUDA path is compared with, never as the thing
 * measured or shipped.
 *
 * It restates, in plain C, the reference's CPU algorithm for the two hot
 * paths of j-arndt/ecc-kv-cache:
 *
 *   compress  = custom_kv/ops_cpu.py:198 compress_cpu
 *               (hadamard_rotate_cpu :29, lloyd_max_params_cpu :64,
 *                lloyd_max_quantize_cpu :78, compute_syndrome_cpu :114)
 *               followed by the 128-byte ECC_KV_Block write of
 *               csrc/ecc_ops.h:22-32 (nibble order :40-49, syndrome bit
 *               order :56-64, fp16 meta as in csrc/compress_ecc.cu:164-166).
 *   decode    = custom_kv/fused_decode.py:200 cpu_reference_decode, with the
 *               GQA mapping kv_head = q_head / (Hq / Hkv) (HF repeat_kv).
 *
 * Bit-exactness of the compress restatement against the reference's torch
 * code (checked by tests/test_oracle_golden.py against fixtures made by
 * tests/golden/make_golden.py from the reference itself):
 *   - WHT butterfly with stride 1,2,...,64 (ops_cpu.py:47-56), fp32 add/sub,
 *     then IEEE fp32 division by fp32(sqrt(128)) (ops_cpu.py:59).
 *   - fp32 sums in the order torch's CPU sum kernel uses for a contiguous
 *     128-float vector: 4 accumulators x 8 lanes, element j into
 *     acc[(j/8)%4][j%8], the 4 blocks of 32 added in order, then
 *     t = ((acc0+acc1)+acc2)+acc3 lane-wise, then t0+t1+...+t7 in order.
 *     mean = sum/128 (ops_cpu.py:72), alpha = sum(|eps|)/128 (:219).
 *   - std (ops_cpu.py:73, unbiased): double accumulation of
 *     (double(x) - double(mean_f32))^2 in element order, /127, sqrt, rounded
 *     to fp32; scale = fp32(double(std_f32) + 1e-8).
 *   - xn = (x - zero) / scale in fp32; q = first index of the minimum of
 *     |xn - C[k]| (ops_cpu.py:99-100); k_tilde = C[q]*scale + zero with two
 *     fp32 roundings (:104); eps = x - k_tilde; bit = eps >= 0 (:126).
 * Build without FMA contraction (-ffp-contract=off, no -march=native).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

#define D 128

/* LM_CENTROIDS_NORM, custom_kv/ops_cpu.py:19-24, as fp32 bit patterns. */
static const uint32_t LM_BITS[16] = {
    0xc019a6b5u, 0xbfebf7cfu, 0xbfb7f2e5u, 0xbf8cb5ddu,
    0xbf4cb296u, 0xbf05bc02u, 0xbe8432cau, 0x00000000u,
    0x3e8432cau, 0x3f05bc02u, 0x3f4cb296u, 0x3f8cb5ddu,
    0x3fb7f2e5u, 0x3febf7cfu, 0x4019a6b5u, 0x404a233au};

static float lm(int k) {
    float f;
    memcpy(&f, &LM_BITS[k], 4);
    return f;
}

void orc_centroids(float out[16]) {
    for (int k = 0; k < 16; ++k) out[k] = lm(k);
}

/* ---- IEEE binary16 <-> binary32 (round to nearest even) ------------------ */
float orc_h2f(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1f;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = s;
        } else { /* subnormal: m * 2^-24 */
            float f = (float)m * 5.9604644775390625e-08f;
            memcpy(&bits, &f, 4);
            bits |= s;
        }
    } else if (e == 31) {
        bits = s | 0x7f800000u | (m << 13);
    } else {
        bits = s | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf or nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7c00u);
    }
    if (ax < 0x38800000u) { /* below the fp16 normal range: subnormal or 0 */
        /* value = ax_float; result = round(value / 2^-24) */
        float a;
        memcpy(&a, &ax, 4);
        /* scale exactly by 2^24 then round to nearest even integer */
        double v = (double)a * 16777216.0;
        double r = nearbyint(v); /* default rounding mode: nearest even */
        return (uint16_t)(sign | (uint32_t)r);
    }
    /* normal: rebias exponent, round mantissa from 23 to 10 bits */
    uint32_t e = (ax >> 23) - 112;
    uint32_t m = ax & 0x7fffffu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1; /* may carry into exponent: ok */
    return (uint16_t)(sign | h);
}

/* ---- hadamard_rotate_cpu (ops_cpu.py:29-59) for one 128-vector ---------- */
static const float SQRT128_F = 0x1.6a09e6p+3f; /* fp32(sqrt(128.0)) */

void orc_wht128(float *x) {
    for (int s = 1; s < D; s <<= 1) {
        for (int base = 0; base < D; base += 2 * s) {
            for (int j = 0; j < s; ++j) {
                float a = x[base + j], b = x[base + s + j];
                x[base + j] = a + b;
                x[base + s + j] = a - b;
            }
        }
    }
    for (int j = 0; j < D; ++j) x[j] = x[j] / SQRT128_F;
}

/* Generic power-of-two length, same butterfly (used for D != 128 tests). */
void orc_wht_any(float *x, int d) {
    for (int s = 1; s < d; s <<= 1)
        for (int base = 0; base < d; base += 2 * s)
            for (int j = 0; j < s; ++j) {
                float a = x[base + j], b = x[base + s + j];
                x[base + j] = a + b;
                x[base + s + j] = a - b;
            }
    float c = (float)sqrt((double)d);
    for (int j = 0; j < d; ++j) x[j] = x[j] / c;
}

/* torch CPU fp32 sum order for a contiguous 128-float vector. */
float orc_tsum128(const float *v) {
    float acc[4][8];
    for (int a = 0; a < 4; ++a)
        for (int l = 0; l < 8; ++l) acc[a][l] = 0.0f;
    for (int blk = 0; blk < 4; ++blk)
        for (int a = 0; a < 4; ++a)
            for (int l = 0; l < 8; ++l) acc[a][l] = acc[a][l] + v[blk * 32 + a * 8 + l];
    float t[8];
    for (int l = 0; l < 8; ++l) t[l] = ((acc[0][l] + acc[1][l]) + acc[2][l]) + acc[3][l];
    float s = t[0];
    for (int l = 1; l < 8; ++l) s = s + t[l];
    return s;
}

/* Full compress of one vector.  x16: 128 fp16 bit patterns.  rotate=0 means
 * the input is already rotated (csrc/ecc_ops.cpp:68 compress_and_store takes
 * x_rot).  Any output pointer may be NULL. */
void orc_compress_detail(const uint16_t *x16, int rotate, float *x_rot_out, uint8_t *q_out,
                         uint8_t *bits_out, float *zero_out, float *scale_out, float *alpha_out,
                         uint8_t *block_out) {
    float x[D];
    for (int j = 0; j < D; ++j) x[j] = orc_h2f(x16[j]);
    if (rotate) orc_wht128(x);

    const float zero = orc_tsum128(x) / 128.0f;
    const double mean_d = (double)zero;
    double acc = 0.0;
    for (int j = 0; j < D; ++j) {
        double dx = (double)x[j] - mean_d;
        acc += dx * dx;
    }
    const float std32 = (float)sqrt(acc / 127.0);
    const float scale = (float)((double)std32 + 1e-8);

    uint8_t q[D], bit[D];
    float aeps[D];
    for (int j = 0; j < D; ++j) {
        float xn = (x[j] - zero) / scale;
        int best = 0;
        float bd = fabsf(xn - lm(0));
        for (int k = 1; k < 16; ++k) {
            float dk = fabsf(xn - lm(k));
            if (dk < bd) {
                bd = dk;
                best = k;
            }
        }
        float kt = lm(best) * scale;
        kt = kt + zero;
        float eps = x[j] - kt;
        q[j] = (uint8_t)best;
        bit[j] = (uint8_t)(eps >= 0.0f);
        aeps[j] = fabsf(eps);
    }
    const float alpha = orc_tsum128(aeps) / 128.0f;

    if (x_rot_out) memcpy(x_rot_out, x, sizeof(x));
    if (q_out) memcpy(q_out, q, D);
    if (bits_out) memcpy(bits_out, bit, D);
    if (zero_out) *zero_out = zero;
    if (scale_out) *scale_out = scale;
    if (alpha_out) *alpha_out = alpha;
    if (block_out) {
        memset(block_out, 0, 128);
        for (int i = 0; i < 64; ++i) block_out[i] = (uint8_t)(q[2 * i] | (q[2 * i + 1] << 4));
        for (int j = 0; j < D; ++j)
            if (bit[j]) block_out[64 + j / 8] |= (uint8_t)(1u << (j % 8));
        uint16_t m[3] = {orc_f2h(scale), orc_f2h(zero), orc_f2h(alpha)};
        for (int i = 0; i < 3; ++i) {
            block_out[80 + 2 * i] = (uint8_t)(m[i] & 0xff);
            block_out[81 + 2 * i] = (uint8_t)(m[i] >> 8);
        }
    }
}

/* Batched compress into 128-byte blocks.  Single-threaded: callers that
 * want several cores split the rows and call this from several threads (the
 * function touches only its own rows). */
void orc_compress(const uint16_t *x16, int64_t n, int rotate, uint8_t *blocks) {
    for (int64_t i = 0; i < n; ++i)
        orc_compress_detail(x16 + i * D, rotate, NULL, NULL, NULL, NULL, NULL, NULL, blocks + i * 128);
}

/* Number of elements of a vector whose normalised value lies within `tol`
 * of a quantiser decision boundary (midpoint of adjacent centroids). */
int64_t orc_count_ties(const uint16_t *x16, int64_t n, int rotate, float tol) {
    int64_t ties = 0;
    for (int64_t i = 0; i < n; ++i) {
        float x[D];
        for (int j = 0; j < D; ++j) x[j] = orc_h2f(x16[i * D + j]);
        if (rotate) orc_wht128(x);
        float zero = orc_tsum128(x) / 128.0f;
        double acc = 0.0;
        for (int j = 0; j < D; ++j) {
            double dx = (double)x[j] - (double)zero;
            acc += dx * dx;
        }
        float scale = (float)((double)(float)sqrt(acc / 127.0) + 1e-8);
        for (int j = 0; j < D; ++j) {
            double xn = ((double)x[j] - (double)zero) / (double)scale;
            for (int k = 0; k < 15; ++k) {
                double mid = 0.5 * ((double)lm(k) + (double)lm(k + 1));
                if (fabs(xn - mid) <= tol) ties++;
            }
        }
    }
    return ties;
}

/* Unpack one block into codes, sign bits and the three fp16 meta words. */
void orc_unpack_block(const uint8_t *blk, uint8_t *q, uint8_t *bits, uint16_t *meta) {
    for (int i = 0; i < 64; ++i) {
        q[2 * i] = blk[i] & 0x0f;
        q[2 * i + 1] = blk[i] >> 4;
    }
    for (int j = 0; j < D; ++j) bits[j] = (blk[64 + j / 8] >> (j % 8)) & 1;
    for (int i = 0; i < 3; ++i) meta[i] = (uint16_t)(blk[80 + 2 * i] | (blk[81 + 2 * i] << 8));
}

/* Reconstruct k_rec = (C[q]*scale + zero) + alpha*s in fp32 exactly as
 * custom_kv/fused_decode.py:229-241 does (two roundings, then one add). */
void orc_reconstruct(const uint8_t *blk, float *out) {
    uint8_t q[D], bits[D];
    uint16_t meta[3];
    orc_unpack_block(blk, q, bits, meta);
    float sc = orc_h2f(meta[0]), zr = orc_h2f(meta[1]), al = orc_h2f(meta[2]);
    for (int j = 0; j < D; ++j) {
        float kt = lm(q[j]) * sc;
        kt = kt + zr;
        float s = bits[j] ? 1.0f : -1.0f;
        out[j] = kt + al * s;
    }
}

/* Decode oracle (fused_decode.py:200-265) with GQA.
 *   q16:   [B, Hq, 128] fp16 (rotated query unless flags&1)
 *   kb/vb: block pools; block (b, h, t) at byte offset
 *          (b*stride_b + h*stride_h + t) * 128
 *   flags: 1 = rotate the query first (q_rot = fp16(WHT(q))),
 *          2 = apply the WHT to the output (values stored rotated).
 *   h_begin/h_end: the query heads this call computes (threads split heads).
 *   out:   [B, Hq, 128] fp32 (caller rounds to fp16 to compare).
 * Scores and softmax are accumulated in double; the reference's fp32 order
 * is not reproducible (BLAS dot), so comparisons use a tolerance. */
void orc_decode(const uint16_t *q16, const uint8_t *kb, const uint8_t *vb, int64_t stride_b,
                int64_t stride_h, int B, int Hq, int Hkv, int64_t L, float sm_scale, int flags,
                int h_begin, int h_end, float *out) {
    const int group = Hq / Hkv;
    if (!(sm_scale > 0.0f)) sm_scale = (float)(1.0 / sqrt((double)D));
    for (int b = 0; b < B; ++b) {
        for (int h = h_begin; h < h_end; ++h) {
            const int kvh = h / group;
            float q[D];
            for (int j = 0; j < D; ++j) q[j] = orc_h2f(q16[((int64_t)b * Hq + h) * D + j]);
            if (flags & 1) {
                orc_wht128(q);
                for (int j = 0; j < D; ++j) q[j] = orc_h2f(orc_f2h(q[j]));
            }
            double *sc = (double *)malloc(sizeof(double) * (size_t)(L > 0 ? L : 1));
            double m = -INFINITY;
            for (int64_t t = 0; t < L; ++t) {
                const uint8_t *blk = kb + ((int64_t)b * stride_b + (int64_t)kvh * stride_h + t) * 128;
                float k[D];
                orc_reconstruct(blk, k);
                double dot = 0.0;
                for (int j = 0; j < D; ++j) dot += (double)q[j] * (double)k[j];
                float s = (float)dot * sm_scale;
                sc[t] = s;
                if (s > m) m = s;
            }
            double l = 0.0, o[D];
            for (int j = 0; j < D; ++j) o[j] = 0.0;
            for (int64_t t = 0; t < L; ++t) {
                double w = exp(sc[t] - m);
                l += w;
                const uint8_t *blk = vb + ((int64_t)b * stride_b + (int64_t)kvh * stride_h + t) * 128;
                float v[D];
                orc_reconstruct(blk, v);
                for (int j = 0; j < D; ++j) o[j] += w * (double)v[j];
            }
            float of[D];
            for (int j = 0; j < D; ++j) of[j] = (L > 0) ? (float)(o[j] / l) : 0.0f;
            if (flags & 2) orc_wht128(of);
            memcpy(out + ((int64_t)b * Hq + h) * D, of, sizeof(of));
            free(sc);
        }
    }
}

/* Log-sum-exp merge of split partials, the host-side statement of the
 * flash-decoding combine.  Each partial i of a row holds its running max
 * m_i, its weight sum l_i = sum_t e^(s_t - m_i) and its UNNORMALISED value
 * sum o_i = sum_t e^(s_t - m_i) v_t.  Merged: m = max m_i over non-empty
 * partials, l = sum l_i e^(m_i-m), o = (sum o_i e^(m_i-m)) / l.
 * pm/pl: [rows, n]; po: [rows, n, 128]; empty partials have l_i == 0. */
void orc_lse_merge(const float *pm, const float *pl, const float *po, int64_t rows, int n, float *out) {
    for (int64_t r = 0; r < rows; ++r) {
        double m = -INFINITY;
        for (int i = 0; i < n; ++i)
            if (pl[r * n + i] > 0 && pm[r * n + i] > m) m = pm[r * n + i];
        double l = 0.0, o[D];
        for (int j = 0; j < D; ++j) o[j] = 0.0;
        for (int i = 0; i < n; ++i) {
            if (!(pl[r * n + i] > 0)) continue;
            double w = exp((double)pm[r * n + i] - m);
            l += w * pl[r * n + i];
            for (int j = 0; j < D; ++j) o[j] += w * po[(r * n + i) * D + j];
        }
        for (int j = 0; j < D; ++j) out[r * D + j] = (l > 0) ? (float)(o[j] / l) : 0.0f;
    }
}

/* Test helper for the product's division by the constant fp32(sqrt(128)):
 * counts x (bit patterns start, start+stride, ... count values) with
 * 2^-100 <= |x| < 2^100 where the remainder-corrected quotient
 * q0 = x*r, rem = fma(-q0, c, x), q = fma(rem, r, q0) (r = RN(1/c)) differs
 * from the IEEE quotient x/c.  Needs a host with FMA. */
__attribute__((target("fma"))) int64_t orc_check_div_sqrt128(uint32_t start, uint32_t count, uint32_t stride) {
    const float c = SQRT128_F;
    const float r = (float)(1.0 / (double)c);
    int64_t bad = 0;
    uint32_t b = start;
    for (uint32_t i = 0; i < count; ++i, b += stride) {
        float x;
        memcpy(&x, &b, 4);
        float ax = fabsf(x);
        if (!(ax >= 0x1p-100f && ax < 0x1p+100f)) continue;
        float q0 = x * r;
        float rem = __builtin_fmaf(-q0, c, x);
        float q = __builtin_fmaf(rem, r, q0);
        float ref = x / c;
        if (memcmp(&q, &ref, 4) != 0) bad++;
    }
    return bad;
}
