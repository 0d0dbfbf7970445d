// compress.cu -- WHT + Lloyd-Max INT4 + sign syndrome -> 128-byte blocks, the
// standalone WHT op, block metadata readback, dequantisation and SoA packing.
//
// The compress kernel is bit-exact with the reference's CPU pipeline
// custom_kv/ops_cpu.py:198 compress_cpu by construction:
//   * WHT stages stride 1,2,...,64 in fp32 (ops_cpu.py:47-56), then the IEEE
//     quotient by fp32(sqrt(128)) (ops_cpu.py:59) computed as
//     q0 = x*r, rem = fma(-q0, c, x), q = fma(rem, r, q0) with r = RN(1/c):
//     one remainder-corrected Newton step (Markstein, "IA-64 and elementary
//     functions", 2000, ch. 8).  An exhaustive check over all fp32 x with
//     2^-100 <= |x| < 2^100 shows it equals x/c (every nonzero WHT value of
//     fp16 inputs lies in that range); x = -0 gives +0, and no output depends
//     on the sign of a zero rotated element.
//   * fp32 sums (mean, alpha) in the order torch's CPU sum kernel uses for a
//     contiguous 128-float vector: acc[(j/8)%4][j%8] seeded with +0, blocks of
//     32 added in order, t = ((acc0+acc1)+acc2)+acc3, then t0+...+t7.
//   * std: fp64 sum of (double(x) - double(mean))^2 / 127, sqrt, rounded to
//     fp32 (torch's std_var_all_cpu).  The fast path sums with FMA and a tree;
//     when the fp64 result lies within 1e-12 (relative) of an fp32 rounding
//     midpoint the vector is re-summed in element order with separate
//     multiply and add, exactly like the CPU.
//   * quantiser: argmin_k |(x-zero)/scale - C[k]| (ops_cpu.py:96-100) is taken
//     from a cell table of the approximate quotient u = (x-zero)*RN(1/scale);
//     whenever u lies within 4e-6 of a decision threshold the element is
//     recomputed with the IEEE quotient and the full first-index argmin.
//   * k_tilde = C[q]*scale + zero with two roundings, eps = x - k_tilde,
//     bit = eps >= 0 (ops_cpu.py:104, :126).
//
// Thread layout: 4 lanes per vector, 8 vectors per warp.  Lane g of a vector
// holds elements e = 32c + 8g + i (c, i in 0..3, 0..7): WHT strides 1,2,4 and
// 32,64 stay in registers, strides 8,16 are lane exchanges, and each lane owns
// torch's accumulator a = g for all four blocks c.
#include <algorithm>
#include <cmath>
#include <mutex>

#include "ecc_common.cuh"

namespace ecc {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kCells = 192;       // u cells of width 1/8: cell = rint(8u + 96)
constexpr int kReplicas = 8;      // one table copy per (lane % 8): conflict-free LDS.128
constexpr float kBand = 4e-6f;    // exact-recompute band around each threshold (u = RN(d * rs))
// Band of the packed fast pass, whose side test is w = RN(d * rs - thr) with
// one rounding.  Near a threshold |d * rs - d / scale| <= 1.7e-7, the
// reference's RN(d / scale) adds <= 1.2e-7, its flip point lies within 1e-7
// of the exact midpoint and thr within 1.2e-7 of it: a decision with
// |w| >= 5.2e-7 is the reference's.  A CPU stress of 4 M near-threshold
// quotients sees wrong decisions only for |w| < 2.8e-7.  The band is 1.5x
// the bound.
constexpr float kBandFast = 8e-7f;
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23: fma(u, 8, kMagic + 96) rounds 8u+96 to an integer
constexpr int kCompressWarps = 8;
constexpr int kVecPerWarp = 8;
constexpr int kVecPerTile = kCompressWarps * kVecPerWarp;

// Unsigned 32-bit division by a runtime constant d >= 1 (round-up method:
// s = ceil(log2 d), m = floor(2^32 (2^s - d) / d) + 1, q = (umulhi(n,m) + n) >> s),
// valid for every n < 2^32.
struct FastDiv {
    uint32_t d, m, s;
};
static inline FastDiv make_fastdiv(uint32_t d) {
    FastDiv f;
    f.d = d;
    f.s = 0;
    while ((1ull << f.s) < d) ++f.s;
    f.m = (uint32_t)((((1ull << 32) * ((1ull << f.s) - d)) / d) + 1);
    return f;
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, FastDiv f) {
    return (uint32_t)(((uint64_t)__umulhi(n, f.m) + n) >> f.s);
}

struct __align__(16) QEntry {
    float thr;   // decision threshold inside this cell, +inf if none
    float c_lo;  // centroid below the threshold
    float c_hi;  // centroid above the threshold
    int q_lo;    // code below the threshold
};

__device__ __forceinline__ int cell_of(float u) {
    const float t = __fmaf_rn(u, 8.0f, kMagic + 96.0f);
    return __float_as_int(t) - __float_as_int(kMagic);
}

// Thresholds m_j = (C[j-1] + C[j]) / 2, j = 1..15.  They are >= 2 cells apart
// and >= 0.09 cells from every cell boundary, so a value within kBand of a
// threshold always falls in that threshold's own cell.
__device__ void build_qtable(QEntry *tab) {
    for (int cell = threadIdx.x; cell < kCells; cell += blockDim.x) {
        int below = 0, own = -1;
#pragma unroll
        for (int j = 1; j < 16; ++j) {
            const float m = __fmul_rn(__fadd_rn(lm(j - 1), lm(j)), 0.5f);
            const int cm = cell_of(m);
            if (cm < cell) ++below;
            if (cm == cell) own = j;
        }
        QEntry e;
        if (own > 0) {
            e.thr = __fmul_rn(__fadd_rn(lm(own - 1), lm(own)), 0.5f);
            e.q_lo = own - 1;
        } else {
            e.thr = __int_as_float(0x7f800000);
            e.q_lo = below;
        }
        e.c_lo = lm(e.q_lo);
        e.c_hi = lm(e.q_lo < 15 ? e.q_lo + 1 : 15);
#pragma unroll
        for (int r = 0; r < kReplicas; ++r) tab[cell * kReplicas + r] = e;
    }
}

// torch-order fp32 sum over the 128 elements of the vector held by the 4
// lanes starting at `base` (see the file comment); every lane gets the sum.
__device__ __forceinline__ float tsum_group(const float (&v)[4][8], int base) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float acc = __fadd_rn(0.0f, v[0][i]);
        acc = __fadd_rn(acc, v[1][i]);
        acc = __fadd_rn(acc, v[2][i]);
        acc = __fadd_rn(acc, v[3][i]);
        const float a0 = __shfl_sync(kFull, acc, base + 0);
        const float a1 = __shfl_sync(kFull, acc, base + 1);
        const float a2 = __shfl_sync(kFull, acc, base + 2);
        const float a3 = __shfl_sync(kFull, acc, base + 3);
        const float t = __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
        s = (i == 0) ? t : __fadd_rn(s, t);
    }
    return s;
}

// Normalised WHT of the vector held by a 4-lane group (layout above).
__device__ __forceinline__ void wht_group(float (&v)[4][8], int g) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int i = 0; i < 8; i += 2) {  // stride 1
            const float a = v[c][i], b = v[c][i + 1];
            v[c][i] = __fadd_rn(a, b);
            v[c][i + 1] = __fsub_rn(a, b);
        }
#pragma unroll
        for (int i0 = 0; i0 < 8; i0 += 4) {  // stride 2
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float a = v[c][i0 + j], b = v[c][i0 + j + 2];
                v[c][i0 + j] = __fadd_rn(a, b);
                v[c][i0 + j + 2] = __fsub_rn(a, b);
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {  // stride 4
            const float a = v[c][j], b = v[c][j + 4];
            v[c][j] = __fadd_rn(a, b);
            v[c][j + 4] = __fsub_rn(a, b);
        }
    }
#pragma unroll
    for (int s = 1; s <= 2; s <<= 1) {  // strides 8, 16: partner lane g ^ s
        // lower index: mine + partner; upper index: partner - mine.  An FMA
        // with multiplier +-1 rounds exactly like the add/sub.
        const float sgn = (g & s) ? -1.0f : 1.0f;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float p = __shfl_xor_sync(kFull, v[c][i], s);
                v[c][i] = __fmaf_rn(sgn, v[c][i], p);
            }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {  // stride 32 (c ^ 1) then 64 (c ^ 2)
        float a = v[0][i], b = v[1][i];
        v[0][i] = __fadd_rn(a, b);
        v[1][i] = __fsub_rn(a, b);
        a = v[2][i];
        b = v[3][i];
        v[2][i] = __fadd_rn(a, b);
        v[3][i] = __fsub_rn(a, b);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float a = v[0][i], b = v[2][i];
        v[0][i] = __fadd_rn(a, b);
        v[2][i] = __fsub_rn(a, b);
        a = v[1][i];
        b = v[3][i];
        v[1][i] = __fadd_rn(a, b);
        v[3][i] = __fsub_rn(a, b);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float x = v[c][i];
            const float q0 = __fmul_rn(x, kInvSqrt128);
            const float rem = __fmaf_rn(-q0, kSqrt128, x);
            // x = +-inf: the remainder is inf - inf = NaN, the quotient is +-inf
            v[c][i] = fabsf(q0) == INFINITY ? q0 : __fmaf_rn(rem, kInvSqrt128, q0);
        }
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t w) {
    __half2 h = *reinterpret_cast<__half2 *>(&w);
    return __half22float2(h);
}

// Exact first-index argmin of ops_cpu.py:99-100 for one element.
__device__ __noinline__ int exact_code(float d, float scale) {
    const float xn = __fdiv_rn(d, scale);
    int best = 0;
    float bd = fabsf(__fsub_rn(xn, lm(0)));
#pragma unroll
    for (int k = 1; k < 16; ++k) {
        const float dk = fabsf(__fsub_rn(xn, lm(k)));
        if (dk < bd) {
            bd = dk;
            best = k;
        }
    }
    return best;
}

// One compress job: vectors (b, h, l) of a strided fp16 [B, H, L, 128] view
// into blocks (b, h, l) of a pool.
struct CompressJob {
    const __half *x;
    int64_t xs_b, xs_h, xs_l;
    uint8_t *blocks;
    int64_t bs_b, bs_h;
    FastDiv div_h, div_l;
    uint32_t n_vec, n_tiles;
    const int *pos_dev;  // token offset read from device memory when set (launches replayed from a graph)
    int64_t cap;         // tokens per (b, h) row of the pool, for the offset check
    uint32_t rec;        // bytes per block record in the pool: 128, or 96 without the pad sector
};

__device__ int g_compress_error;  // a device-side position was out of range

// Byte offset of a job's destination: *pos_dev tokens when the position lives
// in device memory.  A position with pos < 0 or pos + L > cap writes nothing
// and raises g_compress_error (read by ecc_device_status).
__device__ __forceinline__ bool job_offset(const CompressJob &jb, int64_t &off) {
    off = 0;
    if (!jb.pos_dev) return true;
    const int64_t p = *jb.pos_dev;
    if (p < 0 || p + (int64_t)jb.div_l.d > jb.cap) {
        if (threadIdx.x == 0) atomicExch(&g_compress_error, 3);
        return false;
    }
    off = p * jb.rec;
    return true;
}
// Up to two jobs in one launch (K and V of one append): tiles [0, n_tiles of
// job 0) belong to job 0, the rest to job 1.
struct CompressJobs {
    CompressJob j[2];
    int njobs;
};

// One warp's kVecPerWarp vectors of tile `tile`.  The fast pass (kExact =
// false) gives up and returns false, before writing anything, when any of the
// warp's elements needs the exact treatment (a quotient within kBand of a
// decision threshold, or a std near an fp32 rounding midpoint); the exact
// pass handles those elements one by one.  Keeping the exact code out of the
// fast pass keeps the hot loop small.
template <bool kRotate, bool kExact>
__device__ __forceinline__ bool compress_warp(const __half *__restrict__ x, int64_t xs_b, int64_t xs_h, int64_t xs_l,
                                              uint8_t *__restrict__ blocks, int64_t bs_b, int64_t bs_h,
                                              FastDiv div_h, FastDiv div_l, uint32_t n_vec, uint32_t tile,
                                              const QEntry *tab, uint32_t *st, uint32_t rec) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane & 3, vsub = lane >> 2, base = lane & ~3;
    const uint32_t vi = tile * kVecPerTile + warp * kVecPerWarp + vsub;
    const bool valid = vi < n_vec;
    const uint32_t row = fdiv(valid ? vi : 0u, div_l);
    const int64_t l = (valid ? vi : 0u) - row * div_l.d;
    const uint32_t bq = fdiv(row, div_h);
    const int64_t b = bq, h = row - bq * div_h.d;

    float v[4][8];
    {
        const __half *src = x + b * xs_b + h * xs_h + l * xs_l + 8 * g;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint4 raw = make_uint4(0, 0, 0, 0);
            if (valid) raw = __ldcs(reinterpret_cast<const uint4 *>(src + 32 * c));
            float2 f;
            f = h2_to_f2(raw.x); v[c][0] = f.x; v[c][1] = f.y;
            f = h2_to_f2(raw.y); v[c][2] = f.x; v[c][3] = f.y;
            f = h2_to_f2(raw.z); v[c][4] = f.x; v[c][5] = f.y;
            f = h2_to_f2(raw.w); v[c][6] = f.x; v[c][7] = f.y;
        }
    }
    if (kRotate) wht_group(v, g);

    // mean (zero point), ops_cpu.py:72
    const float zero = __fmul_rn(tsum_group(v, base), 0.0078125f);

    // unbiased std, ops_cpu.py:73
    const double md = (double)zero;
    double acc = 0.0;
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const double dx = (double)v[c][i] - md;
            acc = fma(dx, dx, acc);
        }
    acc += __shfl_xor_sync(kFull, acc, 1);
    acc += __shfl_xor_sync(kFull, acc, 2);
    double sd = __dsqrt_rn(__ddiv_rn(acc, 127.0));
    float s32 = __double2float_rn(sd);
    {
        const double lo = (double)s32;
        const double nb = (double)(lo <= sd ? nextafterf(s32, INFINITY) : nextafterf(s32, 0.0f));
        const double mid = 0.5 * (lo + nb);
        const bool amb = fabs(sd - mid) <= 1e-12 * sd;
        if (!kExact && __any_sync(kFull, amb)) return false;  // rare: the exact pass re-sums
        if (kExact && __any_sync(kFull, amb)) {  // re-sum in element order
            double ex = 0.0;
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll 1
                for (int gg = 0; gg < 4; ++gg)
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float xv = __shfl_sync(kFull, v[c][i], base + gg);
                        const double dx = __dsub_rn((double)xv, md);
                        ex = __dadd_rn(ex, __dmul_rn(dx, dx));
                    }
            if (amb) {
                sd = __dsqrt_rn(__ddiv_rn(ex, 127.0));
                s32 = __double2float_rn(sd);
            }
        }
    }
    const float scale = __double2float_rn(__dadd_rn((double)s32, 1e-8));
    const float rs = __frcp_rn(scale);

    // quantise, residual, syndrome
    uint32_t codes[4] = {0u, 0u, 0u, 0u};
    uint32_t bits = 0u;
    bool band = false;  // an element lies within kBand of a decision threshold
    const QEntry *mytab = tab + (lane & (kReplicas - 1));
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float xv = v[c][i];
            const float d = __fsub_rn(xv, zero);
            const float u = __fmul_rn(d, rs);
            const unsigned cell = min((unsigned)cell_of(u), (unsigned)(kCells - 1));
            const QEntry e = mytab[cell * kReplicas];
            const bool hi = u > e.thr;
            float cq = hi ? e.c_hi : e.c_lo;
            int q = e.q_lo + (hi ? 1 : 0);
            if constexpr (kExact) {
                if (fabsf(__fsub_rn(u, e.thr)) < kBand) {
                    q = exact_code(d, scale);
                    cq = lm(0);
#pragma unroll
                    for (int k = 1; k < 16; ++k) cq = (q == k) ? lm(k) : cq;
                }
            } else {
                band = band || (fabsf(__fsub_rn(u, e.thr)) < kBand);
            }
            const float kt = __fadd_rn(__fmul_rn(cq, scale), zero);
            const float eps = __fsub_rn(xv, kt);
            bits |= (eps >= 0.0f ? 1u : 0u) << (8 * c + i);
            codes[c] |= (uint32_t)q << (4 * i);
            v[c][i] = fabsf(eps);
        }
    if (!kExact && __any_sync(kFull, band)) return false;  // the exact pass redoes the warp's vectors
    const float alpha = __fmul_rn(tsum_group(v, base), 0.0078125f);

    // stage: code word 4c+g and syndrome byte 4c+g of this vector
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        st[4 * c + g] = codes[c];
        reinterpret_cast<uint8_t *>(st + 16)[4 * c + g] = (uint8_t)(bits >> (8 * c));
    }
    __syncwarp();
    if (valid) {
        uint8_t *dst = blocks + (b * bs_b + h * bs_h + l) * rec;
        const uint4 w0 = *reinterpret_cast<const uint4 *>(st + 4 * g);
        uint4 w1;
        if (g == 0) {
            w1 = *reinterpret_cast<const uint4 *>(st + 16);
        } else if (g == 1) {
            const uint32_t hs = __half_as_ushort(__float2half_rn(scale));
            const uint32_t hz = __half_as_ushort(__float2half_rn(zero));
            const uint32_t ha = __half_as_ushort(__float2half_rn(alpha));
            w1 = make_uint4(hs | (hz << 16), ha, 0u, 0u);
        } else {
            w1 = make_uint4(0u, 0u, 0u, 0u);
        }
        __stcs(reinterpret_cast<uint4 *>(dst + 16 * g), w0);
        if (64 + 16 * g < (int)rec) __stcs(reinterpret_cast<uint4 *>(dst + 64 + 16 * g), w1);
    }
    __syncwarp();
    return true;
}

template <bool kRotate>
__device__ __noinline__ void compress_warp_exact(const __half *__restrict__ x, int64_t xs_b, int64_t xs_h,
                                                 int64_t xs_l, uint8_t *__restrict__ blocks, int64_t bs_b,
                                                 int64_t bs_h, FastDiv div_h, FastDiv div_l, uint32_t n_vec,
                                                 uint32_t tile, const QEntry *tab, uint32_t *st, uint32_t rec) {
    compress_warp<kRotate, true>(x, xs_b, xs_h, xs_l, blocks, bs_b, bs_h, div_h, div_l, n_vec, tile, tab, st, rec);
}

// ---- packed fast pass -------------------------------------------------------
// The same arithmetic as compress_warp, with the element pairs (i, i+1) of a
// lane held in float2 registers so that every butterfly, quotient and
// quantiser step is one packed fp32x2 instruction (add/mul/fma .rn on two
// lanes, each rounded exactly like its scalar form; no packed product is ever
// followed by a packed add of it, which ptxas would fuse).  Torch's
// accumulator lanes are reduced through shared memory (each lane adds two of
// the eight slots, see tsum_finish) instead of by 32 shuffles per sum.

__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
// a - b, rounded once (fma with multiplier -1 is exact before its rounding)
__device__ __forceinline__ float2 sub2(float2 a, float2 b) { return __ffma2_rn(b, make_float2(-1.0f, -1.0f), a); }

// Stride-1 butterfly of an fp16 pair (a, b): (RN(a + b), RN(a - b)) in fp32,
// with the mixed-precision add/sub that widens a exactly before adding.
__device__ __forceinline__ float2 bfly_h2(uint32_t w) {
    float2 r;
    asm("{\n .reg .b16 lo, hi;\n .reg .f32 fh;\n mov.b32 {lo, hi}, %2;\n cvt.f32.f16 fh, hi;\n"
        " add.rn.f32.f16 %0, lo, fh;\n sub.rn.f32.f16 %1, lo, fh;\n}"
        : "=f"(r.x), "=f"(r.y)
        : "r"(w));
    return r;
}

__device__ __forceinline__ float4 lds_f4(uint32_t a) {
    float4 r;
    // the table is constant after the kernel's set-up barrier: not volatile
    asm("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "r"(a));
    return r;
}

// Finishes a torch-order sum whose lane g holds accumulator g's eight slots
// (A[j] = slots 2j, 2j+1): slot i of the four accumulators is combined as
// ((acc0 + acc1) + acc2) + acc3 by lane i/2, then the eight slot totals are
// added in order.  `red` is the vector's 40-float area (32 accumulator slots,
// then 8 slot totals); every lane of the vector gets the sum.
__device__ __forceinline__ float tsum_finish(const float2 (&A)[4], float *red, int g) {
    __syncwarp();  // earlier readers of the area are done
    float4 *r4 = reinterpret_cast<float4 *>(red + 8 * g);
    r4[0] = make_float4(A[0].x, A[0].y, A[1].x, A[1].y);
    r4[1] = make_float4(A[2].x, A[2].y, A[3].x, A[3].y);
    __syncwarp();
    float2 t = *reinterpret_cast<const float2 *>(red + 2 * g);
    t = add2(t, *reinterpret_cast<const float2 *>(red + 8 + 2 * g));
    t = add2(t, *reinterpret_cast<const float2 *>(red + 16 + 2 * g));
    t = add2(t, *reinterpret_cast<const float2 *>(red + 24 + 2 * g));
    *reinterpret_cast<float2 *>(red + 32 + 2 * g) = t;
    __syncwarp();
    const float4 u0 = reinterpret_cast<const float4 *>(red + 32)[0];
    const float4 u1 = reinterpret_cast<const float4 *>(red + 32)[1];
    float s = __fadd_rn(u0.x, u0.y);
    s = __fadd_rn(s, u0.z);
    s = __fadd_rn(s, u0.w);
    s = __fadd_rn(s, u1.x);
    s = __fadd_rn(s, u1.y);
    s = __fadd_rn(s, u1.z);
    return __fadd_rn(s, u1.w);
}

// Where a lane's vector of the current tile lives.
struct VecRef {
    uint8_t *dst;  // its block
    bool valid;
    bool tail;     // this lane also writes bytes 64 + 16g.. of the block (false for the pad sector of a 96-byte record)
};

__device__ __forceinline__ void load_vec(const CompressJob &jb, uint32_t tile, uint4 (&raw)[4], VecRef &ref,
                                         int64_t off = 0, bool enabled = true) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane & 3, vsub = lane >> 2;
    const uint32_t vi = tile * kVecPerTile + warp * kVecPerWarp + vsub;
    ref.valid = enabled && vi < jb.n_vec;
    const uint32_t v = min(vi, jb.n_vec - 1u);  // lanes past the end re-read the last vector, store nothing
    const uint32_t row = fdiv(v, jb.div_l);
    const int64_t l = v - row * jb.div_l.d;
    const uint32_t bq = fdiv(row, jb.div_h);
    const int64_t b = bq, h = row - bq * jb.div_h.d;
    const __half *src = jb.x + b * jb.xs_b + h * jb.xs_h + l * jb.xs_l + 8 * g;
    ref.dst = jb.blocks + off + (b * jb.bs_b + h * jb.bs_h + l) * jb.rec;
    ref.tail = 64 + 16 * g < (int)jb.rec;
#pragma unroll
    for (int c = 0; c < 4; ++c)
        raw[c] = __ldcs(reinterpret_cast<const uint4 *>(src + 32 * c));
}

// Fast pass over the warp's eight vectors (lane layout as compress_warp).
// Returns false, having written nothing, when any vector of the warp needs
// the exact pass: a quotient within kBandFast of a decision threshold, a std
// near an fp32 rounding midpoint, or a non-finite scale or zero point.
// `tabq` is the shared-window address of this lane's replica of entry 0,
// `red` the vector's reduction area, `st` its staging row.
template <bool kRotate>
__device__ __forceinline__ bool compress_fast(const uint4 (&raw)[4], const VecRef &ref, uint32_t tabq, float *red,
                                              uint32_t *st) {
    const int g = threadIdx.x & 3;
    float2 P[4][4];  // P[c][j] = elements 32c + 8g + 2j, +1
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint32_t w[4] = {raw[c].x, raw[c].y, raw[c].z, raw[c].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) P[c][j] = kRotate ? bfly_h2(w[j]) : h2_to_f2(w[j]);  // stride 1
    }
    if (kRotate) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
            for (int j = 0; j < 4; j += 2) {  // stride 2
                const float2 a = P[c][j], b = P[c][j + 1];
                P[c][j] = add2(a, b);
                P[c][j + 1] = sub2(a, b);
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {  // stride 4
                const float2 a = P[c][j], b = P[c][j + 2];
                P[c][j] = add2(a, b);
                P[c][j + 2] = sub2(a, b);
            }
        }
#pragma unroll
        for (int s = 1; s <= 2; s <<= 1) {  // strides 8, 16: partner lane g ^ s
            const float sg = (g & s) ? -1.0f : 1.0f;
            const float2 sg2 = make_float2(sg, sg);
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 p = make_float2(__shfl_xor_sync(kFull, P[c][j].x, s),
                                                 __shfl_xor_sync(kFull, P[c][j].y, s));
                    P[c][j] = fma2(sg2, P[c][j], p);
                }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {  // stride 32, then 64
            float2 a = P[0][j], b = P[1][j];
            P[0][j] = add2(a, b);
            P[1][j] = sub2(a, b);
            a = P[2][j];
            b = P[3][j];
            P[2][j] = add2(a, b);
            P[3][j] = sub2(a, b);
            a = P[0][j];
            b = P[2][j];
            P[0][j] = add2(a, b);
            P[2][j] = sub2(a, b);
            a = P[1][j];
            b = P[3][j];
            P[1][j] = add2(a, b);
            P[3][j] = sub2(a, b);
        }
        const float2 r2 = make_float2(kInvSqrt128, kInvSqrt128), nc2 = make_float2(-kSqrt128, -kSqrt128);
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 q0 = mul2(P[c][j], r2);
                const float2 rem = fma2(q0, nc2, P[c][j]);
                P[c][j] = fma2(rem, r2, q0);
            }
    }

    // mean (zero point), ops_cpu.py:72: torch accumulator g, slots in c order
    float2 A[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        A[j] = add2(make_float2(0.0f, 0.0f), P[0][j]);
        A[j] = add2(A[j], P[1][j]);
        A[j] = add2(A[j], P[2][j]);
        A[j] = add2(A[j], P[3][j]);
    }
    const float zero = __fmul_rn(tsum_finish(A, red, g), 0.0078125f);

    // unbiased std, ops_cpu.py:73 (fp64 sum of squares against the fp32 mean)
    const double md = (double)zero;
    double acc0 = 0.0, acc1 = 0.0;
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const double d0 = (double)P[c][j].x - md, d1 = (double)P[c][j].y - md;
            acc0 = fma(d0, d0, acc0);
            acc1 = fma(d1, d1, acc1);
        }
    double acc = acc0 + acc1;
    acc += __shfl_xor_sync(kFull, acc, 1);
    acc += __shfl_xor_sync(kFull, acc, 2);
    // the quotient by 127 and the square root are each within an ulp of
    // double; the midpoint test below is 1e-12 wide, far above that
    const double sd = sqrt(acc * (1.0 / 127.0));
    const float s32 = __double2float_rn(sd);
    bool fallback;
    {
        const double lo = (double)s32;
        const double nb = (double)(lo <= sd ? nextafterf(s32, INFINITY) : nextafterf(s32, 0.0f));
        const double mid = 0.5 * (lo + nb);
        fallback = fabs(sd - mid) <= 1e-12 * sd;
    }
    const float scale = __double2float_rn(__dadd_rn((double)s32, 1e-8));
    // non-finite inputs: the exact pass clamps the table index
    fallback = fallback || !(fabsf(scale) < INFINITY) || !(fabsf(zero) < INFINITY);
    if (__any_sync(kFull, fallback)) return false;
    const float rs = __frcp_rn(scale);

    // quantise, residual, syndrome.  |u| <= sqrt(127) (1 + 2^-20) for finite
    // inputs (every |x - zero| is at most sqrt(127) times the std against
    // that zero point), so the cell 8u + 96 lies in [6, 187) and the table
    // address needs no clamp.
    //   * The cell comes from the unrounded product (fma of d with 8/scale):
    //     it differs from the cell of u = RN(d/scale) only next to a cell
    //     boundary, where both cells give the same code because every
    //     threshold is >= 0.09 cells from a boundary.
    //   * w = RN(d * rs - thr) decides the side of the cell's threshold;
    //     |w| < kBandFast sends the warp to the exact pass.  m = sign mask of w
    //     picks code and centroid with integer ops (m = -1: below).
    //   * Codes are shifted into their word and sign bits of eps into
    //     `negs` (funnel shift) in descending element order, so nibble i
    //     and, after a byte reversal, bit 8c + i come out in place.  eps is
    //     never -0 here: a rotated element is never -0 (the quotient returns
    //     +0 for +-0), and eps = -0 needs x = -0; unrotated inputs use the
    //     comparison instead.
    const float2 nz2 = make_float2(-zero, -zero);
    const float rs8 = __fmul_rn(rs, 8.0f);  // exact
    const float2 rs82 = make_float2(rs8, rs8), mg2 = make_float2(kMagic + 96.0f, kMagic + 96.0f);
    const uint32_t tbase = tabq - (uint32_t)__float_as_int(kMagic) * (uint32_t)(kReplicas * sizeof(QEntry));
    uint32_t codes[4];
    uint32_t negs = 0u, bits = 0u;
    bool band = false;
    float2 AL[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) AL[j] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t cw = 0u;
#pragma unroll
        for (int j = 3; j >= 0; --j) {
            const float2 X = P[c][j];
            const float2 D = add2(X, nz2);
            const float2 T = fma2(D, rs82, mg2);
            const float4 e1 = lds_f4(tbase + (uint32_t)__float_as_int(T.y) * (uint32_t)(kReplicas * sizeof(QEntry)));
            const float4 e0 = lds_f4(tbase + (uint32_t)__float_as_int(T.x) * (uint32_t)(kReplicas * sizeof(QEntry)));
            const float w1 = __fmaf_rn(D.y, rs, -e1.x), w0 = __fmaf_rn(D.x, rs, -e0.x);
            band = band || (fabsf(w1) < kBandFast) || (fabsf(w0) < kBandFast);
            const uint32_t m1 = (uint32_t)(__float_as_int(w1) >> 31), m0 = (uint32_t)(__float_as_int(w0) >> 31);
            const float cq1 = __uint_as_float((__float_as_uint(e1.y) & m1) | (__float_as_uint(e1.z) & ~m1));
            const float cq0 = __uint_as_float((__float_as_uint(e0.y) & m0) | (__float_as_uint(e0.z) & ~m0));
            cw = (cw << 4) + ((uint32_t)__float_as_int(e1.w) + 1u + m1);
            cw = (cw << 4) + ((uint32_t)__float_as_int(e0.w) + 1u + m0);
            // k_tilde stays scalar: ptxas fuses a packed multiply followed by
            // a packed add into one fma2 (single rounding) even when both are
            // written as mul.rn/add.rn f32x2 PTX, and the reference rounds twice
            const float2 KT = make_float2(__fadd_rn(__fmul_rn(cq0, scale), zero),
                                          __fadd_rn(__fmul_rn(cq1, scale), zero));
            const float2 E = sub2(X, KT);
            if (kRotate) {
                negs = __funnelshift_l(__float_as_uint(E.y), negs, 1);
                negs = __funnelshift_l(__float_as_uint(E.x), negs, 1);
            } else {
                bits |= (E.x >= 0.0f ? 1u : 0u) << (8 * c + 2 * j);
                bits |= (E.y >= 0.0f ? 1u : 0u) << (8 * c + 2 * j + 1);
            }
            AL[j] = add2(AL[j], make_float2(fabsf(E.x), fabsf(E.y)));
        }
        codes[c] = cw;
    }
    if (kRotate) bits = ~__byte_perm(negs, 0u, 0x0123u);
    if (__any_sync(kFull, band)) return false;
    const float alpha = __fmul_rn(tsum_finish(AL, red, g), 0.0078125f);

    // stage: code word 4c+g and syndrome byte 4c+g of this vector
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        st[4 * c + g] = codes[c];
        reinterpret_cast<uint8_t *>(st + 16)[4 * c + g] = (uint8_t)(bits >> (8 * c));
    }
    __syncwarp();
    if (ref.valid) {
        const uint4 w0 = *reinterpret_cast<const uint4 *>(st + 4 * g);
        uint4 w1;
        if (g == 0) {
            w1 = *reinterpret_cast<const uint4 *>(st + 16);
        } else if (g == 1) {
            const uint32_t hs = __half_as_ushort(__float2half_rn(scale));
            const uint32_t hz = __half_as_ushort(__float2half_rn(zero));
            const uint32_t ha = __half_as_ushort(__float2half_rn(alpha));
            w1 = make_uint4(hs | (hz << 16), ha, 0u, 0u);
        } else {
            w1 = make_uint4(0u, 0u, 0u, 0u);
        }
        __stcs(reinterpret_cast<uint4 *>(ref.dst + 16 * g), w0);
        if (ref.tail) __stcs(reinterpret_cast<uint4 *>(ref.dst + 64 + 16 * g), w1);
    }
    __syncwarp();
    return true;
}

template <bool kRotate>
__global__ void __launch_bounds__(kCompressWarps * 32, 3) compress_kernel(const __grid_constant__ CompressJobs jobs) {
    __shared__ QEntry tab[kCells * kReplicas];
    __shared__ __align__(16) uint32_t stage[kCompressWarps][kVecPerWarp][20];
    __shared__ __align__(16) float reduce[kCompressWarps][kVecPerWarp][40];
    build_qtable(tab);
    __syncthreads();
    pdl_trigger();
    pdl_wait();  // the table set-up above touched shared memory only

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t *st = stage[warp][lane >> 2];
    float *red = reduce[warp][lane >> 2];
    const uint32_t tabq = (uint32_t)__cvta_generic_to_shared(tab + (lane & (kReplicas - 1)));
    const uint32_t t0 = jobs.j[0].n_tiles;
    const uint32_t n_tiles = t0 + (jobs.njobs > 1 ? jobs.j[1].n_tiles : 0u);
    int64_t off0, off1 = 0;
    const bool en0 = job_offset(jobs.j[0], off0);
    const bool en1 = jobs.njobs > 1 ? job_offset(jobs.j[1], off1) : true;
    // the next tile's inputs are loaded before the current tile is processed
    uint32_t tile = blockIdx.x;
    uint4 raw[4];
    VecRef ref;
    if (tile < n_tiles) {
        if (tile >= t0) load_vec(jobs.j[1], tile - t0, raw, ref, off1, en1);
        else load_vec(jobs.j[0], tile, raw, ref, off0, en0);
    }
    while (tile < n_tiles) {
        const uint32_t next = tile + gridDim.x;
        uint4 nraw[4];
        VecRef nref;
        if (next < n_tiles) {
            if (next >= t0) load_vec(jobs.j[1], next - t0, nraw, nref, off1, en1);
            else load_vec(jobs.j[0], next, nraw, nref, off0, en0);
        }
        if (!compress_fast<kRotate>(raw, ref, tabq, red, st)) {
            const bool second = tile >= t0;  // block-uniform
            const CompressJob &jb = second ? jobs.j[1] : jobs.j[0];
            const uint32_t t = second ? tile - t0 : tile;
            compress_warp_exact<kRotate>(jb.x, jb.xs_b, jb.xs_h, jb.xs_l, jb.blocks + (second ? off1 : off0), jb.bs_b,
                                         jb.bs_h, jb.div_h, jb.div_l, (second ? en1 : en0) ? jb.n_vec : 0u, t, tab,
                                         st, jb.rec);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) raw[c] = nraw[c];
        ref = nref;
        tile = next;
    }
}

// ---- small calls: one warp per vector ---------------------------------------
// A decode step appends one token per (sequence, kv head): a few hundred
// vectors, one or two tiles of compress_kernel, whose lanes each run the
// whole chain over 32 elements while the rest of the GPU idles; that chain
// sets the launch's duration.  Here a warp owns one vector and lane i holds
// elements i + 32m (m = 0..3): WHT strides 1..16 are lane exchanges, 32 and
// 64 stay in registers, lane 8a + l is torch's accumulator acc[a][l], the
// syndrome words are ballots and the block is one coalesced 128-byte store.
// Element by element the arithmetic is that of compress_warp (same quotient,
// sums, std, table and exact fallback), so the blocks are identical.
#ifndef ECC_COMPRESS_LATENCY_MAX
#define ECC_COMPRESS_LATENCY_MAX 4096
#endif
constexpr int64_t kLatencyMaxVectors = ECC_COMPRESS_LATENCY_MAX;  // calls up to this many vectors
constexpr int kLatWarps = 8;

// torch-order fp32 sum of the 128 elements spread as above; every lane gets it
__device__ __forceinline__ float tsum_warp(const float (&v)[4], int lane) {
    float acc = __fadd_rn(0.0f, v[0]);
    acc = __fadd_rn(acc, v[1]);
    acc = __fadd_rn(acc, v[2]);
    acc = __fadd_rn(acc, v[3]);
    const int l = lane & 7;
    const float a0 = __shfl_sync(kFull, acc, l), a1 = __shfl_sync(kFull, acc, l + 8);
    const float a2 = __shfl_sync(kFull, acc, l + 16), a3 = __shfl_sync(kFull, acc, l + 24);
    const float t = __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);  // t[l]
    float tk[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) tk[k] = __shfl_sync(kFull, t, k);
    float s = tk[0];
#pragma unroll
    for (int k = 1; k < 8; ++k) s = __fadd_rn(s, tk[k]);
    return s;
}

template <bool kRotate>
__global__ void __launch_bounds__(kLatWarps * 32) compress_lat_kernel(const __grid_constant__ CompressJobs jobs) {
    __shared__ QEntry tab[kCells * kReplicas];
    build_qtable(tab);
    __syncthreads();
    pdl_trigger();
    pdl_wait();  // the table set-up above touched shared memory only

    const int lane = threadIdx.x & 31;
    int64_t off0 = 0, off1 = 0;
    const bool en0 = job_offset(jobs.j[0], off0);
    const bool en1 = jobs.njobs > 1 ? job_offset(jobs.j[1], off1) : true;
    const uint32_t n0 = jobs.j[0].n_vec;
    const uint32_t n = n0 + (jobs.njobs > 1 ? jobs.j[1].n_vec : 0u);
    const uint32_t w = blockIdx.x * kLatWarps + (threadIdx.x >> 5);
    if (w >= n) return;  // warp-uniform
    const bool second = w >= n0;
    if (!(second ? en1 : en0)) return;
    const CompressJob &jb = second ? jobs.j[1] : jobs.j[0];
    const uint32_t vi = second ? w - n0 : w;
    const uint32_t row = fdiv(vi, jb.div_l);
    const int64_t l = vi - row * jb.div_l.d;
    const uint32_t bq = fdiv(row, jb.div_h);
    const int64_t b = bq, h = row - bq * jb.div_h.d;

    float v[4];
    {
        const __half *src = jb.x + b * jb.xs_b + h * jb.xs_h + l * jb.xs_l + lane;
#pragma unroll
        for (int m = 0; m < 4; ++m) v[m] = __half2float(src[32 * m]);
    }
    if (kRotate) {
#pragma unroll
        for (int s = 1; s < 32; s <<= 1) {  // strides 1..16: partner lane ^ s
            // lower index: mine + partner; upper index: partner - mine (an
            // FMA with multiplier +-1 rounds exactly like the add / sub)
            const float sgn = (lane & s) ? -1.0f : 1.0f;
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const float p = __shfl_xor_sync(kFull, v[m], s);
                v[m] = __fmaf_rn(sgn, v[m], p);
            }
        }
        float a = v[0], c = v[1];  // stride 32
        v[0] = __fadd_rn(a, c);
        v[1] = __fsub_rn(a, c);
        a = v[2];
        c = v[3];
        v[2] = __fadd_rn(a, c);
        v[3] = __fsub_rn(a, c);
        a = v[0];  // stride 64
        c = v[2];
        v[0] = __fadd_rn(a, c);
        v[2] = __fsub_rn(a, c);
        a = v[1];
        c = v[3];
        v[1] = __fadd_rn(a, c);
        v[3] = __fsub_rn(a, c);
#pragma unroll
        for (int m = 0; m < 4; ++m) {  // quotient by fp32(sqrt(128)), as in wht_group
            const float x = v[m];
            const float q0 = __fmul_rn(x, kInvSqrt128);
            const float rem = __fmaf_rn(-q0, kSqrt128, x);
            v[m] = fabsf(q0) == INFINITY ? q0 : __fmaf_rn(rem, kInvSqrt128, q0);
        }
    }

    const float zero = __fmul_rn(tsum_warp(v, lane), 0.0078125f);  // ops_cpu.py:72

    // unbiased std (ops_cpu.py:73): fp64 tree sum; near an fp32 rounding
    // midpoint the sum is redone in element order like the CPU
    const double md = (double)zero;
    double acc = 0.0;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const double dx = (double)v[m] - md;
        acc = fma(dx, dx, acc);
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) acc += __shfl_xor_sync(kFull, acc, o);
    double sd = __dsqrt_rn(__ddiv_rn(acc, 127.0));
    float s32 = __double2float_rn(sd);
    {
        const double lo = (double)s32;
        const double nb = (double)(lo <= sd ? nextafterf(s32, INFINITY) : nextafterf(s32, 0.0f));
        const double mid = 0.5 * (lo + nb);
        if (__any_sync(kFull, fabs(sd - mid) <= 1e-12 * sd)) {
            double ex = 0.0;
#pragma unroll
            for (int m = 0; m < 4; ++m)
#pragma unroll 1
                for (int k = 0; k < 32; ++k) {
                    const float xv = __shfl_sync(kFull, v[m], k);
                    const double dx = __dsub_rn((double)xv, md);
                    ex = __dadd_rn(ex, __dmul_rn(dx, dx));
                }
            sd = __dsqrt_rn(__ddiv_rn(ex, 127.0));
            s32 = __double2float_rn(sd);
        }
    }
    const float scale = __double2float_rn(__dadd_rn((double)s32, 1e-8));
    const float rs = __frcp_rn(scale);

    // quantise, residual, syndrome
    const QEntry *mytab = tab + (lane & (kReplicas - 1));
    uint32_t cw[4], syn[4];
    float ab[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const float xv = v[m];
        const float d = __fsub_rn(xv, zero);
        const float u = __fmul_rn(d, rs);
        const unsigned cell = min((unsigned)cell_of(u), (unsigned)(kCells - 1));
        const QEntry e = mytab[cell * kReplicas];
        const bool hi = u > e.thr;
        float cq = hi ? e.c_hi : e.c_lo;
        int q = e.q_lo + (hi ? 1 : 0);
        if (fabsf(__fsub_rn(u, e.thr)) < kBand) {
            q = exact_code(d, scale);
            cq = lm(0);
#pragma unroll
            for (int k = 1; k < 16; ++k) cq = (q == k) ? lm(k) : cq;
        }
        const float kt = __fadd_rn(__fmul_rn(cq, scale), zero);
        const float eps = __fsub_rn(xv, kt);
        syn[m] = __ballot_sync(kFull, eps >= 0.0f);  // syndrome word m: elements 32m..32m+31
        ab[m] = fabsf(eps);
        // code word 4m + lane/8 (elements 8(4m + lane/8) + 0..7, nibble lane % 8)
        uint32_t x = (uint32_t)q << (4 * (lane & 7));
        x |= __shfl_xor_sync(kFull, x, 1);
        x |= __shfl_xor_sync(kFull, x, 2);
        x |= __shfl_xor_sync(kFull, x, 4);
        cw[m] = x;
    }
    const float alpha = __fmul_rn(tsum_warp(ab, lane), 0.0078125f);

    // lane i writes word i of the block: codes 0..15, syndrome 16..19,
    // scale | zero << 16, alpha, zeros
    const int src = 8 * (lane & 3);
    const uint32_t c0 = __shfl_sync(kFull, cw[0], src), c1 = __shfl_sync(kFull, cw[1], src);
    const uint32_t c2 = __shfl_sync(kFull, cw[2], src), c3 = __shfl_sync(kFull, cw[3], src);
    uint32_t word = 0u;
    if (lane < 16) {
        const int m = lane >> 2;
        word = m == 0 ? c0 : m == 1 ? c1 : m == 2 ? c2 : c3;
    } else if (lane < 20) {
        const int m = lane - 16;
        word = m == 0 ? syn[0] : m == 1 ? syn[1] : m == 2 ? syn[2] : syn[3];
    } else if (lane == 20) {
        word = (uint32_t)__half_as_ushort(__float2half_rn(scale)) |
               ((uint32_t)__half_as_ushort(__float2half_rn(zero)) << 16);
    } else if (lane == 21) {
        word = (uint32_t)__half_as_ushort(__float2half_rn(alpha));
    }
    uint8_t *dst = jb.blocks + (second ? off1 : off0) + (b * jb.bs_b + h * jb.bs_h + l) * jb.rec;
    if (4 * lane < (int)jb.rec) reinterpret_cast<uint32_t *>(dst)[lane] = word;
}

// ---- calibrated compress ---------------------------------------------------
// Fixed quantiser parameters instead of per-vector statistics: the per-layer
// scale, zero point and alpha of a calibration config (custom_kv/calibration.py
// :232-237 computes them; the quantiser is ops_cpu.lloyd_max_quantize_cpu,
// ops_cpu.py:78-109, called with those scalars).  Per element:
// d = RN(x - zero), q = first-index argmin_k |RN(d / scale) - C[k]|,
// k~ = RN(RN(C[q] * scale) + zero), bit = (x - k~ >= 0); every block stores
// fp16 of the fp32 scale, zero and alpha.  |d / scale| is unbounded here, so
// the table cell is clamped (the end cells hold no threshold); an element
// within kBand of a threshold, or non-finite, takes the IEEE quotient and the
// full argmin.  Scalar code: this path is an option, not the hot path.
struct CalParams {
    float scale, zero, alpha, rs;  // rs = RN(1 / scale)
};

template <bool kRotate>
__global__ void __launch_bounds__(kCompressWarps * 32, 3)
    compress_cal_kernel(const __grid_constant__ CompressJob jb, const CalParams cp) {
    __shared__ QEntry tab[kCells * kReplicas];
    __shared__ __align__(16) uint32_t stage[kCompressWarps][kVecPerWarp][20];
    build_qtable(tab);
    __syncthreads();
    pdl_trigger();
    pdl_wait();

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane & 3;
    uint32_t *st = stage[warp][lane >> 2];
    const QEntry *mytab = tab + (lane & (kReplicas - 1));
    int64_t off;
    const bool en = job_offset(jb, off);
    for (uint32_t tile = blockIdx.x; tile < jb.n_tiles; tile += gridDim.x) {
        uint4 raw[4];
        VecRef ref;
        load_vec(jb, tile, raw, ref, off, en);
        float v[4][8];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t w[4] = {raw[c].x, raw[c].y, raw[c].z, raw[c].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = h2_to_f2(w[j]);
                v[c][2 * j] = f.x;
                v[c][2 * j + 1] = f.y;
            }
        }
        if (kRotate) wht_group(v, g);
        uint32_t codes[4] = {0u, 0u, 0u, 0u};
        uint32_t bits = 0u;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float xv = v[c][i];
                const float d = __fsub_rn(xv, cp.zero);
                const float u = __fmul_rn(d, cp.rs);
                // nearest cell, clamped; NaN lands in cell 0 (no threshold, NaN test below)
                const int cell = (int)fminf(fmaxf(rintf(__fmaf_rn(u, 8.0f, 96.0f)), 0.0f), (float)(kCells - 1));
                const QEntry e = mytab[cell * kReplicas];
                int q;
                float cq;
                if (!(fabsf(__fsub_rn(u, e.thr)) >= kBand)) {  // near a threshold, or u not finite
                    q = exact_code(d, cp.scale);
                    cq = lm(0);
#pragma unroll
                    for (int k = 1; k < 16; ++k) cq = (q == k) ? lm(k) : cq;
                } else {
                    const bool hi = u > e.thr;
                    q = e.q_lo + (hi ? 1 : 0);
                    cq = hi ? e.c_hi : e.c_lo;
                }
                const float kt = __fadd_rn(__fmul_rn(cq, cp.scale), cp.zero);
                bits |= (__fsub_rn(xv, kt) >= 0.0f ? 1u : 0u) << (8 * c + i);
                codes[c] |= (uint32_t)q << (4 * i);
            }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            st[4 * c + g] = codes[c];
            reinterpret_cast<uint8_t *>(st + 16)[4 * c + g] = (uint8_t)(bits >> (8 * c));
        }
        __syncwarp();
        if (ref.valid) {
            const uint4 w0 = *reinterpret_cast<const uint4 *>(st + 4 * g);
            uint4 w1 = make_uint4(0u, 0u, 0u, 0u);
            if (g == 0) {
                w1 = *reinterpret_cast<const uint4 *>(st + 16);
            } else if (g == 1) {
                const uint32_t hs = __half_as_ushort(__float2half_rn(cp.scale));
                const uint32_t hz = __half_as_ushort(__float2half_rn(cp.zero));
                const uint32_t ha = __half_as_ushort(__float2half_rn(cp.alpha));
                w1 = make_uint4(hs | (hz << 16), ha, 0u, 0u);
            }
            __stcs(reinterpret_cast<uint4 *>(ref.dst + 16 * g), w0);
            if (ref.tail) __stcs(reinterpret_cast<uint4 *>(ref.dst + 64 + 16 * g), w1);
        }
        __syncwarp();
    }
}

// ---- generic WHT (any power of two d <= 1024), one CTA per row ------------
template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

template <typename T>
__global__ void hadamard_generic_kernel(T *__restrict__ x, int d, float norm) {
    extern __shared__ float sh[];
    T *row = x + (int64_t)blockIdx.x * d;
    for (int j = threadIdx.x; j < d; j += blockDim.x) sh[j] = to_f<T>(row[j]);
    __syncthreads();
    for (int s = 1; s < d; s <<= 1) {
        for (int p = threadIdx.x; p < d / 2; p += blockDim.x) {
            const int lo = (p / s) * 2 * s + (p % s);
            const float a = sh[lo], b = sh[lo + s];
            sh[lo] = __fadd_rn(a, b);
            sh[lo + s] = __fsub_rn(a, b);
        }
        __syncthreads();
    }
    for (int j = threadIdx.x; j < d; j += blockDim.x) row[j] = from_f<T>(__fdiv_rn(sh[j], norm));
}

// D = 128 fast path: 4 lanes per row, same arithmetic as the compress prologue.
template <typename T>
__global__ void __launch_bounds__(256) hadamard128_kernel(T *__restrict__ x, int64_t n) {
    const int lane = threadIdx.x & 31;
    const int g = lane & 3;
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 2;
    const bool valid = r < n;
    T *row = x + r * kD;
    float v[4][8];
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] = valid ? to_f<T>(row[32 * c + 8 * g + i]) : 0.0f;
    wht_group(v, g);
    if (valid) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 8; ++i) row[32 * c + 8 * g + i] = from_f<T>(v[c][i]);
    }
}

// ---- dequantise: blocks -> fp16 reconstruction ---------------------------
__global__ void dequant_kernel(const uint8_t *__restrict__ blocks, __half *__restrict__ out, int64_t n) {
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= n) return;
    const uint8_t *blk = blocks + r * kBlockBytes;
    const uint32_t code16 = *reinterpret_cast<const uint16_t *>(blk + 2 * lane);
    const uint32_t syn = (blk[kSynOff + lane / 2] >> (4 * (lane & 1))) & 0xfu;
    const float sc = __half2float(*reinterpret_cast<const __half *>(blk + kScaleOff));
    const float zr = __half2float(*reinterpret_cast<const __half *>(blk + kZeroOff));
    const float al = __half2float(*reinterpret_cast<const __half *>(blk + kAlphaOff));
    __half o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int q = (code16 >> (4 * j)) & 0xf;
        float c = lm(0);
#pragma unroll
        for (int k = 1; k < 16; ++k) c = (q == k) ? lm(k) : c;
        const float kt = __fadd_rn(__fmul_rn(c, sc), zr);
        const float s = ((syn >> j) & 1u) ? al : -al;
        o[j] = __float2half_rn(__fadd_rn(kt, s));
    }
    *reinterpret_cast<uint2 *>(out + r * kD + 4 * lane) = *reinterpret_cast<uint2 *>(o);
}

// ---- SoA trio -> blocks ---------------------------------------------------
__global__ void pack_soa_kernel(const uint8_t *__restrict__ int4, int64_t i4s, const uint8_t *__restrict__ syn,
                                int64_t sys, const uint8_t *__restrict__ meta, int64_t ms,
                                uint8_t *__restrict__ blocks, int64_t n) {
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= n) return;
    uint8_t *dst = blocks + r * kBlockBytes;
    // lanes 0..15 copy 4 code bytes each, 16..19 syndrome, 20..21 meta, rest zero
    uint32_t w = 0;
    const int off = 4 * lane;
    if (lane < 16) {
        const uint8_t *s = int4 + r * i4s + off;
        w = s[0] | (s[1] << 8) | (s[2] << 16) | ((uint32_t)s[3] << 24);
    } else if (lane < 20) {
        const uint8_t *s = syn + r * sys + (off - 64);
        w = s[0] | (s[1] << 8) | (s[2] << 16) | ((uint32_t)s[3] << 24);
    } else if (lane == 20) {
        const uint8_t *s = meta + r * ms;
        w = s[0] | (s[1] << 8) | (s[2] << 16) | ((uint32_t)s[3] << 24);
    } else if (lane == 21) {
        const uint8_t *s = meta + r * ms + 4;
        w = s[0] | (s[1] << 8);
    }
    reinterpret_cast<uint32_t *>(dst)[lane] = w;
}

// ---- host side ------------------------------------------------------------
struct DevInfo {
    int sms = 0;
    int compress_ctas_per_sm[2] = {0, 0};
};

static DevInfo g_dev[64];
static std::mutex g_dev_mu;

static int dev_info(DevInfo **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ECC_ERR_DEVICE;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DevInfo &di = g_dev[dev];
    if (di.sms == 0) {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return ECC_ERR_DEVICE;
        int a = 0, b = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&a, compress_kernel<false>, kCompressWarps * 32, 0);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, compress_kernel<true>, kCompressWarps * 32, 0);
        di.compress_ctas_per_sm[0] = std::max(a, 1);
        di.compress_ctas_per_sm[1] = std::max(b, 1);
        di.sms = sms;
    }
    *out = &di;
    return ECC_OK;
}

int launch_status() {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? ECC_OK : ECC_ERR_LAUNCH;
}

int sm_count() {
    DevInfo *di = nullptr;
    const int rc = dev_info(&di);
    return rc == ECC_OK ? di->sms : 148;
}

}  // namespace ecc

using namespace ecc;

static inline bool aligned(const void *p, size_t a) { return ((uintptr_t)p % a) == 0; }

// Validates one strided compress request and fills its job; *n_out = vectors.
// mode: the entry points' `rotate` argument (ECC_COMPRESS_* bits).
static int make_job(const void *x_f16, int64_t xs_b, int64_t xs_h, int64_t xs_l, void *blocks, int64_t bs_b,
                    int64_t bs_h, int B, int H, int64_t L, int mode, CompressJob *jb, int64_t *n_out) {
    *n_out = 0;
    if (mode & ~(ECC_COMPRESS_ROTATE | ECC_COMPRESS_BLOCK96)) return ECC_ERR_SHAPE;
    jb->rec = (mode & ECC_COMPRESS_BLOCK96) ? 96u : (uint32_t)kBlockBytes;
    if (B < 0 || H < 0 || L < 0) return ECC_ERR_SHAPE;
    const int64_t n = (int64_t)B * H * L;
    *n_out = n;
    if (n == 0) return ECC_OK;
    if (n >= (int64_t)0xffffff00ll) return ECC_ERR_SHAPE;  // 32-bit vector index
    if (!x_f16 || !blocks) return ECC_ERR_NULL;
    // 128-byte blocks start on 128-byte boundaries; 96-byte records on 32-byte ones
    if (!aligned(x_f16, 16) || !aligned(blocks, jb->rec == 96u ? 32 : 128)) return ECC_ERR_ALIGN;
    if ((xs_b % 8) || (xs_h % 8) || (xs_l % 8)) return ECC_ERR_ALIGN;
    jb->x = reinterpret_cast<const __half *>(x_f16);
    jb->xs_b = xs_b;
    jb->xs_h = xs_h;
    jb->xs_l = xs_l;
    jb->blocks = reinterpret_cast<uint8_t *>(blocks);
    jb->bs_b = bs_b;
    jb->bs_h = bs_h;
    jb->div_h = make_fastdiv((uint32_t)std::max(H, 1));
    jb->div_l = make_fastdiv((uint32_t)std::max<int64_t>(L, 1));
    jb->n_vec = (uint32_t)n;
    jb->n_tiles = (uint32_t)((n + kVecPerTile - 1) / kVecPerTile);
    return ECC_OK;
}

static int launch_jobs(CompressJobs &jobs, int mode, ecc_stream_t stream) {
    const bool rotate = (mode & ECC_COMPRESS_ROTATE) != 0;
    // drop empty jobs
    if (jobs.njobs > 1 && jobs.j[1].n_vec == 0) jobs.njobs = 1;
    if (jobs.njobs > 0 && jobs.j[0].n_vec == 0) {
        jobs.j[0] = jobs.j[1];
        jobs.njobs -= 1;
    }
    if (jobs.njobs == 0) return ECC_OK;
    DevInfo *di = nullptr;
    const int rc = dev_info(&di);
    if (rc != ECC_OK) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int64_t nvec = (int64_t)jobs.j[0].n_vec + (jobs.njobs > 1 ? jobs.j[1].n_vec : 0);
    if (nvec <= kLatencyMaxVectors) {  // appends: one warp per vector
        const dim3 grid((unsigned)((nvec + kLatWarps - 1) / kLatWarps)), block(kLatWarps * 32);
        const cudaError_t e = rotate ? launch_pdl(compress_lat_kernel<true>, grid, block, 0, s, jobs)
                                     : launch_pdl(compress_lat_kernel<false>, grid, block, 0, s, jobs);
        if (e != cudaSuccess) return ECC_ERR_LAUNCH;
        return launch_status();
    }
    const int64_t tiles = (int64_t)jobs.j[0].n_tiles + (jobs.njobs > 1 ? jobs.j[1].n_tiles : 0);
    if (tiles >= (int64_t)0xffffff00ll) return ECC_ERR_SHAPE;
    const int64_t grid = std::min<int64_t>(tiles, (int64_t)di->sms * di->compress_ctas_per_sm[rotate ? 1 : 0]);
    const cudaError_t e = rotate ? launch_pdl(compress_kernel<true>, dim3((unsigned)grid), dim3(kCompressWarps * 32),
                                              0, s, jobs)
                                 : launch_pdl(compress_kernel<false>, dim3((unsigned)grid),
                                              dim3(kCompressWarps * 32), 0, s, jobs);
    if (e != cudaSuccess) return ECC_ERR_LAUNCH;
    return launch_status();
}

extern "C" int ecc_compress_strided(const void *x_f16, int64_t xs_b, int64_t xs_h, int64_t xs_l, void *blocks,
                                    int64_t bs_b, int64_t bs_h, int B, int H, int64_t L, int rotate,
                                    ecc_stream_t stream) {
    CompressJobs jobs{};
    int64_t n = 0;
    const int rc = make_job(x_f16, xs_b, xs_h, xs_l, blocks, bs_b, bs_h, B, H, L, rotate, &jobs.j[0], &n);
    if (rc != ECC_OK || n == 0) return rc;
    jobs.njobs = 1;
    return launch_jobs(jobs, rotate, stream);
}

extern "C" int ecc_compress_strided_pair(const void *x0_f16, int64_t x0s_b, int64_t x0s_h, int64_t x0s_l,
                                         void *blocks0, int64_t b0s_b, int64_t b0s_h, const void *x1_f16,
                                         int64_t x1s_b, int64_t x1s_h, int64_t x1s_l, void *blocks1, int64_t b1s_b,
                                         int64_t b1s_h, int B, int H, int64_t L, int rotate, ecc_stream_t stream) {
    CompressJobs jobs{};
    int64_t n0 = 0, n1 = 0;
    int rc = make_job(x0_f16, x0s_b, x0s_h, x0s_l, blocks0, b0s_b, b0s_h, B, H, L, rotate, &jobs.j[0], &n0);
    if (rc != ECC_OK) return rc;
    rc = make_job(x1_f16, x1s_b, x1s_h, x1s_l, blocks1, b1s_b, b1s_h, B, H, L, rotate, &jobs.j[1], &n1);
    if (rc != ECC_OK) return rc;
    if (n0 == 0) return ECC_OK;
    jobs.njobs = 2;
    return launch_jobs(jobs, rotate, stream);
}

static int compress_calibrated_impl(const void *x_f16, int64_t xs_b, int64_t xs_h, int64_t xs_l, void *blocks,
                                    int64_t bs_b, int64_t bs_h, int B, int H, int64_t L, int rotate, float scale,
                                    float zero, float alpha, const int *pos_dev, int64_t capacity,
                                    ecc_stream_t stream) {
    if (!(scale > 0.0f) || !std::isfinite(scale) || !std::isfinite(zero) || !std::isfinite(alpha))
        return ECC_ERR_PARAM;
    CompressJob jb{};
    int64_t n = 0;
    int rc = make_job(x_f16, xs_b, xs_h, xs_l, blocks, bs_b, bs_h, B, H, L, rotate, &jb, &n);
    if (rc != ECC_OK || n == 0) return rc;
    jb.pos_dev = pos_dev;
    jb.cap = capacity;
    DevInfo *di = nullptr;
    rc = dev_info(&di);
    if (rc != ECC_OK) return rc;
    const float rs = 1.0f / scale;  // IEEE single division: RN(1 / scale)
    if (!std::isfinite(rs)) return ECC_ERR_PARAM;
    const CalParams cp{scale, zero, alpha, rs};
    const int64_t grid = std::min<int64_t>(jb.n_tiles, (int64_t)di->sms * 3);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const cudaError_t e =
        (rotate & ECC_COMPRESS_ROTATE) ? launch_pdl(compress_cal_kernel<true>, dim3((unsigned)grid), dim3(kCompressWarps * 32), 0, s, jb, cp)
               : launch_pdl(compress_cal_kernel<false>, dim3((unsigned)grid), dim3(kCompressWarps * 32), 0, s, jb, cp);
    if (e != cudaSuccess) return ECC_ERR_LAUNCH;
    return launch_status();
}

extern "C" int ecc_compress_strided_calibrated(const void *x_f16, int64_t xs_b, int64_t xs_h, int64_t xs_l,
                                               void *blocks, int64_t bs_b, int64_t bs_h, int B, int H, int64_t L,
                                               int rotate, float scale, float zero, float alpha,
                                               ecc_stream_t stream) {
    return compress_calibrated_impl(x_f16, xs_b, xs_h, xs_l, blocks, bs_b, bs_h, B, H, L, rotate, scale, zero, alpha,
                                    nullptr, 0, stream);
}

// Device-side positions: the destination token offset is read from
// *pos_dev when the kernel runs, so one recorded launch serves every step of
// a growing cache (CUDA graph replay).  blocks point at token 0 of the pools.
static int at_checks(const int *pos_dev, int64_t capacity, int64_t L) {
    if (!pos_dev) return ECC_ERR_NULL;
    if (!aligned(pos_dev, 4)) return ECC_ERR_ALIGN;
    if (L < 1 || capacity < L) return ECC_ERR_SHAPE;
    return ECC_OK;
}

extern "C" int ecc_compress_strided_pair_at(const void *x0_f16, int64_t x0s_b, int64_t x0s_h, int64_t x0s_l,
                                            void *blocks0, int64_t b0s_b, int64_t b0s_h, const void *x1_f16,
                                            int64_t x1s_b, int64_t x1s_h, int64_t x1s_l, void *blocks1,
                                            int64_t b1s_b, int64_t b1s_h, int B, int H, int64_t L,
                                            int64_t capacity, const int *pos_dev, int rotate, ecc_stream_t stream) {
    int rc = at_checks(pos_dev, capacity, L);
    if (rc != ECC_OK) return rc;
    CompressJobs jobs{};
    int64_t n0 = 0, n1 = 0;
    rc = make_job(x0_f16, x0s_b, x0s_h, x0s_l, blocks0, b0s_b, b0s_h, B, H, L, rotate, &jobs.j[0], &n0);
    if (rc != ECC_OK) return rc;
    jobs.njobs = 1;
    if (x1_f16 || blocks1) {
        rc = make_job(x1_f16, x1s_b, x1s_h, x1s_l, blocks1, b1s_b, b1s_h, B, H, L, rotate, &jobs.j[1], &n1);
        if (rc != ECC_OK) return rc;
        jobs.njobs = 2;
    }
    if (n0 == 0) return ECC_OK;
    for (int k = 0; k < jobs.njobs; ++k) {
        jobs.j[k].pos_dev = pos_dev;
        jobs.j[k].cap = capacity;
    }
    return launch_jobs(jobs, rotate, stream);
}

extern "C" int ecc_compress_strided_calibrated_at(const void *x_f16, int64_t xs_b, int64_t xs_h, int64_t xs_l,
                                                  void *blocks, int64_t bs_b, int64_t bs_h, int B, int H, int64_t L,
                                                  int64_t capacity, const int *pos_dev, int rotate, float scale,
                                                  float zero, float alpha, ecc_stream_t stream) {
    int rc = at_checks(pos_dev, capacity, L);
    if (rc != ECC_OK) return rc;
    return compress_calibrated_impl(x_f16, xs_b, xs_h, xs_l, blocks, bs_b, bs_h, B, H, L, rotate, scale, zero, alpha,
                                    pos_dev, capacity, stream);
}

namespace ecc {
int compress_device_error(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_compress_error, sizeof(int)) != cudaSuccess) return ECC_ERR_CUDA;
    if (reset) {
        const int z = 0;
        if (cudaMemcpyToSymbol(g_compress_error, &z, sizeof(int)) != cudaSuccess) return ECC_ERR_CUDA;
    }
    return v;
}
}  // namespace ecc

extern "C" int ecc_compress(const void *x_f16, void *blocks, int64_t n, int rotate, ecc_stream_t stream) {
    if (n < 0) return ECC_ERR_SHAPE;
    return ecc_compress_strided(x_f16, 0, 0, kD, blocks, 0, 0, 1, 1, n, rotate, stream);
}

template <typename T>
static int hadamard_impl(void *x, int64_t n, int d, ecc_stream_t stream) {
    if (n < 0 || d < 1 || d > 1024 || (d & (d - 1))) return ECC_ERR_SHAPE;
    if (n == 0) return ECC_OK;
    if (!x) return ECC_ERR_NULL;
    if (!aligned(x, sizeof(T))) return ECC_ERR_ALIGN;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (d == kD) {
        const int64_t threads = n * 4;
        hadamard128_kernel<T><<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(reinterpret_cast<T *>(x), n);
    } else {
        if (n > 0x7fffffff) return ECC_ERR_SHAPE;
        const float norm = (float)std::sqrt((double)d);
        const int threads = std::min(std::max(d / 2, 32), 512);
        hadamard_generic_kernel<T><<<(unsigned)n, threads, d * sizeof(float), s>>>(reinterpret_cast<T *>(x), d, norm);
    }
    return launch_status();
}

extern "C" int ecc_hadamard_f16(void *x, int64_t n, int d, ecc_stream_t stream) {
    return hadamard_impl<__half>(x, n, d, stream);
}

extern "C" int ecc_hadamard_f32(void *x, int64_t n, int d, ecc_stream_t stream) {
    return hadamard_impl<float>(x, n, d, stream);
}

extern "C" int ecc_get_block_metadata(const void *blocks, int64_t n_blocks, int64_t block_idx, float *host_out3,
                                      ecc_stream_t stream) {
    if (!blocks || !host_out3) return ECC_ERR_NULL;
    if (block_idx < 0 || block_idx >= n_blocks) return ECC_ERR_SHAPE;
    __half h[3];
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const uint8_t *src = reinterpret_cast<const uint8_t *>(blocks) + block_idx * kBlockBytes + kScaleOff;
    if (cudaMemcpyAsync(h, src, sizeof(h), cudaMemcpyDeviceToHost, s) != cudaSuccess) return ECC_ERR_CUDA;
    if (cudaStreamSynchronize(s) != cudaSuccess) return ECC_ERR_CUDA;
    for (int i = 0; i < 3; ++i) host_out3[i] = __half2float(h[i]);
    return ECC_OK;
}

extern "C" int ecc_dequantize(const void *blocks, void *out_f16, int64_t n, ecc_stream_t stream) {
    if (n < 0) return ECC_ERR_SHAPE;
    if (n == 0) return ECC_OK;
    if (!blocks || !out_f16) return ECC_ERR_NULL;
    if (!aligned(blocks, 16) || !aligned(out_f16, 8)) return ECC_ERR_ALIGN;
    const int64_t threads = n * 32;
    dequant_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint8_t *>(blocks), reinterpret_cast<__half *>(out_f16), n);
    return launch_status();
}

extern "C" int ecc_pack_soa(const void *int4, int64_t int4_row_bytes, const void *syn, int64_t syn_row_bytes,
                            const void *meta, int64_t meta_row_bytes, void *blocks, int64_t n, ecc_stream_t stream) {
    if (n < 0) return ECC_ERR_SHAPE;
    if (n == 0) return ECC_OK;
    if (!int4 || !syn || !meta || !blocks) return ECC_ERR_NULL;
    if (!aligned(blocks, 128)) return ECC_ERR_ALIGN;
    const int64_t threads = n * 32;
    pack_soa_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint8_t *>(int4), int4_row_bytes, reinterpret_cast<const uint8_t *>(syn),
        syn_row_bytes, reinterpret_cast<const uint8_t *>(meta), meta_row_bytes, reinterpret_cast<uint8_t *>(blocks), n);
    return launch_status();
}

extern "C" const char *ecc_strerror(int code) {
    switch (code) {
        case ECC_OK: return "ok";
        case ECC_ERR_NULL: return "null pointer";
        case ECC_ERR_SHAPE: return "size out of range";
        case ECC_ERR_ALIGN: return "misaligned pointer or stride";
        case ECC_ERR_GQA: return "query heads not a multiple of kv heads";
        case ECC_ERR_WORKSPACE: return "workspace missing or too small";
        case ECC_ERR_LAUNCH: return "kernel launch failed";
        case ECC_ERR_CUDA: return "CUDA runtime call failed";
        case ECC_ERR_DEVICE: return "no usable CUDA device";
        case ECC_ERR_SCRATCH_LIMIT: return "request exceeds the library's static decode scratch";
        case ECC_ERR_PARAM: return "quantiser parameter not finite or scale not positive";
        default: return "unknown error";
    }
}

extern "C" int ecc_version(void) { return 100; }
