// decode_mma.cu -- tensor-core split-KV decode attention over 128-byte blocks
// for GQA groups of up to 8 query heads per KV head (sm_100a, mma.sync).
//
// Per (b, kv head, split) CTA, each warp streams 16-token tiles:
//
//   S  = Q_g . K^T  as three m16n8k16 products per 16-dim step (M = 16 tokens,
//        N = 8 query heads, K = dims):  C_hi(codes), C_lo(codes) and the +-1
//        syndrome signs, so  score = sm * (scale*(q.C) + alpha*(q.s) + zero*sum q)
//        (the decomposition of custom_kv/ops_cpu.py:140-184 with the k_tilde
//        of fused_decode.py:229-241);
//   O += V^T . P    as three products per 16-dim m-tile (M = 16 dims, N = 8
//        heads, K = 16 tokens) with B = p*v_scale for the centroid terms and
//        B = p*v_alpha for the signs; sum p*v_zero is added at the end.
//
// Centroids enter the tensor cores as two fp16 numbers C_hi + C_lo (C_hi =
// fp16(C), C_lo = fp16(C - C_hi)), so the 16-entry fp32 table is represented
// to ~1e-7; a single fp16 copy of the table gives up to 4.6e-3 output error
// on the heavy-outlier single-layer test.  Codes become operands through a
// shared-memory table indexed by one code byte (two nibbles -> a pair of
// fp16 values), replicated per lane so that the 32 lanes of a warp always hit
// 32 different banks; the byte offset of an entry is built with one prmt.
//
// Fragment layouts follow the PTX ISA m16n8k16 .f16 description: lane = 4*g+c
// (groupID g, thread-in-group c); A {a0a1}=(row g, cols 2c..), {a2a3}=(row
// g+8), {a4a5}=(row g, cols 2c+8..), {a6a7}=(row g+8, cols 2c+8..); B {b0b1}=
// (rows 2c.., col g), {b2b3}=(rows 2c+8.., col g); C c0c1=(row g, cols 2c..),
// c2c3=(row g+8).  The K dimension of a product may be any permutation of the
// summed index as long as A and B use the same one; the mappings used are:
//   QK centroid steps m=0..7: k-col 2c+e <-> dim 32c+4m+e, 2c+8+e <-> 32c+4m+2+e
//     (lane c reads code bytes 16c..16c+15 of tokens g and g+8);
//   QK sign steps m=0..7:     k-col 2c+e <-> dim 32c+2m+16e, 2c+8+e <-> 32c+2m+1+16e
//     (syndrome word c of tokens g, g+8; bit p moved to bit 15 by a shift);
//   PV m-tile i=0..7: row g <-> dim 16g+2i, row g+8 <-> dim 16g+2i+1; k-cols =
//     tokens 2c, 2c+1, 2c+8, 2c+9 of the tile (pairs of tokens share one code
//     byte index built from their two code words).
#include <algorithm>
#include <cmath>

#include "ecc_common.cuh"

namespace ecc {

constexpr int kMmaWarps = 4;
constexpr int kTileTok = 16;
constexpr int kLutBytes = 256 * 256;  // 256 code bytes x 32 lanes x 8 B, row stride 256 B
constexpr float kLn2f = 0.6931471805599453f;

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// Table entry (code byte v, lane) -> {C_hi[v&15] | C_hi[v>>4] << 16, C_lo[...] pair}.
// `tab` is the 32-bit shared-window address of the table; the entry offset
// v*256 + lane*8 is assembled by one prmt from byte `byte_idx` of `word` and
// lane8 = lane*8 (< 256).
__device__ __forceinline__ uint2 lut(uint32_t tab, uint32_t word, int byte_idx, uint32_t lane8) {
    const uint32_t off = __byte_perm(word, lane8, 0x5504u | ((uint32_t)byte_idx << 4));
    uint2 r;
    asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(tab + off));
    return r;
}

// 2^x (MUFU.EX2, ~2 ulp; flushes results below 2^-126 to 0, which the
// softmax weights tolerate).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// +-1 pair from bits p and p+16 of w (bit 1 -> +1.0, bit 0 -> -1.0).
__device__ __forceinline__ uint32_t sign_pair(uint32_t w, int p) {
    const uint32_t x = w << (15 - p);
    return (~x & 0x80008000u) | 0x3C003C00u;
}

__device__ __forceinline__ float h_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu))); }
__device__ __forceinline__ float h_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }



constexpr int kQRow = kD + 1;  // padded query row (conflict-free fragment reads)

// Per-lane state of one warp streaming 16-token tiles of one (b, kv head).
struct TileLane {
    uint32_t qc[8][2];  // B fragments of Q for the centroid products
    uint32_t qs[8][2];  // B fragments of Q for the sign products
    float qsum[2];      // sum of the query of heads 2c, 2c+1
    float o[8][4];      // O accumulators: m-tile i, (dim 16g+2i(+1), head 2c(+1))
    float mrun[2], lrun[2], zrun[2];
    uint32_t tab, lane8, sel_half;
    int g, c;
    int koff_c, koff_s, koff_m, voff_c, voff_s;  // byte offsets inside a tile
    float scale_log2;

    template <bool kFull>
    __device__ __forceinline__ void tile(const uint8_t *__restrict__ kt, const uint8_t *__restrict__ vt,
                                         int nvalid) {
        // ---------------- loads ----------------
        const bool va = kFull || g < nvalid, vb8 = kFull || g + 8 < nvalid;
        uint4 kca = make_uint4(0, 0, 0, 0), kcb = make_uint4(0, 0, 0, 0);
        uint32_t ksa = 0, ksb = 0;
        uint2 kma = make_uint2(0, 0), kmb = make_uint2(0, 0), vma = make_uint2(0, 0), vmb = make_uint2(0, 0);
        if (va) {
            kca = __ldg(reinterpret_cast<const uint4 *>(kt + koff_c));
            ksa = __ldg(reinterpret_cast<const uint32_t *>(kt + koff_s));
            kma = __ldg(reinterpret_cast<const uint2 *>(kt + koff_m));
            vma = __ldg(reinterpret_cast<const uint2 *>(vt + koff_m));
        }
        if (vb8) {
            kcb = __ldg(reinterpret_cast<const uint4 *>(kt + koff_c + 8 * kBlockBytes));
            ksb = __ldg(reinterpret_cast<const uint32_t *>(kt + koff_s + 8 * kBlockBytes));
            kmb = __ldg(reinterpret_cast<const uint2 *>(kt + koff_m + 8 * kBlockBytes));
            vmb = __ldg(reinterpret_cast<const uint2 *>(vt + koff_m + 8 * kBlockBytes));
        }
        uint2 vc[4];
        uint32_t vs[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int dt = (u & 1) + 8 * (u >> 1);  // token 2c + dt
            if (kFull || 2 * c + dt < nvalid) {
                vc[u] = __ldg(reinterpret_cast<const uint2 *>(vt + voff_c + dt * kBlockBytes));
                vs[u] = __ldg(reinterpret_cast<const uint32_t *>(vt + voff_s + dt * kBlockBytes));
            } else {
                vc[u] = make_uint2(0, 0);
                vs[u] = 0;
            }
        }

        // ---------------- S = Q K^T ----------------
        float sc[4] = {0.f, 0.f, 0.f, 0.f}, ss[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t kwa[4] = {kca.x, kca.y, kca.z, kca.w};
        const uint32_t kwb[4] = {kcb.x, kcb.y, kcb.z, kcb.w};
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int w = m >> 1, by = 2 * (m & 1);
            const uint2 a0 = lut(tab, kwa[w], by, lane8);
            const uint2 a1 = lut(tab, kwb[w], by, lane8);
            const uint2 a2 = lut(tab, kwa[w], by + 1, lane8);
            const uint2 a3 = lut(tab, kwb[w], by + 1, lane8);
            mma16816(sc, a0.x, a1.x, a2.x, a3.x, qc[m][0], qc[m][1]);
            mma16816(sc, a0.y, a1.y, a2.y, a3.y, qc[m][0], qc[m][1]);
            mma16816(ss, sign_pair(ksa, 2 * m), sign_pair(ksb, 2 * m), sign_pair(ksa, 2 * m + 1),
                     sign_pair(ksb, 2 * m + 1), qs[m][0], qs[m][1]);
        }
        float s2[4];
        {
            const float k_sa = h_lo(kma.x), k_za = h_hi(kma.x), k_aa = h_lo(kma.y);
            const float k_sb = h_lo(kmb.x), k_zb = h_hi(kmb.x), k_ab = h_lo(kmb.y);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float xa = fmaf(k_sa, sc[e], fmaf(k_aa, ss[e], k_za * qsum[e]));
                const float xb = fmaf(k_sb, sc[2 + e], fmaf(k_ab, ss[2 + e], k_zb * qsum[e]));
                s2[e] = va ? xa * scale_log2 : -INFINITY;
                s2[2 + e] = vb8 ? xb * scale_log2 : -INFINITY;
            }
        }
        // ---------------- online softmax ----------------
        float corr[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            float mx = fmaxf(s2[e], s2[2 + e]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mnew = fmaxf(mrun[e], mx);
            corr[e] = ex2(mrun[e] - mnew);  // first tile: ex2(-inf) = 0
            mrun[e] = mnew;
        }
        float p[4];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            p[e] = ex2(s2[e] - mrun[e]);
            p[2 + e] = ex2(s2[2 + e] - mrun[e]);
        }
        if (corr[0] != 1.0f || corr[1] != 1.0f) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                o[i][0] *= corr[0];
                o[i][1] *= corr[1];
                o[i][2] *= corr[0];
                o[i][3] *= corr[1];
            }
        }
        const float v_sa = h_lo(vma.x), v_za = h_hi(vma.x), v_aa = h_lo(vma.y);
        const float v_sb = h_lo(vmb.x), v_zb = h_hi(vmb.x), v_ab = h_lo(vmb.y);
        uint32_t pk[4];  // (p*v_scale, p*v_alpha) per (token g / g+8, head 2c+e)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            lrun[e] = fmaf(lrun[e], corr[e], p[e] + p[2 + e]);
            zrun[e] = fmaf(zrun[e], corr[e], fmaf(p[e], v_za, p[2 + e] * v_zb));
            pk[e] = pack_h2(p[e] * v_sa, p[e] * v_aa);
            pk[2 + e] = pack_h2(p[2 + e] * v_sb, p[2 + e] * v_ab);
        }
        // transpose to the B layout: lane (n=g, c) needs tokens 2c, 2c+1, 2c+8, 2c+9 of head g
        uint32_t bt[4];
        {
            const int srcA = 8 * c + (g >> 1), srcB = srcA + 4;
            const bool odd = g & 1;
            const uint32_t x0e = __shfl_sync(0xffffffffu, pk[0], srcA), x0o = __shfl_sync(0xffffffffu, pk[1], srcA);
            const uint32_t x1e = __shfl_sync(0xffffffffu, pk[0], srcB), x1o = __shfl_sync(0xffffffffu, pk[1], srcB);
            const uint32_t x2e = __shfl_sync(0xffffffffu, pk[2], srcA), x2o = __shfl_sync(0xffffffffu, pk[3], srcA);
            const uint32_t x3e = __shfl_sync(0xffffffffu, pk[2], srcB), x3o = __shfl_sync(0xffffffffu, pk[3], srcB);
            bt[0] = odd ? x0o : x0e;
            bt[1] = odd ? x1o : x1e;
            bt[2] = odd ? x2o : x2e;
            bt[3] = odd ? x3o : x3e;
        }
        const uint32_t b1_0 = __byte_perm(bt[0], bt[1], 0x5410), b1_1 = __byte_perm(bt[2], bt[3], 0x5410);
        const uint32_t b2_0 = __byte_perm(bt[0], bt[1], 0x7632), b2_1 = __byte_perm(bt[2], bt[3], 0x7632);

        // ---------------- O += V^T P ----------------
        const uint32_t sA = __byte_perm(vs[0], vs[1], sel_half), sB = __byte_perm(vs[2], vs[3], sel_half);
#pragma unroll
        for (int w = 0; w < 2; ++w) {
            const uint32_t xa0 = w ? vc[0].y : vc[0].x, xa1 = w ? vc[1].y : vc[1].x;
            const uint32_t xb0 = w ? vc[2].y : vc[2].x, xb1 = w ? vc[3].y : vc[3].x;
            // byte k of ia_e = (even-dim nibble of token 2c) | (same nibble of token 2c+1) << 4
            constexpr uint32_t kLo = 0x0F0F0F0Fu, kHi = 0xF0F0F0F0u;
            const uint32_t ia_e = (xa0 & kLo) | ((xa1 << 4) & kHi), ia_o = ((xa0 >> 4) & kLo) | (xa1 & kHi);
            const uint32_t ib_e = (xb0 & kLo) | ((xb1 << 4) & kHi), ib_o = ((xb0 >> 4) & kLo) | (xb1 & kHi);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int i = 4 * w + k;
                const uint2 r0 = lut(tab, ia_e, k, lane8);
                const uint2 r1 = lut(tab, ia_o, k, lane8);
                const uint2 r2 = lut(tab, ib_e, k, lane8);
                const uint2 r3 = lut(tab, ib_o, k, lane8);
                mma16816(o[i], r0.x, r1.x, r2.x, r3.x, b1_0, b1_1);
                mma16816(o[i], r0.y, r1.y, r2.y, r3.y, b1_0, b1_1);
                mma16816(o[i], sign_pair(sA, 2 * i), sign_pair(sA, 2 * i + 1), sign_pair(sB, 2 * i),
                         sign_pair(sB, 2 * i + 1), b2_0, b2_1);
            }
        }
    }
};

template <int G>
__global__ void __launch_bounds__(kMmaWarps * 32, 3)
decode_mma_kernel(const __half *__restrict__ q, const uint8_t *__restrict__ kb, const uint8_t *__restrict__ vb,
                  int64_t bs_b, int64_t bs_h, float *__restrict__ pm, float *__restrict__ pl,
                  float *__restrict__ po, int Hq, int group, int64_t seq_len, int64_t chunk, int nsplit,
                  float scale_log2, int flags) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t *tab = smem;                                        // 64 KB code-byte table
    float *sq = reinterpret_cast<float *>(smem + kLutBytes);     // [8][kQRow] query (fp16 values)
    float *s_ml = sq + 8 * kQRow;                                // [warps][3][8] m, l, z
    float *s_qsum = s_ml + kMmaWarps * 24;                       // [8]
    uint32_t *s_cent = reinterpret_cast<uint32_t *>(s_qsum + 8);  // [16] C_hi | C_lo << 16
    float *s_o = reinterpret_cast<float *>(smem);  // [warps][8][128], reuses the table after the loop

    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int h0 = kvh * group;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    // ---- centroid pairs, then the code-byte table (row v: 32 lane copies) ----
    if (threadIdx.x < 16) {
        const float cv = lm(threadIdx.x);
        const __half hi = __float2half_rn(cv);
        const __half lo = __float2half_rn(cv - __half2float(hi));
        s_cent[threadIdx.x] = (uint32_t)__half_as_ushort(hi) | ((uint32_t)__half_as_ushort(lo) << 16);
    }
    for (int idx = threadIdx.x; idx < 8 * kD; idx += blockDim.x) {
        const int h = idx >> 7, d = idx & (kD - 1);
        sq[h * kQRow + d] = (h < G) ? __half2float(q[((int64_t)b * Hq + h0 + h) * kD + d]) : 0.0f;
    }
    __syncthreads();
    for (int v = warp; v < 256; v += kMmaWarps) {
        const uint32_t e0 = s_cent[v & 15], e1 = s_cent[v >> 4];
        uint2 e;
        e.x = __byte_perm(e0, e1, 0x5410);  // C_hi(lo nibble) | C_hi(hi nibble) << 16
        e.y = __byte_perm(e0, e1, 0x7632);  // C_lo pair
        reinterpret_cast<uint2 *>(tab + v * 256)[lane] = e;
    }
    if (flags & ECC_DECODE_ROTATE_Q) {  // q_rot = fp16(WHT(q)), like patch.py:106
        for (int h = warp; h < G; h += kMmaWarps) {
            float *row = sq + h * kQRow;
            for (int s = 1; s < kD; s <<= 1) {
                for (int p = lane; p < kD / 2; p += 32) {
                    const int lo = (p / s) * 2 * s + (p % s);
                    const float a = row[lo], bb = row[lo + s];
                    row[lo] = __fadd_rn(a, bb);
                    row[lo + s] = __fsub_rn(a, bb);
                }
                __syncwarp();
            }
            for (int d = lane; d < kD; d += 32) {
                const float x = row[d];
                const float q0 = __fmul_rn(x, kInvSqrt128);
                const float rem = __fmaf_rn(-q0, kSqrt128, x);
                row[d] = __half2float(__float2half_rn(__fmaf_rn(rem, kInvSqrt128, q0)));
            }
        }
    }
    __syncwarp();
    for (int h = warp; h < 8; h += kMmaWarps) {
        const float *row = sq + h * kQRow;
        float s = row[lane] + row[lane + 32] + row[lane + 64] + row[lane + 96];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (lane == 0) s_qsum[h] = s;
    }
    __syncthreads();

    TileLane t;
    t.g = lane >> 2;
    t.c = lane & 3;
    t.lane8 = (uint32_t)lane * 8u;
    t.tab = (uint32_t)__cvta_generic_to_shared(tab);
    t.sel_half = (t.g & 1) ? 0x7632u : 0x5410u;
    t.scale_log2 = scale_log2;
    t.koff_c = t.g * kBlockBytes + 16 * t.c;
    t.koff_s = t.g * kBlockBytes + kSynOff + 4 * t.c;
    t.koff_m = t.g * kBlockBytes + kScaleOff;
    t.voff_c = 2 * t.c * kBlockBytes + 8 * t.g;
    t.voff_s = 2 * t.c * kBlockBytes + kSynOff + 4 * (t.g >> 1);
    {
        const float *qrow = sq + t.g * kQRow;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int d0 = 32 * t.c + 4 * m;
            t.qc[m][0] = pack_h2(qrow[d0], qrow[d0 + 1]);
            t.qc[m][1] = pack_h2(qrow[d0 + 2], qrow[d0 + 3]);
            const int e0 = 32 * t.c + 2 * m;
            t.qs[m][0] = pack_h2(qrow[e0], qrow[e0 + 16]);
            t.qs[m][1] = pack_h2(qrow[e0 + 1], qrow[e0 + 17]);
        }
        t.qsum[0] = s_qsum[2 * t.c];
        t.qsum[1] = s_qsum[2 * t.c + 1];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) t.o[i][k] = 0.0f;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        t.mrun[e] = -INFINITY;
        t.lrun[e] = 0.0f;
        t.zrun[e] = 0.0f;
    }

    const int64_t t0 = (int64_t)split * chunk;
    const int64_t t1 = min(seq_len, t0 + chunk);
    const int64_t row_off = (int64_t)b * bs_b + (int64_t)kvh * bs_h;
    const uint8_t *kbase = kb + row_off * kBlockBytes;
    const uint8_t *vbase = vb + row_off * kBlockBytes;
    for (int64_t tb = t0 + (int64_t)warp * kTileTok; tb < t1; tb += (int64_t)kMmaWarps * kTileTok) {
        const uint8_t *kt = kbase + tb * kBlockBytes;
        const uint8_t *vt = vbase + tb * kBlockBytes;
        if (tb + kTileTok <= t1)
            t.tile<true>(kt, vt, kTileTok);
        else
            t.tile<false>(kt, vt, (int)(t1 - tb));
    }

    // ---------------- combine lanes, then warps ----------------
    const int g = t.g, c = t.c;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            t.lrun[e] += __shfl_xor_sync(0xffffffffu, t.lrun[e], off);
            t.zrun[e] += __shfl_xor_sync(0xffffffffu, t.zrun[e], off);
        }
    }
    __syncthreads();  // every warp is done with the table; s_o overlays it
    float *ml = s_ml + warp * 24;
    if (g == 0) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            ml[2 * c + e] = t.mrun[e];
            ml[8 + 2 * c + e] = t.lrun[e];
            ml[16 + 2 * c + e] = t.zrun[e];
        }
    }
    float *ow = s_o + warp * 8 * kD;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int d0 = 16 * g + 2 * i;
        ow[(2 * c) * kD + d0] = t.o[i][0];
        ow[(2 * c + 1) * kD + d0] = t.o[i][1];
        ow[(2 * c) * kD + d0 + 1] = t.o[i][2];
        ow[(2 * c + 1) * kD + d0 + 1] = t.o[i][3];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * kD; idx += blockDim.x) {
        const int h = idx >> 7, d = idx & (kD - 1);
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kMmaWarps; ++w) M = fmaxf(M, s_ml[w * 24 + h]);
        float L = 0.0f, O = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kMmaWarps; ++w) {
                const float mw = s_ml[w * 24 + h];
                if (mw == -INFINITY) continue;
                const float e = exp2f(mw - M);
                L = fmaf(s_ml[w * 24 + 8 + h], e, L);
                O = fmaf(s_o[(w * 8 + h) * kD + d] + s_ml[w * 24 + 16 + h], e, O);
            }
        }
        const int64_t pi = ((int64_t)b * Hq + h0 + h) * nsplit + split;
        po[pi * kD + d] = O;
        if (d == 0) {
            pm[pi] = (M == -INFINITY) ? -INFINITY : M * kLn2f;
            pl[pi] = L;
        }
    }
}

static_assert(kMmaWarps * 8 * kD * sizeof(float) <= (size_t)kLutBytes, "combine buffer fits in the table");
size_t mma_smem_bytes() { return kLutBytes + (8 * kQRow + kMmaWarps * 24 + 8 + 16) * sizeof(float); }

template <int G>
static int launch_mma_g(const void *q, const void *kbp, const void *vbp, int64_t bs_b, int64_t bs_h, float *pm,
                        float *pl, float *po, int B, int Hq, int Hkv, int64_t seq_len, int64_t chunk, int ns,
                        float scale_log2, int flags, cudaStream_t s) {
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t smem = mma_smem_bytes();
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(decode_mma_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return ECC_ERR_CUDA;
        configured[dev] = true;
    }
    dim3 grid(ns, Hkv, B);
    decode_mma_kernel<G><<<grid, kMmaWarps * 32, smem, s>>>(
        reinterpret_cast<const __half *>(q), reinterpret_cast<const uint8_t *>(kbp),
        reinterpret_cast<const uint8_t *>(vbp), bs_b, bs_h, pm, pl, po, Hq, Hq / Hkv, seq_len, chunk, ns,
        scale_log2, flags);
    return ECC_OK;
}

int launch_decode_mma(const void *q, const void *kbp, const void *vbp, int64_t bs_b, int64_t bs_h, float *pm,
                      float *pl, float *po, int B, int Hq, int Hkv, int64_t seq_len, int64_t chunk, int ns,
                      float scale_log2, int flags, cudaStream_t s) {
    switch (Hq / Hkv) {
        case 1: return launch_mma_g<1>(q, kbp, vbp, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns, scale_log2, flags, s);
        case 2: return launch_mma_g<2>(q, kbp, vbp, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns, scale_log2, flags, s);
        case 3: return launch_mma_g<3>(q, kbp, vbp, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns, scale_log2, flags, s);
        case 4: return launch_mma_g<4>(q, kbp, vbp, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns, scale_log2, flags, s);
        case 5: return launch_mma_g<5>(q, kbp, vbp, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns, scale_log2, flags, s);
        case 6: return launch_mma_g<6>(q, kbp, vbp, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns, scale_log2, flags, s);
        case 7: return launch_mma_g<7>(q, kbp, vbp, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns, scale_log2, flags, s);
        case 8: return launch_mma_g<8>(q, kbp, vbp, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns, scale_log2, flags, s);
        default: return ECC_ERR_GQA;
    }
}

}  // namespace ecc
