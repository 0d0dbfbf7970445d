// decode_tma.cu -- TMA-fed tensor-core decode attention over 128-byte blocks
// (sm_100a), GQA groups of up to 8 query heads per kv head.
//
// Work split: the tiles (16 tokens of one (b, kv head) row) of all rows are
// laid end to end and cut into equal contiguous ranges, one per warp of the
// grid (persistent CTAs, one per SM, kWarps warps each).  A warp therefore
// sees at most a few row segments; for each it builds the query fragments in
// its own registers (loaded straight from global memory, WHT-rotated across
// the four lanes that hold one head) and writes one split partial (m, l, o)
// at the end.  Partial slot of a segment = warp - first warp of the row, so
// every row's partials are contiguous; the last warp of a row marks the
// row's unused slots empty.  No CTA-wide barrier is needed after set-up.
//
// Each warp streams its tiles through its own kStages-stage shared-memory
// ring: one lane issues four cp.async.bulk.tensor boxes per tile (K codes
// 16x64 B, K syndrome+meta 16x32 B, V codes, V syndrome+meta) on an mbarrier
// and later waits on it, then __syncwarp hands the data to the warp.  The
// tensor maps cover [0, seq_len) tokens, so rows past the sequence end come
// back as zeros; such tokens are masked to -inf.  QK: per 16-dim step, one
// m16n8k16 product for the centroids of 8 tokens (rows g / g+8 = fp16 hi /
// lo parts) per token half and one for the signs.  PV: per code byte of the
// lane (two dims in rows g / g+8), four products: centroids hi and lo
// against p*scale_v, centroids hi against its fp16 residual, signs against
// the sign weights.
//
// Every mbarrier wait is bounded (~2 s of clock64); on timeout the warp
// raises a device flag for ecc_device_status(), stops computing and drains
// its outstanding copies (bounded) before exiting.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "ecc_common.cuh"

namespace ecc {

int launch_status();
int sm_count();

__device__ int g_device_error;  // raised by a bounded wait that ran out

namespace tmak {

constexpr int kWarps = 12;          // warps per CTA (384 threads)
constexpr int kStages = 2;          // ring stages per warp
constexpr int kTile = 32;           // tokens per stage (two 16-token MMA sub-tiles)
constexpr int kStageBytes = 6144;
constexpr int kOffKC = 0, kOffKS = 2048, kOffVC = 3072, kOffVS = 5120;  // 32 x 64 B, 32 x 32 B, ...
constexpr int kSubC = 1024, kSubS = 512;  // offset of sub-tile 1 in the code / syndrome boxes
constexpr int kThreads = kWarps * 32;
constexpr int kLutBytes = 65536;
constexpr float kLn2f = 0.6931471805599453f;
constexpr long long kWaitCycles = 4000000000ll;

constexpr int kSmemReserve = 1024;  // shared-window offset of dynamic shared memory
constexpr int kSmLut = 0;
constexpr int kSmRing = kSmLut + kLutBytes;                        // [kWarps][kStages][kStageBytes]
constexpr int kSmCent = kSmRing + kWarps * kStages * kStageBytes;  // [16] u32
constexpr int kSmBar = kSmCent + 16 * 4;                           // [kWarps][kStages] u64
constexpr int kSmBytes = kSmBar + kWarps * kStages * 8;
static_assert(kSmRing % 1024 == 0 && kStageBytes % 128 == 0, "TMA destinations 128-B aligned");
static_assert(kSmBar % 8 == 0, "mbarriers 8-B aligned");
static_assert(kSmBytes <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait by one lane; false when it ran out (the device flag is raised).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, long long limit = kWaitCycles) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try(bar, parity)) {
        if (clock64() - t0 > limit) {
            atomicExch(&g_device_error, 1);
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ void tma_4d(uint32_t dst, const CUtensorMap *map, int x, int y, int z, int w,
                                       uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
    return r;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 r;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(a));
    return r;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t r;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r) : "r"(a));
    return r;
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// 8x8 transpose of 16-bit elements across the warp: lane (g, c) passes row g,
// columns 2c, 2c+1 and receives row g, columns 2c, 2c+1 of the transpose.
__device__ __forceinline__ uint32_t movtrans(uint32_t a) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}
// Code-byte table lookup: for code byte v (codes v & 15, v >> 4) the fp16x2
// word of their hi parts and the fp16x2 word of their lo parts.  Row v of the
// table is 256 bytes: the hi words of the 32 lanes' private copies at v*256 +
// 4*lane, the lo words 128 bytes further.  Every 32-bit load of a warp then
// hits 32 distinct banks, and the two halves arrive in separate registers, so
// the centroid MMA operands (hi words of four lookups in one register quad,
// lo words in another) need no moves.  The offset v*256 + 4*lane is one prmt.
// The table sits at the start of the dynamic shared memory, whose
// shared-window address is the per-block reserve kSmemReserve (checked on the
// host against cudaDevAttrReservedSharedMemoryPerBlock and again by the
// kernel), so the base folds into the loads' immediate offsets.  The table is
// constant after the kernel's set-up barrier, so the loads are not volatile
// and may be scheduled freely.
__device__ __forceinline__ uint2 lut(uint32_t word, int byte_idx, uint32_t lane4) {
    uint2 r;
    const uint32_t a = __byte_perm(word, lane4, 0x5504u | ((uint32_t)byte_idx << 4));
    asm("ld.shared.u32 %0, [%1+%2];" : "=r"(r.x) : "r"(a), "n"(kSmemReserve + kSmLut));
    asm("ld.shared.u32 %0, [%1+%2];" : "=r"(r.y) : "r"(a), "n"(kSmemReserve + kSmLut + 128));
    return r;
}
// +-1 pair from bits p and p+16 of w (bit 1 -> +1.0)
__device__ __forceinline__ uint32_t sign_pair(uint32_t w, int p) {
    const uint32_t x = w << (15 - p);
    return (~x & 0x80008000u) | 0x3C003C00u;
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float h_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu))); }
__device__ __forceinline__ float h_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }

// Sign bit p of both fp16 halves of x kept in place: each half is 0 or the
// fp16 value whose only set bit is p (p <= 14), a power of two sign_weight(p).
// Bit 15 is the fp16 sign bit, so that one moves to bit 14 first.
__device__ __forceinline__ uint32_t sign_bits(uint32_t x, int p) {
    return p == 15 ? ((x >> 1) & 0x40004000u) : (x & (0x00010001u << p));
}
// 1 / (value of the fp16 with only bit p set), bit 15 taken as bit 14
__host__ __device__ constexpr float sign_unweight(int p) {
    return p == 15 ? 0.5f
         : p == 14 ? 0.5f
         : p == 13 ? 128.0f
         : p == 12 ? 2048.0f
         : p == 11 ? 8192.0f
         : p == 10 ? 16384.0f
                   : (float)(1u << (24 - p));  // subnormal 2^(p-24)
}

// K sign bits kept as 0/1 in the exponent field: bit pair (p, p+16) of the
// syndrome word w lands at bit positions (q, q+16), q = kpos(p) in 10..14,
// each half then being 0 or the fp16 2^kexp(p).  x5 = w << 5, x10 = w << 10,
// x1 = w >> 1 are shared by the 16 pairs of a word (3 shifts + 16 masks
// instead of 2 operations per pair).
__host__ __device__ constexpr int kpos(int p) { return p == 15 ? 14 : p >= 10 ? p : p >= 5 ? p + 5 : p + 10; }
__host__ __device__ constexpr int kexp(int p) {
    return kpos(p) == 10 ? -14 : kpos(p) == 11 ? -13 : kpos(p) == 12 ? -11 : kpos(p) == 13 ? -7 : 1;
}
__device__ __forceinline__ uint32_t kbits(uint32_t w, uint32_t x5, uint32_t x10, uint32_t x1, int p) {
    const uint32_t src = p == 15 ? x1 : p >= 10 ? w : p >= 5 ? x5 : x10;
    return src & (0x00010001u << kpos(p));
}

// Consumer lane state for one work item.  For groups of at most 4 query heads
// the PV products use the idle columns 4..7 of the n8 operand for the V sign
// term: lanes g < 4 of the P operand carry p * vscale of head g (columns
// 0..3, centroid products), lanes g >= 4 carry 2 p * valpha of head g - 4
// (columns 4..7, sign-bit products with the bits masked in place, so each
// accumulator row has one power-of-two weight, removed at the end).
template <int G>
struct Lane {
    uint32_t qc[8][2];
    uint32_t qs[8][2];  // q of the sign products, k slot of bit p scaled by 2^-(ssh + kexp(p))
    float sgn2;         // 2^(ssh + 1): q.s = sgn2 * (sign product) - sum(q)
    float qsum[2];
    // PV accumulators: o[i] rows g / g+8 = dims 16g + 2i / 16g + 2i + 1 (code
    // byte i of the lane's 8 V code bytes), columns = the n8 operand columns
    float o[8][4];
    float mrun[2], lrun[2], zrun[2];
    uint32_t lane4, sel_half;
    uint32_t voff;  // this lane's byte offset in the swizzled V code box (see load_v)
    uint32_t soff;  // this lane's byte offset in the swizzled syndrome boxes (see qk, load_v)
    int g, c;
    float scale_log2;

    // Query fragments of a row segment from the lane's fp16 query words qw
    // (dims 32c..32c+31 of its head): the centroid operand qc, the sign
    // operand qs with its exponent sgn2, and the per-head sums qsum.
    __device__ __forceinline__ void set_query(const uint4 (&qw)[4], bool rotate) {
        float x[32];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t wv[4] = {qw[k].x, qw[k].y, qw[k].z, qw[k].w};
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                x[8 * k + 2 * m] = h_lo(wv[m]);
                x[8 * k + 2 * m + 1] = h_hi(wv[m]);
            }
        }
        if (rotate) {  // q_rot = fp16(WHT(q)), like patch.py:106
#pragma unroll
            for (int s = 1; s < 32; s <<= 1)
#pragma unroll
                for (int k = 0; k < 32; ++k)
                    if ((k & s) == 0) {
                        const float a = x[k], bb = x[k + s];
                        x[k] = __fadd_rn(a, bb);
                        x[k + s] = __fsub_rn(a, bb);
                    }
#pragma unroll
            for (int s = 1; s <= 2; s <<= 1) {  // strides 32, 64: partner lane c ^ s
                const float sgn = (c & s) ? -1.0f : 1.0f;
#pragma unroll
                for (int k = 0; k < 32; ++k) {
                    const float p = __shfl_xor_sync(0xffffffffu, x[k], s);
                    x[k] = __fmaf_rn(sgn, x[k], p);
                }
            }
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                const float v = x[k];
                const float q0 = __fmul_rn(v, kInvSqrt128);
                const float rem = __fmaf_rn(-q0, kSqrt128, v);
                x[k] = __half2float(__float2half_rn(__fmaf_rn(rem, kInvSqrt128, q0)));
            }
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            qc[m][0] = pack_h2(x[4 * m], x[4 * m + 1]);
            qc[m][1] = pack_h2(x[4 * m + 2], x[4 * m + 3]);
        }
        // sign-product operand: scale 2^-ssh keeps q * 2^(14 - ssh) < 2^15
        // for the largest |q| of the group (q is fp16, the scalings are
        // exact powers of two)
        {
            float qmax = 0.0f;
#pragma unroll
            for (int k = 0; k < 32; ++k) qmax = fmaxf(qmax, fabsf(x[k]));
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, off));
            const int e2 = (qmax > 0.0f) ? ((__float_as_int(qmax) >> 23) & 0xff) - 127 : 0;
            const int ssh = max(0, e2);
            sgn2 = __int_as_float((ssh + 1 + 127) << 23);
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const float f0 = __int_as_float((127 - ssh - kexp(2 * m)) << 23);
                const float f1 = __int_as_float((127 - ssh - kexp(2 * m + 1)) << 23);
                qs[m][0] = pack_h2(x[2 * m] * f0, x[2 * m + 16] * f0);
                qs[m][1] = pack_h2(x[2 * m + 1] * f1, x[2 * m + 17] * f1);
            }
        }
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < 32; ++k) sum += x[k];
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        qsum[0] = __shfl_sync(0xffffffffu, sum, 4 * (2 * c));       // head 2c
        qsum[1] = __shfl_sync(0xffffffffu, sum, 4 * (2 * c + 1));   // head 2c+1
    }

    // Raw V data of one 16-token sub-tile: tokens 2c, 2c+1, 2c+8, 2c+9 (code
    // bytes 8g..8g+7, syndrome word g/2) and the metadata of tokens g, g+8.
    //
    // The V code box (64-byte rows) is written with the 64-byte swizzle:
    // 16-byte chunk j of row r lands at chunk j ^ ((r >> 1) & 3).  Lane (g,
    // c) reads chunk g/2 of rows 2c + {0, 1, 8, 9}, whose (r >> 1) & 3 is c,
    // so its offset within a row is the lane constant 16 ((g/2) ^ c) + 8 (g &
    // 1) (voff): a half-warp's reads then fall on 16 banks instead of 8.  The
    // syndrome/metadata boxes (32-byte rows) use the 32-byte swizzle: chunk
    // j of row r at chunk j ^ ((r >> 2) & 1) (soff: 16 ((r >> 2) & 1) for the
    // rows a lane reads), which makes the syndrome-word and metadata reads
    // conflict-free.
    struct VRaw {
        uint2 vc[4];
        uint32_t vs[4];
        uint2 vma, vmb;
    };
    __device__ __forceinline__ VRaw load_v(uint32_t vcb, uint32_t vsb) const {
        VRaw v;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int tok = 2 * c + (u & 1) + 8 * (u >> 1);
            v.vc[u] = lds64(vcb + 64 * tok + voff);
            // row tok: (tok >> 2) & 1 = c >> 1
            v.vs[u] = lds32(vsb + 32 * tok + 16 * (c >> 1) + 4 * (g >> 1));
        }
        // metadata: chunk 1 of rows g and g + 8, (row >> 2) & 1 = g >> 2
        v.vma = lds64(vsb + 32 * g + (16 ^ soff));
        v.vmb = lds64(vsb + 32 * (g + 8) + (16 ^ soff));
        return v;
    }

    // log2-scaled scores of one 16-token sub-tile (K codes at kcb, syndrome +
    // metadata at ksb): s2[e] token g, s2[2+e] token g+8, head 2c+e; tokens
    // outside [lo, hi) (sub-tile offsets) are -inf.
    __device__ __forceinline__ void qk(uint32_t kcb, uint32_t ksb, int lo, int hi, float (&s2)[4]) const {
        const uint4 kca = lds128(kcb + 64 * g + 16 * c);
        const uint4 kcb8 = lds128(kcb + 64 * (g + 8) + 16 * c);
        // syndrome box with the 32-byte swizzle (see load_v): rows g, g + 8
        const uint32_t ksa = lds32(ksb + 32 * g + soff + 4 * c);
        const uint32_t ksb8 = lds32(ksb + 32 * (g + 8) + soff + 4 * c);
        const uint32_t ka5 = ksa << 5, ka10 = ksa << 10, ka1 = ksa >> 1;
        const uint32_t kb5 = ksb8 << 5, kb10 = ksb8 << 10, kb1 = ksb8 >> 1;
        const uint2 kma = lds64(ksb + 32 * g + (16 ^ soff));
        const uint2 kmb = lds64(ksb + 32 * (g + 8) + (16 ^ soff));
        const bool va = g >= lo && g < hi, vb8 = g + 8 >= lo && g + 8 < hi;

        // Centroid products: rows g / g+8 of the A operand carry the fp16 hi /
        // lo parts of one token's centroids, so each table entry (hi, lo)
        // lands in the operand registers as loaded; one product per 8 tokens.
        float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f}, ss[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t kwa[4] = {kca.x, kca.y, kca.z, kca.w};
        const uint32_t kwb[4] = {kcb8.x, kcb8.y, kcb8.z, kcb8.w};
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int w = m >> 1, by = 2 * (m & 1);
            const uint2 xa = lut(kwa[w], by, lane4);      // token g, k slots 2c, 2c+1
            const uint2 ya = lut(kwa[w], by + 1, lane4);  // token g, k slots 2c+8, 2c+9
            const uint2 xb = lut(kwb[w], by, lane4);      // token g+8
            const uint2 yb = lut(kwb[w], by + 1, lane4);
            mma16816(sa, xa.x, xa.y, ya.x, ya.y, qc[m][0], qc[m][1]);
            mma16816(sb, xb.x, xb.y, yb.x, yb.y, qc[m][0], qc[m][1]);
            mma16816(ss, kbits(ksa, ka5, ka10, ka1, 2 * m), kbits(ksb8, kb5, kb10, kb1, 2 * m),
                     kbits(ksa, ka5, ka10, ka1, 2 * m + 1), kbits(ksb8, kb5, kb10, kb1, 2 * m + 1), qs[m][0],
                     qs[m][1]);
        }
        // q.C of token g (head 2c+e) = hi row + lo row
        const float sc[4] = {sa[0] + sa[2], sa[1] + sa[3], sb[0] + sb[2], sb[1] + sb[3]};
        // score = scale q.C + alpha (2 q.b - sum q) + zero sum q  (s = 2b - 1)
        const float k_sa = h_lo(kma.x), k_za = h_hi(kma.x), k_aa = h_lo(kma.y);
        const float k_sb = h_lo(kmb.x), k_zb = h_hi(kmb.x), k_ab = h_lo(kmb.y);
        const float k_ga = k_aa * sgn2, k_gb = k_ab * sgn2, k_da = k_za - k_aa, k_db = k_zb - k_ab;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const float xa = fmaf(k_sa, sc[e], fmaf(k_ga, ss[e], k_da * qsum[e]));
            const float xb = fmaf(k_sb, sc[2 + e], fmaf(k_gb, ss[2 + e], k_db * qsum[e]));
            s2[e] = va ? xa * scale_log2 : -INFINITY;
            s2[2 + e] = vb8 ? xb * scale_log2 : -INFINITY;
        }
    }

    // PV products of one 16-token sub-tile with probabilities p (same layout
    // as the scores: p[e] token g, p[2+e] token g+8, head 2c+e).
    //
    // The B operand (k = token, n = column) comes from the score layout (row =
    // token, columns 2c, 2c+1 in lane (g, c)) by one 8x8 transpose per token
    // half (movmatrix).  Its words: ws = p*scale_v with its fp16 residual
    // ws - fp16(ws) (a single fp16 rounding of ws is 2^-11 relative, close to
    // the 2e-3 output tolerance when a few large values dominate), and the
    // sign weights wa = p*alpha_v.  Groups of up to 4 heads use the idle
    // columns 4..7 for the sign products: the score columns 4..7 repeat heads
    // 0..3 (see the query set-up), lanes c >= 2 put 2*wa there, and the
    // sign bits are masked in place (each fp16 half is 0 or the power of two
    // whose only set bit is p), so every accumulator row has one known weight
    // that the epilogue divides out; s = 2b - 1 moves -alpha_v into the
    // zero-point sum.  Groups of 5..8 use +-1 sign operands against wa.
    //
    // Per code byte i of the lane (dims 16g + 2i, 16g + 2i + 1 in rows g,
    // g + 8 of accumulator i), four products: centroids hi x ws, centroids
    // lo x ws, centroids hi x residual, signs x sign weights.
    __device__ __forceinline__ void pv(const VRaw &v, const float (&p)[4]) {
        const float v_sa = h_lo(v.vma.x), v_aa = h_lo(v.vma.y);
        const float v_sb = h_lo(v.vmb.x), v_ab = h_lo(v.vmb.y);
        constexpr bool kSplitCols = G <= 4;
        // rows of the pre-transpose matrices: t = 0 token g, t = 1 token g+8
        uint32_t mw[2], mr[2], ma[2];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const float sc = t ? v_sb : v_sa, al = (kSplitCols ? 2.0f : 1.0f) * (t ? v_ab : v_aa);
            const float w0 = p[2 * t] * sc, w1 = p[2 * t + 1] * sc;
            mw[t] = pack_h2(w0, w1);
            mr[t] = pack_h2(w0 - h_lo(mw[t]), w1 - h_hi(mw[t]));
            ma[t] = pack_h2(p[2 * t] * al, p[2 * t + 1] * al);
        }
        // B words: [0] tokens 2c, 2c+1, [1] tokens 2c+8, 2c+9 of column g
        uint32_t bw[2], br[2], bs[2];
        if constexpr (kSplitCols) {
            const bool cent = g < 4, lo_cols = c < 2;
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const uint32_t x = movtrans(lo_cols ? mw[t] : ma[t]);
                const uint32_t r = movtrans(mr[t]);
                bw[t] = cent ? x : 0u;
                bs[t] = cent ? 0u : x;
                br[t] = cent ? r : 0u;
            }
        } else {
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                bw[t] = movtrans(mw[t]);
                br[t] = movtrans(mr[t]);
                bs[t] = movtrans(ma[t]);
            }
        }

        const uint32_t sA = __byte_perm(v.vs[0], v.vs[1], sel_half), sB = __byte_perm(v.vs[2], v.vs[3], sel_half);
#pragma unroll
        for (int w = 0; w < 2; ++w) {
            const uint32_t xa0 = w ? v.vc[0].y : v.vc[0].x, xa1 = w ? v.vc[1].y : v.vc[1].x;
            const uint32_t xb0 = w ? v.vc[2].y : v.vc[2].x, xb1 = w ? v.vc[3].y : v.vc[3].x;
            constexpr uint32_t kLo = 0x0F0F0F0Fu, kHi = 0xF0F0F0F0u;
            const uint32_t ia_e = (xa0 & kLo) | ((xa1 << 4) & kHi), ia_o = ((xa0 >> 4) & kLo) | (xa1 & kHi);
            const uint32_t ib_e = (xb0 & kLo) | ((xb1 << 4) & kHi), ib_o = ((xb0 >> 4) & kLo) | (xb1 & kHi);
            uint2 r0[4], r1[4], r2[4], r3[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                r0[k] = lut(ia_e, k, lane4);
                r1[k] = lut(ia_o, k, lane4);
                r2[k] = lut(ib_e, k, lane4);
                r3[k] = lut(ib_o, k, lane4);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) mma16816(o[4 * w + k], r0[k].x, r1[k].x, r2[k].x, r3[k].x, bw[0], bw[1]);
#pragma unroll
            for (int k = 0; k < 4; ++k) mma16816(o[4 * w + k], r0[k].y, r1[k].y, r2[k].y, r3[k].y, bw[0], bw[1]);
#pragma unroll
            for (int k = 0; k < 4; ++k) mma16816(o[4 * w + k], r0[k].x, r1[k].x, r2[k].x, r3[k].x, br[0], br[1]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int i = 4 * w + k;
                if constexpr (kSplitCols)
                    mma16816(o[i], sign_bits(sA, 2 * i), sign_bits(sA, 2 * i + 1), sign_bits(sB, 2 * i),
                             sign_bits(sB, 2 * i + 1), bs[0], bs[1]);
                else
                    mma16816(o[i], sign_pair(sA, 2 * i), sign_pair(sA, 2 * i + 1), sign_pair(sB, 2 * i),
                             sign_pair(sB, 2 * i + 1), bs[0], bs[1]);
            }
        }
    }

    // One 32-token stage at `st` (two sub-tiles sharing one softmax update);
    // tokens outside [lo, hi) (offsets within the stage) are masked.
    __device__ __forceinline__ void tile(uint32_t st, int lo, int hi) {
        const VRaw v0 = load_v(st + kOffVC, st + kOffVS);
        float s0[4], s1[4];
        qk(st + kOffKC, st + kOffKS, lo, hi, s0);
        qk(st + kOffKC + kSubC, st + kOffKS + kSubS, lo - 16, hi - 16, s1);

        // mb: the running maximum, or 0 while every token so far is masked
        // (left padding), so that masked scores give p = 0, not NaN
        float corr[2], mb[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            float mx = fmaxf(fmaxf(s0[e], s0[2 + e]), fmaxf(s1[e], s1[2 + e]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mnew = fmaxf(mrun[e], mx);
            mb[e] = mnew == -INFINITY ? 0.0f : mnew;
            corr[e] = ex2(mrun[e] - mb[e]);
            mrun[e] = mnew;
        }
        float p0[4], p1[4];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            p0[e] = ex2(s0[e] - mb[e]);
            p0[2 + e] = ex2(s0[2 + e] - mb[e]);
            p1[e] = ex2(s1[e] - mb[e]);
            p1[2 + e] = ex2(s1[2 + e] - mb[e]);
        }
        // unconditional rescale (32 multiplies): no branch in the middle of
        // the stage, so the compiler schedules the whole stage as one block
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            o[i][0] *= corr[0];
            o[i][1] *= corr[1];
            o[i][2] *= corr[0];
            o[i][3] *= corr[1];
        }
        const VRaw v1 = load_v(st + kOffVC + kSubC, st + kOffVS + kSubS);
        {
            // running sum and zero-point sum (with the split columns the sign
            // s = 2b - 1 moves -valpha into the zero point)
            constexpr bool kSplitCols = G <= 4;
            const float za0 = h_hi(v0.vma.x) - (kSplitCols ? h_lo(v0.vma.y) : 0.0f);
            const float zb0 = h_hi(v0.vmb.x) - (kSplitCols ? h_lo(v0.vmb.y) : 0.0f);
            const float za1 = h_hi(v1.vma.x) - (kSplitCols ? h_lo(v1.vma.y) : 0.0f);
            const float zb1 = h_hi(v1.vmb.x) - (kSplitCols ? h_lo(v1.vmb.y) : 0.0f);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                lrun[e] = fmaf(lrun[e], corr[e], (p0[e] + p0[2 + e]) + (p1[e] + p1[2 + e]));
                zrun[e] = fmaf(zrun[e], corr[e],
                               fmaf(p0[e], za0, fmaf(p0[2 + e], zb0, fmaf(p1[e], za1, p1[2 + e] * zb1))));
            }
        }
        pv(v0, p0);
        pv(v1, p1);
    }
};


// warp that owns global tile t when T tiles are cut into NW equal ranges
// (range w = [floor(w*T/NW), floor((w+1)*T/NW)))
__host__ __device__ __forceinline__ int64_t owner_warp(int64_t t, int64_t T, int64_t NW) {
    return ((t + 1) * NW - 1) / T;
}

template <int G>
__global__ void __launch_bounds__(kThreads, 1)
decode_tma_kernel(const __grid_constant__ CUtensorMap mkc, const __grid_constant__ CUtensorMap mks,
                  const __grid_constant__ CUtensorMap mvc, const __grid_constant__ CUtensorMap mvs,
                  const __half *__restrict__ q, float *__restrict__ pm, float *__restrict__ pl,
                  float *__restrict__ po, int Hq, int Hkv, int64_t seq_len, int tpr, int64_t T, int nslots,
                  float scale_log2, int flags, const int *__restrict__ seq_len_dev,
                  const int *__restrict__ start_dev) {
    extern __shared__ __align__(1024) uint8_t sm[];
    // broadcast from lane 0 so that the compiler treats the warp index, and
    // the tile cursors derived from it, as warp-uniform values
    const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0), lane = threadIdx.x & 31;
    const uint32_t sbase = smem_u32(sm);
    if (sbase != (uint32_t)kSmemReserve) {  // the table loads assume this base
        if (threadIdx.x == 0) atomicExch(&g_device_error, 2);
        return;
    }
    uint32_t *s_cent = reinterpret_cast<uint32_t *>(sm + kSmCent);
    const uint32_t ring = sbase + kSmRing + warp * kStages * kStageBytes;
    const uint32_t bars = sbase + kSmBar + warp * kStages * 8;

    if (threadIdx.x < 16) {
        const float cv = lm(threadIdx.x);
        const __half hi = __float2half_rn(cv);
        const __half lo = __float2half_rn(cv - __half2float(hi));
        s_cent[threadIdx.x] = (uint32_t)__half_as_ushort(hi) | ((uint32_t)__half_as_ushort(lo) << 16);
    }
    if (lane == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(bars + 8 * s, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    for (int v = warp; v < 256; v += kWarps) {
        const uint32_t e0 = s_cent[v & 15], e1 = s_cent[v >> 4];
        uint2 e;
        e.x = __byte_perm(e0, e1, 0x5410);
        e.y = __byte_perm(e0, e1, 0x7632);
        reinterpret_cast<uint32_t *>(sm + kSmLut + v * 256)[lane] = e.x;
        reinterpret_cast<uint32_t *>(sm + kSmLut + v * 256 + 128)[lane] = e.y;
    }
    __syncthreads();
    pdl_trigger();
    pdl_wait();  // everything above touched shared memory only

    if (seq_len_dev) {
        // Length in device memory (a launch recorded once and replayed as the
        // context grows): seq_len, tpr, T above describe the capacity the
        // tensor maps cover; the partition is rebuilt for the current length,
        // clamped to [1, capacity].
        const int64_t rows = T / tpr;
        seq_len = max((int64_t)1, min((int64_t)*seq_len_dev, seq_len));
        tpr = (int)((seq_len + kTile - 1) / kTile);
        T = rows * tpr;
    }
    // at most one warp per tile, so that every range is non-empty and the
    // partial slots of a row have no holes
    const int64_t NW = min((int64_t)gridDim.x * kWarps, T);
    const int64_t wid = (int64_t)blockIdx.x * kWarps + warp;
    if (wid >= NW) return;
    const int64_t tbeg = wid * T / NW;
    const int ntiles = (int)((wid + 1) * T / NW - tbeg);
    const int row_tok = tpr * kTile;  // tokens of a row rounded up to whole tiles

    // Producer cursor: (token base, kv head, batch) of the next tile to issue.
    // Kept by every lane (uniform arithmetic, no divisions per tile); lane 0
    // issues.
    int p_tb, p_kvh, p_b;
    {
        const int64_t r0 = tbeg / tpr;
        p_tb = (int)(tbeg - r0 * tpr) * kTile;
        p_kvh = (int)(r0 % Hkv);
        p_b = (int)(r0 / Hkv);
    }
    auto issue_next = [&](int s) {
        if (lane == 0) {
            const uint32_t bar = bars + 8 * s, dst = ring + s * kStageBytes;
            fence_proxy_async();  // this warp's earlier reads of the stage precede the overwrite
            mbar_expect_tx(bar, kStageBytes);
            tma_4d(dst + kOffKC, &mkc, 0, p_tb, p_kvh, p_b, bar);
            tma_4d(dst + kOffKS, &mks, 64, p_tb, p_kvh, p_b, bar);
            tma_4d(dst + kOffVC, &mvc, 0, p_tb, p_kvh, p_b, bar);
            tma_4d(dst + kOffVS, &mvs, 64, p_tb, p_kvh, p_b, bar);
        }
        p_tb += kTile;
        if (p_tb >= row_tok) {
            p_tb = 0;
            if (++p_kvh == Hkv) {
                p_kvh = 0;
                ++p_b;
            }
        }
    };
    Lane<G> L;
    L.g = lane >> 2;
    L.c = lane & 3;
    // Query words of lane (g, c): dims 32c..32c+31 of query head g of the
    // group (with the split columns, G <= 4, lanes g >= 4 repeat head g - 4,
    // so that the softmax state of columns 4..7, the V sign products, is that
    // of the head they belong to); zero for heads past the group.  The first
    // segment's words are requested before the first stages, so that they do
    // not queue behind the whole grid's first tiles.
    auto load_q = [&](uint4 (&qw)[4], int64_t row) {
        const int qh = (G <= 4) ? (L.g & 3) : L.g;
        const int b_ = (int)(row / Hkv), h0_ = (int)(row % Hkv) * G;
        const uint4 *src = reinterpret_cast<const uint4 *>(q + ((int64_t)b_ * Hq + h0_ + qh) * kD + 32 * L.c);
#pragma unroll
        for (int k = 0; k < 4; ++k) qw[k] = qh < G ? __ldg(src + k) : make_uint4(0u, 0u, 0u, 0u);
    };
    {
        uint4 qw[4];
        load_q(qw, tbeg / tpr);
        for (int s = 0; s < kStages && s < ntiles; ++s) issue_next(s);
        L.set_query(qw, (flags & ECC_DECODE_ROTATE_Q) != 0);
    }

    L.lane4 = (uint32_t)lane * 4u;
    L.sel_half = (L.g & 1) ? 0x7632u : 0x5410u;
    L.voff = 16u * (uint32_t)((L.g >> 1) ^ L.c) + 8u * (uint32_t)(L.g & 1);
    L.soff = 16u * (uint32_t)((L.g >> 2) & 1);
    L.scale_log2 = scale_log2;
    bool ok = true;
    int jfail = -1;        // first tile whose wait ran out
    int j = 0;             // tiles of this warp's range consumed so far
    int stage = 0;         // ring stage of tile j
    uint32_t phase = 0;    // mbarrier parity of tile j
    int64_t r = tbeg / tpr;                  // row of tile j
    int tok0 = (int)(tbeg - r * tpr) * kTile;  // first token of tile j within its row
    while (j < ntiles) {
        // ---------------- new row segment ----------------
        const int seg_tiles = min(ntiles - j, (row_tok - tok0) / kTile);
        const bool row_ends = (tok0 + seg_tiles * kTile == row_tok);
        const int kvh = (int)(r % Hkv), b = (int)(r / Hkv);
        const int h0 = kvh * G;
        // first attended token of the sequence (left padding before it)
        const int t_start = start_dev ? __ldg(start_dev + b) : 0;
        if (j > 0) {
            uint4 qw[4];
            load_q(qw, r);
            L.set_query(qw, (flags & ECC_DECODE_ROTATE_Q) != 0);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int k = 0; k < 4; ++k) L.o[i][k] = 0.0f;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            L.mrun[e] = -INFINITY;
            L.lrun[e] = 0.0f;
            L.zrun[e] = 0.0f;
        }
        // ---------------- tiles of the segment ----------------
        for (int u = 0; u < seg_tiles; ++u) {
            // every lane polls the stage's mbarrier once (one warp-wide
            // try_wait, no divergence); a warp that does not find the phase
            // complete in every lane takes the bounded wait in lane 0
            bool ready = ok;
            if (ok && !__all_sync(0xffffffffu, mbar_try(bars + 8 * stage, phase))) {
                bool r = true;
                if (lane == 0) r = mbar_wait(bars + 8 * stage, phase);
                ready = __shfl_sync(0xffffffffu, r, 0);
            }
            __syncwarp();  // orders the warp's reads of the stage after the wait
            if (ok && !ready) jfail = j;
            ok = ok && ready;
            if (ok) L.tile(ring + stage * kStageBytes, t_start - tok0, (int)min((int64_t)kTile, seq_len - tok0));
            __syncwarp();
            if (ok && j + kStages < ntiles) issue_next(stage);
            ++j;
            tok0 += kTile;
            if (++stage == kStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
        // ---------------- partial of the segment ----------------
#pragma unroll
        for (int e = 0; e < 2; ++e) {
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                L.lrun[e] += __shfl_xor_sync(0xffffffffu, L.lrun[e], off);
                L.zrun[e] += __shfl_xor_sync(0xffffffffu, L.zrun[e], off);
            }
        }
        const int slot = (int)(wid - owner_warp(r * tpr, T, NW));
        const int64_t prow = ((int64_t)b * Hq + h0) * nslots + slot;  // partial of head h0 of the group
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            // accumulator i: rows g / g+8 = dims 16g + 2i / 16g + 2i + 1;
            // with the split columns the sign terms of heads 2c, 2c+1 are in
            // columns 4..7 of lane c + 2, each row with its power-of-two weight
            float sg[4] = {0.f, 0.f, 0.f, 0.f};
            if constexpr (G <= 4) {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    sg[k] = __shfl_down_sync(0xffffffffu, L.o[i][k], 2) * sign_unweight(k < 2 ? 2 * i : 2 * i + 1);
            }
            const int d0 = 16 * L.g + 2 * i;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int h = 2 * L.c + e;
                if (h >= G) continue;
                float2 *pod = reinterpret_cast<float2 *>(po + (prow + (int64_t)h * nslots) * kD + d0);
                *pod = make_float2(L.o[i][e] + (sg[e] + L.zrun[e]), L.o[i][2 + e] + (sg[2 + e] + L.zrun[e]));
            }
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int h = 2 * L.c + e;
            if (h >= G) continue;
            const int64_t pr = ((int64_t)b * Hq + h0 + h) * nslots;
            if (L.g == 0) {
                pm[pr + slot] = (L.mrun[e] == -INFINITY) ? -INFINITY : L.mrun[e] * kLn2f;
                pl[pr + slot] = L.lrun[e];
                if (row_ends) {  // last segment of the row: the rest are empty
                    for (int k = slot + 1; k < nslots; ++k) {
                        pm[pr + k] = -INFINITY;
                        pl[pr + k] = 0.0f;
                    }
                }
            }
        }
        if (row_ends) {
            ++r;
            tok0 = 0;
        }
    }
    if (!ok && lane == 0) {
        // drain the copies still in flight before the warp exits: tiles
        // jfail .. min(ntiles, jfail + kStages) - 1 were issued and not consumed
        for (int k = jfail; k < min(ntiles, jfail + kStages); ++k) {
            const uint32_t bar = bars + 8 * (k % kStages);
            const long long c0 = clock64();
            while (!mbar_try(bar, (uint32_t)((k / kStages) & 1)) && clock64() - c0 < kWaitCycles) {
            }
        }
    }
}

// ---- host ----
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::mutex g_encode_mu;

static int get_encode() {
    std::lock_guard<std::mutex> lk(g_encode_mu);
    if (!g_encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) != cudaSuccess ||
            qr != cudaDriverEntryPointSuccess || !fn)
            return ECC_ERR_CUDA;
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    return ECC_OK;
}

// 4-D map over a block pool: (byte in record, token, kv head, batch); rb =
// bytes per record (128, or 96 without the pad sector).  The boxes read bytes
// 0..63 and 64..95 of a record, so both sizes take the same kernel.
static int make_map(CUtensorMap *m, const void *base, int64_t seq_len, int Hkv, int B, int64_t bs_h, int64_t bs_b,
                    uint32_t box_x, int rb, CUtensorMapSwizzle swz) {
    cuuint64_t dims[4] = {(cuuint64_t)rb, (cuuint64_t)seq_len, (cuuint64_t)Hkv, (cuuint64_t)B};
    cuuint64_t sh = (cuuint64_t)bs_h * rb, sb = (cuuint64_t)bs_b * rb;
    if (Hkv == 1) sh = (cuuint64_t)seq_len * rb;  // stride of an extent-1 dim is unused
    if (B == 1) sb = sh * (cuuint64_t)Hkv;
    cuuint64_t strides[3] = {(cuuint64_t)rb, sh, sb};
    cuuint32_t box[4] = {box_x, (cuuint32_t)kTile, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void *>(base), dims, strides, box,
                                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? ECC_OK : ECC_ERR_CUDA;
}

// The four maps of a launch: K codes (64-byte rows, no swizzle: the K code
// reads are conflict-free as laid out), K syndrome + metadata (32-byte rows,
// 32-byte swizzle), V codes (64-byte swizzle), V syndrome + metadata (32-byte
// swizzle); the kernel's stage reads undo the swizzles.
static int make_maps(CUtensorMap *kc, CUtensorMap *ks, CUtensorMap *vc, CUtensorMap *vs, const void *kb,
                     const void *vb, int64_t len, int Hkv, int B, int64_t bs_h, int64_t bs_b, int rb) {
    if (make_map(kc, kb, len, Hkv, B, bs_h, bs_b, 64, rb, CU_TENSOR_MAP_SWIZZLE_NONE) != ECC_OK ||
        make_map(ks, kb, len, Hkv, B, bs_h, bs_b, 32, rb, CU_TENSOR_MAP_SWIZZLE_32B) != ECC_OK ||
        make_map(vc, vb, len, Hkv, B, bs_h, bs_b, 64, rb, CU_TENSOR_MAP_SWIZZLE_64B) != ECC_OK ||
        make_map(vs, vb, len, Hkv, B, bs_h, bs_b, 32, rb, CU_TENSOR_MAP_SWIZZLE_32B) != ECC_OK)
        return ECC_ERR_CUDA;
    return ECC_OK;
}

template <int G>
static int launch_g(const CUtensorMap &kc, const CUtensorMap &ks, const CUtensorMap &vc, const CUtensorMap &vs,
                    const void *q, float *pm, float *pl, float *po, int Hq, int Hkv, int64_t seq_len, int tpr,
                    int64_t T, int grid, int ns, float scale_log2, int flags, cudaStream_t s,
                    const int *seq_len_dev = nullptr, const int *start_dev = nullptr) {
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(decode_tma_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmBytes) !=
            cudaSuccess)
            return ECC_ERR_CUDA;
        configured[dev] = true;
    }
    if (launch_pdl(decode_tma_kernel<G>, dim3(grid), dim3(kThreads), kSmBytes, s, kc, ks, vc, vs,
                   reinterpret_cast<const __half *>(q), pm, pl, po, Hq, Hkv, seq_len, tpr, T, ns, scale_log2,
                   flags, seq_len_dev, start_dev) != cudaSuccess)
        return ECC_ERR_LAUNCH;
    return launch_status();
}

// The table loads address shared memory with kSmemReserve folded in; the
// driver reports that reserve per device.
static bool reserve_matches() {
    static int known[64];  // 0 unknown, 1 matches, 2 differs
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    if (!known[dev]) {
        int v = -1;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess) return false;
        known[dev] = (v == kSmemReserve) ? 1 : 2;
    }
    return known[dev] == 1;
}

// Grid and partial-slot count of the balanced tile partition for a shape.
struct Plan {
    int grid;
    int64_t tpr, T;
    int nslots;
};
static Plan make_plan(int B, int Hkv, int64_t seq_len) {
    Plan p;
    p.tpr = (std::max<int64_t>(seq_len, 1) + kTile - 1) / kTile;
    const int64_t rows = (int64_t)B * Hkv;
    p.T = rows * p.tpr;
    p.grid = (int)std::max<int64_t>(1, std::min<int64_t>(sm_count(), (p.T + kWarps - 1) / kWarps));
    const int64_t NW = std::min<int64_t>((int64_t)p.grid * kWarps, p.T);
    int64_t mx = 1;
    for (int64_t r = 0; r < rows; ++r) {
        const int64_t n = owner_warp(r * p.tpr + p.tpr - 1, p.T, NW) - owner_warp(r * p.tpr, p.T, NW) + 1;
        mx = std::max(mx, n);
    }
    p.nslots = (int)mx;
    return p;
}

}  // namespace tmak

// Partial slots per (b, query head) of the balanced partition: the split
// count ecc_decode uses by default.
int tma_default_splits(int B, int Hkv, int64_t seq_len) { return tmak::make_plan(B, Hkv, seq_len).nslots; }

// Returns ECC_OK when launched, a positive value when the shape is not one the
// TMA kernel handles (the caller then uses another kernel), or an error.
int launch_decode_tma(const void *q, const void *kb, const void *vb, int64_t bs_b, int64_t bs_h, float *pm,
                      float *pl, float *po, int B, int Hq, int Hkv, int64_t seq_len, int64_t chunk, int ns,
                      float scale_log2, int flags, cudaStream_t s, const int *start_dev) {
    using namespace tmak;
    (void)chunk;
    const int G = Hq / Hkv;
    if (G < 1 || G > 8 || seq_len < 1 || seq_len > (1ll << 30)) return 1;
    if (((uintptr_t)kb % 16) || ((uintptr_t)vb % 16) || ((uintptr_t)q % 16)) return 1;
    const Plan plan = make_plan(B, Hkv, seq_len);
    if (ns < plan.nslots) return 1;  // fewer partial slots than the partition writes
    if (!reserve_matches()) return 1;
    if (get_encode() != ECC_OK) return 1;
    const int rb = (flags & ECC_DECODE_BLOCK96) ? 96 : kBlockBytes;
    flags &= ECC_DECODE_ROTATE_Q;
    CUtensorMap kc, ks, vc, vs;
    if (make_maps(&kc, &ks, &vc, &vs, kb, vb, seq_len, Hkv, B, bs_h, bs_b, rb) != ECC_OK) return 1;
    switch (G) {
#define ECC_TMA_CASE(N) \
    case N: return launch_g<N>(kc, ks, vc, vs, q, pm, pl, po, Hq, Hkv, seq_len, (int)plan.tpr, plan.T, plan.grid, ns, scale_log2, flags, s, nullptr, start_dev);
        ECC_TMA_CASE(1) ECC_TMA_CASE(2) ECC_TMA_CASE(3) ECC_TMA_CASE(4)
        ECC_TMA_CASE(5) ECC_TMA_CASE(6) ECC_TMA_CASE(7)
        default: return launch_g<8>(kc, ks, vc, vs, q, pm, pl, po, Hq, Hkv, seq_len, (int)plan.tpr, plan.T, plan.grid, ns,
                                    scale_log2, flags, s, nullptr, start_dev);
#undef ECC_TMA_CASE
    }
}

// Partial slots that cover the balanced partition of every length up to
// max_len with the grid used for max_len: a row's tiles touch fewer than
// NW / rows + 2 warps (NW <= grid * kWarps), and never more than its tiles.
void tma_dev_plan(int B, int Hkv, int64_t max_len, int *grid, int *nslots) {
    using namespace tmak;
    const Plan p = make_plan(B, Hkv, max_len);
    const int64_t rows = (int64_t)B * Hkv;
    *grid = p.grid;
    *nslots = (int)std::min<int64_t>(p.tpr, (int64_t)p.grid * kWarps / rows + 2);
}

// The TMA decode with the length read from device memory at *seq_len_dev
// (clamped to [1, max_len]); tensor maps over max_len tokens.  Returns ECC_OK,
// a positive value when the shape is not one the TMA kernel handles, or an
// error.
int launch_decode_tma_dev(const void *q, const void *kb, const void *vb, int64_t bs_b, int64_t bs_h, float *pm,
                          float *pl, float *po, int B, int Hq, int Hkv, int64_t max_len, const int *seq_len_dev,
                          int ns, float scale_log2, int flags, cudaStream_t s) {
    using namespace tmak;
    const int G = Hq / Hkv;
    if (G < 1 || G > 8 || max_len < 1 || max_len > (1ll << 30)) return 1;
    if (((uintptr_t)kb % 16) || ((uintptr_t)vb % 16) || ((uintptr_t)q % 16)) return 1;
    int grid = 0, need = 0;
    tma_dev_plan(B, Hkv, max_len, &grid, &need);
    if (ns < need) return 1;
    const Plan plan = make_plan(B, Hkv, max_len);
    if (!reserve_matches()) return 1;
    if (get_encode() != ECC_OK) return 1;
    const int rb = (flags & ECC_DECODE_BLOCK96) ? 96 : kBlockBytes;
    flags &= ECC_DECODE_ROTATE_Q;
    CUtensorMap kc, ks, vc, vs;
    if (make_maps(&kc, &ks, &vc, &vs, kb, vb, max_len, Hkv, B, bs_h, bs_b, rb) != ECC_OK) return 1;
    switch (G) {
#define ECC_TMA_CASE(N) \
    case N: return launch_g<N>(kc, ks, vc, vs, q, pm, pl, po, Hq, Hkv, max_len, (int)plan.tpr, plan.T, grid, ns, scale_log2, flags, s, seq_len_dev);
        ECC_TMA_CASE(1) ECC_TMA_CASE(2) ECC_TMA_CASE(3) ECC_TMA_CASE(4)
        ECC_TMA_CASE(5) ECC_TMA_CASE(6) ECC_TMA_CASE(7)
        default: return launch_g<8>(kc, ks, vc, vs, q, pm, pl, po, Hq, Hkv, max_len, (int)plan.tpr, plan.T, grid, ns,
                                    scale_log2, flags, s, seq_len_dev);
#undef ECC_TMA_CASE
    }
}

}  // namespace ecc

namespace ecc {
namespace tmak {
// Self-test of the bounded wait: one warp arms an mbarrier for bytes that no
// copy will deliver and waits on it with mbar_wait (the decode's wait) and a
// short limit.  The wait runs out, raises the device flag and the kernel
// returns; *out = 1 when the warp saw the wait give up.
__global__ void wait_timeout_selftest_kernel(long long limit, int *out) {
    __shared__ __align__(8) uint64_t bar;
    const uint32_t b = smem_u32(&bar);
    if (threadIdx.x == 0) {
        mbar_init(b, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        mbar_expect_tx(b, 16);  // 16 bytes that never arrive: the phase never completes
    }
    __syncwarp();
    bool ok = true;
    if (threadIdx.x == 0) ok = mbar_wait(b, 0, limit);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (threadIdx.x == 0) *out = ok ? 0 : 1;
}
}  // namespace tmak
}  // namespace ecc

extern "C" int ecc_selftest_wait_timeout(long long limit_cycles, int *host_gave_up) {
    if (!host_gave_up || limit_cycles <= 0 || limit_cycles > (4ll << 30)) return ECC_ERR_SHAPE;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ECC_ERR_DEVICE;
    int *d = nullptr;
    if (cudaMalloc(&d, sizeof(int)) != cudaSuccess) return ECC_ERR_CUDA;
    ecc::tmak::wait_timeout_selftest_kernel<<<1, 32>>>(limit_cycles, d);
    int rc = ecc::launch_status();
    if (rc == ECC_OK && cudaMemcpy(host_gave_up, d, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = ECC_ERR_CUDA;
    cudaFree(d);
    return rc;
}

namespace ecc {
int compress_device_error(int reset);
int exchange_device_error(int reset);
}

extern "C" int ecc_device_status(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, ecc::g_device_error, sizeof(int)) != cudaSuccess) return ECC_ERR_CUDA;
    if (reset) {
        const int z = 0;
        if (cudaMemcpyToSymbol(ecc::g_device_error, &z, sizeof(int)) != cudaSuccess) return ECC_ERR_CUDA;
    }
    const int c = ecc::compress_device_error(reset);
    if (c < 0) return c;
    const int x = ecc::exchange_device_error(reset);
    if (x < 0) return x;
    return v ? v : (c ? c : x);
}
