// decode.cu -- fused ECC-INT4 decode attention over 128-byte blocks
// (replaces the Triton _ecc_decode_kernel of custom_kv/fused_decode.py:30 and
// the dequantise-then-SDPA step of custom_kv/patch.py:100) and the
// log-sum-exp merge of split partials.
//
// Math per (batch b, query head h, token t), kv head = h / (Hq/Hkv):
//   k_rec = C[q_t]*scale_t + zero_t + alpha_t * s_t         (fused_decode.py:229-241)
//   score = sm_scale * <q_rot, k_rec>                         (:242)
//   out   = sum_t softmax(score)_t * v_rec_t                  (:260-262)
// evaluated as split-sequence (flash-decoding) partials: each CTA owns one
// (b, kv head, split) and keeps its GQA query group resident; the merge
// combines (m, l, o) of the splits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "ecc_common.cuh"

namespace ecc {

int launch_status();
int sm_count();
int launch_decode_mma(const void *q, const void *kbp, const void *vbp, int64_t bs_b, int64_t bs_h, float *pm,
                      float *pl, float *po, int B, int Hq, int Hkv, int64_t seq_len, int64_t chunk, int ns,
                      float scale_log2, int flags, cudaStream_t s);
int launch_decode_tma(const void *q, const void *kb, const void *vb, int64_t bs_b, int64_t bs_h, float *pm,
                      float *pl, float *po, int B, int Hq, int Hkv, int64_t seq_len, int64_t chunk, int ns,
                      float scale_log2, int flags, cudaStream_t s, const int *start_dev = nullptr);
int tma_default_splits(int B, int Hkv, int64_t seq_len);
int launch_decode_tma_dev(const void *q, const void *kb, const void *vb, int64_t bs_b, int64_t bs_h, float *pm,
                          float *pl, float *po, int B, int Hq, int Hkv, int64_t max_len, const int *seq_len_dev,
                          int ns, float scale_log2, int flags, cudaStream_t s);
void tma_dev_plan(int B, int Hkv, int64_t max_len, int *grid, int *nslots);

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kV1Warps = 4;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// In-place normalised WHT of sh[0..127] by 128 threads (ascending stride,
// remainder-corrected quotient by fp32(sqrt(128)), as in compress.cu).
__device__ __forceinline__ void smem_wht128(float *sh, int d) {
    __syncthreads();
    for (int s = 1; s < kD; s <<= 1) {
        if ((d & s) == 0) {
            const float a = sh[d], b = sh[d + s];
            sh[d] = __fadd_rn(a, b);
            sh[d + s] = __fsub_rn(a, b);
        }
        __syncthreads();
    }
    const float x = sh[d];
    const float q0 = __fmul_rn(x, kInvSqrt128);
    const float rem = __fmaf_rn(-q0, kSqrt128, x);
    sh[d] = __fmaf_rn(rem, kInvSqrt128, q0);
    __syncthreads();
}

// Dequantise the 4 elements 4*lane .. 4*lane+3 of a block:
// (C[q]*scale + zero) + alpha*s in fp32.
__device__ __forceinline__ void dequant4(const uint8_t *blk, int lane, float (&r)[4]) {
    const uint32_t code16 = __ldg(reinterpret_cast<const uint16_t *>(blk + 2 * lane));
    const uint32_t syn = (__ldg(blk + kSynOff + lane / 2) >> (4 * (lane & 1))) & 0xfu;
    const uint2 meta = __ldg(reinterpret_cast<const uint2 *>(blk + kScaleOff));
    const float sc = __half2float(__ushort_as_half((unsigned short)(meta.x & 0xffffu)));
    const float zr = __half2float(__ushort_as_half((unsigned short)(meta.x >> 16)));
    const float al = __half2float(__ushort_as_half((unsigned short)(meta.y & 0xffffu)));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int q = (code16 >> (4 * j)) & 0xf;
        float c = lm(0);
#pragma unroll
        for (int k = 1; k < 16; ++k) c = (q == k) ? lm(k) : c;
        const float kt = __fadd_rn(__fmul_rn(c, sc), zr);
        r[j] = __fadd_rn(kt, ((syn >> j) & 1u) ? al : -al);
    }
}

// Reference-path kernel: CUDA cores, lane = 4 dims, each warp streams every
// fourth token of the split with an online softmax, warps merged at the end.
template <int G>
__global__ void __launch_bounds__(kV1Warps * 32)
decode_v1_kernel(const __half *__restrict__ q, const uint8_t *__restrict__ kb, const uint8_t *__restrict__ vb,
                 int64_t bs_b, int64_t bs_h, float *__restrict__ pm, float *__restrict__ pl,
                 float *__restrict__ po, int Hq, int group, int n_hchunks, int64_t seq_len, int64_t chunk,
                 int nsplit, float scale_log2, int flags) {
    const int split = blockIdx.x;
    const int kvh = blockIdx.y / n_hchunks, hc = blockIdx.y - kvh * n_hchunks;
    const int b = blockIdx.z;
    const int h0 = kvh * group + hc * G;
    const int nh = min(G, group - hc * G);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    __shared__ float sq[G][kD];
    __shared__ float s_m[kV1Warps][G], s_l[kV1Warps][G];
    __shared__ float s_o[kV1Warps][G][kD];

    for (int idx = threadIdx.x; idx < G * kD; idx += blockDim.x) {
        const int h = idx / kD, d = idx - h * kD;
        sq[h][d] = (h < nh) ? __half2float(q[((int64_t)b * Hq + h0 + h) * kD + d]) : 0.0f;
    }
    static_assert(kV1Warps * 32 == kD, "one thread per dimension for the query WHT");
    if (flags & ECC_DECODE_ROTATE_Q) {  // q_rot = fp16(WHT(q)), like patch.py:106
        for (int h = 0; h < G; ++h) {
            smem_wht128(sq[h], threadIdx.x);
            sq[h][threadIdx.x] = __half2float(__float2half_rn(sq[h][threadIdx.x]));
        }
    }
    __syncthreads();

    float qr[G][4];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
        for (int j = 0; j < 4; ++j) qr[h][j] = sq[h][4 * lane + j];

    float m[G], l[G], o[G][4];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) o[h][j] = 0.0f;
    }

    const int64_t t0 = (int64_t)split * chunk;
    const int64_t t1 = min(seq_len, t0 + chunk);
    const int64_t row_off = (int64_t)b * bs_b + (int64_t)kvh * bs_h;
    for (int64_t t = t0 + warp; t < t1; t += kV1Warps) {
        float kr[4], vr[4];
        dequant4(kb + (row_off + t) * kBlockBytes, lane, kr);
        dequant4(vb + (row_off + t) * kBlockBytes, lane, vr);
#pragma unroll
        for (int h = 0; h < G; ++h) {
            float dot = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) dot = fmaf(qr[h][j], kr[j], dot);
            const float s2 = warp_sum(dot) * scale_log2;
            const float mn = fmaxf(m[h], s2);
            const float corr = exp2f(m[h] - mn);
            const float p = exp2f(s2 - mn);
            l[h] = fmaf(l[h], corr, p);
            m[h] = mn;
#pragma unroll
            for (int j = 0; j < 4; ++j) o[h][j] = fmaf(o[h][j], corr, p * vr[j]);
        }
    }

#pragma unroll
    for (int h = 0; h < G; ++h) {
        if (lane == 0) {
            s_m[warp][h] = m[h];
            s_l[warp][h] = l[h];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) s_o[warp][h][4 * lane + j] = o[h][j];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < nh * kD; idx += blockDim.x) {
        const int h = idx / kD, d = idx - h * kD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kV1Warps; ++w) M = fmaxf(M, s_m[w][h]);
        float L = 0.0f, O = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kV1Warps; ++w) {
                const float e = exp2f(s_m[w][h] - M);
                L = fmaf(s_l[w][h], e, L);
                O = fmaf(s_o[w][h][d], e, O);
            }
        }
        const int64_t prow = (int64_t)b * Hq + h0 + h;
        const int64_t pi = prow * nsplit + split;
        po[pi * kD + d] = O;
        if (d == 0) {
            pm[pi] = (M == -INFINITY) ? -INFINITY : M * kLn2;  // natural-log units
            pl[pi] = L;
        }
    }
}

// LSE combine of n partials (m natural-log units, l, unnormalised o) of one
// row by a 128-thread block, thread d = dim d: M = max over the non-empty
// partials (l > 0; -inf if none), w_j = exp(m_j - M) (0 for empty
// partials), L = sum_j l_j w_j, O = sum_j o_j[d] w_j.  Partial j is read
// through src(j) = {m, l, o[d]}.
//   1. M: thread t takes partials t, t + 128, ...; block maximum.
//   2. Batches of 64 partials, whose o loads go out one batch ahead (two
//      register sets): threads t < 64 put w of partial c0 + t in shared
//      memory and add l w to their own running sum; every thread adds o w
//      of the batch into four accumulators (partial j into j mod 4).
//   3. O = (a0 + a1) + (a2 + a3); L = the 64 running sums reduced by the
//      fixed tree of lse_block_sum64.
// Every step has a fixed order, so the result does not depend on timing,
// and the record merge of the peer exchange (lse_exchange_kernel) uses the
// same helpers so that it equals this function bit for bit.
constexpr int kLseBatch = 64;
static_assert(kLseBatch <= kD, "one thread per partial of a batch");

__device__ __forceinline__ float lse_weight(float m, float l, float M) {
    return (l > 0.0f && M != -INFINITY) ? __expf(m - M) : 0.0f;
}
// o * w with the empty partials' o (possibly never written) left out
__device__ __forceinline__ float lse_term(float o, float w, float acc) { return w != 0.0f ? fmaf(o, w, acc) : acc; }

// Maximum of v over the block's 128 threads (every thread gets it).
__device__ __forceinline__ float lse_block_max(float v, float *red) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    const float r = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();  // red is reused
    return r;
}
// Sum of v over threads 0..63 (the others' v ignored), in one fixed order:
// a shfl_down tree within each of warps 0 and 1, then warp 0 + warp 1.
__device__ __forceinline__ float lse_block_sum64(float v, float *red) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0 || threadIdx.x == 32) red[threadIdx.x >> 5] = v;
    __syncthreads();
    const float r = red[0] + red[1];
    __syncthreads();  // red is reused
    return r;
}

template <class Src>
__device__ __forceinline__ void lse_combine(int n, int d, const Src &src, float &M, float &L, float &O) {
    __shared__ float s_w[kLseBatch];
    __shared__ float s_red[kD / 32];
    float mx = -INFINITY;
    for (int j = d; j < n; j += kD)
        if (src.l(j) > 0.0f) mx = fmaxf(mx, src.m(j));
    M = lse_block_max(mx, s_red);

    float ov[kLseBatch], mv = 0.0f, lv = 0.0f;
    auto fetch = [&](int c0, float (&o)[kLseBatch], float &m, float &l) {
        const int cn = min(kLseBatch, n - c0);
#pragma unroll
        for (int j = 0; j < kLseBatch; ++j) o[j] = (j < cn) ? src.o(c0 + j, d) : 0.0f;
        if (d < cn) {
            m = src.m(c0 + d);
            l = src.l(c0 + d);
        }
    };
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f, lw = 0.0f;
    if (n > 0) fetch(0, ov, mv, lv);
    for (int c0 = 0; c0 < n; c0 += kLseBatch) {
        const int cn = min(kLseBatch, n - c0);
        if (d < kLseBatch) {
            const float w = d < cn ? lse_weight(mv, lv, M) : 0.0f;
            s_w[d] = w;
            if (d < cn) lw = fmaf(lv, w, lw);
        }
        float nv[kLseBatch];
        float nm = 0.0f, nl = 0.0f;
        if (c0 + kLseBatch < n) fetch(c0 + kLseBatch, nv, nm, nl);  // block-uniform
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kLseBatch; j += 4) {
            a0 = lse_term(ov[j], s_w[j], a0);
            a1 = lse_term(ov[j + 1], s_w[j + 1], a1);
            a2 = lse_term(ov[j + 2], s_w[j + 2], a2);
            a3 = lse_term(ov[j + 3], s_w[j + 3], a3);
        }
        __syncthreads();  // s_w is refilled next
        if (c0 + kLseBatch < n) {
#pragma unroll
            for (int j = 0; j < kLseBatch; ++j) ov[j] = nv[j];
            mv = nm;
            lv = nl;
        }
    }
    O = (a0 + a1) + (a2 + a3);
    L = lse_block_sum64(lw, s_red);
}

// Split partials of one row: m, l [row][n], o [row][n][128].
struct SplitSrc {
    const float *pm, *pl, *po;
    int64_t row;
    int n;
    __device__ float m(int i) const { return pm[row * n + i]; }
    __device__ float l(int i) const { return pl[row * n + i]; }
    __device__ float o(int i, int d) const { return po[(row * n + i) * kD + d]; }
};
// Records {m, l, o[128]} of one row, record i at rec + i * stride + row * kRec.
constexpr int kRec = 2 + kD;
struct RecordSrc {
    const float *rec;
    int64_t row, stride;
    __device__ const float *at(int i) const { return rec + i * stride + row * kRec; }
    __device__ float m(int i) const { return at(i)[0]; }
    __device__ float l(int i) const { return at(i)[1]; }
    __device__ float o(int i, int d) const { return at(i)[2 + d]; }
};

__device__ __forceinline__ void write_out(float L, float O, __half *out, int64_t row, int d, int flags, float *sh) {
    float val = (L > 0.0f) ? O / L : 0.0f;
    if (flags & ECC_DECODE_UNROTATE_OUT) {
        sh[d] = val;
        smem_wht128(sh, d);
        val = sh[d];
    }
    out[row * kD + d] = __float2half_rn(val);
}

// Merge n partials per row; 128 threads = 128 dims.
__global__ void __launch_bounds__(kD)
lse_merge_kernel(const float *__restrict__ pm, const float *__restrict__ pl, const float *__restrict__ po,
                 int n, __half *__restrict__ out, int flags) {
    __shared__ float sh[kD];
    pdl_trigger();
    pdl_wait();
    float M, L, O;
    lse_combine(n, threadIdx.x, SplitSrc{pm, pl, po, (int64_t)blockIdx.x, n}, M, L, O);
    write_out(L, O, out, blockIdx.x, threadIdx.x, flags, sh);
}

// Merge n partials per row into one record {M, L, O[128]} (still a partial).
__global__ void __launch_bounds__(kD)
lse_merge_record_kernel(const float *__restrict__ pm, const float *__restrict__ pl, const float *__restrict__ po,
                        int n, float *__restrict__ rec) {
    float M, L, O;
    const int64_t row = blockIdx.x;
    lse_combine(n, threadIdx.x, SplitSrc{pm, pl, po, row, n}, M, L, O);
    float *r = rec + row * kRec;
    if (threadIdx.x == 0) {
        r[0] = M;
        r[1] = L;
    }
    r[2 + threadIdx.x] = O;
}

// Merge n records per row (record i of row r at rec + i * stride + r * kRec).
__global__ void __launch_bounds__(kD)
lse_merge_records_kernel(const float *__restrict__ rec, int n, int64_t stride, __half *__restrict__ out, int flags) {
    __shared__ float sh[kD];
    float M, L, O;
    lse_combine(n, threadIdx.x, RecordSrc{rec, (int64_t)blockIdx.x, stride}, M, L, O);
    write_out(L, O, out, blockIdx.x, threadIdx.x, flags, sh);
}

// ---------------------------------------------------------------------------
// Record exchange over peer memory (sequence-sharded decode, one GPU per
// rank, no NCCL): one kernel per rank and step does the two-level combine of
// lse_merge_record_kernel -> all-gather -> lse_merge_records_kernel.
//
// Every rank owns an exchange buffer that all ranks can store to (a CUDA IPC
// mapping on each peer): records [2][W][rows][kRec] of 64-bit words, each
// word = (epoch << 32) | bits of one float of the record.  Call e (epoch
// e >= 1, the same sequence on every rank) uses half p = e & 1.  The CTA of
// row r on rank s merges its split partials into the row's record and
// stores it into slot [p][s][r] of every rank's buffer with single 64-bit
// stores; it then reads slot [p][q][r] of its own buffer for every rank q,
// polling each word until its tag is e (a word is written by one store, so a
// word with the right tag carries that call's value: no fence and no
// separate flag), and merges the W records with the arithmetic of
// lse_combine.  A CTA depends only on the CTAs of the same row on other GPUs,
// and every CTA of the grid can be resident at once (the grid is capped by
// the kernel's occupancy times the SM count; a CTA takes rows r = b,
// b + grid, ...).  The kernel is a programmatic dependent of the one before
// it (its launch overlaps that kernel's tail; its CTAs start work after
// griddepcontrol.wait) and never lets a dependent of its own start early, so
// once the previous kernel has ended nothing else holds the SMs and no CTA
// waits for one that cannot run.  Half p is reused two calls later: a rank
// can only start call e + 2 after every rank's records of call e + 1
// arrived, which each rank stores after its call-e kernel has ended.  The
// wait is bounded; a CTA that gives up raises g_exchange_error
// (ecc_device_status reports 4) and its rows' output is not valid.
// ---------------------------------------------------------------------------
constexpr int kExchMaxRanks = ECC_EXCHANGE_MAX_RANKS;
constexpr int kExchMaxGrid = 1024;
struct PeerBufs {
    unsigned long long *base[kExchMaxRanks];
};
__device__ int g_exchange_error;

__device__ __forceinline__ void st_relaxed_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long tag(float v, uint32_t epoch) {
    return ((unsigned long long)epoch << 32) | __float_as_uint(v);
}
// Poll one word until it carries `epoch` or the deadline passes (then the
// device flag is raised and *ok cleared); returns its float.
__device__ __forceinline__ float await_word(const unsigned long long *p, unsigned long long w, uint32_t epoch,
                                            long long t0, long long wait_cycles, bool *ok) {
    while ((uint32_t)(w >> 32) != epoch) {
        if (clock64() - t0 > wait_cycles) {
            atomicExch(&g_exchange_error, 4);
            *ok = false;
            break;
        }
        w = ld_relaxed_sys(p);
    }
    return __uint_as_float((uint32_t)w);
}

// Epoch of an exchange call.  Host epochs come as a kernel argument.  With a
// device-side epoch state {counter, done} (calls recorded in a CUDA graph,
// whose arguments are fixed) the epoch is counter % (2^32 - 2) + 1, read after
// the previous kernel: never 0, consecutive calls alternate parity (the
// buffer half).  The last CTA to finish advances the counter -- every CTA
// read it before it counts itself done -- so the next call, ordered after
// this kernel, gets the next epoch.
__device__ __forceinline__ uint32_t call_epoch(uint32_t epoch, const unsigned long long *state) {
    if (!state) return epoch;
    return (uint32_t)(*reinterpret_cast<const volatile unsigned long long *>(state) % 0xFFFFFFFEull) + 1u;
}
__device__ __forceinline__ void advance_epoch(unsigned long long *state) {
    if (!state) return;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(state + 1, 1ull) == (unsigned long long)gridDim.x - 1ull) {
            state[1] = 0ull;
            atomicAdd(state, 1ull);
        }
    }
}

__global__ void __launch_bounds__(kD)
lse_exchange_kernel(const float *__restrict__ pm, const float *__restrict__ pl, const float *__restrict__ po, int n,
                    int64_t rows, int W, int rank, PeerBufs peers, uint32_t epoch_arg, unsigned long long *estate,
                    long long wait_cycles, __half *__restrict__ out, int flags) {
    __shared__ float sh[kD];
    __shared__ float s_m[kExchMaxRanks], s_l[kExchMaxRanks];
    __shared__ float s_w[kLseBatch], s_red[kD / 32];
    const int d = threadIdx.x;
    pdl_wait();  // the partials of the kernel before
    const uint32_t epoch = call_epoch(epoch_arg, estate);
    const int64_t half = epoch & 1u;
    // 1. this rank's record of each row, stored into every rank's buffer
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        float M, L, O;
        lse_combine(n, d, SplitSrc{pm, pl, po, r, n}, M, L, O);
        for (int q = 0; q < W; ++q) {
            unsigned long long *dst = peers.base[q] + ((half * W + rank) * rows + r) * kRec;
            if (d == 0) {
                st_relaxed_sys(dst, tag(M, epoch));
                st_relaxed_sys(dst + 1, tag(L, epoch));
            }
            st_relaxed_sys(dst + 2 + d, tag(O, epoch));
        }
    }
    // 2. every rank's record of each row: the words of all ranks are loaded
    // together, then those not yet carrying this epoch are polled
    const unsigned long long *mine = peers.base[rank] + half * W * rows * kRec;
    const long long t0 = clock64();
    bool ok = true;
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        unsigned long long w[kExchMaxRanks];
        float ov[kExchMaxRanks];
#pragma unroll
        for (int q = 0; q < kExchMaxRanks; ++q)
            if (q < W) w[q] = ld_relaxed_sys(mine + ((int64_t)q * rows + r) * kRec + 2 + d);
        if (d < 2 * W) {  // threads 0..W-1 fetch m of rank d, W..2W-1 l of rank d - W
            const int q = d < W ? d : d - W;
            const unsigned long long *p = mine + ((int64_t)q * rows + r) * kRec + (d < W ? 0 : 1);
            const float v = await_word(p, ld_relaxed_sys(p), epoch, t0, wait_cycles, &ok);
            (d < W ? s_m : s_l)[q] = v;
        }
#pragma unroll
        for (int q = 0; q < kExchMaxRanks; ++q)
            if (q < W) ov[q] = await_word(mine + ((int64_t)q * rows + r) * kRec + 2 + d, w[q], epoch, t0,
                                          wait_cycles, &ok);
        __syncthreads();
        // lse_combine's arithmetic over the W records (bit for bit): the
        // same maximum, weights, accumulator assignment and sum tree
        const float M = lse_block_max((d < W && s_l[d] > 0.0f) ? s_m[d] : -INFINITY, s_red);
        float lw = 0.0f;
        if (d < kLseBatch) {
            const float wt = d < W ? lse_weight(s_m[d], s_l[d], M) : 0.0f;
            s_w[d] = wt;
            if (d < W) lw = fmaf(s_l[d], wt, lw);
        }
        __syncthreads();
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int j = 0; j < kExchMaxRanks; ++j)
            if (j < W) acc[j & 3] = lse_term(ov[j], s_w[j], acc[j & 3]);
        const float O = (acc[0] + acc[1]) + (acc[2] + acc[3]);
        const float L = lse_block_sum64(lw, s_red);  // its barriers also end this row's reads of s_m, s_l, s_w
        write_out(L, O, out, r, d, flags, sh);
    }
    advance_epoch(estate);
}

// ---------------------------------------------------------------------------
// Output gather over peer memory (kv-head-sharded decode, one GPU per rank):
// rank s holds kv heads [s*Hkv/W, (s+1)*Hkv/W) of every sequence and computes
// the outputs of their hq_l query heads.  One kernel per rank and step does
// the merge of the rank's split partials and the all-gather of the ranks'
// fp16 outputs.  The CTA of local row r = (b, j) merges row r's partials
// (lse_combine, write_out's arithmetic), writes the fp16 row at its place in
// this rank's full output [B, W*hq_l, 128] (query head s*hq_l + j) and
// stores it into slot [p][s][r] of every other rank's buffer as 64 words
// (epoch << 32 | two fp16, one store each, the protocol of
// lse_exchange_kernel); then it polls slot [p][q][r] of its own buffer for
// every other rank q until each word carries this epoch and writes rank q's
// row (b, q*hq_l + j).  A CTA waits only for the CTAs of the same local row
// on the other GPUs (every rank has the same rows), the grid is capped by
// residency, and the wait is bounded (then g_exchange_error = 4).
// ---------------------------------------------------------------------------
constexpr int kGatherWords = kD / 2;

__global__ void __launch_bounds__(kD)
lse_gather_kernel(const float *__restrict__ pm, const float *__restrict__ pl, const float *__restrict__ po, int n,
                  int64_t rows, int hq_l, int W, int rank, PeerBufs peers, uint32_t epoch_arg,
                  unsigned long long *estate, long long wait_cycles, __half *__restrict__ out, int flags) {
    __shared__ float sh[kD];
    const int d = threadIdx.x;
    pdl_wait();  // the partials of the kernel before
    const uint32_t epoch = call_epoch(epoch_arg, estate);
    const int64_t half = epoch & 1u;
    const unsigned long long *mine = peers.base[rank] + half * W * rows * kGatherWords;
    const long long t0 = clock64();
    bool ok = true;
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        float M, L, O;
        lse_combine(n, d, SplitSrc{pm, pl, po, r, n}, M, L, O);
        float val = (L > 0.0f) ? O / L : 0.0f;
        if (flags & ECC_DECODE_UNROTATE_OUT) {
            sh[d] = val;
            smem_wht128(sh, d);
            val = sh[d];
        }
        const uint32_t hb = __half_as_ushort(__float2half_rn(val));
        const int64_t b = r / hq_l, j = r - b * hq_l;
        const int64_t stride_q = (int64_t)hq_l * kD;  // one rank's heads of a sequence
        __half *orow = out + (b * W * hq_l + j) * kD;   // rank q's row: orow + q * stride_q
        orow[rank * stride_q + d] = __ushort_as_half((unsigned short)hb);
        const uint32_t hi = __shfl_down_sync(0xffffffffu, hb, 1);
        if ((d & 1) == 0) {
            const unsigned long long tw = ((unsigned long long)epoch << 32) | (hb | (hi << 16));
            for (int q = 0; q < W; ++q)
                if (q != rank)
                    st_relaxed_sys(peers.base[q] + ((half * W + rank) * rows + r) * kGatherWords + (d >> 1), tw);
        }
        // the other ranks' rows: thread d < 64 takes word d of each (its two dims)
        if (d < kGatherWords) {
            unsigned long long w[kExchMaxRanks];
#pragma unroll
            for (int q = 0; q < kExchMaxRanks; ++q)
                if (q < W && q != rank) w[q] = ld_relaxed_sys(mine + ((int64_t)q * rows + r) * kGatherWords + d);
#pragma unroll
            for (int q = 0; q < kExchMaxRanks; ++q)
                if (q < W && q != rank) {
                    const unsigned long long *src = mine + ((int64_t)q * rows + r) * kGatherWords + d;
                    const uint32_t v = __float_as_uint(await_word(src, w[q], epoch, t0, wait_cycles, &ok));
                    reinterpret_cast<uint32_t *>(orow + q * stride_q)[d] = v;
                }
        }
        __syncthreads();  // sh is refilled for the next row
    }
    advance_epoch(estate);
}

int exchange_device_error(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_exchange_error, sizeof(int)) != cudaSuccess) return ECC_ERR_CUDA;
    if (reset) {
        const int z = 0;
        if (cudaMemcpyToSymbol(g_exchange_error, &z, sizeof(int)) != cudaSuccess) return ECC_ERR_CUDA;
    }
    return v;
}

}  // namespace ecc

using namespace ecc;

static inline bool aligned(const void *p, size_t a) { return ((uintptr_t)p % a) == 0; }

// Driver entry points looked up through the runtime (no link against
// libcuda): the current context, and the size of the allocation that
// contains an address.
template <class Fn>
static Fn driver_fn(const char *name) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &qr) != cudaSuccess ||
        qr != cudaDriverEntryPointSuccess)
        return nullptr;
    return reinterpret_cast<Fn>(fn);
}

static CUcontext current_context() {
    static const auto fn = driver_fn<PFN_cuCtxGetCurrent_v4000>("cuCtxGetCurrent");
    CUcontext c = nullptr;
    if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
    return c;
}

static size_t allocation_bytes(const void *p) {
    static const auto fn = driver_fn<PFN_cuMemGetAddressRange_v3020>("cuMemGetAddressRange");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (!fn || fn(&base, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) return 0;
    // bytes from p to the end of its allocation
    return size - (size_t)(reinterpret_cast<CUdeviceptr>(p) - base);
}

static inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

extern "C" int ecc_decode_default_splits(int B, int Hkv, int64_t seq_len) {
    if (B <= 0 || Hkv <= 0 || seq_len <= 0) return 1;
    return tma_default_splits(B, Hkv, seq_len);
}

// Split count and tokens per split.  Default (num_splits <= 0): the partial
// slots of the TMA kernel's balanced partition, kept as is so that the
// partial layout is the one that kernel writes (the register kernel then
// runs one split per slot, trailing ones possibly empty).  Explicit counts
// are rounded to whole 64-token tiles per split.
static int effective_splits(int B, int Hkv, int64_t seq_len, int num_splits, int64_t *chunk_out) {
    const int64_t L = std::max<int64_t>(seq_len, 1);
    if (num_splits <= 0) {
        const int ns = ecc_decode_default_splits(B, Hkv, seq_len);
        if (chunk_out) *chunk_out = cdiv(cdiv(L, ns), 64) * 64;
        return ns;
    }
    int ns = num_splits;
    int64_t chunk = cdiv(cdiv(L, ns), 64) * 64;  // whole 64-token tiles per split
    ns = (int)std::max<int64_t>(1, cdiv(L, chunk));
    if (chunk_out) *chunk_out = chunk;
    return ns;
}

extern "C" size_t ecc_decode_workspace_size(int B, int Hq, int Hkv, int64_t seq_len, int num_splits) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0) return 0;
    const int ns = effective_splits(B, Hkv, seq_len, num_splits, nullptr);
    const size_t parts = (size_t)B * Hq * ns;
    return parts * sizeof(float) * (2 + kD) + 256;
}

static int check_decode_args(const void *q, const void *kb, const void *vb, int B, int Hq, int Hkv,
                             int64_t seq_len) {
    if (!q || !kb || !vb) return ECC_ERR_NULL;
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || seq_len < 0) return ECC_ERR_SHAPE;
    if (Hq % Hkv) return ECC_ERR_GQA;
    if (!aligned(q, 16) || !aligned(kb, 16) || !aligned(vb, 16)) return ECC_ERR_ALIGN;
    return ECC_OK;
}

template <int G>
static void launch_v1(const void *q, const void *kb, const void *vb, int64_t bs_b, int64_t bs_h, float *pm,
                      float *pl, float *po, int B, int Hq, int Hkv, int64_t seq_len, int64_t chunk, int ns,
                      float scale_log2, int flags, cudaStream_t s) {
    const int group = Hq / Hkv;
    const int n_hchunks = (group + G - 1) / G;
    dim3 grid(ns, Hkv * n_hchunks, B);
    decode_v1_kernel<G><<<grid, kV1Warps * 32, 0, s>>>(
        reinterpret_cast<const __half *>(q), reinterpret_cast<const uint8_t *>(kb),
        reinterpret_cast<const uint8_t *>(vb), bs_b, bs_h, pm, pl, po, Hq, group, n_hchunks, seq_len, chunk, ns,
        scale_log2, flags);
}

static int run_partials(const void *q, const void *kb, const void *vb, int64_t bs_b, int64_t bs_h, float *pm,
                        float *pl, float *po, int B, int Hq, int Hkv, int64_t seq_len, int64_t chunk, int ns,
                        float sm_scale, int flags, cudaStream_t s) {
    if (!(sm_scale > 0.0f)) sm_scale = 1.0f / std::sqrt((float)kD);
    const float scale_log2 = sm_scale * kLog2e;
    const int group = Hq / Hkv;
    if (flags & ECC_DECODE_BLOCK96) {  // 96-byte records: the TMA-fed kernel only
        if (group > 8 || (flags & (ECC_DECODE_CUDA_CORES | ECC_DECODE_REGISTER_PATH))) return ECC_ERR_SHAPE;
        const int rc = launch_decode_tma(q, kb, vb, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns,
                                         scale_log2, flags & (ECC_DECODE_ROTATE_Q | ECC_DECODE_BLOCK96), s);
        return rc > 0 ? ECC_ERR_SHAPE : rc;
    }
    if (group <= 8 && !(flags & ECC_DECODE_CUDA_CORES)) {
        if (!(flags & ECC_DECODE_REGISTER_PATH)) {
            const int rc = launch_decode_tma(q, kb, vb, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns,
                                             scale_log2, flags & ECC_DECODE_ROTATE_Q, s);
            if (rc <= 0) return rc;  // launched (or failed); > 0: shape not handled, use the register path
        }
        const int rc = launch_decode_mma(q, kb, vb, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns,
                                         scale_log2, flags & ECC_DECODE_ROTATE_Q, s);
        return rc != ECC_OK ? rc : launch_status();
    }
    if (group == 1)
        launch_v1<1>(q, kb, vb, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns, scale_log2, flags, s);
    else if (group == 2)
        launch_v1<2>(q, kb, vb, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns, scale_log2, flags, s);
    else if (group <= 4)
        launch_v1<4>(q, kb, vb, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns, scale_log2, flags, s);
    else
        launch_v1<8>(q, kb, vb, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns, scale_log2, flags, s);
    return launch_status();
}

extern "C" int ecc_decode_partials(const void *q_f16, const void *k_blocks, const void *v_blocks, int64_t bs_b,
                                   int64_t bs_h, float *part_m, float *part_l, float *part_o, int B, int Hq,
                                   int Hkv, int64_t seq_len, float sm_scale, int flags, int num_splits,
                                   ecc_stream_t stream) {
    int rc = check_decode_args(q_f16, k_blocks, v_blocks, B, Hq, Hkv, seq_len);
    if (rc != ECC_OK) return rc;
    if (!part_m || !part_l || !part_o) return ECC_ERR_NULL;
    if (num_splits <= 0) return ECC_ERR_SHAPE;  // the caller sizes the partial arrays
    int64_t chunk = 0;
    const int ns = effective_splits(B, Hkv, seq_len, num_splits, &chunk);
    if (ns != num_splits) {
        // a split would be empty of whole tiles; keep the caller's count and
        // let trailing splits come out empty (l = 0)
        chunk = cdiv(cdiv(std::max<int64_t>(seq_len, 1), num_splits), 64) * 64;
    }
    return run_partials(q_f16, k_blocks, v_blocks, bs_b, bs_h, part_m, part_l, part_o, B, Hq, Hkv, seq_len, chunk,
                        num_splits, sm_scale, flags & (ECC_DECODE_ROTATE_Q | ECC_DECODE_CUDA_CORES | ECC_DECODE_REGISTER_PATH | ECC_DECODE_BLOCK96),
                        reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ecc_lse_merge(const float *part_m, const float *part_l, const float *part_o, int64_t rows, int n,
                             void *out_f16, int flags, ecc_stream_t stream) {
    if (rows < 0 || n <= 0) return ECC_ERR_SHAPE;
    if (rows == 0) return ECC_OK;
    if (!part_m || !part_l || !part_o || !out_f16) return ECC_ERR_NULL;
    if (rows > 0x7fffffff) return ECC_ERR_SHAPE;
    if (launch_pdl(lse_merge_kernel, dim3((unsigned)rows), dim3(kD), 0, reinterpret_cast<cudaStream_t>(stream),
                   part_m, part_l, part_o, n, reinterpret_cast<__half *>(out_f16), flags) != cudaSuccess)
        return ECC_ERR_LAUNCH;
    return launch_status();
}

extern "C" int ecc_lse_merge_to_record(const float *part_m, const float *part_l, const float *part_o, int64_t rows,
                                       int n, float *records, ecc_stream_t stream) {
    if (rows < 0 || n <= 0) return ECC_ERR_SHAPE;
    if (rows == 0) return ECC_OK;
    if (!part_m || !part_l || !part_o || !records) return ECC_ERR_NULL;
    if (rows > 0x7fffffff) return ECC_ERR_SHAPE;
    lse_merge_record_kernel<<<(unsigned)rows, kD, 0, reinterpret_cast<cudaStream_t>(stream)>>>(part_m, part_l,
                                                                                              part_o, n, records);
    return launch_status();
}

extern "C" int ecc_lse_merge_records(const float *records, int64_t rows, int n, int64_t record_stride, void *out_f16,
                                     int flags, ecc_stream_t stream) {
    if (rows < 0 || n <= 0 || record_stride < 0) return ECC_ERR_SHAPE;
    if (rows == 0) return ECC_OK;
    if (!records || !out_f16) return ECC_ERR_NULL;
    if (rows > 0x7fffffff) return ECC_ERR_SHAPE;
    if (n > 1 && record_stride < rows * kRec) return ECC_ERR_SHAPE;  // record sets may not overlap
    lse_merge_records_kernel<<<(unsigned)rows, kD, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        records, n, record_stride, reinterpret_cast<__half *>(out_f16), flags);
    return launch_status();
}

extern "C" int ecc_decode(const void *q_f16, const void *k_blocks, const void *v_blocks, int64_t bs_b, int64_t bs_h,
                          void *out_f16, void *workspace, size_t workspace_bytes, int B, int Hq, int Hkv,
                          int64_t seq_len, float sm_scale, int flags, int num_splits, ecc_stream_t stream) {
    int rc = check_decode_args(q_f16, k_blocks, v_blocks, B, Hq, Hkv, seq_len);
    if (rc != ECC_OK) return rc;
    if (!out_f16) return ECC_ERR_NULL;
    const size_t need = ecc_decode_workspace_size(B, Hq, Hkv, seq_len, num_splits);
    if (!workspace || workspace_bytes < need) return ECC_ERR_WORKSPACE;
    int64_t chunk = 0;
    const int ns = effective_splits(B, Hkv, seq_len, num_splits, &chunk);
    const size_t parts = (size_t)B * Hq * ns;
    uintptr_t base = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~(uintptr_t)255;
    float *po = reinterpret_cast<float *>(base);
    float *pm = po + parts * kD;
    float *pl = pm + parts;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    rc = run_partials(q_f16, k_blocks, v_blocks, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns, sm_scale,
                      flags & (ECC_DECODE_ROTATE_Q | ECC_DECODE_CUDA_CORES | ECC_DECODE_REGISTER_PATH | ECC_DECODE_BLOCK96), s);
    if (rc != ECC_OK) return rc;
    return ecc_lse_merge(pm, pl, po, (int64_t)B * Hq, ns, out_f16, flags & ECC_DECODE_UNROTATE_OUT, stream);
}

// ---------------------------------------------------------------------------
// Decode of left-padded batches: sequence b attends to tokens
// [start_dev[b], seq_len) only.  The tokens before start_dev[b] are padding
// that a batched prompt put in front of the shorter sequences; they are in
// the pools (the prefill compressed them) but the attention mask excludes
// them.  TMA-fed kernel only (GQA groups up to 8, pools a tensor map can
// describe), with its default partition; the workspace is the one ecc_decode
// needs with num_splits = 0.
// ---------------------------------------------------------------------------
extern "C" int ecc_decode_masked(const void *q_f16, const void *k_blocks, const void *v_blocks, int64_t bs_b,
                                 int64_t bs_h, const int *start_dev, void *out_f16, void *workspace,
                                 size_t workspace_bytes, int B, int Hq, int Hkv, int64_t seq_len, float sm_scale,
                                 int flags, ecc_stream_t stream) {
    int rc = check_decode_args(q_f16, k_blocks, v_blocks, B, Hq, Hkv, seq_len);
    if (rc != ECC_OK) return rc;
    if (!out_f16 || !start_dev) return ECC_ERR_NULL;
    if (seq_len < 1 || Hq / Hkv > 8 || (flags & (ECC_DECODE_CUDA_CORES | ECC_DECODE_REGISTER_PATH)))
        return ECC_ERR_SHAPE;
    const size_t need = ecc_decode_workspace_size(B, Hq, Hkv, seq_len, 0);
    if (!workspace || workspace_bytes < need) return ECC_ERR_WORKSPACE;
    int64_t chunk = 0;
    const int ns = effective_splits(B, Hkv, seq_len, 0, &chunk);
    const size_t parts = (size_t)B * Hq * ns;
    uintptr_t base = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~(uintptr_t)255;
    float *po = reinterpret_cast<float *>(base);
    float *pm = po + parts * kD;
    float *pl = pm + parts;
    if (!(sm_scale > 0.0f)) sm_scale = 1.0f / std::sqrt((float)kD);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    rc = launch_decode_tma(q_f16, k_blocks, v_blocks, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, seq_len, chunk, ns,
                           sm_scale * kLog2e, flags & (ECC_DECODE_ROTATE_Q | ECC_DECODE_BLOCK96), s, start_dev);
    if (rc > 0) return ECC_ERR_SHAPE;  // a pool layout the tensor-map kernel does not take
    if (rc != ECC_OK) return rc;
    return ecc_lse_merge(pm, pl, po, (int64_t)B * Hq, ns, out_f16, flags & ECC_DECODE_UNROTATE_OUT, stream);
}

// ---------------------------------------------------------------------------
// Decode with the context length in device memory, for launches recorded once
// in a CUDA graph and replayed while the context grows.
// ---------------------------------------------------------------------------
extern "C" size_t ecc_decode_dev_workspace_size(int B, int Hq, int Hkv, int64_t max_len) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || max_len <= 0) return 0;
    int grid = 0, ns = 0;
    tma_dev_plan(B, Hkv, max_len, &grid, &ns);
    return (size_t)B * Hq * ns * sizeof(float) * (2 + kD) + 256;
}

extern "C" int ecc_decode_dev_splits(int B, int Hkv, int64_t max_len) {
    if (B <= 0 || Hkv <= 0 || max_len <= 0) return 0;
    int grid = 0, ns = 0;
    tma_dev_plan(B, Hkv, max_len, &grid, &ns);
    return ns;
}

extern "C" int ecc_decode_partials_dev(const void *q_f16, const void *k_blocks, const void *v_blocks, int64_t bs_b,
                                       int64_t bs_h, float *part_m, float *part_l, float *part_o, int B, int Hq,
                                       int Hkv, int64_t max_len, const int *seq_len_dev, float sm_scale, int flags,
                                       int num_splits, ecc_stream_t stream) {
    int rc = check_decode_args(q_f16, k_blocks, v_blocks, B, Hq, Hkv, max_len);
    if (rc != ECC_OK) return rc;
    if (!part_m || !part_l || !part_o || !seq_len_dev) return ECC_ERR_NULL;
    if (max_len < 1 || Hq / Hkv > 8 || num_splits < ecc_decode_dev_splits(B, Hkv, max_len)) return ECC_ERR_SHAPE;
    if (!(sm_scale > 0.0f)) sm_scale = 1.0f / std::sqrt((float)kD);
    rc = launch_decode_tma_dev(q_f16, k_blocks, v_blocks, bs_b, bs_h, part_m, part_l, part_o, B, Hq, Hkv, max_len,
                               seq_len_dev, num_splits, sm_scale * kLog2e, flags & (ECC_DECODE_ROTATE_Q | ECC_DECODE_BLOCK96),
                               reinterpret_cast<cudaStream_t>(stream));
    return rc > 0 ? ECC_ERR_SHAPE : rc;
}

extern "C" int ecc_decode_dev(const void *q_f16, const void *k_blocks, const void *v_blocks, int64_t bs_b,
                              int64_t bs_h, void *out_f16, void *workspace, size_t workspace_bytes, int B, int Hq,
                              int Hkv, int64_t max_len, const int *seq_len_dev, float sm_scale, int flags,
                              ecc_stream_t stream) {
    int rc = check_decode_args(q_f16, k_blocks, v_blocks, B, Hq, Hkv, max_len);
    if (rc != ECC_OK) return rc;
    if (!out_f16 || !seq_len_dev) return ECC_ERR_NULL;
    if (max_len < 1 || Hq / Hkv > 8) return ECC_ERR_SHAPE;
    const size_t need = ecc_decode_dev_workspace_size(B, Hq, Hkv, max_len);
    if (!workspace || workspace_bytes < need) return ECC_ERR_WORKSPACE;
    int grid = 0, ns = 0;
    tma_dev_plan(B, Hkv, max_len, &grid, &ns);
    const size_t parts = (size_t)B * Hq * ns;
    uintptr_t base = (reinterpret_cast<uintptr_t>(workspace) + 255) & ~(uintptr_t)255;
    float *po = reinterpret_cast<float *>(base);
    float *pm = po + parts * kD;
    float *pl = pm + parts;
    if (!(sm_scale > 0.0f)) sm_scale = 1.0f / std::sqrt((float)kD);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    rc = launch_decode_tma_dev(q_f16, k_blocks, v_blocks, bs_b, bs_h, pm, pl, po, B, Hq, Hkv, max_len, seq_len_dev,
                               ns, sm_scale * kLog2e, flags & (ECC_DECODE_ROTATE_Q | ECC_DECODE_BLOCK96), s);
    if (rc > 0) return ECC_ERR_SHAPE;  // a pool layout or device the TMA kernel does not take
    if (rc != ECC_OK) return rc;
    return ecc_lse_merge(pm, pl, po, (int64_t)B * Hq, ns, out_f16, flags & ECC_DECODE_UNROTATE_OUT, stream);
}

// ---------------------------------------------------------------------------
// Decode without any allocation: the split partials live in a fixed device
// array that belongs to this library (ECC_DECODE_STATIC_SCRATCH_BYTES, held on
// every GPU that loads the library until the process exits).  For callers
// that must not call cudaMalloc themselves -- e.g. a host whose device memory
// is owned by another allocator that has already reserved the budget, or a
// latency-critical path that cannot afford cudaMalloc's implicit
// synchronisation.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_decode_scratch[ECC_DECODE_STATIC_SCRATCH_BYTES];

static std::mutex g_scratch_mu;
static void *g_scratch_addr[64];
static CUcontext g_scratch_ctx[64];

// Device address of g_decode_scratch on the current device (the host-side
// name is only a stand-in for it), looked up once per device and context: a
// context that was destroyed and created again (cudaDeviceReset) loads the
// module anew, so the cached address is dropped when the current context is
// not the one it was taken in.
static int static_scratch(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ECC_ERR_DEVICE;
    if (cudaFree(nullptr) != cudaSuccess) return ECC_ERR_CUDA;  // makes the device's primary context current
    const CUcontext ctx = current_context();
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_addr[dev] || g_scratch_ctx[dev] != ctx) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || !p) return ECC_ERR_CUDA;
        g_scratch_addr[dev] = p;
        g_scratch_ctx[dev] = ctx;
    }
    *out = g_scratch_addr[dev];
    return ECC_OK;
}

extern "C" int ecc_decode_static(const void *q_f16, const void *k_blocks, const void *v_blocks, int64_t bs_b,
                                 int64_t bs_h, void *out_f16, int B, int Hq, int Hkv, int64_t seq_len,
                                 float sm_scale, int flags, int num_splits, ecc_stream_t stream) {
    int rc = check_decode_args(q_f16, k_blocks, v_blocks, B, Hq, Hkv, seq_len);
    if (rc != ECC_OK) return rc;
    if (!out_f16) return ECC_ERR_NULL;
    const size_t cap = ECC_DECODE_STATIC_SCRATCH_BYTES;
    int ns_req = num_splits;
    if (ns_req <= 0) {
        // default split count, lowered until the partials fit the array
        const size_t per_split = (size_t)B * Hq * sizeof(float) * (2 + kD);
        const size_t fit = cap > 256 ? (cap - 256) / per_split : 0;
        if (fit < 1) return ECC_ERR_SCRATCH_LIMIT;
        const int dflt = ecc_decode_default_splits(B, Hkv, seq_len);
        // the default count itself when it fits (it selects the same kernel
        // and partition as ecc_decode with num_splits = 0)
        ns_req = (size_t)dflt <= fit ? 0 : (int)std::min<size_t>(fit, 4096);
    }
    if (ecc_decode_workspace_size(B, Hq, Hkv, seq_len, ns_req) > cap) return ECC_ERR_SCRATCH_LIMIT;
    void *scratch = nullptr;
    rc = static_scratch(&scratch);
    if (rc != ECC_OK) return rc;
    return ecc_decode(q_f16, k_blocks, v_blocks, bs_b, bs_h, out_f16, scratch, cap, B, Hq, Hkv, seq_len, sm_scale,
                      flags, ns_req, stream);
}

// ---------------------------------------------------------------------------
// Record exchange over peer memory (lse_exchange_kernel above).
// ---------------------------------------------------------------------------
// CTAs of one exchange call: one per row up to kExchMaxGrid, and never more
// than can be resident at once on the device (the smaller occupancy of the
// two exchange kernels, which both use this grid).
static std::mutex g_exch_mu;
static int g_exch_per_sm[64];

extern "C" int ecc_exchange_grid(int64_t rows) {
    if (rows <= 0) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
    int per_sm;
    {
        std::lock_guard<std::mutex> lk(g_exch_mu);
        if (!g_exch_per_sm[dev]) {
            int na = 0, nb = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&na, lse_exchange_kernel, kD, 0) != cudaSuccess)
                na = 1;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, lse_gather_kernel, kD, 0) != cudaSuccess) nb = 1;
            g_exch_per_sm[dev] = std::max(1, std::min(na, nb));
        }
        per_sm = g_exch_per_sm[dev];
    }
    return (int)std::min<int64_t>({rows, (int64_t)kExchMaxGrid, (int64_t)per_sm * sm_count()});
}

extern "C" size_t ecc_exchange_buffer_bytes(int64_t rows, int world) {
    if (rows <= 0 || world < 1 || world > kExchMaxRanks) return 0;
    return (size_t)2 * world * rows * kRec * sizeof(unsigned long long);
}

// The exchange buffer: a whole cudaMalloc allocation (so that its IPC handle
// maps exactly it), zero-filled; the handle travels to the other ranks, which
// map it on their own device with peer access enabled lazily.
static_assert(sizeof(cudaIpcMemHandle_t) == ECC_IPC_HANDLE_BYTES, "IPC handle size");

// Bytes of every exchange buffer this process allocated or mapped, by the
// address it uses for it: ecc_lse_exchange_merge checks each call's rows and
// world against them, so that no call stores past the end of a buffer on
// another GPU.  A mapped peer buffer's size is the size of the allocation
// behind the IPC handle (cuMemGetAddressRange).
static std::mutex g_bufreg_mu;
static std::unordered_map<const void *, size_t> g_bufreg;

static void bufreg_put(const void *p, size_t bytes) {
    std::lock_guard<std::mutex> lk(g_bufreg_mu);
    g_bufreg[p] = bytes;
}
static void bufreg_drop(const void *p) {
    std::lock_guard<std::mutex> lk(g_bufreg_mu);
    g_bufreg.erase(p);
}
static size_t bufreg_get(const void *p) {
    std::lock_guard<std::mutex> lk(g_bufreg_mu);
    const auto it = g_bufreg.find(p);
    return it == g_bufreg.end() ? 0 : it->second;
}

extern "C" int ecc_exchange_alloc(int64_t rows, int world, void **buffer, void *ipc_handle) {
    const size_t bytes = ecc_exchange_buffer_bytes(rows, world);
    if (!bytes) return ECC_ERR_SHAPE;
    if (!buffer || !ipc_handle) return ECC_ERR_NULL;
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return ECC_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
        cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return ECC_ERR_CUDA;
    }
    std::memcpy(ipc_handle, &h, sizeof(h));
    *buffer = p;
    bufreg_put(p, bytes);
    return ECC_OK;
}

extern "C" int ecc_exchange_open(const void *ipc_handle, void **peer_buffer) {
    if (!ipc_handle || !peer_buffer) return ECC_ERR_NULL;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof(h));
    void *p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return ECC_ERR_CUDA;
    const size_t bytes = allocation_bytes(p);
    if (!bytes) {
        cudaIpcCloseMemHandle(p);
        return ECC_ERR_CUDA;
    }
    bufreg_put(p, bytes);
    *peer_buffer = p;
    return ECC_OK;
}

extern "C" int ecc_exchange_close(void *peer_buffer) {
    if (!peer_buffer) return ECC_ERR_NULL;
    bufreg_drop(peer_buffer);
    return cudaIpcCloseMemHandle(peer_buffer) == cudaSuccess ? ECC_OK : ECC_ERR_CUDA;
}

extern "C" int ecc_exchange_free(void *buffer) {
    if (!buffer) return ECC_ERR_NULL;
    bufreg_drop(buffer);
    return cudaFree(buffer) == cudaSuccess ? ECC_OK : ECC_ERR_CUDA;
}

// Peer pointers of an exchange call, each checked against the registry: a
// buffer this process allocated or mapped, of at least `need` bytes (the
// stores would otherwise land past its end, in another GPU's memory).
static int peer_table(void *const *peer_buffers, int world, size_t need, PeerBufs *pb) {
    for (int q = 0; q < world; ++q) {
        if (!peer_buffers[q]) return ECC_ERR_NULL;
        if ((uintptr_t)peer_buffers[q] % 16) return ECC_ERR_ALIGN;
        const size_t have = bufreg_get(peer_buffers[q]);
        if (have == 0 || have < need) return ECC_ERR_SHAPE;
        pb->base[q] = reinterpret_cast<unsigned long long *>(peer_buffers[q]);
    }
    return ECC_OK;
}

// Host epoch (epoch >= 1, state null) or device-side epoch state (epoch 0).
static int gather_merge(const float *part_m, const float *part_l, const float *part_o, int64_t rows, int n,
                        int hq_local, void *const *peer_buffers, int world, int rank, uint32_t epoch,
                        uint64_t *state, long long wait_cycles, void *out_f16, int flags, ecc_stream_t stream) {
    if (rows <= 0 || n <= 0 || hq_local <= 0 || rows % hq_local || world < 1 || world > kExchMaxRanks || rank < 0 ||
        rank >= world || (epoch == 0) == (state == nullptr) || wait_cycles <= 0 || rows > 0x7fffffff)
        return ECC_ERR_SHAPE;
    if (!part_m || !part_l || !part_o || !peer_buffers || !out_f16) return ECC_ERR_NULL;
    if ((uintptr_t)state % 8) return ECC_ERR_ALIGN;
    PeerBufs pb{};
    // slots [2][world][rows][64 words]: within a buffer made for (rows, world)
    const int rc = peer_table(peer_buffers, world, (size_t)2 * world * rows * kGatherWords * 8, &pb);
    if (rc != ECC_OK) return rc;
    const int grid = ecc_exchange_grid(rows);
    if (launch_pdl(lse_gather_kernel, dim3(grid), dim3(kD), 0, reinterpret_cast<cudaStream_t>(stream), part_m,
                   part_l, part_o, n, rows, hq_local, world, rank, pb, epoch,
                   reinterpret_cast<unsigned long long *>(state), wait_cycles, reinterpret_cast<__half *>(out_f16),
                   flags & ECC_DECODE_UNROTATE_OUT) != cudaSuccess)
        return ECC_ERR_LAUNCH;
    return launch_status();
}

static int exchange_merge(const float *part_m, const float *part_l, const float *part_o, int64_t rows, int n,
                          void *const *peer_buffers, int world, int rank, uint32_t epoch, uint64_t *state,
                          long long wait_cycles, void *out_f16, int flags, ecc_stream_t stream) {
    if (rows <= 0 || n <= 0 || world < 1 || world > kExchMaxRanks || rank < 0 || rank >= world ||
        (epoch == 0) == (state == nullptr) || wait_cycles <= 0 || rows > 0x7fffffff)
        return ECC_ERR_SHAPE;
    if (!part_m || !part_l || !part_o || !peer_buffers || !out_f16) return ECC_ERR_NULL;
    if ((uintptr_t)state % 8) return ECC_ERR_ALIGN;
    PeerBufs pb{};
    const int rc = peer_table(peer_buffers, world, ecc_exchange_buffer_bytes(rows, world), &pb);
    if (rc != ECC_OK) return rc;
    const int grid = ecc_exchange_grid(rows);
    // a programmatic dependent of the previous kernel; it never triggers its
    // own dependents, so none starts before it ends
    if (launch_pdl(lse_exchange_kernel, dim3(grid), dim3(kD), 0, reinterpret_cast<cudaStream_t>(stream), part_m,
                   part_l, part_o, n, rows, world, rank, pb, epoch, reinterpret_cast<unsigned long long *>(state),
                   wait_cycles, reinterpret_cast<__half *>(out_f16), flags & ECC_DECODE_UNROTATE_OUT) != cudaSuccess)
        return ECC_ERR_LAUNCH;
    return launch_status();
}

extern "C" int ecc_lse_gather_merge(const float *part_m, const float *part_l, const float *part_o, int64_t rows, int n,
                                    int hq_local, void *const *peer_buffers, int world, int rank, uint32_t epoch,
                                    long long wait_cycles, void *out_f16, int flags, ecc_stream_t stream) {
    if (epoch == 0) return ECC_ERR_SHAPE;
    return gather_merge(part_m, part_l, part_o, rows, n, hq_local, peer_buffers, world, rank, epoch, nullptr,
                        wait_cycles, out_f16, flags, stream);
}

extern "C" int ecc_lse_gather_merge_dev(const float *part_m, const float *part_l, const float *part_o, int64_t rows,
                                        int n, int hq_local, void *const *peer_buffers, int world, int rank,
                                        uint64_t *epoch_state, long long wait_cycles, void *out_f16, int flags,
                                        ecc_stream_t stream) {
    if (!epoch_state) return ECC_ERR_NULL;
    return gather_merge(part_m, part_l, part_o, rows, n, hq_local, peer_buffers, world, rank, 0, epoch_state,
                        wait_cycles, out_f16, flags, stream);
}

extern "C" int ecc_lse_exchange_merge(const float *part_m, const float *part_l, const float *part_o, int64_t rows,
                                      int n, void *const *peer_buffers, int world, int rank, uint32_t epoch,
                                      long long wait_cycles, void *out_f16, int flags, ecc_stream_t stream) {
    if (epoch == 0) return ECC_ERR_SHAPE;
    return exchange_merge(part_m, part_l, part_o, rows, n, peer_buffers, world, rank, epoch, nullptr, wait_cycles,
                          out_f16, flags, stream);
}

extern "C" int ecc_lse_exchange_merge_dev(const float *part_m, const float *part_l, const float *part_o,
                                          int64_t rows, int n, void *const *peer_buffers, int world, int rank,
                                          uint64_t *epoch_state, long long wait_cycles, void *out_f16, int flags,
                                          ecc_stream_t stream) {
    if (!epoch_state) return ECC_ERR_NULL;
    return exchange_merge(part_m, part_l, part_o, rows, n, peer_buffers, world, rank, 0, epoch_state, wait_cycles,
                          out_f16, flags, stream);
}
