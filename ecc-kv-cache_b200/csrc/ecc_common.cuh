// ecc_common.cuh -- block format, centroid table and small device helpers
// shared by the compress and decode kernels (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ecc_kv_b200.h"

namespace ecc {

constexpr int kD = 128;           // head dim (the block format is fixed to 128)
constexpr int kBlockBytes = 128;  // one ECC_KV_Block
constexpr int kCodesOff = 0;      // 64 bytes of packed INT4 codes
constexpr int kSynOff = 64;       // 16 bytes of sign syndrome
constexpr int kScaleOff = 80;     // fp16 scale
constexpr int kZeroOff = 82;      // fp16 zero point
constexpr int kAlphaOff = 84;     // fp16 alpha

// The reference's block struct (csrc/ecc_ops.h:22-32) restated so its offsets
// are checked at compile time; kernels address bytes through the constants.
struct alignas(128) BlockLayout {
    uint8_t codes[64];
    uint16_t syndrome[8];
    __half scale;
    __half zero;
    __half alpha;
    uint8_t pad[42];
};
static_assert(sizeof(BlockLayout) == kBlockBytes, "block must be 128 bytes");
static_assert(offsetof(BlockLayout, syndrome) == kSynOff, "syndrome @64");
static_assert(offsetof(BlockLayout, scale) == kScaleOff, "scale @80");
static_assert(offsetof(BlockLayout, zero) == kZeroOff, "zero @82");
static_assert(offsetof(BlockLayout, alpha) == kAlphaOff, "alpha @84");

// Lloyd-Max table of custom_kv/ops_cpu.py:19-24 as fp32 bit patterns.
__host__ __device__ constexpr uint32_t lm_bits(int k) {
    return k == 0 ? 0xc019a6b5u : k == 1 ? 0xbfebf7cfu : k == 2 ? 0xbfb7f2e5u : k == 3 ? 0xbf8cb5ddu
         : k == 4 ? 0xbf4cb296u : k == 5 ? 0xbf05bc02u : k == 6 ? 0xbe8432cau : k == 7 ? 0x00000000u
         : k == 8 ? 0x3e8432cau : k == 9 ? 0x3f05bc02u : k == 10 ? 0x3f4cb296u : k == 11 ? 0x3f8cb5ddu
         : k == 12 ? 0x3fb7f2e5u : k == 13 ? 0x3febf7cfu : k == 14 ? 0x4019a6b5u : 0x404a233au;
}
__device__ __forceinline__ float lm(int k) { return __uint_as_float(lm_bits(k)); }

// fp32(sqrt(128)) and its correctly rounded reciprocal (see compress.cu).
constexpr float kSqrt128 = 0x1.6a09e6p+3f;
constexpr float kInvSqrt128 = 0x1.6a09e6p-4f;

__device__ __forceinline__ unsigned lane_id() { return threadIdx.x & 31u; }

// Programmatic dependent launch: the hot kernels are launched as dependents
// of the kernel before them on the stream.  Each calls pdl_wait() before it
// reads or writes memory that earlier work may touch (so its set-up overlaps
// the previous kernel's tail) and pdl_trigger() early so that the next kernel
// can be launched while it runs.  Both are no-ops for a normal launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
static inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                     Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace ecc
