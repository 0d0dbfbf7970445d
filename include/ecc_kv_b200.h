/*
 * ecc_kv_b200.h -- C ABI of libeccb200.so, the B200 (sm_100a) implementation
 * of the ECC-INT4 KV-cache hot path: compress (WHT + Lloyd-Max INT4 + sign
 * syndrome -> 128-byte ECC_KV_Block) and fused decode attention.
 *
 * Plain pointers and sizes only.  Every function is asynchronous on the given
 * stream (NULL = legacy default stream) unless stated otherwise, returns
 * ECC_OK (0) or a negative ECC_ERR_* code, and never aborts; ecc_strerror()
 * names a code.  Pointers are device pointers unless stated otherwise.
 *
 * Block format (one token of one KV head, csrc/ecc_ops.h:22-32 of the
 * reference): bytes 0..63 INT4 codes, byte i = q[2i] | q[2i+1] << 4;
 * bytes 64..79 sign syndrome, bit j in byte j/8 at position j%8 (1 = the
 * quantisation residual is >= 0); fp16 scale @80, zero @82, alpha @84;
 * bytes 86..127 zero.
 */
#ifndef ECC_KV_B200_H
#define ECC_KV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *ecc_stream_t; /* same type as cudaStream_t */

enum {
    ECC_OK = 0,
    ECC_ERR_NULL = -1,        /* a required pointer is NULL */
    ECC_ERR_SHAPE = -2,       /* a size is out of range (D != 128, n < 0, ...) */
    ECC_ERR_ALIGN = -3,       /* a pointer or stride is not suitably aligned */
    ECC_ERR_GQA = -4,         /* Hq is not a multiple of Hkv */
    ECC_ERR_WORKSPACE = -5,   /* workspace missing or smaller than required */
    ECC_ERR_LAUNCH = -6,      /* the CUDA launch failed (cudaGetLastError) */
    ECC_ERR_CUDA = -7,        /* another CUDA runtime call failed */
    ECC_ERR_DEVICE = -8,      /* no usable sm_100 device */
    ECC_ERR_SCRATCH_LIMIT = -9, /* request larger than ECC_DECODE_STATIC_SCRATCH_BYTES */
    ECC_ERR_PARAM = -10         /* a quantiser parameter is not finite, or scale <= 0 */
};

#define ECC_DECODE_ROTATE_Q 1    /* rotate the query (WHT) inside the kernel */
#define ECC_DECODE_UNROTATE_OUT 2 /* apply the WHT to the output (values stored rotated) */
#define ECC_DECODE_CUDA_CORES 4   /* use the CUDA-core kernel instead of the tensor-core one
                                     (groups of more than 8 query heads always use it) */
#define ECC_DECODE_REGISTER_PATH 8 /* tensor-core kernel with per-lane global loads instead of the
                                      TMA-fed warp-specialised one (used automatically when a
                                      pool layout cannot be described by a tensor map) */
#define ECC_DECODE_BLOCK96 16      /* the pools hold 96-byte records (ECC_COMPRESS_BLOCK96); block
                                      strides count records.  TMA-fed kernel only: GQA groups up
                                      to 8 and at least its own split count (ecc_decode: the
                                      default, num_splits <= 0; the partials entry points: any
                                      count >= the default); ECC_ERR_SHAPE for requests only the
                                      other kernels take */

/* Bits of the `rotate` argument of the compress entry points.  0/1 keep
 * their meaning (input already rotated / WHT applied first). */
#define ECC_COMPRESS_ROTATE 1   /* apply the WHT first, as compress_cpu does */
#define ECC_COMPRESS_BLOCK96 2  /* write 96-byte records: the block without its zero pad sector
                                   (bytes 96..127), offsets 0..95 unchanged; block strides and
                                   positions count records; pool base 32-byte aligned.  Not a
                                   format of the reference: an option that cuts cache memory and
                                   decode DRAM traffic by a quarter */

/* Name of an error code (static string). */
const char *ecc_strerror(int code);

/* Library version, e.g. 100 for 0.1.0. */
int ecc_version(void);

/* Device-side error flag of the current device since the last reset
 * (reset != 0 clears it); synchronous:
 *   0  no error;
 *   1  a decode kernel ran out of a bounded wait on its copies and returned
 *      early instead of hanging (its output is not valid);
 *   2  the decode kernel found its shared memory at an unexpected address and
 *      returned without computing;
 *   3  an append at a device-side position (ecc_compress_strided_pair_at,
 *      ..._calibrated_at) was out of range and wrote nothing;
 *   4  ecc_lse_exchange_merge ran out of its wait for another rank's records
 *      (the rows it waited for were not written).
 * When several were raised, the lowest of 1/2 (decode), 3, 4 is returned. */
int ecc_device_status(int reset);

/* Self-test of the bounded device waits (no counterpart in the reference):
 * launches one warp that waits on an mbarrier nothing will complete, with the
 * decode kernel's wait routine and a limit of limit_cycles clocks (at most
 * 2^32).  The wait gives up, raises the flag ecc_device_status reports, and
 * the kernel returns; *host_gave_up = 1 then.  Synchronous; allocates 4 bytes
 * of device memory for the result.  Faults and hangs nothing. */
int ecc_selftest_wait_timeout(long long limit_cycles, int *host_gave_up);

/* ---- WHT ------------------------------------------------------------------
 * In-place normalised Walsh-Hadamard transform of n rows of length d (power
 * of two, 1 <= d <= 1024), contiguous [n, d], fp16 or fp32.  Butterfly with
 * stride 1,2,...,d/2 then an IEEE division by fp32(sqrt(d)) -- the same
 * arithmetic as custom_kv/ops_cpu.py:29 hadamard_rotate_cpu.
 * Replaces launch_hadamard_f16 / launch_hadamard_f32 (csrc/hadamard.cu:107,
 * :119) behind custom_ecc_cuda.hadamard_rotate (csrc/ecc_ops.cpp:32). */
int ecc_hadamard_f16(void *x, int64_t n, int d, ecc_stream_t stream);
int ecc_hadamard_f32(void *x, int64_t n, int d, ecc_stream_t stream);

/* ---- compress -------------------------------------------------------------
 * n contiguous fp16 vectors [n, 128] -> n blocks [n, 128] bytes.  rotate = 1
 * applies the WHT first (custom_kv/ops_cpu.py:198 compress_cpu); rotate = 0
 * takes an already rotated input.  Bit-exact with compress_cpu.
 * Replaces launch_compress_ecc (csrc/compress_ecc.cu:183) behind
 * custom_ecc_cuda.compress_and_store (csrc/ecc_ops.cpp:68) with rotate = 0.
 * x must be 16-byte aligned, blocks 128-byte aligned. */
int ecc_compress(const void *x_f16, void *blocks, int64_t n, int rotate, ecc_stream_t stream);

/* Strided compress of x[b][h][l][0..127] (element strides xs_b, xs_h, xs_l,
 * last dim contiguous, each multiple of 8) into the block pool at
 * block index b*bs_b + h*bs_h + l (token stride one block).  This is the
 * cache write of ErrorCorrectedCache.update (custom_kv/cache.py:103-126). */
int ecc_compress_strided(const void *x_f16, int64_t xs_b, int64_t xs_h, int64_t xs_l,
                         void *blocks, int64_t bs_b, int64_t bs_h,
                         int B, int H, int64_t L, int rotate, ecc_stream_t stream);

/* Two ecc_compress_strided requests of the same [B, H, L] shape in one launch
 * -- the K and V writes of one cache update, which the reference issues as
 * two compress_and_store calls (custom_kv/cache.py:103-126).  The two
 * requests are validated like ecc_compress_strided and run concurrently; for
 * an append of a few tokens that halves the latency of the pair. */
int ecc_compress_strided_pair(const void *x0_f16, int64_t x0s_b, int64_t x0s_h, int64_t x0s_l,
                              void *blocks0, int64_t b0s_b, int64_t b0s_h,
                              const void *x1_f16, int64_t x1s_b, int64_t x1s_h, int64_t x1s_l,
                              void *blocks1, int64_t b1s_b, int64_t b1s_h,
                              int B, int H, int64_t L, int rotate, ecc_stream_t stream);

/* ecc_compress_strided with the quantiser parameters of a calibration config
 * (custom_kv/calibration.py:232-237: per-layer scale, zero, alpha) in place of
 * each vector's own statistics: q = first-index argmin |(x - zero) / scale -
 * C[k]| and k~ = C[q]*scale + zero in fp32 as ops_cpu.lloyd_max_quantize_cpu
 * (ops_cpu.py:78-109) computes them with those scalars, syndrome bit =
 * (x - k~ >= 0), and every block stores fp16(scale), fp16(zero), fp16(alpha).
 * The block format and the decode are unchanged.  ECC_ERR_PARAM unless
 * scale > 0 and all three are finite. */
int ecc_compress_strided_calibrated(const void *x_f16, int64_t xs_b, int64_t xs_h, int64_t xs_l,
                                    void *blocks, int64_t bs_b, int64_t bs_h, int B, int H, int64_t L,
                                    int rotate, float scale, float zero, float alpha, ecc_stream_t stream);

/* Positions and lengths in device memory.  For a decode step recorded once
 * in a CUDA graph and replayed while the context grows (no counterpart in the
 * reference, whose decode runs eagerly, custom_kv/patch.py:100), the token
 * position of an append and the context length of a decode are read from
 * device memory when the kernel runs.  blocks point at token 0 of pools with
 * `capacity` tokens per (b, h) row.
 *
 * ecc_compress_strided_pair_at: ecc_compress_strided_pair into token
 * positions *pos_dev .. *pos_dev + L - 1 (x1_f16 = blocks1 = NULL: one
 * tensor).  A position with pos < 0 or pos + L > capacity writes nothing and
 * raises the flag ecc_device_status reports (3). */
int ecc_compress_strided_pair_at(const void *x0_f16, int64_t x0s_b, int64_t x0s_h, int64_t x0s_l,
                                 void *blocks0, int64_t b0s_b, int64_t b0s_h,
                                 const void *x1_f16, int64_t x1s_b, int64_t x1s_h, int64_t x1s_l,
                                 void *blocks1, int64_t b1s_b, int64_t b1s_h,
                                 int B, int H, int64_t L, int64_t capacity, const int *pos_dev, int rotate,
                                 ecc_stream_t stream);
/* ecc_compress_strided_calibrated at the device-side position *pos_dev. */
int ecc_compress_strided_calibrated_at(const void *x_f16, int64_t xs_b, int64_t xs_h, int64_t xs_l,
                                       void *blocks, int64_t bs_b, int64_t bs_h, int B, int H, int64_t L,
                                       int64_t capacity, const int *pos_dev, int rotate, float scale,
                                       float zero, float alpha, ecc_stream_t stream);

/* ecc_decode over the first *seq_len_dev tokens (read when the kernel runs,
 * clamped to [1, max_len]) of pools holding max_len tokens per row; the split
 * count is fixed by (B, Hkv, max_len), so one recorded launch serves every
 * length.  GQA groups up to 8 and pools the tensor-map kernel takes
 * (ECC_ERR_SHAPE otherwise).  Workspace: ecc_decode_dev_workspace_size. */
size_t ecc_decode_dev_workspace_size(int B, int Hq, int Hkv, int64_t max_len);
/* Split count of the device-length decode for pools of max_len tokens. */
int ecc_decode_dev_splits(int B, int Hkv, int64_t max_len);
/* ecc_decode_partials over the first *seq_len_dev tokens (clamped to
 * [1, max_len]); num_splits >= ecc_decode_dev_splits(B, Hkv, max_len), the
 * partial arrays sized for num_splits. */
int ecc_decode_partials_dev(const void *q_f16, const void *k_blocks, const void *v_blocks, int64_t bs_b,
                            int64_t bs_h, float *part_m, float *part_l, float *part_o, int B, int Hq, int Hkv,
                            int64_t max_len, const int *seq_len_dev, float sm_scale, int flags, int num_splits,
                            ecc_stream_t stream);
int ecc_decode_dev(const void *q_f16, const void *k_blocks, const void *v_blocks, int64_t bs_b, int64_t bs_h,
                   void *out_f16, void *workspace, size_t workspace_bytes, int B, int Hq, int Hkv,
                   int64_t max_len, const int *seq_len_dev, float sm_scale, int flags, ecc_stream_t stream);

/* Copy the fp16 (scale, zero, alpha) of block block_idx to host memory as
 * fp32.  Synchronous on `stream`.  Replaces custom_ecc_cuda.get_block_metadata
 * (csrc/ecc_ops.cpp:98). */
int ecc_get_block_metadata(const void *blocks, int64_t n_blocks, int64_t block_idx,
                           float *host_out3, ecc_stream_t stream);

/* Reconstruct blocks to fp16 vectors: out = (C[q]*scale + zero) + alpha*s
 * (custom_kv/fused_decode.py:229-241), n contiguous blocks -> [n, 128]. */
int ecc_dequantize(const void *blocks, void *out_f16, int64_t n, ecc_stream_t stream);

/* Pack the reference's SoA trio (custom_kv/cache.py:79-84: int4 [N,64] u8,
 * syn [N,16] u8, meta [N,3] fp16, each with its own row stride in bytes)
 * into contiguous 128-byte blocks. */
int ecc_pack_soa(const void *int4, int64_t int4_row_bytes, const void *syn, int64_t syn_row_bytes,
                 const void *meta, int64_t meta_row_bytes, void *blocks, int64_t n, ecc_stream_t stream);

/* ---- decode attention -----------------------------------------------------
 * One decode step of GQA attention over compressed K and V pools.
 *   q:        [B, Hq, 128] fp16, contiguous (rotated query unless flags has
 *             ECC_DECODE_ROTATE_Q).
 *   k_blocks, v_blocks: pools; block (b, kv_head, t) at block index
 *             b*bs_b + kv_head*bs_h + t, t in [0, seq_len).  128-byte aligned.
 *   out:      [B, Hq, 128] fp16, contiguous.
 *   sm_scale: softmax scale; <= 0 selects 1/sqrt(128).
 *   num_splits: sequence partitions per (b, kv_head); <= 0 chooses one.
 *   workspace: device scratch of at least ecc_decode_workspace_size() bytes
 *             for the split partials (may be NULL when that size is 0).
 * Query head h reads kv head h / (Hq / Hkv) (HF repeat_kv convention).
 * Replaces the Triton fused_ecc_decode_attention
 * (custom_kv/fused_decode.py:153) and the dequantise-then-SDPA decode step of
 * custom_kv/patch.py:100 _ecc_decode_step. */
int ecc_decode(const void *q_f16, const void *k_blocks, const void *v_blocks, int64_t bs_b,
               int64_t bs_h, void *out_f16, void *workspace, size_t workspace_bytes, int B, int Hq,
               int Hkv, int64_t seq_len, float sm_scale, int flags, int num_splits,
               ecc_stream_t stream);

/* ecc_decode of a left-padded batch (its attention mask): sequence b attends
 * to tokens [start_dev[b], seq_len) only; the tokens before start_dev[b] are
 * the padding a batched prompt put in front of the shorter sequences.
 *   start_dev: DEVICE int32 [B], read when the kernel runs; a value <= 0
 *              masks nothing, a value >= seq_len masks the whole sequence
 *              (its output is then zero).
 * The other arguments are those of ecc_decode with num_splits = 0 (workspace
 * of ecc_decode_workspace_size(B, Hq, Hkv, seq_len, 0) bytes).  GQA groups up
 * to 8 and pool layouts a TMA tensor map can describe; ECC_ERR_SHAPE
 * otherwise.  Replaces the attention-mask handling the reference's decode
 * step drops (custom_kv/patch.py:87-117 calls SDPA with attn_mask=None). */
int ecc_decode_masked(const void *q_f16, const void *k_blocks, const void *v_blocks, int64_t bs_b,
                      int64_t bs_h, const int *start_dev, void *out_f16, void *workspace,
                      size_t workspace_bytes, int B, int Hq, int Hkv, int64_t seq_len, float sm_scale,
                      int flags, ecc_stream_t stream);

/* Workspace bytes ecc_decode needs for these sizes (0 if it needs none);
 * num_splits as passed to ecc_decode. */
size_t ecc_decode_workspace_size(int B, int Hq, int Hkv, int64_t seq_len, int num_splits);

/* The split count ecc_decode uses when num_splits <= 0. */
int ecc_decode_default_splits(int B, int Hkv, int64_t seq_len);

/* Per-split partials of one decode step without the merge, for combining
 * partials across devices (sequence-chunk sharding): writes m, l
 * [B, Hq, num_splits] fp32 and o [B, Hq, num_splits, 128] fp32 (o is the
 * unnormalised sum of e^(s - m) v, in the stored value basis).  Token
 * positions [0, seq_len) of the pools are this device's chunk. */
int ecc_decode_partials(const void *q_f16, const void *k_blocks, const void *v_blocks,
                        int64_t bs_b, int64_t bs_h, float *part_m, float *part_l, float *part_o,
                        int B, int Hq, int Hkv, int64_t seq_len, float sm_scale, int flags,
                        int num_splits, ecc_stream_t stream);

/* Log-sum-exp merge of n partials per row (rows = B*Hq): m, l [rows, n],
 * o [rows, n, 128] as written by ecc_decode_partials (rows may gather
 * partials of several devices).  out [rows, 128] fp16; flags may hold
 * ECC_DECODE_UNROTATE_OUT. */
int ecc_lse_merge(const float *part_m, const float *part_l, const float *part_o, int64_t rows, int n,
                  void *out_f16, int flags, ecc_stream_t stream);

/* Two-level combine for sequences sharded over devices (no counterpart in
 * the reference, which runs on one GPU).  A partial record is 130 floats
 * {m, l, o[128]} (m in natural-log units, o unnormalised), i.e. one merged
 * split.
 *   ecc_lse_merge_to_record: merges the n split partials of each row (layout
 *     of ecc_lse_merge) into one record per row, records [rows, 130].
 *   ecc_lse_merge_records: merges n records per row, record i of row r at
 *     records + i * record_stride + r * 130 (floats) -- e.g. the [n, rows,
 *     130] result of an all-gather of every device's records, with
 *     record_stride = rows * 130 -- into out [rows, 128] fp16; flags may hold
 *     ECC_DECODE_UNROTATE_OUT.  Record sets may not overlap. */
#define ECC_RECORD_FLOATS 130
int ecc_lse_merge_to_record(const float *part_m, const float *part_l, const float *part_o, int64_t rows, int n,
                            float *records, ecc_stream_t stream);
int ecc_lse_merge_records(const float *records, int64_t rows, int n, int64_t record_stride, void *out_f16,
                          int flags, ecc_stream_t stream);

/* Record exchange over peer memory, for sequences sharded over the GPUs of
 * one node (no counterpart in the reference, which runs on one GPU): the
 * two-level combine above -- ecc_lse_merge_to_record, an all-gather of the
 * records, ecc_lse_merge_records -- as one kernel per rank and step, with the
 * records stored straight into every rank's exchange buffer over NVLink.
 *   ecc_exchange_buffer_bytes(rows, world): bytes of one rank's exchange
 *     buffer (zero-filled once before the first call).
 *   ecc_exchange_grid(rows): CTAs per call (the same on every rank).
 *   ecc_lse_exchange_merge: ECC_ERR_SHAPE unless every entry of peer_buffers
 *     is a buffer this process allocated (ecc_exchange_alloc) or mapped
 *     (ecc_exchange_open) and holds ecc_exchange_buffer_bytes(rows, world)
 *     bytes; part_m/l/o as for ecc_lse_merge (this rank's n
 *     split partials of every row); peer_buffers: HOST array of `world`
 *     device pointers, entry q = rank q's exchange buffer as mapped in this
 *     process (entry `rank` = this rank's own); epoch: 1, 2, 3, ... -- the
 *     same sequence on every rank, one per call; wait_cycles: bound of the
 *     wait for the other ranks' records (SM clock cycles), after which the
 *     kernel raises the ecc_device_status flag (value 4) and returns without
 *     writing those rows.  out [rows, 128] fp16 as ecc_lse_merge_records
 *     writes it (bit-identical); flags may hold ECC_DECODE_UNROTATE_OUT.
 *     Every rank must make the same sequence of calls with the same rows. */
#define ECC_EXCHANGE_MAX_RANKS 8
#define ECC_IPC_HANDLE_BYTES 64
size_t ecc_exchange_buffer_bytes(int64_t rows, int world);
/* Exchange buffers, one per rank, on the current device (synchronous):
 *   ecc_exchange_alloc: allocates and zero-fills this rank's buffer and
 *     writes its CUDA IPC handle (ECC_IPC_HANDLE_BYTES host bytes) for the
 *     other ranks;
 *   ecc_exchange_open: maps another rank's buffer from its handle into this
 *     process on the current device (peer access enabled as needed);
 *   ecc_exchange_close: unmaps a buffer ecc_exchange_open mapped;
 *   ecc_exchange_free: frees this rank's buffer once every rank has closed it. */
int ecc_exchange_alloc(int64_t rows, int world, void **buffer, void *ipc_handle);
int ecc_exchange_open(const void *ipc_handle, void **peer_buffer);
int ecc_exchange_close(void *peer_buffer);
int ecc_exchange_free(void *buffer);
int ecc_exchange_grid(int64_t rows);
int ecc_lse_exchange_merge(const float *part_m, const float *part_l, const float *part_o, int64_t rows, int n,
                           void *const *peer_buffers, int world, int rank, uint32_t epoch, long long wait_cycles,
                           void *out_f16, int flags, ecc_stream_t stream);

/* Output gather over peer memory, for decode sharded by kv head over the GPUs
 * of one node (no counterpart in the reference, which runs on one GPU): the
 * merge of this rank's split partials (ecc_lse_merge) and the all-gather of
 * the ranks' fp16 outputs as one kernel per rank and step.  Rank s serves
 * query heads [s*hq_local, (s+1)*hq_local) of every sequence.
 *   part_m/l/o: this rank's n split partials of rows = B * hq_local rows
 *     (layout of ecc_lse_merge);
 *   peer_buffers, world, rank, epoch, wait_cycles: as for
 *     ecc_lse_exchange_merge; the buffers must hold 2 * world * rows * 512
 *     bytes (a buffer from ecc_exchange_alloc(rows, world) does), else
 *     ECC_ERR_SHAPE;
 *   out: [B, world * hq_local, 128] fp16, the whole attention output of the
 *     step on every rank; flags may hold ECC_DECODE_UNROTATE_OUT.
 * Every rank must make the same sequence of calls (with ecc_lse_exchange_merge
 * calls they share one epoch sequence) with the same rows.  A wait that runs
 * out raises the ecc_device_status flag (4). */
int ecc_lse_gather_merge(const float *part_m, const float *part_l, const float *part_o, int64_t rows, int n,
                         int hq_local, void *const *peer_buffers, int world, int rank, uint32_t epoch,
                         long long wait_cycles, void *out_f16, int flags, ecc_stream_t stream);

/* The two peer-memory merges with the epoch in device memory instead of a
 * kernel argument, so that a step can be recorded once in a CUDA graph and
 * replayed (no counterpart in the reference).  epoch_state: DEVICE array of
 * two uint64 {counter, done}, zero-filled once before the first call; the
 * call's epoch is counter % (2^32 - 2) + 1 and the kernel's last CTA
 * advances the counter, so successive calls (eager or replayed) take
 * successive epochs.  Every rank keeps its own state and makes the same
 * sequence of calls; do not mix these with the host-epoch forms on one set
 * of buffers.  Other arguments as ecc_lse_exchange_merge /
 * ecc_lse_gather_merge. */
int ecc_lse_exchange_merge_dev(const float *part_m, const float *part_l, const float *part_o, int64_t rows, int n,
                               void *const *peer_buffers, int world, int rank, uint64_t *epoch_state,
                               long long wait_cycles, void *out_f16, int flags, ecc_stream_t stream);
int ecc_lse_gather_merge_dev(const float *part_m, const float *part_l, const float *part_o, int64_t rows, int n,
                             int hq_local, void *const *peer_buffers, int world, int rank, uint64_t *epoch_state,
                             long long wait_cycles, void *out_f16, int flags, ecc_stream_t stream);

/* Bytes of the library-owned device array ecc_decode_static uses for its
 * split partials (4 MiB on every GPU that loads the library, kept until the
 * process exits). */
#define ECC_DECODE_STATIC_SCRATCH_BYTES (4u << 20)

/* ecc_decode without a caller workspace and without any allocation, for
 * callers that must not allocate device memory themselves (a host whose
 * device memory is owned by another allocator, a latency-critical path that
 * cannot take cudaMalloc's implicit synchronisation).  No counterpart in the
 * reference.  Same arguments and results as ecc_decode minus the workspace;
 * the split partials go to a fixed library-owned device array of
 * ECC_DECODE_STATIC_SCRATCH_BYTES:
 *   - B * Hq * splits * 520 bytes (+256) must fit; with num_splits <= 0 the
 *     default split count is lowered until it fits, otherwise (or when even
 *     one split does not fit) the call returns ECC_ERR_SCRATCH_LIMIT;
 *   - the first call on a device looks up the array's device address; make
 *     that first call before any stream capture;
 *   - every call on a device shares the one array: calls that overlap on the
 *     GPU (other streams, other threads) race and corrupt each other's
 *     results; serialise them on one stream.  Nothing in the array needs to
 *     start at zero -- each call writes every partial it reads. */
int ecc_decode_static(const void *q_f16, const void *k_blocks, const void *v_blocks, int64_t bs_b,
                      int64_t bs_h, void *out_f16, int B, int Hq, int Hkv, int64_t seq_len,
                      float sm_scale, int flags, int num_splits, ecc_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* ECC_KV_B200_H */
