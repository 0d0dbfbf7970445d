"""custom_ecc_cuda -- the reference's CUDA op module (csrc/ecc_ops.cpp:119-138)
re-implemented over the C ABI of libeccb200.so (sm_100a).

Same op names, argument meaning and error behaviour as the reference's
pybind module:

* ``hadamard_rotate(x)``                 csrc/ecc_ops.cpp:32
* ``compress_and_store(x_rot, cache_raw)`` csrc/ecc_ops.cpp:68
* ``get_block_metadata(cache_raw, idx)``  csrc/ecc_ops.cpp:98

plus the ops the rest of this package is built on (fused rotate+compress into a
strided block pool, fused decode attention, split partials and their merge,
dequantisation, SoA packing).  Every op runs the CUDA library; there is no CPU
path, and CPU tensors raise ``RuntimeError`` like the reference's
``TORCH_CHECK(x.is_cuda())``.  Launches go to torch's current stream.
"""
from __future__ import annotations

import ctypes
import math
import os
import threading

import torch

__all__ = [
    "hadamard_rotate", "compress_and_store", "get_block_metadata", "rotate_and_compress",
    "compress_into", "decode_attention", "decode_partials", "lse_merge", "dequantize", "pack_soa",
    "decode_workspace_size", "default_splits", "library_path", "EccError", "compress_calibrated_into",
    "compress_pair_at", "compress_calibrated_at", "decode_attention_dev", "decode_dev_workspace_size",
    "decode_partials_dev", "decode_dev_splits", "exchange_buffer_bytes", "lse_exchange_merge",
    "exchange_alloc", "exchange_open", "exchange_close", "exchange_free", "lse_gather_merge",
    "decode_attention_masked",
]

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_NAME = "libeccb200.so"
library_path = os.path.join(_HERE, _LIB_NAME)

ROTATE_Q = 1
UNROTATE_OUT = 2
CUDA_CORES = 4
REGISTER_PATH = 8
BLOCK96 = 16           # decode flag: the pools hold 96-byte records
COMPRESS_BLOCK96 = 2   # compress mode bit: write 96-byte records
_KERNEL_FLAGS = {"auto": 0, "tma": 0, "register": REGISTER_PATH, "cuda_cores": CUDA_CORES}
D = 128
BLOCK_BYTES = 128
RECORD96 = 96          # the block without its zero pad sector (bytes 96..127)


class EccError(RuntimeError):
    """A negative status from libeccb200.so."""


def _load():
    if not os.path.exists(library_path):
        raise ImportError(
            f"custom_ecc_cuda: {library_path} is missing; build it with "
            f"`make -C {os.path.join(os.path.dirname(_HERE), 'csrc')}` (sm_100a)")
    lib = ctypes.CDLL(library_path)
    p, i64, i32, f32, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    sig = {
        "ecc_strerror": ([i32], ctypes.c_char_p),
        "ecc_version": ([], i32),
        "ecc_hadamard_f16": ([p, i64, i32, p], i32),
        "ecc_hadamard_f32": ([p, i64, i32, p], i32),
        "ecc_compress": ([p, p, i64, i32, p], i32),
        "ecc_compress_strided": ([p, i64, i64, i64, p, i64, i64, i32, i32, i64, i32, p], i32),
        "ecc_compress_strided_pair": ([p, i64, i64, i64, p, i64, i64, p, i64, i64, i64, p, i64, i64, i32, i32, i64,
                                       i32, p], i32),
        "ecc_compress_strided_calibrated": ([p, i64, i64, i64, p, i64, i64, i32, i32, i64, i32, f32, f32, f32, p],
                                            i32),
        "ecc_compress_strided_pair_at": ([p, i64, i64, i64, p, i64, i64, p, i64, i64, i64, p, i64, i64, i32, i32,
                                          i64, i64, p, i32, p], i32),
        "ecc_compress_strided_calibrated_at": ([p, i64, i64, i64, p, i64, i64, i32, i32, i64, i64, p, i32, f32, f32,
                                                f32, p], i32),
        "ecc_decode_dev_workspace_size": ([i32, i32, i32, i64], sz),
        "ecc_decode_dev_splits": ([i32, i32, i64], i32),
        "ecc_decode_partials_dev": ([p, p, p, i64, i64, p, p, p, i32, i32, i32, i64, p, f32, i32, i32, p], i32),
        "ecc_decode_dev": ([p, p, p, i64, i64, p, p, sz, i32, i32, i32, i64, p, f32, i32, p], i32),
        "ecc_get_block_metadata": ([p, i64, i64, p, p], i32),
        "ecc_dequantize": ([p, p, i64, p], i32),
        "ecc_pack_soa": ([p, i64, p, i64, p, i64, p, i64, p], i32),
        "ecc_decode": ([p, p, p, i64, i64, p, p, sz, i32, i32, i32, i64, f32, i32, i32, p], i32),
        "ecc_decode_masked": ([p, p, p, i64, i64, p, p, p, sz, i32, i32, i32, i64, f32, i32, p], i32),
        "ecc_decode_workspace_size": ([i32, i32, i32, i64, i32], sz),
        "ecc_decode_default_splits": ([i32, i32, i64], i32),
        "ecc_decode_partials": ([p, p, p, i64, i64, p, p, p, i32, i32, i32, i64, f32, i32, i32, p], i32),
        "ecc_lse_merge": ([p, p, p, i64, i32, p, i32, p], i32),
        "ecc_lse_merge_to_record": ([p, p, p, i64, i32, p, p], i32),
        "ecc_lse_merge_records": ([p, i64, i32, i64, p, i32, p], i32),
        "ecc_device_status": ([i32], i32),
        "ecc_exchange_buffer_bytes": ([i64, i32], ctypes.c_size_t),
        "ecc_exchange_grid": ([i64], i32),
        "ecc_exchange_alloc": ([i64, i32, p, p], i32),
        "ecc_exchange_open": ([p, p], i32),
        "ecc_exchange_close": ([p], i32),
        "ecc_exchange_free": ([p], i32),
        "ecc_lse_exchange_merge": ([p, p, p, i64, i32, p, i32, i32, ctypes.c_uint32, ctypes.c_longlong, p, i32, p],
                                   i32),
        "ecc_lse_gather_merge": ([p, p, p, i64, i32, i32, p, i32, i32, ctypes.c_uint32, ctypes.c_longlong, p, i32,
                                  p], i32),
        "ecc_lse_exchange_merge_dev": ([p, p, p, i64, i32, p, i32, i32, p, ctypes.c_longlong, p, i32, p], i32),
        "ecc_lse_gather_merge_dev": ([p, p, p, i64, i32, i32, p, i32, i32, p, ctypes.c_longlong, p, i32, p], i32),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


_lib = _load()
_ws_lock = threading.Lock()
_ws_cache: dict = {}


def _check(rc: int, what: str):
    if rc != 0:
        msg = _lib.ecc_strerror(rc).decode()
        raise EccError(f"{what}: {msg} (code {rc})")


def _stream(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def _require_cuda(t: torch.Tensor, name: str):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")


def _require_input(t: torch.Tensor, name: str):
    _require_cuda(t, name)
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


# ---------------------------------------------------------------------------
# reference op surface (csrc/ecc_ops.cpp)
# ---------------------------------------------------------------------------
def hadamard_rotate(x: torch.Tensor) -> torch.Tensor:
    """In-place normalised WHT of each row of ``x`` [N, D] (fp16/fp32, D a
    power of two <= 1024); returns ``x``.  Arithmetic of
    custom_kv/ops_cpu.py:29 hadamard_rotate_cpu (fp32 butterfly, stride
    1..D/2, division by fp32(sqrt(D))), rounded to fp16 for fp16 input."""
    _require_input(x, "x")
    if x.dim() != 2:
        raise RuntimeError("Expected 2D tensor [N, D]")
    n, d = x.shape
    if d <= 0 or (d & (d - 1)) != 0:
        raise RuntimeError("D must be a power of 2")
    if d > 1024:
        raise RuntimeError("D must be <= 1024 (shared memory limit)")
    with torch.cuda.device(x.device):
        if x.dtype == torch.float16:
            rc = _lib.ecc_hadamard_f16(_ptr(x), n, d, _stream(x))
        elif x.dtype == torch.float32:
            rc = _lib.ecc_hadamard_f32(_ptr(x), n, d, _stream(x))
        else:
            raise RuntimeError("hadamard_rotate only supports float16 and float32")
    _check(rc, "hadamard_rotate")
    return x


def compress_and_store(x_rot: torch.Tensor, cache_raw: torch.Tensor) -> None:
    """Compress already-rotated fp16 vectors ``x_rot`` [N, 128] into the
    128-byte block pool ``cache_raw`` [N', 128] uint8 (N' >= N), row i into
    block i.  Bit-exact with the reference's CPU compress of the same input."""
    _require_input(x_rot, "x_rot")
    _require_input(cache_raw, "cache_raw")
    if x_rot.dtype != torch.float16:
        raise RuntimeError("x_rot must be float16")
    if cache_raw.dtype != torch.uint8:
        raise RuntimeError("cache_raw must be uint8")
    if x_rot.dim() != 2 or x_rot.shape[1] != D:
        raise RuntimeError("Only D=128 supported (hardcoded kernel)")
    if cache_raw.dim() != 2 or cache_raw.shape[1] != BLOCK_BYTES:
        raise RuntimeError("Cache must be [N, 128] bytes")
    if cache_raw.shape[0] < x_rot.shape[0]:
        raise RuntimeError("cache_raw has fewer blocks than x_rot has rows")
    if x_rot.device != cache_raw.device:
        raise RuntimeError("x_rot and cache_raw must be on the same device")
    with torch.cuda.device(x_rot.device):
        rc = _lib.ecc_compress(_ptr(x_rot), _ptr(cache_raw), x_rot.shape[0], 0, _stream(x_rot))
    _check(rc, "compress_and_store")


def get_block_metadata(cache_raw: torch.Tensor, block_idx: int) -> torch.Tensor:
    """(scale, zero_point, alpha) of block ``block_idx`` as a CPU float32[3]
    tensor.  Synchronous, like the reference's debug accessor."""
    _require_input(cache_raw, "cache_raw")
    n_blocks = cache_raw.numel() // BLOCK_BYTES
    out = torch.empty(3, dtype=torch.float32)
    with torch.cuda.device(cache_raw.device):
        rc = _lib.ecc_get_block_metadata(_ptr(cache_raw), n_blocks, int(block_idx),
                                         ctypes.c_void_p(out.data_ptr()), _stream(cache_raw))
    _check(rc, "get_block_metadata")
    return out


# ---------------------------------------------------------------------------
# pool ops used by custom_kv
# ---------------------------------------------------------------------------
def _pool_strides(pool: torch.Tensor, name: str):
    """A block pool is a uint8 tensor [..., B, H, L, R] whose last two dims
    are contiguous records of R = 128 bytes (the block) or 96 (the block
    without its zero pad sector, RECORD96); returns (bs_b, bs_h) in records."""
    _require_cuda(pool, name)
    if pool.dtype != torch.uint8 or pool.dim() < 4 or pool.shape[-1] not in (BLOCK_BYTES, RECORD96):
        raise RuntimeError(f"{name} must be a uint8 block pool [B, H, L, 128] (or [B, H, L, 96])")
    rb = pool.shape[-1]
    if pool.stride(-1) != 1 or pool.stride(-2) != rb:
        raise RuntimeError(f"{name}: blocks along L must be contiguous {rb}-byte rows")
    sb, sh = pool.stride(-4), pool.stride(-3)
    if sb % rb or sh % rb:
        raise RuntimeError(f"{name}: batch/head strides must be whole blocks")
    return sb // rb, sh // rb


def _cmode(rotate: bool, *pools) -> int:
    """The compress entry points' `rotate` argument: WHT bit and record size."""
    rbs = {p.shape[-1] for p in pools if p is not None}
    if len(rbs) != 1:
        raise RuntimeError("the pools of one call must have the same record size")
    return int(bool(rotate)) | (COMPRESS_BLOCK96 if rbs.pop() == RECORD96 else 0)


def _rec_flag(k_pool: torch.Tensor) -> int:
    return BLOCK96 if k_pool.shape[-1] == RECORD96 else 0


def compress_into(x: torch.Tensor, pool: torch.Tensor, pos: int = 0, rotate: bool = True) -> None:
    """Compress ``x`` [B, H, L, 128] fp16 (any strides with a contiguous last
    dim) into ``pool`` [B, H, Lcap, 128] at token positions pos .. pos+L-1.
    ``rotate`` applies the WHT first (custom_kv/ops_cpu.py:198)."""
    _require_cuda(x, "x")
    if x.dtype != torch.float16:
        raise RuntimeError("x must be float16")
    if x.dim() != 4 or x.shape[-1] != D:
        raise RuntimeError("Only D=128 supported (hardcoded kernel)")
    if x.stride(-1) != 1:
        raise RuntimeError("x must have a contiguous last dimension")
    bs_b, bs_h = _pool_strides(pool, "pool")
    B, H, L, _ = x.shape
    if pool.shape[-4] != B or pool.shape[-3] != H:
        raise RuntimeError("pool batch/head dims do not match x")
    if pos < 0 or pos + L > pool.shape[-2]:
        raise RuntimeError(f"positions {pos}..{pos + L} exceed the pool capacity {pool.shape[-2]}")
    if x.device != pool.device:
        raise RuntimeError("x and pool must be on the same device")
    dst = pool[..., pos:, :] if pos else pool
    with torch.cuda.device(x.device):
        rc = _lib.ecc_compress_strided(_ptr(x), x.stride(0), x.stride(1), x.stride(2), _ptr(dst), bs_b, bs_h,
                                       B, H, L, _cmode(rotate, pool), _stream(x))
    _check(rc, "compress_into")


def _compress_dst(x: torch.Tensor, pool: torch.Tensor, pos: int, name: str):
    _require_cuda(x, name)
    if x.dtype != torch.float16:
        raise RuntimeError(f"{name} must be float16")
    if x.dim() != 4 or x.shape[-1] != D:
        raise RuntimeError("Only D=128 supported (hardcoded kernel)")
    if x.stride(-1) != 1:
        raise RuntimeError(f"{name} must have a contiguous last dimension")
    bs = _pool_strides(pool, "pool")
    B, H, L, _ = x.shape
    if pool.shape[-4] != B or pool.shape[-3] != H:
        raise RuntimeError("pool batch/head dims do not match x")
    if pos < 0 or pos + L > pool.shape[-2]:
        raise RuntimeError(f"positions {pos}..{pos + L} exceed the pool capacity {pool.shape[-2]}")
    if x.device != pool.device:
        raise RuntimeError("x and pool must be on the same device")
    return (pool[..., pos:, :] if pos else pool), bs


def compress_calibrated_into(x: torch.Tensor, pool: torch.Tensor, scale: float, zero: float, alpha: float,
                             pos: int = 0, rotate: bool = True) -> None:
    """compress_into with fixed quantiser parameters -- a layer's (scale, zero,
    alpha) from a calibration config (custom_kv/calibration.py:232-237) -- in
    place of each vector's own statistics: the arithmetic of
    ops_cpu.lloyd_max_quantize_cpu(x_rot, scale, zero) + compute_syndrome_cpu,
    every block storing fp16 of the fp32 scale, zero and alpha."""
    dst, bs = _compress_dst(x, pool, pos, "x")
    B, H, L, _ = x.shape
    with torch.cuda.device(x.device):
        rc = _lib.ecc_compress_strided_calibrated(_ptr(x), x.stride(0), x.stride(1), x.stride(2), _ptr(dst), bs[0],
                                                  bs[1], B, H, L, _cmode(rotate, pool), float(scale), float(zero),
                                                  float(alpha), _stream(x))
    _check(rc, "compress_calibrated_into")


def compress_pair_into(k: torch.Tensor, v: torch.Tensor, kpool: torch.Tensor, vpool: torch.Tensor, pos: int = 0,
                       rotate: bool = True) -> None:
    """compress_into of ``k`` into ``kpool`` and ``v`` into ``vpool`` (same
    [B, H, L, 128] shape, same positions) in one launch."""
    if k.shape != v.shape:
        raise RuntimeError("k and v must have the same shape")
    kdst, kbs = _compress_dst(k, kpool, pos, "k")
    vdst, vbs = _compress_dst(v, vpool, pos, "v")
    B, H, L, _ = k.shape
    with torch.cuda.device(k.device):
        rc = _lib.ecc_compress_strided_pair(_ptr(k), k.stride(0), k.stride(1), k.stride(2), _ptr(kdst), kbs[0],
                                            kbs[1], _ptr(v), v.stride(0), v.stride(1), v.stride(2), _ptr(vdst),
                                            vbs[0], vbs[1], B, H, L, _cmode(rotate, kpool, vpool), _stream(k))
    _check(rc, "compress_pair_into")


def rotate_and_compress(x: torch.Tensor, blocks: torch.Tensor | None = None) -> torch.Tensor:
    """WHT + compress of contiguous rows ``x`` [N, 128] fp16 -> blocks [N, 128] u8."""
    _require_input(x, "x")
    if x.dtype != torch.float16 or x.dim() != 2 or x.shape[1] != D:
        raise RuntimeError("x must be float16 [N, 128]")
    if blocks is None:
        blocks = torch.empty((x.shape[0], BLOCK_BYTES), dtype=torch.uint8, device=x.device)
    _require_input(blocks, "blocks")
    with torch.cuda.device(x.device):
        rc = _lib.ecc_compress(_ptr(x), _ptr(blocks), x.shape[0], 1, _stream(x))
    _check(rc, "rotate_and_compress")
    return blocks


def dequantize(blocks: torch.Tensor) -> torch.Tensor:
    """[..., 128] u8 contiguous blocks (or [..., 96] records) -> [..., 128]
    fp16 reconstructions (C[q]*scale + zero) + alpha*s
    (custom_kv/fused_decode.py:229-241)."""
    _require_input(blocks, "blocks")
    if blocks.dim() < 1 or blocks.shape[-1] not in (BLOCK_BYTES, RECORD96):
        raise RuntimeError("blocks must be [..., 128] (or [..., 96]) uint8")
    if blocks.shape[-1] == RECORD96:  # the pad sector back in place (zeros)
        blocks = torch.nn.functional.pad(blocks, (0, BLOCK_BYTES - RECORD96))
    n = blocks.numel() // BLOCK_BYTES
    out = torch.empty(blocks.shape[:-1] + (D,), dtype=torch.float16, device=blocks.device)
    with torch.cuda.device(blocks.device):
        rc = _lib.ecc_dequantize(_ptr(blocks), _ptr(out), n, _stream(blocks))
    _check(rc, "dequantize")
    return out


def pack_soa(int4: torch.Tensor, syn: torch.Tensor, meta: torch.Tensor) -> torch.Tensor:
    """Reference SoA trio (int4 [..., 64] u8, syn [..., 16] u8, meta [..., 3]
    fp16, custom_kv/cache.py:79-84) -> contiguous blocks [..., 128] u8."""
    for t, nme in ((int4, "int4"), (syn, "syn"), (meta, "meta")):
        _require_cuda(t, nme)
    lead = int4.shape[:-1]
    if int4.shape[-1] != 64 or syn.shape[-1] != 16 or meta.shape[-1] != 3 or syn.shape[:-1] != lead \
            or meta.shape[:-1] != lead:
        raise RuntimeError("expected int4 [..., 64], syn [..., 16], meta [..., 3]")
    if int4.dtype != torch.uint8 or syn.dtype != torch.uint8 or meta.dtype != torch.float16:
        raise RuntimeError("expected uint8 int4/syn and float16 meta")
    i4 = int4.reshape(-1, 64)
    sy = syn.reshape(-1, 16)
    me = meta.reshape(-1, 3)
    for t, w in ((i4, 1), (sy, 1), (me, 1)):
        if t.stride(-1) != w:
            raise RuntimeError("SoA tensors need a contiguous last dim")
    n = i4.shape[0]
    out = torch.empty(lead + (BLOCK_BYTES,), dtype=torch.uint8, device=int4.device)
    with torch.cuda.device(int4.device):
        rc = _lib.ecc_pack_soa(_ptr(i4), i4.stride(0), _ptr(sy), sy.stride(0), _ptr(me), me.stride(0) * 2,
                               _ptr(out), n, _stream(int4))
    _check(rc, "pack_soa")
    return out


def default_splits(B: int, hkv: int, seq_len: int) -> int:
    return int(_lib.ecc_decode_default_splits(B, hkv, seq_len))


def decode_workspace_size(B: int, hq: int, hkv: int, seq_len: int, num_splits: int = 0) -> int:
    return int(_lib.ecc_decode_workspace_size(B, hq, hkv, seq_len, num_splits))


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A grow-only per-device workspace reused across calls (stream-ordered:
    calls on one stream never overlap)."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    with _ws_lock:
        ws = _ws_cache.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _ws_cache[key] = ws
    return ws


def _query(q: torch.Tensor):
    _require_cuda(q, "query")
    if q.dtype != torch.float16:
        raise RuntimeError("query must be float16")
    if q.dim() == 4:
        if q.shape[2] != 1:
            raise RuntimeError("decode attention takes one query token ([B, H, 1, D])")
        q3 = q[:, :, 0, :]
    elif q.dim() == 3:
        q3 = q
    else:
        raise RuntimeError("query must be [B, H, 1, D] or [B, H, D]")
    if q3.shape[-1] != D:
        raise RuntimeError(f"Only D=128 supported, got {q3.shape[-1]}")
    return q3.contiguous()


def decode_attention(query: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, seq_len: int,
                     sm_scale: float | None = None, rotate_q: bool = False, unrotate_out: bool = False,
                     num_splits: int = 0, out: torch.Tensor | None = None,
                     workspace: torch.Tensor | None = None, cuda_cores: bool = False,
                     kernel: str = "auto") -> torch.Tensor:
    """One decode step of GQA attention over block pools [B, Hkv, Lcap, 128].

    query [B, Hq, 1, 128] (or [B, Hq, 128]) fp16 -> [B, Hq, 1, 128] fp16.
    Query head h reads kv head h // (Hq // Hkv).  ``sm_scale`` defaults to
    1/sqrt(128) (custom_kv/fused_decode.py:57).  ``kernel`` picks the
    implementation: "auto"/"tma" (TMA-fed warp-specialised tensor-core kernel,
    falling back to "register" for pool layouts a tensor map cannot describe),
    "register" (tensor cores with per-lane global loads) or "cuda_cores"
    (always used for more than 8 query heads per kv head); ``cuda_cores=True``
    is a shorthand for the last."""
    q3 = _query(query)
    kbs = _pool_strides(k_pool, "k_pool")
    vbs = _pool_strides(v_pool, "v_pool")
    if kbs != vbs or k_pool.shape != v_pool.shape:
        raise RuntimeError("k_pool and v_pool must have the same shape and strides")
    B, hq, _ = q3.shape
    hkv = k_pool.shape[-3]
    if k_pool.shape[-4] != B:
        raise RuntimeError("pool batch does not match the query")
    if hq % hkv:
        raise RuntimeError(f"query heads ({hq}) must be a multiple of kv heads ({hkv})")
    if seq_len < 0 or seq_len > k_pool.shape[-2]:
        raise RuntimeError(f"seq_len {seq_len} exceeds the pool capacity {k_pool.shape[-2]}")
    if out is None:
        out = torch.empty((B, hq, 1, D), dtype=torch.float16, device=q3.device)
    elif not out.is_contiguous() or out.dtype != torch.float16 or out.numel() != B * hq * D:
        raise RuntimeError("out must be a contiguous float16 tensor of B*Hq*128 elements")
    flags = (ROTATE_Q if rotate_q else 0) | (UNROTATE_OUT if unrotate_out else 0) | (CUDA_CORES if cuda_cores else 0)
    flags |= _KERNEL_FLAGS[kernel] | _rec_flag(k_pool)
    scale = float(sm_scale) if sm_scale is not None else 0.0
    need = decode_workspace_size(B, hq, hkv, seq_len, num_splits)
    with torch.cuda.device(q3.device):
        ws = workspace if workspace is not None else _workspace(q3.device, need)
        if ws.numel() < need:
            raise RuntimeError(f"workspace too small: {ws.numel()} < {need} bytes")
        rc = _lib.ecc_decode(_ptr(q3), _ptr(k_pool), _ptr(v_pool), kbs[0], kbs[1], _ptr(out), _ptr(ws),
                             ws.numel(), B, hq, hkv, int(seq_len), scale, flags, int(num_splits), _stream(q3))
    _check(rc, "decode_attention")
    return out


def decode_attention_masked(query: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, seq_len: int,
                            start: torch.Tensor, sm_scale: float | None = None, rotate_q: bool = False,
                            unrotate_out: bool = False, out: torch.Tensor | None = None,
                            workspace: torch.Tensor | None = None) -> torch.Tensor:
    """decode_attention of a left-padded batch: sequence b attends to tokens
    [start[b], seq_len) of its pools only (``start`` int32 [B] on the GPU, read
    when the kernel runs); the tokens before start[b] are padding.  GQA groups
    of up to 8 (the TMA-fed kernel); an output row whose whole context is
    masked is zero."""
    q3 = _query(query)
    kbs = _pool_strides(k_pool, "k_pool")
    vbs = _pool_strides(v_pool, "v_pool")
    if kbs != vbs or k_pool.shape != v_pool.shape:
        raise RuntimeError("k_pool and v_pool must have the same shape and strides")
    B, hq, _ = q3.shape
    hkv = k_pool.shape[-3]
    if k_pool.shape[-4] != B or hq % hkv:
        raise RuntimeError("pool batch or GQA shape does not match the query")
    if seq_len < 1 or seq_len > k_pool.shape[-2]:
        raise RuntimeError(f"seq_len {seq_len} must be in [1, {k_pool.shape[-2]}]")
    _dev_int(start, "start", q3.device)
    if start.numel() != B or not start.is_contiguous():
        raise RuntimeError("start must be a contiguous int32 tensor of B elements")
    if out is None:
        out = torch.empty((B, hq, 1, D), dtype=torch.float16, device=q3.device)
    elif not out.is_contiguous() or out.dtype != torch.float16 or out.numel() != B * hq * D:
        raise RuntimeError("out must be a contiguous float16 tensor of B*Hq*128 elements")
    flags = (ROTATE_Q if rotate_q else 0) | (UNROTATE_OUT if unrotate_out else 0) | _rec_flag(k_pool)
    need = decode_workspace_size(B, hq, hkv, seq_len, 0)
    with torch.cuda.device(q3.device):
        ws = workspace if workspace is not None else _workspace(q3.device, need)
        if ws.numel() < need:
            raise RuntimeError(f"workspace too small: {ws.numel()} < {need} bytes")
        rc = _lib.ecc_decode_masked(_ptr(q3), _ptr(k_pool), _ptr(v_pool), kbs[0], kbs[1], _ptr(start), _ptr(out),
                                    _ptr(ws), ws.numel(), B, hq, hkv, int(seq_len),
                                    float(sm_scale) if sm_scale else 0.0, flags, _stream(q3))
    _check(rc, "decode_attention_masked")
    return out


def decode_partials(query: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, seq_len: int,
                    num_splits: int, sm_scale: float | None = None, rotate_q: bool = False,
                    cuda_cores: bool = False, kernel: str = "auto"):
    """Split partials (m, l, o) of one decode step over token positions
    [0, seq_len) of the pools: m, l [B, Hq, num_splits] fp32 (m in natural-log
    units), o [B, Hq, num_splits, 128] fp32 unnormalised."""
    q3 = _query(query)
    kbs = _pool_strides(k_pool, "k_pool")
    vbs = _pool_strides(v_pool, "v_pool")
    if kbs != vbs or k_pool.shape[-1] != v_pool.shape[-1]:
        raise RuntimeError("k_pool and v_pool must have the same strides and record size")
    B, hq, _ = q3.shape
    hkv = k_pool.shape[-3]
    if num_splits <= 0:
        raise RuntimeError("num_splits must be positive")
    dev = q3.device
    pm = torch.empty((B, hq, num_splits), dtype=torch.float32, device=dev)
    pl = torch.empty_like(pm)
    po = torch.empty((B, hq, num_splits, D), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        rc = _lib.ecc_decode_partials(_ptr(q3), _ptr(k_pool), _ptr(v_pool), kbs[0], kbs[1], _ptr(pm), _ptr(pl),
                                      _ptr(po), B, hq, hkv, int(seq_len),
                                      float(sm_scale) if sm_scale is not None else 0.0,
                                      (ROTATE_Q if rotate_q else 0) | (CUDA_CORES if cuda_cores else 0)
                                      | _KERNEL_FLAGS[kernel] | _rec_flag(k_pool), int(num_splits), _stream(q3))
    _check(rc, "decode_partials")
    return pm, pl, po


def lse_merge(pm: torch.Tensor, pl: torch.Tensor, po: torch.Tensor, unrotate_out: bool = False,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """Merge partials along their split axis: pm/pl [..., n], po [..., n, 128]
    -> [..., 128] fp16 (optionally WHT-unrotated)."""
    for t, nme in ((pm, "pm"), (pl, "pl"), (po, "po")):
        _require_input(t, nme)
        if t.dtype != torch.float32:
            raise RuntimeError(f"{nme} must be float32")
    n = pm.shape[-1]
    rows = pm.numel() // max(n, 1)
    if pl.shape != pm.shape or po.shape != pm.shape + (D,):
        raise RuntimeError("partial shapes disagree")
    if out is None:
        out = torch.empty(pm.shape[:-1] + (D,), dtype=torch.float16, device=pm.device)
    with torch.cuda.device(pm.device):
        rc = _lib.ecc_lse_merge(_ptr(pm), _ptr(pl), _ptr(po), rows, n, _ptr(out),
                                UNROTATE_OUT if unrotate_out else 0, _stream(pm))
    _check(rc, "lse_merge")
    return out


RECORD_FLOATS = 2 + D


def _check_partials(pm: torch.Tensor, pl: torch.Tensor, po: torch.Tensor):
    """Contiguous fp32 CUDA split partials pm/pl [..., n], po [..., n, 128];
    returns (rows, n)."""
    for t, nme in ((pm, "pm"), (pl, "pl"), (po, "po")):
        _require_input(t, nme)
        if t.dtype != torch.float32:
            raise RuntimeError(f"{nme} must be float32")
    n = pm.shape[-1]
    rows = pm.numel() // max(n, 1)
    if pl.shape != pm.shape or po.shape != pm.shape + (D,):
        raise RuntimeError("partial shapes disagree")
    return rows, n


def lse_merge_to_record(pm: torch.Tensor, pl: torch.Tensor, po: torch.Tensor,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """Merge partials along their split axis into one partial record per row:
    pm/pl [..., n], po [..., n, 128] -> [..., 130] fp32 {m, l, o[128]} (o
    unnormalised).  Records of several devices merge with lse_merge_records."""
    rows, n = _check_partials(pm, pl, po)
    if out is None:
        out = torch.empty(pm.shape[:-1] + (RECORD_FLOATS,), dtype=torch.float32, device=pm.device)
    elif not out.is_contiguous() or out.dtype != torch.float32 or out.numel() != rows * RECORD_FLOATS:
        raise RuntimeError("out must be a contiguous float32 tensor of rows*130 elements")
    with torch.cuda.device(pm.device):
        rc = _lib.ecc_lse_merge_to_record(_ptr(pm), _ptr(pl), _ptr(po), rows, n, _ptr(out), _stream(pm))
    _check(rc, "lse_merge_to_record")
    return out


def lse_merge_records(records: torch.Tensor, unrotate_out: bool = False,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """Merge n partial records per row: records [n, ..., 130] (e.g. the
    all-gather of every device's lse_merge_to_record result) -> [..., 128] fp16."""
    _require_input(records, "records")
    if records.dtype != torch.float32 or records.shape[-1] != RECORD_FLOATS or records.dim() < 2:
        raise RuntimeError("records must be float32 [n, ..., 130]")
    n = records.shape[0]
    rows = records[0].numel() // RECORD_FLOATS
    if out is None:
        out = torch.empty(records.shape[1:-1] + (D,), dtype=torch.float16, device=records.device)
    with torch.cuda.device(records.device):
        rc = _lib.ecc_lse_merge_records(_ptr(records), rows, n, rows * RECORD_FLOATS, _ptr(out),
                                        UNROTATE_OUT if unrotate_out else 0, _stream(records))
    _check(rc, "lse_merge_records")
    return out


def version() -> int:
    return int(_lib.ecc_version())


def exchange_buffer_bytes(rows: int, world: int) -> int:
    """Bytes of one rank's peer-exchange buffer for ``rows`` rows (B * Hq)."""
    return int(_lib.ecc_exchange_buffer_bytes(rows, world))


IPC_HANDLE_BYTES = 64


def exchange_alloc(rows: int, world: int, device: torch.device):
    """This rank's zero-filled exchange buffer on ``device``: (device address,
    IPC handle bytes for the other ranks).  Free with exchange_free."""
    buf = ctypes.c_void_p()
    handle = (ctypes.c_char * IPC_HANDLE_BYTES)()
    with torch.cuda.device(device):
        rc = _lib.ecc_exchange_alloc(int(rows), int(world), ctypes.byref(buf), handle)
    _check(rc, "exchange_alloc")
    return buf.value, bytes(handle)


def exchange_open(handle: bytes, device: torch.device) -> int:
    """Map another rank's exchange buffer (its IPC handle) on ``device``;
    returns its device address in this process.  Unmap with exchange_close."""
    if len(handle) != IPC_HANDLE_BYTES:
        raise RuntimeError("bad IPC handle")
    ptr = ctypes.c_void_p()
    with torch.cuda.device(device):
        rc = _lib.ecc_exchange_open(ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES), ctypes.byref(ptr))
    _check(rc, "exchange_open")
    return ptr.value


def exchange_close(ptr: int, device: torch.device) -> None:
    with torch.cuda.device(device):
        _check(_lib.ecc_exchange_close(ctypes.c_void_p(ptr)), "exchange_close")


def exchange_free(ptr: int, device: torch.device) -> None:
    with torch.cuda.device(device):
        _check(_lib.ecc_exchange_free(ctypes.c_void_p(ptr)), "exchange_free")


def lse_exchange_merge(pm: torch.Tensor, pl: torch.Tensor, po: torch.Tensor, peer_ptrs, rank: int, epoch: int,
                       unrotate_out: bool = False, out: torch.Tensor | None = None,
                       wait_cycles: int = 10_000_000_000) -> torch.Tensor:
    """Sequence-sharded combine over peer memory: this rank's split partials
    pm/pl [..., n], po [..., n, 128] are merged into one record per row,
    stored into every rank's exchange buffer (``peer_ptrs``: device addresses
    of all ranks' buffers as mapped in this process, ``peer_ptrs[rank]`` this
    rank's own), and the records of all ranks merged into out [..., 128]
    fp16 -- what lse_merge_to_record, an all-gather and lse_merge_records
    give, in one kernel.  ``epoch``: 1, 2, ... in step on every rank, or an
    epoch state (int64 CUDA tensor [2], zero-filled once) that the kernel
    reads and advances itself, for calls recorded in a CUDA graph."""
    rows, n = _check_partials(pm, pl, po)
    W = len(peer_ptrs)
    if out is None:
        out = torch.empty(pm.shape[:-1] + (D,), dtype=torch.float16, device=pm.device)
    elif not out.is_contiguous() or out.dtype != torch.float16 or out.numel() != rows * D:
        raise RuntimeError("out must be a contiguous float16 tensor of rows*128 elements")
    arr = (ctypes.c_void_p * W)(*[int(x) for x in peer_ptrs])
    with torch.cuda.device(pm.device):
        if isinstance(epoch, torch.Tensor):
            _epoch_state(epoch, pm.device)
            rc = _lib.ecc_lse_exchange_merge_dev(_ptr(pm), _ptr(pl), _ptr(po), rows, n, arr, W, int(rank),
                                                 _ptr(epoch), int(wait_cycles), _ptr(out),
                                                 UNROTATE_OUT if unrotate_out else 0, _stream(pm))
        else:
            rc = _lib.ecc_lse_exchange_merge(_ptr(pm), _ptr(pl), _ptr(po), rows, n, arr, W, int(rank), int(epoch),
                                             int(wait_cycles), _ptr(out), UNROTATE_OUT if unrotate_out else 0,
                                             _stream(pm))
    _check(rc, "lse_exchange_merge")
    return out


def _epoch_state(t: torch.Tensor, device) -> None:
    if not t.is_cuda or t.dtype != torch.int64 or t.numel() != 2 or not t.is_contiguous() or t.device != device:
        raise RuntimeError("an epoch state must be a contiguous int64 CUDA tensor of 2 elements on the partials' "
                           "device")


def lse_gather_merge(pm: torch.Tensor, pl: torch.Tensor, po: torch.Tensor, peer_ptrs, rank: int, epoch: int,
                     unrotate_out: bool = False, out: torch.Tensor | None = None,
                     wait_cycles: int = 10_000_000_000) -> torch.Tensor:
    """Kv-head-sharded output gather over peer memory: this rank's split
    partials pm/pl [B, hq_local, n], po [B, hq_local, n, 128] are merged into
    its fp16 output rows, which are stored into every rank's buffer
    (``peer_ptrs`` as for lse_exchange_merge); the result out [B, W*hq_local,
    1, 128] holds every rank's heads (rank q's at heads q*hq_local ..) -- what
    lse_merge and an all-gather of the outputs give, in one kernel.
    ``epoch``: 1, 2, ... in step on every rank, or an epoch state (int64
    CUDA tensor [2], zero-filled once) that the kernel reads and advances
    itself, for calls recorded in a CUDA graph."""
    rows, n = _check_partials(pm, pl, po)
    if pm.dim() != 3:
        raise RuntimeError("partials must be [B, hq_local, n]")
    B, hq_l = pm.shape[0], pm.shape[1]
    W = len(peer_ptrs)
    if out is None:
        out = torch.empty((B, W * hq_l, 1, D), dtype=torch.float16, device=pm.device)
    elif not out.is_contiguous() or out.dtype != torch.float16 or out.numel() != B * W * hq_l * D:
        raise RuntimeError("out must be a contiguous float16 tensor of B*W*hq_local*128 elements")
    arr = (ctypes.c_void_p * W)(*[int(x) for x in peer_ptrs])
    with torch.cuda.device(pm.device):
        if isinstance(epoch, torch.Tensor):
            _epoch_state(epoch, pm.device)
            rc = _lib.ecc_lse_gather_merge_dev(_ptr(pm), _ptr(pl), _ptr(po), rows, n, hq_l, arr, W, int(rank),
                                               _ptr(epoch), int(wait_cycles), _ptr(out),
                                               UNROTATE_OUT if unrotate_out else 0, _stream(pm))
        else:
            rc = _lib.ecc_lse_gather_merge(_ptr(pm), _ptr(pl), _ptr(po), rows, n, hq_l, arr, W, int(rank),
                                           int(epoch), int(wait_cycles), _ptr(out),
                                           UNROTATE_OUT if unrotate_out else 0, _stream(pm))
    _check(rc, "lse_gather_merge")
    return out


def device_status(reset: bool = False) -> int:
    """Device-side error flag of the current device since the last reset:
    1 if a decode kernel gave up a bounded wait (it returned early instead of
    hanging), 2 if the decode kernel found its shared memory at an unexpected
    address (it computed nothing), 3 if an append at a device-side position
    was out of range (it wrote nothing), 4 if lse_exchange_merge gave up
    waiting for another rank's records (those rows were not written), else 0."""
    rc = int(_lib.ecc_device_status(1 if reset else 0))
    if rc < 0:
        _check(rc, "device_status")
    return rc


# ---------------------------------------------------------------------------
# Positions and lengths in device memory (CUDA-graph replay of decode steps)
# ---------------------------------------------------------------------------
def _dev_int(t: torch.Tensor, name: str, device) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype != torch.int32 or t.numel() < 1:
        raise RuntimeError(f"{name} must be an int32 CUDA tensor")
    if t.device != device:
        raise RuntimeError(f"{name} must be on the device of the pools")


def _whole_pool(x: torch.Tensor, pool: torch.Tensor, name: str):
    _require_cuda(x, name)
    if x.dtype != torch.float16 or x.dim() != 4 or x.shape[-1] != D or x.stride(-1) != 1:
        raise RuntimeError(f"{name} must be float16 [B, H, L, 128] with a contiguous last dimension")
    bs = _pool_strides(pool, "pool")
    if pool.shape[-4] != x.shape[0] or pool.shape[-3] != x.shape[1]:
        raise RuntimeError("pool batch/head dims do not match")
    if x.device != pool.device:
        raise RuntimeError(f"{name} and pool must be on the same device")
    return bs


def compress_pair_at(k: torch.Tensor, v: torch.Tensor | None, kpool: torch.Tensor, vpool: torch.Tensor | None,
                     pos_dev: torch.Tensor, rotate: bool = True) -> None:
    """compress_pair_into at token position ``pos_dev[0]`` (int32 on the GPU,
    read when the kernel runs), so that a launch recorded in a CUDA graph
    appends at the current end of a growing cache.  ``v``/``vpool`` None:
    ``k`` alone.  An out-of-range position writes nothing and raises the flag
    device_status() reports."""
    kbs = _whole_pool(k, kpool, "k")
    _dev_int(pos_dev, "pos_dev", k.device)
    B, H, L, _ = k.shape
    if v is not None:
        if v.shape != k.shape or vpool is None or vpool.shape[-2] != kpool.shape[-2]:
            raise RuntimeError("v, vpool must match k, kpool")
        vbs = _whole_pool(v, vpool, "v")
        vargs = (_ptr(v), v.stride(0), v.stride(1), v.stride(2), _ptr(vpool), vbs[0], vbs[1])
    else:
        vargs = (None, 0, 0, 0, None, 0, 0)
    with torch.cuda.device(k.device):
        rc = _lib.ecc_compress_strided_pair_at(_ptr(k), k.stride(0), k.stride(1), k.stride(2), _ptr(kpool), kbs[0],
                                               kbs[1], *vargs, B, H, L, kpool.shape[-2], _ptr(pos_dev),
                                               _cmode(rotate, kpool, vpool if v is not None else None), _stream(k))
    _check(rc, "compress_pair_at")


def compress_calibrated_at(x: torch.Tensor, pool: torch.Tensor, scale: float, zero: float, alpha: float,
                           pos_dev: torch.Tensor, rotate: bool = True) -> None:
    """compress_calibrated_into at the device-side position ``pos_dev[0]``."""
    bs = _whole_pool(x, pool, "x")
    _dev_int(pos_dev, "pos_dev", x.device)
    B, H, L, _ = x.shape
    with torch.cuda.device(x.device):
        rc = _lib.ecc_compress_strided_calibrated_at(_ptr(x), x.stride(0), x.stride(1), x.stride(2), _ptr(pool), bs[0],
                                                     bs[1], B, H, L, pool.shape[-2], _ptr(pos_dev), _cmode(rotate, pool),
                                                     float(scale), float(zero), float(alpha), _stream(x))
    _check(rc, "compress_calibrated_at")


def decode_dev_workspace_size(B: int, hq: int, hkv: int, max_len: int) -> int:
    return int(_lib.ecc_decode_dev_workspace_size(B, hq, hkv, max_len))


def decode_attention_dev(query: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, seq_len_dev: torch.Tensor,
                         sm_scale: float | None = None, rotate_q: bool = False, unrotate_out: bool = False,
                         out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """decode_attention over the first ``seq_len_dev[0]`` tokens (int32 on the
    GPU, read when the kernel runs, clamped to [1, pool capacity]): one
    recorded launch serves every length of a growing cache.  The split count
    is fixed by the pool capacity; GQA groups of up to 8."""
    q3 = _query(query)
    kbs = _pool_strides(k_pool, "k_pool")
    vbs = _pool_strides(v_pool, "v_pool")
    if kbs != vbs or k_pool.shape != v_pool.shape:
        raise RuntimeError("k_pool and v_pool must have the same shape and strides")
    B, hq, _ = q3.shape
    hkv, cap = k_pool.shape[-3], k_pool.shape[-2]
    if k_pool.shape[-4] != B or hq % hkv:
        raise RuntimeError("pool batch or GQA shape does not match the query")
    _dev_int(seq_len_dev, "seq_len_dev", q3.device)
    if out is None:
        out = torch.empty((B, hq, 1, D), dtype=torch.float16, device=q3.device)
    flags = (ROTATE_Q if rotate_q else 0) | (UNROTATE_OUT if unrotate_out else 0) | _rec_flag(k_pool)
    need = decode_dev_workspace_size(B, hq, hkv, cap)
    with torch.cuda.device(q3.device):
        ws = workspace if workspace is not None else _workspace(q3.device, need)
        if ws.numel() < need:
            raise RuntimeError(f"workspace too small: {ws.numel()} < {need} bytes")
        rc = _lib.ecc_decode_dev(_ptr(q3), _ptr(k_pool), _ptr(v_pool), kbs[0], kbs[1], _ptr(out), _ptr(ws), ws.numel(),
                                 B, hq, hkv, cap, _ptr(seq_len_dev), float(sm_scale) if sm_scale else 0.0, flags,
                                 _stream(q3))
    _check(rc, "decode_attention_dev")
    return out


def decode_dev_splits(B: int, hkv: int, max_len: int) -> int:
    """Split count of the device-length decode for pools of max_len tokens."""
    return int(_lib.ecc_decode_dev_splits(B, hkv, max_len))


def decode_partials_dev(query: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, seq_len_dev: torch.Tensor,
                        num_splits: int, sm_scale: float | None = None, rotate_q: bool = False,
                        out: tuple | None = None):
    """decode_partials over the first ``seq_len_dev[0]`` tokens (int32 on the
    GPU, read when the kernel runs); ``num_splits`` >= decode_dev_splits(B,
    Hkv, capacity).  Returns (m, l, o) like decode_partials (``out``: reuse
    three such tensors)."""
    q3 = _query(query)
    kbs = _pool_strides(k_pool, "k_pool")
    if kbs != _pool_strides(v_pool, "v_pool") or k_pool.shape != v_pool.shape:
        raise RuntimeError("k_pool and v_pool must have the same shape and strides")
    B, hq, _ = q3.shape
    hkv, cap = k_pool.shape[-3], k_pool.shape[-2]
    _dev_int(seq_len_dev, "seq_len_dev", q3.device)
    if out is None:
        pm = torch.empty((B, hq, num_splits), dtype=torch.float32, device=q3.device)
        pl = torch.empty_like(pm)
        po = torch.empty((B, hq, num_splits, D), dtype=torch.float32, device=q3.device)
    else:
        pm, pl, po = out
    with torch.cuda.device(q3.device):
        rc = _lib.ecc_decode_partials_dev(_ptr(q3), _ptr(k_pool), _ptr(v_pool), kbs[0], kbs[1], _ptr(pm), _ptr(pl),
                                          _ptr(po), B, hq, hkv, cap, _ptr(seq_len_dev),
                                          float(sm_scale) if sm_scale else 0.0,
                                          (ROTATE_Q if rotate_q else 0) | _rec_flag(k_pool), int(num_splits),
                                          _stream(q3))
    _check(rc, "decode_partials_dev")
    return pm, pl, po
