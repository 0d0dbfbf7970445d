"""CPU oracle for the ECC-INT4 KV-cache hot path -- TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this module.  It is used by ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``, always
as the reference results the CUDA path is compared with, never as the thing
measured or shipped.

Two independent restatements of the reference's CPU algorithm live here:

* ``ecc_oracle.c`` (loaded through ctypes): bit-exact compress
  (custom_kv/ops_cpu.py:198 ``compress_cpu`` + the csrc/ecc_ops.h:22-32 block
  write) and the decode oracle (custom_kv/fused_decode.py:200
  ``cpu_reference_decode`` with HF ``repeat_kv`` GQA).
* ``compress_np``: a vectorised numpy statement of the same compress
  arithmetic, used to cross-check the C code on large inputs.

Both are pinned to the reference by ``tests/test_oracle_golden.py`` against
fixtures that ``tests/golden/make_golden.py`` produced by running the
reference's own ``ops_cpu`` / ``cpu_reference_decode``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libecc_oracle.so")
_lib = None
_lock = threading.Lock()

D = 128
BLOCK_BYTES = 128

# custom_kv/ops_cpu.py:19-24 as fp32 bit patterns (same table as the C file).
LM_BITS = np.array(
    [0xC019A6B5, 0xBFEBF7CF, 0xBFB7F2E5, 0xBF8CB5DD, 0xBF4CB296, 0xBF05BC02, 0xBE8432CA, 0x00000000,
     0x3E8432CA, 0x3F05BC02, 0x3F4CB296, 0x3F8CB5DD, 0x3FB7F2E5, 0x3FEBF7CF, 0x4019A6B5, 0x404A233A],
    dtype=np.uint32)
LM_CENTROIDS = LM_BITS.view(np.float32)
SQRT128_F32 = np.float32(np.sqrt(128.0))


def build() -> str:
    """Compile ecc_oracle.c with the committed Makefile (idempotent)."""
    src = os.path.join(_HERE, "ecc_oracle.c")
    if (not os.path.exists(_LIB_PATH)) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_LIB_PATH)
            p = ctypes.c_void_p
            i64 = ctypes.c_int64
            L.orc_compress.argtypes = [p, i64, ctypes.c_int, p]
            L.orc_compress.restype = None
            L.orc_compress_detail.argtypes = [p, ctypes.c_int, p, p, p, p, p, p, p]
            L.orc_compress_detail.restype = None
            L.orc_count_ties.argtypes = [p, i64, ctypes.c_int, ctypes.c_float]
            L.orc_count_ties.restype = i64
            L.orc_decode.argtypes = [p, p, p, i64, i64, ctypes.c_int, ctypes.c_int, ctypes.c_int, i64,
                                     ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int, p]
            L.orc_decode.restype = None
            L.orc_lse_merge.argtypes = [p, p, p, i64, ctypes.c_int, p]
            L.orc_lse_merge.restype = None
            L.orc_wht128.argtypes = [p]
            L.orc_wht_any.argtypes = [p, ctypes.c_int]
            L.orc_reconstruct.argtypes = [p, p]
            L.orc_f2h.argtypes = [ctypes.c_float]
            L.orc_f2h.restype = ctypes.c_uint16
            L.orc_h2f.argtypes = [ctypes.c_uint16]
            L.orc_h2f.restype = ctypes.c_float
            _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _as_f16_bits(x) -> np.ndarray:
    x = np.ascontiguousarray(x)
    if x.dtype == np.float16:
        return x.view(np.uint16)
    if x.dtype == np.uint16:
        return x
    raise TypeError(f"expected float16 input, got {x.dtype}")


def _threads(n: int) -> int:
    if n and n > 0:
        return n
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


# --------------------------------------------------------------------------
# compress
# --------------------------------------------------------------------------
def compress(x16, rotate: bool = True, threads: int = 0) -> np.ndarray:
    """[N, 128] fp16 -> [N, 128] uint8 ECC_KV_Blocks (bit-exact oracle)."""
    bits = _as_f16_bits(x16).reshape(-1, D)
    n = bits.shape[0]
    out = np.zeros((n, BLOCK_BYTES), dtype=np.uint8)
    L = lib()
    nt = min(_threads(threads), max(1, n // 64))
    if nt <= 1:
        L.orc_compress(_ptr(bits), n, int(rotate), _ptr(out))
        return out
    bounds = np.linspace(0, n, nt + 1).astype(np.int64)

    def work(i):
        a, b = int(bounds[i]), int(bounds[i + 1])
        if b > a:
            L.orc_compress(ctypes.c_void_p(bits.ctypes.data + a * D * 2), b - a, int(rotate),
                           ctypes.c_void_p(out.ctypes.data + a * BLOCK_BYTES))

    with ThreadPoolExecutor(nt) as ex:  # ctypes drops the GIL during the call
        list(ex.map(work, range(nt)))
    return out


def compress_detail(x16_vec, rotate: bool = True) -> dict:
    """All intermediate results of one vector, named like compress_cpu's dict."""
    bits = _as_f16_bits(x16_vec).reshape(D)
    x_rot = np.zeros(D, np.float32)
    q = np.zeros(D, np.uint8)
    syn = np.zeros(D, np.uint8)
    zero = np.zeros(1, np.float32)
    scale = np.zeros(1, np.float32)
    alpha = np.zeros(1, np.float32)
    blk = np.zeros(BLOCK_BYTES, np.uint8)
    lib().orc_compress_detail(_ptr(bits), int(rotate), _ptr(x_rot), _ptr(q), _ptr(syn), _ptr(zero),
                              _ptr(scale), _ptr(alpha), _ptr(blk))
    return {"x_rot": x_rot, "q": q, "syndrome": syn.astype(bool), "zero": zero[0],
            "scale": scale[0], "alpha": alpha[0], "block": blk}


def count_ties(x16, rotate: bool = True, tol: float = 1e-6) -> int:
    """Elements whose normalised value is within `tol` of a decision boundary."""
    bits = _as_f16_bits(x16).reshape(-1, D)
    return int(lib().orc_count_ties(_ptr(bits), bits.shape[0], int(rotate), float(tol)))


def wht(x: np.ndarray) -> np.ndarray:
    """hadamard_rotate_cpu on the last dim (any power of two)."""
    x = np.array(x, dtype=np.float32, copy=True)
    d = x.shape[-1]
    flat = x.reshape(-1, d)
    L = lib()
    for r in range(flat.shape[0]):
        row = np.ascontiguousarray(flat[r])
        if d == D:
            L.orc_wht128(_ptr(row))
        else:
            L.orc_wht_any(_ptr(row), d)
        flat[r] = row
    return flat.reshape(x.shape)


# vectorised numpy statement of the same arithmetic (cross-check of the C)
def _tsum128_np(v: np.ndarray) -> np.ndarray:
    acc = np.zeros((v.shape[0], 4, 8), np.float32)
    for blk in range(4):
        for a in range(4):
            j0 = blk * 32 + a * 8
            acc[:, a, :] = acc[:, a, :] + v[:, j0:j0 + 8]
    t = ((acc[:, 0] + acc[:, 1]) + acc[:, 2]) + acc[:, 3]
    s = t[:, 0].copy()
    for i in range(1, 8):
        s = s + t[:, i]
    return s


def wht_np(x: np.ndarray) -> np.ndarray:
    x = np.array(x, dtype=np.float32, copy=True).reshape(-1, D)
    s = 1
    while s < D:
        v = x.reshape(x.shape[0], D // (2 * s), 2 * s)
        a = v[:, :, :s].copy()
        b = v[:, :, s:].copy()
        v[:, :, :s] = a + b
        v[:, :, s:] = a - b
        s *= 2
    return (x / SQRT128_F32).astype(np.float32)


def compress_np(x16, rotate: bool = True) -> dict:
    """Vectorised restatement; returns blocks plus the intermediate arrays."""
    x = _as_f16_bits(x16).reshape(-1, D).view(np.float16).astype(np.float32)
    xr = wht_np(x) if rotate else x
    zero = (_tsum128_np(xr) / np.float32(128)).astype(np.float32)
    dx = xr.astype(np.float64) - zero.astype(np.float64)[:, None]
    acc = np.zeros(xr.shape[0], np.float64)
    for j in range(D):  # element order, like the C / torch accumulation
        acc = acc + dx[:, j] * dx[:, j]
    std32 = np.sqrt(acc / 127.0).astype(np.float32)
    scale = (std32.astype(np.float64) + 1e-8).astype(np.float32)
    xn = ((xr - zero[:, None]) / scale[:, None]).astype(np.float32)
    dist = np.abs(xn[:, :, None] - LM_CENTROIDS[None, None, :]).astype(np.float32)
    q = dist.argmin(-1).astype(np.uint8)
    kt = ((LM_CENTROIDS[q] * scale[:, None]).astype(np.float32) + zero[:, None]).astype(np.float32)
    eps = (xr - kt).astype(np.float32)
    syn = eps >= 0
    alpha = (_tsum128_np(np.abs(eps)) / np.float32(128)).astype(np.float32)
    blocks = pack_blocks(q, syn, scale, zero, alpha)
    return {"x_rot": xr, "q": q, "syndrome": syn, "zero": zero, "scale": scale, "alpha": alpha,
            "blocks": blocks}


def compress_calibrated_np(x16, scale: float, zero: float, alpha: float, rotate: bool = True) -> np.ndarray:
    """Compress with fixed per-layer quantiser parameters (the values of a
    calibration config, custom_kv/calibration.py:232-237):
    ops_cpu.lloyd_max_quantize_cpu(x_rot, scale, zero) (ops_cpu.py:78-109)
    and compute_syndrome_cpu (ops_cpu.py:114-126), every block storing
    fp16(fp32(scale)), fp16(fp32(zero)), fp16(fp32(alpha)).  The Python
    scalars enter torch's float32 arithmetic rounded to fp32."""
    x = _as_f16_bits(x16).reshape(-1, D).view(np.float16).astype(np.float32)
    xr = wht_np(x) if rotate else x
    s32, z32 = np.float32(scale), np.float32(zero)
    with np.errstate(invalid="ignore", over="ignore"):
        xn = ((xr - z32).astype(np.float32) / s32).astype(np.float32)
        dist = np.abs((xn[:, :, None] - LM_CENTROIDS[None, None, :]).astype(np.float32))
        q = dist.argmin(-1).astype(np.uint8)
        kt = ((LM_CENTROIDS[q] * s32).astype(np.float32) + z32).astype(np.float32)
        syn = (xr - kt).astype(np.float32) >= 0
    n = x.shape[0]
    return pack_blocks(q, syn, np.full(n, s32), np.full(n, z32), np.full(n, np.float32(alpha)))


def pack_blocks(q, syn, scale, zero, alpha) -> np.ndarray:
    """csrc/ecc_ops.h:22-64 layout: codes @0 (byte i = q[2i] | q[2i+1] << 4),
    syndrome @64 (bit j in byte j/8, position j%8), fp16 scale/zero/alpha at
    80/82/84 (fp16 of the fp32 value), zero padding @86..127."""
    q = np.asarray(q, np.uint8).reshape(-1, D)
    syn = np.asarray(syn, bool).reshape(-1, D)
    n = q.shape[0]
    out = np.zeros((n, BLOCK_BYTES), np.uint8)
    out[:, :64] = q[:, 0::2] | (q[:, 1::2] << 4)
    out[:, 64:80] = np.packbits(syn.reshape(n, 16, 8), axis=-1, bitorder="little").reshape(n, 16)
    meta = np.stack([np.asarray(scale, np.float32).reshape(n), np.asarray(zero, np.float32).reshape(n),
                     np.asarray(alpha, np.float32).reshape(n)], axis=1).astype(np.float16)
    out[:, 80:86] = meta.view(np.uint8).reshape(n, 6)
    return out


def unpack_blocks(blocks: np.ndarray):
    """-> codes [N,128] u8, sign bits [N,128] bool, meta [N,3] fp16."""
    b = np.asarray(blocks, np.uint8).reshape(-1, BLOCK_BYTES)
    n = b.shape[0]
    q = np.empty((n, D), np.uint8)
    q[:, 0::2] = b[:, :64] & 0x0F
    q[:, 1::2] = b[:, :64] >> 4
    syn = np.unpackbits(b[:, 64:80], axis=-1, bitorder="little").astype(bool)
    meta = np.ascontiguousarray(b[:, 80:86]).view(np.float16).reshape(n, 3)
    return q, syn, meta


def blocks_to_soa(blocks: np.ndarray):
    """128-byte blocks [..., 128] -> the reference's SoA trio
    (int4 [..., 64] u8, syn [..., 16] u8, meta [..., 3] fp16), cache.py:79-84."""
    b = np.asarray(blocks, np.uint8)
    int4 = np.ascontiguousarray(b[..., :64])
    syn = np.ascontiguousarray(b[..., 64:80])
    meta = np.ascontiguousarray(b[..., 80:86]).view(np.float16)
    return int4, syn, meta


# --------------------------------------------------------------------------
# decode
# --------------------------------------------------------------------------
def decode(q16, k_blocks, v_blocks, hkv: int, seq_len: int, sm_scale: float = 0.0,
           rotate_q: bool = False, unrotate_out: bool = False, threads: int = 0) -> np.ndarray:
    """cpu_reference_decode with GQA.

    q16: [B, Hq, 128] (or [B, Hq, 1, 128]) fp16; k/v_blocks: [B, Hkv, Lcap, 128]
    uint8 pools (only the first seq_len tokens are read).  Returns [B, Hq, 128]
    fp32.  rotate_q: the query is rotated first (q_rot = fp16(WHT(q)));
    unrotate_out: the WHT is applied to the output (values stored rotated)."""
    qb = _as_f16_bits(q16)
    B, Hq = qb.shape[0], qb.shape[1]
    qb = np.ascontiguousarray(qb.reshape(B, Hq, D))
    kb = np.ascontiguousarray(k_blocks, dtype=np.uint8)
    vb = np.ascontiguousarray(v_blocks, dtype=np.uint8)
    assert kb.shape == vb.shape and kb.shape[0] == B and kb.shape[1] == hkv and kb.shape[-1] == 128
    Lcap = kb.shape[2]
    assert 0 <= seq_len <= Lcap and Hq % hkv == 0
    out = np.zeros((B, Hq, D), np.float32)
    flags = (1 if rotate_q else 0) | (2 if unrotate_out else 0)
    L = lib()
    nt = min(_threads(threads), Hq)
    bounds = np.linspace(0, Hq, nt + 1).astype(int)

    def work(i):
        a, b = int(bounds[i]), int(bounds[i + 1])
        if b > a:
            L.orc_decode(_ptr(qb), _ptr(kb), _ptr(vb), hkv * Lcap, Lcap, B, Hq, hkv, seq_len,
                         float(sm_scale), flags, a, b, _ptr(out))

    if nt <= 1:
        work(0)
    else:
        with ThreadPoolExecutor(nt) as ex:
            list(ex.map(work, range(nt)))
    return out


def reconstruct(blocks: np.ndarray) -> np.ndarray:
    """k_rec of every block, fp32, exactly as fused_decode.py:229-241."""
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, BLOCK_BYTES)
    out = np.zeros((b.shape[0], D), np.float32)
    L = lib()
    for i in range(b.shape[0]):
        L.orc_reconstruct(ctypes.c_void_p(b.ctypes.data + i * 128), ctypes.c_void_p(out.ctypes.data + i * D * 4))
    return out


def lse_merge(pm: np.ndarray, pl: np.ndarray, po: np.ndarray) -> np.ndarray:
    """Merge split partials: pm/pl [rows, n], po [rows, n, 128] (unnormalised)."""
    pm = np.ascontiguousarray(pm, np.float32)
    pl = np.ascontiguousarray(pl, np.float32)
    po = np.ascontiguousarray(po, np.float32)
    rows, n = pm.shape
    out = np.zeros((rows, D), np.float32)
    lib().orc_lse_merge(_ptr(pm), _ptr(pl), _ptr(po), rows, n, _ptr(out))
    return out
