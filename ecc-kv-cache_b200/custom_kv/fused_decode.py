"""fused_decode.py -- ``fused_ecc_decode_attention``, the drop-in for the
reference's Triton wrapper (custom_kv/fused_decode.py:153), running the
sm_100a decode kernel of libeccb200.so.

The reference's CPU check ``cpu_reference_decode`` (:200) is test
infrastructure and lives with the oracle, outside this package: the product
has no CPU path.
"""
from __future__ import annotations

from typing import Optional

import torch

import custom_ecc_cuda as ops

from .cache import pool_of_views


def _as_pool(int4: torch.Tensor, syn: torch.Tensor, meta: torch.Tensor) -> torch.Tensor:
    pool = pool_of_views(int4, syn, meta)
    if pool is not None:
        return pool  # zero-copy: the trio are views of one block pool
    return ops.pack_soa(int4, syn, meta)


def fused_ecc_decode_attention(query_rot: torch.Tensor, k_int4: torch.Tensor, k_syn: torch.Tensor,
                               k_meta: torch.Tensor, v_int4: torch.Tensor, v_syn: torch.Tensor,
                               v_meta: torch.Tensor, seq_len: int, sm_scale: Optional[float] = None,
                               num_splits: int = 0) -> torch.Tensor:
    """Attention of the rotated query over ECC-compressed K/V.

    query_rot [B, Hq, 1, 128] fp16; k_int4/v_int4 [B, Hkv, L, 64] u8,
    k_syn/v_syn [B, Hkv, L, 16] u8, k_meta/v_meta [B, Hkv, L, 3] fp16
    (Hq a multiple of Hkv; Hkv == Hq is the reference's case).  Reads tokens
    [0, seq_len).  Returns [B, Hq, 1, 128] fp16 in the stored value basis:
    sum_t softmax(<q, k_rec_t> / sqrt(128)) v_rec_t with
    k_rec = C[q]*scale + zero + alpha*s.
    """
    B, H, _, D = query_rot.shape
    if D != 128:
        raise AssertionError(f"Only D=128 supported, got {D}")
    kp = _as_pool(k_int4, k_syn, k_meta)
    vp = _as_pool(v_int4, v_syn, v_meta)
    q16 = query_rot if query_rot.dtype == torch.float16 else query_rot.to(torch.float16)
    return ops.decode_attention(q16, kp, vp, seq_len=seq_len, sm_scale=sm_scale, num_splits=num_splits)
