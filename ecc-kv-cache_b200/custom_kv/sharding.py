"""Multi-GPU decode over a layer's compressed cache: one process per GPU
(torch.distributed, NCCL over NVLink), two layouts of the cache.

* **kv-head sharding** (``mode="kv"``): rank r holds kv heads
  [r*Hkv/N, (r+1)*Hkv/N) of every sequence and serves their query heads.
  Attention needs no exchange; one all-gather of the ranks' fp16 outputs
  assembles the layer's attention output [B, Hq, 1, 128].  With
  ``exchange="p2p"`` the merge of the split partials and that all-gather are
  one kernel per rank that stores its output rows straight into every rank's
  buffer over NVLink.
* **sequence-chunk sharding** (``mode="seq"``): rank r holds tokens
  [r*L/N, (r+1)*L/N) of every (sequence, kv head) row; new tokens are
  appended on the last rank.  Each rank computes split partials (m, l, o) of
  its chunk, merges them into one 130-float record {m, l, o[128]} per
  (sequence, query head), the records are all-gathered and merged (the
  log-sum-exp combine of flash-decoding).  With ``exchange="p2p"`` the
  record merge, the exchange and the final merge are one kernel per rank
  that stores its records straight into every rank's buffer over NVLink
  (``PeerExchange``) instead of an NCCL all-gather between two kernels.

The reference keeps everything on one device (custom_kv/cache.py:79-84); this
module is the multi-GPU layer around the same fused decode.  Every rank takes
the same collective steps in the same order.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist

D = 128


def kv_head_range(rank: int, world: int, hkv: int) -> Tuple[int, int]:
    """kv heads [lo, hi) of `rank` under kv-head sharding (world must divide hkv)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank out of range")
    if hkv % world:
        raise ValueError(f"{world} ranks do not divide {hkv} kv heads")
    per = hkv // world
    return rank * per, (rank + 1) * per


def q_head_range(rank: int, world: int, hkv: int, hq: int) -> Tuple[int, int]:
    """Query heads [lo, hi) served by `rank` under kv-head sharding (the GQA
    groups of its kv heads, HF repeat_kv order: kv head = q head // (hq/hkv))."""
    if hq % hkv:
        raise ValueError("query heads must be a multiple of kv heads")
    lo, hi = kv_head_range(rank, world, hkv)
    g = hq // hkv
    return lo * g, hi * g


def seq_chunk_range(rank: int, world: int, seq_len: int) -> Tuple[int, int]:
    """Tokens [start, stop) of `rank` under sequence-chunk sharding of a
    context of seq_len tokens: contiguous chunks, the first seq_len % world
    ranks one token longer."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank out of range")
    if seq_len < 0:
        raise ValueError("seq_len must be >= 0")
    base, extra = divmod(seq_len, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _all_gather(out: torch.Tensor, inp: torch.Tensor, group) -> None:
    """out[r] = rank r's inp (out [world, *inp.shape])."""
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, inp, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), inp, group=group)


class PeerExchange:
    """Peer-memory exchange buffers for the records of ``rows`` rows (B * Hq)
    on every rank of ``group`` (one GPU per rank, one node): each rank
    allocates a zero-filled buffer, passes its CUDA IPC handle to the others
    and maps theirs on its own device, so that
    custom_ecc_cuda.lse_exchange_merge can store into all of them.  Made
    collectively (every rank at the same point); calls of ``merge`` must then
    be made in step on every rank, and ``close`` collectively at the end.
    The call epochs live in device memory (``state``, advanced by each
    call's kernel), so calls can be recorded in a CUDA graph and replayed.

    A merge whose bounded wait for another rank ran out raises the device
    status flag (4) and leaves its rows unwritten instead of hanging; the flag
    is read (one synchronisation) every ``check_every`` merges when that is
    > 0, and always at ``close``, and turns into a ``RuntimeError``."""

    def __init__(self, rows: int, group, device: torch.device, ops=None, check_every: int = 0):
        if ops is None:
            import custom_ecc_cuda as ops  # noqa: F811
        self.ops = ops
        self.rows = int(rows)
        self.group = group
        self.device = device
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.own, handle = ops.exchange_alloc(self.rows, self.world, device)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs = [self.own if q == self.rank else ops.exchange_open(h, device) for q, h in enumerate(handles)]
        self.state = torch.zeros(2, dtype=torch.int64, device=device)  # epoch counter, CTAs done
        self.calls = 0
        self.check_every = int(check_every)
        dist.barrier(group=group)  # every buffer zeroed and mapped before the first call

    def merge(self, pm: torch.Tensor, pl: torch.Tensor, po: torch.Tensor, unrotate_out: bool = True,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if not self.ptrs:
            raise RuntimeError("the exchange is closed")
        if pm.dim() != 3 or pm.shape[0] * pm.shape[1] != self.rows:
            raise RuntimeError(f"the exchange was made for {self.rows} rows, got partials of shape {tuple(pm.shape)}")
        res = self.ops.lse_exchange_merge(pm, pl, po, self.ptrs, self.rank, self.state, unrotate_out=unrotate_out,
                                          out=out)
        self._count()
        return res

    def _count(self) -> None:
        self.calls += 1
        if (self.check_every > 0 and self.calls % self.check_every == 0
                and not torch.cuda.is_current_stream_capturing()):
            self._raise_on_status(self.ops.device_status())

    def gather(self, pm: torch.Tensor, pl: torch.Tensor, po: torch.Tensor, unrotate_out: bool = True,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Kv-head sharding: merge this rank's partials of its query heads and
        all-gather the fp16 outputs in one kernel (lse_gather_merge); ``out``
        [B, W*hq_local, 1, 128].  Shares the epoch state of ``merge``."""
        if not self.ptrs:
            raise RuntimeError("the exchange is closed")
        if pm.dim() != 3 or pm.shape[0] * pm.shape[1] != self.rows:
            raise RuntimeError(f"the exchange was made for {self.rows} rows, got partials of shape {tuple(pm.shape)}")
        res = self.ops.lse_gather_merge(pm, pl, po, self.ptrs, self.rank, self.state, unrotate_out=unrotate_out,
                                        out=out)
        self._count()
        return res

    def _raise_on_status(self, status: int) -> None:
        if status != 0:
            raise RuntimeError(f"rank {self.rank}: the peer exchange reported device status {status} (a wait for "
                               f"another rank's records ran out; those outputs are not valid)")

    def close(self) -> None:
        """Unmap the other ranks' buffers and free this rank's (collective;
        every rank's last merge must have finished)."""
        if not self.ptrs:
            return
        torch.cuda.synchronize(self.device)
        status = self.ops.device_status()
        dist.barrier(group=self.group)
        for q, p in enumerate(self.ptrs):
            if q != self.rank:
                self.ops.exchange_close(p, self.device)
        dist.barrier(group=self.group)  # nobody maps this rank's buffer any more
        self.ops.exchange_free(self.own, self.device)
        self.ptrs = []
        self._raise_on_status(status)


class ShardedDecode:
    """One decode step of a sharded layer on this rank.

    ``ops`` provides the per-rank compute (default: the CUDA ops of
    custom_ecc_cuda: decode_attention, decode_partials, lse_merge_to_record,
    lse_merge_records, RECORD_FLOATS).  Buffers for the exchange are made on
    first use and reused, so a steady decode loop allocates nothing.
    ``exchange``: "nccl" (seq mode: all-gather of the records between two
    merge kernels; kv mode: all-gather of the fp16 outputs) or "p2p" (one
    kernel over peer memory, PeerExchange: seq mode merges and exchanges the
    records, kv mode merges and gathers the outputs; GPUs of one node; the
    epochs live in device memory, so a step can be recorded in a CUDA graph).
    """

    def __init__(self, mode: str, group=None, ops=None, exchange: str = "nccl"):
        if mode not in ("kv", "seq"):
            raise ValueError("mode must be 'kv' or 'seq'")
        if exchange not in ("nccl", "p2p"):
            raise ValueError("exchange must be 'nccl' or 'p2p'")
        self.exchange = exchange
        self._peer: Optional[PeerExchange] = None
        if ops is None:
            import custom_ecc_cuda as ops  # noqa: F811
        self.mode = mode
        self.ops = ops
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self._bufs: dict = {}

    def close(self) -> None:
        """Release the peer-memory exchange (its buffers and the peers'
        mappings) and check the device status it reports.  Collective: every
        rank calls it, before destroy_process_group.  A no-op without a peer
        exchange; the next p2p step makes a new one."""
        if self._peer is not None:
            peer, self._peer = self._peer, None
            peer.close()

    def _ensure_peer(self, rows: int, device: torch.device) -> None:
        if self._peer is None or self._peer.rows != rows:
            if self._peer is not None:
                # every rank switches at the same step: release the old
                # buffers collectively before making the new ones
                self._peer.close()
            self._peer = PeerExchange(rows, self.group, device, ops=self.ops)

    def _buf(self, key, shape, dtype, device):
        b = self._bufs.get(key)
        if b is None or b.shape != shape or b.dtype != dtype or b.device != device:
            b = torch.empty(shape, dtype=dtype, device=device)
            self._bufs[key] = b
        return b

    def step(self, query: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, local_len: int,
             num_splits: int = 0, rotate_q: bool = True, unrotate_out: bool = True,
             out: Optional[torch.Tensor] = None, mark: Optional[torch.cuda.Event] = None,
             seq_len_dev: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Attention output of this step for every query head, [B, Hq, 1, 128] fp16.

        kv mode: ``query`` holds this rank's query heads [B, Hq/N, 1, 128] and
        the pools its kv heads; seq mode: ``query`` holds every head and the
        pools this rank's token chunk, of which the first ``local_len`` tokens
        are valid.  ``num_splits`` (seq mode) is the split count of the local
        partials; give one that covers every local length of the run so that
        the exchange shapes stay fixed.  ``mark``, if given, is recorded on
        the current stream after this rank's own attention work and before the
        exchange (to time the two apart).  ``seq_len_dev`` (an int32 CUDA
        tensor): the local length is read from it when the kernels run instead
        of ``local_len``, so the step can be recorded once in a CUDA graph and
        replayed while the cache grows (seq mode then needs num_splits >=
        custom_ecc_cuda.decode_dev_splits(B, Hkv, pool capacity))."""
        ops, W = self.ops, self.world
        B, hq_l = query.shape[0], query.shape[1]
        if self.mode == "kv" and self.exchange == "p2p":
            # partials of this rank's heads, then one kernel: merge + output
            # all-gather over peer memory
            hkv_l, cap = k_pool.shape[-3], k_pool.shape[-2]
            if seq_len_dev is not None:
                splits = max(num_splits, ops.decode_dev_splits(B, hkv_l, cap))
                parts = (self._buf("pm", (B, hq_l, splits), torch.float32, query.device),
                         self._buf("pl", (B, hq_l, splits), torch.float32, query.device),
                         self._buf("po", (B, hq_l, splits, D), torch.float32, query.device))
                pm, pl, po = ops.decode_partials_dev(query, k_pool, v_pool, seq_len_dev, splits, rotate_q=rotate_q,
                                                     out=parts)
            else:
                splits = ops.default_splits(B, hkv_l, local_len)
                pm, pl, po = ops.decode_partials(query, k_pool, v_pool, seq_len=local_len, num_splits=splits,
                                                 rotate_q=rotate_q)
            if mark is not None:
                mark.record()
            if out is None:
                out = torch.empty((B, W * hq_l, 1, D), dtype=torch.float16, device=query.device)
            self._ensure_peer(B * hq_l, query.device)
            return self._peer.gather(pm, pl, po, unrotate_out=unrotate_out, out=out)
        if self.mode == "kv":
            loc = self._buf("loc", (B, hq_l, 1, D), torch.float16, query.device)
            if seq_len_dev is not None:
                ws = self._buf("ws", (ops.decode_dev_workspace_size(B, hq_l, k_pool.shape[-3], k_pool.shape[-2]),),
                               torch.uint8, query.device)
                ops.decode_attention_dev(query, k_pool, v_pool, seq_len_dev, rotate_q=rotate_q,
                                         unrotate_out=unrotate_out, out=loc, workspace=ws)
            else:
                ops.decode_attention(query, k_pool, v_pool, seq_len=local_len, rotate_q=rotate_q,
                                     unrotate_out=unrotate_out, out=loc)
            if mark is not None:
                mark.record()
            if out is None:
                out = torch.empty((B, W * hq_l, 1, D), dtype=torch.float16, device=query.device)
            if W == 1:
                out.copy_(loc)
            elif B == 1 and out.is_contiguous():
                # rank r's heads are one contiguous chunk of the output: gather in place
                _all_gather(out.view(W, 1, hq_l, 1, D), loc, self.group)
            else:
                g = self._buf("gather", (W, B, hq_l, 1, D), torch.float16, query.device)
                _all_gather(g, loc, self.group)
                out.view(B, W, hq_l, 1, D).copy_(g.permute(1, 0, 2, 3, 4))  # one copy into place
            return out
        # sequence chunks
        if num_splits <= 0:
            raise ValueError("seq mode needs a fixed num_splits")
        if seq_len_dev is not None:
            parts = (self._buf("pm", (B, hq_l, num_splits), torch.float32, query.device),
                     self._buf("pl", (B, hq_l, num_splits), torch.float32, query.device),
                     self._buf("po", (B, hq_l, num_splits, D), torch.float32, query.device))
            pm, pl, po = ops.decode_partials_dev(query, k_pool, v_pool, seq_len_dev, num_splits, rotate_q=rotate_q,
                                                 out=parts)
        else:
            pm, pl, po = ops.decode_partials(query, k_pool, v_pool, seq_len=local_len, num_splits=num_splits,
                                             rotate_q=rotate_q)
        if out is None:
            out = torch.empty((B, hq_l, 1, D), dtype=torch.float16, device=query.device)
        if self.exchange == "p2p":
            if mark is not None:
                mark.record()
            self._ensure_peer(B * hq_l, query.device)
            return self._peer.merge(pm, pl, po, unrotate_out=unrotate_out, out=out)
        rec = self._buf("rec", (B, hq_l, ops.RECORD_FLOATS), torch.float32, query.device)
        ops.lse_merge_to_record(pm, pl, po, out=rec)
        if mark is not None:
            mark.record()
        grec = self._buf("grec", (W, B, hq_l, ops.RECORD_FLOATS), torch.float32, query.device)
        if W == 1:
            grec[0].copy_(rec)
        else:
            _all_gather(grec, rec, self.group)
        return ops.lse_merge_records(grec, unrotate_out=unrotate_out, out=out)
