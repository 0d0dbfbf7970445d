"""Multi-GPU decode layouts (custom_kv.sharding) on CPU: two gloo ranks,
each holding its shard of a seeded compressed cache, run ShardedDecode with
the oracle as the per-rank compute; the combined output must equal the
oracle's decode of the whole cache (kv-head and sequence-chunk sharding,
ragged chunk lengths).  The ranks are spawned processes; no GPU is used."""
import os
import socket

import numpy as np
import pytest
import torch

D = 128
TOL = 2e-3


class OracleOps:
    """The per-rank compute of ShardedDecode restated with the oracle (test
    infrastructure): same call signatures as custom_ecc_cuda, CPU tensors."""

    RECORD_FLOATS = 2 + D

    def __init__(self):
        import ecc_oracle
        self.o = ecc_oracle

    def decode_attention(self, q, k_pool, v_pool, seq_len, rotate_q=False, unrotate_out=False, out=None, **_):
        r = self.o.decode(q.numpy(), k_pool.numpy(), v_pool.numpy(), hkv=k_pool.shape[1], seq_len=seq_len,
                          rotate_q=rotate_q, unrotate_out=unrotate_out)
        res = torch.from_numpy(r.astype(np.float16)).reshape(q.shape)
        if out is None:
            return res
        out.copy_(res)
        return out

    def decode_partials(self, q, k_pool, v_pool, seq_len, num_splits, rotate_q=False, **_):
        B, hq = q.shape[0], q.shape[1]
        hkv = k_pool.shape[1]
        g = hq // hkv
        qf = q.float().numpy().reshape(B, hq, D)
        if rotate_q:
            qf = self.o.wht(qf).astype(np.float16).astype(np.float32)
        kr = self.o.reconstruct(k_pool[:, :, :seq_len].numpy()).reshape(B, hkv, seq_len, D).astype(np.float64)
        vr = self.o.reconstruct(v_pool[:, :, :seq_len].numpy()).reshape(B, hkv, seq_len, D).astype(np.float64)
        pm = np.full((B, hq, num_splits), -np.inf, np.float32)
        pl = np.zeros((B, hq, num_splits), np.float32)
        po = np.zeros((B, hq, num_splits, D), np.float32)
        cuts = np.linspace(0, seq_len, num_splits + 1).astype(int)
        for b in range(B):
            for h in range(hq):
                s = kr[b, h // g] @ qf[b, h].astype(np.float64) / np.sqrt(D)
                for i in range(num_splits):
                    lo, hi = cuts[i], cuts[i + 1]
                    if hi > lo:
                        m = s[lo:hi].max()
                        w = np.exp(s[lo:hi] - m)
                        pm[b, h, i], pl[b, h, i] = m, w.sum()
                        po[b, h, i] = w @ vr[b, h // g, lo:hi]
        return torch.from_numpy(pm), torch.from_numpy(pl), torch.from_numpy(po)

    @staticmethod
    def _merge(m, l, o):
        mx = m.max(-1, keepdims=True)
        w = np.where(np.isfinite(m), np.exp(m - np.where(np.isfinite(mx), mx, 0.0)), 0.0)
        return mx[..., 0], (w * l).sum(-1), (w[..., None] * o).sum(-2)

    def lse_merge_to_record(self, pm, pl, po, out=None):
        m, l, o = self._merge(pm.numpy().astype(np.float64), pl.numpy().astype(np.float64),
                              po.numpy().astype(np.float64))
        rec = np.concatenate([m[..., None], l[..., None], o], -1).astype(np.float32)
        out.copy_(torch.from_numpy(rec))
        return out

    def lse_merge_records(self, records, unrotate_out=False, out=None):
        r = np.moveaxis(records.numpy().astype(np.float64), 0, -2)  # [..., n, 130]
        m, l, o = self._merge(r[..., 0], r[..., 1], r[..., 2:])
        res = (o / l[..., None]).astype(np.float32)
        if unrotate_out:
            res = self.o.wht(res)
        res = torch.from_numpy(res.astype(np.float16))
        if out is None:
            return res.unsqueeze(-2) if res.dim() == 3 else res
        out.copy_(res.reshape(out.shape))
        return out


def _cache(B, hkv, hq, L, seed):
    import ecc_oracle
    import workloads
    k16, v16, q16 = workloads.make_c1(seed=seed, B=B, hkv=hkv, hq=hq, L=L)
    kb = ecc_oracle.compress(k16.reshape(-1, D).numpy(), rotate=True).reshape(B, hkv, L, D)
    vb = ecc_oracle.compress(v16.reshape(-1, D).numpy(), rotate=True).reshape(B, hkv, L, D)
    return torch.from_numpy(kb), torch.from_numpy(vb), q16


def _worker(rank, world, port, mode, B, hkv, hq, L, seed):
    import torch.distributed as dist
    from custom_kv.sharding import ShardedDecode, kv_head_range, q_head_range, seq_chunk_range
    import ecc_oracle
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        kb, vb, q = _cache(B, hkv, hq, L, seed)
        shard = ShardedDecode(mode, ops=OracleOps())
        out = torch.empty((B, hq, 1, D), dtype=torch.float16)
        if mode == "kv":
            k0, k1 = kv_head_range(rank, world, hkv)
            q0, q1 = q_head_range(rank, world, hkv, hq)
            shard.step(q[:, q0:q1].contiguous(), kb[:, k0:k1].contiguous(), vb[:, k0:k1].contiguous(), L, out=out)
        else:
            t0, t1 = seq_chunk_range(rank, world, L)
            kp = torch.zeros((B, hkv, t1 - t0 + 5, D), dtype=torch.uint8)
            vp = torch.zeros_like(kp)
            kp[:, :, :t1 - t0] = kb[:, :, t0:t1]
            vp[:, :, :t1 - t0] = vb[:, :, t0:t1]
            shard.step(q, kp, vp, t1 - t0, num_splits=3, out=out)
        ref = ecc_oracle.decode(q.numpy(), kb.numpy(), vb.numpy(), hkv=hkv, seq_len=L, rotate_q=True,
                                unrotate_out=True)
        ref16 = ref.astype(np.float16).astype(np.float32)
        ulp = np.spacing(np.abs(ref16).astype(np.float16)).astype(np.float32)
        err = np.abs(out.float().numpy().reshape(B, hq, D) - ref16)
        assert np.all(err <= TOL + ulp / 2), f"rank {rank} {mode}: max err {err.max()}"
        shard.close()  # collective release; without a peer-memory exchange a no-op
        shard.close()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode,L,B", [("kv", 300, 2), ("kv", 300, 1), ("seq", 300, 2), ("seq", 257, 2)])
def test_two_gloo_ranks_equal_whole_cache_decode(oracle, mode, L, B):
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(2, _free_port(), mode, B, 4, 16, L, 11), nprocs=2, start_method="spawn")


def test_shard_ranges():
    from custom_kv.sharding import kv_head_range, q_head_range, seq_chunk_range
    assert [kv_head_range(r, 4, 8) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert q_head_range(1, 2, 8, 32) == (16, 32)
    chunks = [seq_chunk_range(r, 3, 10) for r in range(3)]
    assert chunks == [(0, 4), (4, 7), (7, 10)]
    assert seq_chunk_range(0, 1, 0) == (0, 0)
    with pytest.raises(ValueError):
        kv_head_range(0, 3, 8)
    with pytest.raises(ValueError):
        seq_chunk_range(2, 2, 5)
