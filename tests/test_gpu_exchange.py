"""The record exchange over peer memory (custom_ecc_cuda.lse_exchange_merge)
on the GPU.  One GPU: with one rank the kernel's merge equals
lse_merge_to_record + lse_merge_records bit for bit over successive epochs
(both buffer halves), and a wait for a rank that never stores gives up,
raises the device flag and leaves the GPU usable.  Two GPUs (skipped with
fewer): sequence-sharded and kv-head-sharded decode steps with the p2p
exchange equal those with the NCCL all-gather bit for bit."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu
D = 128


@pytest.fixture(scope="module")
def ops(cuda_device):
    import custom_ecc_cuda
    return custom_ecc_cuda


class _Buffers:
    """Exchange buffers made by the library (ecc_exchange_alloc), as the
    exchange requires; freed on exit."""

    def __init__(self, ops, dev, rows, world, count):
        self.ops, self.dev = ops, dev
        self.ptrs = [ops.exchange_alloc(rows, world, dev)[0] for _ in range(count)]

    def __enter__(self):
        return self.ptrs

    def __exit__(self, *exc):
        torch.cuda.synchronize(self.dev)
        for p in self.ptrs:
            self.ops.exchange_free(p, self.dev)


def _partials(B, hq, n, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    pm = torch.randn(B, hq, n, device=dev, generator=g) * 3
    pl = torch.rand(B, hq, n, device=dev, generator=g) * 5
    pl[:, :, -1] = 0.0  # an empty split
    pm[:, :, -1] = -float("inf")
    po = torch.randn(B, hq, n, D, device=dev, generator=g)
    return pm, pl, po


@pytest.mark.parametrize("B,hq,n", [(8, 32, 29), (1, 4, 1), (3, 40, 70)])
def test_single_rank_exchange_equals_two_level_merge(ops, cuda_device, B, hq, n):
    rows = B * hq
    with _Buffers(ops, cuda_device, rows, 1, 1) as bufs:
        for epoch in range(1, 5):
            pm, pl, po = _partials(B, hq, n, epoch, cuda_device)
            unrot = bool(epoch & 1)
            ref = ops.lse_merge_records(ops.lse_merge_to_record(pm, pl, po).unsqueeze(0), unrotate_out=unrot)
            got = ops.lse_exchange_merge(pm, pl, po, bufs, 0, epoch, unrotate_out=unrot)
            assert torch.equal(got.reshape(ref.shape), ref), epoch
    assert ops.device_status() == 0


def test_exchange_argument_errors(ops, cuda_device):
    pm, pl, po = _partials(1, 4, 3, 0, cuda_device)
    with _Buffers(ops, cuda_device, 4, 1, 1) as bufs:
        with pytest.raises(RuntimeError):  # epochs start at 1
            ops.lse_exchange_merge(pm, pl, po, bufs, 0, 0)
        with pytest.raises(RuntimeError):  # rank outside the peer list
            ops.lse_exchange_merge(pm, pl, po, bufs, 1, 1)
        with pytest.raises(RuntimeError):  # more ranks than one node's limit
            ops.lse_exchange_merge(pm, pl, po, bufs * 9, 0, 1)
        # a buffer the library did not make or map: refused, nothing is stored
        plain = torch.zeros(ops.exchange_buffer_bytes(4, 1), dtype=torch.uint8, device=cuda_device)
        with pytest.raises(RuntimeError):
            ops.lse_exchange_merge(pm, pl, po, [plain.data_ptr()], 0, 1)
        # more rows than the buffer was made for: refused
        pm8, pl8, po8 = _partials(2, 4, 3, 0, cuda_device)
        with pytest.raises(RuntimeError):
            ops.lse_exchange_merge(pm8, pl8, po8, bufs, 0, 1)
    with _Buffers(ops, cuda_device, 4, 2, 1) as bufs:
        # a buffer made for 2 ranks x 4 rows serves 1 rank x 8 rows (same bytes)
        pm8, pl8, po8 = _partials(2, 4, 3, 0, cuda_device)
        ops.lse_exchange_merge(pm8, pl8, po8, bufs, 0, 1)
    assert ops.exchange_buffer_bytes(4, 9) == 0


def test_wait_for_missing_rank_gives_up(ops, cuda_device):
    """A second 'rank' whose buffer is local memory that no kernel ever flags:
    the wait runs out after ~1e6 cycles, the kernel returns, the device flag
    reads 4 and clears, and the next call on the device works."""
    pm, pl, po = _partials(2, 8, 5, 1, cuda_device)
    rows = 16
    ops.device_status(reset=True)
    with _Buffers(ops, cuda_device, rows, 2, 2) as bufs:
        ops.lse_exchange_merge(pm, pl, po, bufs, 0, 1, wait_cycles=1_000_000)
        torch.cuda.synchronize()
    assert ops.device_status(reset=True) == 4
    assert ops.device_status() == 0
    with _Buffers(ops, cuda_device, rows, 1, 1) as bufs:
        ref = ops.lse_merge_records(ops.lse_merge_to_record(pm, pl, po).unsqueeze(0))
        got = ops.lse_exchange_merge(pm, pl, po, bufs, 0, 1)
        assert torch.equal(got.reshape(ref.shape), ref)


@pytest.mark.parametrize("B,hq_l,n", [(8, 4, 29), (2, 16, 5)])
def test_single_rank_gather_equals_merge(ops, cuda_device, B, hq_l, n):
    """With one rank the fused merge + output gather is lse_merge, bit for bit."""
    rows = B * hq_l
    with _Buffers(ops, cuda_device, rows, 1, 1) as bufs:
        for epoch in range(1, 4):
            pm, pl, po = _partials(B, hq_l, n, epoch, cuda_device)
            unrot = bool(epoch & 1)
            ref = ops.lse_merge(pm, pl, po, unrotate_out=unrot)
            got = ops.lse_gather_merge(pm, pl, po, bufs, 0, epoch, unrotate_out=unrot)
            assert torch.equal(got.reshape(ref.shape), ref), epoch
    assert ops.device_status() == 0


def test_device_epoch_state_and_graph_replay(ops, cuda_device):
    """Epochs from a device-side state: each call (eager or replayed from a
    CUDA graph) takes the next epoch and advances the state itself; results
    equal the host-epoch merges."""
    B, hq, n = 2, 8, 7
    rows = B * hq
    state = torch.zeros(2, dtype=torch.int64, device=cuda_device)
    with _Buffers(ops, cuda_device, rows, 1, 2) as (gbuf, xbuf):
        pm, pl, po = _partials(B, hq, n, 3, cuda_device)
        ref_g = ops.lse_merge(pm, pl, po, unrotate_out=True)
        ref_x = ops.lse_merge_records(ops.lse_merge_to_record(pm, pl, po).unsqueeze(0), unrotate_out=True)
        for _ in range(3):
            got = ops.lse_gather_merge(pm, pl, po, [gbuf], 0, state, unrotate_out=True)
            assert torch.equal(got.reshape(ref_g.shape), ref_g)
        assert state.tolist() == [3, 0]  # counter advanced once per call, done counter reset
        xstate = torch.zeros(2, dtype=torch.int64, device=cuda_device)
        out_g = torch.empty((B, hq, 1, D), dtype=torch.float16, device=cuda_device)
        out_x = torch.empty((B, hq, D), dtype=torch.float16, device=cuda_device)
        side = torch.cuda.Stream(cuda_device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # warm-up off the capture
            ops.lse_gather_merge(pm, pl, po, [gbuf], 0, state, unrotate_out=True, out=out_g)
            ops.lse_exchange_merge(pm, pl, po, [xbuf], 0, xstate, unrotate_out=True, out=out_x)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            ops.lse_gather_merge(pm, pl, po, [gbuf], 0, state, unrotate_out=True, out=out_g)
            ops.lse_exchange_merge(pm, pl, po, [xbuf], 0, xstate, unrotate_out=True, out=out_x)
        for _ in range(5):
            out_g.zero_()
            out_x.zero_()
            graph.replay()
            assert torch.equal(out_g.reshape(ref_g.shape), ref_g)
            assert torch.equal(out_x.reshape(ref_x.shape), ref_x)
        torch.cuda.synchronize()
        assert state.tolist()[0] == 4 + 5 and xstate.tolist()[0] == 1 + 5
        del graph
    assert ops.device_status() == 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_worker(rank, world, port):
    import datetime
    import torch.distributed as dist
    import custom_ecc_cuda as ops
    from custom_kv.sharding import ShardedDecode
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        B, hkv, hq, cap = 2, 4, 16, 3000
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        kp = torch.zeros((B, hkv, cap, 128), dtype=torch.uint8, device=dev)
        vp = torch.zeros_like(kp)
        n0 = 2500 + 137 * rank
        ops.compress_into(torch.randn(B, hkv, n0, D, device=dev, generator=g).half(), kp, pos=0)
        ops.compress_into(torch.randn(B, hkv, n0, D, device=dev, generator=g).half(), vp, pos=0)
        ref, p2p = ShardedDecode("seq"), ShardedDecode("seq", exchange="p2p")
        ns = ops.default_splits(B, hkv, cap) + 1
        for step in range(6):
            q = torch.randn(B, hq, 1, D, generator=torch.Generator().manual_seed(step)).half().to(dev)
            a = ref.step(q, kp, vp, n0 + step, num_splits=ns)
            b = p2p.step(q, kp, vp, n0 + step, num_splits=ns)
            assert torch.equal(a, b), (rank, step)
            if rank == world - 1:  # the last rank's chunk grows
                ops.compress_into(torch.randn(B, hkv, 1, D, device=dev, generator=g).half(), kp, pos=n0 + step)
        # kv-head sharding: each rank serves its hq/world query heads over its
        # own pools; the fused merge + output gather equals lse_merge + the
        # NCCL all-gather bit for bit, and every rank ends with the whole output
        kref, kp2p = ShardedDecode("kv"), ShardedDecode("kv", exchange="p2p")
        hq_l = hq // world
        for step in range(4):
            q = torch.randn(B, hq, 1, D, generator=torch.Generator().manual_seed(50 + step)).half()
            q_l = q[:, rank * hq_l:(rank + 1) * hq_l].contiguous().to(dev)
            a = kref.step(q_l, kp, vp, n0 + step)
            b = kp2p.step(q_l, kp, vp, n0 + step)
            assert a.shape == (B, hq, 1, D) and torch.equal(a, b), (rank, step)
            own = ops.decode_attention(q_l, kp, vp, seq_len=n0 + step, rotate_q=True, unrotate_out=True)
            assert torch.equal(b[:, rank * hq_l:(rank + 1) * hq_l], own)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        p2p.close()
        kp2p.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpus_p2p_exchange_equals_nccl():
    import torch.multiprocessing as mp
    mp.start_processes(_two_gpu_worker, args=(2, _free_port()), nprocs=2, start_method="spawn")
