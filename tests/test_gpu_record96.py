"""The 96-byte record option (a block without its zero pad sector, bytes
96..127) on the GPU: compress writes exactly the first 96 bytes of the
128-byte block through every compress entry point, and the decode over
96-byte pools gives bit-identical results to the decode over 128-byte pools
(the TMA-fed kernel reads bytes 0..95 of a block either way)."""
import numpy as np
import pytest
import torch

import workloads

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(cuda_device):
    import custom_ecc_cuda
    return custom_ecc_cuda


def _pools(B, H, cap, dev, fill=0):
    p128 = torch.full((B, H, cap, 128), fill, dtype=torch.uint8, device=dev)
    p96 = torch.full((B, H, cap, 96), fill, dtype=torch.uint8, device=dev)
    return p128, p96


@pytest.mark.parametrize("B,H,L,pos", [(2, 4, 37, 5), (8, 8, 1, 300), (1, 8, 4096, 0)])
@pytest.mark.parametrize("rotate", [True, False])
def test_compress_records_are_block_prefixes(ops, oracle, cuda_device, B, H, L, pos, rotate):
    """compress_into / compress_pair_into into 96-byte pools (small calls and
    tiled calls, strided input) write the first 96 bytes of the oracle's
    blocks, and nothing outside positions pos..pos+L-1."""
    g = torch.Generator().manual_seed(L + pos)
    k = (torch.randn(B, L, H, 128, generator=g) * 2).half()
    v = workloads.make_heavy(seed=L, n=B * H * L).reshape(B, H, L, 128)
    kd = k.to(cuda_device).transpose(1, 2)  # strided view [B, H, L, 128]
    vd = v.to(cuda_device)
    cap = pos + L + 3
    k128, k96 = _pools(B, H, cap, cuda_device, 0xAB)
    v128, v96 = _pools(B, H, cap, cuda_device, 0xAB)
    ops.compress_into(kd, k96, pos=pos, rotate=rotate)
    ops.compress_pair_into(kd, vd, k128, v128, pos=pos, rotate=rotate)
    k96b, v96b = _pools(B, H, cap, cuda_device, 0xAB)[1], _pools(B, H, cap, cuda_device, 0xAB)[1]
    ops.compress_pair_into(kd, vd, k96b, v96b, pos=pos, rotate=rotate)
    assert torch.equal(k96, k96b)
    assert torch.equal(k96, k128[..., :96]) and torch.equal(v96b, v128[..., :96])
    ref = oracle.compress(k.transpose(1, 2).contiguous().reshape(-1, 128).numpy(), rotate=rotate)
    got = k96[:, :, pos:pos + L].reshape(-1, 96).cpu().numpy()
    assert np.array_equal(got, ref[:, :96])
    outside = torch.cat([k96[:, :, :pos].flatten(), k96[:, :, pos + L:].flatten()])
    assert bool((outside == 0xAB).all())


def test_device_position_and_calibrated_records(ops, cuda_device):
    """compress_pair_at and the calibrated entry points into 96-byte pools
    equal the 128-byte pools' first 96 bytes."""
    B, H, cap = 2, 8, 40
    g = torch.Generator(device=cuda_device).manual_seed(3)
    k = torch.randn(B, H, 1, 128, device=cuda_device, generator=g).half()
    v = torch.randn(B, H, 1, 128, device=cuda_device, generator=g).half()
    pos = torch.tensor([17], dtype=torch.int32, device=cuda_device)
    k128, k96 = _pools(B, H, cap, cuda_device)
    v128, v96 = _pools(B, H, cap, cuda_device)
    ops.compress_pair_at(k, v, k128, v128, pos, rotate=True)
    ops.compress_pair_at(k, v, k96, v96, pos, rotate=True)
    assert torch.equal(k96, k128[..., :96]) and torch.equal(v96, v128[..., :96])
    c128, c96 = _pools(B, H, cap, cuda_device)
    x = torch.randn(B, H, 9, 128, device=cuda_device, generator=g).half()
    ops.compress_calibrated_into(x, c128, 0.9, 0.01, 0.2, pos=4, rotate=True)
    ops.compress_calibrated_into(x, c96, 0.9, 0.01, 0.2, pos=4, rotate=True)
    ops.compress_calibrated_at(k, c128, 0.9, 0.01, 0.2, pos, rotate=False)
    ops.compress_calibrated_at(k, c96, 0.9, 0.01, 0.2, pos, rotate=False)
    assert torch.equal(c96, c128[..., :96])
    with pytest.raises(RuntimeError):  # one call, one record size
        ops.compress_pair_into(k, v, k128, v96, pos=0)


@pytest.mark.parametrize("B,hq,hkv,L", [(1, 32, 8, 2048), (2, 8, 2, 777), (3, 12, 4, 300), (1, 8, 1, 65)])
@pytest.mark.parametrize("flags", [(False, False), (True, True)])
def test_decode_over_records_equals_blocks(ops, oracle, cuda_device, B, hq, hkv, L, flags):
    """decode_attention over 96-byte pools is bit-identical to the TMA
    kernel over the same blocks at 128 bytes, and within the tolerance of
    the oracle."""
    cap = L + 7
    k16, v16, _ = workloads.make_c1(seed=L, B=B, hkv=hkv, hq=hkv, L=L)
    kp = np.zeros((B, hkv, cap, 128), np.uint8)
    vp = np.zeros_like(kp)
    kp[:, :, :L] = oracle.compress(k16.reshape(-1, 128).numpy()).reshape(B, hkv, L, 128)
    vp[:, :, :L] = oracle.compress(v16.reshape(-1, 128).numpy()).reshape(B, hkv, L, 128)
    k128, v128 = torch.from_numpy(kp).to(cuda_device), torch.from_numpy(vp).to(cuda_device)
    k96, v96 = k128[..., :96].contiguous(), v128[..., :96].contiguous()
    q = torch.randn(B, hq, 1, 128, generator=torch.Generator().manual_seed(L)).half().to(cuda_device)
    kw = dict(seq_len=L, rotate_q=flags[0], unrotate_out=flags[1])
    a = ops.decode_attention(q, k128, v128, kernel="tma", **kw)
    b = ops.decode_attention(q, k96, v96, **kw)
    assert torch.equal(a, b)
    ref = oracle.decode(q.cpu().numpy(), kp, vp, hkv=hkv, seq_len=L, rotate_q=flags[0], unrotate_out=flags[1])
    r = ref.astype(np.float32)
    ulp = np.spacing(np.abs(r.astype(np.float16))).astype(np.float32)
    assert float((np.abs(b.float().cpu().numpy().reshape(r.shape) - r) - ulp / 2).max()) <= 2e-3
    # partials (sequence-sharding path) and the device-length decode
    ns = ops.default_splits(B, hkv, L)
    pa = ops.decode_partials(q, k128, v128, L, ns, rotate_q=flags[0], kernel="tma")
    pb = ops.decode_partials(q, k96, v96, L, ns, rotate_q=flags[0])
    assert all(torch.equal(x, y) for x, y in zip(pa, pb))
    n_dev = torch.tensor([L], dtype=torch.int32, device=cuda_device)
    da = ops.decode_attention_dev(q, k128, v128, n_dev, rotate_q=flags[0], unrotate_out=flags[1])
    db = ops.decode_attention_dev(q, k96, v96, n_dev, rotate_q=flags[0], unrotate_out=flags[1])
    assert torch.equal(da, db)


def test_record_decode_errors(ops, cuda_device):
    """Requests only the other kernels take are refused for 96-byte records."""
    k96 = torch.zeros((1, 1, 64, 96), dtype=torch.uint8, device=cuda_device)
    q = torch.zeros((1, 8, 1, 128), dtype=torch.float16, device=cuda_device)
    for kern in ("register", "cuda_cores"):
        with pytest.raises(RuntimeError):
            ops.decode_attention(q, k96, k96, seq_len=64, kernel=kern)
    q12 = torch.zeros((1, 12, 1, 128), dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError):  # GQA group 12
        ops.decode_attention(q12, k96, k96, seq_len=64)
    k96 = torch.zeros((1, 1, 4096, 96), dtype=torch.uint8, device=cuda_device)
    ns = ops.default_splits(1, 1, 4096)
    assert ns > 1
    with pytest.raises(RuntimeError):  # fewer splits than the TMA partition writes
        ops.decode_attention(q, k96, k96, seq_len=4096, num_splits=ns - 1)
    assert ops.decode_attention(q, k96, k96, seq_len=4096).shape == (1, 8, 1, 128)
    pm, pl, po = ops.decode_partials(q, k96, k96, 4096, ns + 3)  # extra partial slots come out empty
    assert bool((pl[..., ns:] == 0).all())


def test_cache_with_records_matches_blocks(cuda_device):
    """ErrorCorrectedCache(block_bytes=96): the same updates and decode steps
    as the 128-byte cache give bit-identical attention outputs, three quarters
    of the memory, and the same reconstructions."""
    from custom_kv import ErrorCorrectedCache

    class Cfg:
        num_hidden_layers = 2
        num_attention_heads = 8
        num_key_value_heads = 2
        hidden_size = 1024
        head_dim = 128

    caches = [ErrorCorrectedCache(Cfg(), batch_size=2, max_cache_len=300, device="cuda", block_bytes=bb)
              for bb in (128, 96)]
    g = torch.Generator(device="cuda").manual_seed(1)
    pre = [torch.randn(2, 2, 200, 128, device="cuda", generator=g).half() for _ in range(2)]
    for c in caches:
        for layer in range(2):
            c.update(pre[0], pre[1], layer_idx=layer)
    for step in range(3):
        k = torch.randn(2, 2, 1, 128, device="cuda", generator=g).half()
        v = torch.randn(2, 2, 1, 128, device="cuda", generator=g).half()
        q = torch.randn(2, 8, 1, 128, device="cuda", generator=g).half()
        outs = []
        for c in caches:
            c.update(k, v, layer_idx=0)
            outs.append(c.decode_attention(q, 0))
        assert torch.equal(outs[0], outs[1]), step
    m128, m96 = (c.memory_bytes()["cache_bytes"] for c in caches)
    assert m96 * 4 == m128 * 3
    a, b = (c.get_kv_fp16_for_layer(0) for c in caches)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    with pytest.raises(RuntimeError):
        ErrorCorrectedCache(Cfg(), max_cache_len=8, device="cuda", block_bytes=64)
