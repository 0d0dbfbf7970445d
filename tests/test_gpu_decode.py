"""Fused decode attention on the GPU through the C ABI against the oracle and
the reference's golden outputs.

Tolerance: every fp16 output element is within 2e-3 of the oracle's value
(fp64-accumulated, fp32 result) beyond the rounding of that value to fp16,
i.e. |out - ref| <= 2e-3 + ulp_fp16(ref) / 2.  (Outputs reach |x| ~ 10 on the
heavy-outlier test, where one fp16 ulp is already 7.8e-3.)"""
import os

import numpy as np
import pytest
import torch

import workloads

pytestmark = pytest.mark.gpu
TOL = 2e-3


@pytest.fixture(scope="module")
def ops(cuda_device):
    import custom_ecc_cuda
    return custom_ecc_cuda


def _dev(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _q(a16_bits, dev):
    return torch.from_numpy(np.ascontiguousarray(a16_bits).view(np.int16)).view(torch.float16).to(dev)


def _ulp16(x: np.ndarray) -> np.ndarray:
    a = np.abs(x.astype(np.float16))
    return (np.nextafter(a, np.float16(np.inf)) - a).astype(np.float32)


def _err(got: torch.Tensor, ref: np.ndarray) -> float:
    """Largest excess of |out - ref| over the fp16 rounding allowance; the
    test bound is TOL on this quantity."""
    g = got.float().cpu().numpy().reshape(ref.shape)
    r = ref.astype(np.float32)
    return float((np.abs(g - r) - 0.5 * _ulp16(r)).max())


@pytest.mark.parametrize("ci", range(4))
@pytest.mark.parametrize("kern", ["tma", "register", "cuda_cores"])
def test_decode_matches_reference_golden(ops, oracle, decode_golden, cuda_device, ci, kern):
    B, hq, hkv, L = [int(v) for v in decode_golden[f"case{ci}_meta"]]
    kb = _dev(decode_golden[f"case{ci}_kblocks"], cuda_device)
    vb = _dev(decode_golden[f"case{ci}_vblocks"], cuda_device)
    q = _q(decode_golden[f"case{ci}_q16"], cuda_device)
    out = ops.decode_attention(q, kb, vb, seq_len=L, kernel=kern)
    ref = decode_golden[f"case{ci}_out16"].view(np.float16).astype(np.float32).reshape(B, hq, 128)
    g = out.float().cpu().numpy().reshape(ref.shape)
    # against the reference's own fp16 output: both sides are rounded to
    # fp16, so the sound bound is TOL plus one ulp (half an ulp each)
    assert float((np.abs(g - ref) - _ulp16(ref)).max()) <= TOL
    # against the oracle's fp32 value (pinned to the same fixture in
    # tests/test_oracle_golden.py): TOL plus half an ulp
    ref32 = oracle.decode(decode_golden[f"case{ci}_q16"], decode_golden[f"case{ci}_kblocks"],
                          decode_golden[f"case{ci}_vblocks"], hkv=hkv, seq_len=L)
    assert _err(out, ref32) <= TOL


def test_fused_ecc_decode_attention_soa_api(decode_golden, cuda_device):
    """The reference wrapper's signature with SoA tensors, both as standalone
    tensors (packed) and as zero-copy views of a pool."""
    from custom_kv.fused_decode import fused_ecc_decode_attention
    from custom_kv.cache import soa_views
    B, hq, hkv, L = [int(v) for v in decode_golden["case1_meta"]]
    kb = _dev(decode_golden["case1_kblocks"], cuda_device)
    vb = _dev(decode_golden["case1_vblocks"], cuda_device)
    q = _q(decode_golden["case1_q16"], cuda_device)
    ref = decode_golden["case1_out16"].view(np.float16).astype(np.float32).reshape(B, hq, 128)
    kv, vv = soa_views(kb), soa_views(vb)
    out_views = fused_ecc_decode_attention(q, *kv, *vv, L)
    standalone = [t.contiguous() for t in kv + vv]
    out_packed = fused_ecc_decode_attention(q, *standalone, L)
    assert _err(out_views, ref) <= TOL and _err(out_packed, ref) <= TOL
    assert out_views.shape == (B, hq, 1, 128) and out_views.dtype == torch.float16


@pytest.mark.parametrize("kern", ["tma", "register", "cuda_cores"])
def test_full_c1_decode_against_reference(ops, oracle, cuda_device, kern):
    """Single-layer op test: GPU compress then decode vs the reference's
    cpu_reference_decode output (GQA via repeat_kv)."""
    path = os.path.join(os.path.dirname(__file__), "golden", "c1_decode_out16.npy")
    if not os.path.exists(path):
        pytest.skip("c1 decode fixture not generated")
    k16, v16, q16 = workloads.make_c1(seed=0)
    kp = torch.empty((1, 8, 2048, 128), dtype=torch.uint8, device=cuda_device)
    vp = torch.empty_like(kp)
    ops.compress_into(k16.to(cuda_device), kp, pos=0, rotate=True)
    ops.compress_into(v16.to(cuda_device), vp, pos=0, rotate=True)
    out = ops.decode_attention(q16.to(cuda_device), kp, vp, seq_len=2048, kernel=kern)
    ref = np.load(path).view(np.float16).astype(np.float32).reshape(1, 32, 128)
    # the reference's output is already fp16: one fp16 ulp (half on each side) on top of TOL
    g = out.float().cpu().numpy().reshape(ref.shape)
    assert float((np.abs(g - ref) - _ulp16(ref)).max()) <= TOL
    # and TOL plus half an ulp against the oracle's fp32 output on the same blocks
    ref32 = oracle.decode(q16.numpy(), kp.cpu().numpy(), vp.cpu().numpy(), hkv=8, seq_len=2048)
    assert _err(out, ref32) <= TOL


def _random_pools(oracle, B, hkv, L, cap, seed):
    k16, v16, _ = workloads.make_c1(seed=seed, B=B, hkv=hkv, hq=hkv, L=L)
    kb = oracle.compress(k16.reshape(-1, 128).numpy()).reshape(B, hkv, L, 128)
    vb = oracle.compress(v16.reshape(-1, 128).numpy()).reshape(B, hkv, L, 128)
    kp = np.zeros((B, hkv, cap, 128), np.uint8)
    vp = np.zeros_like(kp)
    kp[:, :, :L], vp[:, :, :L] = kb, vb
    return kp, vp


@pytest.mark.parametrize("B,hq,hkv,L,splits", [
    (1, 8, 8, 1, 0), (1, 4, 1, 65, 0), (2, 8, 2, 127, 3), (3, 12, 4, 300, 0),   # group 3
    (1, 32, 8, 2048, 1), (1, 32, 8, 2048, 7), (2, 16, 2, 1000, 0),              # group 8
    (1, 48, 4, 640, 0),                                                          # group 12
])
@pytest.mark.parametrize("flags", [(False, False), (True, True)])
@pytest.mark.parametrize("kern", ["tma", "register", "cuda_cores"])
def test_decode_shapes_vs_oracle(ops, oracle, cuda_device, B, hq, hkv, L, splits, flags, kern):
    cap = L + 5
    kp, vp = _random_pools(oracle, B, hkv, L, cap, seed=L + hq)
    g = torch.Generator().manual_seed(L)
    q = torch.randn(B, hq, 1, 128, generator=g).half()
    out = ops.decode_attention(q.to(cuda_device), _dev(kp, cuda_device), _dev(vp, cuda_device), seq_len=L,
                               rotate_q=flags[0], unrotate_out=flags[1], num_splits=splits, kernel=kern)
    ref = oracle.decode(q.numpy(), kp, vp, hkv=hkv, seq_len=L, rotate_q=flags[0], unrotate_out=flags[1])
    assert _err(out, ref) <= TOL


def test_decode_custom_scale_and_prefix(ops, oracle, cuda_device):
    """sm_scale is honoured and only the first seq_len tokens are read."""
    kp, vp = _random_pools(oracle, 1, 2, 200, 256, seed=3)
    kp[:, :, 150:] = 0xFF  # garbage beyond seq_len
    vp[:, :, 150:] = 0xFF
    q = torch.randn(1, 4, 1, 128, generator=torch.Generator().manual_seed(9)).half()
    out = ops.decode_attention(q.to(cuda_device), _dev(kp, cuda_device), _dev(vp, cuda_device), seq_len=150,
                               sm_scale=0.05)
    ref = oracle.decode(q.numpy(), kp, vp, hkv=2, seq_len=150, sm_scale=0.05)
    assert _err(out, ref) <= TOL


@pytest.mark.parametrize("kern", ["tma", "register", "cuda_cores"])
@pytest.mark.parametrize("hq,hkv", [(4, 1), (8, 1)])
def test_sharp_softmax_heavy_values(ops, oracle, cuda_device, kern, hq, hkv):
    """A few tokens dominate (large sm_scale) and the values are heavy-tailed
    with both signs: the output is a near-cancelling mix of large values,
    where a single fp16 rounding of the softmax weights would exceed the
    tolerance."""
    L = 700
    k16 = workloads.make_heavy(seed=11, n=hkv * L)
    v16 = workloads.make_heavy(seed=12, n=hkv * L) * 4
    kp = oracle.compress(k16.numpy()).reshape(1, hkv, L, 128)
    vp = oracle.compress(v16.numpy()).reshape(1, hkv, L, 128)
    for seed in range(4):
        q = (torch.randn(1, hq, 1, 128, generator=torch.Generator().manual_seed(seed)) * 2).half()
        out = ops.decode_attention(q.to(cuda_device), _dev(kp, cuda_device), _dev(vp, cuda_device), seq_len=L,
                                   sm_scale=0.35, rotate_q=True, unrotate_out=True, kernel=kern)
        ref = oracle.decode(q.numpy(), kp, vp, hkv=hkv, seq_len=L, sm_scale=0.35, rotate_q=True, unrotate_out=True)
        assert _err(out, ref) <= TOL, seed


@pytest.mark.parametrize("kern", ["tma", "register", "cuda_cores"])
def test_partials_and_merge_equal_decode(ops, oracle, cuda_device, kern):
    """decode_partials + lse_merge (the cross-device combine) equals decode,
    including partials gathered from two token chunks (sequence sharding)."""
    kp, vp = _random_pools(oracle, 2, 2, 700, 700, seed=8)
    q = torch.randn(2, 8, 1, 128, generator=torch.Generator().manual_seed(2)).half().to(cuda_device)
    K, V = _dev(kp, cuda_device), _dev(vp, cuda_device)
    full = ops.decode_attention(q, K, V, seq_len=700, rotate_q=True, unrotate_out=True, kernel=kern)
    pm, pl, po = ops.decode_partials(q, K, V, seq_len=700, num_splits=5, rotate_q=True, kernel=kern)
    merged = ops.lse_merge(pm, pl, po, unrotate_out=True)

    def close(a, b):  # different split counts: allow 1e-3 beyond one fp16 ulp of the value
        r = b.float().cpu().numpy().reshape(-1)
        return float((np.abs(a.float().cpu().numpy().reshape(-1) - r) - _ulp16(r)).max()) <= 1e-3

    assert close(merged, full)
    # two "devices": tokens [0, 400) and [400, 700)
    a = ops.decode_partials(q, K[:, :, :400], V[:, :, :400], seq_len=400, num_splits=2, rotate_q=True,
                            kernel=kern)
    b = ops.decode_partials(q, K[:, :, 400:], V[:, :, 400:], seq_len=300, num_splits=3, rotate_q=True,
                            kernel=kern)
    cat = [torch.cat([x, y], dim=2).contiguous() for x, y in zip(a, b)]
    merged2 = ops.lse_merge(*cat, unrotate_out=True)
    assert close(merged2, full)
    # two-level combine: each "device" merges its splits into one record per
    # row, the records are stacked as an all-gather would, then merged
    recs = torch.stack([ops.lse_merge_to_record(*a), ops.lse_merge_to_record(*b)])
    assert recs.shape == (2, 2, 8, 130)
    merged3 = ops.lse_merge_records(recs, unrotate_out=True)
    assert close(merged3, full)
    # a device with an empty chunk contributes an empty record
    e = ops.decode_partials(q, K, V, seq_len=0, num_splits=2, rotate_q=True, kernel=kern)
    rec_e = ops.lse_merge_to_record(*e)
    assert (rec_e[..., 1] == 0).all()
    merged4 = ops.lse_merge_records(torch.stack([recs[0], rec_e, recs[1]]), unrotate_out=True)
    assert close(merged4, full)


def test_empty_context_and_empty_splits(ops, cuda_device):
    kp = torch.zeros((1, 1, 64, 128), dtype=torch.uint8, device=cuda_device)
    q = torch.randn(1, 2, 1, 128, device=cuda_device).half()
    out = ops.decode_attention(q, kp, kp, seq_len=0)
    assert torch.count_nonzero(out) == 0
    pm, pl, po = ops.decode_partials(q, kp, kp, seq_len=10, num_splits=4)
    assert (pl[..., 1:] == 0).all()  # 10 tokens fit in the first 64-token split


def test_decode_errors(ops, cuda_device):
    kp = torch.zeros((1, 3, 64, 128), dtype=torch.uint8, device=cuda_device)
    q = torch.randn(1, 4, 1, 128, device=cuda_device).half()
    with pytest.raises(RuntimeError, match="multiple"):
        ops.decode_attention(q, kp, kp, seq_len=8)
    with pytest.raises(RuntimeError, match="capacity"):
        ops.decode_attention(q[:, :3], kp, kp, seq_len=65)
    with pytest.raises(RuntimeError, match="float16"):
        ops.decode_attention(q.float()[:, :3], kp, kp, seq_len=8)


@pytest.mark.parametrize("kern", ["tma", "register", "cuda_cores"])
def test_long_context_vs_oracle(ops, oracle, cuda_device, kern):
    """64k tokens, one batch row, GQA group 4 (the decode benchmark's shape per row)."""
    L, hkv, hq = 65536, 2, 8
    kp, vp = _random_pools(oracle, 1, hkv, L, L, seed=64)
    q = torch.randn(1, hq, 1, 128, generator=torch.Generator().manual_seed(64)).half()
    out = ops.decode_attention(q.to(cuda_device), _dev(kp, cuda_device), _dev(vp, cuda_device), seq_len=L,
                               rotate_q=True, unrotate_out=True, kernel=kern)
    ref = oracle.decode(q.numpy(), kp, vp, hkv=hkv, seq_len=L, rotate_q=True, unrotate_out=True)
    assert _err(out, ref) <= TOL


def test_kernels_agree_at_benchmark_shape(ops, cuda_device):
    """B8 Hq32/Hkv8 at 65536 tokens: all three kernels, same pools, and no
    bounded wait ran out."""
    B, hkv, hq, L = 8, 8, 32, 65536
    g = torch.Generator(device=cuda_device).manual_seed(5)
    kp = torch.empty((B, hkv, L, 128), dtype=torch.uint8, device=cuda_device)
    vp = torch.empty_like(kp)
    for t0 in range(0, L, 16384):
        ops.compress_into(torch.randn(B, hkv, 16384, 128, generator=g, device=cuda_device).half(), kp, pos=t0)
        ops.compress_into(torch.randn(B, hkv, 16384, 128, generator=g, device=cuda_device).half(), vp, pos=t0)
    q = torch.randn(B, hq, 1, 128, generator=g, device=cuda_device).half()
    a = ops.decode_attention(q, kp, vp, seq_len=L - 3, rotate_q=True, unrotate_out=True, kernel="tma")
    b = ops.decode_attention(q, kp, vp, seq_len=L - 3, rotate_q=True, unrotate_out=True, kernel="cuda_cores")
    c = ops.decode_attention(q, kp, vp, seq_len=L - 3, rotate_q=True, unrotate_out=True, kernel="register")
    assert (a.float() - b.float()).abs().max().item() <= 1e-3
    assert (a.float() - c.float()).abs().max().item() <= 1e-3
    assert ops.device_status() == 0


def test_bounded_wait_gives_up_and_reports(ops, cuda_device):
    """A device wait that can never complete (an armed mbarrier without a
    copy) runs out after its limit, raises the device flag and returns: the
    context stays usable and the flag clears."""
    import ctypes
    lib = ctypes.CDLL(ops.library_path)
    lib.ecc_selftest_wait_timeout.argtypes = [ctypes.c_longlong, ctypes.POINTER(ctypes.c_int)]
    lib.ecc_selftest_wait_timeout.restype = ctypes.c_int
    assert ops.device_status(reset=True) == 0
    gave_up = ctypes.c_int(-1)
    assert lib.ecc_selftest_wait_timeout(2_000_000, ctypes.byref(gave_up)) == 0  # ~1 ms at 2 GHz
    assert gave_up.value == 1
    assert ops.device_status(reset=True) == 1
    assert ops.device_status() == 0
    # the device still computes
    x = torch.ones(4, 128, device=cuda_device, dtype=torch.float16)
    assert torch.isfinite(ops.hadamard_rotate(x)).all()
