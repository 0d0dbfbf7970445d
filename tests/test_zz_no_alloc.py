"""ecc_decode_static -- decode attention that allocates nothing.

Some callers cannot allocate device memory themselves: a host whose device
memory is owned by another allocator that has already reserved the budget, or
a latency-critical path that cannot take cudaMalloc's implicit
synchronisation.  For them libeccb200.so keeps the decode's split partials in
a fixed library-owned device array.  This test calls that entry point
directly through the C ABI (ctypes) and checks it against the workspace-based
ecc_decode and the oracle on two calls in a row, with different inputs, so
that the second call cannot pass on what the first left in the shared array.

It lives in a file of its own that pytest collects last, so a run that stops
at the first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import workloads

pytestmark = pytest.mark.gpu
TOL = 2e-3


@pytest.fixture(scope="module")
def lib(cuda_device):
    import custom_ecc_cuda
    L = ctypes.CDLL(custom_ecc_cuda.library_path)
    p, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    L.ecc_decode_static.argtypes = [p, p, p, i64, i64, p, i32, i32, i32, i64, f32, i32, i32, p]
    L.ecc_decode_static.restype = i32
    return L


def _pools(dev, B, hkv, L, seed):
    import custom_ecc_cuda as ops
    k16, v16, _ = workloads.make_c1(seed=seed, B=B, hkv=hkv, hq=hkv, L=L)
    kp = torch.empty((B, hkv, L, 128), dtype=torch.uint8, device=dev)
    vp = torch.empty_like(kp)
    ops.compress_into(k16.to(dev), kp, rotate=True)
    ops.compress_into(v16.to(dev), vp, rotate=True)
    return kp, vp


def _static_decode(lib, q, kp, vp, seq_len, flags, num_splits=0):
    B, hq = q.shape[0], q.shape[1]
    out = torch.empty((B, hq, 1, 128), dtype=torch.float16, device=q.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)
    bs_b, bs_h = kp.stride(0) // 128, kp.stride(1) // 128
    rc = lib.ecc_decode_static(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(kp.data_ptr()),
                               ctypes.c_void_p(vp.data_ptr()), bs_b, bs_h, ctypes.c_void_p(out.data_ptr()),
                               B, hq, kp.shape[1], seq_len, 0.0, flags, num_splits, stream)
    return rc, out


def test_static_decode_matches_workspace_decode_and_oracle_twice(lib, oracle, cuda_device):
    """Two calls in a row with different inputs: each equals the
    workspace-based decode within 2e-3 and the oracle within 2e-3 beyond
    the fp16 rounding of the oracle's value (half an fp16 ulp)."""
    import custom_ecc_cuda as ops
    cases = [  # (B, hq, hkv, L, seq_len, flags, seed)
        (2, 32, 8, 4096, 4000, 3, 1),
        (1, 8, 2, 700, 650, 0, 2),
    ]
    for B, hq, hkv, L, seq_len, flags, seed in cases:
        kp, vp = _pools(cuda_device, B, hkv, L, seed)
        q = torch.randn(B, hq, 1, 128, generator=torch.Generator().manual_seed(seed)).half().to(cuda_device)
        rc, got = _static_decode(lib, q, kp, vp, seq_len, flags)
        assert rc == 0, rc
        ref = ops.decode_attention(q, kp, vp, seq_len=seq_len, rotate_q=bool(flags & 1),
                                   unrotate_out=bool(flags & 2))
        torch.cuda.synchronize()
        err = (got.float() - ref.float()).abs().max().item()
        assert err <= TOL, err
        want = oracle.decode(q.cpu().numpy(), kp.cpu().numpy(), vp.cpu().numpy(), hkv=hkv, seq_len=seq_len,
                             rotate_q=bool(flags & 1), unrotate_out=bool(flags & 2)).astype(np.float32)
        a = np.abs(want.astype(np.float16))
        half_ulp = (np.nextafter(a, np.float16(np.inf)) - a).astype(np.float32) / 2
        g = got.float().cpu().numpy().reshape(want.shape)
        assert float((np.abs(g - want) - half_ulp).max()) <= TOL


def test_static_decode_rejects_requests_beyond_the_array(lib, cuda_device):
    # 4 x 32 query rows x 64 splits x 520 B = 4.26 MB of partials > 4 MiB; the
    # pools are real so that every access would stay in bounds anyway
    kp = torch.zeros((4, 8, 4096, 128), dtype=torch.uint8, device=cuda_device)
    q = torch.zeros((4, 32, 1, 128), dtype=torch.float16, device=cuda_device)
    rc, _ = _static_decode(lib, q, kp, kp, 4096, 0, num_splits=64)
    assert rc == -9
    rc, _ = _static_decode(lib, q, kp, kp, 4096, 0, num_splits=0)  # default splits are lowered to fit
    assert rc == 0
