"""Log-sum-exp combine of many split partials on the GPU (the merge kernels
and the fused exchange kernels all use it): rows of more than 32 partials are
combined in batches of 32 whose loads are issued one batch ahead, and a sum
kept under an earlier batch's maximum is rescaled when a later batch holds a
larger one.  Checked against an fp64 restatement of the combine
(M = max over non-empty partials, L = sum l e^(m - M), O = sum o e^(m - M)):
fp32 records within a relative 1e-5, fp16 outputs within half an fp16 ulp of
the reference plus 1e-6."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
D = 128


@pytest.fixture(scope="module")
def ops(cuda_device):
    import custom_ecc_cuda
    return custom_ecc_cuda


def _partials(rows, n, seed, ramp):
    """Seeded partials: m in natural-log units, l > 0 except every 7th (empty,
    m = -inf), o ~ l * N(0, 1).  ramp > 0 makes m grow with the split index,
    so every batch of 32 raises the running maximum; ramp < 0 lowers it."""
    g = np.random.default_rng(seed)
    m = g.normal(0.0, 2.0, (rows, n)) + ramp * np.arange(n)[None, :]
    l = g.uniform(0.5, 40.0, (rows, n))
    o = g.normal(0.0, 1.0, (rows, n, D)) * l[..., None]
    empty = (np.arange(n)[None, :] + np.arange(rows)[:, None]) % 7 == 3
    m[empty] = -np.inf
    l[empty] = 0.0
    o[empty] = 0.0
    return m.astype(np.float32), l.astype(np.float32), o.astype(np.float32)


def _combine64(m, l, o):
    m64, l64, o64 = m.astype(np.float64), l.astype(np.float64), o.astype(np.float64)
    live = l64 > 0
    M = np.where(live, m64, -np.inf).max(axis=1)
    with np.errstate(invalid="ignore"):  # -inf - -inf in rows with no live partial
        w = np.where(live, np.exp(m64 - M[:, None]), 0.0)
    L = (w * l64).sum(axis=1)
    O = (w[..., None] * o64).sum(axis=1)
    return M, L, O


@pytest.mark.parametrize("n", [1, 31, 32, 33, 64, 100, 223, 257])
@pytest.mark.parametrize("ramp", [0.0, 0.05, -0.05])
def test_many_partials_match_fp64_combine(ops, cuda_device, n, ramp):
    rows = 37
    m, l, o = _partials(rows, n, seed=n * 10 + int(ramp * 100), ramp=ramp)
    pm, pl, po = (torch.from_numpy(a).to(cuda_device) for a in (m, l, o))
    M, L, O = _combine64(m, l, o)

    rec = ops.lse_merge_to_record(pm, pl, po).cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(rec[:, 0], M, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(rec[:, 1], L, rtol=1e-5)
    live = L > 0  # rows whose partials are all empty give a zero output row
    ref = np.zeros_like(O)
    ref[live] = O[live] / L[live, None]
    np.testing.assert_allclose(rec[live, 2:] / rec[live, 1:2], ref[live], rtol=1e-5, atol=1e-6)
    assert not rec[~live, 1].any() and not rec[~live, 2:].any()

    out = ops.lse_merge(pm, pl, po).float().cpu().numpy()
    a = np.abs(ref.astype(np.float16))
    half_ulp = (np.nextafter(a, np.float16(np.inf)) - a).astype(np.float64) / 2
    assert float((np.abs(out - ref) - half_ulp).max()) <= 1e-6


def test_many_partials_records_and_one_call_agree(ops, cuda_device):
    """Partials merged in one call, and in two halves merged as records, give
    the same output within fp32 rounding (the cross-device combine)."""
    rows, n = 16, 223
    m, l, o = _partials(rows, n, seed=5, ramp=0.02)
    pm, pl, po = (torch.from_numpy(a).to(cuda_device) for a in (m, l, o))
    one = ops.lse_merge(pm, pl, po).float()
    h = 100
    ra = ops.lse_merge_to_record(pm[:, :h].contiguous(), pl[:, :h].contiguous(), po[:, :h].contiguous())
    rb = ops.lse_merge_to_record(pm[:, h:].contiguous(), pl[:, h:].contiguous(), po[:, h:].contiguous())
    two = ops.lse_merge_records(torch.stack([ra, rb])).float()
    assert float((one - two).abs().max()) <= 2e-3 * float(one.abs().max()) + 1e-3


def test_all_empty_row_gives_zero(ops, cuda_device):
    rows, n = 3, 70
    pm = torch.full((rows, n), float("-inf"), device=cuda_device)
    pl = torch.zeros((rows, n), device=cuda_device)
    po = torch.zeros((rows, n, D), device=cuda_device)
    pm[1, 40] = 0.5
    pl[1, 40] = 2.0
    po[1, 40] = 4.0
    out = ops.lse_merge(pm, pl, po).float().cpu()
    assert torch.equal(out[0], torch.zeros(D)) and torch.equal(out[2], torch.zeros(D))
    assert torch.allclose(out[1], torch.full((D,), 2.0))
