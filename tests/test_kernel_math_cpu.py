"""CPU checks of the arithmetic the compress kernel relies on (no GPU):
the division by fp32(sqrt(128)) and the table-driven quantiser with its exact
fallback band, emulated in numpy float32 and compared with the oracle."""
import ctypes

import numpy as np
import pytest

import workloads

CELLS, MAGIC, BAND = 192, np.float32(12582912.0), np.float32(4e-6)
BAND_FAST = np.float32(1.5e-6)  # the packed fast pass's band (compress.cu kBandFast)


def test_division_by_sqrt128_sampled(oracle):
    lib = oracle.lib()
    lib.orc_check_div_sqrt128.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]
    lib.orc_check_div_sqrt128.restype = ctypes.c_int64
    # every 4099th bit pattern over the whole fp32 range, plus all mantissas of [1, 2)
    assert lib.orc_check_div_sqrt128(7, (1 << 32) // 4099, 4099) == 0
    assert lib.orc_check_div_sqrt128(0x3F800000, 1 << 23, 1) == 0


def _thresholds(C):
    return np.array([np.float32((np.float32(C[j - 1]) + np.float32(C[j])) * np.float32(0.5)) for j in range(1, 16)],
                    np.float32)


def _cell(u):
    t = (np.float32(8.0) * u.astype(np.float32)).astype(np.float32) + (MAGIC + np.float32(96.0))
    return t.astype(np.float32).view(np.int32) - np.array([MAGIC], np.float32).view(np.int32)[0]


def _table(C):
    m = _thresholds(C)
    cm = _cell(m)
    tab = []
    for cell in range(CELLS):
        own = [j + 1 for j in range(15) if cm[j] == cell]
        if own:
            j = own[0]
            thr, qlo = m[j - 1], j - 1
        else:
            thr, qlo = np.float32(np.inf), int((cm < cell).sum())
        tab.append((thr, C[qlo], C[min(qlo + 1, 15)], qlo))
    return tab, m, cm


def test_threshold_cells_are_separated(oracle):
    C = oracle.LM_CENTROIDS
    _, m, cm = _table(C)
    assert len(set(cm.tolist())) == 15 and np.all(np.diff(cm) >= 2)
    frac = np.abs((np.float64(m) * 8 + 96) - np.rint(np.float64(m) * 8 + 96))
    # distance of every threshold from a cell boundary, in u units, far above the band
    assert np.min((0.5 - frac) / 8) > 100 * BAND


def test_table_quantiser_equals_argmin(oracle):
    """Emulate the kernel's quantiser on real compress inputs and compare the
    codes with the oracle's first-index argmin."""
    C = oracle.LM_CENTROIDS
    tab, _, _ = _table(C)
    thr = np.array([t[0] for t in tab], np.float32)
    qlo = np.array([t[3] for t in tab], np.int64)
    x16 = np.concatenate([workloads.make_heavy(seed=31, n=2048).numpy(),
                          workloads.make_c1(seed=4, L=64)[0].reshape(-1, 128).numpy(),
                          workloads.make_edge().numpy()])
    r = oracle.compress_np(x16, rotate=True)
    xr, zero, scale, q_ref = r["x_rot"], r["zero"], r["scale"], r["q"]
    d = (xr - zero[:, None]).astype(np.float32)
    rs = (np.float64(1.0) / scale.astype(np.float64)).astype(np.float32)  # RN(1/scale)
    u = (d * rs[:, None]).astype(np.float32)
    cell = np.minimum(_cell(u).astype(np.int64) & 0xFFFFFFFF, CELLS - 1)
    hi = u > thr[cell]
    q = qlo[cell] + hi
    band = np.abs((u - thr[cell]).astype(np.float32)) < BAND
    xn = (d / scale[:, None]).astype(np.float32)
    exact = np.abs(xn[..., None] - C[None, None, :]).astype(np.float32).argmin(-1)
    q = np.where(band, exact, q)
    assert np.array_equal(q, q_ref)
    assert band.sum() < 0.001 * band.size


def _fast_pass_codes(d, scale, C, tab):
    """The packed fast pass's quantiser: cell from fma(d, 8 rs, magic + 96),
    side from w = fma(d, rs, -thr), band |w| < BAND_FAST.  float64 holds the
    exact products d*rs (48-bit), so one rounding to float32 emulates each fma."""
    thr = np.array([t[0] for t in tab], np.float32)
    qlo = np.array([t[3] for t in tab], np.int64)
    rs = (np.float64(1.0) / scale.astype(np.float64)).astype(np.float32)
    rs8 = (rs * np.float32(8.0)).astype(np.float32)
    t = (d.astype(np.float64) * rs8.astype(np.float64)[..., None] + np.float64(MAGIC + np.float32(96.0))).astype(np.float32)
    cell = t.view(np.int32) - np.array([MAGIC], np.float32).view(np.int32)[0]
    assert cell.min() >= 0 and cell.max() < CELLS  # no clamp in the kernel
    w = (d.astype(np.float64) * rs.astype(np.float64)[..., None] - thr[cell].astype(np.float64)).astype(np.float32)
    return qlo[cell] + (w >= 0), np.abs(w) < BAND_FAST


def test_fast_pass_quantiser_equals_argmin(oracle):
    """The packed fast pass's decision rule on real compress inputs: outside
    its band the codes are the oracle's first-index argmin."""
    C = oracle.LM_CENTROIDS
    tab, _, _ = _table(C)
    x16 = np.concatenate([workloads.make_heavy(seed=32, n=2048).numpy(),
                          workloads.make_c1(seed=5, L=64)[0].reshape(-1, 128).numpy(),
                          workloads.make_edge().numpy()])
    r = oracle.compress_np(x16, rotate=True)
    d = (r["x_rot"] - r["zero"][:, None]).astype(np.float32)
    q, band = _fast_pass_codes(d, r["scale"], C, tab)
    assert np.array_equal(q[~band], r["q"][~band])
    assert band.sum() < 0.001 * band.size


def test_fast_pass_band_near_thresholds(oracle):
    """Quotients placed within 3e-6 of every decision threshold over scales
    1e-3..1e3: no fast-pass decision outside the band differs from the
    reference's RN(d / scale) argmin, and the closest wrong decision of an
    unbanded rule stays far inside the band."""
    C = oracle.LM_CENTROIDS.astype(np.float32)
    tab, m, _ = _table(C)
    rng = np.random.default_rng(5)
    n = 1_000_000
    j = rng.integers(0, 15, n)
    scale = np.exp(rng.uniform(np.log(1e-3), np.log(1e3), n)).astype(np.float32)
    d = ((m[j].astype(np.float64) + rng.uniform(-3e-6, 3e-6, n)) * scale.astype(np.float64)).astype(np.float32)
    xn = (d.astype(np.float64) / scale.astype(np.float64)).astype(np.float32)
    q_ref = np.abs((xn[:, None] - C[None, :]).astype(np.float32)).argmin(1)
    rs = (np.float64(1.0) / scale.astype(np.float64)).astype(np.float32)
    w = (d.astype(np.float64) * rs.astype(np.float64) - m[j].astype(np.float64)).astype(np.float32)
    wrong = (j + (w >= 0)) != q_ref
    assert not np.any(wrong & (np.abs(w) >= BAND_FAST))
    assert np.abs(w[wrong]).max() < BAND_FAST / 4
