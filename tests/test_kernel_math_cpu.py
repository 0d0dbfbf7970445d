"""CPU checks of the arithmetic the compress kernel relies on (no GPU):
the division by fp32(sqrt(128)) and the table-driven quantiser with its exact
fallback band, emulated in numpy float32 and compared with the oracle."""
import ctypes

import numpy as np
import pytest

import workloads

CELLS, MAGIC, BAND = 192, np.float32(12582912.0), np.float32(4e-6)
BAND_FAST = np.float32(8e-7)  # the packed fast pass's band (compress.cu kBandFast)
BAND_BOUND = 5.2e-7  # |w| beyond which a fast-pass decision is the reference's (error budget in compress.cu)


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
    reference's RN(d / scale) argmin, and every wrong decision of an
    unbanded rule lies inside the error-budget bound, which the band
    exceeds by 1.5x."""
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
    assert BAND_FAST >= 1.5 * BAND_BOUND
    assert not np.any(wrong & (np.abs(w) >= BAND_FAST))
    assert np.abs(w[wrong]).max() < BAND_BOUND


def _lanes_tsum(V):
    """compress_lat_kernel's torch-order sum over lanes: V [N, 32 lanes, 4]
    (lane i holds elements i + 32m); lane 8a + l is accumulator acc[a][l]."""
    acc = np.float32(0.0) + V[..., 0]
    for m in range(1, 4):
        acc = (acc + V[..., m]).astype(np.float32)
    t = [(((acc[:, l] + acc[:, l + 8]).astype(np.float32) + acc[:, l + 16]).astype(np.float32)
          + acc[:, l + 24]).astype(np.float32) for l in range(8)]
    s = t[0]
    for k in range(1, 8):
        s = (s + t[k]).astype(np.float32)
    return s


def test_warp_per_vector_layout(oracle):
    """The small-call compress kernel's lane layout emulated in numpy float32:
    WHT strides 1..16 as lane exchanges (upper lane: partner - mine), 32 and
    64 in registers; mean and alpha summed lane-wise in torch's order; code
    word 4m + i/8 by OR over lanes 8(i/8)..+7, syndrome word m as the ballot
    of element group m, block word i written by lane i.  The result equals the
    oracle's blocks."""
    x16 = np.concatenate([workloads.make_heavy(seed=33, n=512).numpy(),
                          workloads.make_c1(seed=6, L=16)[0].reshape(-1, 128).numpy(),
                          workloads.make_edge().numpy()])
    r = oracle.compress_np(x16, rotate=True)
    n = x16.shape[0]
    lane = np.arange(32)
    V = x16.astype(np.float32).reshape(n, 4, 32).transpose(0, 2, 1).copy()  # V[:, i, m] = x[32m + i]
    with np.errstate(all="ignore"):
        for s in (1, 2, 4, 8, 16):
            P = V[:, lane ^ s, :]
            V = np.where(((lane & s) != 0)[None, :, None], (P - V).astype(np.float32), (V + P).astype(np.float32))
        for a, c in ((0, 1), (2, 3), (0, 2), (1, 3)):
            va, vc = V[..., a].copy(), V[..., c].copy()
            V[..., a], V[..., c] = va + vc, va - vc
        V = (V / np.float32(np.sqrt(128.0))).astype(np.float32)
        xr = V.transpose(0, 2, 1).reshape(n, 128)
        assert np.array_equal(xr, r["x_rot"], equal_nan=True)
        zero = (_lanes_tsum(V) * np.float32(1 / 128)).astype(np.float32)
        assert np.array_equal(zero, r["zero"], equal_nan=True)
        q = r["q"].reshape(n, 4, 32).transpose(0, 2, 1).astype(np.uint32)  # code of lane i, group m
        kt = ((oracle.LM_CENTROIDS[r["q"]] * r["scale"][:, None]).astype(np.float32) + r["zero"][:, None])
        eps = (r["x_rot"] - kt.astype(np.float32)).astype(np.float32)
        E = eps.reshape(n, 4, 32).transpose(0, 2, 1)
        alpha = (_lanes_tsum(np.abs(E)) * np.float32(1 / 128)).astype(np.float32)
        assert np.array_equal(alpha, r["alpha"], equal_nan=True)
    # code words: lanes 8k..8k+7 OR their nibbles q << 4 (lane % 8) -> word 4m + k
    nib = q << (4 * (lane % 8))[None, :, None].astype(np.uint32)
    cw = np.zeros((n, 4, 4), np.uint32)  # [vector, m, k]
    for k in range(4):
        cw[:, :, k] = np.bitwise_or.reduce(nib[:, 8 * k:8 * k + 8, :], axis=1)
    syn = ((E >= 0).astype(np.uint64) << lane[None, :, None].astype(np.uint64)).sum(1).astype(np.uint32)  # ballots
    words = np.zeros((n, 32), np.uint32)
    for i in range(16):
        words[:, i] = cw[:, i >> 2, i & 3]  # lane i reads word i from lane 8 (i % 4), group i / 4
    words[:, 16:20] = syn
    meta = np.stack([r["scale"], r["zero"], r["alpha"]], 1).astype(np.float16).view(np.uint16).astype(np.uint32)
    words[:, 20] = meta[:, 0] | (meta[:, 1] << 16)
    words[:, 21] = meta[:, 2]
    assert np.array_equal(words.view(np.uint8).reshape(n, 128), r["blocks"])
