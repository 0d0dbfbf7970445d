"""Pin the oracle to the reference: every fixture in tests/golden was produced
by the reference's own ops_cpu.compress_cpu / fused_decode.cpu_reference_decode
(tests/golden/make_golden.py).  CPU only."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

import workloads

GROUPS = ["c1", "heavy", "offset", "edge"]
FIELDS = ["x_rot", "q", "syn", "zero", "scale", "alpha", "blocks"]


def test_centroid_table_bits(oracle, compress_golden):
    assert np.array_equal(oracle.LM_BITS, compress_golden["lm_bits"])
    c = np.zeros(16, np.float32)
    lib = oracle.lib()
    lib.orc_centroids(oracle._ptr(c))
    assert np.array_equal(c.view(np.uint32), compress_golden["lm_bits"])


@pytest.mark.parametrize("group", GROUPS)
@pytest.mark.parametrize("rot", [1, 0])
def test_c_oracle_matches_reference(oracle, compress_golden, group, rot):
    x16 = compress_golden[f"{group}_x16"]
    for i in range(x16.shape[0]):
        r = oracle.compress_detail(x16[i], rotate=bool(rot))
        pre = f"{group}_r{rot}_"
        assert np.array_equal(r["x_rot"].view(np.uint32), compress_golden[pre + "x_rot"][i].view(np.uint32)), i
        assert np.array_equal(r["q"], compress_golden[pre + "q"][i]), i
        assert np.array_equal(r["syndrome"], compress_golden[pre + "syn"][i]), i
        for k in ("zero", "scale", "alpha"):
            a = np.float32(r[k]).view(np.uint32)
            b = compress_golden[pre + k][i].view(np.uint32)
            assert a == b or (np.isnan(r[k]) and np.isnan(compress_golden[pre + k][i])), (k, i)
        assert np.array_equal(r["block"], compress_golden[pre + "blocks"][i]), i


@pytest.mark.parametrize("group", GROUPS)
@pytest.mark.parametrize("rot", [1, 0])
def test_numpy_restatement_matches_reference(oracle, compress_golden, group, rot):
    x16 = compress_golden[f"{group}_x16"]
    r = oracle.compress_np(x16, rotate=bool(rot))
    pre = f"{group}_r{rot}_"
    assert np.array_equal(r["q"], compress_golden[pre + "q"])
    assert np.array_equal(r["syndrome"], compress_golden[pre + "syn"])
    assert np.array_equal(r["blocks"], compress_golden[pre + "blocks"])


def test_batched_c_compress_equals_detail(oracle, compress_golden):
    x16 = np.concatenate([compress_golden[f"{g}_x16"] for g in GROUPS])
    for rot in (1, 0):
        blocks = oracle.compress(x16, rotate=bool(rot), threads=4)
        ref = np.concatenate([compress_golden[f"{g}_r{rot}_blocks"] for g in GROUPS])
        assert np.array_equal(blocks, ref)


def test_c_and_numpy_agree_on_large_heavy_tail(oracle):
    x16 = workloads.make_heavy(seed=5, n=4096).numpy()
    a = oracle.compress(x16, rotate=True)
    b = oracle.compress_np(x16, rotate=True)["blocks"]
    assert np.array_equal(a, b)


def test_full_c1_block_digest(oracle):
    """All 2 x 16384 vectors of the single-layer op test, hashed."""
    with open(os.path.join(os.path.dirname(__file__), "golden", "c1_digest.json")) as f:
        dig = json.load(f)
    k16, v16, _ = workloads.make_c1(seed=0)
    kb = oracle.compress(k16.reshape(-1, 128).numpy(), rotate=True)
    vb = oracle.compress(v16.reshape(-1, 128).numpy(), rotate=True)
    assert hashlib.sha256(kb.tobytes()).hexdigest() == dig["k_sha256"]
    assert hashlib.sha256(vb.tobytes()).hexdigest() == dig["v_sha256"]


def _fp16_close(a16: np.ndarray, b16: np.ndarray, atol: float):
    a = a16.astype(np.float32)
    b = b16.astype(np.float32)
    return float(np.max(np.abs(a - b))) if a.size else 0.0


@pytest.mark.parametrize("ci", range(4))
def test_decode_oracle_matches_reference(oracle, decode_golden, ci):
    B, hq, hkv, L = [int(v) for v in decode_golden[f"case{ci}_meta"]]
    q16 = decode_golden[f"case{ci}_q16"].view(np.float16)
    out = oracle.decode(q16, decode_golden[f"case{ci}_kblocks"], decode_golden[f"case{ci}_vblocks"],
                        hkv=hkv, seq_len=L)
    ref = decode_golden[f"case{ci}_out16"].view(np.float16).reshape(B, hq, 128)
    err = _fp16_close(out.astype(np.float16), ref, 0)
    assert err <= 1e-3, err


def test_c1_decode_oracle_matches_reference(oracle):
    path = os.path.join(os.path.dirname(__file__), "golden", "c1_decode_out16.npy")
    if not os.path.exists(path):
        pytest.skip("c1 decode fixture not generated")
    k16, v16, q16 = workloads.make_c1(seed=0)
    kb = oracle.compress(k16.reshape(-1, 128).numpy(), rotate=True).reshape(1, 8, 2048, 128)
    vb = oracle.compress(v16.reshape(-1, 128).numpy(), rotate=True).reshape(1, 8, 2048, 128)
    out = oracle.decode(q16.numpy(), kb, vb, hkv=8, seq_len=2048)
    ref = np.load(path).view(np.float16).reshape(1, 32, 128)
    assert _fp16_close(out.astype(np.float16), ref, 0) <= 1e-3


def test_decode_rotation_flags(oracle, decode_golden):
    """rotate_q rotates the query; unrotate_out applies the WHT to the output."""
    B, hq, hkv, L = [int(v) for v in decode_golden["case2_meta"]]
    q16 = decode_golden["case2_q16"].view(np.float16).reshape(B, hq, 128)
    kb, vb = decode_golden["case2_kblocks"], decode_golden["case2_vblocks"]
    q_rot16 = oracle.wht(q16.astype(np.float32)).astype(np.float16)
    a = oracle.decode(q16, kb, vb, hkv=hkv, seq_len=L, rotate_q=True, unrotate_out=True)
    b = oracle.decode(q_rot16, kb, vb, hkv=hkv, seq_len=L)
    assert np.allclose(a, oracle.wht(b), atol=1e-6)


def test_lse_merge_equals_unsplit(oracle):
    rng = np.random.default_rng(0)
    rows, n = 6, 5
    scores = rng.normal(size=(rows, 40)).astype(np.float32) * 3
    vals = rng.normal(size=(40, 128)).astype(np.float32)
    full = np.exp(scores - scores.max(1, keepdims=True))
    full = (full @ vals) / full.sum(1, keepdims=True)
    pm = np.zeros((rows, n), np.float32)
    pl = np.zeros((rows, n), np.float32)
    po = np.zeros((rows, n, 128), np.float32)
    bounds = [0, 3, 3, 20, 33, 40]  # includes an empty split
    for i in range(n):
        a, b = bounds[i], bounds[i + 1]
        if b == a:
            pm[:, i] = -np.inf
            continue
        s = scores[:, a:b]
        m = s.max(1)
        w = np.exp(s - m[:, None])
        pm[:, i], pl[:, i], po[:, i] = m, w.sum(1), w @ vals[a:b]
    assert np.allclose(oracle.lse_merge(pm, pl, po), full, atol=1e-5)


def test_fp16_conversions(oracle):
    lib = oracle.lib()
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.normal(size=2000) * 10.0 ** rng.integers(-9, 6, size=2000),
                           [0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e9, -1e9, 2 ** -24, 2 ** -25,
                            3 * 2 ** -26, 2 ** -14, 2 ** -14 - 2 ** -25, 5.96e-8]]).astype(np.float32)
    for v in vals:
        h = lib.orc_f2h(float(v))
        assert h == np.float32(v).astype(np.float16).view(np.uint16), v
        back = lib.orc_h2f(h)
        assert np.float32(back).view(np.uint32) == np.float16(np.uint16(h).view(np.float16)).astype(np.float32).view(np.uint32)


def test_wht_properties(oracle):
    rng = np.random.default_rng(2)
    x = rng.normal(size=(4, 128)).astype(np.float32)
    assert np.allclose(oracle.wht(oracle.wht(x)), x, atol=1e-5)
    eye = oracle.wht(np.eye(128, dtype=np.float32))
    assert np.allclose(eye @ eye.T, np.eye(128), atol=1e-5)
    for d in (64, 256):
        y = rng.normal(size=(2, d)).astype(np.float32)
        assert np.allclose(oracle.wht(oracle.wht(y)), y, atol=1e-5)


def test_tie_counter(oracle):
    x16 = workloads.make_heavy(seed=9, n=512).numpy()
    assert oracle.count_ties(x16, tol=1e-6) >= 0
    assert oracle.count_ties(x16, tol=1.0) > 0


def test_calibrated_oracle_matches_reference(oracle):
    """Compress with fixed per-layer parameters: the oracle equals the
    reference's lloyd_max_quantize_cpu + compute_syndrome_cpu fixtures
    (tests/golden/make_calibrated_golden.py) for every parameter set, rotated
    and unrotated, including fp16 extremes far outside the centroid range."""
    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "calibrated_golden.npz")))
    for pi, (scale, zero, alpha) in enumerate(g["params"]):
        for rot in (1, 0):
            got = oracle.compress_calibrated_np(g["x16"], scale, zero, alpha, rotate=bool(rot))
            assert np.array_equal(got, g[f"p{pi}_r{rot}_blocks"]), (pi, rot)
