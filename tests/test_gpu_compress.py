"""Compress path on the GPU through the C ABI, bit-exact against the oracle and
the reference's golden vectors."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

import workloads

pytestmark = pytest.mark.gpu
GROUPS = ["c1", "heavy", "offset", "edge"]


@pytest.fixture(scope="module")
def ops(cuda_device):
    import custom_ecc_cuda
    return custom_ecc_cuda


def _f16(a: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.float16).to(dev)


@pytest.mark.parametrize("group", GROUPS)
def test_rotate_compress_matches_reference_golden(ops, compress_golden, cuda_device, group):
    x = _f16(compress_golden[f"{group}_x16"], cuda_device)
    blocks = ops.rotate_and_compress(x)
    got = blocks.cpu().numpy()
    ref = compress_golden[f"{group}_r1_blocks"]
    bad = np.nonzero((got != ref).any(1))[0]
    assert bad.size == 0, f"rows {bad[:10]} differ"


@pytest.mark.parametrize("group", GROUPS)
def test_compress_and_store_matches_reference_golden(ops, compress_golden, cuda_device, group):
    """Pre-rotated input, the reference op's contract (csrc/ecc_ops.cpp:68)."""
    x = _f16(compress_golden[f"{group}_x16"], cuda_device)
    cache = torch.full((x.shape[0] + 3, 128), 0xAB, dtype=torch.uint8, device=cuda_device)
    ops.compress_and_store(x, cache)
    got = cache.cpu().numpy()
    assert np.array_equal(got[:x.shape[0]], compress_golden[f"{group}_r0_blocks"])
    assert np.all(got[x.shape[0]:] == 0xAB)  # rows past N untouched


def test_full_c1_digest(ops, cuda_device):
    with open(os.path.join(os.path.dirname(__file__), "golden", "c1_digest.json")) as f:
        dig = json.load(f)
    k16, v16, _ = workloads.make_c1(seed=0)
    kp = torch.empty((1, 8, 2048, 128), dtype=torch.uint8, device=cuda_device)
    vp = torch.empty_like(kp)
    ops.compress_into(k16.to(cuda_device), kp, pos=0, rotate=True)
    ops.compress_into(v16.to(cuda_device), vp, pos=0, rotate=True)
    assert hashlib.sha256(kp.cpu().numpy().tobytes()).hexdigest() == dig["k_sha256"]
    assert hashlib.sha256(vp.cpu().numpy().tobytes()).hexdigest() == dig["v_sha256"]


@pytest.mark.parametrize("rotate", [True, False])
def test_large_heavy_tail_equals_oracle(ops, oracle, cuda_device, rotate):
    """2 heads x 131072 tokens of the compress-throughput workload, every block."""
    x16 = workloads.make_heavy(seed=77, n=262144)
    got = ops.rotate_and_compress(x16.to(cuda_device)) if rotate else None
    if not rotate:
        got = torch.empty((x16.shape[0], 128), dtype=torch.uint8, device=cuda_device)
        ops.compress_and_store(x16.to(cuda_device), got)
    ref = oracle.compress(x16.numpy(), rotate=rotate)
    got = got.cpu().numpy()
    bad = np.nonzero((got != ref).any(1))[0]
    ties = oracle.count_ties(x16.numpy()[bad], rotate=rotate, tol=1e-6) if bad.size else 0
    assert bad.size == 0, f"{bad.size} blocks differ ({ties} tie elements among them)"


@pytest.mark.parametrize("B,H,L,pos", [(8, 8, 1, 4095), (2, 4, 37, 5), (1, 8, 2048, 0)])
def test_pair_equals_two_single_compresses(ops, cuda_device, B, H, L, pos):
    """compress_pair_into (K and V of one append in one launch) writes exactly
    what two compress_into calls write, also for strided (transposed) inputs."""
    g = torch.Generator(device=cuda_device).manual_seed(L)
    k = torch.randn((B, L, H, 128), generator=g, device=cuda_device).half().transpose(1, 2)  # strided view
    v = (torch.randn((B, H, L, 128), generator=g, device=cuda_device) * 3).half()
    cap = pos + L + 3
    kp1 = torch.zeros((B, H, cap, 128), dtype=torch.uint8, device=cuda_device)
    vp1, kp2, vp2 = torch.zeros_like(kp1), torch.zeros_like(kp1), torch.zeros_like(kp1)
    ops.compress_into(k, kp1, pos=pos, rotate=True)
    ops.compress_into(v, vp1, pos=pos, rotate=True)
    ops.compress_pair_into(k, v, kp2, vp2, pos=pos, rotate=True)
    assert torch.equal(kp1, kp2) and torch.equal(vp1, vp2)
    assert torch.count_nonzero(kp2[:, :, :pos]) == 0 and torch.count_nonzero(kp2[:, :, pos + L:]) == 0


def test_strided_input_into_pool_positions(ops, oracle, cuda_device):
    """HF key_states are a transposed view [B, H, L, D]; write at pos > 0."""
    B, H, L, cap, pos = 2, 3, 37, 64, 11
    g = torch.Generator().manual_seed(5)
    base = torch.randn(B, L, H, 128, generator=g).half()
    x = base.to(cuda_device).transpose(1, 2)  # [B, H, L, D], non-contiguous
    pool = torch.zeros((B, H, cap, 128), dtype=torch.uint8, device=cuda_device)
    ops.compress_into(x, pool, pos=pos, rotate=True)
    ref = oracle.compress(base.transpose(1, 2).contiguous().reshape(-1, 128).numpy(), rotate=True)
    got = pool.cpu().numpy()
    assert np.array_equal(got[:, :, pos:pos + L].reshape(-1, 128), ref)
    assert not got[:, :, :pos].any() and not got[:, :, pos + L:].any()


@pytest.mark.parametrize("n", [1, 7, 63, 64, 65, 1000])
def test_ragged_counts(ops, oracle, cuda_device, n):
    x16 = workloads.make_heavy(seed=n, n=n)
    got = ops.rotate_and_compress(x16.to(cuda_device)).cpu().numpy()
    assert np.array_equal(got, oracle.compress(x16.numpy(), rotate=True))


@pytest.mark.parametrize("rotate", [True, False])
def test_small_and_tiled_calls_agree(ops, oracle, cuda_device, rotate):
    """Calls of up to 4096 vectors run one warp per vector, larger calls the
    tiled kernel: the same rows give the same blocks through both, equal to
    the oracle's (heavy tails, c1 rows and the hand-made edge rows)."""
    x16 = torch.cat([workloads.make_heavy(seed=58, n=4000), workloads.make_c1(seed=7, L=16)[0].reshape(-1, 128),
                     workloads.make_edge()] * 2)
    n = x16.shape[0]
    assert n > 4096
    xd = x16.to(cuda_device)

    def run(x):
        if rotate:
            return ops.rotate_and_compress(x)
        out = torch.empty((x.shape[0], 128), dtype=torch.uint8, device=cuda_device)
        ops.compress_and_store(x, out)
        return out

    tiled = run(xd).cpu().numpy()
    small = np.concatenate([run(xd[i:i + 4096]).cpu().numpy() for i in range(0, n, 4096)])
    assert np.array_equal(small, tiled)
    assert np.array_equal(small, oracle.compress(x16.numpy(), rotate=rotate))


def test_empty_input(ops, cuda_device):
    x = torch.empty((0, 128), dtype=torch.float16, device=cuda_device)
    assert ops.rotate_and_compress(x).shape == (0, 128)


@pytest.mark.parametrize("d", [1, 2, 16, 64, 128, 256, 1024])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_hadamard_rotate(ops, oracle, cuda_device, d, dtype):
    g = torch.Generator().manual_seed(d)
    x = (torch.randn(33, d, generator=g) * 3).to(dtype)
    y = x.to(cuda_device)
    out = ops.hadamard_rotate(y)
    assert out.data_ptr() == y.data_ptr()  # in place
    ref = oracle.wht(x.float().numpy()) if d > 1 else x.float().numpy()
    if dtype == torch.float32:
        assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    else:
        assert np.array_equal(y.cpu().numpy().view(np.uint16), ref.astype(np.float16).view(np.uint16))


def test_hadamard_errors(ops, cuda_device):
    with pytest.raises(RuntimeError, match="power of 2"):
        ops.hadamard_rotate(torch.zeros(2, 100, device=cuda_device))
    with pytest.raises(RuntimeError, match="1024"):
        ops.hadamard_rotate(torch.zeros(2, 2048, device=cuda_device))
    with pytest.raises(RuntimeError, match="float16 and float32"):
        ops.hadamard_rotate(torch.zeros(2, 128, device=cuda_device, dtype=torch.float64))
    with pytest.raises(RuntimeError, match="2D"):
        ops.hadamard_rotate(torch.zeros(2, 2, 128, device=cuda_device))
    with pytest.raises(RuntimeError, match="contiguous"):
        ops.hadamard_rotate(torch.zeros(128, 4, device=cuda_device).t())


def test_compress_errors(ops, cuda_device):
    x = torch.zeros(4, 128, dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError, match="D=128"):
        ops.compress_and_store(torch.zeros(4, 64, dtype=torch.float16, device=cuda_device),
                               torch.zeros(4, 128, dtype=torch.uint8, device=cuda_device))
    with pytest.raises(RuntimeError, match="\\[N, 128\\]"):
        ops.compress_and_store(x, torch.zeros(4, 64, dtype=torch.uint8, device=cuda_device))
    with pytest.raises(RuntimeError):
        ops.compress_and_store(x.float(), torch.zeros(4, 128, dtype=torch.uint8, device=cuda_device))
    with pytest.raises(RuntimeError, match="capacity"):
        ops.compress_into(x.view(1, 1, 4, 128), torch.zeros((1, 1, 6, 128), dtype=torch.uint8, device=cuda_device),
                          pos=3)


def test_get_block_metadata(ops, compress_golden, cuda_device):
    blocks = torch.from_numpy(compress_golden["heavy_r1_blocks"]).to(cuda_device)
    for i in (0, 5, 255):
        md = ops.get_block_metadata(blocks, i)
        assert md.device.type == "cpu" and md.dtype == torch.float32
        ref = compress_golden["heavy_r1_blocks"][i, 80:86].view(np.float16).astype(np.float32)
        assert np.array_equal(md.numpy(), ref)
    with pytest.raises(RuntimeError):
        ops.get_block_metadata(blocks, 256)


def test_dequantize_matches_reconstruction(ops, oracle, compress_golden, cuda_device):
    blk = np.concatenate([compress_golden[f"{g}_r1_blocks"] for g in ("c1", "heavy")])
    got = ops.dequantize(torch.from_numpy(blk).to(cuda_device)).cpu().numpy()
    ref = oracle.reconstruct(blk).astype(np.float16)
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))


def test_pack_soa_roundtrip(ops, oracle, compress_golden, cuda_device):
    blk = compress_golden["c1_r1_blocks"]
    int4, syn, meta = oracle.blocks_to_soa(blk)
    t = lambda a: torch.from_numpy(a).to(cuda_device)
    packed = ops.pack_soa(t(int4), t(syn), t(meta.view(np.int16)).view(torch.float16)).cpu().numpy()
    assert np.array_equal(packed, blk)


def _calibrated_golden():
    return dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "calibrated_golden.npz")))


@pytest.mark.parametrize("rotate", [True, False])
def test_calibrated_compress_matches_reference_golden(ops, cuda_device, rotate):
    """Fixed per-layer quantiser parameters (a calibration config's scale,
    zero, alpha): blocks equal the reference's lloyd_max_quantize_cpu +
    compute_syndrome_cpu fixtures bit for bit."""
    g = _calibrated_golden()
    x = _f16(g["x16"], cuda_device).reshape(1, 1, -1, 128)
    for pi, (scale, zero, alpha) in enumerate(g["params"]):
        pool = torch.empty((1, 1, x.shape[2], 128), dtype=torch.uint8, device=cuda_device)
        ops.compress_calibrated_into(x, pool, scale, zero, alpha, rotate=rotate)
        got = pool.reshape(-1, 128).cpu().numpy()
        bad = np.nonzero((got != g[f"p{pi}_r{int(rotate)}_blocks"]).any(1))[0]
        assert bad.size == 0, f"parameter set {pi}: rows {bad[:10]} differ"


def test_calibrated_compress_large_and_non_finite(ops, oracle, cuda_device):
    """65536 heavy-tailed vectors under narrow and wide layer parameters,
    plus rows with inf and nan, against the oracle; strided input into a pool
    position; bad parameters raise."""
    x16 = workloads.make_heavy(seed=91, n=65536)
    x16[7, 3] = float("inf")
    x16[8, 100] = float("-inf")
    x16[9, 0] = float("nan")
    for scale, zero, alpha in ((0.05, -0.01, 0.02), (1.05, 0.02, 0.21), (9.0, 1.5, 2.0)):
        # [B, L, H, D] memory seen as [B, H, L, D] (HF layout before its transpose)
        xd = x16.to(cuda_device).reshape(4, 8192, 2, 128).transpose(1, 2)
        pool = torch.zeros((4, 2, 8200, 128), dtype=torch.uint8, device=cuda_device)
        ops.compress_calibrated_into(xd, pool, scale, zero, alpha, pos=5, rotate=True)
        got = pool[:, :, 5:5 + 8192].reshape(-1, 128).cpu().numpy()
        rows = x16.reshape(4, 8192, 2, 128).transpose(1, 2).reshape(-1, 128).numpy()
        ref = oracle.compress_calibrated_np(rows, scale, zero, alpha, rotate=True)
        bad = np.nonzero((got != ref).any(1))[0]
        assert bad.size == 0, f"{bad.size} blocks differ, first {bad[:8]}"
        assert not pool[:, :, :5].any() and not pool[:, :, 5 + 8192:].any()
    x = x16[:4].to(cuda_device).reshape(1, 1, 4, 128)
    pool = torch.empty((1, 1, 4, 128), dtype=torch.uint8, device=cuda_device)
    for bad_args in ((0.0, 0.0, 0.1), (1.0, float("nan"), 0.1)):
        with pytest.raises(RuntimeError):
            ops.compress_calibrated_into(x, pool, *bad_args)


def test_hadamard_rotate_keeps_infinities(ops, oracle, cuda_device):
    """hadamard_rotate_cpu divides by fp32(sqrt(128)): +-inf elements stay
    +-inf (inf - inf butterflies give NaN), like the oracle."""
    x = torch.randn(4, 128)
    x[0, 5] = float("inf")
    x[1, 0] = float("-inf")
    x[2, 7] = float("inf")
    x[2, 9] = float("-inf")
    x[3, 1] = float("nan")
    ref = oracle.wht(x.numpy())
    for dt in (torch.float32, torch.float16):
        got = x.to(dt).to(cuda_device)
        ops.hadamard_rotate(got)
        r = oracle.wht(x.to(dt).float().numpy())
        g = got.float().cpu().numpy()
        if dt == torch.float16:
            r = r.astype(np.float16).astype(np.float32)
        assert np.array_equal(np.isnan(g), np.isnan(r)) and np.array_equal(g[~np.isnan(g)], r[~np.isnan(r)])
    assert np.isinf(ref[0]).all()


def test_full_compress_workload_equals_oracle(ops, oracle, cuda_device):
    """The whole compress benchmark workload -- 8 kv heads x 131072 tokens of
    K and V (heavy-tailed fp16), 2 097 152 vectors -- through the same launch
    shape the benchmark times, every block bit-exact with the oracle."""
    k, v = workloads.make_c2(seed=0, L=131072, device=cuda_device)
    for x in (k, v):
        pool = torch.empty((1, 8, 131072, 128), dtype=torch.uint8, device=cuda_device)
        ops.compress_into(x, pool, rotate=True)
        got = pool.reshape(-1, 128).cpu().numpy()
        ref = oracle.compress(x.reshape(-1, 128).cpu().numpy(), rotate=True)
        bad = np.nonzero((got != ref).any(1))[0]
        assert bad.size == 0, f"{bad.size} of {got.shape[0]} blocks differ, first {bad[:8]}"
