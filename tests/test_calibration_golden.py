"""Calibration statistics against the reference's own calibrate_from_model
(fixture tests/golden/calibration_stats_golden.npz, made by
tests/golden/make_calibration_stats_golden.py): the oracle's restatement on
the CPU pins the fixture, and the package's GPU layer_statistics must match
it.  The reference rounds every value to 6 decimals, so matches are within
2e-6 absolute (float32 reductions in another order may move a value across a
rounding boundary)."""
import os

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "calibration_stats_golden.npz"))
LAYERS = sorted(int(k[5:-4]) for k in GOLD.files if k.endswith("_k16"))
C = np.array([-2.4008, -1.8435, -1.4371, -1.0993, -0.7996, -0.5224, -0.2582, 0.0,
              0.2582, 0.5224, 0.7996, 1.0993, 1.4371, 1.8435, 2.4008, 3.1584], np.float32)


def _keys(i):
    return GOLD[f"layer{i}_k16"].view(np.float16).astype(np.float32)


def _oracle_stats(oracle, k):
    """custom_kv/calibration.py:214-237 restated: full-row WHT (oracle C),
    unbiased std and mean, fp32 quantiser reconstruction, mean |residual|."""
    xr = oracle.wht(k).astype(np.float32)
    sigma = float(xr.astype(np.float64).std(ddof=1))
    mean = float(xr.astype(np.float64).mean())
    s32, z32 = np.float32(sigma), np.float32(mean)
    u = ((xr - z32) / s32).astype(np.float32)
    q = np.abs(u[..., None] - C).argmin(-1)
    recon = (C[q] * s32).astype(np.float32) + z32
    alpha = float(np.abs(xr - recon.astype(np.float32)).astype(np.float64).mean())
    return np.array([sigma, mean, alpha, sigma])


@pytest.mark.parametrize("layer", LAYERS)
def test_oracle_matches_reference_statistics(oracle, layer):
    ref = GOLD[f"layer{layer}_stats"]
    got = _oracle_stats(oracle, _keys(layer))
    assert np.all(np.abs(np.round(got, 6) - ref) <= 2e-6), (got, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("layer", LAYERS)
def test_layer_statistics_match_reference(cuda_device, layer):
    from custom_kv.calibration import layer_statistics
    st = layer_statistics(torch.from_numpy(_keys(layer)), head_dim=128)
    got = np.array([st["scale"], st["zero"], st["alpha"], st["sigma"]])
    ref = GOLD[f"layer{layer}_stats"]
    assert np.all(np.abs(np.round(got, 6) - ref) <= 2e-6), (got, ref)


@pytest.mark.gpu
def test_per_head_statistics_are_the_per_vector_rotation(oracle, cuda_device):
    """per_head=True rotates each 128-dim vector (the cache's rotation)."""
    from custom_kv.calibration import layer_statistics
    k = _keys(1)
    st = layer_statistics(torch.from_numpy(k), head_dim=128, per_head=True)
    xr = oracle.wht(k.reshape(-1, 128)).astype(np.float64)
    assert abs(st["sigma"] - xr.std(ddof=1)) <= 1e-5 * xr.std(ddof=1)
    assert abs(st["zero"] - xr.mean()) <= 1e-5
    full = layer_statistics(torch.from_numpy(k), head_dim=128)
    assert full["sigma"] != st["sigma"] and full["alpha"] != st["alpha"]  # the two rotations differ
