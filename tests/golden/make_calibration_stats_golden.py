"""Golden fixture of the calibration statistics, made by running the
REFERENCE's own calibrate_from_model (custom_kv/calibration.py:170-257) on
fixed key activations.

The reference collects k_proj outputs with forward hooks and a random row
sample (custom_kv/calibration.py:100-164); to pin the statistics rather than
the sampling, this script hands calibrate_from_model fixed activations (its
_collect_kv_activations is replaced by a function returning them) and a stub
model.  The fixture stores the activations (fp16-valued) and the per-layer
{scale, zero, alpha, sigma} the reference computed from them: WHT of each
whole [Hkv*head_dim] row, std / mean of the rotated values, alpha from
lloyd_max_quantize_cpu, each rounded to 6 decimals.  Run once in a checkout
that has the reference:

    python tests/golden/make_calibration_stats_golden.py --reference /path/to/ecc-kv-cache
    (or set ECC_KV_REFERENCE)
"""
from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import workloads  # noqa: E402

# (rows, features, kind): two Llama-8B-shaped layers (8 kv heads x 128) and a
# 2-kv-head layer
LAYERS = [(64, 1024, "heavy"), (64, 1024, "offset"), (64, 256, "plain")]


def activations(seed: int, rows: int, feats: int, kind: str) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, feats, generator=g)
    if kind == "heavy":  # Student-t(3) on 3 % of the channels, x4 spread on a few more
        ch = torch.randperm(feats, generator=g)[: feats * 3 // 100]
        x[:, ch] = workloads.student_t((rows, ch.numel()), 3, g)
        x[:, torch.randperm(feats, generator=g)[:8]] *= 4.0
    elif kind == "offset":
        x = 0.35 * x + 1.75
    return x.half()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ECC_KV_REFERENCE"),
                    help="checkout of the reference project (or set ECC_KV_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or ECC_KV_REFERENCE) is required")
    sys.path.insert(0, os.path.abspath(args.reference))
    from custom_kv import calibration as ref_cal

    acts16 = [activations(100 + i, *spec) for i, spec in enumerate(LAYERS)]
    layer_kvs = {i: {"k": a.float(), "v": a.float()} for i, a in enumerate(acts16)}
    ref_cal._collect_kv_activations = lambda *a, **k: layer_kvs

    class Stub(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.w = torch.nn.Parameter(torch.zeros(1))
            self.config = types.SimpleNamespace(_name_or_path="stub")

    torch.set_num_threads(1)
    cfg = ref_cal.calibrate_from_model(Stub(), tokenizer=None, texts=["unused"], n_samples=1, max_length=8)
    out = {}
    for i, a in enumerate(acts16):
        out[f"layer{i}_k16"] = a.numpy().view(np.uint16)
        st = cfg["layers"][str(i)]
        out[f"layer{i}_stats"] = np.array([st["scale"], st["zero"], st["alpha"], st["sigma"]], np.float64)
    np.savez_compressed(os.path.join(HERE, "calibration_stats_golden.npz"), **out)
    print("wrote calibration_stats_golden.npz:", {k: v for k, v in cfg["layers"].items()})


if __name__ == "__main__":
    main()
