"""Golden fixtures of the calibrated compress (fixed per-layer quantiser
parameters), made by running the REFERENCE's own CPU code: for each input row
x and parameter triple (scale, zero, alpha),

    x_rot    = ops_cpu.hadamard_rotate_cpu(x.float())        (rotate=True rows)
    q, k~    = ops_cpu.lloyd_max_quantize_cpu(x_rot, scale, zero)
    syndrome = ops_cpu.compute_syndrome_cpu(x_rot - k~)

packed in the block layout of csrc/ecc_ops.h:22-64 with fp16(fp32(scale)),
fp16(fp32(zero)), fp16(fp32(alpha)) (how the reference cache stores meta,
custom_kv/cache.py:180).  The parameter triples have the form of
custom_kv/calibration.py:232-237 (6-decimal per-layer values).  Run once in a
checkout that has the reference:

    python tests/golden/make_calibrated_golden.py --reference /path/to/ecc-kv-cache
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import workloads  # noqa: E402
from make_golden import pack  # noqa: E402

D = 128
# (scale, zero, alpha): a layer near the inputs' own spread, a narrow one (most
# values far outside the centroid range), a wide one, an offset one
PARAMS = [(0.998123, 0.004127, 0.197531), (0.052341, -0.031, 0.0123), (7.25, 0.5, 1.1), (1.3, -2.75, 0.25)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ECC_KV_REFERENCE"),
                    help="checkout of the reference project (or set ECC_KV_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or ECC_KV_REFERENCE) is required")
    sys.path.insert(0, os.path.abspath(args.reference))
    from custom_kv import ops_cpu

    x16 = torch.cat([workloads.make_c1(seed=41, L=48)[0].reshape(-1, D)[:96],
                     workloads.make_heavy(seed=42, n=96),
                     workloads.make_edge()])
    n = x16.shape[0]
    out = {"x16": x16.numpy().view(np.uint16), "params": np.array(PARAMS, np.float64)}
    for pi, (scale, zero, alpha) in enumerate(PARAMS):
        for rotate in (True, False):
            q = np.zeros((n, D), np.uint8)
            syn = np.zeros((n, D), bool)
            for i in range(n):
                x = x16[i].float()
                xr = ops_cpu.hadamard_rotate_cpu(x) if rotate else x
                qi, kt = ops_cpu.lloyd_max_quantize_cpu(xr, scale, zero)
                q[i] = qi.numpy().astype(np.uint8)
                syn[i] = ops_cpu.compute_syndrome_cpu(xr - kt).numpy()
            s32 = np.full(n, scale, np.float64).astype(np.float32)
            z32 = np.full(n, zero, np.float64).astype(np.float32)
            a32 = np.full(n, alpha, np.float64).astype(np.float32)
            out[f"p{pi}_r{int(rotate)}_blocks"] = pack(q, syn, s32, z32, a32)
    np.savez_compressed(os.path.join(HERE, "calibrated_golden.npz"), **out)
    print("wrote calibrated_golden.npz:", n, "rows x", len(PARAMS), "parameter sets x 2")


if __name__ == "__main__":
    main()
