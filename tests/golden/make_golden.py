"""Generate the golden fixtures in this folder by running the REFERENCE's own
CPU code (j-arndt/ecc-kv-cache, custom_kv/ops_cpu.py and
custom_kv/fused_decode.py).  Run once in a checkout that has the reference:

    python tests/golden/make_golden.py --reference /path/to/ecc-kv-cache

The fixtures hold inputs (or the seed that regenerates them) and the
reference's outputs; the tests compare the repo's oracle and CUDA path with
them and never need the reference itself.

Block packing follows csrc/ecc_ops.h:22-64 (the reference has no CPU block
writer): codes byte i = q[2i] | q[2i+1] << 4, syndrome bit j in byte j/8 at
position j%8, fp16(fp32(scale)), fp16(zero), fp16(fp32(alpha)) at 80/82/84.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import multiprocessing as mp
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import workloads  # noqa: E402

D = 128


def pack(q, syn, scale32, zero32, alpha32):
    n = q.shape[0]
    out = np.zeros((n, 128), np.uint8)
    out[:, :64] = q[:, 0::2] | (q[:, 1::2] << 4)
    out[:, 64:80] = np.packbits(syn.reshape(n, 16, 8), axis=-1, bitorder="little").reshape(n, 16)
    meta = np.stack([scale32, zero32, alpha32], axis=1).astype(np.float32).astype(np.float16)
    out[:, 80:86] = meta.view(np.uint8).reshape(n, 6)
    return out


def ref_compress(ops, x16: torch.Tensor, rotate: bool):
    """Reference compress of each row.  rotate=True is ops_cpu.compress_cpu;
    rotate=False runs the same steps (ops_cpu.py:215-219) without the WHT,
    i.e. the arithmetic compress_and_store is documented to perform on an
    already rotated input."""
    n = x16.shape[0]
    xr = np.zeros((n, D), np.float32)
    q = np.zeros((n, D), np.uint8)
    syn = np.zeros((n, D), bool)
    zero = np.zeros(n, np.float32)
    scale = np.zeros(n, np.float32)
    scale64 = np.zeros(n, np.float64)
    alpha = np.zeros(n, np.float32)
    for i in range(n):
        x = x16[i].float()
        if rotate:
            r = ops.compress_cpu(x)
        else:
            x_rot = x
            sc, zr = ops.lloyd_max_params_cpu(x_rot)
            qq, kt = ops.lloyd_max_quantize_cpu(x_rot, sc, zr)
            eps = x_rot - kt
            r = {"x_rot": x_rot, "q": qq, "syndrome": ops.compute_syndrome_cpu(eps),
                 "alpha": eps.abs().mean().item(), "scale": sc, "zero": zr}
        xr[i] = r["x_rot"].numpy()
        q[i] = r["q"].numpy().astype(np.uint8)
        syn[i] = r["syndrome"].numpy()
        zero[i] = np.float32(r["zero"])
        scale[i] = np.float32(r["scale"])
        scale64[i] = r["scale"]
        alpha[i] = np.float32(r["alpha"])
    return dict(x_rot=xr, q=q, syn=syn, zero=zero, scale=scale, scale64=scale64, alpha=alpha,
                blocks=pack(q, syn, scale, zero, alpha))


def _compress_chunk(args):
    ref, x16, rotate = args
    sys.path.insert(0, ref)
    from custom_kv import ops_cpu
    torch.set_num_threads(1)
    return ref_compress(ops_cpu, torch.from_numpy(x16).view(torch.float16), rotate)["blocks"]


def par_compress_blocks(ref, x16: torch.Tensor, rotate: bool, procs: int) -> np.ndarray:
    bits = x16.reshape(-1, D).view(torch.int16).numpy().view(np.uint16)
    chunks = np.array_split(bits, procs * 4)
    with mp.get_context("fork").Pool(procs) as pool:
        parts = pool.map(_compress_chunk, [(ref, c, rotate) for c in chunks])
    return np.concatenate(parts)


def _decode_chunk(args):
    ref, h0, h1, qs, soa = args
    sys.path.insert(0, ref)
    from custom_kv import fused_decode
    torch.set_num_threads(1)
    t = [torch.from_numpy(a) for a in soa]
    q = torch.from_numpy(qs).view(torch.float16)
    L = t[0].shape[2]
    out = fused_decode.cpu_reference_decode(q[:, h0:h1], t[0][:, h0:h1], t[1][:, h0:h1],
                                            t[2][:, h0:h1].view(torch.float16), t[3][:, h0:h1],
                                            t[4][:, h0:h1], t[5][:, h0:h1].view(torch.float16), L)
    return h0, out.numpy()


def ref_decode(ref, q16: torch.Tensor, kblk: np.ndarray, vblk: np.ndarray, procs: int):
    """cpu_reference_decode over query heads; K/V blocks [B,Hkv,L,128] are
    expanded to the query heads with HF repeat_kv (head h reads kv head
    h // (Hq/Hkv)) because the reference kernel has no GQA."""
    B, Hq = q16.shape[0], q16.shape[1]
    Hkv = kblk.shape[1]
    rep = Hq // Hkv
    kb = np.repeat(kblk, rep, axis=1)
    vb = np.repeat(vblk, rep, axis=1)
    soa = [np.ascontiguousarray(kb[..., :64]), np.ascontiguousarray(kb[..., 64:80]),
           np.ascontiguousarray(kb[..., 80:86]).view(np.int16),
           np.ascontiguousarray(vb[..., :64]), np.ascontiguousarray(vb[..., 64:80]),
           np.ascontiguousarray(vb[..., 80:86]).view(np.int16)]
    qs = q16.view(torch.int16).numpy()
    bounds = np.linspace(0, Hq, min(procs, Hq) + 1).astype(int)
    jobs = [(ref, int(bounds[i]), int(bounds[i + 1]), qs, soa) for i in range(len(bounds) - 1)]
    out = np.zeros((B, Hq, 1, D), np.float16)
    with mp.get_context("fork").Pool(len(jobs)) as pool:
        for h0, o in pool.map(_decode_chunk, jobs):
            out[:, h0:h0 + o.shape[1]] = o
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ECC_KV_REFERENCE"),
                    help="checkout of the reference project (or set ECC_KV_REFERENCE)")
    ap.add_argument("--procs", type=int, default=os.cpu_count() or 4)
    ap.add_argument("--skip-c1-decode", action="store_true")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or ECC_KV_REFERENCE) is required")
    ref = os.path.abspath(args.reference)
    sys.path.insert(0, ref)
    from custom_kv import ops_cpu
    torch.set_num_threads(1)
    t0 = time.time()

    # 0. the centroid table itself, bit for bit
    lm_bits = ops_cpu.LM_CENTROIDS_NORM.numpy().view(np.uint32)

    # 1. compress cases (per-vector detail, both rotate modes)
    k1, _, _ = workloads.make_c1(seed=0, L=32)          # 8 heads x 32 tokens = 256 rows
    groups = {
        "c1": k1.reshape(-1, D),
        "heavy": workloads.make_heavy(seed=3, n=256),
        "offset": workloads.make_offset(seed=1, n=128),
        "edge": workloads.make_edge(),
    }
    fx = {"lm_bits": lm_bits}
    for name, x16 in groups.items():
        fx[f"{name}_x16"] = x16.view(torch.int16).numpy().view(np.uint16)
        for rot in (1, 0):
            r = ref_compress(ops_cpu, x16, bool(rot))
            for key, val in r.items():
                fx[f"{name}_r{rot}_{key}"] = val
    np.savez_compressed(os.path.join(HERE, "compress_golden.npz"), **fx)
    print(f"compress cases done ({time.time() - t0:.1f}s)")

    # 2. small decode cases (ragged lengths, GQA groups 1/2/4, B>1)
    cases = [
        dict(seed=11, B=1, hq=4, hkv=4, L=1),
        dict(seed=12, B=2, hq=4, hkv=2, L=37),
        dict(seed=13, B=1, hq=8, hkv=2, L=130),
        dict(seed=14, B=2, hq=8, hkv=2, L=64),
    ]
    dx = {}
    for ci, c in enumerate(cases):
        k16, v16, q16 = workloads.make_c1(seed=c["seed"], B=c["B"], hkv=c["hkv"], hq=c["hq"], L=c["L"])
        kb = ref_compress(ops_cpu, k16.reshape(-1, D), True)["blocks"].reshape(c["B"], c["hkv"], c["L"], 128)
        vb = ref_compress(ops_cpu, v16.reshape(-1, D), True)["blocks"].reshape(c["B"], c["hkv"], c["L"], 128)
        out = ref_decode(ref, q16, kb, vb, args.procs)
        dx[f"case{ci}_kblocks"] = kb
        dx[f"case{ci}_vblocks"] = vb
        dx[f"case{ci}_q16"] = q16.view(torch.int16).numpy().view(np.uint16)
        dx[f"case{ci}_out16"] = out.view(np.uint16)
        dx[f"case{ci}_meta"] = np.array([c["B"], c["hq"], c["hkv"], c["L"]], np.int64)
    np.savez_compressed(os.path.join(HERE, "decode_golden.npz"), **dx)
    print(f"decode cases done ({time.time() - t0:.1f}s)")

    # 3. full single-layer op test (B1, Hq32, Hkv8, L2048): block digests and
    #    the decode output; inputs regenerate from workloads.make_c1(seed=0).
    k16, v16, q16 = workloads.make_c1(seed=0)
    kb = par_compress_blocks(ref, k16, True, args.procs).reshape(1, 8, 2048, 128)
    vb = par_compress_blocks(ref, v16, True, args.procs).reshape(1, 8, 2048, 128)
    c1 = {"k_sha256": hashlib.sha256(kb.tobytes()).hexdigest(),
          "v_sha256": hashlib.sha256(vb.tobytes()).hexdigest()}
    print(f"c1 compress done ({time.time() - t0:.1f}s)")
    if not args.skip_c1_decode:
        out = ref_decode(ref, q16, kb, vb, args.procs)
        np.save(os.path.join(HERE, "c1_decode_out16.npy"), out.view(np.uint16))
        print(f"c1 decode done ({time.time() - t0:.1f}s)")
    with open(os.path.join(HERE, "c1_digest.json"), "w") as f:
        json.dump(c1, f, indent=1)


if __name__ == "__main__":
    main()
