"""Seeded synthetic workloads with the shapes and value distributions of the
five benchmark configurations (no dataset is involved on this path).

CPU generators use torch's CPU generator, which is deterministic for a given
torch version, so tests can regenerate the exact inputs that the golden
fixtures were made from.  ``*_cuda`` generators draw on the device (same
distributions, different values) for the full-size benchmark inputs.
"""
from __future__ import annotations

import torch

D = 128


def outlier_channels(hkv: int, n: int, g: torch.Generator) -> torch.Tensor:
    """n fixed outlier channels per KV head: [hkv, n] int64."""
    return torch.stack([torch.randperm(D, generator=g)[:n] for _ in range(hkv)])


def make_c1(seed: int = 0, B: int = 1, hkv: int = 8, hq: int = 32, L: int = 2048):
    """Single-layer op test: K, V ~ N(0,1) fp16 with 4 fixed outlier channels
    per KV head scaled x20; query N(0,1) fp16 from seed+1.
    Returns (k [B,hkv,L,128] fp16, v [B,hkv,L,128] fp16, q [B,hq,1,128] fp16)."""
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(B, hkv, L, D, generator=g)
    v = torch.randn(B, hkv, L, D, generator=g)
    ch = outlier_channels(hkv, 4, g)
    for h in range(hkv):
        k[:, h, :, ch[h]] *= 20.0
        v[:, h, :, ch[h]] *= 20.0
    gq = torch.Generator().manual_seed(seed + 1)
    q = torch.randn(B, hq, 1, D, generator=gq)
    return k.half(), v.half(), q.half()


def student_t(shape, df: float, g: torch.Generator, device="cpu") -> torch.Tensor:
    """Student-t draws as Z / sqrt(chi2_df / df) with chi2 from df squared normals
    (df integer)."""
    z = torch.randn(shape, generator=g, device=device)
    chi = torch.zeros(shape, device=device)
    for _ in range(int(df)):
        chi += torch.randn(shape, generator=g, device=device) ** 2
    return z / torch.sqrt(chi / df)


def make_c2(seed: int = 0, B: int = 1, hkv: int = 8, L: int = 131072, device="cpu"):
    """Compress-only throughput: K, V ~ N(0,1) fp16 [B,hkv,L,128]; on 4 of 128
    channels (3 %), fixed per head, values are Student-t(df=3) draws."""
    g = torch.Generator(device=device).manual_seed(seed)
    gc = torch.Generator().manual_seed(seed + 7)
    ch = outlier_channels(hkv, 4, gc)
    out = []
    for _ in range(2):
        x = torch.randn(B, hkv, L, D, generator=g, device=device)
        for h in range(hkv):
            idx = ch[h].to(device)
            x[:, h, :, idx] = student_t((B, L, 4), 3, g, device)
        out.append(x.half())
    return out[0], out[1]


def make_queries(step: int, B: int = 8, hq: int = 32, device="cpu") -> torch.Tensor:
    """Decode-step query: N(0,1) fp16 [B, hq, 1, 128], seed = step."""
    g = torch.Generator(device=device).manual_seed(1000 + step)
    return torch.randn(B, hq, 1, D, generator=g, device=device).half()


def make_heavy(seed: int, n: int):
    """[n,128] fp16 N(0,1) rows with Student-t(df=3) on 4 channels."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, D, generator=g)
    ch = torch.randperm(D, generator=g)[:4]
    x[:, ch] = student_t((n, 4), 3, g)
    return x.half()


def make_offset(seed: int, n: int):
    """Rows whose rotated value has a large mean relative to its spread (the
    case that pins which mean the reference's std uses)."""
    g = torch.Generator().manual_seed(seed)
    base = 30.0 + 0.003 * torch.randn(n, D, generator=g) * torch.rand(n, 1, generator=g)
    # x = H(x_rot_target): H is self-inverse, so rotating x recovers ~base
    x = base.clone()
    s = 1
    while s < D:
        v = x.view(n, D // (2 * s), 2 * s)
        a = v[:, :, :s].clone()
        b = v[:, :, s:].clone()
        v[:, :, :s] = a + b
        v[:, :, s:] = a - b
        s *= 2
    return (x / D ** 0.5).half()


def make_edge() -> torch.Tensor:
    """Hand-made edge rows: zeros, signed zeros, constants, fp16 extremes,
    subnormals, a single spike, alternating signs, exact centroid grids."""
    rows = []
    z = torch.zeros(D)
    rows.append(z.clone())
    nz = torch.full((D,), -0.0)
    rows.append(nz)
    rows.append(torch.ones(D))
    rows.append(torch.full((D,), -3.5))
    rows.append(torch.full((D,), 65504.0))
    m = torch.full((D,), 65504.0)
    m[::2] = -65504.0
    rows.append(m)
    rows.append(torch.full((D,), 2.0 ** -24))          # smallest subnormal
    sub = torch.arange(D, dtype=torch.float32) * 2.0 ** -24
    rows.append(sub)
    spike = torch.zeros(D)
    spike[5] = 100.0
    rows.append(spike)
    spike2 = torch.zeros(D)
    spike2[0] = 50.0
    spike2[1] = -48.0
    rows.append(spike2)
    alt = torch.ones(D)
    alt[1::2] = -1.0
    rows.append(alt)
    rows.append(torch.arange(D, dtype=torch.float32) / 16.0 - 4.0)
    rows.append(torch.linspace(-60000.0, 60000.0, D))
    cgrid = torch.tensor([-2.4008, -1.8435, -1.4371, -1.0993, -0.7996, -0.5224, -0.2582, 0.0,
                          0.2582, 0.5224, 0.7996, 1.0993, 1.4371, 1.8435, 2.4008, 3.1584]).repeat(8)
    rows.append(cgrid)
    rows.append(torch.tensor([1.0, -1.0] * 64) * 1e-3)
    one_hot = torch.zeros(D)
    one_hot[127] = 1.0
    rows.append(one_hot)
    return torch.stack(rows).half()
