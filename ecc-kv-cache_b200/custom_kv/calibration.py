"""calibration.py -- per-layer key statistics for calibrated quantisation, in
the reference's JSON format (custom_kv/calibration.py:11-20, :243-249):

    {"model_id": ..., "n_samples": N, "max_length": M,
     "layers": {"0": {"scale": s, "zero": z, "alpha": a, "sigma": s}, ...}}

Three steps:

1. ``ProjectionSampler`` -- a context manager that taps the k_proj / v_proj
   output of every attention module (modules are found by their ``layer_idx``
   attribute) and keeps a random sample of up to ``rows_per_pass`` rows of each
   output per forward pass, on the host in fp32.  The reference samples 1000
   rows per pass the same way (custom_kv/calibration.py:117-130).
2. ``layer_statistics`` -- one layer's statistics from its sampled key rows
   k [N, Hkv*head_dim].  Default (``per_head=False``) is what the reference's
   calibrate_from_model computes (custom_kv/calibration.py:214-237): the
   normalised WHT of each whole row (length Hkv*head_dim), sigma = unbiased
   std and mean of all rotated values, scale = sigma, zero = mean, and alpha =
   mean |x - k~| with k~ the 16-level reconstruction (ops_cpu.py:78-109) under
   that scale and zero.  ``per_head=True`` rotates every head_dim vector on
   its own instead -- the rotation the cache applies to the keys it stores, so
   those statistics describe the values the calibrated quantiser actually
   sees; it is an option because its numbers differ from the reference's.
   The WHT runs on the GPU (custom_ecc_cuda.hadamard_rotate, bit-exact with
   hadamard_rotate_cpu); the reductions are torch's GPU reductions, so the
   statistics agree with the reference's CPU ones to float32 rounding.
3. ``calibrate_from_model`` -- runs 1 and 2 over texts and writes the JSON.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Dict, Iterable, List, Optional, Sequence, Union

import torch

# the 16-level table of custom_kv/ops_cpu.py:19-24 (float32)
_LEVELS = (-2.4008, -1.8435, -1.4371, -1.0993, -0.7996, -0.5224, -0.2582, 0.0,
           0.2582, 0.5224, 0.7996, 1.0993, 1.4371, 1.8435, 2.4008, 3.1584)


def lloyd_max_gaussian(n_levels: int = 16, sigma: float = 1.0, n_iter: int = 100) -> List[float]:
    """Lloyd-Max quantiser levels for N(0, sigma^2): alternate the centroid
    condition (each level is the conditional mean of its cell) and the
    nearest-neighbour condition (boundaries at midpoints), starting from the
    equal-probability partition, until the levels move less than 1e-6."""
    import numpy as np
    from scipy import stats

    edges = stats.norm.ppf(np.linspace(0.0, 1.0, n_levels + 1)[1:-1], scale=sigma)
    levels = np.zeros(n_levels)
    for _ in range(n_iter):
        b = np.concatenate([[-np.inf], edges, [np.inf]]) / sigma
        mass = stats.norm.cdf(b[1:]) - stats.norm.cdf(b[:-1])
        dens = stats.norm.pdf(b[:-1]) - stats.norm.pdf(b[1:])
        new = np.where(mass < 1e-10, 0.5 * (b[:-1] + b[1:]) * sigma, sigma * dens / np.maximum(mass, 1e-300))
        converged = np.max(np.abs(new - levels)) < 1e-6
        levels = new
        edges = 0.5 * (levels[:-1] + levels[1:])
        if converged:
            break
    return levels.tolist()


# --------------------------------------------------------------------------
# 1. sampling of the projection outputs
# --------------------------------------------------------------------------
class ProjectionSampler:
    """Samples rows of every attention layer's k_proj and v_proj output.

    Usage::

        with ProjectionSampler(model) as tap:
            for batch in batches:
                model(**batch)
        keys = tap.rows("k")    # {layer: [N, Hkv*head_dim] fp32 CPU tensor}

    Every forward pass contributes min(rows_per_pass, rows of the output)
    rows per layer, drawn without replacement with the sampler's seeded
    generator.
    """

    def __init__(self, model, rows_per_pass: int = 1000, seed: int = 0):
        self.model = model
        self.rows_per_pass = int(rows_per_pass)
        self.seed = int(seed)
        self._gen: Dict[torch.device, torch.Generator] = {}
        self._store: Dict[str, Dict[int, List[torch.Tensor]]] = {"k": {}, "v": {}}
        self._handles: List = []

    def _generator(self, device: torch.device) -> torch.Generator:
        g = self._gen.get(device)
        if g is None:
            g = torch.Generator(device=device)
            g.manual_seed(self.seed)
            self._gen[device] = g
        return g

    def _tap(self, which: str, layer: int):
        def on_output(module, inputs, output):
            flat = output.detach().reshape(-1, output.shape[-1])
            n = flat.shape[0]
            take = min(self.rows_per_pass, n)
            pick = torch.randperm(n, generator=self._generator(flat.device), device=flat.device)[:take]
            self._store[which].setdefault(layer, []).append(flat.index_select(0, pick).float().cpu())
        return on_output

    def __enter__(self) -> "ProjectionSampler":
        found = 0
        for module in self.model.modules():
            layer = getattr(module, "layer_idx", None)
            if not isinstance(layer, int):
                continue
            kp, vp = getattr(module, "k_proj", None), getattr(module, "v_proj", None)
            if kp is None or vp is None:
                continue
            self._handles.append(kp.register_forward_hook(self._tap("k", layer)))
            self._handles.append(vp.register_forward_hook(self._tap("v", layer)))
            found += 1
        if not found:
            raise RuntimeError("ProjectionSampler: no attention module with layer_idx, k_proj and v_proj found")
        return self

    def __exit__(self, *exc) -> None:
        while self._handles:
            self._handles.pop().remove()

    def rows(self, which: str = "k") -> Dict[int, torch.Tensor]:
        """{layer index: sampled rows [N, features]} for "k" or "v"."""
        return {layer: torch.cat(parts) for layer, parts in sorted(self._store[which].items())}


def _encode(tokenizer, text: str, max_length: int, device: torch.device) -> Dict[str, torch.Tensor]:
    enc = tokenizer(text, return_tensors="pt", max_length=max_length, truncation=True)
    items = enc.items() if hasattr(enc, "items") else dict(enc).items()
    return {name: (val.to(device) if isinstance(val, torch.Tensor) else val) for name, val in items}


# --------------------------------------------------------------------------
# 2. statistics of one layer
# --------------------------------------------------------------------------
def _wht_rows(x: torch.Tensor, width: int) -> torch.Tensor:
    """Normalised WHT of every run of ``width`` values of x [N, F] (fp32, GPU)."""
    import custom_ecc_cuda as ops

    if width & (width - 1) or not 1 <= width <= 1024:
        raise RuntimeError(f"the WHT width must be a power of two up to 1024, got {width}")
    y = x.reshape(-1, width).contiguous()
    ops.hadamard_rotate(y)
    return y.reshape(x.shape)


def layer_statistics(k: torch.Tensor, head_dim: int = 128, per_head: bool = False,
                     device: Optional[torch.device] = None) -> Dict[str, float]:
    """Calibration statistics {scale, zero, alpha, sigma} of one layer's key
    rows k [N, Hkv*head_dim].  ``per_head=False`` (the reference's
    statistics): WHT over each whole row; ``per_head=True``: WHT over each
    head_dim vector."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    x = k.to(dev, torch.float32)
    if x.dim() != 2:
        raise RuntimeError(f"k must be [N, features], got {tuple(k.shape)}")
    width = head_dim if per_head else x.shape[1]
    if x.shape[1] % width:
        raise RuntimeError(f"rows of {x.shape[1]} values do not split into heads of {head_dim}")
    xr = _wht_rows(x, width)
    sigma = xr.std().item()
    mean = xr.mean().item()
    # the reconstruction of ops_cpu.lloyd_max_quantize_cpu with the scalars
    # rounded to float32 (torch's cast of a Python scalar operand)
    levels = torch.tensor(_LEVELS, dtype=torch.float32, device=dev)
    sc = torch.tensor(sigma, dtype=torch.float32, device=dev)
    zr = torch.tensor(mean, dtype=torch.float32, device=dev)
    abs_sum = torch.zeros((), dtype=torch.float64, device=dev)
    for part in xr.reshape(-1).split(1 << 20):
        u = (part - zr) / sc
        code = (u[:, None] - levels).abs().argmin(-1)
        recon = levels[code] * sc + zr
        abs_sum += (part - recon).abs().double().sum()
    alpha = abs_sum.item() / xr.numel()
    return {"scale": sigma, "zero": mean, "alpha": alpha, "sigma": sigma}


# --------------------------------------------------------------------------
# 3. the whole calibration
# --------------------------------------------------------------------------
def read_texts(source: Union[str, Path, None], limit: int, max_chars: int = 4000) -> List[str]:
    """Texts for calibration from a directory of .txt files (sorted by name,
    one text per file) or a single .txt file (one text per blank-line
    separated paragraph); each cut to ``max_chars`` characters.  There is no
    download fallback: pass ``texts=`` to calibrate_from_model instead."""
    if source is None:
        return []
    path = Path(source)
    if path.is_dir():
        chunks: Iterable[str] = (f.read_text(encoding="utf-8") for f in sorted(path.glob("*.txt")))
    elif path.is_file():
        chunks = (p for p in path.read_text(encoding="utf-8").split("\n\n") if p.strip())
    else:
        return []
    out: List[str] = []
    for text in chunks:
        if len(out) >= limit:
            break
        out.append(text[:max_chars])
    return out


def calibrate_from_model(model, tokenizer, calibration_data_path: Optional[str] = None,
                         texts: Optional[Sequence[str]] = None, n_samples: int = 512, max_length: int = 2048,
                         output_path: Optional[str] = None, per_head: bool = False, rows_per_pass: int = 1000,
                         seed: int = 0) -> Dict[str, Any]:
    """Per-layer calibration config from ``model`` run over texts (a list, or
    a directory / file read by ``read_texts``); written as JSON to
    ``output_path`` when given.  Values are rounded to 6 decimals as the
    reference's are.  ``per_head`` selects the per-head statistics (see the
    module docstring)."""
    if texts is None:
        texts = read_texts(calibration_data_path, n_samples)
    texts = list(texts)[:n_samples]
    if not texts:
        raise RuntimeError("calibrate_from_model: no calibration texts")
    device = next(model.parameters()).device
    model.eval()
    with torch.no_grad(), ProjectionSampler(model, rows_per_pass=rows_per_pass, seed=seed) as tap:
        for text in texts:
            model(**_encode(tokenizer, text, max_length, device))
    cfg = model.config
    head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    layers = {}
    for layer, k in tap.rows("k").items():
        stats = layer_statistics(k, head_dim=head_dim, per_head=per_head)
        layers[str(layer)] = {name: round(val, 6) for name, val in stats.items()}
    config = {"model_id": getattr(cfg, "_name_or_path", ""), "n_samples": n_samples, "max_length": max_length,
              "layers": layers}
    if per_head:
        config["rotation"] = "per_head"
    if output_path:
        out = Path(output_path)
        out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(json.dumps(config, indent=2))
    return config


def load_calibration_config(path: str) -> Dict[str, Any]:
    """Load a saved calibration config (custom_kv/calibration.py:288)."""
    with open(path) as f:
        return json.load(f)
