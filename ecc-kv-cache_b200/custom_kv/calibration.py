"""calibration.py -- per-layer calibration statistics in the reference's JSON
format (custom_kv/calibration.py:11-20, :243-249):

    {"model_id": ..., "n_samples": N, "max_length": M,
     "layers": {"0": {"scale": s, "zero": z, "alpha": a, "sigma": s}, ...}}

Activations are collected with forward hooks on each layer's k_proj/v_proj
(the reference's approach, :100-164); the rotation and quantisation
statistics run on the GPU through custom_ecc_cuda.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Dict, List, Optional

import torch


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


def _collect_kv_activations(model, tokenizer, texts, max_length: int = 2048, device: str = "cuda") -> Dict[int, dict]:
    """Run ``model`` over ``texts`` and keep up to 1000 random rows of every
    layer's k_proj and v_proj outputs per forward pass (CPU fp32)."""
    num_layers = model.config.num_hidden_layers
    rows: Dict[int, dict] = {i: {"k": [], "v": []} for i in range(num_layers)}
    hooks = []

    def grab(layer_idx: int, which: str):
        def hook(module, inputs, output):
            x = output.detach().float().reshape(-1, output.shape[-1])
            n = min(1000, x.shape[0])
            rows[layer_idx][which].append(x[torch.randperm(x.shape[0], device=x.device)[:n]].cpu())
        return hook

    for i, layer in enumerate(model.model.layers):
        hooks.append(layer.self_attn.k_proj.register_forward_hook(grab(i, "k")))
        hooks.append(layer.self_attn.v_proj.register_forward_hook(grab(i, "v")))
    model.eval()
    try:
        with torch.no_grad():
            for text in texts:
                inputs = tokenizer(text, return_tensors="pt", max_length=max_length, truncation=True)
                if hasattr(inputs, "to"):
                    inputs = inputs.to(device)
                else:
                    inputs = {k: v.to(device) if hasattr(v, "to") else v for k, v in inputs.items()}
                model(**inputs)
    finally:
        for h in hooks:
            h.remove()
    return {i: {"k": torch.cat(r["k"]), "v": torch.cat(r["v"])} for i, r in rows.items() if r["k"]}


def layer_statistics(k: torch.Tensor, head_dim: int = 128, device: Optional[torch.device] = None) -> Dict[str, float]:
    """Calibration statistics of one layer's keys k [N, Hkv*head_dim]: rotate
    every head vector with the WHT (GPU), then sigma/mean of all rotated
    values and alpha = mean |x - Q(x)| under the 16-level table with
    scale = sigma, zero = mean (custom_kv/calibration.py:216-237)."""
    import custom_ecc_cuda as ops

    dev = device or torch.device("cuda", torch.cuda.current_device())
    x = k.to(dev, torch.float32).reshape(-1, head_dim).contiguous()
    ops.hadamard_rotate(x)
    sigma = x.std().item()
    mean = x.mean().item()
    lm = torch.tensor([-2.4008, -1.8435, -1.4371, -1.0993, -0.7996, -0.5224, -0.2582, 0.0,
                       0.2582, 0.5224, 0.7996, 1.0993, 1.4371, 1.8435, 2.4008, 3.1584], device=dev)
    alpha_sum = 0.0
    for chunk in x.split(1 << 16):
        xn = (chunk - mean) / sigma
        q = (xn.unsqueeze(-1) - lm).abs().argmin(-1)
        alpha_sum += (chunk - (lm[q] * sigma + mean)).abs().sum().item()
    return {"scale": sigma, "zero": mean, "alpha": alpha_sum / x.numel(), "sigma": sigma}


def calibrate_from_model(model, tokenizer, calibration_data_path: Optional[str] = None,
                         texts: Optional[List[str]] = None, n_samples: int = 512, max_length: int = 2048,
                         output_path: Optional[str] = None) -> Dict[str, Any]:
    """Per-layer calibration config from a model and texts (a directory of
    .txt files or a list); saved as JSON when ``output_path`` is given."""
    if texts is None:
        texts = _load_calibration_texts(calibration_data_path, n_samples)
    texts = texts[:n_samples]
    device = next(model.parameters()).device
    acts = _collect_kv_activations(model, tokenizer, texts, max_length, str(device))
    head_dim = getattr(model.config, "head_dim", None) or model.config.hidden_size // model.config.num_attention_heads
    layers = {}
    for layer_idx, kv in acts.items():
        st = layer_statistics(kv["k"], head_dim)
        layers[str(layer_idx)] = {k: round(v, 6) for k, v in st.items()}
    config = {"model_id": getattr(model.config, "_name_or_path", ""), "n_samples": n_samples,
              "max_length": max_length, "layers": layers}
    if output_path:
        Path(output_path).parent.mkdir(parents=True, exist_ok=True)
        with open(output_path, "w") as f:
            json.dump(config, f, indent=2)
    return config


def _load_calibration_texts(data_path: Optional[str], n_samples: int) -> List[str]:
    """Up to n_samples texts from the *.txt files of a directory (no network
    fallback)."""
    texts: List[str] = []
    if data_path:
        path = Path(data_path)
        if path.exists():
            for f in sorted(path.glob("*.txt"))[:n_samples]:
                texts.append(f.read_text(encoding="utf-8")[:4000])
    return texts


def load_calibration_config(path: str) -> Dict[str, Any]:
    """Load a saved calibration config (custom_kv/calibration.py:288)."""
    with open(path) as f:
        return json.load(f)
