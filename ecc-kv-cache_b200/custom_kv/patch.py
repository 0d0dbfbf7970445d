"""patch.py -- monkey-patches ``F.scaled_dot_product_attention`` so that
single-token (decode) attention runs the fused ECC-INT4 decode kernel over the
active cache's block pools (custom_kv/patch.py:23-117 of the reference).

Prefill (query length > 1): the original SDPA on the fp16 K/V that
``ErrorCorrectedCache.update`` returned.
Decode (query length 1): ``decode_attention`` over the layer's pools -- query
WHT, GQA, online softmax and the output un-rotation happen inside the kernel;
no fp16 copy of the cache is made (the reference dequantised the whole layer
and called SDPA without GQA, custom_kv/patch.py:100-117).
"""
from __future__ import annotations

from typing import TYPE_CHECKING, Optional

import torch
import torch.nn.functional as F

if TYPE_CHECKING:
    from .cache import ErrorCorrectedCache

_original_sdpa = F.scaled_dot_product_attention
_active_cache: Optional["ErrorCorrectedCache"] = None
_current_layer_idx: int = 0
_is_patched: bool = False
_hook_handles = []


def patch_model(model, cache: "ErrorCorrectedCache") -> None:
    """Route decode attention of ``model`` through ``cache`` (global patch, not
    thread-safe, idempotent)."""
    global _active_cache, _is_patched, _current_layer_idx
    if _is_patched:
        return
    _active_cache = cache
    _current_layer_idx = 0
    F.scaled_dot_product_attention = _ecc_sdpa
    _install_layer_hooks(model)
    _is_patched = True


def unpatch_model() -> None:
    """Restore the original SDPA and remove the layer hooks."""
    global _active_cache, _is_patched, _current_layer_idx
    F.scaled_dot_product_attention = _original_sdpa
    _active_cache = None
    _is_patched = False
    _current_layer_idx = 0
    for handle in _hook_handles:
        handle.remove()
    _hook_handles.clear()


def _install_layer_hooks(model) -> None:
    try:
        layers = model.model.layers
    except AttributeError:
        layers = [m for n, m in model.named_modules() if "self_attn" in n and hasattr(m, "q_proj")]

    def make_hook(layer_idx):
        def pre_hook(module, args):
            global _current_layer_idx
            _current_layer_idx = layer_idx
        return pre_hook

    for i, layer in enumerate(layers):
        attn = layer.self_attn if hasattr(layer, "self_attn") else layer
        _hook_handles.append(attn.register_forward_pre_hook(make_hook(i)))


def _ecc_sdpa(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, attn_mask=None, dropout_p: float = 0.0,
              is_causal: bool = False, scale=None, **kwargs) -> torch.Tensor:
    """Patched SDPA: decode queries go to the ECC kernel, the rest to SDPA."""
    if _active_cache is not None and query.dim() == 4 and query.shape[2] == 1:
        return _ecc_decode_step(query, _current_layer_idx, scale)
    return _original_sdpa(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p, is_causal=is_causal,
                          scale=scale, **kwargs)


def _ecc_decode_step(query: torch.Tensor, layer_idx: int, scale: Optional[float] = None) -> torch.Tensor:
    """query [B, Hq, 1, 128] in the model basis -> attention output
    [B, Hq, 1, 128].  The layer is the one whose ``update`` ran last (the HF
    attention calls ``update`` right before SDPA); the pre-hook index is the
    fallback for callers that bypass ``update``."""
    cache = _active_cache
    layer = cache._last_layer if cache._layer_fill[cache._last_layer] > 0 else layer_idx
    return cache.decode_attention(query, layer, sm_scale=scale)
