"""patch.py -- sends the single-token (decode) attention of a Hugging Face model
to the fused ECC-INT4 decode kernel; ``patch_model`` / ``unpatch_model`` keep
the names and meaning of the reference's custom_kv/patch.py:23-61.

Design.  One ``_DecodeRouter`` instance owns all patch state.  While it is
installed, ``torch.nn.functional.scaled_dot_product_attention`` is the router's
``sdpa`` method:

* a query of length 1 (a decode step) is answered from the cache's block
  pools by ``ErrorCorrectedCache.decode_attention`` -- query WHT, GQA, online
  softmax, output un-rotation and the attention mask (left padding of a
  batch) are handled there; no fp16 copy of the cache is made;
* everything else (prefill) goes to the saved SDPA with its arguments
  untouched.

Which layer a decode call belongs to: Hugging Face attention writes the new
token into the cache (``update``) immediately before it calls SDPA, so the
cache's last updated layer is the layer of the call.  For callers that reach
SDPA without an ``update``, attention modules that carry a ``layer_idx``
attribute (all transformers attention classes do) report their index through a
forward pre-hook; the router uses that hint when the cache has no context for
its last layer.

The patch is process-global (torch's SDPA symbol) and not thread-safe, as in
the reference.
"""
from __future__ import annotations

from typing import TYPE_CHECKING, List, Optional

import torch
import torch.nn.functional as F

if TYPE_CHECKING:
    from .cache import ErrorCorrectedCache


class _DecodeRouter:
    def __init__(self) -> None:
        self.cache: Optional["ErrorCorrectedCache"] = None
        self.saved_sdpa = None
        self.hooks: List = []
        self.layer_hint = 0

    @property
    def active(self) -> bool:
        return self.saved_sdpa is not None

    def install(self, model, cache: "ErrorCorrectedCache") -> None:
        if self.active:  # already installed: keep the first cache, like the reference
            return
        self.cache = cache
        self.layer_hint = 0
        self.saved_sdpa = F.scaled_dot_product_attention
        F.scaled_dot_product_attention = self.sdpa
        for module in _attention_modules(model):
            self.hooks.append(module.register_forward_pre_hook(self._note_layer))

    def remove(self) -> None:
        if self.saved_sdpa is not None:
            F.scaled_dot_product_attention = self.saved_sdpa
        self.saved_sdpa = None
        self.cache = None
        self.layer_hint = 0
        while self.hooks:
            self.hooks.pop().remove()

    def _note_layer(self, module, args) -> None:
        self.layer_hint = int(module.layer_idx)

    def _layer_of_call(self) -> int:
        cache = self.cache
        last = cache._last_layer
        return last if cache._layer_fill[last] > 0 else self.layer_hint

    def sdpa(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, attn_mask=None,
             dropout_p: float = 0.0, is_causal: bool = False, scale=None, **kwargs) -> torch.Tensor:
        if self.cache is not None and query.dim() == 4 and query.shape[2] == 1:
            return self.cache.decode_attention(query, self._layer_of_call(), sm_scale=scale, attn_mask=attn_mask)
        return self.saved_sdpa(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p, is_causal=is_causal,
                               scale=scale, **kwargs)


def _attention_modules(model) -> List[torch.nn.Module]:
    """Attention modules of ``model`` that know their layer index."""
    return [m for m in model.modules() if isinstance(getattr(m, "layer_idx", None), int)
            and any(hasattr(m, name) for name in ("q_proj", "qkv_proj", "query_key_value"))]


_router = _DecodeRouter()


def patch_model(model, cache: "ErrorCorrectedCache") -> None:
    """Route decode attention of ``model`` through ``cache`` (global; a second
    call while patched does nothing)."""
    _router.install(model, cache)


def unpatch_model() -> None:
    """Restore torch's SDPA and remove the layer hooks."""
    _router.remove()


def is_patched() -> bool:
    return _router.active
