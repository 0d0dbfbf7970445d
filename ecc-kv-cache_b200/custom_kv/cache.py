"""ErrorCorrectedCache -- the HF ``Cache`` of custom_kv/cache.py:24, backed by
layer-dimensioned pools of 128-byte ECC_KV_Blocks and the sm_100a kernels of
libeccb200.so.

Differences from the reference that make it usable end to end:

* one block pool per layer, ``[layers, B, Hkv, max_cache_len, 128]`` uint8 for
  K and for V (the reference's SoA tensors have no layer dimension, so every
  layer overwrote the previous one, custom_kv/cache.py:79-84);
* ``update`` compresses with the fused WHT + Lloyd-Max + syndrome kernel and
  returns real fp16 K/V for prefill attention (the reference returned uint8
  placeholders, custom_kv/cache.py:129-130, which SDPA rejects);
* values are rotated too (``rotate_values=True``); the decode kernel undoes the
  rotation on its output.  ``rotate_values=False`` keeps the reference's
  K-only rotation;
* ``get_mask_sizes`` follows the transformers 5.x contract (past + query).

The reference-shaped SoA attributes ``_k_int4 [B,H,L,64]``, ``_k_syn
[B,H,L,16]``, ``_k_meta [B,H,L,3]`` (and ``_v_*``) are zero-copy views of layer
0's pools.  There is no CPU path: a non-CUDA device raises.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import torch

import custom_ecc_cuda as ops

try:
    from transformers.cache_utils import Cache as _HFCache
    _HF_CACHE_IMPORTED = True
except ImportError:  # pragma: no cover
    _HFCache = object
    _HF_CACHE_IMPORTED = False

BLOCK_BYTES = 128
RECORD96 = 96  # the block without its zero pad sector (bytes 96..127)
HEAD_DIM = 128


def soa_views(pool: torch.Tensor):
    """(int4 [...,64] u8, syn [...,16] u8, meta [...,3] fp16) views of a block
    pool [..., 128] u8 -- the reference's SoA trio, zero-copy."""
    int4 = pool[..., 0:64]
    syn = pool[..., 64:80]
    meta = pool[..., 80:86].view(torch.float16)
    return int4, syn, meta


def pool_of_views(int4: torch.Tensor, syn: torch.Tensor, meta: torch.Tensor) -> Optional[torch.Tensor]:
    """If the SoA trio are views of one block pool (as soa_views makes them),
    return that pool [..., 128] (or [..., 96]) u8 as a view; else None."""
    if int4.dtype != torch.uint8 or syn.dtype != torch.uint8 or meta.dtype != torch.float16:
        return None
    if int4.dim() < 2 or int4.stride(-1) != 1 or int4.stride(-2) not in (BLOCK_BYTES, RECORD96):
        return None
    rb = int4.stride(-2)
    base = int4.data_ptr()
    if syn.data_ptr() != base + 64 or meta.data_ptr() != base + 80:
        return None
    if tuple(syn.stride()[:-1]) != tuple(int4.stride()[:-1]):
        return None
    if tuple(s * 2 for s in meta.stride()[:-1]) != tuple(int4.stride()[:-1]):
        return None
    if syn.shape[:-1] != int4.shape[:-1] or meta.shape[:-1] != int4.shape[:-1]:
        return None
    return torch.as_strided(int4, int4.shape[:-1] + (rb,), int4.stride()[:-1] + (1,))


class ErrorCorrectedCache(_HFCache):
    """Drop-in HF KV cache storing every (layer, token, KV head) as one
    128-byte ECC_KV_Block (INT4 codes + sign syndrome + fp16 scale/zero/alpha).

    Usage::

        with ecc_cache(model, max_cache_len=32768) as cache:
            out = model.generate(**inputs, past_key_values=cache, max_new_tokens=200)

    ``calibration`` (a config of custom_kv/calibration.py, e.g. from
    load_calibration_config): the key blocks of every layer the config lists
    are quantised with that layer's calibrated scale / zero point and store its
    alpha, instead of each vector's own statistics; values keep per-vector
    statistics (the config calibrates keys only).

    ``block_bytes=96`` stores each block without its zero pad sector (bytes
    96..127; codes, syndrome and metadata at the same offsets): a quarter
    less cache memory and decode traffic.  Not the reference's format; the
    decode then always takes the TMA-fed kernel (GQA groups up to 8).
    """

    def __init__(self, config, batch_size: int = 1, max_cache_len: int = 128_000, device: Optional[str] = None,
                 rotate_values: bool = True, num_splits: int = 0, calibration: Optional[dict] = None,
                 block_bytes: int = BLOCK_BYTES):
        try:
            super().__init__()
        except (TypeError, ValueError):
            pass
        # transformers 5.x reads self.layers; an empty list makes generate()
        # take the eager path through update() and the patched SDPA.
        self.layers = []

        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device()) \
            if torch.cuda.is_available() else torch.device("cpu")
        if dev.type != "cuda":
            raise RuntimeError("ErrorCorrectedCache needs a CUDA device: the compressed cache lives in GPU memory "
                               "and is read by the sm_100a kernels (there is no CPU path)")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.config = config
        self.batch_size = int(batch_size)
        self._max_cache_len = int(max_cache_len)
        self._device = dev
        self.num_heads = getattr(config, "num_key_value_heads", None) or config.num_attention_heads
        self.num_attention_heads = config.num_attention_heads
        self.head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        if self.head_dim != HEAD_DIM:
            raise RuntimeError(f"ErrorCorrectedCache stores 128-dim heads (the 128-byte block format); "
                               f"got head_dim={self.head_dim}")
        self._num_layers = int(config.num_hidden_layers)
        if block_bytes not in (BLOCK_BYTES, RECORD96):
            raise RuntimeError(f"block_bytes must be {BLOCK_BYTES} or {RECORD96}, got {block_bytes}")
        if block_bytes == RECORD96 and self.num_attention_heads // self.num_heads > 8:
            raise RuntimeError("96-byte records are read by the TMA-fed decode, which takes GQA groups up to 8")
        self.block_bytes = int(block_bytes)
        self.rotate_values = bool(rotate_values)
        self.num_splits = int(num_splits)
        self.calibration = calibration
        self._seen_tokens = 0
        self._layer_fill: List[int] = [0] * self._num_layers
        self._last_layer = 0
        # device-side lengths (CUDA-graph decode), see enable_device_lengths
        self._dev_mode = False
        self._pos_dev: Optional[torch.Tensor] = None
        self._len_dev: Optional[torch.Tensor] = None
        self._dev_ws: Optional[torch.Tensor] = None
        # attention-mask bookkeeping of decode steps (see _mask_window)
        self._mask_memo = None
        self._last_window = None

        shape = (self._num_layers, self.batch_size, self.num_heads, self._max_cache_len, self.block_bytes)
        self._k_pool = torch.zeros(shape, dtype=torch.uint8, device=dev)
        self._v_pool = torch.zeros(shape, dtype=torch.uint8, device=dev)
        # reference-shaped SoA views (custom_kv/cache.py:79-84), layer 0
        self._k_int4, self._k_syn, self._k_meta = soa_views(self._k_pool[0])
        self._v_int4, self._v_syn, self._v_meta = soa_views(self._v_pool[0])

    # ------------------------------------------------------------------ #
    # pools                                                               #
    # ------------------------------------------------------------------ #
    def layer_pools(self, layer_idx: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """(K pool, V pool) of one layer, each [B, Hkv, max_cache_len, block_bytes] u8."""
        return self._k_pool[layer_idx], self._v_pool[layer_idx]

    def _pool_for_store(self, store: torch.Tensor) -> Tuple[torch.Tensor, int]:
        """Find the pool (and layer) an SoA store view belongs to."""
        ptr = store.data_ptr()
        for pool in (self._k_pool, self._v_pool):
            lo = pool.data_ptr()
            per_layer = pool[0].numel()
            if lo <= ptr < lo + pool.numel():
                layer = (ptr - lo) // per_layer
                return pool[layer], int(layer)
        raise RuntimeError("store is not a view of this cache's block pools")

    # ------------------------------------------------------------------ #
    # HuggingFace Cache API                                               #
    # ------------------------------------------------------------------ #
    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[Dict[str, Any]] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Compress the new K/V of ``layer_idx`` into its pools and return the
        K/V attention should use: the new states themselves when they are the
        whole context (first prefill) or a single decode token (the patched
        SDPA then reads the pools), otherwise the dequantised context
        concatenated with the new states."""
        B, H, L_new, D = key_states.shape
        if D != HEAD_DIM or H != self.num_heads or B != self.batch_size:
            raise RuntimeError(f"update: expected [B={self.batch_size}, H={self.num_heads}, L, 128], "
                               f"got {tuple(key_states.shape)}")
        if not key_states.is_cuda:
            raise RuntimeError("key_states must be a CUDA tensor")
        pos = self._layer_fill[layer_idx]
        if pos + L_new > self._max_cache_len:
            raise RuntimeError(f"cache overflow: {pos + L_new} tokens > max_cache_len {self._max_cache_len}")
        k16 = key_states if key_states.dtype == torch.float16 else key_states.to(torch.float16)
        v16 = value_states if value_states.dtype == torch.float16 else value_states.to(torch.float16)
        kp, vp = self.layer_pools(layer_idx)
        kcal = self._key_calibration(layer_idx)
        if self._dev_mode and L_new == 1:
            self._append_at_device_position(k16, v16, kp, vp, kcal)
        elif kcal is not None:
            ops.compress_calibrated_into(k16, kp, kcal["scale"], kcal["zero"], kcal["alpha"], pos=pos, rotate=True)
            ops.compress_into(v16, vp, pos=pos, rotate=self.rotate_values)
        elif self.rotate_values:
            ops.compress_pair_into(k16, v16, kp, vp, pos=pos, rotate=True)
        else:
            ops.compress_into(k16, kp, pos=pos, rotate=True)
            ops.compress_into(v16, vp, pos=pos, rotate=False)

        self._layer_fill[layer_idx] = pos + L_new
        self._last_layer = layer_idx
        if layer_idx == self._num_layers - 1:
            self._seen_tokens += L_new

        if pos == 0 or L_new == 1:
            return key_states, value_states
        k_old, v_old = self._context_fp16(layer_idx, pos)
        return (torch.cat([k_old.to(key_states.dtype), key_states], dim=-2),
                torch.cat([v_old.to(value_states.dtype), value_states], dim=-2))

    def _context_fp16(self, layer_idx: int, length: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Reconstruction of the first ``length`` tokens in the model's basis."""
        kp, vp = self.layer_pools(layer_idx)
        k = ops.dequantize(kp[:, :, :length].contiguous())
        v = ops.dequantize(vp[:, :, :length].contiguous())
        ops.hadamard_rotate(k.view(-1, HEAD_DIM))
        if self.rotate_values:
            ops.hadamard_rotate(v.view(-1, HEAD_DIM))
        return k, v

    def _rotate(self, x: torch.Tensor) -> torch.Tensor:
        """Normalised WHT of the last dim (a rotated copy; custom_kv/cache.py:132)."""
        y = x.to(torch.float32 if x.dtype not in (torch.float16, torch.float32) else x.dtype).contiguous().clone()
        ops.hadamard_rotate(y.view(-1, y.shape[-1]))
        return y.to(x.dtype)

    # ------------------------------------------------------------------ #
    # device-side lengths: decode steps replayed from a CUDA graph         #
    # ------------------------------------------------------------------ #
    def enable_device_lengths(self, enable: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
        """Single-token updates append at, and decode attention reads up to,
        lengths held in two device int32 counters -- ``pos`` (tokens already
        cached; where the next token goes) and ``len = pos + 1`` -- instead of
        the host-side fill, so that a decode step recorded once in a CUDA graph
        can be replayed while the cache grows.  The counters start at the
        current fill; ``advance_device_lengths()`` (recordable in the graph) or
        ``set_device_lengths(n)`` move them.  Every layer shares them, so all
        layers must hold the same number of tokens.  Returns (pos, len)."""
        if enable:
            fill = self._layer_fill[0]
            if any(f != fill for f in self._layer_fill):
                raise RuntimeError("device-side lengths need every layer at the same length")
            self._pos_dev = torch.full((1,), fill, dtype=torch.int32, device=self._device)
            self._len_dev = torch.full((1,), fill + 1, dtype=torch.int32, device=self._device)
            need = ops.decode_dev_workspace_size(self.batch_size, self.num_attention_heads, self.num_heads,
                                                 self._max_cache_len)
            self._dev_ws = torch.empty(need, dtype=torch.uint8, device=self._device)
        self._dev_mode = bool(enable)
        return self._pos_dev, self._len_dev

    def set_device_lengths(self, n_cached: int) -> None:
        """pos = n_cached, len = n_cached + 1 (stream-ordered device writes)."""
        self._pos_dev.fill_(int(n_cached))
        self._len_dev.fill_(int(n_cached) + 1)

    def advance_device_lengths(self) -> None:
        """pos += 1, len += 1 on the device: the end of one decode step."""
        self._pos_dev.add_(1)
        self._len_dev.add_(1)

    def _append_at_device_position(self, k16, v16, kp, vp, kcal) -> None:
        if kcal is not None:
            ops.compress_calibrated_at(k16, kp, kcal["scale"], kcal["zero"], kcal["alpha"], self._pos_dev, rotate=True)
            ops.compress_pair_at(v16, None, vp, None, self._pos_dev, rotate=self.rotate_values)
        elif self.rotate_values:
            ops.compress_pair_at(k16, v16, kp, vp, self._pos_dev, rotate=True)
        else:
            ops.compress_pair_at(k16, None, kp, None, self._pos_dev, rotate=True)
            ops.compress_pair_at(v16, None, vp, None, self._pos_dev, rotate=False)

    def _key_calibration(self, layer_idx: int) -> Optional[Dict[str, float]]:
        """The calibrated {scale, zero, alpha} of a layer's keys, or None."""
        if not self.calibration:
            return None
        entry = self.calibration.get("layers", {}).get(str(layer_idx))
        if entry is None:
            return None
        return {k: float(entry[k]) for k in ("scale", "zero", "alpha")}

    def _compress(self, x: torch.Tensor, int4_store: torch.Tensor, syn_store: torch.Tensor,
                  meta_store: torch.Tensor, pos: int, L_new: int) -> None:
        """Quantise ``x`` [B, H, L_new, 128] as given (no rotation) into the
        pool behind the SoA stores at positions pos..pos+L_new-1
        (custom_kv/cache.py:136)."""
        pool = pool_of_views(int4_store, syn_store, meta_store)
        if pool is None:
            pool, _ = self._pool_for_store(int4_store)
        x16 = x[:, :, :L_new].to(torch.float16)
        ops.compress_into(x16, pool, pos=pos, rotate=False)

    def _dequantize(self, int4: torch.Tensor, syn: torch.Tensor, meta: torch.Tensor) -> torch.Tensor:
        """Reconstruct fp16 ``(C[q]*scale + zero) + alpha*s`` from the SoA trio
        (views of a pool or standalone tensors), in the stored basis
        (custom_kv/cache.py:204)."""
        pool = pool_of_views(int4, syn, meta)
        blocks = pool.contiguous() if pool is not None else ops.pack_soa(int4, syn, meta)
        return ops.dequantize(blocks)

    def get_kv_fp16_for_layer(self, layer_idx: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Reconstructed (K, V) [B, H, L, 128] fp16 of a layer in the stored
        (rotated) basis, as custom_kv/cache.py:187 returns them."""
        L = self._layer_fill[layer_idx]
        kp, vp = self.layer_pools(layer_idx)
        return ops.dequantize(kp[:, :, :L].contiguous()), ops.dequantize(vp[:, :, :L].contiguous())

    def decode_attention(self, query: torch.Tensor, layer_idx: int, sm_scale: Optional[float] = None,
                         attn_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One decode step of attention of ``query`` [B, Hq, 1, 128] over the
        compressed context of ``layer_idx`` (the new token already appended).

        ``attn_mask``: the SDPA mask of the step ([B, 1, 1, kv_len] or [B,
        kv_len], bool with True = attend, or additive float), or None.  Left
        padding (each sequence attends to a suffix of the context, as batched
        ``generate()`` with a left-padded prompt produces) runs the fused
        kernel with a per-sequence start; a mask of any other shape of
        attended positions takes the reconstructed context and the masked
        SDPA.  The mask is read once per forward pass (every layer gets the
        same tensor)."""
        kp, vp = self.layer_pools(layer_idx)
        q16 = query if query.dtype == torch.float16 else query.to(torch.float16)
        if self._dev_mode:
            # device-side lengths (CUDA-graph replay): the mask is not read
            # while recording; GraphDecoder refuses padded batches
            out = ops.decode_attention_dev(q16, kp, vp, self._len_dev, sm_scale=sm_scale, rotate_q=True,
                                           unrotate_out=self.rotate_values, workspace=self._dev_ws)
            return out if query.dtype == torch.float16 else out.to(query.dtype)
        fill = self._layer_fill[layer_idx]
        window = self._mask_window(attn_mask, fill) if attn_mask is not None else None
        if window is None:
            out = ops.decode_attention(q16, kp, vp, seq_len=fill, sm_scale=sm_scale, rotate_q=True,
                                       unrotate_out=self.rotate_values, num_splits=self.num_splits)
        elif isinstance(window, torch.Tensor) and self.num_attention_heads // self.num_heads <= 8:
            out = ops.decode_attention_masked(q16, kp, vp, seq_len=fill, start=window, sm_scale=sm_scale,
                                              rotate_q=True, unrotate_out=self.rotate_values)
        else:
            out = self._masked_sdpa(q16, layer_idx, fill, attn_mask, sm_scale)
        return out if query.dtype == torch.float16 else out.to(query.dtype)

    def _mask_window(self, attn_mask: torch.Tensor, fill: int):
        """None when the mask attends to every cached token; an int32 [B]
        device tensor of first attended positions when every sequence attends
        to a suffix of the context (left padding); False otherwise.  Cached per
        mask tensor and length, so one forward pass reads the mask once."""
        key = (attn_mask.data_ptr(), tuple(attn_mask.shape), attn_mask.dtype, fill)
        hit = self._mask_memo
        if hit is not None and hit[0] == key:
            return hit[1]
        m = attn_mask
        if m.dim() == 4:
            m = m[:, 0, -1, :]
        elif m.dim() != 2:
            raise RuntimeError(f"decode attention mask must be [B, 1, 1, L] or [B, L], got {tuple(attn_mask.shape)}")
        if m.shape[0] not in (1, self.batch_size) or m.shape[-1] < fill:
            raise RuntimeError(f"decode attention mask {tuple(attn_mask.shape)} does not cover the batch of "
                               f"{self.batch_size} and the {fill} cached tokens")
        attend = m[:, :fill] if m.dtype == torch.bool else m[:, :fill] > torch.finfo(m.dtype).min / 2
        attend = attend.expand(self.batch_size, fill)
        any_ = attend.any(-1)
        first = torch.where(any_, attend.int().argmax(-1), torch.full_like(any_, fill, dtype=torch.int64))
        suffix = attend.sum(-1) == fill - first
        padded, is_suffix = torch.stack([(first > 0).any(), suffix.all()]).tolist()
        if not is_suffix:
            window = False
        elif not padded:
            window = None
        else:
            window = first.to(torch.int32).contiguous()
        self._mask_memo = (key, window)
        self._last_window = window
        return window

    def _masked_sdpa(self, q16: torch.Tensor, layer_idx: int, fill: int, attn_mask: torch.Tensor,
                     sm_scale: Optional[float]) -> torch.Tensor:
        """Decode under an arbitrary mask: the layer's context reconstructed
        on the GPU (dequantise kernel + inverse WHT) and torch's masked SDPA."""
        k, v = self._context_fp16(layer_idx, fill)
        mask = attn_mask[..., :fill]
        if mask.dim() == 2:
            mask = mask[:, None, None, :]
        return torch.nn.functional.scaled_dot_product_attention(q16, k, v, attn_mask=mask, scale=sm_scale,
                                                                enable_gqa=self.num_attention_heads != self.num_heads)

    # ------------------------------------------------------------------ #
    # HuggingFace Cache protocol                                          #
    # ------------------------------------------------------------------ #
    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self._layer_fill[layer_idx]

    def get_max_cache_shape(self, layer_idx: int = 0) -> int:
        return self._max_cache_len

    @property
    def is_compileable(self) -> bool:
        """Runtime SDPA patching is not torch.compile-compatible."""
        return False

    @property
    def is_initialized(self) -> bool:
        return True

    @property
    def is_sliding(self) -> List[bool]:
        return [False] * self._num_layers

    @property
    def max_batch_size(self) -> int:
        return self.batch_size

    @property
    def max_cache_len(self) -> int:
        return self._max_cache_len

    def __len__(self) -> int:
        return self._num_layers

    def get_mask_sizes(self, query_length, layer_idx: int = 0) -> tuple:
        """(kv_length, kv_offset) for mask construction: the cached length plus
        the query length, offset 0 (transformers 5.x layer contract)."""
        if isinstance(query_length, torch.Tensor):
            query_length = int(query_length.shape[0]) if query_length.dim() > 0 else int(query_length)
        return (self.get_seq_length(layer_idx) + int(query_length), 0)

    def reset(self) -> None:
        self._layer_fill = [0] * self._num_layers
        self._seen_tokens = 0
        self._mask_memo = None
        self._last_window = None

    def crop(self, max_length: int) -> None:
        if max_length < 0:
            max_length = max(0, max(self._layer_fill) + max_length)
        for i in range(self._num_layers):
            self._layer_fill[i] = min(self._layer_fill[i], max_length)
        self._seen_tokens = min(self._seen_tokens, max_length)

    def batch_select_indices(self, indices: torch.Tensor) -> None:
        idx = indices.to(self._device)
        self._k_pool = self._k_pool.index_select(1, idx).contiguous()
        self._v_pool = self._v_pool.index_select(1, idx).contiguous()
        self.batch_size = int(idx.numel())
        self._k_int4, self._k_syn, self._k_meta = soa_views(self._k_pool[0])
        self._v_int4, self._v_syn, self._v_meta = soa_views(self._v_pool[0])

    def reorder_cache(self, beam_idx: torch.LongTensor) -> None:
        idx = beam_idx.to(self._device)
        self._k_pool.copy_(self._k_pool.index_select(1, idx))
        self._v_pool.copy_(self._v_pool.index_select(1, idx))

    @property
    def seen_tokens(self) -> int:
        return self._seen_tokens

    def get_usable_length(self, new_seq_length: int, layer_idx: int = 0) -> int:
        return self._layer_fill[layer_idx]

    def get_max_length(self):
        return self._max_cache_len

    def memory_bytes(self) -> dict:
        """Pool bytes and the fp16 cache they replace (256 B per token-head)."""
        total = self._k_pool.numel() + self._v_pool.numel()
        fp16 = 2 * self._num_layers * self.batch_size * self.num_heads * self._max_cache_len * HEAD_DIM * 2
        return {"cache_bytes": total, "cache_gb": total / 1e9, "fp16_equivalent_gb": fp16 / 1e9,
                "compression_ratio": fp16 / total if total else 0.0}

    def __repr__(self) -> str:
        mem = self.memory_bytes()
        return (f"ErrorCorrectedCache(seq_len={self._seen_tokens}, max_len={self._max_cache_len}, "
                f"layers={self._num_layers}, vram={mem['cache_gb']:.2f}GB, "
                f"compression={mem['compression_ratio']:.1f}x)")
