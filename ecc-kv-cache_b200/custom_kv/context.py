"""context.py -- ``ecc_cache()`` context manager (custom_kv/context.py:19 of the
reference): allocate the cache, patch SDPA, yield, and always unpatch."""
from contextlib import contextmanager
from typing import Generator, Optional

import torch

from .cache import ErrorCorrectedCache
from .patch import patch_model, unpatch_model


@contextmanager
def ecc_cache(model, batch_size: int = 1, max_cache_len: int = 128_000, device: Optional[str] = None,
              **cache_kwargs) -> Generator[ErrorCorrectedCache, None, None]:
    """Patch ``model`` for ECC-cached inference for the duration of the block.

    Usage::

        with ecc_cache(model, max_cache_len=32768) as cache:
            out = model.generate(**inputs, past_key_values=cache, max_new_tokens=200)

    The SDPA patch is global (not thread-safe).  Extra keyword arguments go to
    ``ErrorCorrectedCache`` (``rotate_values``, ``num_splits``, ``calibration``).
    """
    cache = ErrorCorrectedCache(config=model.config, batch_size=batch_size, max_cache_len=max_cache_len,
                                device=device, **cache_kwargs)
    patch_model(model, cache)
    try:
        yield cache
    finally:
        unpatch_model()
        del cache
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
