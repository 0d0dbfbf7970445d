"""custom_kv -- ECC-INT4 KV cache for HF transformers on B200 (sm_100a).

Public API (same names as the reference, custom_kv/__init__.py:11-26):
    ErrorCorrectedCache  -- HF cache of 128-byte ECC_KV_Blocks (pass as past_key_values)
    ecc_cache            -- context manager: allocate, patch SDPA, always unpatch
    patch_model          -- install the decode-attention patch
    unpatch_model        -- restore the original SDPA
    calibrate_from_model -- per-layer calibration statistics (reference JSON format)
    load_calibration_config
"""
from .cache import ErrorCorrectedCache
from .calibration import calibrate_from_model, load_calibration_config
from .context import ecc_cache
from .patch import patch_model, unpatch_model

__version__ = "0.1.0"

__all__ = [
    "ErrorCorrectedCache",
    "ecc_cache",
    "patch_model",
    "unpatch_model",
    "calibrate_from_model",
    "load_calibration_config",
]
