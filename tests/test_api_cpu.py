"""Host-side logic of the Python API that needs no GPU: construction errors
(no CPU path), the SDPA patch lifecycle, calibration hooks and format."""
import json
import types

import pytest
import torch
import torch.nn.functional as F


class FakeConfig:
    num_hidden_layers = 32
    num_attention_heads = 32
    num_key_value_heads = 8
    hidden_size = 4096
    head_dim = 128
    _name_or_path = "random-init/llama-3.1-8b-shape"


def test_package_imports_and_api_surface():
    import custom_kv
    for name in ("ErrorCorrectedCache", "ecc_cache", "patch_model", "unpatch_model", "calibrate_from_model",
                 "load_calibration_config"):
        assert hasattr(custom_kv, name)
    import custom_ecc_cuda
    for name in ("hadamard_rotate", "compress_and_store", "get_block_metadata"):
        assert callable(getattr(custom_ecc_cuda, name))


def test_cache_refuses_cpu_device():
    from custom_kv import ErrorCorrectedCache
    with pytest.raises(RuntimeError, match="CUDA"):
        ErrorCorrectedCache(FakeConfig(), batch_size=1, max_cache_len=64, device="cpu")


def test_cache_subclasses_hf_cache():
    from transformers.cache_utils import Cache
    from custom_kv import ErrorCorrectedCache
    assert issubclass(ErrorCorrectedCache, Cache)


def test_ops_reject_cpu_tensors():
    import custom_ecc_cuda as ops
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        ops.hadamard_rotate(torch.zeros(4, 128))
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        ops.compress_and_store(torch.zeros(4, 128, dtype=torch.float16), torch.zeros(4, 128, dtype=torch.uint8))
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        ops.get_block_metadata(torch.zeros(4, 128, dtype=torch.uint8), 0)


def test_patch_and_unpatch_restore_sdpa():
    from custom_kv import patch_model, unpatch_model
    from custom_kv import patch as P

    class Attn(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = torch.nn.Linear(4, 4)

    class Layer(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.self_attn = Attn()

    model = types.SimpleNamespace(model=types.SimpleNamespace(layers=[Layer(), Layer()]))
    original = F.scaled_dot_product_attention
    for _ in range(3):
        patch_model(model, cache=object())
        assert F.scaled_dot_product_attention is not original
        patch_model(model, cache=object())  # idempotent
        unpatch_model()
        assert F.scaled_dot_product_attention is original
        assert not P._hook_handles


def test_patched_sdpa_passes_prefill_through():
    from custom_kv import patch as P
    P._active_cache = None
    q = torch.randn(1, 2, 3, 8)
    assert torch.allclose(P._ecc_sdpa(q, q, q, is_causal=True), P._original_sdpa(q, q, q, is_causal=True))


def test_calibration_hooks_capture_all_layers():
    """Mirrors the reference's hook test (tests/integration/test_colab_compat.py:256)."""
    from custom_kv.calibration import _collect_kv_activations
    n_layers, d_model, d_kv = 4, 64, 32

    class SA(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.k_proj = torch.nn.Linear(d_model, d_kv, bias=False)
            self.v_proj = torch.nn.Linear(d_model, d_kv, bias=False)

    class L(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.self_attn = SA()

        def forward(self, x):
            self.self_attn.k_proj(x)
            self.self_attn.v_proj(x)
            return x

    class Top(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.config = types.SimpleNamespace(num_hidden_layers=n_layers)
            self.model = torch.nn.Module()
            self.model.layers = torch.nn.ModuleList([L() for _ in range(n_layers)])

        def forward(self, input_ids=None, **kw):
            x = torch.randn(1, input_ids.shape[1], d_model)
            for layer in self.model.layers:
                x = layer(x)
            return x

    def tok(text, return_tensors=None, max_length=None, truncation=None):
        return {"input_ids": torch.randint(0, 100, (1, min(len(text.split()), max_length or 32)))}

    res = _collect_kv_activations(Top(), tok, ["hello world " * 20] * 3, max_length=32, device="cpu")
    assert len(res) == n_layers
    for i in range(n_layers):
        assert res[i]["k"].shape[-1] == d_kv and res[i]["v"].shape[-1] == d_kv


def test_lloyd_max_gaussian_is_symmetric_and_sorted():
    from custom_kv.calibration import lloyd_max_gaussian
    c = lloyd_max_gaussian(16)
    assert len(c) == 16 and all(a < b for a, b in zip(c, c[1:]))
    assert abs(c[0] + c[-1]) < 1e-4 and abs(c[-1] - 2.733) < 0.02


def test_calibration_config_roundtrip(tmp_path):
    from custom_kv import load_calibration_config
    cfg = {"model_id": "x", "n_samples": 2, "max_length": 16,
           "layers": {"0": {"scale": 1.0, "zero": 0.0, "alpha": 0.1, "sigma": 1.0}}}
    p = tmp_path / "cal.json"
    p.write_text(json.dumps(cfg))
    assert load_calibration_config(str(p)) == cfg
