"""Host-side logic of the Python API that needs no GPU: construction errors
(no CPU path), the SDPA patch lifecycle, calibration sampling and format."""
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


class _Attn(torch.nn.Module):
    """Stand-in for a transformers attention module: layer_idx and projections."""

    def __init__(self, layer_idx, d_model=4, d_kv=4):
        super().__init__()
        self.layer_idx = layer_idx
        self.q_proj = torch.nn.Linear(d_model, d_kv, bias=False)
        self.k_proj = torch.nn.Linear(d_model, d_kv, bias=False)
        self.v_proj = torch.nn.Linear(d_model, d_kv, bias=False)

    def forward(self, x):
        self.k_proj(x)
        self.v_proj(x)
        return x


class _Model(torch.nn.Module):
    def __init__(self, n_layers=2, d_model=4, d_kv=4):
        super().__init__()
        self.d_model = d_model
        self.config = types.SimpleNamespace(num_hidden_layers=n_layers, hidden_size=d_model,
                                            num_attention_heads=1, head_dim=d_kv)
        self.layers = torch.nn.ModuleList([_Attn(i, d_model, d_kv) for i in range(n_layers)])

    def forward(self, input_ids=None, **kw):
        x = torch.randn(1, input_ids.shape[1], self.d_model)
        for layer in self.layers:
            x = layer(x)
        return x


def test_patch_and_unpatch_restore_sdpa():
    from custom_kv import patch_model, unpatch_model
    from custom_kv import patch as P
    model = _Model()
    original = F.scaled_dot_product_attention
    for _ in range(3):
        patch_model(model, cache=object())
        assert F.scaled_dot_product_attention is not original and P.is_patched()
        assert len(P._router.hooks) == 2  # one pre-hook per attention module
        patch_model(model, cache=object())  # a second call while patched does nothing
        assert len(P._router.hooks) == 2
        unpatch_model()
        assert F.scaled_dot_product_attention is original and not P.is_patched()
        assert not P._router.hooks


def test_patched_sdpa_passes_prefill_through_and_notes_layers():
    from custom_kv import patch_model, unpatch_model
    from custom_kv import patch as P
    model = _Model(n_layers=3)
    original = F.scaled_dot_product_attention
    patch_model(model, cache=object())
    try:
        q = torch.randn(1, 2, 3, 8)
        got = F.scaled_dot_product_attention(q, q, q, is_causal=True)
        assert torch.equal(got, original(q, q, q, is_causal=True))
        model.layers[2](torch.zeros(1, 1, 4))
        assert P._router.layer_hint == 2
    finally:
        unpatch_model()


def test_projection_sampler_taps_every_layer():
    """Every attention module's k_proj / v_proj output is sampled, up to
    rows_per_pass rows per forward pass (the reference's hook test is
    tests/integration/test_colab_compat.py:256)."""
    from custom_kv.calibration import ProjectionSampler, _encode
    n_layers, d_model, d_kv = 4, 64, 32
    model = _Model(n_layers, d_model, d_kv)

    def tok(text, return_tensors=None, max_length=None, truncation=None):
        return {"input_ids": torch.randint(0, 100, (1, min(len(text.split()), max_length or 32)))}

    with ProjectionSampler(model, rows_per_pass=20, seed=3) as tap:
        for text in ["hello world " * 20] * 3:
            model(**_encode(tok, text, 32, torch.device("cpu")))
    k, v = tap.rows("k"), tap.rows("v")
    assert sorted(k) == list(range(n_layers)) and sorted(v) == list(range(n_layers))
    for i in range(n_layers):
        assert k[i].shape == (60, d_kv) and v[i].shape == (60, d_kv)  # 3 passes x 20 of 32 rows
    assert not any(m._forward_hooks for m in model.modules())  # hooks removed on exit


def test_read_texts(tmp_path):
    from custom_kv.calibration import read_texts
    (tmp_path / "b.txt").write_text("second " * 1000)
    (tmp_path / "a.txt").write_text("first")
    assert read_texts(tmp_path, 5) == ["first", ("second " * 1000)[:4000]]
    assert read_texts(tmp_path, 1) == ["first"]
    f = tmp_path / "one.txt"
    f.write_text("p1\n\np2\n\n\np3")
    assert read_texts(f, 2) == ["p1", "p2"]
    assert read_texts(tmp_path / "missing", 3) == [] and read_texts(None, 3) == []


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
