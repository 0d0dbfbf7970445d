"""ErrorCorrectedCache, the SDPA patch and ecc_cache on the GPU: the
reference's cache-contract tests re-targeted to CUDA, plus a real
transformers LlamaForCausalLM generate() through the compressed cache."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


class FakeConfig:
    num_hidden_layers = 32
    num_attention_heads = 32
    num_key_value_heads = 8
    hidden_size = 4096
    head_dim = 128
    _name_or_path = "random-init/llama-3.1-8b-shape"


class TinyConfig(FakeConfig):
    num_hidden_layers = 2
    num_attention_heads = 4
    num_key_value_heads = 2
    hidden_size = 512


def _cache(cfg=None, L=64, **kw):
    from custom_kv import ErrorCorrectedCache
    return ErrorCorrectedCache(cfg or TinyConfig(), batch_size=1, max_cache_len=L, device="cuda", **kw)


def _kv(L, H=2, B=1, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(B, H, L, 128, device="cuda", generator=g).half(),
            torch.randn(B, H, L, 128, device="cuda", generator=g).half())


def test_contract_attributes(cuda_device):
    from transformers.cache_utils import Cache
    c = _cache()
    assert isinstance(c, Cache) and isinstance(c.layers, list) and c.is_compileable is False
    c.update(*_kv(8), layer_idx=0)
    assert c.get_mask_sizes(1, 0) == (9, 0)  # past 8 + query 1
    for m in ("update", "get_seq_length", "get_max_cache_shape", "reset", "crop", "batch_select_indices",
              "reorder_cache"):
        assert hasattr(c, m)


def test_reference_shapes_and_memory(cuda_device):
    c = _cache(FakeConfig(), L=512)
    assert c._k_int4.shape == (1, 8, 512, 64) and c._k_syn.shape == (1, 8, 512, 16)
    assert c._k_meta.shape == (1, 8, 512, 3) and c._k_meta.dtype == torch.float16
    assert c._v_int4.shape == (1, 8, 512, 64)
    mem = c.memory_bytes()
    assert mem["cache_gb"] > 0 and mem["compression_ratio"] == 2.0
    assert "ErrorCorrectedCache" in repr(c) and c._max_cache_len == 512


def test_reset_crop_seen_tokens(cuda_device):
    c = _cache()
    c.update(*_kv(10), layer_idx=0)
    assert c.seen_tokens == 0
    c.update(*_kv(10), layer_idx=1)
    assert c.seen_tokens == 10 and c.get_seq_length(0) == 10
    c.crop(7)
    assert c.get_seq_length(0) == 7 and c.get_seq_length(1) == 7
    c.reset()
    assert c.get_seq_length(0) == 0 and c.get_seq_length(1) == 0 and c.seen_tokens == 0


def test_update_returns_usable_kv(cuda_device):
    c = _cache()
    k, v = _kv(12)
    ko, vo = c.update(k, v, layer_idx=0)
    assert ko is k and vo is v  # first prefill: the uncompressed states
    k2, v2 = _kv(5, seed=1)
    ko, vo = c.update(k2, v2, layer_idx=0)  # chunked prefill: context + new
    assert ko.shape == (1, 2, 17, 128) and ko.dtype == torch.float16
    assert torch.equal(ko[:, :, 12:], k2)
    rel = (ko[:, :, :12].float() - k.float()).norm() / k.float().norm()
    assert rel < 0.15  # INT4 + sign correction reconstruction of the first chunk


def test_compress_dequantize_roundtrip(oracle, cuda_device):
    c = _cache(FakeConfig(), L=64)
    x = torch.randn(1, 8, 16, 128, device="cuda").half()
    c._compress(x, c._k_int4, c._k_syn, c._k_meta, pos=0, L_new=16)
    rec = c._dequantize(c._k_int4[:, :, :16], c._k_syn[:, :, :16], c._k_meta[:, :, :16])
    assert rec.shape == x.shape
    ref = oracle.reconstruct(oracle.compress(x.cpu().numpy().reshape(-1, 128), rotate=False))
    assert np.array_equal(rec.cpu().numpy().reshape(-1, 128).view(np.uint16),
                          ref.astype(np.float16).view(np.uint16))
    assert ((x.float() - rec.float()).abs().mean() / x.float().abs().mean()) < 0.5
    assert (x.sign() == rec.float().sign()).float().mean() > 0.7
    # standalone SoA tensors go through the pack kernel
    rec2 = c._dequantize(c._k_int4[:, :, :16].contiguous(), c._k_syn[:, :, :16].contiguous(),
                         c._k_meta[:, :, :16].contiguous())
    assert torch.equal(rec, rec2)


def test_get_kv_fp16_for_layer(cuda_device):
    c = _cache()
    c.update(*_kv(12), layer_idx=1)
    k, v = c.get_kv_fp16_for_layer(1)
    assert k.shape == (1, 2, 12, 128) and v.shape == (1, 2, 12, 128) and k.dtype == torch.float16


def test_layers_do_not_overwrite_each_other(cuda_device):
    c = _cache()
    k0, v0 = _kv(6, seed=10)
    k1, v1 = _kv(6, seed=11)
    c.update(k0, v0, 0)
    c.update(k1, v1, 1)
    a, _ = c.get_kv_fp16_for_layer(0)
    b, _ = c.get_kv_fp16_for_layer(1)
    assert not torch.equal(a, b)


def test_ecc_cache_context_manager(cuda_device):
    from custom_kv import ecc_cache

    class M(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.config = TinyConfig()
            self.model = torch.nn.Module()
            self.model.layers = torch.nn.ModuleList()

    model = M()
    original = F.scaled_dot_product_attention
    for _ in range(3):
        with ecc_cache(model, batch_size=1, max_cache_len=32, device="cuda") as cache:
            assert F.scaled_dot_product_attention is not original
            cache.update(*_kv(4), layer_idx=0)
            cache.update(*_kv(4), layer_idx=1)
            assert cache.get_seq_length(0) == 4 and cache.seen_tokens == 4
        assert F.scaled_dot_product_attention is original
    with pytest.raises(RuntimeError, match="intentional"):
        with ecc_cache(model, batch_size=1, max_cache_len=32, device="cuda"):
            raise RuntimeError("intentional")
    assert F.scaled_dot_product_attention is original


def _tiny_llama(seed=0, layers=2):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=layers, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=128, vocab_size=1000, max_position_embeddings=4096,
                      rope_theta=500000.0, attn_implementation="sdpa")
    return LlamaForCausalLM(cfg).half().cuda().eval()


def test_decode_step_matches_oracle_through_patch(oracle, cuda_device):
    """The patched SDPA's decode result equals the oracle's decode on the
    cache's own blocks (GQA 4/2, rotated K and V)."""
    from custom_kv import ErrorCorrectedCache, patch_model, unpatch_model
    model = _tiny_llama()
    cache = ErrorCorrectedCache(model.config, batch_size=1, max_cache_len=256, device="cuda")
    patch_model(model, cache)
    try:
        k, v = _kv(100, seed=3)
        cache.update(k, v, layer_idx=1)
        q = torch.randn(1, 4, 1, 128, device="cuda").half()
        out = F.scaled_dot_product_attention(q, k[:, :, -1:], v[:, :, -1:], scale=128 ** -0.5)
    finally:
        unpatch_model()
    kp, vp = cache.layer_pools(1)
    ref = oracle.decode(q.cpu().numpy(), kp[:, :, :100].cpu().numpy(), vp[:, :, :100].cpu().numpy(), hkv=2,
                        seq_len=100, rotate_q=True, unrotate_out=True)
    err = np.abs(out.float().cpu().numpy().reshape(1, 4, 128) - ref.astype(np.float16).astype(np.float32)).max()
    assert err <= 2e-3
    # and it approximates exact fp16 attention on the uncompressed K/V
    exact = F.scaled_dot_product_attention(q, k, v, scale=128 ** -0.5, enable_gqa=True)
    cos = F.cosine_similarity(out.float().flatten(), exact.float().flatten(), dim=0)
    assert cos > 0.95


def test_llama_generate_through_ecc_cache(cuda_device, monkeypatch):
    """transformers generate() end to end: prefill on fp16 K/V, every decode
    step through the ECC kernel, logits close to the fp16-cache run."""
    import custom_ecc_cuda as ops
    from custom_kv import ecc_cache
    model = _tiny_llama(seed=1)
    prompt = torch.randint(0, 1000, (1, 300), generator=torch.Generator().manual_seed(0)).cuda()
    calls = {"n": 0}
    real = ops.decode_attention

    def counting(*a, **k):
        calls["n"] += 1
        return real(*a, **k)

    monkeypatch.setattr(ops, "decode_attention", counting)
    with torch.no_grad():
        ref = model.generate(prompt, max_new_tokens=12, do_sample=False, output_logits=True,
                             return_dict_in_generate=True)
        with ecc_cache(model, batch_size=1, max_cache_len=512, device="cuda") as cache:
            got = model.generate(prompt, past_key_values=cache, max_new_tokens=12, do_sample=False,
                                 output_logits=True, return_dict_in_generate=True)
            assert cache.get_seq_length(0) == 300 + 11
    assert got.sequences.shape == (1, 312)
    assert calls["n"] == 11 * 2  # 11 decode steps x 2 layers
    # first generated token comes from the (uncompressed) prefill: identical
    assert torch.equal(got.sequences[0, 300], ref.sequences[0, 300])
    cos = F.cosine_similarity(got.logits[1].float().flatten(), ref.logits[1].float().flatten(), dim=0)
    assert cos > 0.98


def test_cache_consumes_calibration_for_keys(oracle, cuda_device):
    """With a calibration config the cache's key blocks of the listed layers
    carry that layer's scale / zero / alpha and the calibrated quantisation;
    values and unlisted layers keep per-vector statistics; decode through the
    pools still matches the oracle."""
    import custom_ecc_cuda as ops
    cal = {"layers": {"1": {"scale": 0.93, "zero": 0.011, "alpha": 0.18, "sigma": 0.93}}}
    cache = _cache(L=128, calibration=cal)
    k, v = _kv(100, seed=9)
    for layer in (0, 1):
        cache.update(k, v, layer_idx=layer)
    kp1, vp1 = cache.layer_pools(1)
    kp0, _ = cache.layer_pools(0)
    k_blocks = kp1[:, :, :100].reshape(-1, 128).cpu().numpy()
    ref_k = oracle.compress_calibrated_np(k.reshape(-1, 128).cpu().numpy(), 0.93, 0.011, 0.18, rotate=True)
    assert np.array_equal(k_blocks, ref_k)
    assert np.array_equal(vp1[:, :, :100].reshape(-1, 128).cpu().numpy(),
                          oracle.compress(v.reshape(-1, 128).cpu().numpy(), rotate=True))
    assert np.array_equal(kp0[:, :, :100].reshape(-1, 128).cpu().numpy(),
                          oracle.compress(k.reshape(-1, 128).cpu().numpy(), rotate=True))
    q = torch.randn(1, 4, 1, 128, device="cuda").half()
    out = ops.decode_attention(q, kp1, vp1, seq_len=100, rotate_q=True, unrotate_out=True)
    ref = oracle.decode(q.cpu().numpy(), kp1[:, :, :100].cpu().numpy(), vp1[:, :, :100].cpu().numpy(), hkv=2,
                        seq_len=100, rotate_q=True, unrotate_out=True)
    ref16 = ref.astype(np.float16).astype(np.float32)
    err = np.abs(out.float().cpu().numpy().reshape(1, 4, 128) - ref16)
    assert np.all(err <= 2e-3 + np.spacing(np.abs(ref16).astype(np.float16)).astype(np.float32) / 2)
