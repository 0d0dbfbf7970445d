"""Decode under an attention mask (left-padded batches).

The reference's decode step drops the mask (custom_kv/patch.py:87-117 calls
SDPA with attn_mask=None), so a batched generate() with left padding attends
to the pad tokens.  Here sequence b of a decode attends to tokens
[start[b], L) only: the kernel-level entry point against the oracle on the
unpadded suffix, and transformers generate() on a left-padded batch against
each sequence run on its own."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import workloads

pytestmark = pytest.mark.gpu


def _ulp16(x):
    a = np.abs(x.astype(np.float16))
    return (np.nextafter(a, np.float16(np.inf)) - a).astype(np.float32)


def _pools(B, hkv, L, cap, seed):
    import custom_ecc_cuda as ops
    k16, v16, _ = workloads.make_c1(seed=seed, B=B, hkv=hkv, hq=hkv, L=L)
    kb = torch.zeros((B, hkv, cap, 128), dtype=torch.uint8, device="cuda")
    vb = torch.zeros_like(kb)
    ops.compress_into(k16.cuda(), kb, pos=0, rotate=True)
    ops.compress_into(v16.cuda(), vb, pos=0, rotate=True)
    return kb, vb


@pytest.mark.parametrize("hq,hkv", [(8, 2), (4, 4), (16, 2)])
def test_masked_decode_matches_oracle_on_suffix(oracle, cuda_device, hq, hkv):
    import custom_ecc_cuda as ops
    B, L = 4, 300
    kb, vb = _pools(B, hkv, L, 320, seed=31)
    q = torch.randn(B, hq, 1, 128, generator=torch.Generator().manual_seed(5)).half()
    starts = [0, 37, 255, 299]
    start = torch.tensor(starts, dtype=torch.int32, device="cuda")
    out = ops.decode_attention_masked(q.cuda(), kb, vb, seq_len=L, start=start, rotate_q=True, unrotate_out=True)
    got = out.float().cpu().numpy().reshape(B, hq, 128)
    kh, vh = kb.cpu().numpy(), vb.cpu().numpy()
    for b, s in enumerate(starts):
        ref = oracle.decode(q[b:b + 1].numpy(), kh[b:b + 1, :, s:L], vh[b:b + 1, :, s:L], hkv=hkv, seq_len=L - s,
                            rotate_q=True, unrotate_out=True)[0]
        assert np.all(np.abs(got[b] - ref) <= 2e-3 + 0.5 * _ulp16(ref)), (b, s)
    # start 0 everywhere is the unmasked decode, bit for bit (same kernel and partition)
    zero = torch.zeros(B, dtype=torch.int32, device="cuda")
    a = ops.decode_attention_masked(q.cuda(), kb, vb, seq_len=L, start=zero, rotate_q=True, unrotate_out=True)
    b_ = ops.decode_attention(q.cuda(), kb, vb, seq_len=L, rotate_q=True, unrotate_out=True)
    assert torch.equal(a, b_)
    # a sequence masked entirely gives zeros, the others are unaffected
    allm = torch.tensor([L, 0, L + 5, 0], dtype=torch.int32, device="cuda")
    c = ops.decode_attention_masked(q.cuda(), kb, vb, seq_len=L, start=allm, rotate_q=True, unrotate_out=True)
    assert torch.all(c[0] == 0) and torch.all(c[2] == 0)
    assert torch.equal(c[1], b_[1]) and torch.equal(c[3], b_[3])


def test_masked_decode_rejects_bad_start(cuda_device):
    import custom_ecc_cuda as ops
    kb, vb = _pools(2, 2, 64, 64, seed=1)
    q = torch.randn(2, 4, 1, 128, device="cuda").half()
    with pytest.raises(RuntimeError):
        ops.decode_attention_masked(q, kb, vb, seq_len=64, start=torch.zeros(2, dtype=torch.int64, device="cuda"))
    with pytest.raises(RuntimeError):
        ops.decode_attention_masked(q, kb, vb, seq_len=64, start=torch.zeros(3, dtype=torch.int32, device="cuda"))


def _tiny_llama(seed=0):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=128, vocab_size=1000, max_position_embeddings=4096,
                      rope_theta=500000.0, attn_implementation="sdpa", pad_token_id=0)
    return LlamaForCausalLM(cfg).half().cuda().eval()


def test_left_padded_generate_matches_each_sequence_alone(cuda_device):
    """Batch of two prompts (200 and 120 tokens), left-padded, through
    generate() with the ECC cache: each row's logits equal (to rounding) those
    of the same prompt run alone, and the greedy tokens agree."""
    from custom_kv import ecc_cache
    model = _tiny_llama(seed=2)
    g = torch.Generator().manual_seed(7)
    p0 = torch.randint(1, 1000, (200,), generator=g)
    p1 = torch.randint(1, 1000, (120,), generator=g)
    ids = torch.zeros((2, 200), dtype=torch.long)
    mask = torch.zeros((2, 200), dtype=torch.long)
    ids[0], mask[0] = p0, 1
    ids[1, 80:], mask[1, 80:] = p1, 1
    new = 8
    with torch.no_grad():
        with ecc_cache(model, batch_size=2, max_cache_len=256, device="cuda") as cache:
            got = model.generate(ids.cuda(), attention_mask=mask.cuda(), past_key_values=cache, max_new_tokens=new,
                                 do_sample=False, output_logits=True, return_dict_in_generate=True)
            assert cache._last_window is not None  # the masked kernel ran
        alone = []
        for p in (p0, p1):
            with ecc_cache(model, batch_size=1, max_cache_len=256, device="cuda") as cache:
                alone.append(model.generate(p[None].cuda(), past_key_values=cache, max_new_tokens=new,
                                            do_sample=False, output_logits=True, return_dict_in_generate=True))
    for row, ref in enumerate(alone):
        assert torch.equal(got.sequences[row, 200:], ref.sequences[0, -new:])
        for step in range(1, new):
            cos = F.cosine_similarity(got.logits[step][row].float(), ref.logits[step][0].float(), dim=0)
            assert cos > 0.999, (row, step, float(cos))


def test_mask_with_holes_takes_masked_sdpa(cuda_device):
    """A mask that is not a suffix of the context (a hole in the middle) is
    served by reconstruction + masked SDPA and equals it exactly."""
    from custom_kv import ErrorCorrectedCache

    class Cfg:
        num_hidden_layers, num_attention_heads, num_key_value_heads = 1, 4, 2
        hidden_size, head_dim = 512, 128

    cache = ErrorCorrectedCache(Cfg(), batch_size=2, max_cache_len=64, device="cuda")
    gk = torch.Generator(device="cuda").manual_seed(3)
    k = torch.randn(2, 2, 40, 128, device="cuda", generator=gk).half()
    v = torch.randn(2, 2, 40, 128, device="cuda", generator=gk).half()
    cache.update(k, v, 0)
    mask = torch.ones(2, 1, 1, 40, dtype=torch.bool, device="cuda")
    mask[0, ..., 10:20] = False
    q = torch.randn(2, 4, 1, 128, device="cuda").half()
    out = cache.decode_attention(q, 0, attn_mask=mask)
    assert cache._last_window is False
    kr, vr = cache._context_fp16(0, 40)
    ref = F.scaled_dot_product_attention(q, kr, vr, attn_mask=mask, enable_gqa=True)
    assert torch.equal(out, ref)
