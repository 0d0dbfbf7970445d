"""Positions and lengths in device memory: the append and the decode read
them when the kernel runs, so one CUDA graph of a decode step serves every
step of a growing cache.  Checked against the eager ops and the oracle."""
import numpy as np
import pytest
import torch

import workloads

pytestmark = pytest.mark.gpu
TOL = 2e-3


@pytest.fixture(scope="module")
def ops(cuda_device):
    import custom_ecc_cuda
    return custom_ecc_cuda


def _close(out, ref):
    """fp16 output within 2e-3 of the fp32 reference plus its own rounding
    (half an fp16 ulp).  Rounding the reference to fp16 first would add a
    second half ulp for values on an fp16 rounding midpoint."""
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)
    err = np.abs(out.float().cpu().numpy().reshape(ref.shape) - ref)
    assert np.all(err <= TOL + ulp / 2), err.max()


def test_append_at_device_position_equals_host_position(ops, cuda_device):
    B, H, cap = 2, 4, 300
    g = torch.Generator(device=cuda_device).manual_seed(4)
    k = torch.randn(B, H, 3, 128, device=cuda_device, generator=g).half()
    v = torch.randn(B, H, 3, 128, device=cuda_device, generator=g).half()
    pos = torch.tensor([171], dtype=torch.int32, device=cuda_device)
    a_k = torch.zeros((B, H, cap, 128), dtype=torch.uint8, device=cuda_device)
    a_v = torch.zeros_like(a_k)
    b_k, b_v = torch.zeros_like(a_k), torch.zeros_like(a_k)
    ops.compress_pair_at(k, v, a_k, a_v, pos, rotate=True)
    ops.compress_pair_into(k, v, b_k, b_v, pos=171, rotate=True)
    assert torch.equal(a_k, b_k) and torch.equal(a_v, b_v)
    ops.compress_pair_at(k, None, a_k, None, pos, rotate=False)  # one tensor
    ops.compress_into(k, b_k, pos=171, rotate=False)
    assert torch.equal(a_k, b_k)
    c_k = torch.zeros_like(a_k)
    ops.compress_calibrated_at(k, c_k, 0.9, 0.01, 0.2, pos, rotate=True)
    d_k = torch.zeros_like(a_k)
    ops.compress_calibrated_into(k, d_k, 0.9, 0.01, 0.2, pos=171, rotate=True)
    assert torch.equal(c_k, d_k)
    # out of range: nothing written, the device flag says so
    ops.device_status(reset=True)
    before = a_k.clone()
    pos.fill_(cap - 2)
    ops.compress_pair_at(k, v, a_k, a_v, pos, rotate=True)
    torch.cuda.synchronize()
    assert torch.equal(a_k, before)
    assert ops.device_status(reset=True) == 3
    assert ops.device_status() == 0


@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 8), (16, 2)])
def test_decode_with_device_length_equals_oracle(ops, oracle, cuda_device, hq, hkv):
    B, cap = 2, 3000
    k16, v16, _ = workloads.make_c1(seed=17, B=B, hkv=hkv, hq=hq, L=cap)
    kp = torch.empty((B, hkv, cap, 128), dtype=torch.uint8, device=cuda_device)
    vp = torch.empty_like(kp)
    ops.compress_into(k16.to(cuda_device), kp, rotate=True)
    ops.compress_into(v16.to(cuda_device), vp, rotate=True)
    kb, vb = kp.cpu().numpy(), vp.cpu().numpy()
    n = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    q = torch.randn(B, hq, 1, 128, generator=torch.Generator().manual_seed(3)).half().to(cuda_device)
    for L in (1, 31, 32, 33, 1000, 2999, 3000):
        n.fill_(L)
        out = ops.decode_attention_dev(q, kp, vp, n, rotate_q=True, unrotate_out=True)
        ref = oracle.decode(q.cpu().numpy(), kb, vb, hkv=hkv, seq_len=L, rotate_q=True, unrotate_out=True)
        _close(out, ref)
    n.fill_(10 ** 6)  # clamped to the capacity
    _close(ops.decode_attention_dev(q, kp, vp, n, rotate_q=True, unrotate_out=True),
           oracle.decode(q.cpu().numpy(), kb, vb, hkv=hkv, seq_len=cap, rotate_q=True, unrotate_out=True))


def test_partials_with_device_length(ops, oracle, cuda_device):
    """decode_partials_dev + lse_merge equals decode_attention_dev bit for bit
    and the oracle within tolerance; too few splits are rejected."""
    B, hq, hkv, cap = 2, 16, 4, 2500
    k16, v16, _ = workloads.make_c1(seed=29, B=B, hkv=hkv, hq=hq, L=cap)
    kp = torch.empty((B, hkv, cap, 128), dtype=torch.uint8, device=cuda_device)
    vp = torch.empty_like(kp)
    ops.compress_into(k16.to(cuda_device), kp, rotate=True)
    ops.compress_into(v16.to(cuda_device), vp, rotate=True)
    q = torch.randn(B, hq, 1, 128, generator=torch.Generator().manual_seed(8)).half().to(cuda_device)
    ns = ops.decode_dev_splits(B, hkv, cap)
    for L in (1, 100, 2047, 2500):
        n = torch.tensor([L], dtype=torch.int32, device=cuda_device)
        pm, pl, po = ops.decode_partials_dev(q, kp, vp, n, ns + 3, rotate_q=True)
        merged = ops.lse_merge(pm, pl, po, unrotate_out=True)
        whole = ops.decode_attention_dev(q, kp, vp, n, rotate_q=True, unrotate_out=True)
        assert torch.equal(merged.reshape(whole.shape), whole)
        ref = oracle.decode(q.cpu().numpy(), kp.cpu().numpy(), vp.cpu().numpy(), hkv=hkv, seq_len=L, rotate_q=True,
                            unrotate_out=True)
        _close(whole, ref)
    with pytest.raises(RuntimeError):
        ops.decode_partials_dev(q, kp, vp, n, ns - 1, rotate_q=True)


def test_graph_of_append_and_decode_replays_a_growing_cache(ops, oracle, cuda_device):
    """Record append + decode once; replay for 6 steps while the device-side
    length grows; every step equals the oracle on the pools at that length."""
    B, hq, hkv, cap, L0 = 1, 8, 2, 1024, 700
    k16, v16, _ = workloads.make_c1(seed=23, B=B, hkv=hkv, hq=hq, L=L0)
    kp = torch.zeros((B, hkv, cap, 128), dtype=torch.uint8, device=cuda_device)
    vp = torch.zeros_like(kp)
    ops.compress_into(k16.to(cuda_device), kp, rotate=True)
    ops.compress_into(v16.to(cuda_device), vp, rotate=True)
    pos = torch.tensor([L0], dtype=torch.int32, device=cuda_device)
    length = torch.tensor([L0 + 1], dtype=torch.int32, device=cuda_device)
    newk = torch.zeros(B, hkv, 1, 128, dtype=torch.float16, device=cuda_device)
    newv = torch.zeros_like(newk)
    q = torch.zeros(B, hq, 1, 128, dtype=torch.float16, device=cuda_device)
    out = torch.empty_like(q)
    ws = torch.empty(ops.decode_dev_workspace_size(B, hq, hkv, cap), dtype=torch.uint8, device=cuda_device)
    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(s):  # warm-up off the capture
        ops.compress_pair_at(newk, newv, kp, vp, pos, rotate=True)
        ops.decode_attention_dev(q, kp, vp, length, rotate_q=True, unrotate_out=True, out=out, workspace=ws)
    torch.cuda.current_stream(cuda_device).wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.compress_pair_at(newk, newv, kp, vp, pos, rotate=True)
        ops.decode_attention_dev(q, kp, vp, length, rotate_q=True, unrotate_out=True, out=out, workspace=ws)
    gen = torch.Generator().manual_seed(5)
    for step in range(6):
        L = L0 + step
        newk.copy_(torch.randn(B, hkv, 1, 128, generator=gen).half())
        newv.copy_(torch.randn(B, hkv, 1, 128, generator=gen).half())
        q.copy_(torch.randn(B, hq, 1, 128, generator=gen).half())
        pos.fill_(L)
        length.fill_(L + 1)
        graph.replay()
        torch.cuda.synchronize()
        ref = oracle.decode(q.cpu().numpy(), kp.cpu().numpy(), vp.cpu().numpy(), hkv=hkv, seq_len=L + 1,
                            rotate_q=True, unrotate_out=True)
        _close(out, ref)
        # the appended token is the eager compress of the step's K and V
        blk = torch.empty((B, hkv, 1, 128), dtype=torch.uint8, device=cuda_device)
        ops.compress_into(newk, blk, rotate=True)
        assert torch.equal(blk[:, :, 0], kp[:, :, L])
    del graph


def _tiny_llama(seed=0, layers=2):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=layers, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=128, vocab_size=1000, max_position_embeddings=4096,
                      rope_theta=500000.0, attn_implementation="sdpa")
    return LlamaForCausalLM(cfg).half().cuda().eval()


def test_graph_decoder_replays_eager_decode_steps(cuda_device):
    """transformers Llama over the ECC cache: every replayed step (model
    forward, appends, fused decodes, argmax) gives the logits and token of the
    same step run eagerly with device-side lengths, bit for bit; and the
    tokens follow the ordinary eager ECC decode."""
    from custom_kv import ecc_cache
    from custom_kv.graph import GraphDecoder
    model = _tiny_llama(seed=2, layers=3)
    prompt = torch.randint(0, 1000, (1, 200), generator=torch.Generator().manual_seed(1)).cuda()
    steps = 8
    with torch.no_grad():
        # eager, device-side lengths
        with ecc_cache(model, batch_size=1, max_cache_len=256, device="cuda") as cache:
            logits = model(prompt, past_key_values=cache, use_cache=True).logits[:, -1]
            tok = logits.argmax(-1, keepdim=True)
            cache.enable_device_lengths()
            eager_logits, eager_toks = [], []
            pos = 200
            for _ in range(steps):
                out = model(input_ids=tok, position_ids=torch.tensor([[pos]], device="cuda"),
                            cache_position=torch.tensor([pos], device="cuda"), past_key_values=cache, use_cache=True)
                eager_logits.append(out.logits[:, -1].clone())
                tok = out.logits[:, -1].argmax(-1, keepdim=True)
                eager_toks.append(tok.clone())
                cache.advance_device_lengths()
                pos += 1
        # graph replays
        with ecc_cache(model, batch_size=1, max_cache_len=256, device="cuda") as cache:
            logits = model(prompt, past_key_values=cache, use_cache=True).logits[:, -1]
            dec = GraphDecoder(model, cache, logits.argmax(-1, keepdim=True))
            for i in range(steps):
                t = dec.step()
                torch.cuda.synchronize()
                assert torch.equal(dec.logits, eager_logits[i]), f"step {i}"
                assert torch.equal(t, eager_toks[i])
            assert dec.sync_host_lengths() == 200 + steps
        # the ordinary eager path (host lengths) follows the same tokens
        with ecc_cache(model, batch_size=1, max_cache_len=256, device="cuda") as cache:
            got = model.generate(prompt, past_key_values=cache, max_new_tokens=4, do_sample=False)
    assert torch.equal(got[0, 201:204].cpu(), torch.cat(eager_toks[:3]).flatten().cpu())
