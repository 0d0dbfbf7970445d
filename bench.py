#!/usr/bin/env python
"""Benchmark of the ECC-INT4 KV-cache hot path on B200.

Default workload (one "step"): one decode step of the single-layer decode
benchmark -- batch 8, 32 query heads over 8 KV heads (GQA 4), head dim 128,
65536-token compressed context that grows by one token per step:
compress the step's new K and V token into the block pools, then fused decode
attention of the step's queries over the whole context.  Inputs are seeded
synthetic N(0,1) fp16 (no dataset is involved on this path).  The pools
(2 x 8 x 8 x 65536 x 128 B = 1.07 GB) are far larger than the 126 MB L2, so
no L2 flush is needed between steps.

Also measured in the same run: compress throughput on the compress benchmark
(8 KV heads x 131072 tokens, K and V, heavy-tailed fp16).

N > 1 GPUs (torchrun): the same job split over the ranks (strong scaling):
by kv head by default (rank r holds kv heads [8r/N, 8(r+1)/N) of every
sequence; one kernel per step merges the rank's partials and gathers the
ranks' fp16 outputs over peer memory, or NCCL with ``--exchange nccl``), or by
sequence chunk with ``--shard seq`` (LSE combine of the ranks' partial
records over peer memory or NCCL).  With N > 1 the K timed steps are
recorded once as a CUDA graph and replayed (``--graph off``: issued eagerly,
which the host's issue time bounds at 8 GPUs).  Rank 0 checks the final
step's sharded output against a one-GPU decode of the same pools.

``--impl reference`` times the reference algorithm's CPU implementation (the
oracle port in oracle/, all host threads) on a bounded sample of the same
workload and prints the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(ROOT, "ecc-kv-cache_b200"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "ECC-INT4 decode-attn HBM GB/s (% peak); decode tok/s @64k ctx; compress tok/s"
B, HQ, HKV, D, CTX = 8, 32, 8, 128, 65536
BLOCK = 128
COMPRESS_TOKENS = 131072

# DRAM bytes per unit measured with ncu (dram__bytes_read.sum +
# dram__bytes_write.sum of one launch of the decode kernel at B8 x 8 kv heads x
# 65541 tokens, and of one compress launch of 8 x 131072 vectors, divided by the
# units each processed).
# Decode: per (token, kv head), algorithmic 256 B.  Compress: per vector,
# algorithmic 384 B; the output blocks of a launch partly stay in the 126 MB L2
# when the launch ends, so DRAM writes are counted below 128 B per vector.
DECODE_DRAM_BYTES_PER_UNIT = (1.074460e9 + 3.663104e6) / (B * HKV * 65541)
COMPRESS_DRAM_BYTES_PER_VECTOR = (268.652032e6 + 97.288704e6) / (HKV * COMPRESS_TOKENS)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 20 ms with host
    timestamps; summary() reports the samples inside the window mark_start()
    .. mark_stop() (the timed region), or the nearest ones if the window was
    shorter than the sampling interval."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu = gpu_id
        self.proc = None
        self.samples = []  # (host time, line)
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            deadline = time.time() + 10.0  # let nvidia-smi come up before the timed region
            while not self.samples and time.time() < deadline and self.proc.poll() is None:
                time.sleep(0.01)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def mark_start(self):
        self.t0 = time.time()

    def mark_stop(self):
        self.t1 = time.time()
        time.sleep(0.06)  # the sample that covers the end of the window

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        picked = [ln for t, ln in self.samples if self.t0 is not None and self.t0 <= t <= (self.t1 or t)]
        window = "timed region"
        if not picked and self.samples and self.t0 is not None:
            mid = 0.5 * (self.t0 + (self.t1 or self.t0))
            picked = [min(self.samples, key=lambda s: abs(s[0] - mid))[1]]
            window = "nearest sample"
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in picked:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "window": window}


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def compress_bench(ops, workloads, dev, stream, K, peak, peak_kind):
    """Compress throughput: 8 KV heads x 131072 tokens of heavy-tailed fp16,
    K then V, each one launch of 1 048 576 vectors into a block pool."""
    import torch
    ck, cv = workloads.make_c2(seed=0, L=COMPRESS_TOKENS, device=dev)
    cpool_k = torch.empty((1, HKV, COMPRESS_TOKENS, BLOCK), dtype=torch.uint8, device=dev)
    cpool_v = torch.empty_like(cpool_k)
    for _ in range(3):
        ops.compress_into(ck, cpool_k, rotate=True)
        ops.compress_into(cv, cpool_v, rotate=True)
    reps = max(5, min(50, K))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    torch.cuda.synchronize()
    for a, b in evs:
        a.record(stream)
        ops.compress_into(ck, cpool_k, rotate=True)
        ops.compress_into(cv, cpool_v, rotate=True)
        b.record(stream)
    torch.cuda.synchronize()
    cms = [a.elapsed_time(b) for a, b in evs]
    c_avg = sum(cms) / len(cms)
    n_vec = 2 * HKV * COMPRESS_TOKENS
    cbytes = n_vec * (2 * D + BLOCK)
    c_gbs = cbytes / (c_avg / 1e3) / 1e9
    return {"workload": "compress 8 KV heads x 131072 tokens, K and V, fp16 N(0,1) + Student-t(3) on 3% of "
                        "channels -> 128-B blocks",
            "tok_s": HKV * COMPRESS_TOKENS / (c_avg / 1e3), "vectors_per_s": n_vec / (c_avg / 1e3),
            "ms_per_pass": c_avg, "gbs": c_gbs,
            # input vectors and the blocks the kernel wrote for them, for the
            # oracle parity check of the CPU leg (removed before printing)
            "_sample": (ck[0, 0, :32768].cpu().numpy(), cpool_k[0, 0, :32768].cpu().numpy()),
            "roofline": {"bound": "hbm", "achieved": c_gbs, "peak": peak, "unit": "GB/s",
                         "frac": c_gbs / peak,
                         "traffic": COMPRESS_DRAM_BYTES_PER_VECTOR * HKV * COMPRESS_TOKENS,
                         "note": f"per launch of {HKV * COMPRESS_TOKENS} vectors: 384 B per vector (256 B fp16 "
                                 f"in + 128 B block out); traffic from ncu; peak {peak_kind}"}}


def run_compress_only(args):
    import torch
    import custom_ecc_cuda as ops
    import workloads
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak, peak_kind = peaks()
    comp = compress_bench(ops, workloads, dev, torch.cuda.current_stream(dev), args.steps, peak, peak_kind)
    comp.pop("_sample")
    print(json.dumps({"compress": comp}), flush=True)


def run_model_e2e(args):
    """Model-level run: a Llama-3.1-8B-shaped model (32 layers, 32 q / 8 kv
    heads, hidden 4096, MLP 14336, vocab 128256, rope theta 5e5) with seeded
    random fp16 weights (no checkpoint is available offline), a 32768-token
    seeded random prompt, 200 greedy tokens through transformers generate():
    once with the ECC cache (prefill on fp16 K/V with every layer compressed
    into the block pools, every decode step through the fused kernel), once
    with transformers' own fp16 cache, and once with the ECC cache and every
    decode step one CUDA-graph replay (custom_kv.graph: same kernels, lengths
    in device memory, no per-token host work).  Prints one JSON object."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    from custom_kv import ecc_cache
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    prompt_len, new_tokens = 32768, 200
    cfg = LlamaConfig(hidden_size=4096, intermediate_size=14336, num_hidden_layers=32, num_attention_heads=32,
                      num_key_value_heads=8, head_dim=128, vocab_size=128256, rope_theta=500000.0,
                      max_position_embeddings=131072)
    torch.manual_seed(0)
    with torch.device(dev):
        model = LlamaForCausalLM(cfg).half().eval()  # torch's default init, seeded, on the GPU
    prompt = torch.randint(0, cfg.vocab_size, (1, prompt_len), generator=torch.Generator().manual_seed(0)).to(dev)
    mask = torch.ones_like(prompt)

    def timed_generate(n, cache_ctx):
        # time generate() only: the cache context's set-up and exit (pool
        # allocation, allocator cache release) are outside the timed region
        with torch.no_grad(), cache_ctx() as cache:
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            out = model.generate(prompt, attention_mask=mask, past_key_values=cache, max_new_tokens=n,
                                 min_new_tokens=n, do_sample=False)
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            extra = cache.memory_bytes() if hasattr(cache, "memory_bytes") else None
        return dt, out, extra

    class _NoCache:  # transformers' default (fp16 DynamicCache)
        def __enter__(self):
            return None

        def __exit__(self, *a):
            return False

    def ecc_ctx():
        return ecc_cache(model, batch_size=1, max_cache_len=prompt_len + new_tokens + 8, device=str(dev))

    def graph_decode():
        # prefill eagerly, then every decode step one CUDA-graph replay
        from custom_kv.graph import GraphDecoder
        with torch.no_grad(), ecc_ctx() as cache:
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            logits = model(prompt, attention_mask=mask, past_key_values=cache, use_cache=True).logits[:, -1]
            first = logits.argmax(-1, keepdim=True)
            torch.cuda.synchronize()
            t_pre = time.perf_counter() - t0
            t0 = time.perf_counter()
            dec = GraphDecoder(model, cache, first)
            torch.cuda.synchronize()
            t_setup = time.perf_counter() - t0
            toks = torch.empty((new_tokens,), dtype=torch.long, device=dev)
            toks[0] = first[0, 0]
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for i in range(1, new_tokens):
                toks[i] = dec.step()[0, 0]
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            n = new_tokens - 1
            return {"prefill_s": t_pre, "graph_setup_s": t_setup, "decode_tok_s": n / dt,
                    "decode_ms_per_token": 1e3 * dt / n, "tokens": toks.tolist()[:8]}

    res = {}
    graph_decode()  # warm-up
    res["ecc_cache_cuda_graph"] = graph_decode()
    torch.cuda.empty_cache()
    for name, ctx in (("ecc_cache", ecc_ctx), ("fp16_cache", _NoCache)):
        timed_generate(2, ctx)  # warm-up: kernels, allocator, tensor maps
        t_pre, _, _ = timed_generate(1, ctx)
        t_all, out, mem = timed_generate(new_tokens + 1, ctx)
        dec = t_all - t_pre
        res[name] = {"prefill_s": t_pre, "decode_tok_s": new_tokens / dec, "decode_ms_per_token": 1e3 * dec / new_tokens,
                     "tokens": out[0, prompt_len:].tolist()[:8]}
        if mem:
            res[name]["cache_memory"] = mem
        torch.cuda.empty_cache()
    same_first = (res["ecc_cache"]["tokens"][0] == res["fp16_cache"]["tokens"][0]
                  == res["ecc_cache_cuda_graph"]["tokens"][0])
    print(json.dumps({"workload": f"Llama-3.1-8B shape, random fp16 weights, {prompt_len}-token prompt, "
                                  f"{new_tokens} greedy tokens, batch 1, transformers generate()",
                      "data": "synthetic", **res, "first_token_equal": same_first}), flush=True)


def run_prefill(args):
    """One 32768-token prefill of the Llama-3.1-8B-shaped model (seeded
    random fp16 weights, seeded random prompt) through the ECC cache, after
    one warm-up prefill: every layer's K and V are compressed into the block
    pools by the fused WHT + compress kernel while attention runs on the fp16
    K/V.  Under ncu's launch list (gpu__time_duration only) this gives the
    compress kernels' share of the prefill's GPU time.  Prints the wall time."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    from custom_kv import ecc_cache
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    prompt_len = 32768
    cfg = LlamaConfig(hidden_size=4096, intermediate_size=14336, num_hidden_layers=32, num_attention_heads=32,
                      num_key_value_heads=8, head_dim=128, vocab_size=128256, rope_theta=500000.0,
                      max_position_embeddings=131072)
    torch.manual_seed(0)
    with torch.device(dev):
        model = LlamaForCausalLM(cfg).half().eval()
    prompt = torch.randint(0, cfg.vocab_size, (1, prompt_len), generator=torch.Generator().manual_seed(0)).to(dev)
    times = []
    with torch.no_grad():
        for rep in range(2):
            with ecc_cache(model, batch_size=1, max_cache_len=prompt_len + 8, device=str(dev)) as cache:
                torch.cuda.synchronize()
                if rep == 1:
                    torch.cuda.profiler.start()  # ncu --profile-from-start off records this prefill only
                t0 = time.perf_counter()
                model(prompt, past_key_values=cache, use_cache=True, logits_to_keep=1)
                torch.cuda.synchronize()
                times.append(time.perf_counter() - t0)
                if rep == 1:
                    torch.cuda.profiler.stop()
    print(json.dumps({"workload": f"Llama-3.1-8B shape, random fp16 weights, {prompt_len}-token prefill through "
                                  f"the ECC cache", "prefill_s": times[-1], "warmup_s": times[0]}), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def _fill_decode_pools(ops, kpool, vpool, heads, tok_range, dev):
    """Blocks of the decode workload for kv heads ``heads`` (global indices)
    and tokens [t0, t1) of every sequence, written to kpool / vpool at local
    head index and token t - t0.  Kv head h's tokens come from a generator
    seeded by h alone, so every rank of a kv-head or sequence-chunk split holds
    exactly its part of the one-GPU pools (rank 0 rebuilds those for the
    sharded parity check)."""
    import torch
    t0, t1 = tok_range
    chunk = 8192
    for li, h in enumerate(heads):
        gen = torch.Generator(device=dev).manual_seed(5000 + h)
        for c0 in range(0, CTX, chunk):
            xk = torch.randn((B, 1, chunk, D), generator=gen, device=dev).half()
            xv = torch.randn((B, 1, chunk, D), generator=gen, device=dev).half()
            a, b = max(c0, t0), min(c0 + chunk, t1)
            if a < b:
                ops.compress_into(xk[:, :, a - c0:b - c0], kpool[:, li:li + 1], pos=a - t0, rotate=True)
                ops.compress_into(xv[:, :, a - c0:b - c0], vpool[:, li:li + 1], pos=a - t0, rotate=True)


def _step_inputs(n_steps, dev):
    """New K / V token per step for every (b, kv head), and the step's queries."""
    import torch
    import workloads
    gen = torch.Generator(device=dev).manual_seed(777)
    new_k = torch.randn((n_steps, B, HKV, 1, D), generator=gen, device=dev).half()
    new_v = torch.randn((n_steps, B, HKV, 1, D), generator=gen, device=dev).half()
    qs = torch.stack([workloads.make_queries(i, B, HQ, device=dev) for i in range(n_steps)])
    return new_k, new_v, qs


def run_ours(args):
    """The decode benchmark (B8, Hq32/Hkv8, 65536-token context growing by one
    token per step; append + fused decode per step).  One GPU: the whole job.
    N GPUs (torchrun): the same job split over the ranks (strong scaling) --
    by kv head (default: rank r holds kv heads [8r/N, 8(r+1)/N) of every
    sequence, and the ranks' fp16 outputs are all-gathered) or by sequence
    chunk (``--shard seq``: rank r holds tokens [rL/N, (r+1)L/N) of every row,
    the last rank also the appended ones; LSE combine of the ranks'
    records)."""
    import torch
    import custom_ecc_cuda as ops

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist.group.WORLD
    mode = "single" if world == 1 else args.shard
    if mode == "kv" and HKV % world:
        raise SystemExit(f"{world} ranks do not divide {HKV} kv heads")
    K, W = args.steps, args.warmup
    rb = args.block_bytes  # 128-byte blocks, or the 96-byte records of the option
    n_steps = W + K
    growth = n_steps + K + 8  # timed steps, then the e2e steps
    last = rank == world - 1
    if mode == "kv":
        heads = list(range(rank * HKV // world, (rank + 1) * HKV // world))
        toks = (0, CTX)
    elif mode == "seq":
        heads = list(range(HKV))
        toks = (rank * CTX // world, (rank + 1) * CTX // world)
    else:
        heads, toks = list(range(HKV)), (0, CTX)
    hkv_l, hq_l = len(heads), len(heads) * (HQ // HKV)
    grows = mode != "seq" or last  # this rank appends the new tokens
    cap = toks[1] - toks[0] + (growth if grows else 0)
    kpool = torch.empty((B, hkv_l, cap, rb), dtype=torch.uint8, device=dev)
    vpool = torch.empty_like(kpool)
    _fill_decode_pools(ops, kpool, vpool, heads, toks, dev)
    new_k, new_v, qs = _step_inputs(n_steps + K, dev)
    h0, q0 = heads[0], heads[0] * (HQ // HKV)
    if mode == "kv":
        new_k, new_v = new_k[:, :, h0:h0 + hkv_l].contiguous(), new_v[:, :, h0:h0 + hkv_l].contiguous()
        qs = qs[:, :, q0:q0 + hq_l].contiguous()
    out = torch.empty((B, HQ, 1, D), dtype=torch.float16, device=dev)
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize()
    shard, nspl = None, 0
    if world > 1:
        from custom_kv.sharding import ShardedDecode
        shard = ShardedDecode(mode, pg, exchange=args.exchange)
        if mode == "seq":
            lens = [toks[1] - toks[0] + (g if grows else 0) for g in (0, growth)]
            nspl = max(ops.default_splits(B, HKV, s) for s in lens) + 1

    def local_len(seq_len):
        return seq_len - toks[0] if grows else toks[1] - toks[0]

    def step(i, seq_len, q=None, nk=None, nv=None, dst=None, events=None, append=True):
        """Append step i's token (at global position seq_len - 1), then
        decode at context length seq_len; the output lands in dst."""
        q = qs[i] if q is None else q
        nk = new_k[i] if nk is None else nk
        nv = new_v[i] if nv is None else nv
        dst = out if dst is None else dst
        if grows and append:
            ops.compress_pair_into(nk, nv, kpool, vpool, pos=local_len(seq_len) - 1, rotate=True)
        if events is not None:
            events[0].record(stream)
        if world == 1:
            ops.decode_attention(q, kpool, vpool, seq_len=seq_len, rotate_q=True, unrotate_out=True, out=dst)
            if events is not None:
                events[1].record(stream)
        else:
            shard.step(q, kpool, vpool, local_len(seq_len), num_splits=nspl, out=dst,
                       mark=events[1] if events is not None else None)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        import torch.distributed as dist
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    try:
        gpu_id = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        gpu_id = str(local)
    clk = ClockSampler(gpu_id).__enter__()  # up and sampling before the warm-up steps

    seq = CTX
    for i in range(W):
        seq += 1
        step(i, seq)
    barrier()

    # ---- timed region: K device-resident steps.  No event inside: an event
    # between two launches would keep the next kernel from starting early
    # (programmatic dependent launch).  With --graph the K steps are recorded
    # once as a CUDA graph (the same launches, lengths baked into each) and
    # the timed region is one replay: no host work per step ----
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    seq0 = seq
    graph = None
    if args.graph:
        # workspaces for the longest step exist before the capture
        ops._workspace(dev, ops.decode_workspace_size(B, hq_l, hkv_l, local_len(seq0 + K) + 64, 0) + (1 << 20))
        barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            s_ = seq0
            for i in range(K):
                s_ += 1
                step(W + i, s_)
    barrier()
    clk.mark_start()
    start.record(stream)
    h0 = time.perf_counter()
    if graph is not None:
        graph.replay()
        seq += K
    else:
        for i in range(K):
            seq += 1
            step(W + i, seq)
    host_ms = (time.perf_counter() - h0) * 1e3 / K  # host time to issue one step
    stop.record(stream)
    barrier()
    clk.mark_stop()
    clk.__exit__(None, None, None)
    total_ms = max_over_ranks(start.elapsed_time(stop))
    final = out.clone()
    final_seq = seq

    # ---- per-launch times for the roofline and the exchange: the same K
    # decode steps again (same lengths and queries, the tokens already
    # appended), one event pair around this rank's attention launches and one
    # more after the exchange ----
    ev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(K)]
    barrier()
    for i in range(K):
        step(W + i, seq0 + 1 + i, events=ev[i], append=False)
        ev[i][2].record(stream)
    barrier()
    dec_ms = sum(a.elapsed_time(b) for a, b, _ in ev) / K
    xch_ms = sum(b.elapsed_time(c) for _, b, c in ev) / K if world > 1 else 0.0

    mean_ctx = seq0 + (K + 1) / 2.0
    job_bytes_per_step = B * HKV * mean_ctx * 2 * rb
    rank_units = B * hkv_l * ((mean_ctx - toks[0]) if grows else float(toks[1] - toks[0]))
    value = job_bytes_per_step * K / (total_ms / 1e3) / 1e9
    tok_s = B * K / (total_ms / 1e3)
    achieved = rank_units * 2 * rb / (dec_ms / 1e3) / 1e9
    peak, peak_kind = peaks()
    clocks = clk.summary()

    # ---- sharded output against the one-GPU decode of the same rows ----
    shard_parity = None
    if world > 1:
        if rank == 0:
            fk = torch.empty((B, HKV, CTX + growth, rb), dtype=torch.uint8, device=dev)
            fv = torch.empty_like(fk)
            _fill_decode_pools(ops, fk, fv, list(range(HKV)), (0, CTX), dev)
            fnk, fnv, fqs = _step_inputs(n_steps + K, dev)
            for i in range(n_steps):
                ops.compress_pair_into(fnk[i], fnv[i], fk, fv, pos=CTX + i, rotate=True)
            one = ops.decode_attention(fqs[n_steps - 1], fk, fv, seq_len=final_seq, rotate_q=True,
                                       unrotate_out=True)
            d = (one.float() - final.float()).abs()
            ulp = (torch.nextafter(one.abs(), torch.full_like(one, float("inf"))) - one.abs()).float()
            shard_parity = {"rows": B * HQ, "max_abs_vs_one_gpu": d.max().item(),
                            "over_1e-3_plus_ulp": int((d > 1e-3 + ulp).sum().item()),
                            "note": "final timed step's gathered output vs the one-GPU decode of the same pools "
                                    "(different partition: rounding-level differences)"}
            del fk, fv, fnk, fnv, fqs, one
        barrier()

    # ---- e2e: host buffers in, result out, every step (reference-facing API) ----
    hq = torch.empty((K, B, hq_l if mode == "kv" else HQ, 1, D), dtype=torch.float16).pin_memory()
    hk = torch.empty((K, B, new_k.shape[2], 1, D), dtype=torch.float16).pin_memory()
    hv = torch.empty_like(hk).pin_memory()
    hq.copy_(qs[n_steps:].cpu())
    hk.copy_(new_k[n_steps:].cpu())
    hv.copy_(new_v[n_steps:].cpu())
    hout = torch.empty((K, B, HQ, 1, D), dtype=torch.float16).pin_memory()
    # Pipelined like a serving loop: a copy stream brings step i+1's inputs
    # in and step i's output out while step i computes; device inputs and
    # outputs are double-buffered.  Every step's copies are inside the timed
    # region, which runs from the first input copy to the last output copy
    # (both on the copy stream).
    cs = torch.cuda.Stream(dev)
    dq = [torch.empty(hq.shape[1:], dtype=torch.float16, device=dev) for _ in range(2)]
    dk = [torch.empty(hk.shape[1:], dtype=torch.float16, device=dev) for _ in range(2)]
    dv = [torch.empty(hk.shape[1:], dtype=torch.float16, device=dev) for _ in range(2)]
    dout = [torch.empty((B, HQ, 1, D), dtype=torch.float16, device=dev) for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(K)]
    ev_done = [torch.cuda.Event() for _ in range(K)]
    ev_out = [torch.cuda.Event() for _ in range(K)]

    def h2d(i):
        b = i % 2
        with torch.cuda.stream(cs):
            if i >= 2:
                cs.wait_event(ev_done[i - 2])  # step i-2 has read buffer b
            dq[b].copy_(hq[i], non_blocking=True)
            dk[b].copy_(hk[i], non_blocking=True)
            dv[b].copy_(hv[i], non_blocking=True)
            ev_in[i].record(cs)

    seq_e = seq
    barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(cs)
    h2d(0)
    for i in range(K):
        b = i % 2
        if i + 1 < K:
            h2d(i + 1)
        seq_e += 1
        stream.wait_event(ev_in[i])
        if i >= 2:
            stream.wait_event(ev_out[i - 2])  # step i-2's output has left buffer b
        step(None, seq_e, q=dq[b], nk=dk[b], nv=dv[b], dst=dout[b])
        ev_done[i].record(stream)
        with torch.cuda.stream(cs):
            cs.wait_event(ev_done[i])
            hout[i].copy_(dout[b], non_blocking=True)
            ev_out[i].record(cs)
    e2.record(cs)
    barrier()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2))
    mean_ctx_e = seq + (K + 1) / 2.0
    e2e = {"value": B * HKV * mean_ctx_e * 2 * rb * K / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
           "tok_s": B * K / (e2e_ms / 1e3), "ms_per_step": e2e_ms / K,
           "h2d_bytes_per_step": (dq[0].numel() + dk[0].numel() + dv[0].numel()) * 2,
           "d2h_bytes_per_step": dout[0].numel() * 2,
           "pipelining": "copy stream overlaps step i+1's input and step i's output copies with step i"
                         + ("; per rank: its own query heads / kv heads in, the whole output out"
                            if world > 1 else "")}

    # ---- compress throughput (8 KV heads x 131072 tokens, K and V) ----
    comp = None
    if world == 1 and not args.skip_compress:
        pools_host = None
        if rank == 0 and not args.skip_cpu:
            # the decode parity check of the CPU leg reads two batch rows of
            # the final timed step's pools (blocks beyond that length unused)
            pools_host = (kpool[[0, B - 1], :, :final_seq].cpu().numpy(),
                          vpool[[0, B - 1], :, :final_seq].cpu().numpy(),
                          qs[n_steps - 1][[0, B - 1]].cpu().numpy(), final[[0, B - 1]].float().cpu().numpy())
        del kpool, vpool
        torch.cuda.empty_cache()
        comp = compress_bench(ops, __import__("workloads"), dev, stream, K, peak, peak_kind)
    sample = comp.pop("_sample") if comp else None

    # ---- CPU leg (rank 0, one GPU): timed oracle baseline and the oracle parity check ----
    cpu, parity = None, None
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu = cpu_baseline(args.cpu_tokens)
        if sample is not None:
            parity = cpu_parity(pools_host, final_seq, sample)

    launches_per_step = {"single": 3, "kv": 3,
                         "seq": (1 if args.exchange == "p2p" else 2) + 1 + (1 if last else 0)}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": total_ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp16 MMA (split operands), fp32 accumulate", "data": "synthetic",
            "config": decode_config(world, mode, rb),
            "decode_tok_s": tok_s, "pct_peak": value / world / peak,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": DECODE_DRAM_BYTES_PER_UNIT * rank_units if rb == BLOCK else None,
                         "note": f"rank 0's decode (split partials + merge) per step: {2 * rb} B per (token, kv "
                                 f"head), {rank_units:.0f} units, timed per launch with CUDA events in a second "
                                 f"pass over the timed steps; traffic from ncu (per launch of the decode kernel); "
                                 f"peak {peak_kind}"},
            "rank0_ms": {"attention": dec_ms, "exchange": xch_ms, "host_issue": host_ms,
                         "note": "per step: attention and exchange by CUDA events around each launch in a second "
                                 "pass over the same steps; host_issue = host wall time to issue one step in the "
                                 "timed loop (a step is host-bound when it is not below ms_per_step)"},
            "gpu_launches": K * launches_per_step[mode], "cuda_graph": bool(args.graph),
            "clocks": clocks, "e2e": e2e, "compress": comp, "cpu_baseline": cpu, "parity": parity,
        }
        if world > 1:
            line["exchange"] = {("kv", "p2p"): "one kernel: merge of the split partials, fp16 output rows stored "
                                               "into every rank's buffer over NVLink (CUDA IPC), epoch-tagged words",
                                ("kv", "nccl"): "merge, then NCCL all-gather of the ranks' fp16 outputs",
                                ("seq", "p2p"): "one kernel: records stored into every rank's buffer over NVLink "
                                                "(CUDA IPC), epoch-tagged words, merge",
                                ("seq", "nccl"): "merge to records, NCCL all-gather, merge"}[(mode, args.exchange)]
            line["parity"] = shard_parity
        if comp:
            line["compress_tok_s"] = comp["tok_s"]
        print(json.dumps(line), flush=True)
    del graph  # a graph holding NCCL work is released before the process group
    if world > 1:
        import torch.distributed as dist
        torch.cuda.synchronize()
        if ops.device_status() != 0:  # a bounded wait gave up: the numbers are void
            raise RuntimeError(f"rank {rank}: device status {ops.device_status()}")
        shard.close()
        dist.barrier()
        dist.destroy_process_group()


def decode_config(world: int, mode: str, rb: int = BLOCK) -> dict:
    """The benchmark's config object (both arms print the same one)."""
    hkv_l = HKV // world if mode == "kv" else HKV
    toks = CTX // world if mode == "seq" else CTX
    rank_bytes = B * hkv_l * toks * 2 * rb
    return {"workload": f"decode step: B{B} Hq{HQ}/Hkv{HKV} D{D}, {CTX}-token compressed context growing 1 "
                        f"token/step, append + fused decode; the whole job on every N",
            "batch": B, "q_heads": HQ, "kv_heads": HKV, "head_dim": D, "context": CTX,
            "parallelism": {"single": "single", "kv": f"kv-head x{world}", "seq": f"seq-chunk x{world}"}[mode],
            "per_rank": f"{hkv_l} kv heads x {toks} tokens",
            "l2": f"pools {rank_bytes / 1e9:.2f} GB per rank " + (
                "> 126 MB L2 (no flush needed)" if rank_bytes > 126e6 else
                "(not larger than the 126 MB L2 at this N: every step re-reads the pools)"),
            "block_bytes": rb}


def cpu_parity(pools_host, seq_len, comp_sample):
    """Oracle checks of the benchmarked data (part of the CPU leg; nothing
    is timed here): the final timed decode step's
    output for two batch rows (all 32 query heads) against the oracle's
    decode of the same pools, and a sample of the compress benchmark's input
    against the oracle's blocks (bit for bit) with the count of elements
    within 1e-6 of a quantiser decision boundary."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ecc_oracle
    threads = len(os.sched_getaffinity(0))
    kb, vb, q, got = pools_host
    ref = ecc_oracle.decode(q, kb, vb, hkv=HKV, seq_len=seq_len, rotate_q=True, unrotate_out=True,
                            threads=threads)
    got = got.reshape(ref.shape)
    err = np.abs(got - ref)
    a = np.abs(ref.astype(np.float16))
    half_ulp = 0.5 * (np.nextafter(a, np.float16(np.inf)) - a).astype(np.float32)
    x16, blocks = comp_sample
    oracle_blocks = ecc_oracle.compress(x16, rotate=True, threads=threads)
    mism = int((oracle_blocks.reshape(-1, BLOCK) != blocks.reshape(-1, BLOCK)).any(axis=1).sum())
    return {"decode": {"rows": f"batch rows 0 and {B - 1}, {HQ} q heads, final step ({seq_len} tokens)",
                       "max_abs_err": float(err.max()), "elements": int(err.size),
                       "over_plain_2e-3": int((err > 2e-3).sum()),
                       "over_2e-3_plus_half_ulp": int((err > 2e-3 + half_ulp).sum())},
            "compress": {"vectors": int(x16.shape[0]), "blocks_differing": mism,
                         "elements_within_1e-6_of_a_boundary": ecc_oracle.count_ties(x16, rotate=True),
                         "note": "vectors of the compress benchmark's K input; oracle = compress_cpu restated"}}


LONG_B, LONG_CTX = 16, 131072


def run_long(args):
    """Long-context decode at the Llama-3.1-8B long-context shapes: batch 16,
    32 query heads over 8 kv heads, 131072-token compressed context per
    sequence; a step is one layer's decode attention (append the new K/V
    token, fused decode).  The work is split over the ranks (strong scaling,
    the total work is fixed as N grows):

    * ``--long kv``: rank r holds kv heads [8r/N, 8(r+1)/N) of every sequence
      and their query heads; attention needs no exchange, and one all-gather
      of the ranks' fp16 outputs assembles the layer's attention output.
    * ``--long seq``: rank r holds tokens [rL/N, (r+1)L/N) of every (b, kv head)
      row (the last rank also the appended ones); each rank merges its split
      partials into one record per (b, q head), the records are all-gathered
      and merged (LSE combine).
    """
    import torch
    import custom_ecc_cuda as ops
    import workloads

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    mode = args.long
    if HKV % world:
        raise SystemExit(f"--long: {world} ranks do not divide {HKV} kv heads")
    K, W = args.steps, args.warmup
    Bl = LONG_B
    hkv_l = HKV // world if mode == "kv" else HKV
    hq_l = HQ // world if mode == "kv" else HQ
    chunk_ctx = LONG_CTX if mode == "kv" else LONG_CTX // world
    last = rank == world - 1
    grows = mode == "kv" or last  # this rank appends the new tokens
    cap = chunk_ctx + W + K + 8
    gen = torch.Generator(device=dev).manual_seed(4321 + rank)
    kpool = torch.empty((Bl, hkv_l, cap, BLOCK), dtype=torch.uint8, device=dev)
    vpool = torch.empty_like(kpool)
    fill = 4096
    for t0 in range(0, chunk_ctx, fill):
        for pool in (kpool, vpool):
            x = torch.randn((Bl, hkv_l, fill, D), generator=gen, device=dev).half()
            ops.compress_into(x, pool, pos=t0, rotate=True)
            del x
    torch.cuda.synchronize()
    n = W + K
    new_k = torch.randn((n, Bl, hkv_l, 1, D), generator=gen, device=dev).half()
    new_v = torch.randn((n, Bl, hkv_l, 1, D), generator=gen, device=dev).half()
    # every rank draws the full query set of a step and keeps its heads
    qs = torch.stack([workloads.make_queries(i, Bl, HQ, device=dev) for i in range(n)])
    if mode == "kv":
        qs = qs[:, :, rank * hq_l:(rank + 1) * hq_l].contiguous()
    out = torch.empty((Bl, hq_l, 1, D), dtype=torch.float16, device=dev)
    stream = torch.cuda.current_stream(dev)
    if world > 1:
        import torch.distributed as dist
        from custom_kv.sharding import ShardedDecode
        shard = ShardedDecode(mode)
        nspl = max(ops.default_splits(Bl, HKV, s) for s in (chunk_ctx, cap)) + 1
        full = torch.empty((Bl, HQ, 1, D), dtype=torch.float16, device=dev)  # the layer's whole output

    def step(i, local_len, events=None):
        if grows:
            ops.compress_pair_into(new_k[i], new_v[i], kpool, vpool, pos=local_len - 1, rotate=True)
        if events is not None:
            events[0].record(stream)
        if world == 1:
            ops.decode_attention(qs[i], kpool, vpool, seq_len=local_len, rotate_q=True, unrotate_out=True, out=out)
            if events is not None:
                events[1].record(stream)
        else:
            shard.step(qs[i], kpool, vpool, local_len, num_splits=nspl, out=full,
                       mark=events[1] if events is not None else None)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    try:
        gpu_id = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        gpu_id = str(local)
    clk = ClockSampler(gpu_id).__enter__()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ln = chunk_ctx
    graph = None
    if args.graph:
        # every step one CUDA-graph replay: the append position, the local
        # length and the step's inputs come from device counters that the
        # recorded step advances itself
        pos_dev = torch.full((1,), chunk_ctx, dtype=torch.int32, device=dev)
        len_dev = torch.full((1,), chunk_ctx + (1 if grows else 0), dtype=torch.int32, device=dev)
        step_dev = torch.zeros((1,), dtype=torch.long, device=dev)
        if world > 1 and mode == "seq":
            nspl = max(nspl, ops.decode_dev_splits(Bl, HKV, cap))
        ws1 = torch.empty(ops.decode_dev_workspace_size(Bl, hq_l, hkv_l, cap), dtype=torch.uint8, device=dev)

        def body():
            q_i = torch.index_select(qs, 0, step_dev)[0]
            if grows:
                k_i = torch.index_select(new_k, 0, step_dev)[0]
                v_i = torch.index_select(new_v, 0, step_dev)[0]
                ops.compress_pair_at(k_i, v_i, kpool, vpool, pos_dev, rotate=True)
            if world == 1:
                ops.decode_attention_dev(q_i, kpool, vpool, len_dev, rotate_q=True, unrotate_out=True, out=out,
                                         workspace=ws1)
            else:
                shard.step(q_i, kpool, vpool, 0, num_splits=nspl, out=full, seq_len_dev=len_dev)
            if grows:
                pos_dev.add_(1)
                len_dev.add_(1)
            step_dev.add_(1)

        def reset():
            pos_dev.fill_(chunk_ctx)
            len_dev.fill_(chunk_ctx + (1 if grows else 0))
            step_dev.zero_()

        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(2):
                body()
        stream.wait_stream(side)
        barrier()
        reset()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            body()
        reset()
        for i in range(W):
            graph.replay()
        ln += W if grows else 0
        barrier()
        ln0 = ln
        clk.mark_start()
        start.record(stream)
        for i in range(K):
            graph.replay()
        stop.record(stream)
        ln += K if grows else 0
        barrier()
        dec_ms = None
    else:
        for i in range(W):
            ln += 1 if grows else 0
            step(i, ln)
        barrier()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
        ln0 = ln
        clk.mark_start()
        start.record(stream)
        for i in range(K):
            ln += 1 if grows else 0
            step(W + i, ln, ev[i])
        stop.record(stream)
        barrier()
        dec_ms = sum(a.elapsed_time(b) for a, b in ev) / K
    clk.mark_stop()
    clk.__exit__(None, None, None)
    total_ms = start.elapsed_time(stop)
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = t.item()
    # K + V blocks the whole job reads per step (mean over the timed steps)
    job_ctx = LONG_CTX + W + (K + 1) / 2.0
    job_bytes = Bl * HKV * job_ctx * 2 * BLOCK
    rank_ctx = (ln0 + (K + 1) / 2.0) if grows else float(chunk_ctx)
    rank_bytes = Bl * hkv_l * rank_ctx * 2 * BLOCK
    peak, peak_kind = peaks()
    if rank == 0:
        line = {
            "metric": "long-context ECC-INT4 decode attention: job HBM GB/s; decode tok/s", "value":
                job_bytes * K / (total_ms / 1e3) / 1e9, "unit": "GB/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": total_ms / K, "higher_is_better": True, "scaling": "strong", "dtype": "fp16 MMA (split operands), fp32 accumulate",
            "data": "synthetic",
            "config": {"workload": f"long-context decode step: B{Bl} Hq{HQ}/Hkv{HKV} D{D}, {LONG_CTX}-token "
                                   f"compressed context per sequence, one layer, append + fused decode",
                       "batch": Bl, "context": LONG_CTX,
                       "parallelism": {"kv": "kv-head", "seq": "seq-chunk"}[mode] if world > 1 else "single",
                       "per_rank": f"{hkv_l} kv heads x {chunk_ctx} tokens"},
            "decode_tok_s": Bl * K / (total_ms / 1e3),
            "rank0_decode_gbs": rank_bytes / (dec_ms / 1e3) / 1e9 if dec_ms else None,
            "cuda_graph": bool(args.graph), "peak": peak, "peak_kind": peak_kind,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    del graph  # a graph holding NCCL work is released before the process group
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU baseline / reference arm: the oracle port of the reference's CPU path
# ---------------------------------------------------------------------------
def _cpu_sample(tokens: int, seed: int = 0):
    import numpy as np
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ecc_oracle
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(1, HKV, tokens, D, generator=g).half().numpy()
    v = torch.randn(1, HKV, tokens, D, generator=g).half().numpy()
    kb = ecc_oracle.compress(k.reshape(-1, D), rotate=True).reshape(1, HKV, tokens, BLOCK)
    vb = ecc_oracle.compress(v.reshape(-1, D), rotate=True).reshape(1, HKV, tokens, BLOCK)
    q = torch.randn(1, HQ, 1, D, generator=g).half().numpy()
    return ecc_oracle, np, q, kb, vb


def cpu_baseline(tokens: int, min_seconds: float = 10.0):
    """Oracle decode (cpu_reference_decode restated in C, GQA) on one batch
    row x 8 KV heads x `tokens` tokens with all host threads, repeated until
    at least `min_seconds` of CPU work has been timed."""
    orc, np, q, kb, vb = _cpu_sample(tokens)
    threads = len(os.sched_getaffinity(0))
    orc.decode(q, kb[:, :, :64], vb[:, :, :64], hkv=HKV, seq_len=64, threads=threads)
    reps, t0 = 0, time.perf_counter()
    while True:
        orc.decode(q, kb, vb, hkv=HKV, seq_len=tokens, rotate_q=True, unrotate_out=True, threads=threads)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= min_seconds and reps >= 2:
            break
    gbs = HKV * tokens * 2 * BLOCK * reps / dt / 1e9
    return {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"oracle decode (C port of cpu_reference_decode) of 1 batch row x {HQ} q heads / {HKV} kv "
                      f"heads x {tokens} tokens, {reps} times ({dt:.1f} s)"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    orc, np, q, kb, vb = _cpu_sample(args.cpu_tokens)
    threads = len(os.sched_getaffinity(0))
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        orc.decode(q, kb, vb, hkv=HKV, seq_len=args.cpu_tokens, rotate_q=True, unrotate_out=True, threads=threads)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
    total = sum(times)
    gbs = HKV * args.cpu_tokens * 2 * BLOCK * len(times) / total / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic", "config": decode_config(world, "single" if world == 1 else args.shard),
            "decode_tok_s": 1.0 / (total / len(times)) * (args.cpu_tokens / CTX),
            "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": f"each step: oracle decode (C port of cpu_reference_decode) of 1 batch row "
                                       f"x {HQ} q heads / {HKV} kv heads x {args.cpu_tokens} tokens of this "
                                       f"workload, on {threads} host threads; GB/s per the same 256 B per "
                                       f"(token, kv head)"},
            "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-tokens", type=int, default=CTX)
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-compress", action="store_true")
    ap.add_argument("--shard", default="kv", choices=["kv", "seq"],
                    help="N > 1: split the decode job by kv head (default) or by sequence chunk")
    ap.add_argument("--exchange", default="p2p", choices=["nccl", "p2p"],
                    help="N > 1: how the ranks' results are combined: one kernel over peer memory (default), "
                         "or NCCL all-gather between merge kernels")
    ap.add_argument("--block-bytes", type=int, default=BLOCK, choices=[BLOCK, 96],
                    help="record size of the decode pools: the 128-byte block (default, the reference's "
                         "format) or the 96-byte record without the pad sector")
    ap.add_argument("--compress-only", action="store_true",
                    help="run only the compress benchmark and print its JSON object")
    ap.add_argument("--model-e2e", action="store_true",
                    help="run the Llama-3.1-8B-shaped 32k-prompt generate() comparison and print its JSON object")
    ap.add_argument("--prefill", action="store_true",
                    help="run one Llama-3.1-8B-shaped 32k-token prefill through the ECC cache (for ncu launch "
                         "lists of the prefill)")
    ap.add_argument("--long", choices=["kv", "seq"], default=None,
                    help="long-context decode (B16, 131072 tokens) sharded by kv head or by sequence chunk")
    ap.add_argument("--graph", choices=["auto", "on", "off"], default="auto",
                    help="decode benchmark: the K timed steps recorded once as a CUDA graph and replayed "
                         "(auto: with more than one GPU, where an eager step is bound by host issue time); with "
                         "--long: every step one CUDA-graph replay (device-side lengths)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    args.graph = args.graph == "on" or (args.graph == "auto" and world > 1 and not args.long)
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.compress_only:
        run_compress_only(args)
    elif args.model_e2e:
        run_model_e2e(args)
    elif args.prefill:
        run_prefill(args)
    elif args.long:
        run_long(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
