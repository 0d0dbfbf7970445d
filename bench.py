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

N > 1 GPUs (torchrun): sequence-chunk sharding, weak scaling -- every rank
holds its own 65536-token chunk of a context N x 65536 tokens long, computes
split partials, all-gathers them over NCCL and merges them (LSE combine).

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
# 65542 tokens, and of one compress launch of 8 x 131072 vectors, divided by the
# units each processed).
# Decode: per (token, kv head), algorithmic 256 B.  Compress: per vector,
# algorithmic 384 B; the output blocks of a launch partly stay in the 126 MB L2
# when the launch ends, so DRAM writes are counted below 128 B per vector.
DECODE_DRAM_BYTES_PER_UNIT = (1.074092e9 + 4.958208e6) / (B * HKV * 65542)
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


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import custom_ecc_cuda as ops
    import workloads

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist.group.WORLD
    K, W = args.steps, args.warmup
    cap = CTX + W + K + 2 * (K + W) + 8
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)

    # --- block pools filled by the compress kernel from seeded N(0,1) ---
    rb = args.block_bytes  # 128-byte blocks, or the 96-byte records of the option
    kpool = torch.empty((B, HKV, cap, rb), dtype=torch.uint8, device=dev)
    vpool = torch.empty_like(kpool)
    chunk = 8192
    for t0 in range(0, CTX, chunk):
        for pool in (kpool, vpool):
            x = torch.randn((B, HKV, chunk, D), generator=gen, device=dev).half()
            ops.compress_into(x, pool, pos=t0, rotate=True)
    torch.cuda.synchronize()

    n_steps = W + K
    new_k = torch.randn((n_steps, B, HKV, 1, D), generator=gen, device=dev).half()
    new_v = torch.randn((n_steps, B, HKV, 1, D), generator=gen, device=dev).half()
    qs = torch.stack([workloads.make_queries(i, B, HQ, device=dev) for i in range(n_steps)])
    out = torch.empty((B, HQ, 1, D), dtype=torch.float16, device=dev)
    # one rank: the library's default split count (the TMA kernel's balanced
    # partition for each step's length); sharded: a fixed count that covers
    # the partition of every length the run reaches
    splits = 0
    nspl = max(ops.default_splits(B, HKV, s) for s in (CTX, CTX + (cap - CTX) // 2, cap)) + 1
    stream = torch.cuda.current_stream(dev)

    if world > 1:
        import torch.distributed as dist
        from custom_kv.sharding import ShardedDecode
        # two-level combine: each rank merges its splits into one record
        # {m, l, o[128]} per (b, q head); one all-gather of the records
        shard = ShardedDecode("seq", pg, exchange=args.exchange)

    def step(i, seq_len, events=None):
        # append the new token (sharded run: the last rank owns the newest chunk)
        if world == 1 or rank == world - 1:
            ops.compress_pair_into(new_k[i], new_v[i], kpool, vpool, pos=seq_len - 1, rotate=True)
        if events is not None:
            events[0].record(stream)
        if world == 1:
            ops.decode_attention(qs[i], kpool, vpool, seq_len=seq_len, rotate_q=True, unrotate_out=True,
                                 num_splits=splits, out=out)
            if events is not None:
                events[1].record(stream)
        else:
            # ranks before the last hold a full, fixed chunk; the last rank's grows
            local_len = seq_len if rank == world - 1 else CTX
            shard.step(qs[i], kpool, vpool, local_len, num_splits=nspl, out=out,
                       mark=events[1] if events is not None else None)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

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

    # ---- timed region: K device-resident steps ----
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    seq0 = seq
    barrier()
    clk.mark_start()
    start.record(stream)
    for i in range(K):
        seq += 1
        step(W + i, seq, ev[i])
    stop.record(stream)
    barrier()
    clk.mark_stop()
    clk.__exit__(None, None, None)
    total_ms = start.elapsed_time(stop)
    dec_ms = [a.elapsed_time(b) for a, b in ev]
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = t.item()

    mean_ctx = seq0 + (K + 1) / 2.0
    # K + V blocks read per step: the last rank's chunk grows, the others' are CTX
    rank_ctx = mean_ctx if (world == 1 or rank == world - 1) else float(CTX)
    bytes_per_step = B * HKV * rank_ctx * 2 * rb
    job_bytes_per_step = B * HKV * ((world - 1) * CTX + mean_ctx) * 2 * rb
    value = job_bytes_per_step * K / (total_ms / 1e3) / 1e9
    tok_s = B * K / (total_ms / 1e3)
    dec_avg_ms = sum(dec_ms) / len(dec_ms)
    achieved = bytes_per_step / (dec_avg_ms / 1e3) / 1e9
    peak, peak_kind = peaks()
    clocks = clk.summary()

    # ---- e2e: host buffers in, result out, every step (reference-facing API) ----
    e2e = None
    if world == 1:
        hq = torch.empty((K, B, HQ, 1, D), dtype=torch.float16).pin_memory()
        hk = torch.empty((K, B, HKV, 1, D), dtype=torch.float16).pin_memory()
        hv = torch.empty_like(hk).pin_memory()
        hq.copy_(qs[W:].cpu())
        hk.copy_(new_k[W:].cpu())
        hv.copy_(new_v[W:].cpu())
        hout = torch.empty((K, B, HQ, 1, D), dtype=torch.float16).pin_memory()
        # Pipelined like a serving loop: a copy stream brings step i+1's
        # inputs in and step i's output out while step i computes; device
        # inputs and outputs are double-buffered.  Every step's copies are
        # inside the timed region, which runs from the first input copy to
        # the last output copy (both on the copy stream).
        cs = torch.cuda.Stream(dev)
        dq = [torch.empty((B, HQ, 1, D), dtype=torch.float16, device=dev) for _ in range(2)]
        dk = [torch.empty((B, HKV, 1, D), dtype=torch.float16, device=dev) for _ in range(2)]
        dv = [torch.empty((B, HKV, 1, D), dtype=torch.float16, device=dev) for _ in range(2)]
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
            ops.compress_pair_into(dk[b], dv[b], kpool, vpool, pos=seq_e - 1, rotate=True)
            ops.decode_attention(dq[b], kpool, vpool, seq_len=seq_e, rotate_q=True, unrotate_out=True,
                                 num_splits=splits, out=dout[b])
            ev_done[i].record(stream)
            with torch.cuda.stream(cs):
                cs.wait_event(ev_done[i])
                hout[i].copy_(dout[b], non_blocking=True)
                ev_out[i].record(cs)
        e2.record(cs)
        barrier()
        e2e_ms = s2.elapsed_time(e2)
        mean_ctx_e = seq + (K + 1) / 2.0
        e2e = {"value": B * HKV * mean_ctx_e * 2 * rb * K / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
               "tok_s": B * K / (e2e_ms / 1e3), "ms_per_step": e2e_ms / K,
               "h2d_bytes_per_step": (dq[0].numel() + dk[0].numel() + dv[0].numel()) * 2,
               "d2h_bytes_per_step": dout[0].numel() * 2,
               "pipelining": "copy stream overlaps step i+1's input and step i's output copies with step i"}

    # ---- compress throughput (8 KV heads x 131072 tokens, K and V) ----
    comp = None
    if world == 1 and not args.skip_compress:
        del kpool, vpool
        torch.cuda.empty_cache()
        comp = compress_bench(ops, workloads, dev, stream, K, peak, peak_kind)

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu = cpu_baseline(args.cpu_tokens)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": total_ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp32", "data": "synthetic",
            "config": {"workload": f"decode step: B{B} Hq{HQ}/Hkv{HKV} D{D}, {CTX}-token compressed context "
                                   f"per rank growing 1 token/step, append + fused decode",
                       "batch": B, "q_heads": HQ, "kv_heads": HKV, "head_dim": D, "context_per_rank": CTX,
                       "parallelism": "seq-chunk" if world > 1 else "single",
                       "num_splits": nspl if world > 1 else "default (balanced tile partition)",
                       "l2": f"inputs {B * HKV * CTX * 2 * rb / 1e9:.2f} GB/rank > L2 (no flush needed)",
                       "block_bytes": rb},
            "decode_tok_s": tok_s, "pct_peak": value / world / peak,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": DECODE_DRAM_BYTES_PER_UNIT * B * HKV * rank_ctx if rb == BLOCK else None,
                         "note": f"decode (split partials + merge) per step: {2 * rb} B per (token, kv head), "
                                 f"{B * HKV} (b, kv head) rows x mean {rank_ctx:.0f} tokens; traffic from ncu "
                                 f"(per launch of the decode kernel); peak {peak_kind}"},
            "gpu_launches": K * (3 if world == 1 else
                                 (2 if args.exchange == "p2p" else 3) + (1 if rank == world - 1 else 0)),
            "clocks": clocks, "e2e": e2e, "compress": comp, "cpu_baseline": cpu,
        }
        if world > 1:
            line["exchange"] = {"p2p": "one kernel: records stored into every rank's buffer over NVLink "
                                       "(CUDA IPC), epoch flags, merge",
                                "nccl": "merge to records, NCCL all-gather, merge"}[args.exchange]
        if comp:
            line["compress_tok_s"] = comp["tok_s"]
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        torch.cuda.synchronize()
        if args.exchange == "p2p":
            if ops.device_status() != 0:  # a bounded wait in the exchange gave up: the numbers are void
                raise RuntimeError(f"rank {rank}: peer exchange reported device status {ops.device_status()}")
            shard._peer.close()
        dist.barrier()
        dist.destroy_process_group()


LONG_B, LONG_CTX = 16, 131072
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
            "ms_per_step": total_ms / K, "higher_is_better": True, "scaling": "strong", "dtype": "fp32",
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
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": f"decode step sample: 1 batch row x Hq{HQ}/Hkv{HKV} D{D} x {args.cpu_tokens} "
                                   f"tokens of the {CTX}-token decode workload", "parallelism": "host threads"},
            "decode_tok_s": 1.0 / (total / len(times)) * (args.cpu_tokens / CTX),
            "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": f"oracle decode (C port of cpu_reference_decode) per step: 1 row x "
                                       f"{args.cpu_tokens} tokens"},
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
    ap.add_argument("--exchange", default="p2p", choices=["nccl", "p2p"],
                    help="N > 1: how the ranks' records are combined (NCCL all-gather, or one kernel over "
                         "peer memory)")
    ap.add_argument("--block-bytes", type=int, default=BLOCK, choices=[BLOCK, 96],
                    help="record size of the decode pools: the 128-byte block (default, the reference's "
                         "format) or the 96-byte record without the pad sector")
    ap.add_argument("--compress-only", action="store_true",
                    help="run only the compress benchmark and print its JSON object")
    ap.add_argument("--model-e2e", action="store_true",
                    help="run the Llama-3.1-8B-shaped 32k-prompt generate() comparison and print its JSON object")
    ap.add_argument("--long", choices=["kv", "seq"], default=None,
                    help="long-context decode (B16, 131072 tokens) sharded by kv head or by sequence chunk")
    ap.add_argument("--graph", action="store_true",
                    help="with --long: every step one CUDA-graph replay (device-side lengths)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.compress_only:
        run_compress_only(args)
    elif args.model_e2e:
        run_model_e2e(args)
    elif args.long:
        run_long(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
