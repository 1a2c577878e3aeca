#!/usr/bin/env python
"""Decode throughput of the 102.45M SparDA model on B200 with the forecast-guided
block-sparse attention path (batch 64 per GPU, 16K cached
tokens, block 64, top-k 8, bf16), plus the roofline of the fused decode kernel.

    python bench.py [--gpus N --steps K --warmup W]              # this build
    python bench.py --impl reference [--steps K --warmup W]      # the reference's
                                                                 # algorithm on the host CPU
N > 1 runs under torchrun, one rank per GPU, each rank decoding its own batch of
64 sequences (batch sharding, no collective on the hot path).

A step is one greedy decode step of every sequence: 12 layers of fused
(RoPE + KV append + compressor update + forecast selection + block-sparse
attention) kernels around cuBLAS projections/FFN, the tied LM head and argmax,
replayed as one CUDA graph.  The cache is pre-filled with seeded N(0,1) keys and
values (random-init weights, synthetic data).  The decode position cycles
through one 64-token window starting at the 16K context (lengths are rewound
every 64 steps), so every timed step decodes at 16,385..16,448 cached tokens.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "decode tok/s (B=64, 16K ctx) + sparse-attn HBM GB/s vs peak, at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4096)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=16384)
    ap.add_argument("--rule", choices=["reference", "absolute"], default="absolute")
    ap.add_argument("--window", type=int, default=64)
    ap.add_argument("--prefill", action="store_true",
                    help="BASELINE config 3: prefill of one --ctx-token sequence (e.g. --ctx 32768) through the "
                         "12-layer model; roofline of the tensor-core block-sparse prefill attention")
    ap.add_argument("--offload", action="store_true",
                    help="BASELINE config 5 sample: K/V rows in pinned host memory, forecast-guided prefetch of the "
                         "selected blocks into device slots (use with e.g. --ctx 32768)")
    ap.add_argument("--cache-blocks", type=int, default=None,
                    help="with --offload: device slots per (sequence, kv head) for selected blocks (top-k..32; more "
                         "than top-k make them a block cache with least-recently-used replacement)")
    ap.add_argument("--selection", choices=["kernel", "side-stream", "chain"], default="chain",
                    help="forecast selection inside the fused decode kernel, layer L+1's candidates computed on a "
                         "side stream during layer L, or at the end of layer L's fused kernel")
    ap.add_argument("--pdl", choices=["on", "off"], default="off",
                    help="programmatic dependent launch of the library's decode-step kernels")
    ap.add_argument("--projections", choices=["cublas", "tc"], default="cublas",
                    help="decode-step projections: cuBLAS GEMMs with the library's RMSNorm and SwiGLU kernels, or "
                         "the library's fused tensor-core projections (sd_linear)")
    ap.add_argument("--e2e-steps", type=int, default=1024)
    ap.add_argument("--probe-steps", type=int, default=64)
    ap.add_argument("--cpu-seqs", type=int, default=1, help="sequences per CPU worker thread")
    ap.add_argument("--kernels-only", action="store_true",
                    help="only the standalone kernel measurements (compressor, gather, prefill selector and list "
                         "builder at BASELINE sizes), one JSON line; for profiler captures of those kernels")
    ap.add_argument("--backward", action="store_true",
                    help="only the block-sparse attention backward (sd_prefill_attention_backward) and its forward "
                         "on one --ctx-token sequence (12 query / 4 kv heads, bf16, the masked forecast lists up to "
                         "8192 tokens, chunked above), one JSON line; for training-path timing and profiler captures")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the config-3 prefill and standalone-kernel sub-measurements of the default run")
    ap.add_argument("--cpu-budget-s", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=12,
                    help="layers of the model (12 = the benchmark model; fewer only for small profiler captures)")
    return ap.parse_args()


# ------------------------------------------------------------------ helpers
def read_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def read_traffic(kernel_tag: str):
    """DRAM bytes per launch of the fused decode kernel from the committed ncu
    summary (profiles/), or None."""
    path = os.path.join(REPO, "profiles", "decode_layer_b64_ctx16k.md")
    try:
        txt = open(path).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples every 200 ms while running."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(parts)
            except Exception:
                pass
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "", 1).isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "", 1).isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def gpu_id_for(dev_index: int) -> str:
    import torch
    try:
        u = str(torch.cuda.get_device_properties(dev_index).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(dev_index)


# ------------------------------------------------------------------ CPU leg
def cpu_reference(ctx: int, seqs: int, budget_s: float, rule: str, max_steps: int = 1000, warmup: int = 1,
                  workers: int = 0):
    """The reference's decode-step algorithm (oracle restatement, numpy fp32)
    on the host cores: full 12-layer model at ``ctx`` cached tokens, O(T)
    block compression every layer and step as the reference does
    (model/attention/sparse.py:134-135).

    Every host core is used whatever the launcher set (torchrun exports
    OMP_NUM_THREADS=1): ``workers`` threads (default: all cores, at most 32)
    each decode their own ``seqs`` sequences with their own caches, BLAS pools
    pinned to one thread each so the cores are not oversubscribed (numpy
    releases the GIL inside its kernels).  The reported rate is sequences
    decoded per second over all workers; it does not depend on the batch the
    GPU arm runs, because each sequence's step is independent work."""
    import concurrent.futures as cf

    import numpy as np
    from oracle import sparda_oracle as O
    from oracle.synthetic import SmallModelConfig, model_state
    try:
        from threadpoolctl import threadpool_limits
    except Exception:
        threadpool_limits = None
    workers = workers or min(os.cpu_count() or 1, 32)
    cfg = SmallModelConfig(vocab_size=32000, n_layer=12)
    m = O.OracleModel(model_state(cfg, seed=0), n_layer=12, block_size=64, top_k=8, max_seq_len=ctx + 64,
                      rule=rule, dtype=np.float32)
    rng = np.random.default_rng(5)
    kc0 = [rng.standard_normal((seqs, 4, ctx + 64, 64), dtype=np.float32) for _ in range(12)]
    vc0 = [rng.standard_normal((seqs, 4, ctx + 64, 64), dtype=np.float32) for _ in range(12)]
    state = [([c.copy() for c in kc0], [c.copy() for c in vc0], rng.integers(0, cfg.vocab_size, size=seqs))
             for _ in range(workers)]
    del kc0, vc0

    def one(w):
        kc, vc, ids = state[w]
        logits = m.decode_step(ids, kc, vc, ctx)  # fixed position: each step decodes token ctx
        state[w] = (kc, vc, logits.argmax(-1))

    import contextlib
    limits = threadpool_limits(limits=1) if threadpool_limits is not None else contextlib.nullcontext()
    with limits, cf.ThreadPoolExecutor(max_workers=workers) as ex:
        times = []
        t_start = time.perf_counter()
        i = 0
        while i < max_steps + warmup:
            t0 = time.perf_counter()
            list(ex.map(one, range(workers)))
            if i >= warmup:
                times.append(time.perf_counter() - t0)
            i += 1
            if time.perf_counter() - t_start > budget_s and len(times) >= 2:
                break
    step_s = statistics.mean(times)
    total = seqs * workers
    return {"value": total / step_s, "unit": "tok/s", "cores": int(workers), "kind": "port",
            "sample": f"{workers} threads x {seqs} sequence(s) each = {total} sequences x {len(times)} decode steps "
                      f"at {ctx} cached tokens, 12 layers, fp32 numpy (oracle/sparda_oracle.py OracleModel, the "
                      f"reference algorithm restated; the reference's own PyTorch code cannot travel to the GPU "
                      f"box); rate = sequences decoded per second, independent of the GPU arm's batch",
            "step_s": step_s, "steps": len(times), "sequences": total}


# ------------------------------------------------------------------ GPU leg
def run_b200(args, rank, world, local):
    import torch
    import torch.distributed as dist

    from local_research_small_language_model_b200 import ModelConfig, ops
    from local_research_small_language_model_b200.model import DecodeEngine, SparDAB200Model

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.manual_seed(1234 + rank)
    ops.set_programmatic_launch(args.pdl == "on")
    B, ctx, W = args.batch, args.ctx, args.window
    cfg = ModelConfig(block_size=64, top_k_blocks=8, context_length=4096, selector_rule=args.rule,
                      n_layer=args.layers)
    model = SparDAB200Model(cfg).to(dev, torch.bfloat16).eval()
    for layer in model.layers:
        layer.use_tc_linear = args.projections == "tc"
    caches = model.allocate_caches(B, ctx + W + 64, selection=args.selection, offload=args.offload,
                                   cache_blocks=args.cache_blocks if args.offload else None)
    gen = torch.Generator(device=dev)
    gen.manual_seed(99 + rank)
    with torch.no_grad():
        for c in caches:
            if args.offload:  # one prompt per layer: host store, block sums and slots
                k = torch.randn(B, ctx, 4, 64, generator=gen, device=dev, dtype=torch.bfloat16)
                v = torch.randn(B, ctx, 4, 64, generator=gen, device=dev, dtype=torch.bfloat16)
                c.update(k, v)
                del k, v
                continue
            for s in range(0, ctx, 2048):
                n = min(2048, ctx - s)
                k = torch.randn(B, n, 4, 64, generator=gen, device=dev, dtype=torch.bfloat16)
                v = torch.randn(B, n, 4, 64, generator=gen, device=dev, dtype=torch.bfloat16)
                c.update(k, v)
    torch.cuda.synchronize()

    def rewind(delta):
        model._lens.sub_(delta)
        for c in caches:
            c.current_len -= delta

    plain = DecodeEngine(model, caches, B)
    plain.ids.random_(0, cfg.vocab_size)
    plain.capture()

    # instrumented twin: timing events around each layer's fused kernel and its
    # selected lists, for the roofline numerator
    probes = []
    for layer in model.layers:
        p = {"start": torch.cuda.Event(enable_timing=True, external=True),
             "end": torch.cuda.Event(enable_timing=True, external=True),
             "cstart": torch.cuda.Event(enable_timing=True, external=True),
             "cend": torch.cuda.Event(enable_timing=True, external=True),
             "sel": torch.full((B, 4, 16), -1, dtype=torch.int32, device=dev),
             "cnt": torch.zeros(B, 4, dtype=torch.int32, device=dev)}
        if args.offload:  # the compute stream's wait for the layer's prefetch
            p["wstart"] = torch.cuda.Event(enable_timing=True, external=True)
            p["wend"] = torch.cuda.Event(enable_timing=True, external=True)
        layer.probe = p
        probes.append(p)
    inst = DecodeEngine(model, caches, B)
    inst.ids.copy_(plain.ids)
    inst.capture()
    for layer in model.layers:
        layer.probe = None

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.no_grad():
        # warm-up, then back to the start of the window
        for i in range(args.warmup):
            plain.step()
        rewind(caches[0].current_len - ctx)
        torch.cuda.synchronize()

        # ---- timed: device-resident inputs, graph replays back to back
        clocks = ClockSampler(gpu_id_for(local))
        clocks.start()
        barrier()
        torch.cuda.synchronize()
        stats0 = sum(c.stats.clone() for c in caches) if args.offload else None
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for i in range(args.steps):
            plain.step()
            if (i + 1) % W == 0:
                rewind(W)
        ev1.record()
        torch.cuda.synchronize()
        barrier()
        clock_info = clocks.stop()
        ms = max_over_ranks(ev0.elapsed_time(ev1))
        stats1 = sum(c.stats.clone() for c in caches) if args.offload else None
        rewind(caches[0].current_len - ctx)

        # ---- e2e: the public API with host buffers, greedy loop that reads
        # every step's tokens on the host
        host_ids = torch.randint(0, cfg.vocab_size, (B, 1), dtype=torch.long).pin_memory()
        host_next = torch.empty(B, 1, dtype=torch.long).pin_memory()
        ke = min(args.e2e_steps, args.steps)
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(ke):
            plain.ids.copy_(host_ids, non_blocking=True)
            plain.step()
            host_next.copy_(plain.next_ids, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            host_ids.copy_(host_next)
            if (i + 1) % W == 0:
                rewind(W)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1))
        rewind(caches[0].current_len - ctx)

        # ---- roofline of the fused decode kernel (instrumented graph)
        side = args.selection == "side-stream"
        chain = args.selection == "chain"
        k_ms, k_bytes, k_launch = 0.0, 0.0, 0
        w_ms = 0.0
        c_ms, c_bytes, c_launch = 0.0, 0.0, 0
        np_ = __import__("numpy")
        for i in range(args.probe_steps):
            inst.step()
            torch.cuda.synchronize()
            L = caches[0].current_len  # tokens after the step (the new one included)
            nb = (L + 63) // 64
            for li, p in enumerate(probes):
                k_ms += p["start"].elapsed_time(p["end"])
                if args.offload:
                    w_ms += p["wstart"].elapsed_time(p["wend"])
                k_launch += 1
                sel = p["sel"].cpu().numpy()
                cnt = p["cnt"].cpu().numpy()
                rows = 0
                for (b_, h_), c_ in np_.ndenumerate(cnt):
                    for j in sel[b_, h_, :c_]:
                        rows += min(64, L - int(j) * 64)
                n_sc = (nb - 1) if args.rule == "absolute" else 1  # cached sums scored (current one in smem)
                k_bytes += (rows * 64 * 2 * 2            # selected K and V rows (bf16)
                            + B * (1280 + 256 + 768) * 2  # q|k|v in, forecast in, attention out
                            + B * 4 * 64 * 2 * 2         # new K and V rows written
                            + B * 4 * 64 * 4 * 2)        # current block's running sum read + write
                if li > 0:  # forecast-driven layers
                    k_bytes += B * 4 * 8 * 8 if (side or chain) else B * 4 * n_sc * 64 * 4  # candidates, or sums
                if chain and li + 1 < len(probes):  # the next layer's candidates, computed by this kernel
                    k_bytes += B * 4 * (n_sc * 64 * 4 + 64 * 2 + 8 * 8)
                if (side or args.offload) and li + 1 < len(probes):  # layer li+1's candidates (+ prefetch)
                    c_ms += p["cstart"].elapsed_time(p["cend"])
                    c_launch += 1
                    c_bytes += B * 4 * (n_sc * 64 * 4 + 64 * 2 + 8 * 8)  # fp32 sums scored, forecast, output
            if (i + 1) % W == 0:
                rewind(W)
        rewind(caches[0].current_len - ctx)
        ops.check_device_errors(dev)
        kern_only = None
        if chain and not args.offload:
            kern_only = decode_kernels_graph_us(model, caches, args, dev)
        ops.check_device_errors(dev)

    value = world * B * args.steps / (ms / 1000.0)
    e2e = world * B * ke / (e2e_ms / 1000.0)
    hbm, src = read_peaks()
    in_step_s = k_ms / 1000.0 / k_launch
    # the kernel's duration: from the graph of the decode kernels alone when
    # measured (events around every launch inside the step add their own
    # nodes), else from the per-launch events of the instrumented step
    avg_launch_s = kern_only / 1e6 if kern_only else in_step_s
    bytes_per_launch = k_bytes / k_launch
    c_avg_s = c_ms / 1000.0 / max(c_launch, 1)
    c_gbs = (c_bytes / max(c_launch, 1)) / c_avg_s / 1e9 if c_launch else None
    achieved = bytes_per_launch / avg_launch_s / 1e9
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "BASELINE config 2: 102.45M SparDA decode step, random-init N(0,0.02) weights, "
                               "seeded N(0,1) bf16 KV pre-fill",
                   "model": "SparDA-102.45M (12L, 768, 12q/4kv x 64, SwiGLU 2048, vocab 32000)",
                   "global_batch": B * world, "per_gpu_batch": B, "seq_len": ctx,
                   "ctx_window": [ctx + 1, ctx + W], "block_size": 64, "top_k": 8,
                   "selector_rule": args.rule, "selection": args.selection, "pdl": args.pdl,
                   "projections": args.projections,
                   "parallelism": f"batch-shard x{world}, no collective",
                   "l2": "no flush: per-step working set (~0.9 GB of weights, prototypes and selected KV) "
                         "exceeds the 126 MB L2"},
        "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": B * 8, "d2h_bytes_per_step": B * 8,
                "steps": ke, "note": "pinned host token ids in, argmax ids out and read on the host every step"},
        # per step: fused decode (12) + side-stream candidates (11, side-stream
        # selection only) + RMSNorm (25) + SwiGLU gate (12) + length bump (1)
        # kernels of libspardab200.so
        "gpu_launches": args.steps * (cfg.n_layer + (cfg.n_layer - 1 if side else 0) + (2 * cfg.n_layer + 1)
                                      + cfg.n_layer + 1),
        "roofline": {"bound": "hbm", "kernel": "sd::decode_layer_kernel<bf16,bf16,3>",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "peak_source": src,
                     "traffic": read_traffic("decode_layer"),
                     "bytes_per_launch": round(bytes_per_launch), "avg_launch_us": round(avg_launch_s * 1e6, 3),
                     "duration_source": ("CUDA events around replays of a graph holding the 12 layers' fused "
                                         "decode kernels alone (the step's caches, chained candidates), / 12"
                                         if kern_only else "CUDA events around each launch in the step graph"),
                     "in_step_event_us": round(in_step_s * 1e6, 3),
                     "in_step_frac": round(bytes_per_launch / in_step_s / 1e9 / hbm, 4),
                     "launches_sampled": k_launch,
                     "selector_kernel": {"kernel": "sd::decode_candidates_kernel<bf16> (side stream)",
                                         "achieved": round(c_gbs, 1) if c_gbs else None, "unit": "GB/s",
                                         "frac": round(c_gbs / hbm, 4) if c_gbs else None,
                                         "bytes_per_launch": round(c_bytes / max(c_launch, 1)),
                                         "avg_launch_us": round(c_avg_s * 1e6, 3), "launches_sampled": c_launch}
                     if side else None,
                     "path": {"achieved": round((k_bytes + c_bytes) / ((k_ms + c_ms) / 1000.0) / 1e9, 1),
                              "note": "decode + candidate kernels' algorithmic bytes over their summed time"}},
        "clocks": clock_info,
    }
    if args.offload:
        wanted, hits, h2d = (float(x) for x in (stats1 - stats0).tolist())
        result["metric"] = "KV-offload decode tok/s (BASELINE config 5 sample)"
        result["config"]["workload"] = (f"BASELINE config 5 sample: {B} sequences per GPU at {ctx} cached tokens, "
                                        "K/V in pinned host memory, forecast-guided prefetch into device slots")
        result["offload"] = {
            "host_store_gb": round(sum(2 * c.host_k.numel() * c.host_k.element_size() for c in caches) / 1e9, 2),
            "h2d_bytes_per_step": round(h2d / args.steps),
            "h2d_gbs": round(h2d / (ms / 1000.0) / 1e9, 2),
            "device_slots_per_head": caches[0].kslots,
            "prefetch_hit_rate": round(hits / wanted, 4) if wanted else None,
            "exposed_wait_us_per_step": round(w_ms * 1000.0 / max(args.probe_steps, 1), 2),
            "prefetch_us_per_layer": round(c_ms * 1000.0 / max(c_launch, 1), 2),
            "note": "exposed wait = compute-stream time blocked on the layers' prefetch events (instrumented "
                    "graph); prefetch time includes the candidate kernel"}
    return result


def decode_kernels_graph_us(model, caches, args, dev, reps: int = 20, warm: int = 3) -> float:
    """Average duration (us) of one fused decode-layer launch: CUDA events
    around replays of a graph that holds only the layers' fused decode kernels,
    chained as in the step (layer L's kernel computes layer L+1's candidates;
    layer 0 takes the static window), on the step's own caches at the first
    position of the timed window, with random projection rows.  Every replay
    rewrites the same new token; the block sums it touches are restored after."""
    import torch
    from local_research_small_language_model_b200 import ops
    B = args.batch
    n = len(model.layers)
    a0 = model.layers[0].attention
    nq = (a0.n_head + 2 * a0.n_kv_head) * a0.head_dim
    fd = model.config.forecast_heads * model.config.forecast_dim
    g = torch.Generator(device=dev).manual_seed(77)
    proj = [torch.randn(B, nq + fd, generator=g, device=dev, dtype=torch.bfloat16) for _ in range(n)]
    for c in caches:
        if getattr(c, "cand", None) is None:
            c.cand = (torch.empty(B, a0.n_kv_head, a0.top_k_blocks, dtype=torch.int32, device=dev),
                      torch.empty(B, a0.n_kv_head, a0.top_k_blocks, dtype=torch.float32, device=dev))
    j = caches[0].current_len // a0.block_size
    snap = [c.proto_sum[:, :, j].clone() for c in caches]
    cos, sin = model.rotary_emb.cos, model.rotary_emb.sin

    def body():
        for li, layer in enumerate(model.layers):
            a, c = layer.attention, caches[li]
            nxt = (caches[li + 1].proto_sum, proj[li][:, nq:], caches[li + 1].cand) if li + 1 < n else None
            ops.decode_layer(proj[li][:, :nq], proj[li - 1][:, nq:] if li > 0 else None, cos, sin, c.len_dev,
                             c.k_store, c.v_store, c.proto_sum, a.n_head, a.n_kv_head, a.block_size, a.top_k_blocks,
                             a.rule, cand=c.cand if li > 0 else None, next_cand=nxt)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        body()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        body()
    for _ in range(warm):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (reps * n)
    for c, r in zip(caches, snap):
        c.proto_sum[:, :, j].copy_(r)
    del graph
    torch.cuda.synchronize()
    return us


def prefill_flops(lists, counts, T, G, causal=True):
    """Algorithmic attention FLOPs of one prefill: 4*D per valid (query head,
    query, key) triple of the block lists (QK^T and PV, 2 flops per MAC)."""
    import numpy as np
    lists = lists.cpu().numpy()
    counts = counts.cpu().numpy()
    total = 0
    b_, h_, nqt, _ = lists.shape
    for ib in range(b_):
        for ih in range(h_):
            for qt in range(nqt):
                q0, q1 = qt * 64, min(T, qt * 64 + 64)
                tq = np.arange(q0, q1)
                for j in lists[ib, ih, qt, :counts[ib, ih, qt]]:
                    if j < 0:
                        continue
                    k0, k1 = j * 64, min(T, j * 64 + 64)
                    if causal:
                        total += int(np.clip(np.minimum(tq + 1, k1) - k0, 0, None).sum())
                    else:
                        total += (q1 - q0) * (k1 - k0)
    return 4 * 64 * G * total


def run_prefill(args, rank, world, local):
    import torch
    from local_research_small_language_model_b200 import ModelConfig, ops
    from local_research_small_language_model_b200.model import SparDAB200Model
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.manual_seed(1234 + rank)
    T = args.ctx
    cfg = ModelConfig(block_size=64, top_k_blocks=8, context_length=4096, n_layer=args.layers)
    model = SparDAB200Model(cfg).to(dev, torch.bfloat16).eval()
    caches = model.allocate_caches(1, T + 64)
    gen = torch.Generator(device="cpu").manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (1, T), generator=gen).to(dev)
    with torch.no_grad():
        def step():
            for c in caches:
                c.reset()
            return model(ids, kv_caches=caches)["logits"]
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        clocks = ClockSampler(gpu_id_for(local))
        clocks.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        clock_info = clocks.stop()
        ms = max_over_ranks_simple(e0.elapsed_time(e1))
        # the attention kernel alone on one layer's shapes (chunked forecast lists)
        q = torch.randn(1, T, 12, 64, device=dev, dtype=torch.bfloat16)
        k = torch.randn(1, 4, T, 64, device=dev, dtype=torch.bfloat16)
        v = torch.randn(1, 4, T, 64, device=dev, dtype=torch.bfloat16)
        f = torch.randn(1, T, 4, 64, device=dev, dtype=torch.bfloat16)
        reps = ops.compress_blocks(k.transpose(1, 2), 64)
        _, topk = ops.select_blocks(f, reps, 8, 64, False)
        lists, counts = ops.prefill_lists("chunked_forecast", 1, 4, T, 64, 8, topk, True, device=dev)
        for _ in range(3):
            ops.prefill_attention(q, k, v, lists, counts, 64, None, True)
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps_n = 10
        a0.record()
        for _ in range(reps_n):
            ops.prefill_attention(q, k, v, lists, counts, 64, None, True)
        a1.record()
        torch.cuda.synchronize()
        att_s = a0.elapsed_time(a1) / 1000.0 / reps_n
    flops = prefill_flops(lists, counts, T, 3)
    peak = read_peak_tflops()
    achieved = flops / att_s / 1e12
    value = world * args.steps * T / (ms / 1000.0)
    return {
        "metric": "prefill tok/s (BASELINE config 3: one 32K-token sequence, 12 layers)", "value": round(value, 1),
        "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"BASELINE config 3: prefill of one {T}-token sequence of uniform random ids, "
                               "random-init 102.45M model, chunked block-sparse path, block 64, top-k 8",
                   "seq_len": T, "layers": args.layers},
        "roofline": {"bound": "tensor", "kernel": "sd::prefill_tc_kernel<bf16> (chunked forecast lists, one layer)",
                     "achieved": round(achieved, 2), "peak": peak[0], "unit": "TFLOP/s",
                     "frac": round(achieved / peak[0], 4), "peak_source": peak[1],
                     "flops_per_launch": flops, "avg_launch_us": round(att_s * 1e6, 2), "traffic": None},
        "clocks": clock_info,
    }


def _event_time_s(fn, reps=10, warm=3):
    """Average device time of fn() over `reps` launches (CUDA events on the
    current stream, after `warm` untimed calls)."""
    import torch
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1000.0 / reps


def _graph_time_s(fns):
    """Average device time per call of the calls fns[i]() captured back to
    back in one CUDA graph (no host launch gaps between them), from one timed
    replay after a warm one."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for fn in fns:
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for fn in fns:
            fn()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / 1000.0 / len(fns)


def run_backward(args, local: int):
    """Event-timed attention backward and forward of one prefill layer's
    shapes.  Per listed key block, query block and head the backward runs
    seven 64x64x64 products on the tensor cores (mma.sync): S and dP in both
    passes, and dQ, dK, dV twice each (bf16 high and low parts of P and dS)."""
    import torch
    from local_research_small_language_model_b200 import ops
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(0)
    T, hq, hkv = args.ctx, 12, 4
    q = torch.randn(1, T, hq, 64, generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn(1, hkv, T, 64, generator=g, device=dev, dtype=torch.bfloat16)
    v = torch.randn(1, hkv, T, 64, generator=g, device=dev, dtype=torch.bfloat16)
    go = torch.randn(1, T, hq, 64, generator=g, device=dev, dtype=torch.bfloat16)
    f = torch.randn(1, T, hkv, 64, generator=g, device=dev, dtype=torch.bfloat16)
    chunked = T > 8192
    reps = ops.compress_blocks(k.transpose(1, 2).contiguous(), 64)
    _, topk = ops.select_blocks(f, reps, 8, 64, not chunked, return_scores=False)
    mode = "chunked_forecast" if chunked else "masked_forecast"
    lists, counts = ops.prefill_lists(mode, 1, hkv, T, 64, 8, topk, True, device=dev)
    row_topk = None if chunked else topk
    bwd_s = _event_time_s(lambda: ops.prefill_attention_backward(q, k, v, go, lists, counts, 64, row_topk, True))
    fwd_s = _event_time_s(lambda: ops.prefill_attention(q, k, v, lists, counts, 64, row_topk, True))
    ops.check_device_errors(dev)
    blocks = int(counts.clamp_min(0).sum().item()) * (hq // hkv)
    per_product = 2 * 64 ** 3
    flops = blocks * 7 * per_product  # S and dP in both passes, dQ, dK, dV
    mma = blocks * (4 + 2 * 3) * per_product  # dQ, dK, dV run twice (bf16 high and low parts of P / dS)
    peak = read_peak_tflops()
    return {"kernel": "sd::bwd::prefill_bwd_tc_kernel<bf16, true> (sd_prefill_attention_backward)",
            "mode": mode, "seq_len": T, "us": round(bwd_s * 1e6, 2), "forward_us": round(fwd_s * 1e6, 2),
            "flops": flops, "tflops": round(flops / bwd_s / 1e12, 2), "mma_flops": mma,
            "mma_tflops": round(mma / bwd_s / 1e12, 2), "peak_bf16_tflops": peak[0],
            "frac": round(mma / bwd_s / 1e12 / peak[0], 4), "peak_source": peak[1],
            "bound": "mma.sync chains per 64-key block (legacy tensor path, 8 warps per CTA), the exponentials, "
                     "fp32 atomics of dK / dV; at small T too few CTAs"}


def run_kernels(local: int):
    """Standalone device time of the path's other kernels on BASELINE-sized
    inputs, against the HBM roofline (algorithmic bytes per launch / time):
    the compressor over one config-2 layer cache (64 x 16,384 tokens, bf16),
    the block gather of 10 blocks per (sequence, kv head) from that cache, the
    config-3 prefill selector (32,768 forecast rows x 512 blocks, fp32 scores +
    top-8 in registers; fp32 CUDA-core bound) and the config-3 block-list
    builder.  Inputs exceed the 126 MB L2 except the selector's, whose bound is
    arithmetic."""
    import torch
    from local_research_small_language_model_b200 import ops
    dev = torch.device("cuda", local)
    hbm, src = read_peaks()
    g = torch.Generator(device=dev).manual_seed(5)
    out = {}
    B, T, H = 64, 16384, 4
    k_store = torch.randn(B, H, T, 64, generator=g, device=dev, dtype=torch.bfloat16)
    v_store = torch.randn(B, H, T, 64, generator=g, device=dev, dtype=torch.bfloat16)
    k_tok = k_store.permute(0, 2, 1, 3)  # the reference's [B, T, H, D] view of the block-major store
    s = _event_time_s(lambda: ops.compress_blocks(k_tok, 64))
    by = k_store.numel() * 2 + B * (T // 64) * H * 64 * 4
    out["compress_blocks"] = {"kernel": "sd::compress_blocks_vec_kernel (sd_compress_blocks)", "us": round(s * 1e6, 2),
                              "bytes": by, "gbs": round(by / s / 1e9, 1), "frac": round(by / s / 1e9 / hbm, 4),
                              "shape": "K [64, 16384, 4, 64] bf16 -> prototypes fp32 [64, 256, 4, 64]"}
    # ten index sets, one per call: 10 x 42 MB of rows, beyond the L2, and no
    # host launch gaps (one graph of the ten calls)
    idxs = [torch.randint(0, T // 64, (B, H, 10), generator=g, device=dev) for _ in range(10)]
    s = _graph_time_s([lambda i=i: ops.gather_kv_blocks(k_store, v_store, i, 64) for i in idxs])
    by = 2 * 2 * B * H * 10 * 64 * 64 * 2  # K and V rows read and written
    out["gather_kv_blocks"] = {"kernel": "sd::gather_kv_vec_kernel (sd_gather_kv_blocks)", "us": round(s * 1e6, 2),
                               "bytes": by, "gbs": round(by / s / 1e9, 1), "frac": round(by / s / 1e9 / hbm, 4),
                               "shape": "10 blocks of 64 rows per (sequence, kv head), 64 x 4, bf16"}
    del k_store, v_store, k_tok
    Tp = 32768
    f = torch.randn(1, Tp, H, 64, generator=g, device=dev, dtype=torch.bfloat16)
    reps = torch.randn(1, Tp // 64, H, 64, generator=g, device=dev, dtype=torch.float32)
    s = _event_time_s(lambda: ops.select_blocks(f, reps, 8, 64, False, return_scores=False))
    fl = 2 * Tp * H * (Tp // 64) * 64
    tpeak, tsrc = read_peak_tflops()
    # the fp32 scores run as 3 bf16 MMAs per product (prototype split in hi /
    # mid / lo parts): 3 x fl on the tensor cores, against the bf16 peak
    out["select_blocks_prefill"] = {"kernel": "sd::seltc::select_rows_tc_kernel (sd_select_blocks, no score tensor)",
                                    "us": round(s * 1e6, 2), "flops": fl, "tflops": round(fl / s / 1e12, 2),
                                    "mma_flops": 3 * fl, "peak_bf16_tflops": round(tpeak, 1),
                                    "frac": round(3 * fl / s / 1e12 / tpeak, 4),
                                    "bound": "issue: the per-row top-8 scan of the scores read from tensor memory",
                                    "shape": "forecast [1, 32768, 4, 64] bf16 x prototypes [1, 512, 4, 64] fp32"}
    _, topk = ops.select_blocks(f, reps, 8, 64, False, return_scores=False)
    s = _graph_time_s([lambda: ops.prefill_lists("chunked_forecast", 1, H, Tp, 64, 8, topk, True, device=dev)] * 10)
    by = topk.numel() * 8 + H * (Tp // 64) * (10 + 1) * 4
    out["prefill_lists"] = {"kernel": "sd::prefill_lists_kernel (sd_prefill_lists, chunked forecast)",
                            "us": round(s * 1e6, 2), "bytes": by, "gbs": round(by / s / 1e9, 1),
                            "frac": round(by / s / 1e9 / hbm, 4),
                            "shape": "top-8 of 32768 rows x 4 heads -> 512 lists per head"}
    out["peak_source"] = src
    return out


def max_over_ranks_simple(x):
    from local_research_small_language_model_b200.sharding import max_over_ranks
    return max_over_ranks(x)


def read_peak_tflops():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return 0
        steps = max(1, args.steps if args.steps < 50 else 8)
        r = cpu_reference(args.ctx, args.cpu_seqs, args.cpu_budget_s * 4, args.rule, max_steps=steps,
                          warmup=min(args.warmup, 2))
        out = {"impl": "reference", "metric": METRIC, "value": round(r["value"], 3), "unit": "tok/s",
               "n_gpus": world, "steps": r["steps"], "warmup": min(args.warmup, 2),
               "ms_per_step": round(r["step_s"] * 1000.0, 3), "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "f32", "data": "synthetic",
               "config": {"workload": "BASELINE config 2 decode step (the GPU arm's workload), timed on a bounded "
                                      "sample of its sequences on the host cores",
                          "global_batch": args.batch * world, "per_gpu_batch": args.batch,
                          "sample_sequences": r["sequences"], "seq_len": args.ctx, "selector_rule": args.rule},
               "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
               "e2e": {"value": round(r["value"], 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                       "d2h_bytes_per_step": 0}}
        print(json.dumps(out), flush=True)
        return 0

    if args.kernels_only:
        import torch
        torch.cuda.set_device(local)
        print(json.dumps({"kernels": run_kernels(local)}), flush=True)
        return 0

    if args.backward:
        import torch
        torch.cuda.set_device(local)
        print(json.dumps({"backward": run_backward(args, local)}), flush=True)
        return 0

    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    try:
        res = run_prefill(args, rank, world, local) if args.prefill else run_b200(args, rank, world, local)
        if world == 1 and not args.prefill and not args.offload and not args.no_extras:
            # BASELINE config 3 (prefill of one 32K-token sequence) and the
            # standalone path kernels, so the default run records them too
            pa = argparse.Namespace(**vars(args))
            pa.ctx, pa.steps, pa.warmup, pa.layers = 32768, 2, 1, args.layers
            pre = run_prefill(pa, rank, world, local)
            res["prefill"] = {k: pre[k] for k in ("metric", "value", "unit", "ms_per_step", "steps", "warmup",
                                                  "config", "roofline", "clocks")}
            res["kernels"] = run_kernels(local)
        if rank == 0:
            if world == 1 and not args.no_cpu_baseline and not args.prefill:
                r = cpu_reference(args.ctx, args.cpu_seqs, args.cpu_budget_s, args.rule)
                res["cpu_baseline"] = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
