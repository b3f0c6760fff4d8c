"""Benchmark of the paged KV-cache decode path: Qwen3-4B layer-shape decode
at 32k context on one GPU, and the same KV-head sharded over N GPUs.

Workload: Qwen3-4B layer shape (Hq=32, Hkv=8, D=128, bf16), 36 layers, each
with 32768 cached tokens in a fragmented block table over a 4096-page pool
(seeded permutation; synthetic N(0,1) values — the reference has no dataset).
A step is one decode token through all 36 layers: per layer one call of the
public API, whose fused launch appends the token's K/V into its page and
attends over the 32k+ tokens (split-K flash-decoding), then the split
combine. Before timing, layer 0's output is checked against a torch fp32
recomputation (`parity` in the line). The one-GPU default run also measures
the 0.6B-layer decode (config 1) and the chunked prefill (config 4) under
`other_configs`. The KV data of a step (36 x 128 MiB) is far larger than L2
(126 MB), so no L2 flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N>1 (launched by torch.distributed.run, one rank per GPU): the 8 KV heads are
sharded over the ranks (8/N each, the matching query heads with them), block
tables are identical on every rank, and each layer's outputs are all-gathered
inside the split combine over NVLink (--gather p2p, the default) or with NCCL
(--gather nccl). Total work is fixed as N grows (strong scaling).

--impl reference times the reference's own CPU op (oracle/_ref, compiled from
the Genllm sources; else the C restatement) on the host cores on the same
config: one process, one thread per layer (the op itself is single-threaded).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "paged-attn decode HBM GB/s (% of 8 TB/s) @32k ctx; tok/s Qwen3-4B-shape"
UNIT = "GB/s"
NOMINAL_HBM_GBS = 8000.0
HQ, HKV, D, LAYERS, CTX, POOL = 32, 8, 128, 36, 32768, 4096


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--ctx", type=int, default=CTX)
    ap.add_argument("--pool", type=int, default=0, help="pages per pool (0: max(4096, ctx/16 + 64))")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="skip the config-1 and config-4 side measurements of the default decode line")
    ap.add_argument("--e2e-steps", type=int, default=0, help="0 = same as --steps")
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "prefill", "qknorm", "flash", "export", "append", "qkrope"],
                    help="decode: config 3 (the headline line); prefill: config 4, chunked prefill on tensor "
                         "cores; qknorm: config 3 fed the Q/K/V projections, QK-norm + RoPE fused into the step; "
                         "export: config 3's 36 layers exported to head-major e4m3 (KV format row); append: the "
                         "chunk append kernel alone (8192 tokens in 512-token chunks into 36 layers' pages); "
                         "qkrope: the standalone QK-norm + RoPE + permute kernel on 512-token chunks")
    ap.add_argument("--gather", default="p2p", choices=["p2p", "nccl"],
                    help="N>1: head all-gather fused into the decode (NVLink peer stores) or NCCL all_gather")
    ap.add_argument("--no-kernel-events", action="store_true",
                    help="skip the per-launch CUDA events (kernel time then comes from the step time)")
    return ap.parse_args()


def pool_pages(args):
    return args.pool or max(POOL, args.ctx // 16 + 64)


def config(args, world):
    return {"workload": "Qwen3-4B layer-shape paged-attention decode, 36 layers back to back",
            "n_q_heads": HQ, "n_kv_heads": HKV, "head_dim": D, "layers": args.layers, "ctx": args.ctx,
            "page_size": 16, "pool_pages": pool_pages(args), "block_table": "seeded random permutation (fragmented)",
            "batch": 1, "parallelism": f"kv-head shard x{world}" if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (36 x 128 MiB of KV per step), no flush"}


# --------------------------------------------------------------------------
# clocks during the timed region (NVML polling thread)
class ClockSampler:
    def __init__(self, index):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    _NAMES = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
              0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
              0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def _run(self):
        while not self._stop.is_set():
            self.sample()
            time.sleep(0.005)

    def sample(self):
        if not self.nv:
            return
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for bit, name in self._NAMES.items():
                if r & bit and name != "gpu_idle":
                    self.reasons.add(name)
        except Exception:
            pass

    def start(self):
        if self.nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        self._stop.set()
        if self._t:
            self._t.join()
        self.sample()
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def profiled_traffic(args, world, summary="paged_decode_kernel_qwen3_4b_32k.md"):
    """DRAM bytes (read + write) of one launch of the summary's kernel from the
    committed ncu summary of this exact configuration, or None."""
    if world != 1 or args.ctx != CTX:
        return None
    try:
        with open(os.path.join(ROOT, "profiles", summary)) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":")[1])
    except OSError:
        pass
    return None


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy burst)"
    except Exception:
        return 6650.0, "fallback 6.65 TB/s"


# --------------------------------------------------------------------------
def run_reference_arm(args, rank, world):
    """The reference's CPU implementation of the path, timed alone."""
    if rank != 0:
        return
    vals, dts, byts = [], [], []
    info = None
    for i in range(args.warmup + args.steps):
        g, cores, kind, sample, dt, nbytes = cpu_step(args)
        info = (cores, kind, sample)
        if i >= args.warmup:
            dts.append(dt)
            byts.append(nbytes)
    value = sum(byts) / sum(dts) / 1e9
    cores, kind, sample = info
    line = {"metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1e3 * sum(dts) / len(dts), 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config(args, world), "impl": "reference",
            "frac_of_8TBps": round(value / NOMINAL_HBM_GBS, 6),
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


_cpu = {}


def cpu_step(args):
    """One timed step of the reference CPU op on the host: one decode token
    (append + attention) of T layers at once, one host thread per layer (the
    op itself is single-threaded; distinct layers share no state), T = the
    host's cores, at most the config's 36 layers. Falls back to the C
    restatement (one layer, threads over its heads) when oracle/_ref is absent.
    Returns (GB/s, cores, kind, sample, seconds, algorithmic bytes)."""
    import numpy as np
    from genllm_b200.synth import bf16_bits
    from oracle.oracle import Oracle, RefSession, ref_available

    c = _cpu
    if not c:
        T = max(1, min(os.cpu_count() or 1, args.layers))
        n_pages = (args.ctx + 15) // 16
        pool = n_pages + 64
        tile = bf16_bits(np.random.default_rng(0).standard_normal(1 << 20, dtype=np.float32))
        c.update(T=T, n_pages=n_pages, pool=pool, tile=tile, ctx=args.ctx)
        c["q"] = [np.resize(tile, HQ * D).reshape(HQ, 1, D).copy() for _ in range(T)]
        c["kv"] = [np.resize(tile[7:], HKV * D).reshape(HKV, 1, D).copy() for _ in range(T)]
        c["out"] = [np.zeros((HQ, 1, D), np.uint16) for _ in range(T)]
        if ref_available():
            s = RefSession(T, HKV, D, pool)
            for l in range(T):
                for w in (0, 1):
                    view = s.pool_view(l, w).reshape(-1)
                    view[:] = np.resize(tile, view.size)
                    for _ in range(pool):
                        s.alloc(l, w)
                    for pid in range(pool - 1, n_pages - 1, -1):
                        s.free(l, w, pid)
                ids = np.random.default_rng(l).permutation(n_pages).astype(np.int32)
                s.set_table(l, ids, ids, args.ctx)
            c.update(s=s, kind="reference", layers=T,
                     sample=(f"{T} layers at once (one host thread each; the op is single-threaded), one decode "
                             f"token per layer per step, ctx {args.ctx} and growing, reference CPU op "
                             f"(ops::PagedAttentionImpl<CPU>::execute) built from the Genllm sources"))
        else:
            c.update(s=None, kind="port", layers=1, o=Oracle(), kp=np.resize(tile, pool * 16 * HKV * D),
                     ids=np.random.default_rng(0).permutation(pool)[: n_pages + 1].astype(np.int32),
                     sample=f"one layer-token at ctx {args.ctx}, C restatement over {T} threads")
    total = c["ctx"] + 1
    if c["s"] is not None:
        t0 = time.perf_counter()
        c["s"].paged_attention_layers(c["q"], c["kv"], c["kv"], c["out"], HQ, 1, 1 / np.sqrt(D))
        dt = time.perf_counter() - t0
        c["ctx"] += 1
    else:
        t0 = time.perf_counter()
        c["o"].paged_attention_f32(c["q"][0], c["kp"], c["kp"], c["ids"], c["ids"], total, HQ, HKV, 1, D,
                                   1 / np.sqrt(D), threads=c["T"])
        dt = time.perf_counter() - t0
    per_layer = 2 * (total - 1) * HKV * D * 2 + 2 * 2 * HKV * D * 2 + 2 * HQ * D * 2 + ((total + 15) // 16) * 8
    nbytes = c["layers"] * per_layer
    return nbytes / dt / 1e9, c["T"], c["kind"], c["sample"], dt, nbytes


def measure_config1(args):
    """Config 1 (Qwen3-0.6B layer: Hq 16, Hkv 8, D 128, 1024 cached tokens in
    a fragmented 256-page pool, one token appended per step): the decode step
    through the public API (one call per step) and captured in a CUDA graph
    (device time), 200 steps each; the reference CPU op timed beside it on
    the same shape (one thread, its own implementation). Returns a dict for
    the bench line."""
    import numpy as np
    import torch
    from genllm_b200.paged_attention import DecodeGraph
    from genllm_b200.workload import DecodeWorkload

    hq, hkv, ctx, pool, n = 16, 8, 1024, 256, 200
    wl = DecodeWorkload(0, n_layers=1, ctx=ctx, pool_pages=pool, n_q_heads=hq, n_kv_heads=hkv, head_dim=D, seed=0)
    stream = torch.cuda.current_stream()
    sh = __import__("ctypes").c_void_p(stream.cuda_stream)
    for _ in range(5):
        wl.layer_step(0, sh)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0 = wl.cached(0)
    e0.record(stream)
    for _ in range(n):
        wl.layer_step(0, sh)
    e1.record(stream)
    torch.cuda.synchronize()
    call_us = e0.elapsed_time(e1) * 1e3 / n
    byts = sum(wl.bytes_per_layer_token(c0 + k + 1) for k in range(n)) / n
    L0 = wl.layers[0]
    graph = DecodeGraph(wl.mgr, [0], [L0.q], [L0.k], [L0.v], [L0.out], hq, wl.scale)
    for _ in range(5):
        graph.run()
    torch.cuda.synchronize()
    c1 = wl.cached(0)
    e0.record(stream)
    for _ in range(n):
        graph.run()
    e1.record(stream)
    torch.cuda.synchronize()
    graph_us = e0.elapsed_time(e1) * 1e3 / n
    gbyts = sum(wl.bytes_per_layer_token(c1 + k + 1) for k in range(n)) / n
    graph.close()
    out = {"workload": "config 1: Qwen3-0.6B layer decode, 1024 cached tokens (+1 per step), 256-page fragmented "
                       "pool, Hq 16 / Hkv 8 / D 128, bf16",
           "public_api_us_per_step": round(call_us, 3), "public_api_gbs": round(byts / (call_us * 1e-6) / 1e9, 1),
           "captured_us_per_step": round(graph_us, 3), "captured_gbs": round(gbyts / (graph_us * 1e-6) / 1e9, 1),
           "bytes_per_step": round(byts)}
    try:
        from genllm_b200.synth import bf16_bits
        from oracle.oracle import RefSession, ref_available
        if ref_available():
            s = RefSession(1, hkv, D, pool)
            tile = bf16_bits(np.random.default_rng(0).standard_normal(1 << 20, dtype=np.float32))
            for w in (0, 1):
                view = s.pool_view(0, w).reshape(-1)
                view[:] = np.resize(tile, view.size)
                for _ in range(pool):
                    s.alloc(0, w)
                for pid in range(pool - 1, ctx // 16 - 1, -1):
                    s.free(0, w, pid)
            ids = np.random.default_rng(0).permutation(ctx // 16).astype(np.int32)
            s.set_table(0, ids, ids, ctx)
            q = [np.resize(tile, hq * D).reshape(hq, 1, D).copy()]
            kv = [np.resize(tile[7:], hkv * D).reshape(hkv, 1, D).copy()]
            o = [np.zeros((hq, 1, D), np.uint16)]
            reps, t = 0, 0.0
            while reps < 20:
                h0 = time.perf_counter()
                s.paged_attention_layers(q, kv, kv, o, hq, 1, 1 / np.sqrt(D))
                t += time.perf_counter() - h0
                reps += 1
            us = t / reps * 1e6
            out["cpu_baseline"] = {"value": round(us, 1), "unit": "us per step", "cores": 1, "kind": "reference",
                                   "sample": f"{reps} decode steps of the reference CPU op (growing from 1024 "
                                             "cached tokens), one thread"}
    except Exception as exc:  # noqa: BLE001
        out["cpu_baseline"] = {"unavailable": str(exc)[:200]}
    return out


def measure_config4(args):
    """Config 4 (chunked prefill on the tensor cores) for the bench line:
    causal-exact TFLOP/s over an 8192-token prompt in 512-token chunks."""
    return prefill_numbers(argparse.Namespace(steps=20, warmup=3))


# --------------------------------------------------------------------------
def run_prefill(args):
    line = prefill_numbers(args)
    print(json.dumps(line), flush=True)


def prefill_numbers(args):
    """Config 4: Qwen3-1.7B layer shape (Hq 16, Hkv 8, D 128), an 8192-token
    prompt in 512-token chunks; each chunk appended into pages and attended
    causally over all prior pages by the tensor-core kernel. A step = the
    whole prompt for one layer (cache reset first). Metric: causal-exact
    attention TFLOP/s (4 * D * Hq * sum of visible keys)."""
    import torch
    from genllm_b200.paged_attention import PagedAttentionManager, paged_attention

    hq, hkv, d, chunk, prompt = 16, 8, 128, 512, 8192
    torch.cuda.set_device(0)
    m = PagedAttentionManager(0)
    m.init_layer(0, hkv, d)
    m.reserve_layer(0, prompt // 16 + 8)
    g = torch.Generator(device="cuda").manual_seed(4)
    n_chunks = prompt // chunk
    Q = [torch.randn(1, hq, chunk, d, generator=g, device="cuda").to(torch.bfloat16) for _ in range(n_chunks)]
    K = [torch.randn(1, hkv, chunk, d, generator=g, device="cuda").to(torch.bfloat16) for _ in range(n_chunks)]
    V = [torch.randn(1, hkv, chunk, d, generator=g, device="cuda").to(torch.bfloat16) for _ in range(n_chunks)]
    out = torch.empty(1, hq, chunk, d, dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.current_stream()

    def step(events=None):
        m.reset_layer(0)
        for c in range(n_chunks):
            if events is not None:
                events[c][0].record(stream)
            paged_attention(m, 0, Q[c], K[c], V[c], out=out)
            if events is not None:
                events[c][1].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(0)
    clocks.start()
    t0.record(stream)
    h0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    flops = 4.0 * d * hq * sum(p + 1 for p in range(prompt))
    ev = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(n_chunks)]
    step(ev)
    torch.cuda.synchronize()
    chunk_ms = [a.elapsed_time(b) for a, b in ev]
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, src = float(json.load(f)["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except Exception:
        peak, src = 1590.0, "fallback 1.59 PFLOP/s"
    tflops = flops / (ms / 1e3) / 1e12
    last = chunk_ms[-1]
    last_flops = 4.0 * d * hq * sum(p + 1 for p in range(prompt - chunk, prompt))
    line = {"metric": "chunked-prefill paged attention TFLOP/s (causal-exact), Qwen3-1.7B layer shape",
            "value": round(tflops, 2), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config 4: 8192-token prompt in 16 chunks of 512, append + causal attention "
                                   "over all prior pages", "n_q_heads": hq, "n_kv_heads": hkv, "head_dim": d},
            "gpu_launches": 2 * n_chunks * args.steps,
            "host_enqueue_ms_per_step": round(host_ms, 4),
            "roofline": {"bound": "tensor", "achieved": round(last_flops / (last / 1e3) / 1e12, 2), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(last_flops / (last / 1e3) / 1e12 / peak, 4),
                         "traffic": None, "peak_source": src,
                         "kernel": "prefill_tc_kernel (+ kv_append_kernel), last chunk (8192 visible keys)",
                         "chunk_ms": [round(x, 4) for x in chunk_ms]},
            "clocks": clk}
    return line


def run_flash(args):
    """The reference's non-paged attention op (FlashAttentionImpl) on the
    tcgen05 kernel: one causal self-attention call over an 8192-token
    sequence, Qwen3-1.7B layer shape (Hq 16, Hkv 8, D 128, bf16). Metric:
    causal-exact TFLOP/s (4 * D * Hq * sum of visible keys)."""
    import torch
    from genllm_b200.paged_attention import flash_attention

    torch.cuda.set_device(0)
    B, hq, hkv, d, S = 1, 16, 8, 128, 8192
    g = torch.Generator(device="cuda").manual_seed(9)
    Q = torch.randn(B, hq, S, d, generator=g, device="cuda").to(torch.bfloat16)
    K = torch.randn(B, hkv, S, d, generator=g, device="cuda").to(torch.bfloat16)
    V = torch.randn(B, hkv, S, d, generator=g, device="cuda").to(torch.bfloat16)
    out = torch.empty_like(Q)
    for _ in range(args.warmup):
        flash_attention(Q, K, V, out=out)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(0)
    clocks.start()
    e0.record(stream)
    for _ in range(args.steps):
        flash_attention(Q, K, V, out=out)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    flops = 4.0 * d * hq * B * sum(p + 1 for p in range(S))
    tf = flops / (ms / 1e3) / 1e12
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, src = float(json.load(f)["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except Exception:
        peak, src = 1590.0, "fallback 1.59 PFLOP/s"
    line = {"metric": "non-paged causal attention TFLOP/s (causal-exact), Qwen3-1.7B layer shape, 8192 tokens",
            "value": round(tf, 2), "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "FlashAttentionImpl: one self-attention call, B 1, S 8192, causal",
                       "n_q_heads": hq, "n_kv_heads": hkv, "head_dim": d},
            "gpu_launches": args.steps,
            "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(tf / peak, 4), "traffic": None, "peak_source": src,
                         "kernel": "prefill_tc_kernel (contiguous K/V)"},
            "clocks": clk}
    print(json.dumps(line), flush=True)


def run_export(args):
    """KV format export: config 3's cache (36 layers x 32k tokens, Hkv 8, D
    128, fragmented 4096-page pools) exported to dense head-major e4m3 with
    per (head, 16-token block) scales -- one kv_export_kernel launch per
    layer. A step = all 36 layers. Metric: algorithmic HBM GB/s (pages read
    2 B/element, e4m3 written 1 B/element, scales 4 B per block). Also timed:
    the bf16 export and the e4m3 import (same bytes in the other direction);
    e2e = the export plus the device-to-host copy of its output into pinned
    host memory (a KV offload)."""
    import torch
    from genllm_b200.paged_attention import PagedAttentionManager

    torch.cuda.set_device(0)
    L, n, hkv, pages = args.layers, args.ctx, HKV, pool_pages(args)
    dev = torch.device("cuda:0")
    m = PagedAttentionManager(0)
    g = torch.Generator(device=dev).manual_seed(6)
    for l in range(L):
        m.init_layer(l, hkv, D)
        m.reserve_layer(l, pages)
        kp, vp = m.pool_tensors(l)
        kp.copy_(torch.randn(kp.shape, generator=g, device=dev).to(torch.bfloat16))
        vp.copy_(torch.randn(vp.shape, generator=g, device=dev).to(torch.bfloat16))
        for w in (0, 1):
            pool = m.pool(l, w)
            for _ in range(pages):
                pool.alloc()
        pk = torch.randperm(pages, generator=torch.Generator().manual_seed(100 + l))[: (n + 15) // 16]
        pv = torch.randperm(pages, generator=torch.Generator().manual_seed(200 + l))[: (n + 15) // 16]
        m.set_page_table(l, pk.tolist(), pv.tolist(), n)
    nb = (n + 15) // 16
    elems = 2 * hkv * n * D
    fp8_bytes = elems * 3 + 2 * hkv * nb * 4       # read bf16, write e4m3 + scales
    bf16_bytes = elems * 4
    # preallocated outputs: the export writes into them through the raw C ABI
    import ctypes as C
    from genllm_b200 import _lib
    K8 = [torch.empty((hkv, n, D), dtype=torch.uint8, device=dev) for _ in range(L)]
    V8 = [torch.empty_like(K8[0]) for _ in range(L)]
    KS = [torch.empty((hkv, nb), dtype=torch.float32, device=dev) for _ in range(L)]
    VS = [torch.empty_like(KS[0]) for _ in range(L)]
    K16 = torch.empty((hkv, n, D), dtype=torch.bfloat16, device=dev)
    V16 = torch.empty_like(K16)
    stream = torch.cuda.current_stream()
    sh = C.c_void_p(stream.cuda_stream)
    cnt = C.c_int32()

    def export(l, fmt):
        if fmt == _lib.GKV_KV_FP8_E4M3:
            args_ = (K8[l], V8[l], KS[l], VS[l])
        else:
            args_ = (K16, V16, None, None)
        _lib.check(_lib.lib().gkv_export_kv(m.handle, l, fmt, *[C.c_void_p(t.data_ptr() if t is not None else 0)
                                                                  for t in args_], C.byref(cnt), sh))

    def step(fmt=_lib.GKV_KV_FP8_E4M3, events=None):
        for l in range(L):
            if events is not None:
                events[l][0].record(stream)
            export(l, fmt)
            if events is not None:
                events[l][1].record(stream)

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / steps

    # headline: the e4m3 export, per-launch events inside the timed region
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ev = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(L)]
          for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(0)
    clocks.start()
    t0.record(stream)
    for k in range(args.steps):
        step(events=ev[k])
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    launch_ms = statistics.mean(a.elapsed_time(b) for e in ev for a, b in e)
    gbs = fp8_bytes * L / (ms / 1e3) / 1e9
    ms_bf16 = timed(lambda: step(_lib.GKV_KV_BF16), args.steps)

    # e4m3 import of the exported layers into a second manager (reset per step)
    m2 = PagedAttentionManager(0)
    for l in range(L):
        m2.init_layer(l, hkv, D)
        m2.reserve_layer(l, pages)

    def import_step():
        m2.reset()
        for l in range(L):
            _lib.check(_lib.lib().gkv_import_kv(m2.handle, l, _lib.GKV_KV_FP8_E4M3, C.c_void_p(K8[l].data_ptr()),
                                                C.c_void_p(V8[l].data_ptr()), C.c_void_p(KS[l].data_ptr()),
                                                C.c_void_p(VS[l].data_ptr()), n, sh))
    ms_import = timed(import_step, args.steps)

    # e2e: export + D2H of every layer's e4m3 output and scales into pinned memory
    host = [(torch.empty(K8[0].shape, dtype=torch.uint8, pin_memory=True),
             torch.empty(V8[0].shape, dtype=torch.uint8, pin_memory=True),
             torch.empty(KS[0].shape, dtype=torch.float32, pin_memory=True),
             torch.empty(VS[0].shape, dtype=torch.float32, pin_memory=True)) for _ in range(L)]

    def e2e_step():
        for l in range(L):
            export(l, _lib.GKV_KV_FP8_E4M3)
            for dst, src in zip(host[l], (K8[l], V8[l], KS[l], VS[l])):
                dst.copy_(src, non_blocking=True)
    e2e_steps = max(3, min(args.steps, 5))
    ms_e2e = timed(e2e_step, e2e_steps)
    d2h = L * (2 * hkv * n * D + 2 * hkv * nb * 4)

    peak, src = measured_peak()
    achieved = fp8_bytes / (launch_ms / 1e3) / 1e9
    cpu = None
    if not args.no_cpu_baseline:
        cpu = export_cpu_baseline()
    line = {"metric": "KV export to head-major e4m3 + block scales, algorithmic HBM GB/s, 36 layers x 32k tokens",
            "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u8", "data": "synthetic",
            "config": {"workload": "config 3's KV cache exported (KV format row): 36 layers x 32768 tokens, "
                                   "Hkv 8, D 128, fragmented 4096-page pools",
                       "layers": L, "ctx": n, "n_kv_heads": hkv, "head_dim": D, "pool_pages": pages,
                       "l2": "inputs larger than L2 (36 x 128 MiB of pages per step), no flush"},
            "gpu_launches": L * args.steps,
            "bf16_export_gbs": round(bf16_bytes * L / (ms_bf16 / 1e3) / 1e9, 1),
            "fp8_import_gbs": round(fp8_bytes * L / (ms_import / 1e3) / 1e9, 1),
            "e2e": {"value": round(fp8_bytes * L / (ms_e2e / 1e3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": 0, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e2e, 3),
                    "what": "export + device-to-host copy of the e4m3 output into pinned memory"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "traffic": profiled_traffic(args, 1, "kv_export_kernel_qwen3_4b_32k.md"),
                         "peak_source": src, "kernel": "kv_export_kernel", "bytes_per_launch": fp8_bytes,
                         "launch_ms": round(launch_ms, 5)},
            "cpu_baseline": cpu,
            "clocks": clk}
    print(json.dumps(line), flush=True)


def export_cpu_baseline():
    """The oracle's export (a scalar C port; the reference has no export) on a
    bounded sample: one layer of 4096 tokens, Hkv 8."""
    import numpy as np
    from oracle.oracle import Oracle
    o = Oracle()
    hkv, n, pages = HKV, 4096, 256
    rng = np.random.default_rng(1)
    kp = rng.integers(0, 0x4000, size=(pages, 16, hkv, D), dtype=np.uint16)
    vp = rng.integers(0, 0x4000, size=(pages, 16, hkv, D), dtype=np.uint16)
    ids = rng.permutation(pages).astype(np.int32)
    reps, t = 0, 0.0
    while t < 10.0 and reps < 50:
        h0 = time.perf_counter()
        o.export_kv(kp, vp, ids, ids, n, hkv, fp8=True)
        t += time.perf_counter() - h0
        reps += 1
    nbytes = 2 * hkv * n * D * 3 + 2 * hkv * (n // 16) * 4
    return {"value": round(nbytes * reps / t / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"oracle export of one layer, 4096 tokens x 8 heads, {reps} repetitions"}


def run_qknorm(args):
    """Config 3 on the projections: each layer-token's Q/K/V arrive as the
    Q/K/V projections ([1, H*128] bf16) and go through QK-norm + RoPE before
    the append and the attention (src/model/Qwen3.cpp:136-158). Fused: one
    gkv_paged_attention_qknorm per layer (the norm and rotation run inside
    the decode kernel). Unfused: gkv_qk_norm_rope (one launch for the
    permutes, norms and rotations the reference runs as seven ops) then
    gkv_paged_attention. Both are timed; `value` is the fused one."""
    import ctypes as C
    import numpy as np
    import torch
    from genllm_b200 import _lib
    from genllm_b200.paged_attention import QkNorm
    from genllm_b200.workload import DecodeWorkload

    torch.cuda.set_device(0)
    wl = DecodeWorkload(0, n_layers=args.layers, ctx=args.ctx, pool_pages=pool_pages(args), n_q_heads=HQ,
                        n_kv_heads=HKV, head_dim=D, seed=0)
    g = torch.Generator().manual_seed(5)
    max_seq = args.ctx + 2 * (args.steps + args.warmup) + 64
    qk = QkNorm(1 + 0.25 * torch.randn(D, generator=g), 1 + 0.25 * torch.randn(D, generator=g), 1e-6, 1e6,
                max_seq, 0)
    L = _lib.lib()
    stream = torch.cuda.current_stream()
    sh = C.c_void_p(stream.cuda_stream)
    tq = torch.empty((HQ, 1, D), dtype=torch.bfloat16, device="cuda")
    tk = torch.empty((HKV, 1, D), dtype=torch.bfloat16, device="cuda")
    tv = torch.empty((HKV, 1, D), dtype=torch.bfloat16, device="cuda")
    sc = C.c_float(1.0 / D ** 0.5)

    def fused_step():
        for l, b in enumerate(wl.layers):
            _lib.check(L.gkv_paged_attention_qknorm(wl.mgr.handle, l, C.c_void_p(b.q.data_ptr()),
                                                    C.c_void_p(b.k.data_ptr()), C.c_void_p(b.v.data_ptr()),
                                                    C.c_void_p(b.out.data_ptr()), HQ, 1, sc, 1, _lib.GKV_BF16,
                                                    C.byref(qk.desc), sh))

    pos = [args.ctx]  # every layer holds the same number of tokens

    def unfused_step():
        for l, b in enumerate(wl.layers):
            _lib.check(L.gkv_qk_norm_rope(C.c_void_p(b.q.data_ptr()), C.c_void_p(b.k.data_ptr()),
                                          C.c_void_p(b.v.data_ptr()), 1, HQ, HKV, C.byref(qk.desc), pos[0],
                                          C.c_void_p(tq.data_ptr()), C.c_void_p(tk.data_ptr()),
                                          C.c_void_p(tv.data_ptr()), sh))
            _lib.check(L.gkv_paged_attention(wl.mgr.handle, l, C.c_void_p(tq.data_ptr()), C.c_void_p(tk.data_ptr()),
                                             C.c_void_p(tv.data_ptr()), C.c_void_p(b.out.data_ptr()), 1, HQ, 1, D,
                                             HKV, sc, 1, HQ // HKV, _lib.GKV_BF16, _lib.GKV_BF16, sh))
        pos[0] += 1

    def counted_fused():
        fused_step()
        pos[0] += 1

    def plain_step():
        for l in range(args.layers):
            wl.layer_step(l, sh)
        pos[0] += 1

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    clocks = ClockSampler(0)
    clocks.start()
    ms_fused = timed(counted_fused)
    clk = clocks.stop()
    ms_unfused = timed(unfused_step)
    ms_plain = timed(plain_step)
    per_layer = ms_fused * 1e3 / args.layers
    ctx_now = wl.mgr.get_layer(0).num_cached
    bytes_lt = 2 * ctx_now * HKV * D * 2 + HQ * D * 2 * 2 + 2 * HKV * D * 2
    gbs = bytes_lt / (per_layer * 1e-6) / 1e9
    peak, src = measured_peak()
    cpu = None
    try:
        from oracle.oracle import RefOps
        from genllm_b200.synth import randn_bf16
        R = RefOps()
        rng = np.random.default_rng(0)
        cos, sin = R.rope_cache(1e6, D, 64)
        xq = randn_bf16(rng, (HQ, 1, D))
        xk = randn_bf16(rng, (HKV, 1, D))
        wq = np.ones(D, np.float32)
        n = 2000
        t0 = time.perf_counter()
        for _ in range(n):
            R.apply_rope_bf16(R.rms_norm_bf16(xq, wq, 1e-6), cos, sin, 5)
            R.apply_rope_bf16(R.rms_norm_bf16(xk, wq, 1e-6), cos, sin, 5)
        us = (time.perf_counter() - t0) / n * 1e6
        cpu = {"value": round(us, 2), "unit": "us per layer-token (QK-norm + RoPE only)", "cores": 1,
               "kind": "reference", "sample": f"{n} layer-tokens of the reference CPU rms_norm + apply_rope ops "
                                               "(Hq 32, Hkv 8), ctypes call overhead included"}
    except Exception as exc:  # noqa: BLE001
        cpu = {"unavailable": str(exc)[:200]}
    line = {"metric": "paged-attn decode on the Q/K/V projections (QK-norm + RoPE + append + attention), "
                      "us per layer-token @32k; Qwen3-4B shape",
            "value": round(per_layer, 3), "unit": "us/layer-token", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_fused, 4), "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config 3 fed the projections: 36 layers at 32k, per layer-token QK-norm "
                                   "(RMSNorm eps 1e-6) + RoPE (theta 1e6) + append + decode",
                       "n_q_heads": HQ, "n_kv_heads": HKV, "head_dim": D, "l2": "KV of a step (4.8 GB) >> L2"},
            "unfused_us_per_layer_token": round(ms_unfused * 1e3 / args.layers, 3),
            "plain_decode_us_per_layer_token": round(ms_plain * 1e3 / args.layers, 3),
            "gpu_launches": 2 * args.layers * args.steps,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "traffic": None, "peak_source": src,
                         "kernel": "paged_decode_kernel (QK-norm + RoPE fused) + combine, whole layer-token"},
            "cpu_baseline": cpu, "clocks": clk}
    print(json.dumps(line), flush=True)


def run_append(args):
    """The chunk append (append_kv_from_tensor, src/core/page_attention.cpp:
    104-139) alone: Qwen3-1.7B KV shape (Hkv 8, D 128, bf16), an 8192-token
    prompt appended in 512-token chunks into each of 36 layers' fragmented
    pools (a step = 36 x 16 launches of kv_append_kernel). Inputs (36 x 32 MiB
    of K and V) and pools exceed L2. Metric: algorithmic HBM GB/s (K and V
    read once, written once, plus the published table entries)."""
    import torch
    from genllm_b200.paged_attention import PagedAttentionManager

    torch.cuda.set_device(0)
    L, hkv, d, chunk, prompt = args.layers, 8, 128, 512, 8192
    dev = torch.device("cuda", 0)
    m = PagedAttentionManager(0)
    g = torch.Generator(device=dev).manual_seed(12)
    K, V = [], []
    for l in range(L):
        m.init_layer(l, hkv, d)
        m.reserve_layer(l, prompt // 16 + 64)
        K.append(torch.randn(hkv, prompt, d, generator=g, device=dev).to(torch.bfloat16))
        V.append(torch.randn(hkv, prompt, d, generator=g, device=dev).to(torch.bfloat16))
    n_chunks = prompt // chunk
    Kc = [[K[l][:, c * chunk:(c + 1) * chunk].contiguous() for c in range(n_chunks)] for l in range(L)]
    Vc = [[V[l][:, c * chunk:(c + 1) * chunk].contiguous() for c in range(n_chunks)] for l in range(L)]
    del K, V
    stream = torch.cuda.current_stream()

    def launches():
        for l in range(L):
            for c in range(n_chunks):
                m.append_kv_from_tensor(l, Kc[l][c], Vc[l][c])

    def step():
        m.reset()
        launches()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(0)
    clocks.start()
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    # The same launches captured once (pages allocated at capture) and
    # replayed: device time without the host's per-call cost, which is
    # larger than one 4 MiB launch.
    m.reset()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        launches()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    t0.record(stream)
    for _ in range(args.steps):
        graph.replay()
    t1.record(stream)
    torch.cuda.synchronize()
    ms_graph = t0.elapsed_time(t1) / args.steps
    launch_ms = ms_graph / (L * n_chunks)
    per_launch = 2 * 2 * hkv * chunk * d * 2 + (chunk // 16) * 8
    gbs = per_launch * L * n_chunks / (ms / 1e3) / 1e9
    peak, src = measured_peak()
    achieved = per_launch / (launch_ms / 1e3) / 1e9
    line = {"metric": "KV chunk append (append_kv_from_tensor) algorithmic HBM GB/s, Qwen3-1.7B KV shape",
            "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "8192-token prompt appended in 512-token chunks into 36 layers' pages",
                       "layers": L, "n_kv_heads": hkv, "head_dim": d, "chunk": chunk,
                       "l2": "36 x 32 MiB of inputs per step, larger than L2"},
            "gpu_launches": L * n_chunks * args.steps,
            "captured_step_ms": round(ms_graph, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None, "peak_source": src,
                         "kernel": "kv_append_kernel", "bytes_per_launch": per_launch,
                         "launch_us": round(launch_ms * 1e3, 3),
                         "how": "mean per launch of the step's 576 launches replayed from a CUDA graph"},
            "clocks": clk}
    print(json.dumps(line), flush=True)


def run_qkrope(args):
    """The standalone QK-norm + RoPE + head-major permute (gkv_qk_norm_rope;
    src/model/Qwen3.cpp:136-154 as one launch instead of seven): Qwen3-4B
    shape (Hq 32, Hkv 8), 512-token chunks at positions 0..511, distinct
    inputs for 36 layers (36 x 6 MiB, larger than L2). Metric: algorithmic
    HBM GB/s (projections read, the three head-major outputs written, the
    position's cos/sin rows read once per launch)."""
    import torch
    from genllm_b200.paged_attention import QkNorm, qk_norm_rope

    torch.cuda.set_device(0)
    L, hq, hkv, d, S = args.layers, HQ, HKV, D, 512
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(13)
    qk = QkNorm(1 + 0.25 * torch.randn(d), 1 + 0.25 * torch.randn(d), 1e-6, 1e6, S, 0)
    ins = [tuple(torch.randn(S, h * d, generator=g, device=dev).to(torch.bfloat16) for h in (hq, hkv, hkv))
           for _ in range(L)]
    stream = torch.cuda.current_stream()

    def step():
        for l in range(L):
            qk_norm_rope(*ins[l], hq, hkv, qk, 0)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(0)
    clocks.start()
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    t0.record(stream)
    for _ in range(args.steps):
        graph.replay()
    t1.record(stream)
    torch.cuda.synchronize()
    ms_graph = t0.elapsed_time(t1) / args.steps
    launch_ms = ms_graph / L
    per_launch = 2 * S * (hq + 2 * hkv) * d * 2 + 2 * S * d * 4 + 2 * d * 4
    gbs = per_launch * L / (ms / 1e3) / 1e9
    peak, src = measured_peak()
    achieved = per_launch / (launch_ms / 1e3) / 1e9
    line = {"metric": "QK-norm + RoPE + permute (one launch) algorithmic HBM GB/s, Qwen3-4B shape, 512-token chunks",
            "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "gkv_qk_norm_rope on a 512-token chunk for each of 36 layers",
                       "layers": L, "n_q_heads": hq, "n_kv_heads": hkv, "head_dim": d, "chunk": S,
                       "l2": "36 x 6 MiB of projections per step, larger than L2"},
            "gpu_launches": L * args.steps,
            "captured_step_ms": round(ms_graph, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None, "peak_source": src,
                         "kernel": "qk_norm_rope_kernel", "bytes_per_launch": per_launch,
                         "launch_us": round(launch_ms * 1e3, 3),
                         "how": "mean per launch of the step's 36 launches replayed from a CUDA graph"},
            "clocks": clk}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.workload == "prefill":
        run_prefill(args)
        return
    if args.workload == "qknorm":
        run_qknorm(args)
        return
    if args.workload == "flash":
        run_flash(args)
        return
    if args.workload == "export":
        run_export(args)
        return
    if args.workload == "append":
        run_append(args)
        return
    if args.workload == "qkrope":
        run_qkrope(args)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from genllm_b200.workload import DecodeWorkload, allgather_heads

    wl = DecodeWorkload(local, n_layers=args.layers, ctx=args.ctx, pool_pages=pool_pages(args), n_q_heads=HQ, n_kv_heads=HKV,
                        head_dim=D, seed=0, world=world, rank=rank)
    stream = torch.cuda.current_stream()
    sh = __import__("ctypes").c_void_p(stream.cuda_stream)
    gathered_all = torch.empty((args.layers, HQ * D), dtype=torch.bfloat16, device="cuda")
    gathered = [gathered_all[l].view(1, HQ, 1, D) for l in range(args.layers)]

    hg = None
    if world > 1 and args.gather == "p2p":
        import ctypes as C
        from genllm_b200 import _lib
        from genllm_b200.gather import HeadGather
        hg = HeadGather(local, args.layers, HQ)
        gfn = _lib.lib().gkv_paged_attention_gather
        gargs = [(wl.mgr.handle, l, C.c_void_p(b.q.data_ptr()), C.c_void_p(b.k.data_ptr()), C.c_void_p(b.v.data_ptr()),
                  hg.handle, l * hg.layer_bytes, wl.hq_local, C.c_float(wl.scale), _lib.GKV_BF16, sh)
                 for l, b in enumerate(wl.layers)]
        gathered_all = hg.full.view(args.layers, HQ * D)

    def layer_call(l):
        if hg is not None:
            st = gfn(*gargs[l])
            if st:
                _lib.check(st)
        else:
            wl.layer_step(l, sh)
            if world > 1:
                allgather_heads(wl.layers[l].out, gathered[l])

    # One GPU: the same step is also captured as a CUDA graph
    # (gkv_decode_graph_step: host page allocation + one graph launch),
    # timed separately below. The headline keeps one call per layer.
    graph = None
    if hg is None and world == 1:
        from genllm_b200.paged_attention import DecodeGraph
        graph = DecodeGraph(wl.mgr, list(range(args.layers)), [b.q for b in wl.layers], [b.k for b in wl.layers],
                            [b.v for b in wl.layers], [b.out for b in wl.layers], wl.hq_local, wl.scale)

    def step(events=None):
        for l in range(args.layers):
            if events is not None:
                events[l][0].record(stream)
            layer_call(l)
            if events is not None:
                events[l][1].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # Self-check before timing: layer 0's output of the last warm-up step,
    # gathered over the ranks, against a torch fp32 recomputation of all
    # heads from the workload's seeded values (rank 0).
    parity = None
    if args.warmup > 0 and rank == 0:
        got = (gathered_all[0] if world > 1 else wl.layers[0].out).float().reshape(HQ, D)
        want = wl.reference_output(0)
        err = (got - want).abs()
        big = want.abs() >= 1e-3
        max_abs = float(err.max())
        max_rel = float((err[big] / want[big].abs()).max()) if bool(big.any()) else 0.0
        parity = {"layer": 0, "max_abs": max_abs, "max_rel": max_rel, "ok": max_abs <= 2e-3 and max_rel <= 1e-2,
                  "bounds": "max-abs 2e-3; max-rel 1e-2 over |want| >= 1e-3",
                  "against": "torch fp32 recomputation of all heads from the seeded workload (bf16 output rounded)"}
        del want, got, err
        torch.cuda.empty_cache()
    ctx0 = wl.cached(0)

    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    t_start.record(stream)
    h0 = time.perf_counter()
    for k in range(args.steps):
        step()
    host_enqueue_s = time.perf_counter() - h0
    t_end.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
    ms = t_start.elapsed_time(t_end)
    captured = None
    if graph is not None:
        # The same steps through the captured multi-layer step: the layers are
        # distinct and their inputs ready before the step, so each combine
        # releases the next layer's decode at entry and the layers after the
        # first do not wait for their predecessor before computing.
        for _ in range(args.warmup):
            graph.run()
        torch.cuda.synchronize()
        ctx_g = wl.cached(0)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(args.steps):
            graph.run()
        g1.record(stream)
        torch.cuda.synchronize()
        g_ms = g0.elapsed_time(g1)
        g_bytes = sum(args.layers * wl.bytes_per_layer_token(ctx_g + k + 1) for k in range(args.steps))
        captured = {"value": round(g_bytes / (g_ms / 1e3) / 1e9, 2), "unit": UNIT,
                    "ms_per_step": round(g_ms / args.steps, 4),
                    "us_per_token_layer": round(1e3 * g_ms / (args.steps * args.layers), 3),
                    "path": "gkv_decode_graph_step: the 36 layers' decode + combine kernels replayed from one CUDA "
                            "graph; combines release the next layer's decode at entry, layers after the first "
                            "skip the wait on their predecessor (their inputs were ready before the step)"}
    # Per-launch device time of one layer's decode step (decode + combine
    # kernels), from CUDA events around each call on the launching stream in a
    # separate instrumented pass (events between launches serialise them).
    kern_steps = 0 if args.no_kernel_events else min(args.steps, 5)
    ev = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(args.layers)]
          for _ in range(kern_steps)]
    ctx_k = wl.cached(0)
    for k in range(kern_steps):
        step(ev[k])
    torch.cuda.synchronize()
    if kern_steps:
        kern_ms = [ev[k][l][0].elapsed_time(ev[k][l][1]) for k in range(kern_steps) for l in range(args.layers)]
        kern_avg_ms = sum(kern_ms) / len(kern_ms)
        kern_bytes = sum(wl.bytes_per_layer_token(ctx_k + k + 1) for k in range(kern_steps)) / kern_steps
    else:
        kern_avg_ms = ms / (args.steps * args.layers)
        kern_bytes = None

    # Algorithmic bytes: this rank's launches over the timed steps.
    byts = 0
    for k in range(args.steps):
        byts += args.layers * wl.bytes_per_layer_token(ctx0 + k + 1)
    per_launch_bytes = byts / (args.steps * args.layers)
    t = torch.tensor([ms, kern_avg_ms], device="cuda")
    b = torch.tensor([float(byts)], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(b, op=dist.ReduceOp.SUM)
    ms_max, kern_max = t.tolist()
    total_bytes = b.item()
    value = total_bytes / (ms_max / 1e3) / 1e9

    # ---- end to end: host buffers through the public API ---------------
    e2e_steps = args.e2e_steps or args.steps
    from genllm_b200.paged_attention import paged_attention
    hq_l, hkv_l = wl.hq_local, wl.hkv_local
    # One pinned host buffer with every layer's Q/K/V for the step, one for
    # the outputs: a step is H2D copy, 36 calls of the public API, D2H copy.
    h_in = torch.empty_like(wl.inbuf, device="cpu").pin_memory()
    h_in.copy_(wl.inbuf)
    h_out = torch.empty((args.layers, (HQ if world > 1 else hq_l) * D), dtype=torch.bfloat16).pin_memory()

    from genllm_b200.paged_attention import DecodeStep
    one_call = None
    if graph is not None:
        # The whole step's 36 layers through one library call, beside the
        # captured step (one graph launch per step).
        bound = ([b.q for b in wl.layers], [b.k for b in wl.layers], [b.v for b in wl.layers],
                 [b.out for b in wl.layers])
        one_call = DecodeStep(wl.mgr, list(range(args.layers)), *bound, hq_l, wl.scale)
    enqueue = [0.0]

    def e2e_step(runner=None):
        wl.inbuf.copy_(h_in, non_blocking=True)
        if runner is not None:
            h0 = time.perf_counter()
            runner.run()
            enqueue[0] += time.perf_counter() - h0
            h_out.copy_(wl.outbuf, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            return float(h_out[-1, 0])
        h0 = time.perf_counter()
        for l in range(args.layers):
            L = wl.layers[l]
            if hg is not None:
                hg.decode(wl.mgr, l, L.q, L.k, L.v, wl.scale)
            else:
                paged_attention(wl.mgr, l, L.q, L.k, L.v, out=L.out, scale=wl.scale)
                if world > 1:
                    allgather_heads(L.out, gathered[l])
        enqueue[0] += time.perf_counter() - h0
        h_out.copy_(gathered_all if world > 1 else wl.outbuf, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return float(h_out[-1, 0])  # the step's result, read on the host

    def e2e_run(runner):
        for _ in range(2):
            e2e_step(runner)
        ctx1 = wl.cached(0)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        enqueue[0] = 0.0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step(runner)
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1)
        eb = 0
        for k in range(e2e_steps):
            eb += args.layers * wl.bytes_per_layer_token(ctx1 + k + 1)
        te = torch.tensor([e_ms], device="cuda")
        be = torch.tensor([float(eb)], device="cuda", dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
            dist.all_reduce(be, op=dist.ReduceOp.SUM)
        return be.item() / (te.item() / 1e3) / 1e9, te.item() / e2e_steps, 1e3 * enqueue[0] / e2e_steps

    extra_e2e = {}
    e2e_value, e2e_ms, e2e_enq = e2e_run(None)
    e2e_path = ("one pinned H2D copy of all layers Q/K/V, per-layer C ABI calls, one D2H copy of the "
                "outputs, host reads the result")
    if graph is not None:
        v1, ms1, enq1 = e2e_run(one_call)
        v2, ms2, enq2 = e2e_run(graph)
        extra_e2e = {"one_call": {"value": round(v1, 2), "ms_per_step": round(ms1, 4),
                                  "host_call_ms_per_step": round(enq1, 4),
                                  "path": "same copies, one gkv_decode_layers call per step"},
                     "captured_step": {"value": round(v2, 2), "ms_per_step": round(ms2, 4),
                                       "host_call_ms_per_step": round(enq2, 4),
                                       "path": "same copies, one gkv_decode_graph_step call per step"}}
    h2d = h_in.numel() * 2
    d2h = h_out.numel() * 2

    peak, peak_src = measured_peak()
    # Per launch pair (decode + combine of one layer), averaged over the
    # timed region (CUDA events around the K timed steps, launches
    # overlapping as they do in use); the instrumented per-launch pass (events
    # between launches serialise them) is reported beside it.
    pair_ms = ms_max / (args.steps * args.layers)
    achieved = per_launch_bytes / (pair_ms / 1e3) / 1e9
    serialized = (kern_bytes or per_launch_bytes) / (kern_max / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config(args, world),
        "frac_of_8TBps": round(value / NOMINAL_HBM_GBS, 4),
        "us_per_token_layer": round(1e3 * ms_max / (args.steps * args.layers), 3),
        "tok_per_s_qwen3_4b_attention": round(args.steps / (ms_max / 1e3), 2),
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps, "ms_per_step": round(e2e_ms, 4), "host_call_ms_per_step": round(e2e_enq, 4),
                "path": e2e_path, **extra_e2e},
        "gpu_launches": (1 if os.environ.get("GKV_DECODE_FUSED_MERGE") == "1" and not (world > 1 and args.gather == "p2p") else 2) * args.steps * args.layers,
        "gather": (args.gather if world > 1 else None),
        "host_enqueue_ms_per_step": round(1e3 * host_enqueue_s / args.steps, 4),
        "timed_path": "per-layer C ABI calls (decode + combine kernels each), one call per layer",
        "captured_step": captured,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": profiled_traffic(args, world),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of paged_decode_kernel "
                                       "(profiles/paged_decode_kernel_qwen3_4b_32k.md)",
                     "peak_source": peak_src,
                     "kernel": "paged_decode_kernel + paged_decode_combine_kernel (one decode step of one layer)",
                     "kernel_avg_us": round(1e3 * pair_ms, 3),
                     "bytes_per_launch": round(per_launch_bytes),
                     "serialized_launch": {"avg_us": round(1e3 * kern_max, 3), "achieved": round(serialized, 1),
                                           "how": "separate pass, CUDA events recorded between launches (no "
                                                  "overlap of consecutive launches)"}},
        "clocks": clk,
        "parity": parity,
    }
    if rank == 0 and world == 1 and not args.no_other_configs:
        # The other single-GPU configs, measured in the same run (not the
        # headline): config 1 (0.6B layer decode) and config 4 (chunked
        # prefill on the tensor cores).
        c4 = measure_config4(args)
        line["other_configs"] = {
            "config1": measure_config1(args),
            "config4": {"workload": c4["config"]["workload"], "tflops": c4["value"], "ms_per_prompt": c4["ms_per_step"],
                        "last_chunk_tflops": c4["roofline"]["achieved"], "peak": c4["roofline"]["peak"],
                        "frac_of_peak": round(c4["value"] / c4["roofline"]["peak"], 4)}}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_step(args)  # warm-up (and set-up) step, untimed
        runs = [cpu_step(args) for _ in range(3)]
        g = sum(r[5] for r in runs) / sum(r[4] for r in runs) / 1e9
        _, cores, kind, sample, _, _ = runs[0]
        line["cpu_baseline"] = {"value": round(g, 4), "unit": UNIT, "cores": cores, "kind": kind,
                                "sample": sample + "; 3 timed steps after one untimed",
                                "seconds_per_step": round(sum(r[4] for r in runs) / 3, 3)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        if hg is not None:
            hg.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
