#!/usr/bin/env python
"""Benchmark: Qwen1.5-MoE-A2.7B-shaped MoE layer with exponent-compressed
experts on B200.

Workload (one step = one layer forward over one 512-token batch): hidden 2048,
60 routed SwiGLU experts (intermediate 1408), softmax top-4 without
renormalisation, a shared SwiGLU expert (intermediate 5632) with a sigmoid
gate.  Router weights N(0, 0.02) plus a per-expert logit bias giving Zipf(1.0)
expert popularity.  Every routed expert is stored as LZ4HC-9 exponent chunks
(3 per matrix) + raw sign+mantissa plane in HBM; 16 decoded experts are cached
(the 16 most popular are decoded before timing); every other activated expert
is decoded on the GPU inside the step.  Seeded synthetic data (no checkpoint):
weights N(0, 0.02) BF16, activations N(0, 1) BF16.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
Under torchrun (N > 1) the layer is expert-parallel: rank r owns experts
[r*60//N, (r+1)*60//N) (compressed in its HBM, decoded on its GPU), every rank
routes its own 512 tokens (weak scaling) and token rows go to their expert's
rank and back by NCCL all-to-all.  The decoded-expert cache stays 16 experts
for the whole box, split over the ranks in proportion to the experts they own.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from typing import Optional

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "zipmoe-icml26_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "MoE-layer tokens/s"
UNIT = "tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=512)
    ap.add_argument("--cache", type=int, default=16)
    ap.add_argument("--chunks", type=int, default=3)
    ap.add_argument("--codec", default="LZ4HC")
    ap.add_argument("--level", type=int, default=9)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--store", default="device", choices=["device", "host"],
                    help="where the compressed experts live (host: pinned memory, copied in per miss)")
    ap.add_argument("--sm-slots", type=int, default=0,
                    help="host store: experts whose sign+mantissa planes stay in HBM (the SMCACHE pool)")
    ap.add_argument("--matrices", type=int, default=180,
                    help="encode: expert matrices converted per step (180 = one layer's 60 experts)")
    ap.add_argument("--attempts", type=int, default=256,
                    help="encode: hash-chain candidates tried per position (LZ4HC level 9 tries 256)")
    ap.add_argument("--config", default="qwen", choices=["qwen", "decode-sweep", "switch", "deepseek-stack", "encode"],
                    help="qwen: the Qwen1.5-MoE layer (default; the headline line, with a token-count sweep); "
                         "decode-sweep: decode+recombine GB/s over sizes and weight distributions; "
                         "switch: the Switch-large-128 layer at 4096 tokens; deepseek-stack: 26 "
                         "DeepSeek-V2-Lite MoE layers at decode batch sizes, with and without next-layer prefetch; "
                         "encode: the offload conversion (plane split + LZ4 encode) of one layer's 60 experts")
    ap.add_argument("--timeline", default=None,
                    help="write the GPU timeline of 3 more steps (kernels and copies per stream, "
                         "torch.profiler over CUPTI) to this text file")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """SM clock and throttle reasons around and during the timed region, on
    one GPU (inactive when index is None, so that only one rank takes part).

    During the region the clock is measured on the GPU itself: at five points
    of the loop (probe()) a one-thread kernel on a side stream counts SM cycles
    against the GPU's nanosecond timer for 100 us, next to the step's own
    kernels.  The driver is not queried while steps run: an NVML or
    nvidia-smi query stalls the host's synchronisations for milliseconds, and
    in expert-parallel steps every rank then waits at the next collective (it
    cost a third of the 2-GPU throughput).  The throttle reasons, the max
    clock and one more clock reading come from NVML before the region (then
    100 ms pass and the ranks meet at a barrier) and right after it (the GPU
    found by UUID); without NVML they come from one nvidia-smi query at each
    edge."""
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    Q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PROBE_NS = 100_000

    def __init__(self, index: Optional[int]):
        self.index = index
        self.edges = []          # (sm_mhz, sm_max_mhz, [active flags in NAMES order]) before and after
        self.probes = []
        self.source = None

    def _edge(self):
        try:
            import pynvml
            if self.source is None:
                pynvml.nvmlInit()
                uid = str(torch.cuda.get_device_properties(self.index).uuid)
                self.h = None
                for key in (uid, "GPU-" + uid):
                    try:
                        self.h = pynvml.nvmlDeviceGetHandleByUUID(key)
                        break
                    except pynvml.NVMLError:
                        continue
                if self.h is None:
                    raise RuntimeError("no NVML device with UUID " + uid)
                self.source = "nvml"
            nv, h = pynvml, self.h
            bits = [nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                    nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap]
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            self.edges.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                               nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM), [bool(r & b) for b in bits]))
        except Exception:
            self.source = "nvidia-smi"
            try:
                line = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                      timeout=30).stdout.strip().splitlines()[0]
                parts = [x.strip() for x in line.split(",")]
                self.edges.append((float(parts[0]), float(parts[1]), [v.lower() == "active" for v in parts[2:6]]))
            except Exception:
                pass

    def __enter__(self):
        if self.index is None:
            return self
        self._edge()
        time.sleep(0.1)          # driver work that a query starts can outlast the call
        from zmoe._lib import lib
        self.lib = lib
        self.buf = torch.zeros(5, 2, dtype=torch.int64, device=torch.device("cuda", self.index))
        self.side = torch.cuda.Stream(device=torch.device("cuda", self.index))
        return self

    def probe(self, i: int, steps: int):
        """Call before step i of steps: probes at 5 evenly spread steps."""
        if self.index is None:
            return
        points = sorted({0, steps // 4, steps // 2, (3 * steps) // 4, max(steps - 1, 0)})
        if i in points and len(self.probes) < 5:
            slot = len(self.probes)
            self.probes.append(slot)
            st = self.lib.zmoe_clock_probe(self.buf[slot].data_ptr(), self.PROBE_NS, self.side.cuda_stream)
            if st != 0:
                self.probes.pop()

    def __exit__(self, *a):
        if self.index is None:
            return
        torch.cuda.synchronize(self.index)
        self._edge()

    def summary(self):
        if self.index is None:
            return None
        got = self.buf[: len(self.probes)].cpu().tolist() if self.probes else []
        mhz = [c * 1000.0 / ns for c, ns in got if ns > 0]
        if not mhz and not self.edges:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        reasons = sorted({self.NAMES[i] for _, _, r in self.edges for i, v in enumerate(r) if v})
        return {"sm_mhz": round(statistics.median(mhz), 1) if mhz else statistics.median(e[0] for e in self.edges),
                "sm_max_mhz": max((e[1] for e in self.edges), default=None), "reasons": reasons,
                "samples": len(mhz),
                "edge_sm_mhz": [e[0] for e in self.edges],
                "source": f"SM cycles / GPU timer on the GPU during the loop; {self.source} at its edges"}


def build_workload(args, device_index=0, threads=0):
    from zmoe import synthetic as syn
    from zmoe.layer import MoELayer
    s = syn.QWEN
    w = syn.expert_weights(s, 1)[0]
    wr, sg = syn.router_weights(s)
    sh = syn.shared_weights(s)
    bias = syn.zipf_bias(s, 0)
    L = MoELayer(s, max_tokens=args.tokens, cache_slots=args.cache, device=device_index,
                 store=getattr(args, "store", "device"), sm_slots=getattr(args, "sm_slots", 0))
    L.set_router(wr, bias, sg)
    L.set_shared(*sh)
    enc = L.load_experts(w, num_file_chunks=args.chunks, codec=args.codec, level=args.level, threads=threads)
    warm = syn.popularity_order(s, 0)[: args.cache]
    L.warm_cache(warm)
    return s, L, enc, (wr, bias, sg, sh, warm)


def cpu_reference_layer(s, enc, extra, threads):
    from oracle.reference_cpu import ReferenceCPULayer
    wr, bias, sg, sh, warm = extra
    shapes = [(s.inter, s.hidden), (s.inter, s.hidden), (s.hidden, s.inter)]
    return ReferenceCPULayer(shapes, enc, wr, bias, sg, sh, s.topk, warm, threads=threads)


def cpu_model() -> str:
    """Host CPU model name (lscpu "Model name", else /proc/cpuinfo)."""
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for ln in out.splitlines():
            if ln.strip().lower().startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.lower().startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def bench_config(args, s, world):
    """The workload as both arms print it (the same dict, so the lines compare)."""
    return {"workload": "qwen1.5-moe-layer", "tokens_per_gpu": args.tokens, "hidden": s.hidden,
            "experts": s.num_experts, "inter": s.inter, "topk": s.topk, "shared_inter": s.shared_inter,
            "cached_experts": args.cache, "codec": f"{args.codec}-{args.level}",
            "num_file_chunks": args.chunks, "zipf_s": s.zipf_s,
            "parallelism": f"ep{world}" if world > 1 else "single", "store": args.store,
            "sm_slots": args.sm_slots,
            "l2": "inputs larger than L2 (decoded + compressed experts > 1 GB)"}


def run_reference(args):
    """The reference's CPU path (oracle port: liblz4 + torch CPU) on the host
    cores; prints the reference line.  Nothing of this repository's library is
    loaded in this process: the experts are encoded by the oracle's liblz4
    bindings too."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from oracle import codec as oc
    from zmoe import synthetic as syn      # pure Python: seeded tensors, no native code
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    s = syn.QWEN
    w = syn.expert_weights(s, 1)[0]
    wr, sg = syn.router_weights(s)
    sh = syn.shared_weights(s)
    bias = syn.zipf_bias(s, 0)
    flat = oc.encode_tensors([t for e in w for t in e], args.chunks, args.codec, args.level, threads)
    enc = [flat[i * 3:(i + 1) * 3] for i in range(s.num_experts)]
    warm = syn.popularity_order(s, 0)[: args.cache]
    L = cpu_reference_layer(s, enc, (wr, bias, sg, sh, warm), threads)
    x = syn.activations(args.tokens, s.hidden)
    for _ in range(args.warmup):
        L.forward(x)
    t0 = time.perf_counter()
    st = None
    for _ in range(args.steps):
        _, st = L.forward(x)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    L.close()
    v = args.tokens / dt
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
            "config": bench_config(args, s, world),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "cpu_model": cpu_model(), "kind": "port",
                             "sample": f"{args.steps} full {args.tokens}-token layer steps: liblz4 decode of "
                                       f"{st['misses']} missed experts on {threads} threads + torch CPU BF16 layer"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def write_timeline(step, steps, path):
    """Runs step() `steps` times under torch.profiler (CUDA activity only) and
    writes every kernel and copy with its stream, start and duration (us,
    relative to the first), then which kernels ran while a decode kernel ran
    on another stream."""
    import tempfile
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            step()
        torch.cuda.synchronize()
    with tempfile.TemporaryDirectory() as d:
        tp = os.path.join(d, "trace.json")
        prof.export_chrome_trace(tp)
        tr = json.load(open(tp))
    ev = [e for e in tr.get("traceEvents", []) if e.get("cat") in ("kernel", "gpu_memcpy", "gpu_memset")]
    ev.sort(key=lambda e: e["ts"])
    t0 = ev[0]["ts"] if ev else 0.0
    short = lambda n: n.split("(")[0].replace("void ", "").replace("zmoe::", "").replace("(anonymous namespace)::", "")
    lines = [f"# {len(ev)} GPU activities over {steps} steps (us from the first; stream = CUDA stream id)",
             f"{'start':>10} {'dur':>8} {'stream':>6}  name"]
    for e in ev:
        lines.append(f"{e['ts'] - t0:10.1f} {e['dur']:8.1f} {e['args'].get('stream', -1):>6}  {short(e['name'])}")
    dec = [e for e in ev if e.get("cat") == "kernel" and ("map_kernel" in e["name"] or "resolve_kernel" in e["name"])]
    lines.append("")
    lines.append("# kernels that overlapped a decode kernel of another stream (us of overlap)")
    tot = {}
    for e in ev:
        if e.get("cat") != "kernel" or e in dec:
            continue
        a, b = e["ts"], e["ts"] + e["dur"]
        ov = sum(max(0.0, min(b, d["ts"] + d["dur"]) - max(a, d["ts"])) for d in dec
                 if d["args"].get("stream") != e["args"].get("stream"))
        if ov > 0:
            k = short(e["name"])
            tot[k] = tot.get(k, 0.0) + ov
    for k, v in sorted(tot.items(), key=lambda kv: -kv[1]):
        lines.append(f"{v / steps:10.1f} per step  {k}")
    with open(path, "w") as f:
        f.write("\n".join(lines) + "\n")


def run_ours(args):
    world, rank, local = dist_env()
    if world > 1:
        return run_ep(args)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    threads = max(1, (os.cpu_count() or 1) // max(world, 1))
    s, L, enc, extra = build_workload(args, local, threads)
    from zmoe import synthetic as syn
    x = syn.activations(args.tokens, s.hidden, seed=1 + rank).cuda()
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        L.forward(x, out)
    L.sync()
    L.reset_stats()
    L.set_timing(True)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:          # its first driver reading comes before the barrier
        barrier()
        start.record(stream)
        for i in range(args.steps):
            clk.probe(i, args.steps)
            L.forward(x, out)
        stop.record(stream)
        torch.cuda.synchronize()
    L.sync()
    barrier()
    ms = start.elapsed_time(stop) / args.steps
    st = L.stats()
    L.set_timing(False)
    if args.timeline and rank == 0:
        write_timeline(lambda: L.forward(x, out), 3, args.timeline)
    sweep = token_sweep(L, s, args) if args.config == "qwen" else None

    # end to end through the public API with pinned host buffers: every step
    # copies its input in and its output back (zmoe_layer_submit_host, copies
    # pipelined with the neighbouring steps' compute); the timed region ends
    # when the last output copy has landed
    xh = x.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    for _ in range(2):
        L.forward_host(xh, oh)
    if not torch.equal(oh, out.cpu()):
        raise RuntimeError("forward_host output differs from forward")
    oh.zero_()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        L.submit_host(xh, oh)
    L.join_host()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if not torch.equal(oh, out.cpu()):
        raise RuntimeError("submit_host output differs from forward")

    t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = float(t[0]), float(t[1])
    clocks = clk.summary()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args, s, enc, extra)
    if rank == 0:
        hbm, tfl, src = peaks()
        dec_s = st["decode_ns"] * 1e-9
        launches = max(st["decode_timed_launches"], 1)
        achieved = (st["decode_timed_bytes"] / launches) / (dec_s / launches) / 1e9 if dec_s > 0 else 0.0
        traffic, traffic_src = None, None
        tp = os.path.join(ROOT, "profiles", "decode_traffic.json")
        if os.path.exists(tp):          # an ncu figure for this launch, not measured in this run
            traffic = json.load(open(tp)).get("bytes_per_launch")
            traffic_src = "ncu dram__bytes_read.sum + dram__bytes_write.sum of one 252-chunk launch pair " \
                          "(profiles/decode_traffic.json), not measured in this run"
        line = {
            "metric": METRIC, "value": world * args.tokens / (ms / 1e3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
            "config": bench_config(args, s, world),
            "e2e": {"value": world * args.tokens / (e2e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": x.numel() * 2},
            "roofline": {"bound": "hbm", "kernel": "map_kernel+resolve_kernel (fused LZ4 decode)", "achieved": achieved,
                         "peak": hbm, "unit": "GB/s", "frac": achieved / hbm, "peak_source": src, "traffic": traffic,
                         "traffic_source": traffic_src,
                         "algorithmic_bytes_per_launch": st["decode_timed_bytes"] / launches,
                         "kernel_ms_per_launch": dec_s * 1e3 / launches},
            "decode": {"experts_per_step": st["decoded_experts"] / args.steps,
                       "gb_per_s": achieved, "share_of_step": dec_s / (ms * 1e-3 * args.steps)},
            "ffn_ms_per_step": st["ffn_ns"] * 1e-6 / args.steps,
            "cache": {"hits": st["hits"], "misses": st["misses"], "evictions": st["evictions"]},
            "gpu_launches": st["launches"],
            "clocks": clocks,
        }
        if sweep is not None:
            line["tokens_sweep"] = sweep
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    L.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_ep(args):
    """Expert-parallel layer over WORLD_SIZE ranks (one GPU each)."""
    import datetime
    import torch.distributed as dist
    from zmoe import codec as zc
    from zmoe import ep
    from zmoe import synthetic as syn
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    s = syn.QWEN
    part = ep.ExpertPartition(s.num_experts, world)
    mine = part.owned(rank)
    w = syn.expert_weights(s, 1)[0]
    wr, sg = syn.router_weights(s)
    sh = syn.shared_weights(s)
    bias = syn.zipf_bias(s, 0)
    threads = max(1, (os.cpu_count() or 1) // world)
    flat = zc.encode_tensors([t for e in mine for t in w[e]], args.chunks, args.codec, args.level, threads)
    enc = [None] * s.num_experts
    for j, e in enumerate(mine):
        enc[e] = flat[j * 3:(j + 1) * 3]
    cache = max(1, round(args.cache * len(mine) / s.num_experts))
    warm = syn.popularity_order(s, 0)[: args.cache]
    L = ep.build_gpu_layer(s, enc, wr, bias, sg, sh, max_tokens=args.tokens, cache_slots=cache, device=local,
                           warm=warm)
    eng = L.engine
    x = syn.activations(args.tokens, s.hidden, seed=1 + rank).cuda()
    stream = torch.cuda.current_stream()

    def barrier():
        dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        L(x)
    eng.sync()
    eng.reset_stats()
    eng.set_timing(True)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local if rank == 0 else None) as clk:   # first driver reading before the barrier
        barrier()
        start.record(stream)
        for i in range(args.steps):
            clk.probe(i, args.steps)
            L(x)
        stop.record(stream)
        torch.cuda.synchronize()
    eng.sync()
    barrier()
    ms = start.elapsed_time(stop) / args.steps
    st = eng.stats()
    eng.set_timing(False)

    # end to end: pinned host tokens in, host output back, every step
    xh = x.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    xd = torch.empty_like(x)

    def host_step():
        xd.copy_(xh, non_blocking=True)
        oh.copy_(L(xd), non_blocking=True)

    for _ in range(2):
        host_step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local if rank == 0 else None) as clk2:   # its driver reading comes before the barrier
        barrier()
        e0.record(stream)
        for i in range(args.steps):
            clk2.probe(i, args.steps)                 # the same side-stream probes as the device-timed loop
            host_step()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    # every rank's own step times, then the max over ranks
    per = torch.tensor([ms, e2e_ms], dtype=torch.float64, device="cuda")
    gathered = [torch.zeros_like(per) for _ in range(world)]
    dist.all_gather(gathered, per)
    per_rank = [[round(float(g[0]), 4), round(float(g[1]), 4)] for g in gathered]
    ms = max(p[0] for p in per_rank)
    e2e_ms = max(p[1] for p in per_rank)
    clocks = clk.summary()
    if rank == 0:
        hbm, tfl, src = peaks()
        dec_s = st["decode_ns"] * 1e-9
        launches = max(st["decode_timed_launches"], 1)
        achieved = (st["decode_timed_bytes"] / launches) / (dec_s / launches) / 1e9 if dec_s > 0 else 0.0
        # per step: router 1, permute 3, gathers 2, shared FFN 2, combine 1 + the engine's own
        # (NCCL's own kernels are not counted)
        ep_launches = 9 * args.steps
        line = {
            "metric": METRIC, "value": world * args.tokens / (ms / 1e3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
            "config": bench_config(args, s, world),
            "ep": {"cached_experts_rank0": cache, "experts_rank0": len(mine),
                   "exchange": "libzmoe.so zmoe_ep_forward: grouped ncclSend/ncclRecv of counts, BF16 rows out "
                               "and BF16 rows back on torch's NCCL communicator; one host wait per step",
                   "per_rank_ms_value_e2e": per_rank},
            "e2e": {"value": world * args.tokens / (e2e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": x.numel() * 2},
            "roofline": {"bound": "hbm", "kernel": "map_kernel+resolve_kernel (fused LZ4 decode)", "achieved": achieved,
                         "peak": hbm, "unit": "GB/s", "frac": achieved / hbm, "peak_source": src, "traffic": None,
                         "algorithmic_bytes_per_launch": st["decode_timed_bytes"] / launches,
                         "kernel_ms_per_launch": dec_s * 1e3 / launches},
            "decode": {"experts_per_step_rank0": st["decoded_experts"] / args.steps,
                       "gb_per_s": achieved, "share_of_step": dec_s / (ms * 1e-3 * args.steps)},
            "cache": {"hits": st["hits"], "misses": st["misses"], "evictions": st["evictions"]},
            "gpu_launches": st["launches"] + ep_launches,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    if hasattr(L, "close"):
        L.close()                                      # the native layer before its engine and the communicator
    eng.close()
    dist.barrier()
    dist.destroy_process_group()


def token_sweep(L, s, args):
    """The same layer (same cache state going in) at the other batch sizes of
    the Qwen config: tokens/s, step time and experts decoded per step."""
    from zmoe import synthetic as syn
    out = {}
    for T in (1, 16, 128):
        xs = syn.activations(T, s.hidden, seed=50 + T).cuda()
        os_ = torch.empty_like(xs)
        for _ in range(3):
            L.forward(xs, os_)
        L.sync()
        before = L.stats()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            L.forward(xs, os_)
        b.record()
        torch.cuda.synchronize()
        L.sync()
        ms = a.elapsed_time(b) / args.steps
        st = L.stats()
        dec = (st["decoded_experts"] - before["decoded_experts"]) / args.steps
        touched = (st["hits"] + st["misses"] - before["hits"] - before["misses"]) / args.steps
        out[str(T)] = {"tokens_per_s": T / (ms * 1e-3), "ms_per_step": ms, "experts_touched_per_step": touched,
                       "experts_decoded_per_step": dec}
    return out


def weight_family(name: str, scale: float, shape, seed: int):
    """BF16 matrices whose exponent planes compress differently: normal(sd),
    laplace(b) and uniform(+-a) draws, seeded."""
    gen = torch.Generator().manual_seed(seed)
    if name == "normal":
        w = torch.randn(*shape, generator=gen) * scale
    elif name == "laplace":
        u = torch.rand(*shape, generator=gen) - 0.5
        w = -scale * torch.sign(u) * torch.log1p(-2 * u.abs())
    else:
        w = (torch.rand(*shape, generator=gen) * 2 - 1) * scale
    return w.to(torch.bfloat16)


def run_decode_sweep(args):
    """Decode+recombine throughput over total sizes and weight distributions
    (the decompression-bandwidth sweep): for each family a pool of 8 distinct
    Qwen-shaped matrices is encoded (LZ4HC-9, 3 chunks), copied on the device
    until the requested size is reached (every copy has its own source bytes,
    so nothing is served from L2), and decoded in launches of up to 1 GiB of
    output.  Each rank decodes its own copies (weak scaling); value is the
    sum over ranks at the largest size for normal(0.02)."""
    import datetime
    from zmoe import codec as zc
    from zmoe import ops
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    families = [("normal", 0.005), ("normal", 0.02), ("normal", 0.08), ("normal", 0.0283), ("laplace", 0.02),
                ("uniform", 0.05)]
    sizes_mb = [1, 16, 256, 1024, 4096, 8192]
    shape = (1408, 2048)
    n_el = shape[0] * shape[1]
    results = []
    hbm, _, src = peaks()
    threads = max(1, (os.cpu_count() or 1) // world)
    for fi, (fam, scale) in enumerate(families):
        pool = [weight_family(fam, scale, shape, 1000 * fi + i) for i in range(8)]
        enc = zc.encode_tensors(pool, args.chunks, args.codec, args.level, threads)
        ratio = sum(e.compressed_bytes for e in enc) / sum(e.numel for e in enc)
        base = [ops.CompressedTensor(e.blocks, e.original_sizes, e.sm) for e in enc]
        for mb in sizes_mb:
            n_mat = max(1, int(round(mb * 2 ** 20 / (2 * n_el))))
            small = mb * 2 ** 20 < 2 * n_el
            if small:                                   # 1 MB: the leading rows of one matrix
                rows = max(1, mb * 2 ** 20 // (2 * shape[1]))
                e = zc.encode_tensors([pool[0][:rows]], args.chunks, args.codec, args.level, threads)[0]
                cts = [ops.CompressedTensor(e.blocks, e.original_sizes, e.sm)]
                n_out = [e.numel]
            else:
                cts = []
                for i in range(n_mat):
                    b = base[i % len(base)]
                    c = object.__new__(ops.CompressedTensor)
                    c.__dict__.update(b.__dict__)
                    if i >= len(base):                  # its own device copy of the source bytes
                        c.blocks, c.sm = b.blocks.clone(), b.sm.clone()
                        c.indexes = b.indexes.clone()
                    cts.append(c)
                n_out = [n_el] * n_mat
            total = sum(n_out)
            dst = torch.empty(total, dtype=torch.bfloat16, device="cuda")
            launches, pos, cur = [], 0, []
            cap = 2 ** 29                               # elements (1 GiB of BF16) per launch
            for c, n in zip(cts, n_out):
                if cur and sum(d[4] for d in cur) + n > cap:
                    launches.append(cur)
                    cur = []
                cur.extend(c.descs(dst[pos:pos + n]))
                pos += n
            launches.append(cur)
            tables = []
            for d in launches:
                scratch = ops.map_scratch([x[4] for x in d], "cuda")
                tables.append((ops.chunk_table(d, "cuda", scratch), len(d), scratch,
                               torch.zeros(len(d), dtype=torch.int32, device="cuda")))
            alg = sum(x[3] + 3 * x[4] for d in launches for x in d)

            def once():
                for tab, n, _, st in tables:
                    ops.check(ops.lib.zmoe_decode_chunks(tab.data_ptr(), n, st.data_ptr(),
                                                         torch.cuda.current_stream().cuda_stream), "decode")
            for _ in range(2):
                once()
            torch.cuda.synchronize()
            if dist is not None:
                dist.barrier()
            reps = max(1, min(args.steps, int(2e9 // max(alg, 1)) + 1))
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(reps):
                once()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / reps
            ok = all(bool((t[3] == 0).all()) for t in tables)
            if mb == sizes_mb[-1] or small:             # bit-exact check of the first matrix
                want = codec_bits(pool[0][:rows] if small else pool[0]).reshape(-1)
                ok = ok and torch.equal(dst[:want.numel()].view(torch.int16).cpu(), want)
            t = torch.tensor([ms], dtype=torch.float64, device="cuda")
            if dist is not None:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t[0])
            gbs = world * alg / (ms * 1e-3) / 1e9
            results.append({"family": f"{fam}({scale})", "exp_ratio": round(ratio, 4), "size_mb": mb,
                            "chunks": sum(len(d) for d in launches), "ms": round(ms, 4), "gb_per_s": round(gbs, 1),
                            "frac_of_hbm": round(gbs / world / hbm, 4), "status_ok": ok})
            del tables, dst, cts
            torch.cuda.empty_cache()
    head = [r for r in results if r["family"] == "normal(0.02)" and r["size_mb"] == sizes_mb[-1]][0]
    if rank == 0:
        cpu = cpu_decode_baseline(args) if not args.no_cpu_baseline and world == 1 else None
        line = {"metric": "expert decode+recombine GB/s (algorithmic bytes)", "value": head["gb_per_s"],
                "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": 2,
                "ms_per_step": head["ms"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "u8", "data": "synthetic (seeded weight families, see results)",
                "config": {"workload": "decode-sweep", "codec": f"{args.codec}-{args.level}",
                           "num_file_chunks": args.chunks, "sizes_mb_per_gpu": sizes_mb,
                           "l2": "inputs larger than L2 from 256 MB up"},
                "roofline": {"bound": "hbm", "achieved": head["gb_per_s"] / world, "peak": hbm, "unit": "GB/s",
                             "frac": head["gb_per_s"] / world / hbm, "peak_source": src, "traffic": None},
                "results": results}
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_switch(args):
    """Switch-large-128 layer (d_model 1024, 128 ReLU experts of 2816, top-1,
    capacity factor 1.25, overflow tokens passed through) over 4096 tokens:
    one GPU holds all 128 experts (16 decoded in the cache, the rest
    compressed); under torchrun the experts are sharded (16 per GPU at 8 GPUs)
    and each rank routes 4096 / N tokens as its own sequence, so the capacity
    is floor(1.25 * (4096 / N) / 128) per rank."""
    import dataclasses
    import datetime
    from zmoe import ep
    from zmoe import synthetic as syn
    from zmoe.layer import MoELayer
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    T = 4096 // world
    s = dataclasses.replace(syn.SWITCH, capacity=(125 * T) // (100 * syn.SWITCH.num_experts), seq_len=T)
    w = syn.expert_weights(s, 1)[0]
    wr, _ = syn.router_weights(s)
    threads = max(1, (os.cpu_count() or 1) // world)
    cache = max(1, 16 // world)
    if world == 1:
        L = MoELayer(s, max_tokens=T, cache_slots=cache, device=local)
        L.set_router(wr, None, None)
        L.load_experts(w, num_file_chunks=args.chunks, codec=args.codec, level=args.level, threads=threads)
        eng = L
    else:
        from zmoe import codec as zc
        part = ep.ExpertPartition(s.num_experts, world)
        mine = part.owned(rank)
        flat = zc.encode_tensors([t for e in mine for t in w[e]], args.chunks, args.codec, args.level, threads)
        enc = [None] * s.num_experts
        for j, e in enumerate(mine):
            enc[e] = flat[j * 2:(j + 1) * 2]
        L = ep.build_gpu_layer(s, enc, wr, None, None, None, max_tokens=T, cache_slots=cache, device=local)
        eng = L.engine
    x = syn.activations(T, s.hidden, seed=1 + rank).cuda()
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        L(x, out) if world == 1 else L(x)
    eng.sync()
    eng.reset_stats()
    eng.set_timing(True)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local if rank == 0 else None) as clk:
        barrier()
        a.record(stream)
        for i in range(args.steps):
            clk.probe(i, args.steps)
            L(x, out) if world == 1 else L(x)
        b.record(stream)
        torch.cuda.synchronize()
    eng.sync()
    ms = a.elapsed_time(b) / args.steps
    st = eng.stats()
    eng.set_timing(False)
    xh = x.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    xd = torch.empty_like(x)

    def host_step():
        xd.copy_(xh, non_blocking=True)
        oh.copy_(L(xd), non_blocking=True)

    for _ in range(2):
        host_step()
    a2, b2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local if rank == 0 else None) as clk2:
        barrier()
        a2.record(stream)
        for i in range(args.steps):
            clk2.probe(i, args.steps)
            host_step()
        b2.record(stream)
        torch.cuda.synchronize()
    e2e_ms = a2.elapsed_time(b2) / args.steps
    t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = float(t[0]), float(t[1])
    if rank == 0:
        hbm, _, src = peaks()
        dec_s = st["decode_ns"] * 1e-9
        launches = max(st["decode_timed_launches"], 1)
        achieved = (st["decode_timed_bytes"] / launches) / (dec_s / launches) / 1e9 if dec_s > 0 else 0.0
        line = {"metric": "MoE-layer tokens/s", "value": world * T / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations, uniform router)",
                "config": {"workload": "switch-large-128-layer", "tokens_total": 4096, "tokens_per_gpu": T,
                           "hidden": s.hidden, "experts": s.num_experts, "inter": s.inter, "topk": 1,
                           "capacity_per_rank": s.capacity, "cached_experts_per_gpu": cache,
                           "codec": f"{args.codec}-{args.level}", "num_file_chunks": args.chunks,
                           "parallelism": f"ep{world}" if world > 1 else "single"},
                "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s",
                        "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": x.numel() * 2},
                "roofline": {"bound": "hbm", "kernel": "map_kernel+resolve_kernel (fused LZ4 decode)",
                             "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                             "peak_source": src, "traffic": None},
                "decode": {"experts_per_step_rank0": st["decoded_experts"] / args.steps},
                "cache": {"hits": st["hits"], "misses": st["misses"]},
                "gpu_launches": st["launches"], "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    if world > 1 and hasattr(L, "close"):
        L.close()
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_deepseek_stack(args):
    """26 DeepSeek-V2-Lite-shaped MoE layers (64 SwiGLU experts of 1408, top-6
    softmax, routed_scaling 1.0, 2 shared experts of combined 2816, Zipf(1.2)
    popularity with a per-layer seeded permutation), one GPU, decode batches
    of 1 and 64 tokens, 16 decoded experts cached per layer.  The stack's
    input is the layer-to-layer chain: layer l + 1 takes layer l's output,
    and every step feeds new tokens, as decoding does.
    Each batch size runs twice: without prefetch, and with the next-layer
    predictor (ExpertPredictor: 0.8 * count + 0.2 * last-5 visits, top-6)
    asking layer l + 1 to decode its predicted experts into its cache before
    layer l runs, so those decodes overlap layer l.  Expert weights: a seeded
    pool of 64 experts, each layer taking them in its own seeded order (every
    layer holds and decodes its own copy of the compressed bytes)."""
    from zmoe import codec as zc
    from zmoe import synthetic as syn
    from zmoe.layer import MoELayer
    from zmoe.predictor import ExpertPredictor
    world, rank, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    s = syn.DEEPSEEK
    n_layers, cache, Tmax = 26, 16, 64
    threads = os.cpu_count() or 1
    pool = syn.expert_weights(s, 1)[0]
    enc = zc.encode_tensors([t for e in pool for t in e], args.chunks, args.codec, args.level, threads)
    enc = [enc[3 * e:3 * e + 3] for e in range(s.num_experts)]
    layers = []
    for li in range(n_layers):
        perm = torch.randperm(s.num_experts, generator=torch.Generator().manual_seed(100 + li)).tolist()
        wr, _ = syn.router_weights(s, seed=2 + 1000 * li)
        sh = syn.shared_weights(s, seed=4 + 1000 * li)
        L = MoELayer(s, max_tokens=Tmax, cache_slots=cache, device=local)
        L.set_router(wr, syn.zipf_bias(s, li), None)
        L.set_shared(*sh)
        for e in range(s.num_experts):
            for t, et in enumerate(enc[perm[e]]):
                L.load_encoded(e, t, et)
        L.warm_cache(syn.popularity_order(s, li)[:cache])
        layers.append(L)
    stream = torch.cuda.current_stream()
    results = {}
    for T in (1, 64):
        for prefetch in (False, True):
            pred = ExpertPredictor(n_layers, s.topk)
            n_in = max(args.warmup, 3) + args.steps
            xs = syn.activations(n_in * T, s.hidden, seed=1).view(n_in, T, s.hidden).cuda()   # new tokens every step
            outs = [torch.empty_like(xs[0]) for _ in range(n_layers)]
            step_no = [0]

            def stack():
                x = xs[step_no[0] % n_in]
                step_no[0] += 1
                for li, L in enumerate(layers):
                    if prefetch and li + 1 < n_layers:
                        _, want = pred.predict_next_layer(li)
                        if want:
                            layers[li + 1].prefetch(want[:cache])
                    L.forward(x, outs[li])
                    pred.update(li, [e for e, c in enumerate(L.last_counts()) if c > 0])
                    x = outs[li]
                return x

            for _ in range(max(args.warmup, 3)):
                stack()
            torch.cuda.synchronize()
            before = [L.stats() for L in layers]
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(args.steps):
                stack()
            b.record(stream)
            torch.cuda.synchronize()
            for L in layers:
                L.sync()
            ms = a.elapsed_time(b) / args.steps
            after = [L.stats() for L in layers]
            hits = sum(y["hits"] - x["hits"] for x, y in zip(before, after))
            misses = sum(y["misses"] - x["misses"] for x, y in zip(before, after))
            dec = sum(y["decoded_experts"] - x["decoded_experts"] for x, y in zip(before, after))
            results[f"T{T}_{'prefetch' if prefetch else 'no_prefetch'}"] = {
                "tokens_per_s": T / (ms * 1e-3), "ms_per_stack": ms, "hit_rate": hits / max(hits + misses, 1),
                "experts_decoded_per_stack": dec / args.steps}
    head = results["T64_prefetch"]
    line = {"metric": "MoE-stack tokens/s (26 layers)", "value": head["tokens_per_s"], "unit": "tokens/s",
            "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": head["ms_per_stack"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) expert pool, per-layer routers, N(0,1) input)",
            "config": {"workload": "deepseek-v2-lite-moe-stack", "layers": n_layers, "experts": s.num_experts,
                       "inter": s.inter, "topk": s.topk, "shared_inter": s.shared_inter, "zipf_s": s.zipf_s,
                       "cached_experts_per_layer": cache, "codec": f"{args.codec}-{args.level}",
                       "num_file_chunks": args.chunks, "parallelism": "single"},
            "results": results}
    print(json.dumps(line), flush=True)
    for L in layers:
        L.close()


def codec_bits(t):
    return t.contiguous().view(torch.int16).cpu()


def cpu_decode_baseline(args):
    """liblz4 decode (LZ4_decompress_safe_partial, one chunk per task) plus the
    numpy recombine on every host thread, over 32 Qwen chunks of normal(0.02)."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import codec as oc
    threads = os.cpu_count() or 1
    mats = [weight_family("normal", 0.02, (1408, 2048), 7000 + i) for i in range(11)]
    enc = oc.encode_tensors(mats, args.chunks, args.codec, args.level, threads)
    chunks = [(b, o) for e in enc for b, o in zip(e.blocks, e.original_sizes)][:32]
    sms = [np.frombuffer(e.sm, np.uint8) for e in enc]
    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        outs = list(ex.map(lambda c: oc.lz4_decompress(c[0], c[1]), chunks))
        rec = list(ex.map(lambda i: oc.recombine(outs[i], sms[i // 3][(i % 3) * outs[0].size:][:outs[i].size]),
                          range(len(outs))))
    dt = time.perf_counter() - t0
    alg = sum(len(b) + 3 * o for b, o in chunks)
    del rec
    return {"value": alg / dt / 1e9, "unit": "GB/s", "cores": threads, "cpu_model": cpu_model(), "kind": "port",
            "sample": f"{len(chunks)} LZ4 chunks of 961,195 B decoded and recombined on {threads} threads"}


def cpu_baseline(args, s, enc, extra):
    from zmoe import synthetic as syn
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    enc_py = enc
    L = cpu_reference_layer(s, enc_py, extra, threads)
    x = syn.activations(args.tokens, s.hidden, seed=1)
    L.forward(x)
    n, t0 = 0, time.perf_counter()
    st = None
    while n < 3 and time.perf_counter() - t0 < 20:
        _, st = L.forward(x)
        n += 1
    dt = (time.perf_counter() - t0) / n
    L.close()
    return {"value": args.tokens / dt, "unit": UNIT, "cores": threads, "cpu_model": cpu_model(), "kind": "port",
            "sample": f"{n} full {args.tokens}-token layer steps ({st['misses']} misses decoded by liblz4 on "
                      f"{threads} threads, torch CPU BF16 experts)"}


ENCODE_METRIC = "expert LZ4 encode GB/s (exponent bytes in)"


def encode_config(args):
    m = args.matrices
    return {"workload": "qwen1.5-moe-layer-offload" if m == 180 else f"qwen1.5-moe-offload-{m}-matrices",
            "experts": -(-m // 3), "matrices": m, "matrices_shape": "gate/up 1408 x 2048, down 2048 x 1408",
            "num_file_chunks": args.chunks, "chunks": m * args.chunks, "exponent_bytes": m * 1408 * 2048,
            "l2": f"inputs {'larger' if m * 1408 * 2048 > 126e6 else 'smaller'} than L2 "
                  f"({m * 1408 * 2048 / 1e6:.0f} MB of exponent bytes)"}


def cpu_encode_baseline(args, mats, threads):
    """liblz4 LZ4_compress_HC at the configured level, one exponent chunk per
    task on every host thread (TensorEngine::PipelineCompress's compute pool),
    over the chunks of the first 8 matrices."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import codec as oc
    chunks = []
    for m in mats[:8]:
        exp, _ = oc.split_planes(codec_bits(m).numpy().view(np.uint16))
        chunks += oc.chunk_exponents(exp, args.chunks)
    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        out = list(ex.map(lambda c: len(oc.lz4_compress_hc(c, args.level)), chunks))
    dt = time.perf_counter() - t0
    n = sum(c.size for c in chunks)
    return {"value": n / dt / 1e9, "unit": "GB/s", "cores": threads, "cpu_model": cpu_model(), "kind": "port",
            "ratio": sum(out) / n,
            "sample": f"{len(chunks)} exponent chunks of 961,195 B compressed by liblz4 LZ4_compress_HC level "
                      f"{args.level} on {threads} threads"}


def run_encode(args):
    """Offload conversion of one Qwen1.5-MoE layer's 60 routed experts (180
    BF16 matrices of 1408 x 2048): per matrix the plane split and its exponent
    plane cut into 3 chunks, then every chunk LZ4-encoded in one launch
    (zmoe_lz4_encode_chunks, 256 hash-chain candidates per position, as LZ4HC
    level 9).  value: exponent bytes per second with the weights resident;
    e2e: the same through ops.encode_tensors with the BF16 weights copied in
    from pinned host memory and the blocks and sign+mantissa planes copied
    back every step."""
    from zmoe import ops
    from zmoe import synthetic as syn
    world, rank, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    s = syn.QWEN
    mats = [t for e in syn.expert_weights(s, 1)[0] for t in e][:args.matrices]
    dev = [m.cuda() for m in mats]
    n_exp = sum(m.numel() for m in mats)
    for _ in range(max(args.warmup, 3)):
        enc = ops.encode_tensors(dev, args.chunks, args.attempts)
    torch.cuda.synchronize()
    # parity of every block of the first matrix against the oracle's statement
    from oracle import codec as oc
    exp0, _ = oc.split_planes(codec_bits(mats[0]).numpy().view(np.uint16))
    for c, b in zip(oc.chunk_exponents(exp0, args.chunks), enc[0][0]):
        if b.cpu().numpy().tobytes() != oc.lz4_encode_chains(c, args.attempts):
            raise RuntimeError("GPU LZ4 block differs from the oracle's")
    out_bytes = sum(b.numel() for e in enc for b in e[0])
    del enc
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        a.record(stream)
        for i in range(args.steps):
            clk.probe(i, args.steps)
            enc = ops.encode_tensors(dev, args.chunks, args.attempts)
        b.record(stream)
        torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    # end to end: pinned host weights in, blocks and sm planes out, every step
    hw = [m.contiguous().pin_memory() for m in mats]
    caps = sum(m.numel() + m.numel() // 255 + 16 for m in mats)
    hb = torch.empty(caps, dtype=torch.uint8).pin_memory()
    hs = torch.empty(n_exp, dtype=torch.uint8).pin_memory()
    dw = [torch.empty_like(d) for d in dev]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d2h = 0
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        for h, d in zip(hw, dw):
            d.copy_(h, non_blocking=True)
        enc = ops.encode_tensors(dw, args.chunks, args.attempts)
        bo = so = 0
        d2h = 0
        for blocks, _, sm in enc:
            for blk in blocks:
                hb[bo:bo + blk.numel()].copy_(blk, non_blocking=True)
                bo += blk.numel()
            hs[so:so + sm.numel()].copy_(sm, non_blocking=True)
            so += sm.numel()
        d2h = bo + so
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    threads = os.cpu_count() or 1
    cpu = None if args.no_cpu_baseline else cpu_encode_baseline(args, mats, threads)
    hbm, _, src = peaks()
    alg = n_exp + out_bytes                              # exponent bytes read, block bytes written
    line = {"metric": ENCODE_METRIC, "value": n_exp / (ms * 1e-3) / 1e9, "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic (seeded N(0,0.02) BF16 weights)", "config": encode_config(args),
            "attempts": args.attempts, "ratio": out_bytes / n_exp,
            "e2e": {"value": n_exp / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": 2 * n_exp,
                    "d2h_bytes_per_step": d2h},
            "roofline": {"bound": "hbm", "kernel": "chain+match+plan+scan+write (LZ4 encode)",
                         "achieved": alg / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": alg / (ms * 1e-3) / 1e9 / hbm, "peak_source": src, "traffic": None,
                         "note": "the match search is bound by instruction issue in shared memory, not by HBM"},
            "gpu_launches": 5 * args.steps, "clocks": clk.summary()}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def run_encode_reference(args):
    """The reference's offload compression on the host cores: liblz4
    LZ4_compress_HC per exponent chunk on every thread (oracle bindings; no
    code of this repository's library)."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from zmoe import synthetic as syn
    mats = [t for e in syn.expert_weights(syn.QWEN, 1)[0] for t in e][:args.matrices]
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_encode_baseline(args, mats[:1], threads)
    vals = [cpu_encode_baseline(args, mats, threads) for _ in range(args.steps)]
    v = statistics.median(x["value"] for x in vals)
    cb = dict(vals[0], value=v)
    n = min(8, len(mats)) * 1408 * 2048
    line = {"impl": "reference", "metric": ENCODE_METRIC, "value": v, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": n / (v * 1e9) * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic (seeded N(0,0.02) BF16 weights)", "config": encode_config(args),
            "cpu_baseline": cb, "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference" and args.config == "encode":
        run_encode_reference(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.config == "encode":
        run_encode(args)
    elif args.config == "decode-sweep":
        run_decode_sweep(args)
    elif args.config == "switch":
        run_switch(args)
    elif args.config == "deepseek-stack":
        run_deepseek_stack(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
