"""Benchmark of the sm_100a attention path (one JSON line on rank 0).

Default workload: BASELINE config 3 -- batched ragged GQA decode, Llama-3-8B
attention shape (32 q / 8 kv heads, head_dim 128, 32 layers), 64 sequences
with seeded context lengths in [1024, 8192], fp16 KV cache.  One step = one
decode step of attention: 32 per-layer launches over all sequences, as the
engine calls it layer by layer.  At N GPUs the 64 sequences are sharded by
sequence (strong scaling, no collective in the data path); value = the job's
tokens/s.  The same line carries config 4 (131072-key decode, split-KV over
the N GPUs with the partial exchange) as its long_decode sub-object.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


# roofline.traffic: DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum)
# from one ncu capture of exactly the launch the bench times (the commands and the
# rest of those captures are summarised under profiles/).  Workloads without such a
# capture report null.
# dram__bytes_read.sum + dram__bytes_write.sum of one launch of each workload's dominant kernel, from the ncu
# captures summarised under profiles/ (same workloads; --layers-reduced steps have the same per-launch bytes)
NCU_TRAFFIC = {"decode": 1225510144, "prefill": 25232128, "gated_prefill": 168607744, "gated_decode": 274070272,
               "long_decode": 541052160, "gdn_inputs": 225114112, "rope_store": 1590784,
               "gdn_decode": 78914048, "gdn_prefill_state": 257715456, "fused_decode": 1226680832,
               "gemv_q4k_gate_up": 66095388}


class ClockSampler:
    """SM clock / throttle-reason sampling during the timed region: NVML every
    5 ms in a thread (read-only queries), nvidia-smi every 200 ms if NVML is
    missing.  Only samples taken while the region runs are kept; a region
    shorter than the poll period gets one sample taken as it ends."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None
        self.nvml = None
        self.samples: list[tuple[float, float, float, set]] = []
        self.running = False
        self.t_begin = 0.0

    def begin(self):
        """Marks the start of the timed region (NVML samples before it are dropped)."""
        self.t_begin = time.perf_counter()

    def start(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = (pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu))
        except Exception:  # noqa: BLE001 -- no NVML: fall back to nvidia-smi
            self.nvml = None
        self.running = True
        if self.nvml is not None:
            self.thread = threading.Thread(target=self._poll_nvml, daemon=True)
            self.thread.start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _sample_nvml(self):
        nv, h = self.nvml
        bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
        try:
            sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
            smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            self.samples.append((time.perf_counter(), float(sm), float(smax),
                                 {n for n, b in bits.items() if r & b}))
        except Exception:  # noqa: BLE001
            pass

    def _poll_nvml(self):
        while self.running:
            self._sample_nvml()
            time.sleep(0.005)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        self.running = False
        if self.nvml is not None:
            if self.thread:
                self.thread.join(timeout=2)
            source = "nvml 5 ms"
            if not any(x[0] >= self.t_begin for x in self.samples):
                self._sample_nvml()   # region shorter than the poll period: sample as it ends
                source = "nvml, one sample as the region ended (region < 5 ms)"
            kept = [x for x in self.samples if x[0] >= self.t_begin]
            sm = [x[1] for x in kept]
            smax = [x[2] for x in kept]
            reasons = set().union(*[x[3] for x in kept]) if kept else set()
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                    "reasons": sorted(reasons), "samples": len(sm), "source": source}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(self.NAMES, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi 200 ms"}


# --------------------------------------------------------------- CPU side

class CpuReference:
    """The reference's CPU attention for config 3: oracle/_ref (the
    reference's matvec.c/platform.c under the restated engine.c:1074-1096
    loop, OpenMP over query heads, every host core), or the port if _ref is
    absent.

    A step is a bounded sample of the workload, timed whole: n_sample of the
    64 sequences -- every (64/n_sample)-th by context length, so their mean
    context is the config's -- through all 32 layers, one engine attention
    call per (layer, sequence).  The K/V/q of fix_layers distinct layers are
    generated (the same seeded bytes as the GPU arm) and cycled over the 32
    layers: each layer's sample is ~150 MB, and consecutive calls alternate
    between layers, so the working set (~600 MB) stays far beyond any L3."""

    def __init__(self, cfg, n_sample: int = 8, fix_layers: int = 4):
        sys.path.insert(0, str(ROOT / "tests"))
        import oracle

        self.oracle = oracle
        self.kind = "reference" if oracle.has_ref() else "port"
        self.lib = oracle.load("ref" if self.kind == "reference" else "port")
        # every host core (torchrun exports OMP_NUM_THREADS=1 to its ranks)
        self.lib.orc_set_threads(len(os.sched_getaffinity(0)))
        self.cores = int(self.lib.orc_max_threads())
        self.cfg = cfg
        ctx = cfg.ctx()
        order = sorted(range(cfg.n_seqs), key=lambda s: (ctx[s], s))
        stride = cfg.n_seqs // n_sample
        self.seqs = [order[i * stride + stride // 2] for i in range(n_sample)]
        self.keys = sum(ctx[s] for s in self.seqs)
        self.fx = [[oracle.decode_fixture(cfg, layer, s, lib=self.lib) for s in self.seqs]
                   for layer in range(fix_layers)]

    def time_step(self) -> float:
        """Seconds for one sample step: every layer of every sampled sequence."""
        c = self.cfg
        t0 = time.perf_counter()
        for layer in range(c.layers):
            for f in self.fx[layer % len(self.fx)]:
                self.oracle.attn_decode(f["q"], f["k"], f["v"], f["pos"], c.n_heads, c.n_kv_heads, c.head_dim,
                                        c.kv_dim, lib=self.lib)
        return time.perf_counter() - t0

    def describe(self, n_steps: int, seconds: float) -> str:
        c = self.cfg
        return (f"{len(self.seqs)} of the {c.n_seqs} sequences (every {c.n_seqs // len(self.seqs)}th by context "
                f"length: {self.keys} keys per layer, mean {self.keys / len(self.seqs):.0f} against the config's "
                f"{sum(c.ctx()) / c.n_seqs:.0f}) x all {c.layers} layers per step; {n_steps} steps timed "
                f"({seconds:.1f} s)")

    def rate(self, budget_s: float) -> dict:
        times = []
        while not times or (sum(times) < budget_s and len(times) < 8):
            times.append(self.time_step())
        step_s = statistics.median(times)
        return {"value": round(len(self.seqs) / step_s, 4), "unit": "tok/s", "cores": self.cores,
                "kind": self.kind, "sample": self.describe(len(times), sum(times))}


def config3_dict(cfg, world: int, n_layers: int, n_seqs: int, profile: bool = False) -> dict:
    """The config of the config-3 line: the same keys and values for the GPU arm and for the reference arm
    launched at the same N."""
    keys = sum(cfg.ctx_of(s) for s in range(n_seqs))
    return {
        "workload": cfg.name + ("" if not profile else f"-profile-{n_seqs}seq-{n_layers}layer"),
        "n_heads": cfg.n_heads, "n_kv_heads": cfg.n_kv_heads, "head_dim": cfg.head_dim,
        "layers": n_layers, "n_seqs": n_seqs, "ctx_range": [cfg.ctx_lo, cfg.ctx_hi],
        "total_keys_per_layer": keys, "kv_bytes_per_step": keys * cfg.kv_dim * 2 * 2 * n_layers,
        "parallelism": (f"the {n_seqs} sequences sharded by sequence over {world} GPU(s), longest-first by "
                        "context length; no collective"),
        "l2": "inputs larger than L2 (KV per GPU >> 126 MB)",
    }


# --------------------------------------------------------------- GPU side

def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from yllm_b200 import attn, dist as ydist, fixtures
    from yllm_b200.configs import CFG3 as cfg

    rank, world, local = ydist.init("nccl" if args.gpus > 1 else "gloo")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # --seqs / --layers shrink the workload for profiler captures only; the
    # default (and every reported number) is the full config.
    n_layers = args.layers or cfg.layers
    # Strong scaling (the config as stated): the config's 64 sequences are dealt to the ranks
    # longest-first by context length, so each GPU holds about 1/N of the keys; no data-path
    # collective.  --weak instead gives every rank a whole batch of the config's size.
    n_per_rank = args.seqs or cfg.n_seqs
    n_total = n_per_rank * world if args.weak else n_per_rank
    ctx_all = [cfg.ctx_of(s) for s in range(n_total)]
    seqs = ydist.shard_by_length(ctx_all, world)[rank]
    log(f"[rank {rank}] {len(seqs)} seqs, {sum(ctx_all[s] for s in seqs)} keys/layer, {n_layers} layers")

    d = fixtures.decode_inputs(cfg, layers=list(range(n_layers)), seqs=seqs, device=dev)
    torch.cuda.synchronize()
    # every sequence's KV lives in one pool: the pooled plan streams it with tensor copies
    plan = attn.DecodePlan.build([c - 1 for c in d.ctx], cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.kv_dim,
                                 device=dev, pool=(d.kv_pool.data_ptr(), d.kv_pool.numel() * 2))
    items = [attn.make_items([(d.q[l, i], d.out[l, i], d.k_ptr(l, i), d.v_ptr(l, i), None, d.ctx[i] - 1)
                              for i in range(len(seqs))], device=dev) for l in range(n_layers)]
    stream = torch.cuda.current_stream()

    def step():
        for l in range(n_layers):
            plan.run(items[l], stream)

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident timing ----
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps * n_layers)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    clocks.begin()
    t0.record(stream)
    k = 0
    for _ in range(args.steps):
        for l in range(n_layers):
            ev[k][0].record(stream)
            plan.run(items[l], stream)
            ev[k][1].record(stream)
            k += 1
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier()
    elapsed_ms = t0.elapsed_time(t1)
    launch_ms = sum(a.elapsed_time(b) for a, b in ev) / len(ev)
    t = torch.tensor([elapsed_ms, launch_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t[0].item())
    ms_per_step = elapsed_ms / args.steps
    value = n_total / (ms_per_step / 1e3)

    # ---- end to end: pinned host q in, host out back, every step ----
    # The copies run on streams of their own, one event per layer: layer l's q lands while the layers before it
    # compute, and its output goes back while the layers after it compute.  A step starts its copies only after
    # the previous step has ended, and ends when its last layer's output is on the host.
    n_q = d.q.numel()
    q_host = torch.empty(n_q, dtype=torch.float32, pin_memory=True)
    q_host.copy_(d.q.reshape(-1).cpu())
    out_host = torch.empty(n_q, dtype=torch.float32, pin_memory=True)
    q_host_l, out_host_l = q_host.view(n_layers, -1), out_host.view(n_layers, -1)
    q_dev_l, out_dev_l = d.q.view(n_layers, -1), d.out.view(n_layers, -1)
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(n_layers)]
    ev_done = [torch.cuda.Event() for _ in range(n_layers)]
    # the same timing-event pair around every launch as the device-resident loop above carries, so that the two
    # numbers differ by the copies only
    ev_l = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_layers)]

    def e2e_step():
        s_in.wait_stream(stream)
        with torch.cuda.stream(s_in):
            for l in range(n_layers):
                q_dev_l[l].copy_(q_host_l[l], non_blocking=True)
                ev_in[l].record(s_in)
        for l in range(n_layers):
            stream.wait_event(ev_in[l])
            ev_l[l][0].record(stream)
            plan.run(items[l], stream)
            ev_l[l][1].record(stream)
            ev_done[l].record(stream)
        with torch.cuda.stream(s_out):
            for l in range(n_layers):
                s_out.wait_event(ev_done[l])
                out_host_l[l].copy_(out_dev_l[l], non_blocking=True)
        stream.wait_stream(s_out)

    e2e_value = None
    if not args.no_e2e:
        for _ in range(max(1, args.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        te = torch.tensor([e0.elapsed_time(e1)], device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_value = n_total / (float(te.item()) / args.steps / 1e3)
    h2d = torch.tensor([n_q * 4], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(h2d)   # every rank's q bytes (the out bytes are the same)
    io_bytes = int(h2d.item())

    # ---- roofline of the decode kernel (per launch = one layer of this rank's seqs; slowest rank) ----
    bytes_per_launch = sum(d.ctx) * cfg.kv_dim * 2 * 2 + len(seqs) * cfg.n_heads * cfg.head_dim * 4 * 2
    bt = torch.tensor([bytes_per_launch / (launch_ms / 1e3)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(bt, op=dist.ReduceOp.MIN)
    achieved = float(bt.item()) / 1e9
    peaks, peak_src = load_peaks()
    st = attn.device_status()
    if st != 0:
        raise RuntimeError(f"device status {st}: a kernel gave up waiting")
    del d, plan, items
    torch.cuda.empty_cache()

    # ---- config 4 in the same run: the one cross-GPU exchange (split-KV over the ranks) ----
    long = None if args.no_long else _long_decode(args, rank, world, local, dist, sub=True)

    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1 and not (args.seqs or args.layers):
            cpu = CpuReference(cfg).rate(args.cpu_budget)
        line = {
            "metric": "attn decode tok/s (batched ragged GQA decode, all layers)",
            "value": round(value, 2),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True,
            "scaling": "weak" if args.weak else "strong",
            "vs_baseline": None,
            "dtype": "f32 math, fp16 KV",
            "data": "synthetic (seeded splitmix64 + Box-Muller, N(0,1) fp16 KV cache)",
            "config": config3_dict(cfg, world, n_layers, n_total, profile=bool(args.seqs or args.layers)),
            "e2e": None if e2e_value is None else {
                "value": round(e2e_value, 2), "unit": "tok/s",
                "h2d_bytes_per_step": io_bytes, "d2h_bytes_per_step": io_bytes,
                "path": ("plan.run per layer; each layer's q copied in from pinned host memory and its output copied "
                         "back on copy streams, overlapped with the other layers' kernels (one event per layer)")},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "traffic": None if (args.seqs or args.layers or world > 1) else NCU_TRAFFIC["decode"],
                         "kernel": "k_decode<128,4,TM> (pooled tensor copies)",
                         "peak_source": peak_src,
                         "bytes_per_launch": bytes_per_launch, "launch_ms": round(launch_ms, 5),
                         "note": "per GPU: the slowest rank's bytes per launch / its mean launch time"},
            "gpu_launches": args.steps * n_layers,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                       "samples": clk["samples"], "source": clk.get("source")},
        }
        if world > 1:
            line["config"]["seqs_per_gpu"] = [len(x) for x in ydist.shard_by_length(ctx_all, world)]
        if long is not None:
            line["long_decode"] = long
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_decode_small(args) -> None:
    """BASELINE config 1 (Qwen2.5-0.5B shape: one sequence, ctx 512, 24 layers)
    and config 5c decode (qwen3.5 gated full attention, 32 sequences at ctx
    4096, one layer).  A step is every layer of the batch through the batched
    plan, replayed as one CUDA graph (the launches are shorter than the Python
    call that makes them); L2 is scrubbed between timed steps when the step's
    KV fits in it.  Weak scaling: each rank serves its own batch."""
    import torch
    import torch.distributed as dist

    from yllm_b200 import attn, dist as ydist, fixtures
    from yllm_b200.configs import CFG1, CFG5_GATED_DECODE

    cfg = CFG1 if args.workload == "config1_decode" else CFG5_GATED_DECODE
    rank, world, local = ydist.init("nccl" if args.gpus > 1 else "gloo")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    seqs = list(range(rank * cfg.n_seqs, (rank + 1) * cfg.n_seqs))
    d = fixtures.decode_inputs(cfg, seqs=seqs, device=dev)
    torch.cuda.synchronize()
    plan = attn.DecodePlan.build([c - 1 for c in d.ctx], cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.kv_dim,
                                 device=dev, pool=(d.kv_pool.data_ptr(), d.kv_pool.numel() * 2))
    items = [attn.make_items([(d.q[l, i], d.out[l, i], d.k_ptr(l, i), d.v_ptr(l, i),
                               d.gate[l, i] if d.gate is not None else None, d.ctx[i] - 1)
                              for i in range(len(seqs))], device=dev) for l in range(d.n_layers)]

    def step():
        for l in range(d.n_layers):
            plan.run(items[l])

    kv_bytes = sum(d.ctx) * cfg.kv_dim * 2 * 2 * d.n_layers
    flush = kv_bytes < (512 << 20)
    ms, per_call, clk = _timed(step, args, stream, world, dist, local, graph=True, flush_l2=flush)
    qo_bytes = d.n_layers * len(seqs) * cfg.n_heads * cfg.head_dim * 4 * (3 if cfg.gated else 2)
    step_bytes = kv_bytes + qo_bytes
    peaks, src = load_peaks()
    ach = step_bytes / (per_call / 1e3) / 1e9
    G = -(-cfg.n_heads // cfg.n_kv_heads)
    roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(ach / peaks["hbm_gbs"], 4), "traffic": NCU_TRAFFIC["gated_decode"] if cfg.gated else None,
            "kernel": f"k_decode<{cfg.head_dim},{G},TM> (pooled tensor copies)",
            "peak_source": src, "bytes_per_step": step_bytes,
            "note": f"{d.n_layers} launches per step in one graph; achieved = step bytes / step device time"}
    e2e = None
    if not args.no_e2e:
        n_q = d.q.numel()
        qh = torch.empty(n_q, dtype=torch.float32, pin_memory=True)
        qh.copy_(d.q.reshape(-1).cpu())
        oh = torch.empty(n_q, dtype=torch.float32, pin_memory=True)

        def e2e_step():
            d.q.view(-1).copy_(qh, non_blocking=True)
            step()
            oh.copy_(d.out.view(-1), non_blocking=True)

        ems, _, _ = _timed(e2e_step, args, stream, world, dist, local)
        e2e = {"value": round(len(seqs) * world / (ems / 1e3), 2), "unit": "tok/s",
               "h2d_bytes_per_step": n_q * 4 * world, "d2h_bytes_per_step": n_q * 4 * world,
               "path": "DecodePlan.run per layer per step (no graph), pinned host q in, out back"}
    st = attn.device_status()
    if st != 0:
        raise RuntimeError(f"device status {st}: a kernel gave up waiting")
    if rank == 0:
        metric = ("attn decode tok/s (Qwen2.5-0.5B shape, 24 layers, ctx 512)" if cfg is CFG1
                  else "gated attn decode tok/s (qwen3.5 shape, batch 32, ctx 4096)")
        line = _line(args, world, metric, len(seqs) * world / (ms / 1e3), "tok/s", ms,
                     {"workload": cfg.name, "n_heads": cfg.n_heads, "n_kv_heads": cfg.n_kv_heads,
                      "head_dim": cfg.head_dim, "layers": d.n_layers, "n_seqs": len(seqs) * world,
                      "ctx": cfg.ctx_hi, "gated": cfg.gated, "kv_bytes_per_step": kv_bytes * world,
                      "parallelism": f"data-parallel x{world}: a batch per GPU, no collective",
                      "launch": "CUDA graph replay of the step (device-timed value)",
                      "l2": ("L2 scrubbed between timed steps outside the step's events (256 MB write, then "
                             "256 MB read of another buffer, so no dirty scrub lines remain)" if flush
                             else "KV per step larger than L2")},
                     roof, args.steps * d.n_layers, clk, e2e, scaling="weak")
        line["dtype"] = "f32 math, fp16 KV" + (", bf16-valued q and gate" if cfg.gated else "")
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args) -> None:
    """The reference's own CPU attention for the config-3 workload (rank 0 only;
    the other ranks exit without work).  Each step is a bounded sample of the
    workload (CpuReference), timed whole: value = the sample's tokens / the
    median step time, so ms_per_step x steps is the time actually spent."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return
    from yllm_b200.configs import CFG3 as cfg

    ref = CpuReference(cfg)
    times = []
    for i in range(args.warmup + args.steps):
        t = ref.time_step()
        if i >= args.warmup:
            times.append(t)
    step_s = statistics.median(times)
    value = len(ref.seqs) / step_s
    sample = ref.describe(len(times), sum(times))
    line = {
        "impl": "reference",
        "metric": "attn decode tok/s (batched ragged GQA decode, all layers)",
        "value": round(value, 4),
        "unit": "tok/s",
        "n_gpus": world,
        "runs_on": (f"host cores of rank 0 ({ref.cores} threads; OpenMP over query heads, as the engine); no GPU "
                    "work"),
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_s * 1e3, 2),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32 math, fp16 KV",
        "data": "synthetic (seeded splitmix64 + Box-Muller, N(0,1) fp16 KV cache)",
        "config": config3_dict(cfg, world, cfg.layers, cfg.n_seqs),
        "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": ref.cores, "kind": ref.kind,
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------- other workloads
#
# `--workload` selects one of the other BASELINE configs.  Each prints one line
# of the same shape; the driver's default (no flag) is config 3 above.

def _timed(fn, args, stream, world, dist, local, graph=False, flush_l2=False):
    """Warm-up, then args.steps calls of fn between CUDA events on the stream
    (one event pair per call), clocks sampled meanwhile; max over ranks.

    graph=True captures one call of fn (which must launch on the current
    stream) into a CUDA graph and times its replays: the device-resident number
    for kernels shorter than the Python call that launches them.

    flush_l2=True scrubs L2 between timed calls, outside each call's event
    pair, for inputs that fit in L2: it writes a 256 MB buffer (twice the L2),
    then reads another 256 MB buffer, so the call starts with none of its
    inputs in L2 and no dirty lines of the scrub left to write back during
    it.  The step time is then the sum of the per-call device times."""
    import torch

    scrub = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local}") if flush_l2 else None
    scrub_rd = torch.ones(64 << 20, dtype=torch.float32, device=f"cuda:{local}") if flush_l2 else None

    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        torch.cuda.synchronize()
        fn = g.replay
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.begin()
    t0.record(stream)
    for a, b in ev:
        if scrub is not None:
            scrub.fill_(1)
            scrub_rd.sum()
        a.record(stream)
        fn()
        b.record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    per_call = sum(a.elapsed_time(b) for a, b in ev) / len(ev)
    total = torch.tensor([per_call * args.steps if scrub is not None else t0.elapsed_time(t1)],
                         device=f"cuda:{local}")
    if world > 1:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
    return float(total.item()) / args.steps, per_call, clk


def _line(args, world, metric, value, unit, ms, cfg_dict, roofline, launches, clk, e2e=None, cpu=None,
          higher=True, scaling="strong"):
    line = {"metric": metric, "value": round(value, 4), "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": higher, "scaling": scaling,
            "vs_baseline": None, "dtype": "f32 math, fp16 Q/K/V/P hi+lo", "data": "synthetic (seeded)",
            "config": cfg_dict, "e2e": e2e, "roofline": roofline, "gpu_launches": launches,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                       "samples": clk["samples"], "source": clk.get("source")}}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


def run_prefill(args, gated: bool) -> None:
    import torch
    import torch.distributed as dist

    from yllm_b200 import attn, dist as ydist, fixtures
    from yllm_b200.configs import CFG2, CFG5_GATED_PREFILL

    cfg = CFG5_GATED_PREFILL if gated else CFG2
    rank, world, local = ydist.init("nccl" if args.gpus > 1 else "gloo")
    torch.cuda.set_device(local)
    stream = torch.cuda.current_stream()
    S, H, hd = cfg.seq_len, cfg.n_heads, cfg.head_dim
    p = fixtures.prefill_inputs(cfg)
    # Weak scaling: every rank prefills its own S-token prompt (prompts are
    # independent units; no collective).
    r0, r1 = 0, S
    B = r1 - r0
    qs = H * hd

    # The config's q is fp16 by construction (drawn in fp16), so the step uses the q hi-only kernel
    # (YATTN_PREFILL_Q_F16, which checks the claim on the device).  The default kernel -- q split into
    # hi + lo, what the engine's fp32 projections need -- is timed beside it on the same inputs.
    def step(q_f16=True):
        attn.attn_prefill(p.out[r0:r1], p.q[r0:r1], p.k, p.v, r0, B, H, cfg.n_kv_heads, hd, cfg.kv_dim, qs,
                          gate=p.gate[r0:r1] if p.gate is not None else None, q_f16=q_f16)

    ms, per_call, clk = _timed(step, args, stream, world, dist, local, graph=True, flush_l2=True)
    ms_lo, per_call_lo, _ = _timed(lambda: step(False), args, stream, world, dist, local, graph=True, flush_l2=True)
    flops = cfg.causal_flops() * world
    my_flops = cfg.causal_flops()
    e2e = None
    if not args.no_e2e:
        qh = torch.empty(B * qs, dtype=torch.float32, pin_memory=True)
        qh.copy_(p.q[r0:r1].reshape(-1).cpu())
        kh = torch.empty(r1 * cfg.kv_dim, dtype=torch.uint16, pin_memory=True)
        kh.copy_(p.k[:r1].reshape(-1).cpu())
        vh = torch.empty_like(kh)
        vh.copy_(p.v[:r1].reshape(-1).cpu())
        oh = torch.empty(B * qs, dtype=torch.float32, pin_memory=True)

        def e2e_step():
            p.q[r0:r1].view(-1).copy_(qh, non_blocking=True)
            p.k[:r1].view(-1).copy_(kh, non_blocking=True)
            p.v[:r1].view(-1).copy_(vh, non_blocking=True)
            step()
            oh.copy_(p.out[r0:r1].view(-1), non_blocking=True)

        ems, _, _ = _timed(e2e_step, args, stream, world, dist, local)
        nb = B * qs * 4
        e2e = {"value": round(flops / (ems / 1e3) / 1e12, 3), "unit": "TFLOP/s",
               "h2d_bytes_per_step": int((nb + 2 * r1 * cfg.kv_dim * 2) * world), "d2h_bytes_per_step": int(nb * world),
               "path": "attn_prefill API call per step, no graph"}
    peaks, src = load_peaks()
    achieved = my_flops / (per_call / 1e3) / 1e12
    roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
            "frac": round(achieved / peaks["bf16_tflops"], 4),
            "traffic": NCU_TRAFFIC["gated_prefill" if gated else "prefill"],
            "kernel": f"k_prefill<{hd},QLO=false> (q hi only)", "peak_source": src + " (dense bf16 burst)"}
    fp32_q = {"value": round(flops / (ms_lo / 1e3) / 1e12, 4), "unit": "TFLOP/s", "ms_per_step": round(ms_lo, 5),
              "frac": round(my_flops / (per_call_lo / 1e3) / 1e12 / peaks["bf16_tflops"], 4),
              "kernel": f"k_prefill<{hd},QLO=true> (q hi + lo: the default, and the drop-in's, for fp32 q)"}
    st = attn.device_status()
    if st != 0:
        raise RuntimeError(f"device status {st}")
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_prefill_rate(cfg, args.cpu_budget)
    if rank == 0:
        print(json.dumps(_line(args, world, "prefill attn TFLOP/s (causal, counted causal FLOPs)",
                               flops / (ms / 1e3) / 1e12, "TFLOP/s", ms,
                               {"workload": cfg.name, "seq_len": S, "n_heads": H, "n_kv_heads": cfg.n_kv_heads,
                                "head_dim": hd, "gated": gated, "flops": flops,
                                "parallelism": f"data-parallel x{world}: one {S}-token prompt per GPU, no collective",
                                "launch": "CUDA graph replay of the step (device-timed value)",
                                "q": "fp16-valued (the config's q/k/v are drawn in fp16): YATTN_PREFILL_Q_F16",
                                "l2": ("L2 scrubbed between timed steps outside the step's events (256 MB write, "
                                       "then 256 MB read of another buffer)")},
                               roof, args.steps, clk, e2e, cpu, scaling="weak") | {"fp32_q_kernel": fp32_q}),
              flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def cpu_prefill_rate(cfg, budget_s: float) -> dict:
    """Reference CPU prefill (oracle/_ref) on the last 128 query rows, scaled to
    the whole causal prefill by FLOP count."""
    sys.path.insert(0, str(ROOT / "tests"))
    import oracle

    kind = "reference" if oracle.has_ref() else "port"
    lib = oracle.load("ref" if kind == "reference" else "port")
    f = oracle.prefill_fixture(cfg, lib=lib)
    S, H, hd, B = cfg.seq_len, cfg.n_heads, cfg.head_dim, 128
    times = []
    while not times or (sum(times) < budget_s and len(times) < 5):
        t0 = time.perf_counter()
        oracle.attn_prefill(f["q"][S - B:], f["k"], f["v"], S - B, B, H, cfg.n_kv_heads, hd, cfg.kv_dim, H * hd,
                            gate=None if f["gate"] is None else f["gate"][S - B:], lib=lib)
        times.append(time.perf_counter() - t0)
    sample_flops = 4.0 * hd * H * sum(r + 1 for r in range(S - B, S))
    rate = sample_flops / statistics.median(times)
    return {"value": round(rate / 1e12, 6), "unit": "TFLOP/s", "cores": int(lib.orc_max_threads()), "kind": kind,
            "sample": f"last {B} rows of the {S}-token prefill (keys 0..{S - 1}), {len(times)} runs; "
                      f"rate = sample FLOPs / time"}


def run_gdn(args, decode: bool) -> None:
    import torch
    import torch.distributed as dist

    from yllm_b200 import attn, dist as ydist, fixtures
    from yllm_b200.configs import CFG5_GDN as c

    rank, world, local = ydist.init("nccl" if args.gpus > 1 else "gloo")
    torch.cuda.set_device(local)
    stream = torch.cuda.current_stream()
    D, NK, NV = c.head_dim, c.num_k_heads, c.n_v_heads
    if decode:
        s0, s1 = 0, c.batch      # weak scaling: every rank serves its own batch
        n = s1 - s0
        g = fixtures.gdn_inputs(c, c.batch, 1, seeded_state=True)
        S, q, k, v, o = g.S[s0:s1], g.q[s0:s1], g.k[s0:s1], g.v[s0:s1], g.out[s0:s1]
        gt, bt, z = g.gate[s0:s1], g.beta[s0:s1], g.z[s0:s1]

        def step():
            if n:
                attn.gdn_decode(S, o, q, k, v, gt, bt, n, NK, D, NV, D, norm_w=g.norm_w, z=z, eps=c.eps)
        ms, per_call, clk = _timed(step, args, stream, world, dist, local, graph=True)
        nbytes = c.batch * world * NV * D * D * 4 * 2
        mine = n * NV * D * D * 4 * 2
        peaks, src = load_peaks()
        ach = mine / (per_call / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(ach / peaks["hbm_gbs"], 4), "traffic": NCU_TRAFFIC["gdn_decode"],
                "traffic_note": "below the state bytes: part of the 134 MB state stays in L2 across launches",
                "kernel": "k_gdn_decode",
                "peak_source": src}
        if rank == 0:
            print(json.dumps(_line(args, world, "GDN batch-32 decode tok/s (state read+write)",
                                   c.batch * world / (ms / 1e3), "tok/s", ms,
                                   {"workload": c.name + "-decode-b32", "n_v_heads": NV, "num_k_heads": NK,
                                    "head_dim": D, "batch": c.batch * world, "state_bytes_per_step": nbytes,
                                    "parallelism": f"data-parallel x{world}: a batch of {c.batch} per GPU",
                                    "launch": "CUDA graph replay of the step", "l2": "state 134 MB per GPU > L2"},
                                   roof, args.steps, clk, scaling="weak")), flush=True)
    else:
        T = c.tokens
        g = fixtures.gdn_inputs(c, 1, T, seeded_state=False)

        def step():
            attn.gdn_prefill(g.S, g.out, g.q, g.k, g.v, g.gate, g.beta, 1, T, NK, D, NV, D, norm_w=g.norm_w,
                             z=g.z, eps=c.eps)
        ms, per_call, clk = _timed(step, args, stream, world, dist, local, graph=True)
        flops = T * NV * 7.0 * D * D
        peaks, src = load_peaks()
        ach = flops / (per_call / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": round(ach, 2), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": round(ach / peaks["bf16_tflops"], 4), "traffic": NCU_TRAFFIC["gdn_prefill_state"],
                "traffic_note": "k_gdn_chunk_state, the larger of the step's two kernels", "kernel": "k_gdn_prefill",
                "peak_source": src + " (dense bf16 burst)"}
        if rank == 0:
            print(json.dumps(_line(args, world, "GDN 4096-token prefill TFLOP/s (recurrent-equivalent FLOPs)",
                                   flops * world / (ms / 1e3) / 1e12, "TFLOP/s", ms,
                                   {"workload": c.name + "-prefill-4096", "n_v_heads": NV, "num_k_heads": NK,
                                    "head_dim": D, "tokens": T, "flops": flops * world,
                                    "parallelism": f"data-parallel x{world}: one sequence per GPU",
                                    "launch": "CUDA graph replay of the step"},
                                   roof, args.steps, clk, scaling="weak")), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _long_decode(args, rank, world, local, dist, sub=False):
    """Config 4: one 131072-key decode, the key range split over the ranks.
    Each rank reduces its range to (m, l, o) partials; at N > 1 the partials are
    exchanged over NVLink (k_exchange_merge: pushed into every rank's area,
    merged on every GPU) or by an NCCL all-gather.  Returns the line's fields
    (rank 0) -- a sub-object of the config-3 line when sub is True."""
    import torch

    from yllm_b200 import attn, dist as ydist, fixtures
    from yllm_b200.configs import CFG4 as c

    stream = torch.cuda.current_stream()
    d = fixtures.decode_inputs(c)
    n = d.ctx[0]
    k0, k1 = ydist.split_range(n, world, rank)
    H, hd = c.n_heads, c.head_dim
    peer = world > 1 and args.exchange in ("peer", "peer2")
    fused = peer and args.exchange == "peer"
    ex = (ydist.PeerExchange if peer else ydist.PartialExchange)(H, hd, device=f"cuda:{local}")
    out = d.out[0, 0]
    kv, vv = d.k_view(0, 0), d.v_view(0, 0)

    def partial():
        attn.decode_partial(ex.ml, ex.o, d.q[0, 0], kv, vv, k0, k1, H, c.n_kv_heads, hd, c.kv_dim)

    def step():
        # launches on the current stream, so the step (NCCL included) can be graph-captured
        if world == 1:
            attn.attn_decode(out, d.q[0, 0], kv, vv, n - 1, H, c.n_kv_heads, hd, c.kv_dim)
        elif fused:   # two launches: the shard's split decode, then merge + exchange + merge in one kernel
            ex.decode(out, d.q[0, 0], kv, vv, k0, k1, c.n_kv_heads, c.kv_dim)
        else:         # the shard's partial decode, then the exchange (peer memory or NCCL) as its own call
            partial()
            ex.run(out)

    ms, per_call, clk = _timed(step, args, stream, world, dist, local, graph=True)
    # the split: the partial decode alone (graph-replayed), slowest rank
    split = None
    if world > 1:
        ms_p, _, _ = _timed(partial, args, stream, world, dist, local, graph=True)
        split = {"partial_decode_ms": round(ms_p, 5), "exchange_and_merge_ms": round(ms - ms_p, 5),
                 "note": "partial_decode_ms: this rank's shard reduced to one (m, l, o) per head on its GPU "
                         "(yattn_decode_partial); the rest of the step is the exchange"}
    e2e = None
    if not args.no_e2e:
        qh = torch.empty(H * hd, dtype=torch.float32, pin_memory=True)
        qh.copy_(d.q[0, 0].cpu())
        oh = torch.empty(H * hd, dtype=torch.float32, pin_memory=True)

        def e2e_step():
            d.q[0, 0].copy_(qh, non_blocking=True)
            step()
            oh.copy_(out, non_blocking=True)

        ems, _, _ = _timed(e2e_step, args, stream, world, dist, local)
        e2e = {"value": round(n * c.kv_dim * 4 / (ems / 1e3) / 1e9, 1), "unit": "GB/s",
               "h2d_bytes_per_step": H * hd * 4 * world, "d2h_bytes_per_step": H * hd * 4 * world,
               "path": "API calls per step (no graph), pinned host q in, out back"}
    torch.cuda.synchronize()
    st = attn.device_status()
    if st != 0:
        raise RuntimeError(f"device status {st}: a kernel gave up waiting")
    nbytes = n * c.kv_dim * 2 * 2
    peaks, src = load_peaks()
    ach = nbytes / (ms / 1e3) / 1e9
    roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"] * world, "unit": "GB/s",
            "frac": round(ach / (peaks["hbm_gbs"] * world), 4),
            "traffic": NCU_TRAFFIC["long_decode"] if world == 1 else None,
            "kernel": "k_decode<128,4,TM>" + ((" + k_merge_splits<EX> (split merge + exchange + merge)" if fused
                                               else " + k_merge_splits, then k_exchange_merge" if peer
                                               else " + NCCL all-gather + merge")
                                              if world > 1 else " + k_merge_splits"),
            "peak_source": src + f" x{world} GPUs"}
    cfg_d = {"workload": c.name, "ctx": n, "n_heads": H, "n_kv_heads": c.n_kv_heads, "head_dim": hd,
             "kv_bytes": nbytes,
             "parallelism": (f"split-KV x{world}, " + (
                 "(m,l,o) pushed into every GPU over NVLink + LSE merge, one kernel" if fused
                 else "(m,l,o) pushed into every GPU over NVLink + LSE merge, its own launch" if peer
                 else "NCCL all-gather of (m,l,o) + LSE merge")) if world > 1 else "one GPU",
             "launch": "CUDA graph replay of the step (partial decode, exchange, merge)",
             "l2": "KV 537 MB > L2"}
    if peer:
        ex.close()
    del d
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    if sub:
        return {"metric": "long-context decode GB/s (131072 keys, one layer)", "value": round(ach, 1),
                "unit": "GB/s", "ms_per_step": round(ms, 5), "scaling": "strong", "config": cfg_d,
                "roofline": roof, "split": split, "e2e": e2e,
                "clocks": {"sm_mhz": clk["sm_mhz"], "reasons": clk["reasons"], "samples": clk["samples"]}}
    line = _line(args, world, "long-context decode GB/s (131072 keys, one layer)", ach, "GB/s", ms, cfg_d, roof,
                 args.steps * (2 if world > 1 else 1), clk, e2e)
    if split:
        line["split"] = split
    return line


def run_long_decode(args) -> None:
    """Config 4 on its own line (see _long_decode)."""
    import torch
    import torch.distributed as dist

    from yllm_b200 import dist as ydist

    rank, world, local = ydist.init("nccl" if args.gpus > 1 else "gloo")
    torch.cuda.set_device(local)
    line = _long_decode(args, rank, world, local, dist)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_rope_store(args) -> None:
    """The decode step's RoPE + KV store (engine.c:1052-1072 per sequence and
    layer; cuda_fwd.c:136-147 launches three kernels per sequence) at config
    3's shape: every layer's q rotated in place and k/v rounded into the
    pooled cache at each sequence's newest position, one launch per layer for
    all 64 sequences.  Inputs fit in L2, so L2 is scrubbed between timed
    steps.  Weak scaling: each rank serves its own batch."""
    import ctypes as C

    import torch
    import torch.distributed as dist

    from yllm_b200 import attn, dist as ydist
    from yllm_b200.configs import CFG3 as c

    rank, world, local = ydist.init("nccl" if args.gpus > 1 else "gloo")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    L, n, H, KV, hd, kd = c.layers, c.n_seqs, c.n_heads, c.n_kv_heads, c.head_dim, c.kv_dim
    L = args.layers or L   # --layers shrinks the step for profiler captures only
    theta = 500000.0   # Llama-3 rope_theta
    ctx = c.ctx()
    offs = [sum(ctx[:i]) for i in range(n)]
    rows = sum(ctx)
    pool = torch.empty(2 * L * rows * kd, dtype=torch.int16, device=dev)   # [K layers | V layers][rows][kd]
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    q = torch.randn(L, n, H * hd, generator=g, device=dev)
    k = torch.randn(L, n, kd, generator=g, device=dev)
    v = torch.randn(L, n, kd, generator=g, device=dev)
    base = pool.data_ptr()
    items = [attn.make_rope_items([(q[l, i], k[l, i], v[l, i], base + 2 * (l * rows + offs[i]) * kd,
                                    base + 2 * ((L + l) * rows + offs[i]) * kd, ctx[i] - 1) for i in range(n)],
                                  device=dev) for l in range(L)]

    def step():
        for l in range(L):
            attn.rope_store_kv(items[l], n, H, KV, hd, kd, attn.ROPE_LLAMA, theta)

    ms, per_call, clk = _timed(step, args, stream, world, dist, local, graph=True, flush_l2=True)
    per_item = 2 * H * hd * 4 + 2 * kd * 4 + 2 * kd * 2     # q read + write, k and v read, k and v rows written
    step_bytes = L * n * per_item
    e2e = None
    if not args.no_e2e:
        hq = torch.empty(q.numel(), dtype=torch.float32, pin_memory=True)
        hk = torch.empty(k.numel(), dtype=torch.float32, pin_memory=True)
        hv = torch.empty(v.numel(), dtype=torch.float32, pin_memory=True)
        hq.copy_(q.reshape(-1).cpu())
        hk.copy_(k.reshape(-1).cpu())
        hv.copy_(v.reshape(-1).cpu())
        oq = torch.empty(q.numel(), dtype=torch.float32, pin_memory=True)

        def e2e_step():
            q.view(-1).copy_(hq, non_blocking=True)
            k.view(-1).copy_(hk, non_blocking=True)
            v.view(-1).copy_(hv, non_blocking=True)
            step()
            oq.copy_(q.view(-1), non_blocking=True)

        ems, _, _ = _timed(e2e_step, args, stream, world, dist, local)
        e2e = {"value": round(n * world / (ems / 1e3), 2), "unit": "tok/s",
               "h2d_bytes_per_step": (q.numel() + k.numel() + v.numel()) * 4 * world,
               "d2h_bytes_per_step": q.numel() * 4 * world,
               "path": "rope_store_kv per layer per step (no graph), pinned host q/k/v in, rotated q back"}
    st = attn.device_status()
    if st != 0:
        raise RuntimeError(f"device status {st}")
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        import numpy as np

        sys.path.insert(0, str(ROOT / "tests"))
        import oracle

        kind = "reference" if oracle.has_ref() else "port"
        lib = oracle.load("ref" if kind == "reference" else "port")
        qh, kh, vh = q[0].cpu().numpy().copy(), k[0].cpu().numpy().copy(), v[0].cpu().numpy().copy()
        kc = np.zeros(max(ctx) * kd, np.uint16)
        vc = np.zeros(max(ctx) * kd, np.uint16)
        times = []
        while not times or (sum(times) < min(args.cpu_budget, 5.0) and len(times) < 50):
            t0 = time.perf_counter()
            for i in range(n):
                lib.orc_rope_store(qh[i], kh[i], vh[i], kc, vc, H, KV, hd, kd, 0, hd, ctx[i] - 1, theta)
            times.append(time.perf_counter() - t0)
        step_s = statistics.median(times) * L
        cpu = {"value": round(n / step_s, 2), "unit": "tok/s", "cores": 1, "kind": kind,
               "sample": f"layer 0 of {n} seqs (engine.c:1052-1072 per sequence, one thread as in the engine), "
                         f"timed {len(times)}x, x{L} layers per step"}
    peaks, src = load_peaks()
    ach = step_bytes / (per_call / 1e3) / 1e9
    roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(ach / peaks["hbm_gbs"], 4), "traffic": NCU_TRAFFIC["rope_store"], "kernel": "k_rope_store",
            "peak_source": src, "bytes_per_step": step_bytes,
            "note": f"{L} launches of {per_item * n / 1e6:.2f} MB each per step in one graph: launch-latency "
                    "bound, the HBM fraction is small by construction"}
    if rank == 0:
        line = _line(args, world, "RoPE + KV store tok/s (Llama-3-8B shape, 64 sequences, 32 layers)",
                     n * world / (ms / 1e3), "tok/s", ms,
                     {"workload": c.name + "-rope-store" + (f"-profile-{L}-layers" if args.layers else ""), "n_heads": H, "n_kv_heads": KV, "head_dim": hd,
                      "layers": L, "n_seqs": n * world, "rope": "llama pairs, theta 500000",
                      "parallelism": f"data-parallel x{world}: a batch per GPU, no collective",
                      "launch": "CUDA graph replay of the step (one launch per layer)",
                      "l2": "L2 scrubbed between timed steps outside the step's events"},
                     roof, args.steps * L, clk, e2e, cpu=cpu, scaling="weak")
        line["dtype"] = "f32 math, fp16 KV rows (engine rounding)"
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_fused_decode(args) -> None:
    """Config 3's whole attention step with the decode step's RoPE + KV store
    (engine.c:1052-1096 per sequence and layer): per layer, the new token's k and
    v rotated / rounded into every sequence's cache row pos, q rotated, and the
    attention over keys 0..pos.  Timed two ways on the same inputs: one fused
    launch per layer (yattn_decode_run_pooled_rope), and two (yattn_rope_store_kv,
    then yattn_decode_run_pooled).  KV per GPU far above L2.  Weak scaling."""
    import torch
    import torch.distributed as dist

    from yllm_b200 import attn, dist as ydist, fixtures
    from yllm_b200.configs import CFG3 as cfg

    rank, world, local = ydist.init("nccl" if args.gpus > 1 else "gloo")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    n_layers = args.layers or cfg.layers
    seqs = list(range(args.seqs or cfg.n_seqs))
    H, KV, hd, kd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.kv_dim
    theta = 500000.0   # Llama-3 rope_theta
    d = fixtures.decode_inputs(cfg, layers=list(range(n_layers)), seqs=seqs, device=dev)
    n = len(seqs)
    g = torch.Generator(device=dev)
    g.manual_seed(77 + rank)
    kn = torch.randn(n_layers, n, kd, generator=g, device=dev)
    vn = torch.randn(n_layers, n, kd, generator=g, device=dev)
    q_raw = d.q.clone()   # the fused path reads q unrotated and leaves it so
    pool = (d.kv_pool.data_ptr(), d.kv_pool.numel() * 2)
    pos = [c - 1 for c in d.ctx]
    plan = attn.DecodePlan.build(pos, H, KV, hd, kd, device=dev, pool=pool)
    items = [attn.make_items([(q_raw[l, i], d.out[l, i], d.k_ptr(l, i), d.v_ptr(l, i), None, pos[i])
                              for i in range(n)], device=dev) for l in range(n_layers)]
    rows = [attn.make_new_rows([(kn[l, i], vn[l, i]) for i in range(n)], device=dev) for l in range(n_layers)]
    ritems = [attn.make_rope_items([(d.q[l, i], kn[l, i], vn[l, i], d.k_ptr(l, i), d.v_ptr(l, i), pos[i])
                                    for i in range(n)], device=dev) for l in range(n_layers)]
    items2 = [attn.make_items([(d.q[l, i], d.out[l, i], d.k_ptr(l, i), d.v_ptr(l, i), None, pos[i])
                               for i in range(n)], device=dev) for l in range(n_layers)]

    def fused():
        for l in range(n_layers):
            plan.run_rope(items[l], rows[l], attn.ROPE_LLAMA, theta)

    def two_launch():
        # the store rotates q in place, so repeated steps rotate an already rotated q: the same work
        for l in range(n_layers):
            attn.rope_store_kv(ritems[l], n, H, KV, hd, kd, attn.ROPE_LLAMA, theta)
            plan.run(items2[l])

    ms_f, _, clk = _timed(fused, args, stream, world, dist, local)
    ms_2, _, _ = _timed(two_launch, args, stream, world, dist, local)
    st = attn.device_status()
    if st != 0:
        raise RuntimeError(f"device status {st}")
    keys = sum(d.ctx)
    step_bytes = n_layers * (keys * kd * 2 * 2 + n * (H * hd * 4 * 2 + kd * 4 * 2))
    peaks, src = load_peaks()
    roof = {"bound": "hbm", "achieved": round(step_bytes / (ms_f / 1e3) / 1e9, 1), "peak": peaks["hbm_gbs"],
            "unit": "GB/s", "frac": round(step_bytes / (ms_f / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
            "traffic": None if (args.seqs or args.layers or world > 1) else NCU_TRAFFIC["fused_decode"],
            "kernel": "k_decode<128,4,TM,ROPE> (pooled tensor copies, RoPE + store fused)", "peak_source": src,
            "bytes_per_step": step_bytes}
    if rank == 0:
        line = _line(args, world, "attn decode tok/s with the RoPE + KV store (batched ragged GQA decode, all layers)",
                     n * world / (ms_f / 1e3), "tok/s", ms_f,
                     {"workload": cfg.name + "-rope-store-fused", "n_heads": H, "n_kv_heads": KV, "head_dim": hd,
                      "layers": n_layers, "n_seqs": n * world, "rope": "llama pairs, theta 500000",
                      "parallelism": f"data-parallel x{world}: a batch per GPU, no collective",
                      "launch": "one API call per layer per step (no graph)",
                      "l2": "inputs larger than L2 (KV per GPU >> 126 MB)"},
                     roof, args.steps * n_layers, clk, scaling="weak")
        line["two_launch"] = {"value": round(n * world / (ms_2 / 1e3), 2), "unit": "tok/s", "ms_per_step": round(ms_2, 4),
                              "path": "yattn_rope_store_kv, then yattn_decode_run_pooled, per layer"}
        line["dtype"] = "f32 math, fp16 KV (engine rounding of the new rows)"
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_gemv(args, fmt: str = "q4k") -> None:
    """The per-layer linear layers of a Llama-3-8B decode step (cuda_fwd.c:94-168
    brackets attention with these GEMVs): per layer q, k, v, o (4096/1024 x
    4096), gate and up (14336 x 4096) and down (4096 x 14336), 218 M weights:
    123 MB as Q4_K (fmt "q4k"), 436 MB as fp16 (fmt "f16"); 32 layers, each
    with its own weights (far above L2).  Q4_K runs q/k/v and gate/up, which
    read the same x, as one launch each (128 launches per step); fp16 runs the
    224 matrices one by one.  The step is replayed as a CUDA graph.  Bound:
    HBM on the weight bytes.  Weak scaling: each rank streams its own copy."""
    import ctypes as C

    import torch
    import torch.distributed as dist

    from yllm_b200 import attn, dist as ydist

    rank, world, local = ydist.init("nccl" if args.gpus > 1 else "gloo")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    L, H = args.layers or 32, 4096   # --layers shrinks the step for profiler captures only
    shapes = [(4096, H), (1024, H), (1024, H), (H, 4096), (14336, H), (14336, H), (H, 14336)]
    f16 = fmt == "f16"
    nbytes_of = (lambda o, i: o * i * 2) if f16 else (lambda o, i: o * (i // 256) * 144)
    per_layer = sum(nbytes_of(o, i) for o, i in shapes)
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    if f16:
        wbuf = torch.empty(L * per_layer // 2, dtype=torch.float16, device=dev).normal_(0.0, 0.02, generator=g)
        wbuf = wbuf.view(torch.uint8)
    else:
        wbuf = torch.randint(0, 256, (L * per_layer,), dtype=torch.uint8, device=dev, generator=g)
        # d and dmin of every block: small positive fp16 so the outputs stay finite
        blocks = wbuf.view(-1, 144)
        dd = (torch.rand(blocks.shape[0], 2, device=dev, generator=g) * 1e-3 + 5e-4).half()
        blocks[:, 0:4] = dd.view(torch.uint8).view(-1, 4)
    xs = {i: torch.randn(i, device=dev, generator=g) for i in (H, 14336)}
    ys = {o: torch.empty(o, device=dev) for o in (1024, 4096, 14336)}
    mats = []
    off = 0
    for l in range(L):
        for o, i in shapes:
            n = nbytes_of(o, i)
            mats.append((wbuf[off:off + n].view(torch.int16) if f16 else wbuf[off:off + n], o, i))
            off += n
    gemv = attn.gemv_f16 if f16 else attn.gemv_q4k
    # Q4_K: the matrices that read the same x go in one launch (q, k, v; gate, up), 4 launches per layer
    if f16:
        calls = [(lambda w=w, o=o, i=i: gemv(ys[o], w, xs[i], o, i, 1)) for w, o, i in mats]
    else:
        yq = {o: torch.empty(o, device=dev) for o in (1024, 4096, 14336)}   # second outputs of a group
        calls = []
        for l in range(L):
            q, k, v, o_, gt, up, dn = mats[7 * l:7 * l + 7]
            calls.append(lambda q=q, k=k, v=v: attn.gemv_q4k_multi([ys[4096], ys[1024], yq[1024]], [q[0], k[0], v[0]],
                                                                  [4096, 1024, 1024], xs[H], H))
            calls.append(lambda o_=o_: gemv(ys[4096], o_[0], xs[H], 4096, H, 1))
            calls.append(lambda gt=gt, up=up: attn.gemv_q4k_multi([ys[14336], yq[14336]], [gt[0], up[0]],
                                                                 [14336, 14336], xs[H], H))
            calls.append(lambda dn=dn: gemv(ys[4096], dn[0], xs[14336], 4096, 14336, 1))

    def step():
        for c in calls:
            c()

    ms, per_call, clk = _timed(step, args, stream, world, dist, local, graph=True)
    step_bytes = L * per_layer
    peaks, src = load_peaks()
    ach = step_bytes / (per_call / 1e3) / 1e9
    roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(ach / peaks["hbm_gbs"], 4),
            "traffic": None if (f16 or args.layers) else NCU_TRAFFIC["gemv_q4k_gate_up"],
            "kernel": "k_gemv_f16<4,1,2>" if f16 else "k_gemv_q4k_tc(_multi)<MT,KS,U> (mma.sync)",
            "peak_source": src, "bytes_per_step": step_bytes,
            "note": (f"{len(calls)} launches per step in one graph; achieved = weight bytes / step device time"
                     + ("" if f16 else "; traffic: one gate + up launch (two 14336 x 4096), 66,060,288 B of weights"))}
    e2e = None
    if not args.no_e2e:
        hx = torch.empty(H, dtype=torch.float32, pin_memory=True)
        hx.copy_(xs[H].cpu())
        hy = torch.empty(H, dtype=torch.float32, pin_memory=True)

        def e2e_step():
            xs[H].copy_(hx, non_blocking=True)
            step()
            hy.copy_(ys[4096], non_blocking=True)

        ems, _, _ = _timed(e2e_step, args, stream, world, dist, local)
        e2e = {"value": round(world / (ems / 1e3), 2), "unit": "tok/s", "h2d_bytes_per_step": H * 4 * world,
               "d2h_bytes_per_step": H * 4 * world,
               "path": (f"yattn_gemv_{fmt} per matrix" if f16 else
                        "yattn_gemv_q4k_multi for q/k/v and gate/up, yattn_gemv_q4k for o and down")
                       + " per step (no graph), pinned x in, y back"}
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        import numpy as np

        sys.path.insert(0, str(ROOT / "tests"))
        import oracle

        kind = "reference" if oracle.has_ref() else "port"
        lib = oracle.load("ref" if kind == "reference" else "port")
        lib.orc_set_threads(len(os.sched_getaffinity(0)))
        host = [(mats[j][0].cpu().numpy().view(np.uint16 if f16 else np.uint8), mats[j][1], mats[j][2])
                for j in range(len(shapes))]   # layer 0
        hxs = {i: xs[i].cpu().numpy() for i in xs}
        hys = {o: np.zeros(o, np.float32) for o in ys}
        times = []
        while not times or (sum(times) < min(args.cpu_budget, 10.0) and len(times) < 20):
            t0 = time.perf_counter()
            for w, o, i in host:
                (lib.orc_matmul_f16 if f16 else lib.orc_matmul_q4k)(hys[o], hxs[i], w, o, i)
            times.append(time.perf_counter() - t0)
        step_s = statistics.median(times) * L
        cpu = {"value": round(1 / step_s, 3), "unit": "tok/s", "cores": int(lib.orc_max_threads()), "kind": kind,
               "sample": f"layer 0's seven {'fp16 matmuls (matvec.c:111' if f16 else 'Q4_K matmuls (matvec.c:514'}"
                         f", the engine's path), timed {len(times)}x, x{L} layers"}
    if rank == 0:
        name = "fp16" if f16 else "Q4_K"
        line = _line(args, world, f"{name} linear layers tok/s (Llama-3-8B decode step, 32 layers, batch 1)",
                     world / (ms / 1e3), "tok/s", ms,
                     {"workload": f"llama3-8b-{fmt}-gemv-decode" + (f"-profile-{L}-layers" if args.layers else ""),
                      "layers": L, "hidden": H, "ffn": 14336,
                      "weight_bytes_per_step": step_bytes, "parallelism": f"replicas x{world}",
                      "launch": "CUDA graph replay of the step",
                      "l2": f"weights per step {step_bytes / 1e9:.1f} GB > L2"},
                     roof, args.steps * len(calls), clk, e2e, cpu=cpu, scaling="weak")
        line["dtype"] = f"{name} weights, f32 x and accumulation"
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_gdn_inputs(args) -> None:
    """The qwen35 GDN layer's input preparation (engine.c:785-821) for config
    5a's 4096-token chunk: gates, conv1d delay line + silu, q/k l2norm, one
    launch.  Bound: HBM (the projection read, q/k/v written).  Inputs above L2.
    Weak scaling: each rank prepares its own sequence."""
    import torch
    import torch.distributed as dist

    from yllm_b200 import attn, dist as ydist
    from yllm_b200.configs import CFG5_GDN as c

    rank, world, local = ydist.init("nccl" if args.gpus > 1 else "gloo")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    T, NK, NV, D, KW = c.tokens, c.num_k_heads, c.n_v_heads, c.head_dim, 4
    CC = 2 * NK * D + NV * D
    g = torch.Generator(device=dev)
    g.manual_seed(11 + rank)
    qkv = torch.randn(1, T, CC, device=dev, generator=g)
    st = torch.randn(1, KW, CC, device=dev, generator=g)
    wc = 0.5 * torch.randn(CC, KW, device=dev, generator=g)
    al = torch.randn(1, T, NV, device=dev, generator=g)
    bi = torch.randn(1, T, NV, device=dev, generator=g)
    dt = torch.randn(NV, device=dev, generator=g)
    a = -dt.abs()
    q = torch.empty(1, T, NK * D, device=dev)
    k = torch.empty_like(q)
    v = torch.empty(1, T, NV * D, device=dev)
    ga = torch.empty(1, T, NV, device=dev)
    be = torch.empty_like(ga)

    def step():
        attn.gdn_inputs(qkv, st, wc, al, bi, dt, a, q, k, v, ga, be, 1, T, KW, NK, D, NV, D, eps=c.eps)

    ms, per_call, clk = _timed(step, args, stream, world, dist, local, graph=True, flush_l2=True)
    nbytes = (qkv.numel() + q.numel() + k.numel() + v.numel() + 4 * al.numel()) * 4
    peaks, src = load_peaks()
    ach = nbytes / (per_call / 1e3) / 1e9
    roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(ach / peaks["hbm_gbs"], 4), "traffic": NCU_TRAFFIC["gdn_inputs"], "kernel": "k_gdn_inputs<4,32>",
            "peak_source": src, "bytes_per_step": nbytes}
    if rank == 0:
        line = _line(args, world, "GDN layer inputs tok/s (qwen3.5 shape, one 4096-token chunk)",
                     T * world / (ms / 1e3), "tok/s", ms,
                     {"workload": c.name + "-inputs-4096", "tokens": T, "conv_chan": CC, "kwidth": KW,
                      "num_k_heads": NK, "n_v_heads": NV, "head_dim": D,
                      "parallelism": f"data-parallel x{world}: one sequence per GPU",
                      "launch": "CUDA graph replay of the step",
                      "l2": "L2 scrubbed between timed steps outside the step's events"},
                     roof, args.steps, clk, scaling="weak")
        line["dtype"] = "f32"
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_sess_kv(args) -> None:
    """The session KV file of a Llama-3-8B-shaped engine (32 blocks, kv_dim
    1024, max_seq 8192, every row filled: 1 GiB of K and V) saved from and
    loaded back into HBM through the library (cache.c:174-247 on the host
    blob in the reference).  A step is one save plus one load.  The file sits
    in the host's page cache (tmpfs or disk cache); the bound is the host
    side: PCIe for the device copies, memory bandwidth for the file copy.
    Rank 0 only (a host file per GPU adds nothing)."""
    import ctypes as C
    import tempfile

    import torch

    from yllm_b200 import attn

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    nb, kd, max_seq, pos = 32, 1024, 8192, 8192
    n = (2 * nb + 1) * max_seq * kd
    blob = torch.randint(-32768, 32768, (n,), dtype=torch.int32, device="cuda").to(torch.int16)
    back = torch.zeros_like(blob)
    nbytes = 2 * nb * pos * kd * 2
    # tmpfs where the host has one, so the line measures the library's path and not the box's virtual disk
    # (a 1 GB write to the disk-backed /tmp runs at its writeback rate, under 2 GB/s for either arm)
    shm = "/dev/shm" if os.path.isdir("/dev/shm") and os.access("/dev/shm", os.W_OK) else None
    d = tempfile.mkdtemp(prefix="yattn_sess_", dir=shm)
    path = os.path.join(d, "s.kv")

    def step():
        attn.sess_kv_save(blob, nb, kd, max_seq, pos, path)
        attn.sess_kv_load(back, nb, kd, max_seq, path)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert torch.equal(back.view(2 * nb + 1, max_seq, kd)[1:], blob.view(2 * nb + 1, max_seq, kd)[1:])
    clocks = ClockSampler(0)
    clocks.start()
    time.sleep(0.3)
    clocks.begin()
    ts, tsave = [], []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        attn.sess_kv_save(blob, nb, kd, max_seq, pos, path)
        t1 = time.perf_counter()
        attn.sess_kv_load(back, nb, kd, max_seq, path)
        ts.append(time.perf_counter() - t0)
        tsave.append(t1 - t0)
    clk = clocks.stop()
    ms = statistics.median(ts) * 1e3
    save_ms = statistics.median(tsave) * 1e3
    # the host-side peak this is bound by: pinned D2H + H2D of the same bytes (CUDA events)
    pin = torch.empty(64 << 20, dtype=torch.uint8, pin_memory=True)
    src = torch.empty(64 << 20, dtype=torch.uint8, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        pin.copy_(src, non_blocking=True)
    e0.record()
    for _ in range(16):
        pin.copy_(src, non_blocking=True)
        src.copy_(pin, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    pcie = 2 * 16 * (64 << 20) / (e0.elapsed_time(e1) / 1e3) / 1e9
    ach = 2 * nbytes / (ms / 1e3) / 1e9
    cpu = None
    if not args.no_cpu_baseline:
        sys.path.insert(0, str(ROOT / "tests"))
        import numpy as np
        import oracle

        kind = "reference" if oracle.has_ref() else "port"
        lib = oracle.load("ref" if kind == "reference" else "port")
        hb = blob.cpu().numpy().view(np.uint16)
        hback = np.zeros_like(hb)
        p = C.c_uint32(0)
        cts, csave = [], []
        for _ in range(3):
            t0 = time.perf_counter()
            lib.orc_sess_kv_save(hb, nb, kd, max_seq, pos, path.encode())
            t1 = time.perf_counter()
            lib.orc_sess_kv_load(hback, nb, kd, max_seq, path.encode(), C.byref(p))
            cts.append(time.perf_counter() - t0)
            csave.append(t1 - t0)
        cpu = {"value": round(2 * nbytes / statistics.median(cts) / 1e9, 3), "unit": "GB/s", "cores": 1,
               "kind": kind, "sample": "the same 1 GiB file saved from and loaded into a host blob, 3x",
               "save_gbs": round(nbytes / statistics.median(csave) / 1e9, 3)}
    os.remove(path)
    os.rmdir(d)
    roof = {"bound": "pcie", "achieved": round(ach, 2), "peak": round(pcie, 2), "unit": "GB/s",
            "frac": round(ach / pcie, 4), "traffic": None, "kernel": "cudaMemcpyAsync D2H / H2D via pinned staging",
            "peak_source": "pinned D2H + H2D copy measured in this run (64 MiB x 16 each way)",
            "note": "file bytes each way per step / step wall time; the page-cache copy shares the host memory"}
    line = {"metric": "session KV save + load GB/s (device blob <-> engine session file)", "value": round(ach, 3),
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "u16 (fp16 bits)",
            "data": "synthetic (random fp16 bits)",
            "config": {"workload": "sess-kv-llama3-8b", "n_blocks": nb, "kv_dim": kd, "max_seq": max_seq, "pos": pos,
                       "file_bytes": 24 + nbytes, "timing": "host wall clock around save + load (host I/O path)",
                       "save_gbs": round(nbytes / (save_ms / 1e3) / 1e9, 3),
                       "load_gbs": round(nbytes / ((ms - save_ms) / 1e3) / 1e9, 3), "dir": d},
            "e2e": {"value": round(ach, 3), "unit": "GB/s", "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
                    "path": "yattn_sess_kv_save then yattn_sess_kv_load (the public calls)"},
            "roofline": roof, "gpu_launches": 0,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                       "samples": clk["samples"], "source": clk.get("source")}}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "prefill", "gated_prefill", "gdn_prefill", "gdn_decode", "long_decode",
                             "config1_decode", "gated_decode", "rope_store", "sess_kv", "gemv", "gemv_f16", "gdn_inputs",
                             "fused_decode"],
                    help="decode = BASELINE config 3 (the default bench line)")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--seqs", type=int, default=0, help="profiling only: first N sequences")
    ap.add_argument("--layers", type=int, default=0, help="profiling only: first L layers")
    ap.add_argument("--cpu-budget", type=float, default=20.0, help="seconds of CPU attention in the baseline")
    ap.add_argument("--weak", action="store_true",
                    help="decode at N>1: every rank serves a whole 64-sequence batch (default: the 64 sharded)")
    ap.add_argument("--no-long", action="store_true", help="decode: skip the config-4 long_decode sub-object")
    ap.add_argument("--exchange", choices=["peer", "peer2", "nccl"], default="peer",
                    help="long_decode at N>1: split-KV exchange over peer memory fused into the split merge (peer), "
                         "over peer memory as its own launch after the partial decode (peer2), or NCCL all-gather")
    args = ap.parse_args()
    if args.warmup < 3:
        log("warmup raised to 3 (timing rule)")
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "decode":
        run_ours(args)
    elif args.workload in ("prefill", "gated_prefill"):
        run_prefill(args, gated=args.workload == "gated_prefill")
    elif args.workload in ("gdn_prefill", "gdn_decode"):
        run_gdn(args, decode=args.workload == "gdn_decode")
    elif args.workload in ("config1_decode", "gated_decode"):
        run_decode_small(args)
    elif args.workload == "rope_store":
        run_rope_store(args)
    elif args.workload == "sess_kv":
        run_sess_kv(args)
    elif args.workload in ("gemv", "gemv_f16"):
        run_gemv(args, "f16" if args.workload == "gemv_f16" else "q4k")
    elif args.workload == "gdn_inputs":
        run_gdn_inputs(args)
    elif args.workload == "fused_decode":
        run_fused_decode(args)
    else:
        run_long_decode(args)


if __name__ == "__main__":
    main()
