#!/usr/bin/env python3
"""Benchmark of the B200 kernel backend on the encoder-block workload.

Default workload: the BERT-base post-LN encoder block (hidden 768, 12 heads,
head dim 64, FFN 3072, tanh-GELU, no mask) at batch 8, sequence 512, fp16, seven
sm_100a kernels captured in one CUDA graph. A step is one forward of that block
over 4096 tokens; metric = encoder-block tokens/s.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl lunara|reference]
                  [--workload block|stack|gemm|attention|attention_causal|layernorm|bias_gelu]

Timing: W untimed warm-up steps, then K steps, each bracketed by CUDA events on
the launching stream, with a 256 MB L2-flush write between steps (outside the
events); a barrier and torch.cuda.synchronize() on both sides of the K steps;
the max over ranks is reported. Multi-GPU (torchrun, one rank per GPU, NCCL) is
batch sharding with no collective on the data path: every rank runs its own
batch-8 block (weak scaling). `e2e` repeats the step through the host-facing
API (pinned host input -> device, block, device -> pinned host output).
`--impl reference` times the reference's CPU path (torch eager fp32 on the host
cores, the oracle) on the same workload.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

TOKENS_METRIC = "encoder-block tokens/s (B8,S512,H768)"


def _rank_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), \
        int(os.environ.get("LOCAL_RANK", "0"))


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def _traffic_from_profiles(kernel: str, workload: str):
    """DRAM bytes per launch recorded in profiles/<kernel>_<workload>.md (line 'dram_bytes_per_launch: N')."""
    for f in sorted((ROOT / "profiles").glob(f"{kernel}_{workload}*.md")):
        for line in f.read_text().splitlines():
            if line.strip().startswith("dram_bytes_per_launch:"):
                try:
                    return float(line.split(":", 1)[1].strip().split()[0])
                except ValueError:
                    return None
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    INTERVAL_MS = 20

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.window = None

    def mark(self, start: bool):
        """Host wall-clock bounds of the timed region (samples outside it are dropped)."""
        now = datetime.datetime.now()
        if start:
            self.window = [now, None]
        elif self.window is not None:
            self.window[1] = now

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", str(self.INTERVAL_MS), "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.path is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
            except ValueError:
                continue
            rows.append((ts, parts[1:]))
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        inside = rows
        if self.window is not None and self.window[1] is not None:
            lo, hi = self.window
            inside = [r for r in rows if lo <= r[0] <= hi]
            if not inside:   # timed region shorter than the sampling interval: nearest sample after its start
                after = [r for r in rows if r[0] >= lo] or rows[-1:]
                inside = after[:1]
        rows = [r[1] for r in inside]
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows),
                "window_ms": round((self.window[1] - self.window[0]).total_seconds() * 1e3, 1)
                if self.window and self.window[1] else None}


# ─────────────────────────────────────────────────────────── reference arm ──

def cpu_block_sample(budget_s: float, steps: int = 0, warmup: int = 1, batch: int = 8, seq: int = 512):
    """Time the oracle (torch eager fp32 on the host cores) on the block workload."""
    from oracle import inputs, oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    x, w = inputs.block_inputs(batch, seq, seed=0)
    for _ in range(warmup):
        oracle.encoder_block(x, w, num_heads=12)
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        oracle.encoder_block(x, w, num_heads=12)
        times.append(time.perf_counter() - t0)
        if steps and len(times) >= steps:
            break
        if budget_s and time.perf_counter() - t_start > budget_s:
            break
        if not steps and len(times) >= 50:
            break
    tokens = batch * seq
    return {"value": tokens * len(times) / sum(times), "unit": "tokens/s", "cores": threads,
            "kind": "port", "sample": f"{len(times)} full block forwards B{batch} S{seq} fp32, "
                                      f"median {statistics.median(times) * 1e3:.1f} ms"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    # K steps of one block forward each, stopped after 90 s of host time so that
    # a long --steps run still ends within minutes (the sample says how many ran).
    cb = cpu_block_sample(budget_s=90.0, steps=args.steps, warmup=min(args.warmup, 3))
    line = {"impl": "reference", "metric": TOKENS_METRIC, "value": cb["value"], "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 4096 / cb["value"] * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights)",
            "config": {"workload": "encoder block B8 S512 H768 heads12 FFN3072 tanh-GELU post-LN",
                       "global_batch": 8, "seq_len": 512, "parallelism": "host CPU (torch eager fp32)"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ──────────────────────────────────────────────────────────── lunara arm ──

def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def bench_block(args, rank, world, device):
    from oracle import inputs
    from lunara_b200.runtime.encoder import EncoderBlock, GraphRunner, KERNEL_ORDER, block_flops
    batch, seq = 8, 512
    x, w = inputs.block_inputs(batch, seq, seed=rank)
    blk = EncoderBlock(w, batch, seq, num_heads=12, dtype=torch.float16, device=device)
    blk.x.copy_(x.half().view(batch * seq, 768).to(device))
    flops = block_flops(batch * seq, seq)

    # Timed graph: the seven kernels alone (adjacent kernel nodes keep their
    # programmatic-launch overlap). A second copy of the graph with an event
    # between kernels (external events) gives per-kernel durations; it is
    # replayed in its own loop after the timed one, since event nodes between
    # kernels serialise them.
    runner = GraphRunner(lambda: blk.run_kernels())
    n_ev = len(KERNEL_ORDER) + 1
    evs = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(n_ev)]
    idx = {name: i for i, name in enumerate(KERNEL_ORDER)}

    def hook(name, where):
        if where == "begin" and name == KERNEL_ORDER[0]:
            evs[0].record()
        elif where == "end":
            evs[idx[name] + 1].record()

    try:
        prof_runner = GraphRunner(lambda: blk.run_kernels(hook=hook))
    except Exception as e:  # graph event nodes unsupported: per-kernel times from eager launches
        print(f"[bench] per-kernel events in graph unavailable ({e}); timing kernels eagerly", file=sys.stderr)
        prof_runner = None

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        flush.zero_()
        runner.replay()
    torch.cuda.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(torch.cuda.current_device()) as clk:
        _barrier(world)
        torch.cuda.synchronize()
        clk.mark(True)
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            runner.replay()
            ends[i].record(stream)
        torch.cuda.synchronize()
        clk.mark(False)
        _barrier(world)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = _max_over_ranks(sum(step_ms), world)

    kernel_ms = {k: [] for k in KERNEL_ORDER}
    if prof_runner is not None:
        for i in range(args.steps + 1):
            flush.zero_()
            prof_runner.replay()
            torch.cuda.synchronize()
            if i > 0:
                for k, name in enumerate(KERNEL_ORDER):
                    kernel_ms[name].append(evs[k].elapsed_time(evs[k + 1]))
        prof_runner.release()
    else:
        eager = {k: [] for k in KERNEL_ORDER}
        cur = {}

        def ehook(name, where):
            if where == "begin":
                cur[name] = torch.cuda.Event(enable_timing=True)
                cur[name].record()
            else:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                eager[name].append((cur[name], e))
        for _ in range(args.steps):
            flush.zero_()
            blk.run_kernels(hook=ehook)
        torch.cuda.synchronize()
        kernel_ms = {k: [a.elapsed_time(b) for a, b in v] for k, v in eager.items()}

    # End to end through host buffers: pinned input -> device, block, device -> pinned output.
    x_host = x.half().view(batch * seq, 768).pin_memory()
    y_host = torch.empty(batch * seq, 768, dtype=torch.float16).pin_memory()
    e2e_ms = []
    for i in range(args.steps + args.warmup):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        blk.x.copy_(x_host, non_blocking=True)
        out = runner.replay()
        y_host.copy_(out, non_blocking=True)
        e.record(stream)
        e.synchronize()
        if i >= args.warmup:
            e2e_ms.append(s.elapsed_time(e))
    e2e_total = _max_over_ranks(sum(e2e_ms), world)
    runner.release()

    mean_k = {k: statistics.mean(v) for k, v in kernel_ms.items() if v}
    dom = max(mean_k, key=mean_k.get)
    tokens = batch * seq
    return {
        "tokens_per_step": tokens * world,
        "total_ms": total_ms,
        "e2e_total_ms": e2e_total,
        "h2d": x_host.numel() * 2, "d2h": y_host.numel() * 2,
        "kernel_ms": mean_k, "dominant": dom, "dominant_flops": flops[dom],
        "launches_per_step": len(KERNEL_ORDER),
        "clocks": clk.summary(),
        "per_kernel_events": prof_runner is not None,
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["lunara", "reference"], default="lunara")
    ap.add_argument("--workload", default="block",
                    choices=["block", "stack", "gemm", "attention", "attention_causal", "layernorm", "bias_gelu"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    assert args.warmup >= 0 and args.steps >= 1
    rank, world, local = _rank_env()

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    from lunara_b200.runtime import _lib
    _lib.load()

    if args.workload != "block":
        from lunara_b200 import kernel_bench
        line = kernel_bench.run(args.workload, args, rank, world, device)
        if rank == 0:
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    r = bench_block(args, rank, world, device)
    peaks = _peaks()
    if rank == 0:
        value = r["tokens_per_step"] * args.steps / (r["total_ms"] * 1e-3)
        e2e = r["tokens_per_step"] * args.steps / (r["e2e_total_ms"] * 1e-3)
        dom_ms = r["kernel_ms"][r["dominant"]]
        achieved = r["dominant_flops"] / (dom_ms * 1e-3) / 1e12
        traffic = _traffic_from_profiles(r["dominant"], "block_b8s512")
        line = {
            "metric": TOKENS_METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["total_ms"] / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights, zero biases, LN 1/0)",
            "config": {"workload": "encoder block B8 S512 H768 heads12 FFN3072 tanh-GELU post-LN, fp16",
                       "global_batch": 8 * world, "seq_len": 512,
                       "parallelism": f"batch-sharded replicas x{world} (no collective)",
                       "l2": "256 MB flush write between timed steps",
                       "graph": "7 kernels in one CUDA graph (programmatic dependent launch)",
                       "kernel_timing": "per-kernel CUDA events from an instrumented replay of the same graph"},
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": r["h2d"] * world,
                    "d2h_bytes_per_step": r["d2h"] * world},
            "gpu_launches": r["launches_per_step"] * args.steps,
            "roofline": {"kernel": r["dominant"], "bound": "tensor", "achieved": achieved,
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": achieved / peaks["bf16_tflops"], "traffic": traffic,
                         "peak_source": f"{peaks['source']} bf16 burst"},
            "kernel_ms": {k: round(v, 5) for k, v in r["kernel_ms"].items()},
            "clocks": r["clocks"],
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_block_sample(budget_s=15.0)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
