#!/usr/bin/env python3
"""Benchmark of the B200 kernel backend on the encoder-block workload.

Default workload: the BERT-base post-LN encoder block (hidden 768, 12 heads,
head dim 64, FFN 3072, tanh-GELU, no mask) at batch 8, sequence 512, fp16, seven
sm_100a kernels captured in one CUDA graph. A step is one forward of that block
over 4096 tokens; metric = encoder-block tokens/s.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl lunara|reference]
                  [--workload block|stack|gemm|attention|attention_causal|layernorm|bias_gelu|softmax|qkv_split|tp_ffn]

Timing: W untimed warm-up steps, then K steps, each bracketed by CUDA events on
the launching stream, with a 256 MB L2-flush write between steps (outside the
events); a barrier and torch.cuda.synchronize() on both sides of the K steps;
the max over ranks is reported. Multi-GPU (torchrun, one rank per GPU, NCCL) is
batch sharding with no collective on the data path: every rank runs its own
batch-8 block (weak scaling). `e2e` runs the step as a serving loop does: the
input copied from pinned host memory, the block, the output copied back to
pinned host memory, every step, with the copies of neighbouring steps
overlapping the kernels on their own streams (two buffer pairs).
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
    """DRAM bytes per launch of a kernel, from the ncu summary profiles/<workload>*.md
    (line 'dram_bytes_per_launch[<kernel>]: N')."""
    key = f"dram_bytes_per_launch[{kernel}]:"
    for f in sorted((ROOT / "profiles").glob(f"{workload}*.md")):
        for line in f.read_text().splitlines():
            if line.strip().startswith(key):
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
    # programmatic-launch overlap).
    runner = GraphRunner(lambda: blk.run_kernels())
    # Per-kernel durations: one graph per kernel holding REPS back-to-back
    # launches of it on the block's own buffers (every launch is idempotent),
    # timed with events around the replay, replayed after the timed loop.
    reps = 20
    fns = blk.kernel_fns()
    kernel_runners = {name: GraphRunner(lambda f=f: [f() for _ in range(reps)]) for name, f in fns.items()}

    # 256 MB (twice the 126 MB L2), int64 so that the fill kernel stores wide words.
    flush = torch.empty(32 * 1024 * 1024, dtype=torch.int64, device=device)
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
    for name, kr in kernel_runners.items():
        for i in range(6):
            flush.zero_()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            kr.replay()
            s1.record(stream)
            s1.synchronize()
            if i > 0:
                kernel_ms[name].append(s0.elapsed_time(s1) / reps)
        kr.release()

    # End to end through host buffers, as a serving loop runs it: every step
    # copies its input from pinned host memory (H2D stream), runs the block
    # (compute stream, with the L2 flush) and copies its output back to pinned
    # host memory (D2H stream). Two input/output buffer pairs let step i+1's
    # H2D and step i-1's D2H overlap step i's kernels; events order the reuse
    # of each buffer. Whole-loop time / steps.
    x_host = x.half().view(batch * seq, 768).pin_memory()
    y_hosts = [torch.empty(batch * seq, 768, dtype=torch.float16).pin_memory() for _ in range(2)]
    xb = [blk.x, torch.empty_like(blk.x)]
    yb = [blk.y, torch.empty_like(blk.y)]
    e2e_runners = [runner, GraphRunner(lambda: blk.run_kernels(x=xb[1], out=yb[1]))]
    h2d_s, d2h_s = torch.cuda.Stream(), torch.cuda.Stream()

    def e2e_loop(n):
        ev = lambda: torch.cuda.Event()  # noqa: E731
        h2d_done, comp_done, d2h_done = [ev(), ev()], [ev(), ev()], [ev(), ev()]
        for i in range(n):
            k = i % 2
            if i >= 2:
                h2d_s.wait_event(comp_done[k])        # step i-2 has finished reading xb[k]
            with torch.cuda.stream(h2d_s):
                xb[k].copy_(x_host, non_blocking=True)
                h2d_done[k].record(h2d_s)
            stream.wait_event(h2d_done[k])
            if i >= 2:
                stream.wait_event(d2h_done[k])        # step i-2's output has left yb[k]
            flush.zero_()
            e2e_runners[k].replay()
            comp_done[k].record(stream)
            d2h_s.wait_event(comp_done[k])
            with torch.cuda.stream(d2h_s):
                y_hosts[k].copy_(yb[k], non_blocking=True)
                d2h_done[k].record(d2h_s)
        stream.wait_stream(d2h_s)
        stream.wait_stream(h2d_s)

    e2e_loop(max(args.warmup, 2))
    torch.cuda.synchronize()
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_loop(args.steps)
    e1.record(stream)
    e1.synchronize()
    _barrier(world)
    e2e_total = _max_over_ranks(e0.elapsed_time(e1), world)
    assert torch.equal(y_hosts[(args.steps - 1) % 2], yb[(args.steps - 1) % 2].cpu()), "e2e output mismatch"
    for r_ in e2e_runners:
        r_.release()

    mean_k = {k: statistics.median(v) for k, v in kernel_ms.items() if v}
    dom = max(mean_k, key=mean_k.get)
    tokens = batch * seq
    return {
        "tokens_per_step": tokens * world,
        "total_ms": total_ms,
        "e2e_total_ms": e2e_total,
        "h2d": x_host.numel() * 2, "d2h": y_hosts[0].numel() * 2,
        "kernel_ms": mean_k, "dominant": dom, "dominant_flops": flops[dom],
        "launches_per_step": len(KERNEL_ORDER),
        "clocks": clk.summary(),
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["lunara", "reference"], default="lunara")
    ap.add_argument("--workload", default="block",
                    choices=["block", "stack", "gemm", "attention", "attention_causal", "layernorm", "bias_gelu",
                             "softmax", "qkv_split", "tp_ffn"])
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
                       "kernel_timing": "per kernel: CUDA events around a graph of 20 back-to-back launches "
                                        "on the block's buffers, / 20 (median of 5)"},
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
