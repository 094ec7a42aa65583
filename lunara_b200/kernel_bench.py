"""Per-kernel benchmark workloads (the non-block benchmark configurations).

  gemm              C = A B, M=N=K=4096 fp16, plus the bias+GELU epilogue variant
  attention         B2 H12 S2048 D64 fp16, non-causal   (25.77 GFLOP)
  attention_causal  same, causal                          (12.88 GFLOP, half)
  layernorm         16384 x 768 fp16                      (50.33 MB moved)
  bias_gelu         16384 x 3072 fp16 + bias, tanh GELU   (201.33 MB moved)
  softmax           49152 x 512 fp16 row softmax, the block's score shape
                    (B8 H12 S512 rows of 512 keys; 100.66 MB moved)
  qkv_split         [8, 512, 2304] fp16 fused projection -> 3 x [8, 12, 512, 64]
                    (the QKV split + head reshape graph op, bit-exact; 37.75 MB moved)
  stack             12-layer encoder stack, batch 64 split over the ranks

Each step replays a CUDA graph of 10 back-to-back launches between CUDA
events, with a 256 MB L2-flush write between steps outside the events; the
launches cycle over enough distinct buffer sets that none finds its inputs
in L2; the per-launch time is the step time / 10. Used by bench.py.
"""
from __future__ import annotations

import json
import statistics
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def _sustained_tflops() -> float:
    """cuBLAS bf16 throughput held for seconds under the 1 kW power cap: the
    denominator for a GEMM loop that itself runs for seconds."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops_sustained", d["bf16_tflops"])
    return 1400.0


def _time_steps(fns, steps, warmup, flush):
    """Per-launch device time (ms), one value per step.

    ``fns`` are launches on distinct buffer sets, enough of them that their
    working sets together exceed L2 (no launch finds its inputs left in L2 by
    the previous one). They are captured back to back, REPS = 10 launches
    cycling over the sets, into one CUDA graph; a step replays the graph
    between CUDA events after a 256 MB L2-flush write outside them and counts
    time / REPS, so host launch cost is not in the number.
    """
    from lunara_b200.runtime.encoder import GraphRunner
    reps = 10
    runner = GraphRunner(lambda: [fns[i % len(fns)]() for i in range(reps)])
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        flush.zero_()
        runner.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        runner.replay()
        e.record(stream)
        e.synchronize()
        times.append(s.elapsed_time(e) / reps)
    runner.release()
    return times


def _rotations(working_set_bytes: int) -> int:
    """Buffer sets needed so that consecutive launches never share data in L2."""
    return max(1, min(10, -(-(256 << 20) // working_set_bytes)))


def _same_size_copy_gbs(nbytes: int, steps: int, warmup: int, flush, device) -> float:
    """Device-to-device copy rate (read + write GB/s) for a transfer of ``nbytes``
    each way, timed exactly like the kernels (same rotation, flush and graph).

    A bandwidth kernel of a few tens of MB pays a fixed ramp and drain per
    launch that a multi-GB copy (the HBM peak) does not; this figure is the
    roofline of a pure copy at the kernel's own size.
    """
    words = max(1, nbytes // 8)
    n = _rotations(2 * words * 8)
    sets = [(torch.ones(words, dtype=torch.int64, device=device), torch.empty(words, dtype=torch.int64, device=device))
            for _ in range(n)]
    t = _time_steps([lambda s=s_: s[1].copy_(s[0]) for s_ in sets], min(steps, 200), warmup, flush)
    return 2.0 * words * 8 / (statistics.median(t) * 1e-3) / 1e9


def config_kernel_map(device, steps: int = 20, warmup: int = 3):
    """Every single-kernel benchmark configuration, timed as the workloads above
    (rotated buffer sets, 256 MB flush between steps, graphs of 10 launches),
    with a short step count: {name: {ms, value, unit, frac, peak_source}}.

      gemm4096_{f16,bf16}[_bias_gelu]   M=N=K=4096, tensor roof
      attention_s2048[_causal]          B2 H12 S2048 D64 fp16, tensor roof (causal: half the FLOPs)
      layernorm_16384x768               fp16, HBM roof
      bias_gelu_16384x3072              fp16, HBM roof
    """
    from oracle import inputs
    from lunara_b200.runtime import ops
    hbm, tflops_peak, src = _peaks()
    flush = torch.empty(32 << 20, dtype=torch.int64, device=device)
    out = {}

    def put(name, t, work, unit):
        ms = statistics.median(t)
        if unit == "TFLOP/s":
            val, peak = work / (ms * 1e-3) / 1e12, tflops_peak
        else:
            val, peak = work / (ms * 1e-3) / 1e9, hbm
        out[name] = {"ms": round(ms, 5), "value": round(val, 1), "unit": unit, "frac": round(val / peak, 3),
                     "peak_source": f"{src} {'bf16 burst' if unit == 'TFLOP/s' else 'copy'}"}

    a, b, bias = inputs.gemm_inputs()
    for dt, tag in ((torch.float16, "f16"), (torch.bfloat16, "bf16")):
        ad, bd, biasd = a.to(dt).to(device), b.to(dt).to(device), bias.to(dt).to(device)
        sets = [(ad.clone(), bd.clone(), torch.empty(4096, 4096, dtype=dt, device=device))
                for _ in range(_rotations(3 * 4096 * 4096 * 2))]
        put(f"gemm4096_{tag}", _time_steps([lambda s=s_: ops.gemm(s[0], s[1], s[2]) for s_ in sets],
                                           steps, warmup, flush), 2.0 * 4096 ** 3, "TFLOP/s")
        put(f"gemm4096_{tag}_bias_gelu",
            _time_steps([lambda s=s_: ops.gemm(s[0], s[1], s[2], bias=biasd, activation="gelu_tanh") for s_ in sets],
                        steps, warmup, flush), 2.0 * 4096 ** 3, "TFLOP/s")
        del sets, ad, bd
    q, k, v = (t.half().to(device) for t in inputs.attention_inputs())
    sets = [(q.clone(), k.clone(), v.clone(), torch.empty_like(q)) for _ in range(_rotations(4 * q.numel() * 2))]
    for causal in (False, True):
        t = _time_steps([lambda s=s_: ops.attention(s[0], s[1], s[2], causal=causal, out=s[3]) for s_ in sets],
                        steps, warmup, flush)
        put("attention_s2048" + ("_causal" if causal else ""), t,
            4.0 * 2 * 12 * 2048 * 2048 * 64 * (0.5 if causal else 1.0), "TFLOP/s")
    del sets
    x, w, b = inputs.layernorm_inputs()
    x, w, b = x.half().to(device), w.half().to(device), b.half().to(device)
    sets = [(x.clone(), torch.empty_like(x)) for _ in range(_rotations(2 * x.numel() * 2))]
    put("layernorm_16384x768", _time_steps([lambda s=s_: ops.layernorm(s[0], w, b, 1e-5, out=s[1]) for s_ in sets],
                                           steps, warmup, flush), 2.0 * 16384 * 768 * 2 + 2 * 768 * 2, "GB/s")
    del sets
    x, bias = inputs.bias_gelu_inputs()
    x, bias = x.half().to(device), bias.half().to(device)
    sets = [(x.clone(), torch.empty_like(x)) for _ in range(_rotations(2 * x.numel() * 2))]
    put("bias_gelu_16384x3072", _time_steps([lambda s=s_: ops.bias_act(s[0], bias, "gelu_tanh", out=s[1])
                                             for s_ in sets], steps, warmup, flush),
        2.0 * 16384 * 3072 * 2 + 3072 * 2, "GB/s")
    return out


def run(workload, args, rank, world, device):
    from oracle import inputs
    from lunara_b200.runtime import ops
    hbm, tflops_peak, src = _peaks()
    flush = torch.empty(32 << 20, dtype=torch.int64, device=device)   # 256 MB, wide stores
    line = {"steps": args.steps, "warmup": args.warmup, "n_gpus": world, "data": "synthetic (seeded)"}
    if workload == "gemm":
        a, b, bias = inputs.gemm_inputs()
        a, b, bias = a.half().to(device), b.half().to(device), bias.half().to(device)
        n = _rotations(3 * 4096 * 4096 * 2)
        sets = [(a.clone(), b.clone(), torch.empty(4096, 4096, dtype=torch.float16, device=device)) for _ in range(n)]
        t_plain = _time_steps([lambda s=s_: ops.gemm(s[0], s[1], s[2]) for s_ in sets], args.steps, args.warmup, flush)
        t_fused = _time_steps([lambda s=s_: ops.gemm(s[0], s[1], s[2], bias=bias, activation="gelu_tanh")
                               for s_ in sets], args.steps, args.warmup, flush)
        flops = 2.0 * 4096 ** 3
        tp = flops / (statistics.median(t_plain) * 1e-3) / 1e12
        tf = flops / (statistics.median(t_fused) * 1e-3) / 1e12
        line.update(metric="GEMM 4096^3 fp16 TFLOP/s", value=tp, unit="TFLOP/s", dtype="f16",
                    config={"workload": "GEMM M=N=K=4096 fp16 row-major, fp32 accumulate"},
                    ms_per_step=statistics.median(t_plain), bias_gelu_tflops=tf,
                    timed_seconds=sum(t_plain) * 10 * 1e-3,
                    roofline={"bound": "tensor", "achieved": tp, "peak": tflops_peak, "unit": "TFLOP/s",
                              "frac": tp / tflops_peak, "peak_source": f"{src} bf16 burst",
                              "sustained_peak": _sustained_tflops(),
                              "frac_of_sustained": tp / _sustained_tflops()})
    elif workload in ("attention", "attention_causal"):
        causal = workload == "attention_causal"
        q, k, v = (t.half().to(device) for t in inputs.attention_inputs())
        n = _rotations(4 * q.numel() * 2)
        sets = [(q.clone(), k.clone(), v.clone(), torch.empty_like(q)) for _ in range(n)]
        t = _time_steps([lambda s=s_: ops.attention(s[0], s[1], s[2], causal=causal, out=s[3]) for s_ in sets],
                        args.steps, args.warmup, flush)
        flops = 4.0 * 2 * 12 * 2048 * 2048 * 64 * (0.5 if causal else 1.0)
        ach = flops / (statistics.median(t) * 1e-3) / 1e12
        line.update(metric=f"attention B2 H12 S2048 D64 fp16 {'causal' if causal else 'non-causal'} TFLOP/s",
                    value=ach, unit="TFLOP/s", dtype="f16", ms_per_step=statistics.median(t),
                    config={"workload": "SDPA B2 H12 S2048 D64 fp16, scale 1/8",
                            "flops_convention": "4*B*H*S^2*D, halved for causal"},
                    roofline={"bound": "tensor", "achieved": ach, "peak": tflops_peak, "unit": "TFLOP/s",
                              "frac": ach / tflops_peak, "peak_source": f"{src} bf16 burst"})
    elif workload == "layernorm":
        x, w, b = inputs.layernorm_inputs()
        x, w, b = x.half().to(device), w.half().to(device), b.half().to(device)
        n = _rotations(2 * x.numel() * 2)
        sets = [(x.clone(), torch.empty_like(x)) for _ in range(n)]
        t = _time_steps([lambda s=s_: ops.layernorm(s[0], w, b, 1e-5, out=s[1]) for s_ in sets],
                        args.steps, args.warmup, flush)
        nbytes = 2.0 * 16384 * 768 * 2 + 2 * 768 * 2
        gbs = nbytes / (statistics.median(t) * 1e-3) / 1e9
        cp = _same_size_copy_gbs(16384 * 768 * 2, args.steps, args.warmup, flush, device)
        line.update(metric="LayerNorm 16384x768 fp16 GB/s", value=gbs, unit="GB/s", dtype="f16",
                    ms_per_step=statistics.median(t), config={"workload": "LayerNorm 16384x768 fp16"},
                    roofline={"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                              "peak_source": f"{src} copy", "same_size_copy_gbs": cp,
                              "frac_of_same_size_copy": gbs / cp})
    elif workload == "bias_gelu":
        x, bias = inputs.bias_gelu_inputs()
        x, bias = x.half().to(device), bias.half().to(device)
        n = _rotations(2 * x.numel() * 2)
        sets = [(x.clone(), torch.empty_like(x)) for _ in range(n)]
        t = _time_steps([lambda s=s_: ops.bias_act(s[0], bias, "gelu_tanh", out=s[1]) for s_ in sets],
                        args.steps, args.warmup, flush)
        nbytes = 2.0 * 16384 * 3072 * 2 + 3072 * 2
        gbs = nbytes / (statistics.median(t) * 1e-3) / 1e9
        cp = _same_size_copy_gbs(16384 * 3072 * 2, args.steps, args.warmup, flush, device)
        line.update(metric="bias+GELU 16384x3072 fp16 GB/s", value=gbs, unit="GB/s", dtype="f16",
                    ms_per_step=statistics.median(t), config={"workload": "bias + tanh-GELU 16384x3072 fp16"},
                    roofline={"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                              "peak_source": f"{src} copy", "same_size_copy_gbs": cp,
                              "frac_of_same_size_copy": gbs / cp})
    elif workload == "softmax":
        g = torch.Generator().manual_seed(5)
        x = (2.0 * torch.randn(49152, 512, generator=g)).half().to(device)
        n = _rotations(2 * x.numel() * 2)
        sets = [(x.clone(), torch.empty_like(x)) for _ in range(n)]
        t = _time_steps([lambda s=s_: ops.softmax(s[0], out=s[1]) for s_ in sets], args.steps, args.warmup, flush)
        nbytes = 2.0 * 49152 * 512 * 2
        gbs = nbytes / (statistics.median(t) * 1e-3) / 1e9
        cp = _same_size_copy_gbs(49152 * 512 * 2, args.steps, args.warmup, flush, device)
        line.update(metric="softmax 49152x512 fp16 GB/s", value=gbs, unit="GB/s", dtype="f16",
                    ms_per_step=statistics.median(t),
                    config={"workload": "row softmax 49152x512 fp16 (B8 H12 S512 attention scores)"},
                    roofline={"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                              "peak_source": f"{src} copy", "same_size_copy_gbs": cp,
                              "frac_of_same_size_copy": gbs / cp})
    elif workload == "qkv_split":
        from lunara_b200.runtime import _lib
        lib = _lib.load()
        g = torch.Generator().manual_seed(6)
        B, S, H, D = 8, 512, 12, 64
        qkv = torch.randn(B, S, 3 * H * D, generator=g).half().to(device)
        n = _rotations(2 * qkv.numel() * 2)
        sets = [(qkv.clone(), *(torch.empty(B, H, S, D, dtype=torch.half, device=device) for _ in range(3)))
                for _ in range(n)]
        def split(s):
            _lib.check(lib.lunara_qkv_split(s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), s[3].data_ptr(),
                                            B, S, H, D, 2, torch.cuda.current_stream().cuda_stream))
        t = _time_steps([lambda s=s_: split(s) for s_ in sets], args.steps, args.warmup, flush)
        nbytes = 2.0 * qkv.numel() * 2
        gbs = nbytes / (statistics.median(t) * 1e-3) / 1e9
        cp = _same_size_copy_gbs(qkv.numel() * 2, args.steps, args.warmup, flush, device)
        line.update(metric="QKV split [8,512,2304] -> 3x[8,12,512,64] fp16 GB/s", value=gbs, unit="GB/s", dtype="f16",
                    ms_per_step=statistics.median(t),
                    config={"workload": "QKV split + head reshape, B8 S512 H12 D64 fp16 (bit-exact copy)"},
                    roofline={"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                              "peak_source": f"{src} copy", "same_size_copy_gbs": cp,
                              "frac_of_same_size_copy": gbs / cp})
    elif workload == "stack":
        from lunara_b200.runtime.encoder import EncoderStack
        per_rank = 64 // world
        x, ws = inputs.stack_inputs(batch=64, seq=512, layers=12, seed=4)
        xs = x[rank * per_rank:(rank + 1) * per_rank]
        st = EncoderStack(ws, batch=per_rank, seq=512, num_heads=12, device=device)
        st.x.copy_(xs.half().reshape(-1, 768).to(device))
        t = _time_steps([st.run_kernels], args.steps, args.warmup, flush)
        total = sum(t)
        if world > 1:
            import torch.distributed as dist
            tt = torch.tensor([total], dtype=torch.float64, device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            total = float(tt.item())
        tokens = 64 * 512 * args.steps
        val = tokens / (total * 1e-3)
        flops = 12 * 8 * 64.42e9 * args.steps
        ach = flops / (total * 1e-3) / 1e12
        line.update(metric="12-layer encoder stack tokens/s (B64,S512,H768)", value=val, unit="tokens/s",
                    dtype="f16", scaling="strong", ms_per_step=total / args.steps,
                    config={"workload": "12-layer encoder stack B64 S512 fp16", "global_batch": 64,
                            "per_rank_batch": per_rank, "parallelism": f"batch-sharded x{world}"},
                    roofline={"bound": "tensor", "achieved": ach, "peak": tflops_peak * world,
                              "unit": "TFLOP/s", "frac": ach / (tflops_peak * world),
                              "peak_source": f"{src} bf16 burst x {world} GPUs"})
    elif workload == "tp_ffn":
        line.update(_tp_ffn(args, rank, world, device, tflops_peak, src))
    else:
        raise ValueError(workload)
    return line


def _tp_ffn(args, rank, world, device, tflops_peak, src):
    """One tensor-parallel encoder layer over B64 S512 (32768 tokens): attention
    replicated on every rank, FFN W1 column-split / W2 row-split over ``world``
    ranks, one NCCL all-reduce (sum) of the [32768, 768] fp16 partials per layer.

    Eager launches (every kernel here runs for tens of microseconds or more, so
    host launch cost stays hidden); CUDA events around ``steps`` layers after a
    barrier, max over ranks. Working set (x 50 MB, QKV 151 MB, ...) exceeds L2.
    The all-reduce alone is timed the same way for its bus bandwidth.
    """
    import torch.distributed as dist
    from oracle import inputs
    from lunara_b200.runtime.sharding import TPEncoderBlock
    x, ws = inputs.stack_inputs(batch=64, seq=512, layers=1, seed=4)
    allreduce = None if world > 1 else (lambda t: None)
    blk = TPEncoderBlock(ws[0], batch=64, seq=512, num_heads=12, world=world, rank=rank, device=device,
                         allreduce=allreduce)
    blk.x.copy_(x.half().reshape(-1, 768).to(device))
    stream = torch.cuda.current_stream()

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(steps):
            fn()
        e.record(stream)
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
        if world > 1:
            tt = torch.tensor([ms], dtype=torch.float64, device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        return ms / steps

    steps = min(args.steps, 200)
    layer_ms = timed(blk.run_kernels, steps)
    ar_ms = timed(lambda: blk.allreduce(blk.g), steps) if world > 1 else 0.0
    tokens = 64 * 512
    ffn_flops = 2.0 * 2 * tokens * 768 * 3072
    rank_flops = 8 * (64.42e9 - 38.66e9) + ffn_flops / world   # replicated attention part + FFN shard
    ach = rank_flops / (layer_ms * 1e-3) / 1e12
    ar_bytes = tokens * 768 * 2
    bus = (2.0 * (world - 1) / world * ar_bytes / (ar_ms * 1e-3) / 1e9) if world > 1 else None
    return dict(metric="tensor-parallel FFN encoder layer tokens/s (B64,S512,H768)",
                value=tokens / (layer_ms * 1e-3), unit="tokens/s", dtype="f16", scaling="strong",
                ms_per_step=layer_ms, steps=steps,
                config={"workload": "encoder layer B64 S512 fp16, FFN split over ranks, NCCL all-reduce",
                        "global_batch": 64, "parallelism": f"tp-ffn x{world}", "l2": "working set > L2"},
                allreduce={"ms": ar_ms, "bytes": ar_bytes, "bus_gbs": bus,
                           "share_of_layer": (ar_ms / layer_ms) if world > 1 else 0.0},
                roofline={"bound": "tensor", "achieved": ach, "peak": tflops_peak, "unit": "TFLOP/s per rank",
                          "frac": ach / tflops_peak, "peak_source": f"{src} bf16 burst"})
