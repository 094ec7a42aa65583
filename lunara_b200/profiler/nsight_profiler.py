"""Profiler and roofline API: the drop-in counterpart of lunara/profiler/nsight_profiler.py.

Same public names and shapes (``GPUSpec``, ``GPU_SPECS``, ``detect_gpu``,
``KernelMetrics``, ``ProfileResult``, ``CUDAEventProfiler``, ``NsightProfiler``;
nsight_profiler.py:36-379) with three changes:

  * a ``B200`` entry; its peaks are the measured copy bandwidth and bf16 GEMM
    throughput of this machine pool when ``MEASURED_PEAKS.json`` is present,
    otherwise the datasheet figures (7.7 TB/s HBM3e, 2250 TFLOP/s dense fp16);
  * the event profiler can flush L2 (a 256 MB write) between timed calls, so a
    working set that fits in the 126 MB L2 does not inflate HBM figures;
  * the ncu path really profiles the callable: it is serialised with
    cloudpickle into a launcher script that ncu runs with ``--clock-control
    none`` (the reference's launcher is a placeholder, 250-257), and the CSV
    is parsed per kernel.
"""
from __future__ import annotations

import csv
import io
import json
import os
import shutil
import subprocess
import sys
import tempfile
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Dict, List, Optional, Tuple

import torch


@dataclass
class GPUSpec:
    name: str
    peak_flops_fp16: float   # TFLOPS (dense tensor core)
    peak_flops_fp32: float   # TFLOPS
    peak_bw_hbm: float       # TB/s
    peak_bw_l2: float        # TB/s
    num_sms: int
    shared_mem_per_sm: int   # bytes


def _b200_spec() -> GPUSpec:
    """B200: measured peaks when MEASURED_PEAKS.json exists, else datasheet dense figures."""
    fp16, hbm = 2250.0, 7.7
    for cand in (Path(os.environ.get("LUNARA_PEAKS", "")), Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"):
        if cand.is_file():
            try:
                d = json.loads(cand.read_text())
                fp16, hbm = float(d["bf16_tflops"]), float(d["hbm_gbs"]) / 1000.0
            except (KeyError, ValueError):
                pass
            break
    return GPUSpec("B200", fp16, 80.0, hbm, 20.0, 148, 228 * 1024)


GPU_SPECS: Dict[str, GPUSpec] = {
    "A100": GPUSpec("A100", 312.0, 19.5, 2.0, 12.0, 108, 164 * 1024),
    "A10G": GPUSpec("A10G", 125.0, 31.2, 0.6, 4.0, 80, 100 * 1024),
    "V100": GPUSpec("V100", 125.0, 14.1, 0.9, 3.1, 80, 96 * 1024),
    "H100": GPUSpec("H100", 989.0, 51.2, 3.35, 33.0, 132, 228 * 1024),
    "RTX4090": GPUSpec("RTX4090", 330.0, 82.6, 1.008, 8.0, 128, 100 * 1024),
    "B200": _b200_spec(),
}


def detect_gpu() -> GPUSpec:
    name = torch.cuda.get_device_name(0) if torch.cuda.is_available() else ""
    for key in GPU_SPECS:
        if key in name:
            return GPU_SPECS[key]
    props = torch.cuda.get_device_properties(0) if torch.cuda.is_available() else None
    if props:
        clock_ghz = getattr(props, "clock_rate", 1_500_000) * 1e-6
        return GPUSpec(name=props.name,
                       peak_flops_fp16=float(props.multi_processor_count) * 128 * 2 * clock_ghz * 1e-3,
                       peak_flops_fp32=float(props.multi_processor_count) * 64 * 2 * clock_ghz * 1e-3,
                       peak_bw_hbm=0.9, peak_bw_l2=4.0, num_sms=props.multi_processor_count,
                       shared_mem_per_sm=props.shared_memory_per_multiprocessor)
    return GPU_SPECS["B200"]


@dataclass
class KernelMetrics:
    kernel_name: str = ""
    duration_us: float = 0.0
    sm_active_pct: float = 0.0
    achieved_occupancy: float = 0.0
    warp_efficiency: float = 0.0
    hbm_read_bw_gbs: float = 0.0
    hbm_write_bw_gbs: float = 0.0
    l2_read_bw_gbs: float = 0.0
    l2_write_bw_gbs: float = 0.0
    l1_hit_rate: float = 0.0
    achieved_flops_t: float = 0.0
    arithmetic_intensity: float = 0.0
    roofline_bound: str = "unknown"
    roofline_efficiency: float = 0.0
    raw_metrics: Dict[str, str] = field(default_factory=dict)


@dataclass
class ProfileResult:
    kernels: List[KernelMetrics] = field(default_factory=list)
    gpu_spec: Optional[GPUSpec] = None
    total_duration_us: float = 0.0

    @property
    def primary(self) -> Optional[KernelMetrics]:
        """The kernel with the longest duration."""
        if not self.kernels:
            return None
        return max(self.kernels, key=lambda k: k.duration_us)


def classify_roofline(m: KernelMetrics, flops: Optional[float], bytes_accessed: Optional[float],
                      gpu: GPUSpec) -> None:
    """Memory- or compute-bound by arithmetic intensity vs the ridge point (nsight_profiler.py:161-171)."""
    if flops is None or bytes_accessed is None or bytes_accessed <= 0:
        return
    m.arithmetic_intensity = flops / bytes_accessed
    ridge = gpu.peak_flops_fp16 / gpu.peak_bw_hbm   # FLOP per byte (TFLOPS / TB/s)
    if m.arithmetic_intensity < ridge:
        m.roofline_bound = "memory"
        m.roofline_efficiency = m.hbm_read_bw_gbs / (gpu.peak_bw_hbm * 1000)
    else:
        m.roofline_bound = "compute"
        m.roofline_efficiency = m.achieved_flops_t / gpu.peak_flops_fp16


class CUDAEventProfiler:
    """Latency by CUDA events (median), optional L2 flush between calls; no ncu needed."""

    def __init__(self, n_warmup: int = 5, n_trials: int = 20, flush_l2: bool = True):
        self.n_warmup = n_warmup
        self.n_trials = n_trials
        self.flush_l2 = flush_l2
        self._flush = None

    def _do_flush(self):
        if self.flush_l2:
            if self._flush is None:
                self._flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
            self._flush.zero_()

    def profile(self, fn: Callable, flops: Optional[float] = None, bytes_accessed: Optional[float] = None,
                gpu_spec: Optional[GPUSpec] = None) -> KernelMetrics:
        gpu_spec = gpu_spec or detect_gpu()
        for _ in range(self.n_warmup):
            fn()
        torch.cuda.synchronize()
        times_us = []
        for _ in range(self.n_trials):
            self._do_flush()
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            times_us.append(s.elapsed_time(e) * 1000)
        times_us.sort()
        med = times_us[len(times_us) // 2]
        m = KernelMetrics(duration_us=med)
        if flops is not None:
            m.achieved_flops_t = flops / (med * 1e-6) / 1e12
        if bytes_accessed is not None and med > 0:
            m.hbm_read_bw_gbs = bytes_accessed / (med * 1e-6) / 1e9
        classify_roofline(m, flops, bytes_accessed, gpu_spec)
        return m


_NCU_METRICS = [
    "gpu__time_duration.sum",
    "sm__cycles_active.avg.pct_of_peak_sustained_elapsed",
    "sm__warps_active.avg.pct_of_peak_sustained_active",
    "smsp__warps_eligible.avg.pct_of_peak_sustained_active",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "dram__throughput.avg.pct_of_peak_sustained_elapsed",
    "lts__t_sectors_srcunit_tex_op_read.sum",
    "lts__t_sectors_srcunit_tex_op_write.sum",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
]

_LAUNCHER = """\
import sys, cloudpickle, torch
sys.path[:0] = {paths!r}
with open({blob!r}, "rb") as f:
    fn, args, kwargs, warmup = cloudpickle.load(f)
for _ in range(warmup):
    fn(*args, **kwargs)
torch.cuda.synchronize()
fn(*args, **kwargs)
torch.cuda.synchronize()
"""


class NsightProfiler:
    """Profile a callable with ncu (per-kernel metrics) or, without ncu, with CUDA events."""

    def __init__(self, ncu_path: str = "ncu", fallback_to_events: bool = True, launch_count: int = 8,
                 kernel_regex: Optional[str] = None, warmup: int = 1):
        self.ncu_path = ncu_path
        self.fallback = fallback_to_events
        self.launch_count = launch_count
        self.kernel_regex = kernel_regex
        self.warmup = warmup
        self._has_ncu = self._check_ncu()
        self.gpu_spec = detect_gpu()
        self._event_profiler = CUDAEventProfiler()
        if not self._has_ncu:
            print("[profiler] ncu not found; using CUDA event profiler")

    def _check_ncu(self) -> bool:
        try:
            subprocess.run([self.ncu_path, "--version"], capture_output=True, check=True)
            return True
        except (subprocess.CalledProcessError, FileNotFoundError, OSError):
            return False

    def profile_kernel(self, fn: Callable, args: Tuple = (), kwargs: Optional[Dict] = None,
                       flops: Optional[float] = None, bytes_accessed: Optional[float] = None,
                       kernel_name: str = "kernel") -> ProfileResult:
        kwargs = kwargs or {}
        if self._has_ncu and torch.cuda.is_available():
            try:
                return self._profile_with_ncu(fn, args, kwargs, kernel_name, flops, bytes_accessed)
            except Exception as e:
                if not self.fallback:
                    raise
                print(f"[profiler] ncu profiling failed ({e}); using CUDA events")
        m = self._event_profiler.profile(lambda: fn(*args, **kwargs), flops, bytes_accessed, self.gpu_spec)
        m.kernel_name = kernel_name
        return ProfileResult(kernels=[m], gpu_spec=self.gpu_spec, total_duration_us=m.duration_us)

    def ncu_command(self, launcher: Path, csv_out: Path) -> List[str]:
        cmd = [self.ncu_path, "--clock-control", "none", "--csv", "--page", "raw",
               "--metrics", ",".join(_NCU_METRICS), "--launch-skip", str(self.warmup),
               "--launch-count", str(self.launch_count), "--log-file", str(csv_out)]
        if self.kernel_regex:
            cmd += ["--kernel-name", f"regex:{self.kernel_regex}"]
        return cmd + [sys.executable, str(launcher)]

    def _profile_with_ncu(self, fn, args, kwargs, kernel_name, flops, bytes_accessed) -> ProfileResult:
        import cloudpickle
        with tempfile.TemporaryDirectory() as tmp:
            blob = Path(tmp) / "call.pkl"
            with open(blob, "wb") as f:
                cloudpickle.dump((fn, args, kwargs, self.warmup), f)
            launcher = Path(tmp) / "launch.py"
            launcher.write_text(_LAUNCHER.format(paths=[p for p in sys.path if p], blob=str(blob)))
            csv_out = Path(tmp) / "metrics.csv"
            subprocess.run(self.ncu_command(launcher, csv_out), check=True, capture_output=True, timeout=600)
            return self._parse_ncu_csv(csv_out, kernel_name, flops, bytes_accessed)

    def _parse_ncu_csv(self, csv_path: Path, name: str, flops: Optional[float] = None,
                       bytes_accessed: Optional[float] = None) -> ProfileResult:
        """Parse `ncu --csv --page raw` output: one row per kernel launch, one column per metric."""
        result = ProfileResult(gpu_spec=self.gpu_spec)
        if not csv_path.exists():
            return result
        text = "\n".join(ln for ln in csv_path.read_text().splitlines() if ln.startswith('"'))
        rows = list(csv.reader(io.StringIO(text)))
        if len(rows) < 2:
            return result
        header, body = rows[0], rows[1:]
        if body and body[0] and body[0][0] == "":   # units row
            body = body[1:]
        col = {h: i for i, h in enumerate(header)}

        def val(r, key, default=0.0):
            i = col.get(key)
            if i is None or i >= len(r):
                return default
            try:
                return float(r[i].replace(",", ""))
            except ValueError:
                return default
        for r in body:
            m = KernelMetrics(kernel_name=r[col["Kernel Name"]] if "Kernel Name" in col else name)
            m.raw_metrics = {h: r[i] for h, i in col.items() if i < len(r)}
            m.duration_us = val(r, "gpu__time_duration.sum") / 1000.0   # ns -> us
            m.sm_active_pct = val(r, "sm__cycles_active.avg.pct_of_peak_sustained_elapsed")
            m.achieved_occupancy = val(r, "sm__warps_active.avg.pct_of_peak_sustained_active") / 100.0
            m.warp_efficiency = val(r, "smsp__warps_eligible.avg.pct_of_peak_sustained_active") / 100.0
            if m.duration_us > 0:
                m.hbm_read_bw_gbs = val(r, "dram__bytes_read.sum") / (m.duration_us * 1e-6) / 1e9
                m.hbm_write_bw_gbs = val(r, "dram__bytes_write.sum") / (m.duration_us * 1e-6) / 1e9
                if flops is not None:
                    m.achieved_flops_t = flops / (m.duration_us * 1e-6) / 1e12
            classify_roofline(m, flops, bytes_accessed, self.gpu_spec)
            result.kernels.append(m)
        result.total_duration_us = sum(k.duration_us for k in result.kernels)
        return result

    @staticmethod
    def print_summary(result: ProfileResult) -> None:
        sep = "─" * 60
        print(f"\n{sep}")
        print("  Lunara Kernel Profile Summary")
        print(sep)
        if result.gpu_spec:
            g = result.gpu_spec
            print(f"  GPU:  {g.name}  |  FP16 peak: {g.peak_flops_fp16:.0f} TFLOPS  |  HBM BW: {g.peak_bw_hbm:.1f} TB/s")
        print()
        for k in result.kernels:
            print(f"  Kernel: {k.kernel_name}")
            print(f"    Duration:    {k.duration_us:>10.2f} µs")
            print(f"    SM util:     {k.sm_active_pct:>9.1f}%")
            print(f"    Occupancy:   {k.achieved_occupancy * 100:>9.1f}%")
            print(f"    HBM read BW: {k.hbm_read_bw_gbs:>9.1f} GB/s")
            print(f"    Achieved:    {k.achieved_flops_t:>9.2f} TFLOPS")
            print(f"    Arith. Int.: {k.arithmetic_intensity:>9.2f} FLOP/B")
            print(f"    Roofline:    {k.roofline_bound:>9s} ({k.roofline_efficiency * 100:.1f}% of peak)")
        print(sep + "\n")

    def plot_roofline(self, result: ProfileResult, output_path: str = "roofline.png") -> None:
        """Roofline chart with matplotlib; skipped (with a message) when matplotlib is absent."""
        try:
            import matplotlib.pyplot as plt
            import numpy as np
        except ImportError:
            print("[profiler] matplotlib not available; skipping roofline plot")
            return
        if not result.gpu_spec:
            return
        g = result.gpu_spec
        fig, ax = plt.subplots(figsize=(10, 6))
        ax.set_xscale("log", base=2)
        ax.set_yscale("log", base=2)
        ai = np.logspace(-2, 10, 500, base=2)
        ax.plot(ai, np.minimum(g.peak_bw_hbm * 1000 * ai, np.full_like(ai, g.peak_flops_fp16 * 1000)), "k-",
                linewidth=2.5, label="Roofline (FP16 TC)")
        for k in result.kernels:
            if k.arithmetic_intensity > 0 and k.achieved_flops_t > 0:
                ax.scatter(k.arithmetic_intensity, k.achieved_flops_t * 1000, s=120, zorder=5,
                           label=f"{k.kernel_name} ({k.achieved_flops_t:.1f}T, {k.roofline_efficiency * 100:.0f}%)")
        ax.set_xlabel("Arithmetic Intensity (FLOP/byte)")
        ax.set_ylabel("Performance (GFLOPS)")
        ax.set_title(f"Roofline Model — {g.name}")
        ax.legend(loc="lower right")
        ax.grid(True, which="both", alpha=0.3)
        plt.tight_layout()
        plt.savefig(output_path, dpi=150)
        plt.close(fig)
        print(f"[profiler] Roofline saved → {output_path}")


def ncu_available(path: str = "ncu") -> bool:
    return shutil.which(path) is not None
