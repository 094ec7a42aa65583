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
    cloudpickle into a launcher script, which is first run once without ncu
    (a call that fails there is never profiled) and then under ncu with
    ``--clock-control none``, a kernel filter and a launch count (the
    reference's launcher is a placeholder, 250-257); the CSV is parsed per
    kernel;
  * memory-bound kernels are graded on read + write bytes, and the report and
    the roofline chart show each kernel against both roofs (HBM and tensor).

``python -m lunara_b200.profiler.nsight_profiler --selfcheck`` profiles one
small GEMM launch through the ncu path and compares its duration with the
CUDA-event timing of the same launch.
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


# Where each GPU's peak figures come from, for the report ("measured" or "datasheet").
PEAK_SOURCE: Dict[str, str] = {}


def _b200_spec() -> GPUSpec:
    """B200: measured peaks when MEASURED_PEAKS.json exists, else datasheet dense figures."""
    fp16, hbm, src = 2250.0, 7.7, "datasheet"
    for cand in (Path(os.environ.get("LUNARA_PEAKS", "")), Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"):
        if cand.is_file():
            try:
                d = json.loads(cand.read_text())
                fp16, hbm, src = float(d["bf16_tflops"]), float(d["hbm_gbs"]) / 1000.0, "measured"
            except (KeyError, ValueError):
                pass
            break
    PEAK_SOURCE["B200"] = src
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
    """Memory- or compute-bound by arithmetic intensity vs the ridge point (nsight_profiler.py:161-171).

    A memory-bound kernel is graded on every byte it moves: read plus write
    bandwidth against the HBM peak (a copy-like kernel writes as much as it reads).
    """
    if flops is None or bytes_accessed is None or bytes_accessed <= 0:
        return
    m.arithmetic_intensity = flops / bytes_accessed
    ridge = gpu.peak_flops_fp16 / gpu.peak_bw_hbm   # FLOP per byte (TFLOPS / TB/s)
    if m.arithmetic_intensity < ridge:
        m.roofline_bound = "memory"
        m.roofline_efficiency = (m.hbm_read_bw_gbs + m.hbm_write_bw_gbs) / (gpu.peak_bw_hbm * 1000)
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
            # Event timing sees no counters: the algorithmic bytes (reads and
            # writes together) are reported as the read figure, the write figure stays 0.
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
                 kernel_regex: Optional[str] = None, warmup: int = 1, metrics: Optional[List[str]] = None):
        self.ncu_path = ncu_path
        self.fallback = fallback_to_events
        self.launch_count = launch_count
        self.kernel_regex = kernel_regex
        self.warmup = warmup
        self.metrics = list(metrics) if metrics else list(_NCU_METRICS)
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
               "--metrics", ",".join(self.metrics), "--launch-skip", str(self.warmup),
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
            # The same launcher runs once without ncu first: a call that fails (or
            # faults) there is reported as an error and never profiled.
            subprocess.run([sys.executable, str(launcher)], check=True, capture_output=True, timeout=300)
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
        """One table row per kernel: time, achieved TFLOP/s and HBM GB/s, each as a
        fraction of its roof, and the roof that bounds the kernel."""
        g = result.gpu_spec
        rows = []
        for k in sorted(result.kernels, key=lambda k: -k.duration_us):
            hbm = k.hbm_read_bw_gbs + k.hbm_write_bw_gbs
            tc_frac = k.achieved_flops_t / g.peak_flops_fp16 if g and g.peak_flops_fp16 else 0.0
            bw_frac = hbm / (g.peak_bw_hbm * 1000.0) if g and g.peak_bw_hbm else 0.0
            name = k.kernel_name if len(k.kernel_name) <= 34 else k.kernel_name[:31] + "..."
            rows.append((name, f"{k.duration_us:.2f}", f"{k.achieved_flops_t:.1f}", f"{tc_frac:.2f}",
                         f"{hbm:.0f}", f"{bw_frac:.2f}", f"{k.arithmetic_intensity:.1f}", k.roofline_bound))
        head = ("kernel", "us", "TFLOP/s", "x tensor", "GB/s", "x HBM", "FLOP/B", "bound")
        widths = [max(len(r[i]) for r in rows + [head]) for i in range(len(head))]
        src = PEAK_SOURCE.get(g.name, "datasheet") if g else "-"
        print(f"\nLunara Profile Summary -- {g.name if g else 'unknown GPU'}")
        if g:
            print(f"roofs ({src}): tensor {g.peak_flops_fp16:.0f} TFLOP/s, HBM {g.peak_bw_hbm * 1000:.0f} GB/s, "
                  f"ridge {g.peak_flops_fp16 / g.peak_bw_hbm:.0f} FLOP/B")
        line = "  ".join(h.rjust(w) if i else h.ljust(w) for i, (h, w) in enumerate(zip(head, widths)))
        print(line)
        print("-" * len(line))
        for r in rows:
            print("  ".join(c.rjust(w) if i else c.ljust(w) for i, (c, w) in enumerate(zip(r, widths))))
        print(f"total {result.total_duration_us:.2f} us over {len(result.kernels)} kernel launch(es)\n")

    def plot_roofline(self, result: ProfileResult, output_path: str = "roofline.png") -> None:
        """Log-log roofline: the HBM roof (bandwidth x intensity) and the tensor roof,
        the ridge between them, and one marker per kernel at (intensity, achieved);
        skipped with a message when matplotlib is absent."""
        try:
            import matplotlib
            matplotlib.use("Agg")
            import matplotlib.pyplot as plt
        except ImportError:
            print("[profiler] matplotlib not available; skipping roofline plot")
            return
        g = result.gpu_spec
        if g is None:
            return
        bw_gflops_per_flop_b = g.peak_bw_hbm * 1000.0          # GB/s = GFLOP/s per (FLOP/B)
        tensor_gflops = g.peak_flops_fp16 * 1000.0
        ridge = tensor_gflops / bw_gflops_per_flop_b
        pts = [k for k in result.kernels if k.arithmetic_intensity > 0]
        lo = min([ridge / 64] + [k.arithmetic_intensity / 2 for k in pts])
        hi = max([ridge * 64] + [k.arithmetic_intensity * 2 for k in pts])
        fig, ax = plt.subplots(figsize=(9, 5.5))
        ax.loglog([lo, ridge], [bw_gflops_per_flop_b * lo, tensor_gflops], color="tab:blue",
                  label=f"HBM roof {g.peak_bw_hbm * 1000:.0f} GB/s")
        ax.loglog([ridge, hi], [tensor_gflops, tensor_gflops], color="tab:red",
                  label=f"tensor roof {g.peak_flops_fp16:.0f} TFLOP/s")
        ax.axvline(ridge, color="gray", linestyle=":", linewidth=1)
        for k in pts:
            y = k.achieved_flops_t * 1000.0 if k.achieved_flops_t > 0 else \
                (k.hbm_read_bw_gbs + k.hbm_write_bw_gbs) * k.arithmetic_intensity
            ax.scatter([k.arithmetic_intensity], [y], zorder=3)
            ax.annotate(f"{k.kernel_name[:24]} {k.roofline_efficiency:.0%}", (k.arithmetic_intensity, y),
                        textcoords="offset points", xytext=(5, -12), fontsize=8)
        ax.set_xlabel("FLOP per DRAM byte")
        ax.set_ylabel("GFLOP/s")
        ax.set_title(f"{g.name}: kernels against the HBM and tensor roofs ({PEAK_SOURCE.get(g.name, 'datasheet')})")
        ax.legend(loc="upper left")
        fig.tight_layout()
        fig.savefig(output_path, dpi=130)
        plt.close(fig)
        print(f"[profiler] roofline chart written to {output_path}")


def ncu_available(path: str = "ncu") -> bool:
    return shutil.which(path) is not None


def _selfcheck() -> int:
    """Profile one 2048^3 fp16 GEMM launch through the ncu path (duration and DRAM
    bytes only) and compare its duration with CUDA-event timing of the same call.
    Prints one JSON line; exit status 0 when the two agree within 2x."""
    import torch as _torch
    from lunara_b200.runtime import ops
    n = 2048
    a = _torch.randn(n, n, dtype=_torch.float16, device="cuda")
    b = _torch.randn(n, n, dtype=_torch.float16, device="cuda")
    c = _torch.empty(n, n, dtype=_torch.float16, device="cuda")
    flops, nbytes = 2.0 * n ** 3, 3.0 * n * n * 2
    prof = NsightProfiler(fallback_to_events=False, launch_count=1, kernel_regex="gemm_tc", warmup=2,
                          metrics=["gpu__time_duration.sum", "dram__bytes_read.sum", "dram__bytes_write.sum"])
    ncu_res = prof.profile_kernel(ops.gemm, (a, b, c), {}, flops=flops, bytes_accessed=nbytes, kernel_name="gemm")
    ev = CUDAEventProfiler(n_warmup=3, n_trials=20).profile(lambda: ops.gemm(a, b, c), flops, nbytes)
    k = ncu_res.primary
    out = {"ncu_kernels": len(ncu_res.kernels), "ncu_kernel": k.kernel_name if k else None,
           "ncu_duration_us": k.duration_us if k else None, "event_duration_us": ev.duration_us,
           "ncu_dram_read_bytes": k.raw_metrics.get("dram__bytes_read.sum") if k else None,
           "ncu_dram_write_bytes": k.raw_metrics.get("dram__bytes_write.sum") if k else None,
           "ratio": (k.duration_us / ev.duration_us) if k and ev.duration_us else None}
    print(json.dumps(out))
    if k is not None:
        NsightProfiler.print_summary(ncu_res)
    return 0 if out["ratio"] is not None and 0.5 <= out["ratio"] <= 2.0 else 1


if __name__ == "__main__":
    if "--selfcheck" in sys.argv:
        sys.exit(_selfcheck())
    print("usage: python -m lunara_b200.profiler.nsight_profiler --selfcheck")
