"""Profiler: ncu integration, CUDA-event timing and roofline analysis."""

from lunara_b200.profiler.nsight_profiler import (
    GPU_SPECS, CUDAEventProfiler, GPUSpec, KernelMetrics, NsightProfiler, ProfileResult, detect_gpu,
)

__all__ = ["NsightProfiler", "CUDAEventProfiler", "ProfileResult", "KernelMetrics", "GPUSpec", "GPU_SPECS",
           "detect_gpu"]
