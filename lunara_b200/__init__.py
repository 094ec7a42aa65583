"""lunara_b200 -- B200 (sm_100a) kernel backend for Lunara's kernel kinds.

Public API (same names as the reference package ``lunara``):

    from lunara_b200 import Compiler, KernelSpec, KernelKind, TileConfig
    from lunara_b200.profiler import NsightProfiler
    from lunara_b200.codegen import Autotuner

The kernels (tcgen05 GEMM and attention, vectorised LayerNorm / Softmax /
elementwise / index kernels) live in ``liblunara_b200.so`` behind the C ABI of
``include/lunara_b200.h``; ``lunara_b200.runtime.ops`` is the torch-facing
layer over it and ``lunara_b200.runtime.encoder`` runs the encoder block.
"""

__version__ = "0.1.0"
__license__ = "Apache-2.0"

from lunara_b200.codegen.autotuner import Autotuner, TuningResult
from lunara_b200.codegen.kernel_emitter import (
    KernelEmitter, KernelKind, KernelSpec, TileConfig, TritonEmitter, emit_transformer_block,
)
from lunara_b200.driver import CompiledModel, Compiler
from lunara_b200.profiler.nsight_profiler import GPUSpec, KernelMetrics, NsightProfiler, ProfileResult, detect_gpu

__all__ = [
    "Compiler", "CompiledModel",
    "KernelKind", "KernelSpec", "TileConfig", "TritonEmitter", "KernelEmitter",
    "emit_transformer_block",
    "Autotuner", "TuningResult",
    "NsightProfiler", "ProfileResult", "KernelMetrics", "GPUSpec",
    "detect_gpu",
]
