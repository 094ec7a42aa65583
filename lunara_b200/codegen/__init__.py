"""Codegen: KernelSpec -> launcher modules over the sm_100a C ABI, and the autotuner."""

from lunara_b200.codegen.autotuner import Autotuner, TuningCache, TuningResult
from lunara_b200.codegen.kernel_emitter import (
    KernelEmitter, KernelKind, KernelSpec, TileConfig, TritonEmitter, emit_attention, emit_elementwise, emit_gemm,
    emit_layernorm, emit_softmax, emit_transformer_block,
)

__all__ = [
    "KernelKind", "KernelSpec", "TileConfig", "TritonEmitter", "KernelEmitter",
    "emit_gemm", "emit_attention", "emit_softmax", "emit_layernorm",
    "emit_elementwise", "emit_transformer_block",
    "Autotuner", "TuningResult", "TuningCache",
]
