"""Import-path alias of ``lunara_b200.codegen.kernel_emitter``.

The reference keeps its emitter at ``lunara/codegen/triton_emitter.py``; code
written against that module path keeps working. Nothing here uses Triton.
"""
from lunara_b200.codegen.kernel_emitter import (  # noqa: F401
    _ELTWISE_BODIES, KernelEmitter, KernelKind, KernelSpec, TileConfig, TritonEmitter, emit_attention,
    emit_elementwise, emit_gemm, emit_layernorm, emit_softmax, emit_transformer_block, gemm_block_n,
    transformer_block_specs,
)
