"""Compiler driver: the drop-in counterpart of lunara/driver.py.

    from lunara_b200 import Compiler
    compiler = Compiler(opt_level=2, dtype="float16")
    compiled = compiler.compile_transformer(768, 12, 512)
    compiled.benchmark(batch_size=8, seq_len=512)
    compiled.save("bert_kernels/")

``Compiler`` and ``CompiledModel`` keep the reference's constructor arguments,
fields, methods, return types and failure behaviour (lunara/driver.py:41-259):
``compile`` runs the external ``lunara-opt`` tool when it is installed and
otherwise warns and continues, the kernel specs come from
``_default_transformer_specs`` (driver.py:208-216, 266-283), the emitted
module is loaded with ``load_kernels``, ``get_launch_fn`` raises ``KeyError``,
and ``benchmark`` returns ``{kernel_name: latency_ms}`` with NaN for kernels
that fail. The emitted kernels call the sm_100a C ABI instead of Triton; the
default ``gpu_arch`` is ``sm_100a``.
"""
from __future__ import annotations

import shutil
import statistics
import subprocess
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, List, Optional

import torch

from lunara_b200.codegen.autotuner import Autotuner, TuningResult
from lunara_b200.codegen.kernel_emitter import (
    KernelEmitter, KernelKind, KernelSpec, TileConfig, emit_transformer_block, transformer_block_specs,
)
from lunara_b200.profiler.nsight_profiler import NsightProfiler


@dataclass
class CompiledModel:
    name: str
    kernel_module: Path
    mlir_path: Optional[Path]
    kernel_specs: List[KernelSpec] = field(default_factory=list)
    tuning_results: Dict[str, TuningResult] = field(default_factory=dict)
    _ns: dict = field(default_factory=dict, repr=False)

    def load_kernels(self) -> None:
        """exec() the generated launcher module to make kernels callable."""
        src = self.kernel_module.read_text()
        exec(compile(src, str(self.kernel_module), "exec"), self._ns)
        self._apply_tuning()

    def _apply_tuning(self) -> None:
        # Tuned GEMM tiles replace the emitted defaults (same effect as re-emitting).
        from lunara_b200.codegen.autotuner import gemm_call_args
        for name, res in self.tuning_results.items():
            key = f"_TILE_{name}"
            if key in self._ns and res is not None:
                self._ns[key].update(gemm_call_args(res.config))

    def get_launch_fn(self, name: str):
        fn = self._ns.get(f"{name}_launch")
        if fn is None:
            raise KeyError(f"No launch function for kernel '{name}'")
        return fn

    def benchmark(self, batch_size: int = 1, seq_len: int = 512, n_warmup: int = 5,
                  n_trials: int = 20) -> Dict[str, float]:
        """Per-kernel latency in ms (median of CUDA-event timed launches); NaN for failures."""
        results: Dict[str, float] = {}
        for spec in self.kernel_specs:
            try:
                fn = self.get_launch_fn(spec.name)
                inputs = self._make_dummy_inputs(spec, batch_size, seq_len)
                for _ in range(n_warmup):
                    fn(*inputs)
                torch.cuda.synchronize()
                times = []
                for _ in range(n_trials):
                    s = torch.cuda.Event(enable_timing=True)
                    e = torch.cuda.Event(enable_timing=True)
                    s.record()
                    fn(*inputs)
                    e.record()
                    e.synchronize()
                    times.append(s.elapsed_time(e))
                results[spec.name] = statistics.median(times)
            except Exception as e:  # keep the reference's "NaN on failure" contract
                results[spec.name] = float("nan")
                print(f"  [warn] benchmark {spec.name}: {e}")
        return results

    def _make_dummy_inputs(self, spec: KernelSpec, B: int, S: int) -> List[torch.Tensor]:
        """Inputs shaped as the reference's benchmark makes them (lunara/driver.py:88-103)."""
        dtype = getattr(torch, spec.dtype, torch.float16)
        dev = "cuda"
        if spec.kind == KernelKind.GEMM:
            M = B * S
            return [torch.randn(M, 768, dtype=dtype, device=dev),
                    torch.randn(768, 768, dtype=dtype, device=dev),
                    torch.empty(M, 768, dtype=dtype, device=dev)] + \
                   ([torch.zeros(768, dtype=dtype, device=dev)] if spec.has_bias else [])
        if spec.kind == KernelKind.ATTENTION:
            return [torch.randn(B, spec.num_heads, S, spec.tile.HEAD_DIM, dtype=dtype, device=dev)] * 3
        if spec.kind == KernelKind.LAYERNORM:
            return [torch.randn(B * S, 768, dtype=dtype, device=dev),
                    torch.ones(768, dtype=dtype, device=dev),
                    torch.zeros(768, dtype=dtype, device=dev)]
        if spec.kind == KernelKind.SOFTMAX:
            return [torch.randn(B * S, S, dtype=dtype, device=dev)]
        if spec.kind == KernelKind.ELEMENTWISE:
            x = [torch.randn(B * S, 768, dtype=dtype, device=dev)]
            return x + ([torch.zeros(768, dtype=dtype, device=dev)] if spec.has_bias else [])
        return []

    def save(self, directory: str) -> None:
        dst = Path(directory)
        dst.mkdir(parents=True, exist_ok=True)
        shutil.copy(self.kernel_module, dst / self.kernel_module.name)
        if self.mlir_path and self.mlir_path.exists():
            shutil.copy(self.mlir_path, dst / self.mlir_path.name)
        print(f"[lunara] Saved compiled model → {dst}")


class Compiler:
    """End-to-end driver: model -> kernel specs -> sm_100a launcher module.

    opt_level : 0-3, passed to lunara-opt when it is installed
    dtype     : "float16" | "float32" | "bfloat16"
    autotune  : tune GEMM tiles on the device after codegen
    gpu_arch  : target architecture (this backend builds sm_100a only)
    lunara_opt_path : path of the lunara-opt binary (optional)
    """

    def __init__(self, opt_level: int = 2, dtype: str = "float16", autotune: bool = False,
                 gpu_arch: str = "sm_100a", lunara_opt_path: str = "lunara-opt"):
        if gpu_arch not in ("sm_100a", "sm_100"):
            print(f"[warn] gpu_arch {gpu_arch!r} requested; this backend's kernels are built for sm_100a only")
        self.opt_level = opt_level
        self.dtype = dtype
        self.autotune = autotune
        self.gpu_arch = gpu_arch
        self.lunara_opt_path = lunara_opt_path
        self._tuner = Autotuner() if autotune else None
        self._profiler = NsightProfiler(fallback_to_events=True)

    def compile(self, model_path: str, output_dir: Optional[str] = None,
                model_name: Optional[str] = None) -> CompiledModel:
        """Full pipeline; returns a CompiledModel ready to run."""
        model_path = Path(model_path)
        name = model_name or model_path.stem
        out = Path(output_dir or f"lunara_compiled_{name}")
        out.mkdir(parents=True, exist_ok=True)
        print(f"[lunara] Compiling {model_path.name} → {out}/")
        mlir_path = out / "lowered.mlir"
        self._run_lunara_opt(model_path, mlir_path)
        self._model_path = model_path
        specs = self._extract_kernel_specs(mlir_path, name)
        emitter = KernelEmitter(str(out / "kernels"))
        for spec in specs:
            emitter.emit(spec)
        kernel_module = emitter.write_module(name)
        tuning: Dict[str, TuningResult] = {}
        if self.autotune and torch.cuda.is_available():
            tuning = self._autotune(specs)
        compiled = CompiledModel(name=name, kernel_module=kernel_module, mlir_path=mlir_path,
                                 kernel_specs=specs, tuning_results=tuning)
        compiled.load_kernels()
        print(f"[lunara] Compilation complete: {len(specs)} kernels")
        return compiled

    def _run_lunara_opt(self, model_path: Path, mlir_out: Path) -> None:
        """Invoke the external lunara-opt tool when it is installed (its MLIR output is informational)."""
        cmd = [self.lunara_opt_path, str(model_path), "--emit=mlir", f"--opt={self.opt_level}",
               f"--out={mlir_out.parent}"]
        try:
            result = subprocess.run(cmd, capture_output=True, text=True, check=True)
            if result.stdout:
                print(result.stdout)
        except FileNotFoundError:
            print(f"[warn] lunara-opt not found at '{self.lunara_opt_path}'; generating synthetic specs from model name")
        except subprocess.CalledProcessError as e:
            print(f"[warn] lunara-opt failed:\n{e.stderr}")

    def _extract_kernel_specs(self, mlir_path: Path, model_name: str) -> List[KernelSpec]:
        """Kernel specs of the model being compiled.

        The reference returns the canonical encoder-block kernel set here
        whatever the model (driver.py:208-216). This reads the ONNX graph
        itself (lunara_b200.frontend.onnx_graph) and derives the kernel list
        from it; a file that is not a readable ONNX model, or a graph with no
        kernel-producing node, falls back to the canonical block set.
        """
        from lunara_b200.frontend.onnx_graph import OnnxFormatError, graph_kernel_specs, load_onnx
        model_path = getattr(self, "_model_path", None)
        if model_path is not None:
            try:
                specs = graph_kernel_specs(load_onnx(model_path), self.dtype)
            except (OSError, OnnxFormatError) as e:
                print(f"[warn] {model_path}: not a readable ONNX model ({e}); using the encoder-block kernels")
                specs = []
            if specs:
                return specs
        return _default_transformer_specs(model_name, self.dtype)

    def _autotune(self, specs: List[KernelSpec]) -> Dict[str, TuningResult]:
        results: Dict[str, TuningResult] = {}
        for spec in specs:
            if spec.kind == KernelKind.GEMM and self._tuner is not None:
                try:
                    results[spec.name] = self._tuner.tune_gemm(4096, 4096, 768, spec=spec)
                except Exception as e:
                    print(f"  [warn] autotune {spec.name}: {e}")
        return results

    def compile_transformer(self, hidden_dim: int = 768, num_heads: int = 12, seq_len: int = 512,
                            output_dir: Optional[str] = None) -> CompiledModel:
        """Emit an encoder-block kernel set without a model file."""
        name = f"transformer_h{hidden_dim}_H{num_heads}_s{seq_len}"
        out = Path(output_dir or f"lunara_compiled_{name}")
        out.mkdir(parents=True, exist_ok=True)
        kernel_module = emit_transformer_block(hidden_dim=hidden_dim, num_heads=num_heads, seq_len=seq_len,
                                               dtype=self.dtype, output_dir=str(out / "kernels"))
        specs = _default_transformer_specs(name, self.dtype, hidden_dim, num_heads)
        tuning: Dict[str, TuningResult] = {}
        if self.autotune and torch.cuda.is_available():
            tuning = self._autotune(specs)
        compiled = CompiledModel(name=name, kernel_module=kernel_module, mlir_path=None, kernel_specs=specs,
                                 tuning_results=tuning)
        compiled.load_kernels()
        return compiled


def _default_transformer_specs(name: str, dtype: str, hidden: int = 768, heads: int = 12) -> List[KernelSpec]:
    """The seven kernels of one encoder block (lunara/driver.py:266-283)."""
    return transformer_block_specs(hidden, heads, dtype)


def _main():
    import argparse
    p = argparse.ArgumentParser(description="Lunara B200 driver")
    sub = p.add_subparsers(dest="command")
    cp = sub.add_parser("compile", help="Compile a model")
    cp.add_argument("model")
    cp.add_argument("--out", default=None)
    cp.add_argument("--opt", type=int, default=2)
    cp.add_argument("--dtype", default="float16")
    cp.add_argument("--tune", action="store_true")
    ep = sub.add_parser("emit", help="Emit encoder-block kernels")
    ep.add_argument("--hidden", type=int, default=768)
    ep.add_argument("--heads", type=int, default=12)
    ep.add_argument("--seq", type=int, default=512)
    ep.add_argument("--dtype", default="float16")
    ep.add_argument("--out", default=None)
    ep.add_argument("--tune", action="store_true")
    ep.add_argument("--bench", action="store_true")
    args = p.parse_args()
    if args.command is None:
        p.print_help()
        return
    if args.command == "compile":
        compiled = Compiler(opt_level=args.opt, dtype=args.dtype, autotune=args.tune).compile(args.model, args.out)
        print(f"Kernels: {compiled.kernel_module}")
    elif args.command == "emit":
        compiled = Compiler(dtype=args.dtype, autotune=args.tune).compile_transformer(
            args.hidden, args.heads, args.seq, args.out)
        print(f"Kernels: {compiled.kernel_module}")
        if args.bench and torch.cuda.is_available():
            for k, v in compiled.benchmark().items():
                print(f"  {k:<30s}: {v:.3f} ms")


if __name__ == "__main__":
    _main()
