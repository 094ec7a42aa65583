"""Autotuner over the sm_100a kernel configurations.

Drop-in counterpart of lunara/codegen/autotuner.py: ``TuningResult``,
``TuningCache`` (same JSON format and key, autotuner.py:35-46, 107-138),
``Autotuner.tune_gemm`` / ``tune_attention`` (172-283) and ``_gemm_configs``.
The search space is the tcgen05 GEMM's: MMA N tile (64/128/192/256) x
shared-memory ring depth (2 .. what fits in 227 KB for that tile); M tile 128
and K tile 64 are fixed by the kernel. Each candidate is timed as the median of
CUDA-event measured launches (autotuner.py:77-95) and the best is cached.
"""
from __future__ import annotations

import hashlib
import json
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Callable, Dict, List, Optional, Tuple

import torch

from lunara_b200.codegen.kernel_emitter import KernelKind, KernelSpec, TileConfig


@dataclass
class TuningResult:
    config: TileConfig
    latency_ms: float
    tflops: float
    config_hash: str = ""

    def __post_init__(self):
        if not self.config_hash:
            d = asdict(self.config)
            self.config_hash = hashlib.md5(json.dumps(d, sort_keys=True).encode()).hexdigest()[:8]


# sm_100a GEMM search space.
BLOCK_M = 128
BLOCK_K = 64
_BLOCK_N_CHOICES = [64, 128, 192, 256]
_SMEM_LIMIT = 232448          # 227 KB opt-in dynamic shared memory per CTA
_SMEM_RESERVED = 22528        # barriers, bias and output staging, 1 KB alignment slack


def max_stages(block_n: int, elem_bytes: int = 2) -> int:
    """Deepest ring that fits: stages * (A tile + B tile) <= 227 KB - reserved (capped at 8)."""
    per_stage = (BLOCK_M + block_n) * BLOCK_K * elem_bytes
    return min(8, (_SMEM_LIMIT - _SMEM_RESERVED) // per_stage)


def _gemm_configs() -> List[TileConfig]:
    configs = []
    for bn in _BLOCK_N_CHOICES:
        for s in range(2, max_stages(bn) + 1):
            configs.append(TileConfig(BLOCK_M=BLOCK_M, BLOCK_N=bn, BLOCK_K=BLOCK_K, num_stages=s, num_warps=4))
    return configs


def _bench(fn: Callable, n_warmup: int = 5, n_trials: int = 20) -> float:
    """Median latency in ms over CUDA-event timed calls."""
    for _ in range(n_warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(n_trials):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end))
    times.sort()
    return times[len(times) // 2]


def _tflops_gemm(M: int, N: int, K: int, latency_ms: float) -> float:
    return 2 * M * N * K / (latency_ms * 1e-3) / 1e12


class TuningCache:
    def __init__(self, path: str = ".lunara_tuning_cache.json"):
        self.path = Path(path)
        self._data: Dict[str, dict] = {}
        if self.path.exists():
            self._data = json.loads(self.path.read_text())

    def _key(self, spec: KernelSpec, shape: Tuple) -> str:
        return f"{spec.kind.name}_{spec.name}_{'x'.join(map(str, shape))}"

    def get(self, spec: KernelSpec, shape: Tuple) -> Optional[TuningResult]:
        k = self._key(spec, shape)
        if k not in self._data:
            return None
        d = self._data[k]
        return TuningResult(config=TileConfig(**d["config"]), latency_ms=d["latency_ms"], tflops=d["tflops"],
                            config_hash=d["config_hash"])

    def put(self, spec: KernelSpec, shape: Tuple, result: TuningResult) -> None:
        self._data[self._key(spec, shape)] = {
            "config": asdict(result.config),
            "latency_ms": result.latency_ms,
            "tflops": result.tflops,
            "config_hash": result.config_hash,
        }
        self.path.write_text(json.dumps(self._data, indent=2))


class Autotuner:
    """Tune one kernel for one problem shape on the current device."""

    def __init__(self, cache_path: str = ".lunara_tuning_cache.json", n_warmup: int = 3, n_trials: int = 10,
                 verbose: bool = True):
        self.cache = TuningCache(cache_path)
        self.n_warmup = n_warmup
        self.n_trials = n_trials
        self.verbose = verbose

    def _log(self, msg: str):
        if self.verbose:
            print(f"[autotuner] {msg}")

    def tune_gemm(self, M: int, N: int, K: int, dtype: torch.dtype = torch.float16,
                  spec: Optional[KernelSpec] = None, b_layout: str = "kn") -> TuningResult:
        from lunara_b200.runtime import ops
        if spec is None:
            spec = KernelSpec(KernelKind.GEMM, "gemm_tuned")
        cached = self.cache.get(spec, (M, N, K))
        if cached:
            self._log(f"Cache hit: GEMM {M}x{N}x{K} → {cached.tflops:.2f} TFLOPS @ {cached.latency_ms:.3f}ms")
            return cached
        A = torch.randn(M, K, dtype=dtype, device="cuda")
        B = torch.randn(K, N, dtype=dtype, device="cuda") if b_layout == "kn" else \
            torch.randn(N, K, dtype=dtype, device="cuda")
        C = torch.empty(M, N, dtype=dtype, device="cuda")
        bias = torch.zeros(N, dtype=dtype, device="cuda") if spec.has_bias else None
        configs = _gemm_configs()
        self._log(f"Tuning GEMM {M}x{N}x{K}: {len(configs)} configs")
        best: Optional[TuningResult] = None
        for i, cfg in enumerate(configs):
            try:
                def fn(cfg=cfg):
                    return ops.gemm(A, B, C, bias=bias, activation=spec.activation, b_layout=b_layout,
                                    block_n=cfg.BLOCK_N, stages=cfg.num_stages)
                lat = _bench(fn, self.n_warmup, self.n_trials)
                tfl = _tflops_gemm(M, N, K, lat)
                if best is None or lat < best.latency_ms:
                    best = TuningResult(config=cfg, latency_ms=lat, tflops=tfl)
            except Exception as e:
                self._log(f"  Config {i} failed: {e}")
        if best is None:
            raise RuntimeError("All GEMM configs failed during tuning")
        self._log(f"Best: BN={best.config.BLOCK_N} stages={best.config.num_stages} → {best.tflops:.2f} TFLOPS")
        self.cache.put(spec, (M, N, K), best)
        return best

    def tune_attention(self, B: int, H: int, M: int, N: int, D: int, dtype: torch.dtype = torch.float16,
                       causal: bool = False) -> TuningResult:
        """The tcgen05 attention kernel has one tiling (128-query tiles, 128-key blocks); this measures it."""
        from lunara_b200.runtime import ops
        spec = KernelSpec(KernelKind.ATTENTION, "attn_tuned", is_causal=causal)
        cached = self.cache.get(spec, (B, H, M, N, D))
        if cached:
            self._log(f"Cache hit: Attention {B}x{H}x{M}x{N}x{D}")
            return cached
        Q = torch.randn(B, H, M, D, dtype=dtype, device="cuda")
        K = torch.randn(B, H, N, D, dtype=dtype, device="cuda")
        V = torch.randn(B, H, N, D, dtype=dtype, device="cuda")
        cfg = TileConfig(BLOCK_SEQ=128, HEAD_DIM=D, num_warps=4)
        lat = _bench(lambda: ops.attention(Q, K, V, causal=causal), self.n_warmup, self.n_trials)
        flops = 4.0 * B * H * M * N * D * (0.5 if causal else 1.0)
        best = TuningResult(config=cfg, latency_ms=lat, tflops=flops / (lat * 1e-3) / 1e12)
        self.cache.put(spec, (B, H, M, N, D), best)
        self._log(f"Attention: {best.tflops:.2f} TFLOPS")
        return best
