"""Autotuner over the sm_100a kernel configurations.

Drop-in counterpart of lunara/codegen/autotuner.py: ``TuningResult``,
``TuningCache`` (same JSON layout and key format, autotuner.py:35-46,
107-138), ``Autotuner.tune_gemm`` / ``tune_attention`` (172-283) and
``_gemm_configs``. The search space is the tcgen05 GEMM's own choices
(autotuner.py:50-70 searched every tile parameter of the Triton kernel; these
are the parameters of this one):

  * tile shape: single-CTA 128-row tiles (``BLOCK_M=128``) or 256-row tiles
    of a CTA pair (``BLOCK_M=256``, cta_group::2), by MMA N (``BLOCK_N``
    64/128/192/256 single, 128/192/256 paired; 192-wide pairs need B as a
    [N, K] weight);
  * shared-memory ring depth (``num_stages``, 2 .. what fits in 227 KB per
    CTA for that tile after the epilogue's staging);
  * persistent grid (``num_ctas``): every SM, or, when the last round of
    tiles is partly empty, the smallest grid that keeps the same number of
    rounds (fewer busy SMs draw less power, so the busy ones clock higher).

M tile per CTA (128) and K tile (64) are fixed by the kernel. Each candidate
is timed as the median of CUDA-event measured launches (autotuner.py:77-95)
and the best is cached.
"""
from __future__ import annotations

import hashlib
import json
import math
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Callable, Dict, List, Optional, Tuple

import torch

from lunara_b200.codegen.kernel_emitter import KernelKind, KernelSpec, TileConfig, gemm_cta_pair


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


# sm_100a GEMM search space (lunara_b200/csrc/gemm.cu).
BLOCK_M = 128                 # rows per CTA (a CTA pair's tile has 256)
BLOCK_K = 64
_BLOCK_N_SINGLE = [64, 128, 192, 256]
_BLOCK_N_PAIR = [128, 192, 256]
_SMEM_LIMIT = 232448          # 227 KB opt-in dynamic shared memory per CTA
# Barriers, 12 epilogue warps' bias staging (96 fp32 each) and output staging
# (2 KB each), 1 KB alignment slack: gemm.cu kSmemReserve.
_SMEM_RESERVED = 1024 + 512 + 12 * 96 * 4 + 12 * 2048
_NUM_SMS = 148


def max_stages(block_n: int, elem_bytes: int = 2, pair: bool = False) -> int:
    """Deepest ring that fits one CTA: stages * (A rows + B rows it holds) * BLOCK_K * elem
    <= 227 KB - reserved, capped at 8. A CTA of a pair holds 128 A rows and BLOCK_N/2 B rows."""
    b_rows = block_n // 2 if pair else block_n
    per_stage = (BLOCK_M + b_rows) * BLOCK_K * elem_bytes
    return min(8, (_SMEM_LIMIT - _SMEM_RESERVED) // per_stage)


def grid_choices(M: Optional[int], N: Optional[int], block_m: int, block_n: int, sms: int = _NUM_SMS) -> List[int]:
    """Persistent grid sizes worth timing: 0 (every SM or SM pair) and, when the
    last round of tiles is partly empty, the smallest grid with the same round count."""
    if M is None or N is None:
        return [0]
    units = sms // 2 if block_m == 256 else sms
    tiles = math.ceil(M / block_m) * math.ceil(N / block_n)
    rounds = math.ceil(tiles / units)
    fill = math.ceil(tiles / rounds)
    if tiles <= units or fill >= units:
        return [0]
    return [0, fill * (2 if block_m == 256 else 1)]


def _gemm_configs(M: Optional[int] = None, N: Optional[int] = None, b_layout: str = "nk",
                  sms: int = _NUM_SMS) -> List[TileConfig]:
    """Every (tile shape, ring depth, grid) the tcgen05 GEMM accepts for this problem."""
    configs = []
    shapes = [(BLOCK_M, bn) for bn in _BLOCK_N_SINGLE] + \
             [(2 * BLOCK_M, bn) for bn in _BLOCK_N_PAIR if bn != 192 or b_layout == "nk"]
    for bm, bn in shapes:
        for s in range(2, max_stages(bn, pair=bm == 256) + 1):
            for g in grid_choices(M, N, bm, bn, sms):
                configs.append(TileConfig(BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=BLOCK_K, num_stages=s, num_warps=4,
                                          num_ctas=g))
    return configs


def gemm_call_args(cfg: TileConfig) -> Dict[str, int]:
    """The ops.gemm / lunara_gemm_config request for a tuned TileConfig."""
    return dict(block_n=cfg.BLOCK_N, stages=cfg.num_stages, num_ctas=cfg.num_ctas,
                cta_pair=gemm_cta_pair(cfg) or 1)


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
        configs = _gemm_configs(M, N, b_layout, torch.cuda.get_device_properties(0).multi_processor_count)
        self._log(f"Tuning GEMM {M}x{N}x{K}: {len(configs)} configs")
        best: Optional[TuningResult] = None
        for i, cfg in enumerate(configs):
            try:
                def fn(cfg=cfg):
                    return ops.gemm(A, B, C, bias=bias, activation=spec.activation, b_layout=b_layout,
                                    **gemm_call_args(cfg))
                lat = _bench(fn, self.n_warmup, self.n_trials)
                tfl = _tflops_gemm(M, N, K, lat)
                if best is None or lat < best.latency_ms:
                    best = TuningResult(config=cfg, latency_ms=lat, tflops=tfl)
            except Exception as e:
                self._log(f"  Config {i} failed: {e}")
        if best is None:
            raise RuntimeError("All GEMM configs failed during tuning")
        self._log(f"Best: {'CTA pair' if best.config.BLOCK_M == 256 else 'single CTA'} BN={best.config.BLOCK_N} "
                  f"stages={best.config.num_stages} grid={best.config.num_ctas or 'all'} → {best.tflops:.2f} TFLOPS")
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
