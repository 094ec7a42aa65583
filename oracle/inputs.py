"""Seeded synthetic inputs for the benchmark configurations -- TEST INFRASTRUCTURE.

Each generator draws fp32 tensors on the CPU from a ``torch.Generator`` with
the configuration's seed, in a fixed order, so the GPU run (after a cast to
fp16/bf16) and the CPU oracle see the same values. The shapes and
distributions are those of the benchmark configurations:

  block   BERT-base post-LN encoder block: hidden 768, 12 heads, FFN 3072,
          x ~ N(0,1) [B,S,768], Linear weights N(0,0.02) as [out,in],
          biases 0, LN gamma 1, beta 0 (seed 0; examples/01_transformer_block.py)
  gemm    M=N=K=4096, A,B ~ N(0,1) row-major, bias ~ N(0,0.1) (seed 1)
  attn    B2 H12 S2048 D64, Q,K,V ~ N(0,1), scale 1/8 (seed 2)
  ln      16384 x 768, x ~ N(0,1), gamma 1+N(0,0.1), beta N(0,0.1) (seed 3)
  gelu    16384 x 3072, x ~ N(0,1), bias ~ N(0,0.1) (seed 3)
  stack   12 independent block layers, x [64,512,768] (seed 4)
"""
from __future__ import annotations

from typing import Dict, List

import torch

HIDDEN, HEADS, FFN = 768, 12, 3072


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def block_weights(g: torch.Generator, hidden: int = HIDDEN, ffn: int = FFN,
                  std: float = 0.02) -> Dict[str, torch.Tensor]:
    return {
        "w_qkv": torch.randn(3 * hidden, hidden, generator=g) * std,
        "b_qkv": torch.zeros(3 * hidden),
        "w_o": torch.randn(hidden, hidden, generator=g) * std,
        "b_o": torch.zeros(hidden),
        "ln1_w": torch.ones(hidden),
        "ln1_b": torch.zeros(hidden),
        "w_1": torch.randn(ffn, hidden, generator=g) * std,
        "b_1": torch.zeros(ffn),
        "w_2": torch.randn(hidden, ffn, generator=g) * std,
        "b_2": torch.zeros(hidden),
        "ln2_w": torch.ones(hidden),
        "ln2_b": torch.zeros(hidden),
    }


def block_inputs(batch: int = 8, seq: int = 512, seed: int = 0, hidden: int = HIDDEN,
                 ffn: int = FFN):
    """(x [B,S,H], weights) of the encoder-block configuration."""
    g = _gen(seed)
    x = torch.randn(batch, seq, hidden, generator=g)
    return x, block_weights(g, hidden, ffn)


def stack_inputs(batch: int = 64, seq: int = 512, layers: int = 12, seed: int = 4,
                 hidden: int = HIDDEN, ffn: int = FFN):
    g = _gen(seed)
    x = torch.randn(batch, seq, hidden, generator=g)
    ws: List[Dict[str, torch.Tensor]] = [block_weights(g, hidden, ffn) for _ in range(layers)]
    return x, ws


def gemm_inputs(M: int = 4096, N: int = 4096, K: int = 4096, seed: int = 1):
    g = _gen(seed)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(K, N, generator=g)
    bias = torch.randn(N, generator=g) * 0.1
    return a, b, bias


def attention_inputs(B: int = 2, H: int = 12, S: int = 2048, D: int = 64, seed: int = 2):
    g = _gen(seed)
    return tuple(torch.randn(B, H, S, D, generator=g) for _ in range(3))


def layernorm_inputs(rows: int = 16384, cols: int = 768, seed: int = 3):
    g = _gen(seed)
    x = torch.randn(rows, cols, generator=g)
    w = 1.0 + 0.1 * torch.randn(cols, generator=g)
    b = 0.1 * torch.randn(cols, generator=g)
    return x, w, b


def bias_gelu_inputs(rows: int = 16384, cols: int = 3072, seed: int = 3):
    g = _gen(seed)
    x = torch.randn(rows, cols, generator=g)
    bias = 0.1 * torch.randn(cols, generator=g)
    return x, bias
