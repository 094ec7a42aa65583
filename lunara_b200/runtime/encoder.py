"""Encoder block / stack executor over the sm_100a kernels.

Runs the kernel set of one post-LN transformer encoder block -- the seven
kernels of lunara/driver.py:275-283 (qkv_proj, flash_attn, out_proj,
layernorm_attn, ffn1, ffn2, layernorm_ffn) -- on device-resident weights and
activation buffers, optionally captured once into a CUDA graph and replayed.
Each LayerNorm can be fused into the GEMM before it (lunara_gemm_layernorm,
the reference's FusionOptions.fuse_layernorm, lunara/passes/operator_fusion.h:19-20),
so the block runs five kernels: qkv_proj, flash_attn, out_proj+layernorm_attn,
ffn1, ffn2+layernorm_ffn. By default the fused form is used from
FUSE_LAYERNORM_MIN_TOKENS tokens per block up, the seven-kernel form below it.

Data layout in HBM (tokens T = B*S, hidden Hd, heads H, head dim D = Hd/H):
  x      [T, Hd]            input / residual of the attention sub-layer
  qkv    [T, 3*Hd]          = [B, S, 3, H, D]; attention reads Q, K and V from
                            it in place through 4-D tensor maps (no split copy)
  attn   [T, Hd]            attention output written as [B, S, H, D]
  h      [T, Hd]            out_proj + bias + residual(x)   (fused epilogue; unused when
                            the LayerNorm is fused as well)
  x1     [T, Hd]            LayerNorm(h)
  f      [T, F]             GELU(x1 W1^T + b1)               (fused epilogue)
  g      [T, Hd]            f W2^T + b2 + residual(x1)       (unused when fused)
  y      [T, Hd]            LayerNorm(g)
Linear weights are kept as [out, in] (K-major for the tcgen05 B operand).
"""
from __future__ import annotations

import math
from collections import OrderedDict
from typing import Callable, Dict, List, Optional

import torch

from lunara_b200.runtime import ops

WEIGHT_NAMES = ("w_qkv", "b_qkv", "w_o", "b_o", "ln1_w", "ln1_b", "w_1", "b_1", "w_2", "b_2", "ln2_w", "ln2_b")

# Kernel names in execution order, as in the reference's block spec list.
KERNEL_ORDER = ("qkv_proj", "flash_attn", "out_proj", "layernorm_attn", "ffn1", "ffn2", "layernorm_ffn")
# The same block with each LayerNorm fused into the GEMM before it.
FUSED_KERNEL_ORDER = ("qkv_proj", "flash_attn", "out_proj+layernorm_attn", "ffn1", "ffn2+layernorm_ffn")

# Default choice between the two forms, by tokens per block (batch * seq). The
# fused GEMM + LayerNorm kernel keeps each row's 768 columns in one cluster of
# single-CTA 128 x 192 tiles (a 4-stage ring at most), while the unfused ffn2
# runs on 256 x 192 CTA pairs with a 5-stage ring. Measured on B200, 12-layer
# stacks, interleaved repeats: the seven-kernel form was 2.7 % faster at 4096
# tokens (B8 S512: 1.052 against 1.081 ms per forward; block step 94.6 against
# 95.8 us) and 2 % faster at 8192; at 16384 and 32768 the two were within the
# run-to-run spread (3.79 / 3.79 and 7.95 / 8.07 ms).
FUSE_LAYERNORM_MIN_TOKENS = 16384


def default_fuse_layernorm(batch: int, seq: int) -> bool:
    """The block form used when the caller does not choose: fused from
    FUSE_LAYERNORM_MIN_TOKENS tokens per block up."""
    return batch * seq >= FUSE_LAYERNORM_MIN_TOKENS


def block_flops(tokens: int, seq: int, hidden: int = 768, heads: int = 12, ffn: int = 3072) -> Dict[str, float]:
    """Algorithmic FLOPs per kernel of one block (2MNK per GEMM, 4*B*H*S^2*D attention)."""
    batch = tokens // seq
    d = hidden // heads
    f = {
        "qkv_proj": 2.0 * tokens * hidden * 3 * hidden,
        "flash_attn": 4.0 * batch * heads * seq * seq * d,
        "out_proj": 2.0 * tokens * hidden * hidden,
        "layernorm_attn": 0.0,
        "ffn1": 2.0 * tokens * hidden * ffn,
        "ffn2": 2.0 * tokens * ffn * hidden,
        "layernorm_ffn": 0.0,
    }
    f["out_proj+layernorm_attn"] = f["out_proj"]
    f["ffn2+layernorm_ffn"] = f["ffn2"]
    return f


class EncoderBlock:
    """One encoder layer with static buffers for a fixed [batch, seq] shape."""

    def __init__(self, weights: Dict[str, torch.Tensor], batch: int, seq: int, num_heads: int = 12,
                 dtype: torch.dtype = torch.float16, device: Optional[torch.device] = None,
                 eps: float = 1e-5, ffn_activation: str = "gelu_tanh",
                 gemm_tiles: Optional[Dict[str, Dict[str, int]]] = None,
                 fuse_layernorm: Optional[bool] = None):
        device = torch.device(device or "cuda")
        self.batch, self.seq, self.heads, self.dtype, self.eps = batch, seq, num_heads, dtype, eps
        self.fuse_layernorm = default_fuse_layernorm(batch, seq) if fuse_layernorm is None else fuse_layernorm
        self.ffn_activation = ffn_activation
        self.gemm_tiles = gemm_tiles or {}
        self.w = {k: weights[k].to(device=device, dtype=dtype).contiguous() for k in WEIGHT_NAMES}
        self.hidden = self.w["w_o"].shape[0]
        self.ffn = self.w["w_1"].shape[0]
        assert self.hidden % num_heads == 0
        self.head_dim = self.hidden // num_heads
        T = batch * seq
        e = lambda n: torch.empty(T, n, dtype=dtype, device=device)  # noqa: E731
        self.x = e(self.hidden)
        self.qkv = e(3 * self.hidden)
        self.attn = e(self.hidden)
        self.h = e(self.hidden)
        self.x1 = e(self.hidden)
        self.f = e(self.ffn)
        self.g = e(self.hidden)
        self.y = e(self.hidden)
        self.scale = 1.0 / math.sqrt(self.head_dim)

    # Views of the fused QKV buffer as [B, H, S, D] with the buffer's strides.
    def _qkv_views(self):
        B, S, H, D = self.batch, self.seq, self.heads, self.head_dim
        t = self.qkv.view(B, S, 3, H, D)
        return tuple(t[:, :, i].permute(0, 2, 1, 3) for i in range(3))

    def _tile(self, name: str) -> Dict[str, int]:
        return self.gemm_tiles.get(name, {})

    def kernel_names(self):
        return FUSED_KERNEL_ORDER if self.fuse_layernorm else KERNEL_ORDER

    def kernel_fns(self, x: Optional[torch.Tensor] = None,
                   out: Optional[torch.Tensor] = None) -> "OrderedDict[str, Callable[[], object]]":
        """The launches of one block forward (x, default self.x -> out, default self.y), in
        order, keyed by the names of FUSED_KERNEL_ORDER (LayerNorm fused) or KERNEL_ORDER."""
        x = self.x if x is None else x
        y = self.y if out is None else out
        w = self.w
        B, S, H, D = self.batch, self.seq, self.heads, self.head_dim
        q, k, v = self._qkv_views()
        o = self.attn.view(B, S, H, D).permute(0, 2, 1, 3)
        if self.fuse_layernorm:
            return OrderedDict([
                ("qkv_proj", lambda: ops.gemm(x, w["w_qkv"], self.qkv, bias=w["b_qkv"], b_layout="nk",
                                              **self._tile("qkv_proj"))),
                ("flash_attn", lambda: ops.attention(q, k, v, causal=False, scale=self.scale, out=o)),
                ("out_proj+layernorm_attn",
                 lambda: ops.gemm_layernorm(self.attn, w["w_o"], w["ln1_w"], w["ln1_b"], bias=w["b_o"], residual=x,
                                            eps=self.eps, out=self.x1)),
                ("ffn1", lambda: ops.gemm(self.x1, w["w_1"], self.f, bias=w["b_1"], activation=self.ffn_activation,
                                          b_layout="nk", **self._tile("ffn1"))),
                ("ffn2+layernorm_ffn",
                 lambda: ops.gemm_layernorm(self.f, w["w_2"], w["ln2_w"], w["ln2_b"], bias=w["b_2"],
                                            residual=self.x1, eps=self.eps, out=y)),
            ])
        return OrderedDict([
            ("qkv_proj", lambda: ops.gemm(x, w["w_qkv"], self.qkv, bias=w["b_qkv"], b_layout="nk",
                                          **self._tile("qkv_proj"))),
            ("flash_attn", lambda: ops.attention(q, k, v, causal=False, scale=self.scale, out=o)),
            ("out_proj", lambda: ops.gemm(self.attn, w["w_o"], self.h, bias=w["b_o"], residual=x, b_layout="nk",
                                          **self._tile("out_proj"))),
            ("layernorm_attn", lambda: ops.layernorm(self.h, w["ln1_w"], w["ln1_b"], self.eps, out=self.x1)),
            ("ffn1", lambda: ops.gemm(self.x1, w["w_1"], self.f, bias=w["b_1"], activation=self.ffn_activation,
                                      b_layout="nk", **self._tile("ffn1"))),
            ("ffn2", lambda: ops.gemm(self.f, w["w_2"], self.g, bias=w["b_2"], residual=self.x1, b_layout="nk",
                                      **self._tile("ffn2"))),
            ("layernorm_ffn", lambda: ops.layernorm(self.g, w["ln2_w"], w["ln2_b"], self.eps, out=y)),
        ])

    def run_kernels(self, x: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                    hook: Optional[Callable[[str, str], None]] = None) -> torch.Tensor:
        """Launch the seven kernels on the current stream: x (default self.x) -> out (default self.y).

        ``hook(kernel_name, "begin"|"end")`` is called around each launch (used
        to record CUDA events inside a captured graph).
        """
        y = self.y if out is None else out
        for name, fn in self.kernel_fns(x, y).items():
            if hook:
                hook(name, "begin")
            fn()
            if hook:
                hook(name, "end")
        return y


class EncoderStack:
    """A stack of encoder blocks sharing one set of activation buffers per shape."""

    def __init__(self, layers: List[Dict[str, torch.Tensor]], batch: int, seq: int, num_heads: int = 12,
                 dtype: torch.dtype = torch.float16, device: Optional[torch.device] = None,
                 eps: float = 1e-5, ffn_activation: str = "gelu_tanh", fuse_layernorm: Optional[bool] = None):
        self.blocks = [EncoderBlock(w, batch, seq, num_heads, dtype, device, eps, ffn_activation,
                                    fuse_layernorm=fuse_layernorm) for w in layers]
        # Share activation buffers between layers: only the weights differ.
        first = self.blocks[0]
        for blk in self.blocks[1:]:
            for name in ("qkv", "attn", "h", "x1", "f", "g"):
                setattr(blk, name, getattr(first, name))
        self.x = first.x
        self._ping = torch.empty_like(first.y)
        self._pong = torch.empty_like(first.y)
        self.y = self._pong if len(self.blocks) % 2 == 0 else self._ping

    def run_kernels(self, x: Optional[torch.Tensor] = None, hook=None) -> torch.Tensor:
        cur = self.x if x is None else x
        bufs = (self._ping, self._pong)
        for i, blk in enumerate(self.blocks):
            nxt = bufs[i % 2]
            blk.run_kernels(cur, nxt, hook=hook)
            cur = nxt
        return cur


class GraphRunner:
    """Capture ``fn`` (a sequence of kernel launches on static buffers) into a CUDA graph.

    ``replay()`` relaunches the whole sequence with one host call; it is what
    removes the per-kernel host launch cost from a block or stack step.
    """

    def __init__(self, fn: Callable[[], object], warmup: int = 1):
        self.stream = torch.cuda.Stream()
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            for _ in range(warmup):
                fn()
        torch.cuda.current_stream().wait_stream(self.stream)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.out = fn()
        torch.cuda.synchronize()

    def replay(self):
        self.graph.replay()
        return self.out

    def release(self) -> None:
        self.graph.reset()
