"""CPU oracle for the Lunara kernel kinds -- TEST INFRASTRUCTURE ONLY.

Torch-eager fp32 restatements, on the host CPU, of what each kernel of the
reference computes (lunara/codegen/triton_emitter.py), plus the post-LN
encoder block those kernels are emitted for (lunara/driver.py:266-283,
examples/01_transformer_block.py). Only the tests, ``__graft_entry__.smoke()``
and bench.py's CPU-baseline leg may use this module, and only as the checker or
as the timed CPU baseline; the product path (``lunara_b200``) never calls it.

Pinning: tests/test_oracle_golden.py checks every function here against golden
fixtures produced by running the reference's own Triton kernels under Triton's
CPU interpreter (tests/golden/make_golden.py).

Deliberate differences from the reference, each also pinned by a test:
  * LayerNorm takes the variance over exactly N elements. The reference sums
    (0 - mean)^2 for the padding lanes of its power-of-two block
    (triton_emitter.py:390-393); ``layernorm_reference_padded`` restates that
    behaviour for the pin, ``layernorm`` is what the kernels must match.
  * The encoder block's FFN uses the tanh-form GELU named for the benchmark
    configuration; the reference's GEMM epilogue and elementwise "gelu" are the
    erf form (triton_emitter.py:86, 454), available here as ``gelu_erf``.
  * GEMM epilogues stay in fp32 until one final rounding; the reference casts
    the accumulator to the output dtype before bias and activation
    (triton_emitter.py:145-147).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch

F32 = torch.float32


# ─────────────────────────────────────────────────────────── activations ──

def relu(x: torch.Tensor) -> torch.Tensor:
    """tl.maximum(x, 0.0) -- triton_emitter.py:84, 453."""
    return torch.clamp_min(x, 0.0)


def gelu_erf(x: torch.Tensor) -> torch.Tensor:
    """x * 0.5 * (1 + erf(x * 0.70710678)) -- triton_emitter.py:86, 454."""
    return x * 0.5 * (1.0 + torch.erf(x * 0.70710678))


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    """0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), the encoder block's GELU."""
    return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x * x * x)))


def sigmoid(x: torch.Tensor) -> torch.Tensor:
    """1 / (1 + exp(-x)) -- triton_emitter.py:88, 455."""
    return 1.0 / (1.0 + torch.exp(-x))


def tanh(x: torch.Tensor) -> torch.Tensor:
    """tanh(x) -- triton_emitter.py:456."""
    return torch.tanh(x)


ACTIVATIONS = {
    None: lambda x: x, "none": lambda x: x, "identity": lambda x: x,
    "relu": relu, "gelu": gelu_erf, "gelu_erf": gelu_erf, "gelu_tanh": gelu_tanh,
    "sigmoid": sigmoid, "tanh": tanh,
}


def unary(x: torch.Tensor, activation: Optional[str]) -> torch.Tensor:
    """ELEMENTWISE kind: y = body(x) -- triton_emitter.py:432-439."""
    return ACTIVATIONS[activation](x.to(F32))


def binary(x: torch.Tensor, y: torch.Tensor, op: str) -> torch.Tensor:
    return x.to(F32) + y.to(F32) if op == "add" else x.to(F32) * y.to(F32)


def bias_act(x: torch.Tensor, bias: torch.Tensor, activation: Optional[str]) -> torch.Tensor:
    """act(x + bias[col]) -- the ELEMENTWISE kind with KernelSpec.has_bias."""
    return ACTIVATIONS[activation](x.to(F32) + bias.to(F32))


# ────────────────────────────────────────────────────────────────── GEMM ──

def gemm(a: torch.Tensor, b: torch.Tensor, bias: Optional[torch.Tensor] = None,
         activation: Optional[str] = None, residual: Optional[torch.Tensor] = None,
         b_layout: str = "kn") -> torch.Tensor:
    """C = act(A @ B + bias) + residual with fp32 accumulation.

    GEMM template, triton_emitter.py:107-152: K-loop of tl.dot into an fp32
    accumulator (135-143), then bias (146, 181-182) and activation (147).
    ``b_layout="nk"`` takes B as [N, K] (a Linear weight).
    """
    bb = b.to(F32) if b_layout == "kn" else b.to(F32).t()
    c = a.to(F32) @ bb
    if bias is not None:
        c = c + bias.to(F32)
    c = ACTIVATIONS[activation](c)
    if residual is not None:
        c = c + residual.to(F32)
    return c


# ───────────────────────────────────────────────────────────── attention ──

def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
              scale: Optional[float] = None) -> torch.Tensor:
    """softmax(Q K^T * scale, causal keep row >= col) V over [B, H, S, D].

    Attention template, triton_emitter.py:212-293: scale 1/sqrt(D) (302),
    causal mask row >= col (265-268), fp32 online softmax -- restated here as
    the exact (non-online) softmax it converges to.
    """
    q32, k32, v32 = q.to(F32), k.to(F32), v.to(F32)
    D = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    s = (q32 @ k32.transpose(-1, -2)) * scale
    if causal:
        Sq, Skv = s.shape[-2], s.shape[-1]
        keep = torch.arange(Sq)[:, None] >= torch.arange(Skv)[None, :]
        s = s.masked_fill(~keep, float("-inf"))
    return torch.softmax(s, dim=-1) @ v32


# ────────────────────────────────────────────────────────── row kernels ──

def layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """(x - mean) / sqrt(var + eps) * w + b over the last dim, population variance over N.

    LayerNorm template, triton_emitter.py:382-398 (two-pass fp32 statistics),
    without the padding-lane term in the variance.
    """
    x32 = x.to(F32)
    mean = x32.mean(dim=-1, keepdim=True)
    var = ((x32 - mean) ** 2).mean(dim=-1, keepdim=True)
    return (x32 - mean) / torch.sqrt(var + eps) * weight.to(F32) + bias.to(F32)


def layernorm_reference_padded(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                               eps: float = 1e-5) -> torch.Tensor:
    """The reference kernel's actual arithmetic when N is not a power of two.

    Lanes N..BLOCK-1 load 0 (triton_emitter.py:390) and still contribute
    (0 - mean)^2 to the variance sum (392), which is divided by N.
    Used only to pin the oracle to the reference's golden output.
    """
    x32 = x.to(F32)
    N = x.shape[-1]
    block = 1 << (N - 1).bit_length()
    mean = x32.sum(dim=-1, keepdim=True) / N
    var = (((x32 - mean) ** 2).sum(dim=-1, keepdim=True) + (block - N) * mean ** 2) / N
    return (x32 - mean) / torch.sqrt(var + eps) * weight.to(F32) + bias.to(F32)


def softmax(x: torch.Tensor) -> torch.Tensor:
    """exp(x - max) / sum over the last dim -- triton_emitter.py:341-353."""
    x32 = x.to(F32)
    e = torch.exp(x32 - x32.max(dim=-1, keepdim=True).values)
    return e / e.sum(dim=-1, keepdim=True)


# ──────────────────────────────────────────────────────────── index ops ──

def gather(src: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """Gather along dim 0 (graph op Gather, lunara/frontend/graph_ir.h:23)."""
    return torch.index_select(src, 0, index)


def slice_(src: torch.Tensor, starts, ends, steps=None) -> torch.Tensor:
    """ONNX-style Slice with positive steps (graph op Slice)."""
    steps = steps or [1] * src.dim()
    idx = tuple(slice(s, e, st) for s, e, st in zip(starts, ends, steps))
    return src[idx].contiguous()


def qkv_split(qkv: torch.Tensor, num_heads: int):
    """[B, S, 3*H*D] -> three [B, H, S, D] (QKV split + head reshape of the block)."""
    B, S, three_hd = qkv.shape
    D = three_hd // (3 * num_heads)
    t = qkv.view(B, S, 3, num_heads, D).permute(2, 0, 3, 1, 4)
    return t[0].contiguous(), t[1].contiguous(), t[2].contiguous()


# ──────────────────────────────────────────────────────── encoder block ──

BLOCK_WEIGHT_NAMES = ("w_qkv", "b_qkv", "w_o", "b_o", "ln1_w", "ln1_b", "w_1", "b_1", "w_2", "b_2",
                      "ln2_w", "ln2_b")


def encoder_block(x: torch.Tensor, w: Dict[str, torch.Tensor], num_heads: int,
                  eps: float = 1e-5, ffn_activation: str = "gelu_tanh") -> torch.Tensor:
    """Post-LN BERT encoder block, the kernel set of lunara/driver.py:275-283.

    qkv_proj -> flash_attn -> out_proj (+residual) -> layernorm_attn ->
    ffn1 (+GELU) -> ffn2 (+residual) -> layernorm_ffn. Linear weights are
    [out, in] (``y = x W^T + b``); no attention mask.
    """
    B, S, Hd = x.shape
    D = Hd // num_heads
    x32 = x.to(F32).reshape(B * S, Hd)
    qkv = gemm(x32, w["w_qkv"], w["b_qkv"], b_layout="nk")
    q, k, v = qkv_split(qkv.view(B, S, 3 * Hd), num_heads)
    a = attention(q, k, v).permute(0, 2, 1, 3).reshape(B * S, Hd)
    h = gemm(a, w["w_o"], w["b_o"], residual=x32, b_layout="nk")
    x1 = layernorm(h, w["ln1_w"], w["ln1_b"], eps)
    f = gemm(x1, w["w_1"], w["b_1"], activation=ffn_activation, b_layout="nk")
    g = gemm(f, w["w_2"], w["b_2"], residual=x1, b_layout="nk")
    return layernorm(g, w["ln2_w"], w["ln2_b"], eps).view(B, S, Hd)


def encoder_stack(x: torch.Tensor, layers: List[Dict[str, torch.Tensor]], num_heads: int,
                  eps: float = 1e-5) -> torch.Tensor:
    for w in layers:
        x = encoder_block(x, w, num_heads, eps)
    return x


# ─────────────────────────────────────────────────────── error metrics ──

def max_abs(out: torch.Tensor, ref: torch.Tensor) -> float:
    return (out.detach().to(F32).cpu() - ref.to(F32).cpu()).abs().max().item()


def rel_l2(out: torch.Tensor, ref: torch.Tensor) -> float:
    o, r = out.detach().to(F32).cpu(), ref.to(F32).cpu()
    return ((o - r).norm() / r.norm().clamp_min(1e-30)).item()
