"""Torch-facing wrappers over the C ABI: one function per KernelSpec kind.

torch owns every buffer; these functions pass raw device pointers, sizes and
torch's current CUDA stream to the library. Argument errors mirror the
reference launchers (``AssertionError`` for non-CUDA inputs and shape
mismatches, ``lunara/codegen/triton_emitter.py:155-160``); library errors raise
``ValueError`` (bad argument) or ``LunaraError``.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence

import torch

from lunara_b200.runtime import _lib

_DTYPES = {torch.float16: _lib.F16, torch.bfloat16: _lib.BF16, torch.float32: _lib.F32}

ACTIVATIONS = {
    None: _lib.ACT_NONE, "none": _lib.ACT_NONE, "identity": _lib.ACT_NONE,
    "relu": _lib.ACT_RELU,
    "gelu": _lib.ACT_GELU_ERF, "gelu_erf": _lib.ACT_GELU_ERF,
    "gelu_tanh": _lib.ACT_GELU_TANH,
    "sigmoid": _lib.ACT_SIGMOID,
    "tanh": _lib.ACT_TANH,
}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float16, bfloat16 or float32") from None


def _act_code(activation) -> int:
    if isinstance(activation, int):
        return activation
    try:
        return ACTIVATIONS[activation]
    except KeyError:
        raise ValueError(f"unknown activation {activation!r}") from None


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _require_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None:
            assert t.is_cuda, "lunara kernels take CUDA tensors"


# ─────────────────────────────────────────────────────────────── GEMM ──

def gemm(A: torch.Tensor, B: torch.Tensor, C: Optional[torch.Tensor] = None,
         bias: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
         activation=None, b_layout: str = "kn", block_n: int = 0, stages: int = 0,
         num_ctas: int = 0, cta_pair: int = 0) -> torch.Tensor:
    """C = act(A @ B + bias) + residual.

    ``b_layout="kn"``: B is [K, N] (the reference launcher's B);
    ``b_layout="nk"``: B is [N, K] (a Linear weight, C = A @ B^T).
    A, B, C and residual need a unit inner stride; leading dimensions are free.
    ``block_n`` / ``stages`` / ``num_ctas`` / ``cta_pair`` (1 single-CTA tiles,
    2 CTA-pair tiles) override the automatic tile choice; 0 means automatic.
    """
    _require_cuda(A, B, C, bias, residual)
    assert A.dim() == 2 and B.dim() == 2, "GEMM operands must be 2-D"
    M, K = A.shape
    if b_layout == "kn":
        K2, N = B.shape
        layout = _lib.B_KN
    elif b_layout == "nk":
        N, K2 = B.shape
        layout = _lib.B_NK
    else:
        raise ValueError(f"b_layout must be 'kn' or 'nk', got {b_layout!r}")
    assert K == K2, f"Dimension mismatch: A{(M, K)} B{tuple(B.shape)}"
    if C is None:
        C = torch.empty(M, N, dtype=A.dtype, device=A.device)
    assert C.shape == (M, N), f"C must be {(M, N)}, got {tuple(C.shape)}"
    assert A.dtype == B.dtype == C.dtype, "A, B and C must share a dtype"
    for t, name in ((A, "A"), (B, "B"), (C, "C")):
        assert t.stride(1) == 1 or t.shape[1] == 1, f"{name} needs a unit inner stride"
    if bias is not None:
        assert bias.numel() == N and bias.is_contiguous() and bias.dtype == A.dtype, "bias must be [N], contiguous"
    ldr = 0
    if residual is not None:
        assert residual.shape == (M, N) and residual.dtype == A.dtype, "residual must be [M, N]"
        assert residual.stride(1) == 1 or N == 1, "residual needs a unit inner stride"
        ldr = residual.stride(0)
    cfg = _lib.GemmConfig(block_n, stages, num_ctas, cta_pair)
    lib = _lib.load()
    _lib.check(lib.lunara_gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), _ptr(bias), _ptr(residual),
                               M, N, K, max(A.stride(0), K), max(B.stride(0), 1), max(C.stride(0), N), ldr,
                               layout, _dtype_code(A), _act_code(activation), cfg, _stream()))
    return C


def gemm_layernorm(A: torch.Tensor, B: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor,
                   bias: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
                   eps: float = 1e-5, b_layout: str = "nk", out: Optional[torch.Tensor] = None,
                   block_n: int = 0, stages: int = 0, num_ctas: int = 0) -> torch.Tensor:
    """LayerNorm(A @ B + bias + residual) * gamma + beta over the last dimension, in one
    kernel (lunara_gemm_layernorm). Shapes the fused kernel does not take (N not a
    multiple of 128/192/256 in 2..8 slices, fp32, unaligned views) run the GEMM into a
    temporary and the LayerNorm kernel after it -- two launches, same result."""
    _require_cuda(A, B, gamma, beta, bias, residual, out)
    assert A.dim() == 2 and B.dim() == 2, "GEMM operands must be 2-D"
    M, K = A.shape
    if b_layout == "kn":
        K2, N = B.shape
        layout = _lib.B_KN
    elif b_layout == "nk":
        N, K2 = B.shape
        layout = _lib.B_NK
    else:
        raise ValueError(f"b_layout must be 'kn' or 'nk', got {b_layout!r}")
    assert K == K2, f"Dimension mismatch: A{(M, K)} B{tuple(B.shape)}"
    assert gamma.numel() == N and beta.numel() == N, "gamma/beta must have N elements"
    if out is None:
        out = torch.empty(M, N, dtype=A.dtype, device=A.device)
    assert out.shape == (M, N) and out.dtype == A.dtype and out.stride(1) == 1, "out must be [M, N]"
    g = gamma.contiguous().to(A.dtype)
    b = beta.contiguous().to(A.dtype)
    ldr = 0
    if residual is not None:
        assert residual.shape == (M, N) and residual.dtype == A.dtype and residual.stride(1) == 1
        ldr = residual.stride(0)
    if bias is not None:
        assert bias.numel() == N and bias.is_contiguous() and bias.dtype == A.dtype, "bias must be [N], contiguous"
    lib = _lib.load()
    rc = lib.lunara_gemm_layernorm(A.data_ptr(), B.data_ptr(), out.data_ptr(), _ptr(bias), _ptr(residual),
                                   g.data_ptr(), b.data_ptr(), M, N, K, max(A.stride(0), K), max(B.stride(0), 1),
                                   max(out.stride(0), N), ldr, layout, _dtype_code(A), float(eps),
                                   _lib.GemmConfig(block_n, stages, num_ctas, 0), _stream())
    if rc == _lib.ERR_UNSUPPORTED:
        h = gemm(A, B, bias=bias, residual=residual, b_layout=b_layout)
        return layernorm(h, g, b, eps, out=out)
    _lib.check(rc)
    return out


# ────────────────────────────────────────────────────────── attention ──

def attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, causal: bool = False,
              scale: Optional[float] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """softmax(Q K^T * scale [causal]) V for [B, H, S, D] views (any strides, unit dim stride)."""
    _require_cuda(Q, K, V, out)
    assert Q.dim() == 4 and K.dim() == 4 and V.dim() == 4, "attention takes [B, H, S, D] tensors"
    B, H, Sq, D = Q.shape
    Bk, Hk, Skv, Dk = K.shape
    assert (Bk, Hk, Dk) == (B, H, D) and V.shape == K.shape, "Q/K/V shape mismatch"
    assert Q.dtype == K.dtype == V.dtype, "Q/K/V must share a dtype"
    if out is None:
        out = torch.empty(B, H, Sq, D, dtype=Q.dtype, device=Q.device)
    assert out.shape == Q.shape and out.dtype == Q.dtype
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    lib = _lib.load()
    _lib.check(lib.lunara_attention(
        Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), B, H, Sq, Skv, D,
        _lib.i64_array(Q.stride()), _lib.i64_array(K.stride()), _lib.i64_array(V.stride()),
        _lib.i64_array(out.stride()), float(scale), 1 if causal else 0, _dtype_code(Q), _stream()))
    return out


# ─────────────────────────────────────────────────── row-wise kernels ──

def layernorm(X: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """LayerNorm over the last dimension of a tensor of any rank."""
    _require_cuda(X, weight, bias, out)
    shape = X.shape
    N = shape[-1]
    X2 = X.contiguous().view(-1, N)
    assert weight.numel() == N and bias.numel() == N, "weight/bias must have the last dim's size"
    w = weight.contiguous().to(X.dtype)
    b = bias.contiguous().to(X.dtype)
    Y = torch.empty_like(X2) if out is None else out.view(-1, N)
    lib = _lib.load()
    _lib.check(lib.lunara_layernorm(X2.data_ptr(), w.data_ptr(), b.data_ptr(), Y.data_ptr(),
                                    X2.shape[0], N, float(eps), _dtype_code(X), _stream()))
    return Y.view(shape)


def softmax(X: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Row softmax over the last dimension."""
    _require_cuda(X, out)
    shape = X.shape
    N = shape[-1]
    X2 = X.contiguous().view(-1, N)
    Y = torch.empty_like(X2) if out is None else out.view(-1, N)
    lib = _lib.load()
    _lib.check(lib.lunara_softmax(X2.data_ptr(), Y.data_ptr(), X2.shape[0], N, _dtype_code(X), _stream()))
    return Y.view(shape)


# ──────────────────────────────────────────────────────── elementwise ──

def unary(X: torch.Tensor, activation="relu", out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _require_cuda(X, out)
    Xc = X.contiguous()
    Y = torch.empty_like(Xc) if out is None else out
    lib = _lib.load()
    _lib.check(lib.lunara_eltwise_unary(_act_code(activation), Xc.data_ptr(), Y.data_ptr(), Xc.numel(),
                                        _dtype_code(X), _stream()))
    return Y


def binary(X: torch.Tensor, Y: torch.Tensor, op: str = "add", out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _require_cuda(X, Y, out)
    assert X.shape == Y.shape and X.dtype == Y.dtype, "binary ops take same-shape, same-dtype tensors"
    Xc, Yc = X.contiguous(), Y.contiguous()
    O = torch.empty_like(Xc) if out is None else out
    code = {"add": _lib.BIN_ADD, "mul": _lib.BIN_MUL}[op]
    lib = _lib.load()
    _lib.check(lib.lunara_eltwise_binary(code, Xc.data_ptr(), Yc.data_ptr(), O.data_ptr(), Xc.numel(),
                                         _dtype_code(X), _stream()))
    return O


def bias_act(X: torch.Tensor, bias: torch.Tensor, activation="gelu_tanh",
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """act(X + bias) with bias broadcast over the last dimension."""
    _require_cuda(X, bias, out)
    cols = X.shape[-1]
    assert bias.numel() == cols and bias.dtype == X.dtype, "bias must match the last dim and dtype"
    Xc = X.contiguous()
    Y = torch.empty_like(Xc) if out is None else out
    lib = _lib.load()
    _lib.check(lib.lunara_bias_act(Xc.data_ptr(), bias.contiguous().data_ptr(), Y.data_ptr(),
                                   Xc.numel() // max(cols, 1), cols, _act_code(activation), _dtype_code(X),
                                   _stream()))
    return Y


# ─────────────────────────────────────────────────────────── index ops ──

def gather(src: torch.Tensor, index: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Row gather along dim 0 (``index_select(src, 0, index)``), bit-exact."""
    _require_cuda(src, index, out)
    assert index.dtype == torch.int64 and index.dim() == 1, "index must be 1-D int64"
    s = src.contiguous()
    rows = s.shape[0]
    row_bytes = s[0].numel() * s.element_size() if rows > 0 else 0
    if out is None:
        out = torch.empty((index.numel(),) + tuple(s.shape[1:]), dtype=s.dtype, device=s.device)
    idx = index.contiguous()
    lib = _lib.load()
    _lib.check(lib.lunara_gather(s.data_ptr(), idx.data_ptr(), out.data_ptr(), idx.numel(), rows,
                                 row_bytes, _stream()))
    return out


def contiguous_copy(src: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Materialise any strided view (Reshape / Transpose / Slice result) contiguously, bit-exact."""
    _require_cuda(src, out)
    if out is None:
        out = torch.empty(src.shape, dtype=src.dtype, device=src.device)
    lib = _lib.load()
    _lib.check(lib.lunara_copy_strided(src.data_ptr(), out.data_ptr(), src.dim(), _lib.i64_array(src.shape),
                                       _lib.i64_array(src.stride()), src.element_size(), _stream()))
    return out


def slice(src: torch.Tensor, starts: Sequence[int], ends: Sequence[int],
          steps: Optional[Sequence[int]] = None) -> torch.Tensor:
    """ONNX-style Slice on every dimension (positive steps), into a new contiguous tensor."""
    _require_cuda(src)
    s = src.contiguous()
    nd = s.dim()
    steps = list(steps) if steps is not None else [1] * nd
    assert len(starts) == len(ends) == len(steps) == nd, "one start/end/step per dimension"
    dst_sizes = []
    for k in range(nd):
        n = s.shape[k]
        st = max(0, min(starts[k] + n if starts[k] < 0 else starts[k], n))
        en = max(0, min(ends[k] + n if ends[k] < 0 else ends[k], n))
        dst_sizes.append(max(0, (en - st + steps[k] - 1) // steps[k]))
        starts = list(starts)
        starts[k] = st
    out = torch.empty(dst_sizes, dtype=s.dtype, device=s.device)
    if out.numel() == 0:
        return out
    lib = _lib.load()
    _lib.check(lib.lunara_slice(s.data_ptr(), out.data_ptr(), nd, _lib.i64_array(s.shape),
                                _lib.i64_array(starts), _lib.i64_array(steps), _lib.i64_array(dst_sizes),
                                s.element_size(), _stream()))
    return out


def reshape(src: torch.Tensor, shape: Sequence[int]) -> torch.Tensor:
    """Reshape: a zero-copy view when the source is contiguous, else a strided copy first."""
    if src.is_contiguous():
        return src.view(*shape)
    return contiguous_copy(src).view(*shape)


def qkv_split(qkv: torch.Tensor, num_heads: int):
    """[B, S, 3*H*D] fused projection -> three contiguous [B, H, S, D] tensors, bit-exact."""
    _require_cuda(qkv)
    B, S, three_hd = qkv.shape
    assert three_hd % (3 * num_heads) == 0, "last dim must be 3 * heads * head_dim"
    D = three_hd // (3 * num_heads)
    src = qkv.contiguous()
    q, k, v = (torch.empty(B, num_heads, S, D, dtype=qkv.dtype, device=qkv.device) for _ in range(3))
    lib = _lib.load()
    _lib.check(lib.lunara_qkv_split(src.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), B, S, num_heads, D,
                                    src.element_size(), _stream()))
    return q, k, v


def device_error(clear: bool = True) -> int:
    """Synchronize the current stream and return (and clear) the library's device error word."""
    lib = _lib.load()
    v = lib.lunara_device_error(_stream(), 1 if clear else 0)
    if v < 0:
        _lib.check(-v)
    return v
