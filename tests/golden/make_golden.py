"""Generate golden fixtures from the reference's own kernels.

Runs the reference's Triton templates (lunara/codegen/triton_emitter.py) under
Triton's CPU interpreter (TRITON_INTERPRET=1) on small seeded inputs and saves
inputs and outputs as .npz files next to this script. The fixtures pin the CPU
oracle (oracle/oracle.py) to the reference's arithmetic; the GPU parity tests
then compare the sm_100a kernels with that oracle.

Needs the reference checkout (default /root/reference, or $LUNARA_REFERENCE)
and runs on CPU only. The committed .npz files are what the tests read; this
script only regenerates them.

Two in-memory patches make the shipped templates runnable, without changing
their arithmetic:
  * the GEMM launcher's assert message is not a valid f-string
    (triton_emitter.py:160), so the module does not parse; the message is
    dropped from that one assert, and the fixtures call the @triton.jit kernel
    directly with the launcher's own argument list;
  * the bias load of the GEMM template uses `mask_n` before it is defined
    (triton_emitter.py:146-150, 181-182); the mask is dropped, which is exact
    because the template wraps its column index `rn` modulo N (line 129).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

if "LUNARA_REFERENCE" not in os.environ:
    sys.exit("make_golden.py: set LUNARA_REFERENCE to the reference checkout (the directory holding lunara/)")
REF = Path(os.environ["LUNARA_REFERENCE"])
OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(REF))

from lunara.codegen import triton_emitter as te  # noqa: E402


def _exec(src: str, name: str) -> dict:
    ns: dict = {}
    exec(compile(src, f"<reference {name}>", "exec"), ns)
    return ns


def _save(name: str, **arrays) -> None:
    path = OUT / f"{name}.npz"
    np.savez_compressed(path, **{k: (v.numpy() if isinstance(v, torch.Tensor) else v) for k, v in arrays.items()})
    print(f"wrote {path.name}: " + ", ".join(f"{k}{tuple(np.shape(v))}" for k, v in arrays.items()))


def gen_softmax() -> None:
    spec = te.KernelSpec(te.KernelKind.SOFTMAX, "sm", dtype="float32")
    ns = _exec(te.emit_softmax(spec), "softmax")
    g = torch.Generator().manual_seed(100)
    for M, N in ((6, 100), (4, 64)):
        x = torch.randn(M, N, generator=g) * 3.0
        y = torch.empty_like(x)
        block = 1 << (N - 1).bit_length()
        ns["sm"][(M,)](x, y, M, N, BLOCK=block)  # launcher args, triton_emitter.py:356-363
        _save(f"softmax_f32_{M}x{N}", x=x, y=y)


def gen_layernorm() -> None:
    spec = te.KernelSpec(te.KernelKind.LAYERNORM, "ln", dtype="float32")
    ns = _exec(te.emit_layernorm(spec), "layernorm")
    g = torch.Generator().manual_seed(101)
    for M, N in ((5, 64), (5, 96)):
        x = torch.randn(M, N, generator=g) * 2.0 + 0.5
        w = 1.0 + 0.1 * torch.randn(N, generator=g)
        b = 0.1 * torch.randn(N, generator=g)
        y = torch.empty_like(x)
        block = 1 << (N - 1).bit_length()
        ns["ln"][(M,)](x, w, b, y, N, 1e-5, BLOCK=block)  # launcher args, triton_emitter.py:401-411
        _save(f"layernorm_f32_{M}x{N}", x=x, w=w, b=b, eps=np.float32(1e-5), y=y)


def gen_elementwise() -> None:
    g = torch.Generator().manual_seed(102)
    x = torch.randn(3000, generator=g) * 2.5
    for op, body in te._ELTWISE_BODIES.items():
        if op == "tanh":
            # The body `tl.math.tanh(x)` (triton_emitter.py:456) names a function
            # this Triton release does not have, so the reference cannot run it;
            # the oracle's tanh is pinned to torch.tanh instead.
            continue
        spec = te.KernelSpec(te.KernelKind.ELEMENTWISE, f"ew_{op}")
        ns = _exec(te.emit_elementwise(spec, body=body), f"eltwise {op}")
        y = torch.empty_like(x)
        n = x.numel()
        ns[f"ew_{op}"][((n + 1023) // 1024,)](x, y, n, BLOCK=1024)  # triton_emitter.py:442-449
        _save(f"eltwise_{op}_f32", x=x, y=y)


def gen_gemm() -> None:
    g = torch.Generator().manual_seed(103)
    M, K, N = 96, 80, 72
    for dtype, tdt in (("float32", torch.float32), ("float16", torch.float16)):
        for act, has_bias in ((None, False), ("relu", False), ("gelu", False), ("sigmoid", False),
                              (None, True), ("gelu", True)):
            name = f"gemm_{dtype}_{act or 'none'}_{'bias' if has_bias else 'nobias'}"
            spec = te.KernelSpec(te.KernelKind.GEMM, "gk", dtype=dtype, has_bias=has_bias, activation=act)
            src = te.emit_gemm(spec)
            src = src.replace("bias = tl.load(bias_ptr + rn, mask=mask_n, other=0.0)", "bias = tl.load(bias_ptr + rn)")
            src = "\n".join("    assert K == K2" if ln.strip().startswith("assert K == K2") else ln
                            for ln in src.splitlines())
            ns = _exec(src, name)
            a = torch.randn(M, K, generator=g).to(tdt)
            b = torch.randn(K, N, generator=g).to(tdt)
            bias = (0.1 * torch.randn(N, generator=g)).to(tdt)
            c = torch.empty(M, N, dtype=tdt)
            t = spec.tile
            grid = (((M + t.BLOCK_M - 1) // t.BLOCK_M) * ((N + t.BLOCK_N - 1) // t.BLOCK_N),)
            args = [a, b, c] + ([bias] if has_bias else [])
            try:
                ns["gk"][grid](*args, a.stride(0), a.stride(1), b.stride(0), b.stride(1), c.stride(0), c.stride(1),
                               M, N, K, BLOCK_M=t.BLOCK_M, BLOCK_N=t.BLOCK_N, BLOCK_K=t.BLOCK_K)
            except Exception as e:  # the reference itself cannot run this variant
                # fp16 output + erf/exp activation: the template casts the
                # accumulator to fp16 before the activation (lines 145-147) and
                # tl.math.erf / tl.math.exp accept fp32/fp64 only.
                print(f"skipped {name}: reference kernel fails: {str(e).splitlines()[-1][:120]}")
                continue
            arrays = dict(a=a, b=b, c=c)
            if has_bias:
                arrays["bias"] = bias
            _save(name, **arrays)


def gen_attention() -> None:
    g = torch.Generator().manual_seed(104)
    B, H, S, D = 1, 2, 128, 64
    for dtype, tdt in (("float32", torch.float32), ("float16", torch.float16)):
        spec = te.KernelSpec(te.KernelKind.ATTENTION, "fa", dtype=dtype, tile=te.TileConfig(BLOCK_SEQ=64, HEAD_DIM=D))
        ns = _exec(te.emit_attention(spec), "attention")
        for causal in (False, True):
            q = torch.randn(B, H, S, D, generator=g).to(tdt)
            k = torch.randn(B, H, S, D, generator=g).to(tdt)
            v = torch.randn(B, H, S, D, generator=g).to(tdt)
            o = torch.empty_like(q)
            scale = 1.0 / (D ** 0.5)  # triton_emitter.py:302
            ns["fa"][((S + 63) // 64, B * H)](
                q, k, v, o, scale, *q.stride(), *k.stride(), *v.stride(), *o.stride(), B, H, S, S, D,
                BLOCK_M=64, BLOCK_N=64, HEAD_DIM=D, IS_CAUSAL=causal)
            _save(f"attention_{dtype}_{'causal' if causal else 'full'}", q=q, k=k, v=v, o=o)


def main() -> None:
    if not (REF / "lunara" / "codegen" / "triton_emitter.py").exists():
        raise SystemExit(f"reference checkout not found under {REF}")
    gen_softmax()
    gen_layernorm()
    gen_elementwise()
    gen_gemm()
    gen_attention()


if __name__ == "__main__":
    main()
