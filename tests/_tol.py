"""Tolerances of the parity tests against the fp32 CPU oracle.

fp16 outputs: max-abs <= 2e-2 (scaled by the reference's RMS when that is
above 1, e.g. the 4096^3 GEMM whose outputs have std 64) and relative-L2
<= 1e-3. bf16 outputs (8-bit mantissa; output rounding alone gives a
relative-L2 near 1e-3): max-abs <= 6e-2 (same scaling) and relative-L2 <= 5e-3.
fp32 outputs: max-abs <= 1e-4 (scaled) and relative-L2 <= 1e-5.
Index ops are compared bit for bit.

GOLDEN_TOL: the reference's own kernel outputs (tests/golden) as the
expected values instead of the fp32 oracle. For fp16 those outputs are
themselves rounded to fp16 by the reference's kernel, so a comparison
carries two output roundings (the reference's and ours) plus the
reference's fp16 P: relative-L2 is allowed 2e-3 instead of 1e-3. fp32
golden outputs keep the fp32 bound.
"""
import torch

TOL = {
    torch.float16: (2e-2, 1e-3),
    torch.bfloat16: (6e-2, 5e-3),
    torch.float32: (1e-4, 1e-5),
}

# A stack of L layers stores every kernel's output in fp16/bf16 between
# kernels, and each layer's rounding error (relative-L2 ~4e-4 per fp16 block
# against the fp32 oracle) feeds the next layer's input: the errors add up
# like a random walk. Each layer is checked on its own at TOL (its input taken
# from the GPU's previous layer); the end-to-end output of L layers is
# allowed sqrt(L) times TOL's relative-L2 bound.
def stack_rel_l2(dtype, layers: int) -> float:
    return TOL[dtype][1] * layers ** 0.5


GOLDEN_TOL = {
    torch.float16: (2e-2, 2e-3),
    torch.float32: (1e-4, 1e-5),
}


def check_close(out: torch.Tensor, ref: torch.Tensor, dtype: torch.dtype = None, what: str = "",
                max_abs: float = None, rel_l2: float = None):
    dtype = dtype or out.dtype
    a_tol, r_tol = TOL[dtype]
    a_tol = a_tol if max_abs is None else max_abs
    r_tol = r_tol if rel_l2 is None else rel_l2
    o = out.detach().float().cpu()
    r = ref.detach().float().cpu()
    assert o.shape == r.shape, f"{what}: shape {tuple(o.shape)} vs {tuple(r.shape)}"
    assert torch.isfinite(o).all(), f"{what}: non-finite output"
    rms = r.pow(2).mean().sqrt().item()
    scale = max(1.0, rms)
    err = (o - r).abs().max().item()
    rl2 = ((o - r).norm() / r.norm().clamp_min(1e-30)).item()
    assert err <= a_tol * scale, f"{what}: max-abs {err:.3e} > {a_tol * scale:.3e} (rms {rms:.3g})"
    assert rl2 <= r_tol, f"{what}: rel-L2 {rl2:.3e} > {r_tol:.1e}"
    return err, rl2
