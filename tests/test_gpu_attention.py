"""GPU parity of scaled-dot-product attention against the CPU oracle.

The tcgen05 kernel (head dim 64, fp16/bf16) is checked causal and non-causal,
at sequence lengths that fill whole 256-query CTAs, half CTAs and ragged
tails in both the query and the key dimension, with Q/K/V read in place from
a fused [B, S, 3, H, D] projection and the output written as [B, S, H, D],
and at the benchmark shape (B2 H12 S2048). The CUDA-core kernel covers other
head dims and fp32. The reference's own attention kernel outputs (golden
fixtures) are matched as well."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import inputs, oracle
from tests._tol import GOLDEN_TOL, check_close

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _ops():
    from lunara_b200.runtime import ops
    return ops


def _qkv(B, H, Sq, Skv, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, Sq, D, generator=g).to(dtype)
    k = torch.randn(B, H, Skv, D, generator=g).to(dtype)
    v = torch.randn(B, H, Skv, D, generator=g).to(dtype)
    return q, k, v


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("S", [128, 256, 512, 200, 777])
def test_attention_tcgen05(dtype, causal, S):
    q, k, v = _qkv(1, 3, S, S, 64, dtype, S)
    o = _ops().attention(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    check_close(o, oracle.attention(q, k, v, causal), dtype, f"attention S={S} causal={causal}")


@pytest.mark.parametrize("Sq,Skv", [(128, 384), (300, 129), (64, 1000)])
def test_attention_cross_lengths(Sq, Skv):
    q, k, v = _qkv(2, 2, Sq, Skv, 64, torch.float16, Sq + Skv)
    o = _ops().attention(q.cuda(), k.cuda(), v.cuda())
    check_close(o, oracle.attention(q, k, v), torch.float16, f"attention {Sq}x{Skv}")


@pytest.mark.parametrize("Sq,Skv", [(300, 129), (129, 300), (257, 640)])
def test_attention_cross_lengths_causal(Sq, Skv):
    """Causal mask on absolute positions (key <= query) with different query / key lengths."""
    q, k, v = _qkv(2, 3, Sq, Skv, 64, torch.float16, 7 * Sq + Skv)
    o = _ops().attention(q.cuda(), k.cuda(), v.cuda(), causal=True)
    check_close(o, oracle.attention(q, k, v, True), torch.float16, f"causal attention {Sq}x{Skv}")


@pytest.mark.parametrize("causal", [False, True])
def test_attention_many_items_bf16(causal):
    """More 128-row work items than SMs (ragged last tile): persistent CTAs take several items."""
    q, k, v = _qkv(3, 8, 1000, 1000, 64, torch.bfloat16, 5)
    o = _ops().attention(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    check_close(o, oracle.attention(q, k, v, causal), torch.bfloat16, f"bf16 attention B3H8S1000 causal={causal}")


def test_attention_fused_qkv_layout():
    ops = _ops()
    B, S, H, D = 2, 384, 4, 64
    g = torch.Generator().manual_seed(21)
    qkv = torch.randn(B, S, 3, H, D, generator=g).half()
    dev = qkv.cuda()
    q, k, v = (dev[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    out = torch.empty(B, S, H, D, dtype=torch.float16, device="cuda")
    ops.attention(q, k, v, out=out.permute(0, 2, 1, 3))
    rq, rk, rv = (qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    ref = oracle.attention(rq, rk, rv).permute(0, 2, 1, 3)
    check_close(out, ref, torch.float16, "attention on fused qkv")


@pytest.mark.parametrize("causal", [False, True])
def test_attention_benchmark_shape(causal):
    q, k, v = inputs.attention_inputs()
    q, k, v = q.half(), k.half(), v.half()
    o = _ops().attention(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    check_close(o, oracle.attention(q, k, v, causal), torch.float16, f"attention B2H12S2048 causal={causal}")


@pytest.mark.parametrize("D,dtype", [(32, torch.float16), (128, torch.float16), (64, torch.float32),
                                     (80, torch.bfloat16)])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_simt_path(D, dtype, causal):
    q, k, v = _qkv(1, 2, 100, 100, D, dtype, D)
    o = _ops().attention(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    check_close(o, oracle.attention(q, k, v, causal), dtype, f"simt attention D={D}")


@pytest.mark.parametrize("name", ["attention_float16_full", "attention_float16_causal",
                                  "attention_float32_full", "attention_float32_causal"])
def test_attention_matches_reference_golden(name):
    z = np.load(GOLDEN / f"{name}.npz")
    q, k, v, o = (torch.from_numpy(z[n]) for n in ("q", "k", "v", "o"))
    causal = name.endswith("causal")
    out = _ops().attention(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    a_tol, r_tol = GOLDEN_TOL[q.dtype]
    check_close(out, o, q.dtype, name, max_abs=a_tol, rel_l2=r_tol)


def test_attention_deterministic_and_no_device_error():
    ops = _ops()
    q, k, v = _qkv(2, 4, 512, 512, 64, torch.float16, 3)
    o1 = ops.attention(q.cuda(), k.cuda(), v.cuda())
    o2 = ops.attention(q.cuda(), k.cuda(), v.cuda())
    assert torch.equal(o1, o2)
    assert ops.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_nan_score_poisons_its_rows_only(dtype, causal):
    """A NaN in one key makes every score against it NaN: the softmax of each row that
    sees that key is NaN (as torch's is), whichever pipe computed its exponential; rows
    that do not see it (causal, earlier queries) and other heads stay finite and exact."""
    q, k, v = _qkv(1, 2, 384, 384, 64, dtype, 77)
    k[0, 0, 200, 5] = float("nan")
    o = _ops().attention(q.cuda(), k.cuda(), v.cuda(), causal=causal).float().cpu()
    first = 200 if causal else 0
    assert torch.isnan(o[0, 0, first:]).all(dim=-1).all()
    assert torch.isfinite(o[0, 0, :first]).all() and torch.isfinite(o[0, 1]).all()
    ref = oracle.attention(q, k, v, causal)
    check_close(o[0, 1], ref[0, 1], dtype, "head without the NaN")
    if causal:
        check_close(o[0, 0, :first], ref[0, 0, :first], dtype, "rows before the NaN key")
