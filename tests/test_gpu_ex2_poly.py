"""The attention softmax computes part of its exponentials with a cubic on the
FMA pipe instead of the MUFU unit (lunara_b200/csrc/common.cuh ex2_poly /
ex2_poly2: 2^x = 2^j * p(f), j = rint(x), f in [-0.5, 0.5], p a cubic fitted to
minimise relative error, stated maximum 7.5e-5). These tests bound its error
against float64 exp2 over the softmax's input range: exponents of scores minus
a running maximum that may trail the true maximum by up to 2^8, so x <= 8.
Relative error is bounded on [-125, 8], where every result is a normal float;
on [-126, -125] the scaled result can fall into the subnormal encoding (p(0)
is slightly below 1), so the error there is bounded in absolute terms (these
values are ~1e-38 and vanish in the 16-bit P anyway). Outside the range the
result is what MUFU ex2.approx.ftz gives: exactly 0 below -126 (a masked -inf
score contributes a zero probability, in bf16 P too) and NaN for NaN.
"""
import pytest
import torch

from lunara_b200.runtime import _lib

pytestmark = pytest.mark.gpu


def _run(x: torch.Tensor, pair: int) -> torch.Tensor:
    fn = _lib.load().lunara_selftest_ex2_poly
    y = torch.empty_like(x)
    rc = fn(x.data_ptr(), y.data_ptr(), x.numel(), pair, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("pair", [0, 1, 2])
def test_ex2_poly_relative_error(pair):
    g = torch.Generator().manual_seed(13)
    dense = torch.linspace(-125.0, 8.0, 1 << 20, dtype=torch.float32)
    rand = torch.rand(1 << 20, generator=g) * 133.0 - 125.0
    near_int = torch.arange(-125, 9, dtype=torch.float32).repeat_interleave(8) + \
        torch.tensor([-0.5, -0.49999, -1e-6, 0.0, 1e-6, 0.25, 0.49999, 0.5]).repeat(134)
    x = torch.cat([dense, rand, near_int.clamp(-125.0, 8.0)]).cuda()
    y = _run(x, pair).double().cpu()
    ref = torch.exp2(x.double().cpu())
    rel = ((y - ref).abs() / ref).max().item()
    assert rel <= 1.0e-4, rel
    low = torch.linspace(-126.0, -125.0, 1 << 12, dtype=torch.float32).cuda()
    err = (_run(low, pair).double().cpu() - torch.exp2(low.double().cpu())).abs().max().item()
    assert err <= 2.0 ** -126, err


def test_ex2_poly_pair_equals_scalar():
    x = (torch.rand(1 << 16, generator=torch.Generator().manual_seed(14)) * 134.0 - 126.0).cuda()
    assert torch.equal(_run(x, 0).view(torch.int32), _run(x, 1).view(torch.int32))
    # on [-126, 8] the clamped form the softmax runs is the same function
    assert torch.equal(_run(x, 1).view(torch.int32), _run(x, 2).view(torch.int32))


def test_ex2_poly_clamped_form_below_range():
    """The softmax's clamped form gives a tiny non-negative value below -126 (-inf included);
    the softmax zeroes masked columns itself where bf16 would keep it."""
    below = torch.tensor([-126.5, -200.0, float("-inf"), -1.0e30], dtype=torch.float32).cuda()
    y = _run(below, 2).cpu()
    assert torch.isfinite(y).all() and (y >= 0).all() and (y <= 2.0 ** -125).all(), y


@pytest.mark.parametrize("pair", [0, 1])
def test_ex2_poly_underflow_and_nan(pair):
    below = torch.tensor([-126.5, -127.5, -200.0, -1.0e30, float("-inf"), -150.25], dtype=torch.float32).cuda()
    y = _run(below, pair).cpu()
    assert torch.equal(y, torch.zeros_like(y)), y
    edge = _run(torch.tensor([-126.0, -126.0], dtype=torch.float32).cuda(), pair).cpu()
    assert ((edge - 2.0 ** -126).abs() <= 2.0 ** -135).all(), edge
    nan = _run(torch.tensor([float("nan"), 1.0], dtype=torch.float32).cuda(), pair).cpu()
    assert torch.isnan(nan[0]) and nan[1].item() == pytest.approx(2.0, rel=1e-4), nan
