"""Failure paths on the GPU, made to happen without a fault.

Every warp-specialised kernel bounds each mbarrier wait with a %globaltimer
budget; when a wait runs out the kernel records a site code in the library's
device error word, drains its own work and returns, so the context stays
usable. The self-test entry point lunara_selftest_bounded_wait runs that same
wait against a barrier nothing arrives on, with a 1 ms budget; the test checks
that the call returns, that lunara_device_error reports the site code, and
that normal kernels still run and match the oracle afterwards. (The
reference's only failure handling is try/except -> NaN in
CompiledModel.benchmark, lunara/driver.py:83-85.)
"""
import time

import pytest
import torch

from lunara_b200.runtime import _lib, ops
from oracle import inputs, oracle
from tests._tol import check_close

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports_its_site():
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    assert ops.device_error(clear=True) == 0
    t0 = time.perf_counter()
    assert lib.lunara_selftest_bounded_wait(1_000_000, 0x401, stream) == _lib.OK
    code = lib.lunara_device_error(stream, 1)          # synchronizes the stream, then reads and clears
    elapsed = time.perf_counter() - t0
    assert code == 0x401, hex(code)
    assert elapsed < 2.0, elapsed                       # 1 ms budget; far below the 4 s product budget
    assert lib.lunara_device_error(stream, 0) == 0      # cleared
    # The first failure wins: a second self-test with another site is recorded only once cleared.
    assert lib.lunara_selftest_bounded_wait(1_000_000, 0x402, stream) == _lib.OK
    assert lib.lunara_selftest_bounded_wait(1_000_000, 0x403, stream) == _lib.OK
    assert lib.lunara_device_error(stream, 1) == 0x402
    # The context is intact: a GEMM and an attention call still match the oracle.
    a, b, bias = (t.half() for t in inputs.gemm_inputs(512, 384, 256, seed=9))
    c = ops.gemm(a.cuda(), b.cuda(), bias=bias.cuda(), activation="gelu_tanh")
    check_close(c, oracle.gemm(a, b, bias, activation="gelu_tanh"), torch.float16, "GEMM after the self-test")
    q, k, v = (t.half() for t in inputs.attention_inputs(1, 2, 256, 64, seed=10))
    o = ops.attention(q.cuda(), k.cuda(), v.cuda(), causal=True)
    check_close(o, oracle.attention(q, k, v, True), torch.float16, "attention after the self-test")
    assert ops.device_error() == 0


def test_attention_with_broadcast_kv_views():
    """K/V expanded over the batch (stride 0) are valid torch views; the call must not fail
    (the tensor-core path takes only stepped strides, the CUDA-core kernel takes the rest)."""
    g = torch.Generator().manual_seed(17)
    q = torch.randn(3, 4, 200, 64, generator=g).half()
    k1 = torch.randn(1, 4, 300, 64, generator=g).half()
    v1 = torch.randn(1, 4, 300, 64, generator=g).half()
    kx, vx = k1.cuda().expand(3, -1, -1, -1), v1.cuda().expand(3, -1, -1, -1)
    assert kx.stride(0) == 0
    o = ops.attention(q.cuda(), kx, vx)
    check_close(o, oracle.attention(q, k1.expand(3, -1, -1, -1), v1.expand(3, -1, -1, -1)), torch.float16,
                "attention with batch-broadcast K/V")


def test_attention_single_batch_any_batch_stride():
    """A dimension of extent 1 is never stepped: any stride torch reports for it (here a
    sliced batch of 1 with an odd stride) keeps the tensor-core path and the right result."""
    g = torch.Generator().manual_seed(18)
    big = torch.randn(1, 3, 256, 64, generator=g).half().cuda()
    q = big[:, :2]                                      # batch stride 3*256*64, extent 1
    k = torch.randn(1, 2, 256, 64, generator=g).half()
    v = torch.randn(1, 2, 256, 64, generator=g).half()
    o = ops.attention(q, k.cuda(), v.cuda(), causal=True)
    check_close(o, oracle.attention(q.cpu(), k, v, True), torch.float16, "attention, batch of one")
