"""GPU parity of the GEMM (tcgen05 path and CUDA-core path) against the CPU oracle.

Covers every tile width (BN 64/128/192/256), both B layouts ([K,N] as the
reference launcher passes it, [N,K] as a Linear weight), fp16 and bf16, every
epilogue (bias, each activation, residual), ragged shapes that leave partial
tiles in M, N and K (TMA zero fill), several tiles per persistent CTA, the
benchmark GEMM (4096^3, plain and bias+GELU) and the CUDA-core path for
strides TMA cannot take and for fp32."""
import pytest
import torch

from oracle import inputs, oracle
from tests._tol import check_close

pytestmark = pytest.mark.gpu


def _ops():
    from lunara_b200.runtime import ops
    return ops


def _mk(M, N, K, dtype, seed, layout="kn", scale=1.0):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(M, K, generator=g) * scale).to(dtype)
    b = (torch.randn(K, N, generator=g) * scale).to(dtype) if layout == "kn" else \
        (torch.randn(N, K, generator=g) * scale).to(dtype)
    bias = (0.1 * torch.randn(N, generator=g)).to(dtype)
    res = torch.randn(M, N, generator=g).to(dtype)
    return a, b, bias, res


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("layout", ["kn", "nk"])
@pytest.mark.parametrize("bn", [64, 128, 192, 256])
def test_gemm_tile_widths(dtype, layout, bn):
    M, N, K = 256, 512, 192
    a, b, _, _ = _mk(M, N, K, dtype, bn, layout, scale=0.5)
    c = _ops().gemm(a.cuda(), b.cuda(), b_layout=layout, block_n=bn, cta_pair=1)
    check_close(c, oracle.gemm(a, b, b_layout=layout), dtype, f"gemm bn={bn} {layout}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("layout", ["kn", "nk"])
@pytest.mark.parametrize("bn", [128, 192, 256])
def test_gemm_cta_pair_tiles(dtype, layout, bn):
    """256-row tiles computed by a CTA pair (cta_group::2 MMA), several tiles per pair.
    (N=192 pair tiles take B as [N,K]; with B as [K,N] the request runs on single-CTA tiles.)"""
    M, N, K = 1024, 768, 320
    a, b, bias, res = _mk(M, N, K, dtype, bn + 1, layout, scale=0.5)
    ops = _ops()
    c = ops.gemm(a.cuda(), b.cuda(), bias=bias.cuda(), residual=res.cuda(), b_layout=layout, block_n=bn,
                 cta_pair=2, num_ctas=4)
    check_close(c, oracle.gemm(a, b, bias, residual=res, b_layout=layout), dtype, f"pair gemm bn={bn} {layout}")


@pytest.mark.parametrize("layout", ["kn", "nk"])
@pytest.mark.parametrize("M,N,K", [(300, 136, 72), (129, 512, 1000), (600, 264, 64)])
def test_gemm_cta_pair_ragged(layout, M, N, K):
    a, b, bias, _ = _mk(M, N, K, torch.float16, M + N, layout, scale=0.5)
    for act in (None, "gelu_tanh", "relu"):
        c = _ops().gemm(a.cuda(), b.cuda(), bias=bias.cuda(), activation=act, b_layout=layout, cta_pair=2)
        check_close(c, oracle.gemm(a, b, bias, activation=act, b_layout=layout), torch.float16,
                    f"pair gemm {M}x{N}x{K} {act}")


@pytest.mark.parametrize("layout", ["kn", "nk"])
@pytest.mark.parametrize("M,N,K", [(200, 136, 72), (1, 64, 64), (129, 300, 1000), (64, 8, 8), (300, 1000, 40)])
def test_gemm_ragged_shapes(layout, M, N, K):
    a, b, bias, res = _mk(M, N, K, torch.float16, M + N + K, layout, scale=0.5)
    c = _ops().gemm(a.cuda(), b.cuda(), bias=bias.cuda(), residual=res.cuda(), b_layout=layout)
    check_close(c, oracle.gemm(a, b, bias, residual=res, b_layout=layout), torch.float16, f"gemm {M}x{N}x{K}")


@pytest.mark.parametrize("act", [None, "relu", "gelu", "gelu_tanh", "sigmoid", "tanh"])
@pytest.mark.parametrize("with_res", [False, True])
def test_gemm_epilogues(act, with_res):
    M, N, K = 384, 768, 256
    a, b, bias, res = _mk(M, N, K, torch.float16, 11, "nk", scale=0.3)
    c = _ops().gemm(a.cuda(), b.cuda(), bias=bias.cuda(), residual=res.cuda() if with_res else None,
                    activation=act, b_layout="nk")
    ref = oracle.gemm(a, b, bias, activation=act, residual=res if with_res else None, b_layout="nk")
    check_close(c, ref, torch.float16, f"gemm epilogue {act} res={with_res}")


def test_gemm_many_tiles_per_cta_and_stages():
    ops = _ops()
    M, N, K = 1024, 1024, 512
    a, b, bias, _ = _mk(M, N, K, torch.float16, 12, "kn", scale=0.5)
    ref = oracle.gemm(a, b, bias)
    for bn, stages, ctas in [(128, 2, 3), (256, 3, 5), (64, 8, 1), (192, 5, 7)]:
        c = ops.gemm(a.cuda(), b.cuda(), bias=bias.cuda(), block_n=bn, stages=stages, num_ctas=ctas, cta_pair=1)
        check_close(c, ref, torch.float16, f"gemm bn={bn} stages={stages} ctas={ctas}")


def test_gemm_strided_operands_and_output():
    ops = _ops()
    M, N, K = 256, 256, 128
    g = torch.Generator().manual_seed(13)
    big_a = torch.randn(M, K + 64, generator=g).half()
    big_b = torch.randn(K, N + 128, generator=g).half()
    a, b = big_a[:, 32:32 + K], big_b[:, 64:64 + N]
    c_buf = torch.zeros(M, N + 64, dtype=torch.float16, device="cuda")
    c = c_buf[:, 16:16 + N]
    a_dev = big_a.cuda()[:, 32:32 + K]   # lda = K + 64, base offset 64 bytes
    b_dev = big_b.cuda()[:, 64:64 + N]   # ldb = N + 128, base offset 128 bytes
    ops.gemm(a_dev, b_dev, c)            # ldc = N + 64, base offset 32 bytes
    check_close(c, oracle.gemm(a, b), torch.float16, "strided gemm")
    assert torch.count_nonzero(c_buf[:, :16]) == 0 and torch.count_nonzero(c_buf[:, 16 + N:]) == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_gemm_benchmark_4096(dtype):
    a, b, bias = inputs.gemm_inputs()
    a, b, bias = a.to(dtype), b.to(dtype), bias.to(dtype)
    ops = _ops()
    c = ops.gemm(a.cuda(), b.cuda())
    check_close(c, oracle.gemm(a, b), dtype, "gemm 4096^3")
    c2 = ops.gemm(a.cuda(), b.cuda(), bias=bias.cuda(), activation="gelu_tanh")
    check_close(c2, oracle.gemm(a, b, bias, activation="gelu_tanh"), dtype, "gemm 4096^3 bias+gelu")


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_gemm_simt_path(dtype):
    ops = _ops()
    M, N, K = 70, 33, 45   # K, N not multiples of 8 -> no TMA -> CUDA-core kernel
    a, b, bias, res = _mk(M, N, K, dtype, 14, "kn", scale=0.5)
    c = ops.gemm(a.cuda(), b.cuda(), bias=bias.cuda(), residual=res.cuda(), activation="relu")
    check_close(c, oracle.gemm(a, b, bias, activation="relu", residual=res), dtype, "simt gemm")
    a2, b2, _, _ = _mk(M, N, K, dtype, 15, "nk", scale=0.5)
    check_close(ops.gemm(a2.cuda(), b2.cuda(), b_layout="nk"), oracle.gemm(a2, b2, b_layout="nk"), dtype,
                "simt gemm nk")


def test_gemm_deterministic():
    ops = _ops()
    a, b, bias, _ = _mk(512, 768, 768, torch.float16, 16, "nk")
    c1 = ops.gemm(a.cuda(), b.cuda(), bias=bias.cuda(), b_layout="nk")
    c2 = ops.gemm(a.cuda(), b.cuda(), bias=bias.cuda(), b_layout="nk")
    assert torch.equal(c1, c2)
    assert ops.device_error() == 0


def test_gemm_shape_errors_like_reference():
    ops = _ops()
    a = torch.randn(8, 16).half().cuda()
    b = torch.randn(12, 8).half().cuda()
    with pytest.raises(AssertionError):
        ops.gemm(a, b)
    with pytest.raises(AssertionError):
        ops.gemm(a.cpu(), b.cpu())
