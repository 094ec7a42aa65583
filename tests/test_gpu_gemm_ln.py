"""GPU parity of the fused GEMM + bias + residual + LayerNorm kernel
(lunara_gemm_layernorm) against the CPU oracle's unfused composition
LayerNorm(gemm(A, B, bias, residual)) -- the out_proj + layernorm_attn and
ffn2 + layernorm_ffn pairs of the encoder block (lunara/driver.py:275-283).

Each row's N columns are split over a cluster of N / slice CTAs that
exchange row statistics through distributed shared memory; the cases cover
every slice width (128, 192, 256) and cluster size from 2 to 8, ragged row and
K counts, both B layouts, fp16 and bf16, and grids small enough that every
cluster walks many row blocks (the statistics buffers alternate between
blocks)."""
import pytest
import torch

from lunara_b200.runtime import _lib, ops
from oracle import oracle
from tests._tol import check_close

pytestmark = pytest.mark.gpu


def _case(M, N, K, dtype, seed, bias=True, residual=True, scale=3.0, shift=0.5):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).to(dtype)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(dtype)                 # [N, K] Linear weight
    b = (0.1 * torch.randn(N, generator=g)).to(dtype) if bias else None
    r = (scale * torch.randn(M, N, generator=g) + shift).to(dtype) if residual else None
    gamma = (1.0 + 0.1 * torch.randn(N, generator=g)).to(dtype)
    beta = (0.1 * torch.randn(N, generator=g)).to(dtype)
    return a, w, b, r, gamma, beta


def _ref(a, w, b, r, gamma, beta, eps=1e-5):
    h = oracle.gemm(a, w, b, residual=r, b_layout="nk")
    return oracle.layernorm(h, gamma, beta, eps)


def _cuda(*ts):
    return [t.cuda() if t is not None else None for t in ts]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(4096, 768, 768), (4096, 768, 3072), (1000, 768, 200), (128, 768, 64),
                                   (777, 384, 512), (512, 1024, 256), (640, 512, 320), (300, 2048, 128)])
def test_gemm_layernorm_matches_oracle(dtype, M, N, K):
    a, w, b, r, gamma, beta = _case(M, N, K, dtype, seed=M + N + K)
    y = ops.gemm_layernorm(*_cuda(a, w, gamma, beta), bias=b.cuda(), residual=r.cuda())
    check_close(y, _ref(a, w, b, r, gamma, beta), dtype, f"gemm+layernorm {M}x{N}x{K} {dtype}")


@pytest.mark.parametrize("bias,residual", [(False, False), (True, False), (False, True)])
def test_gemm_layernorm_optional_terms(bias, residual):
    a, w, b, r, gamma, beta = _case(1024, 768, 768, torch.float16, seed=3, bias=bias, residual=residual)
    y = ops.gemm_layernorm(*_cuda(a, w, gamma, beta), bias=b.cuda() if bias else None,
                           residual=r.cuda() if residual else None)
    check_close(y, _ref(a, w, b, r, gamma, beta), torch.float16, f"bias={bias} residual={residual}")


def test_gemm_layernorm_kn_layout():
    a, w, b, r, gamma, beta = _case(2048, 768, 384, torch.float16, seed=4)
    wkn = w.t().contiguous()                                                   # [K, N]
    y = ops.gemm_layernorm(a.cuda(), wkn.cuda(), gamma.cuda(), beta.cuda(), bias=b.cuda(), residual=r.cuda(),
                           b_layout="kn")
    check_close(y, _ref(a, w, b, r, gamma, beta), torch.float16, "gemm+layernorm, B as [K, N]")


@pytest.mark.parametrize("block_n", [128, 192, 256])
def test_gemm_layernorm_each_slice_width(block_n):
    """N = 768 as 6 x 128, 4 x 192 or 3 x 256 columns per cluster."""
    a, w, b, r, gamma, beta = _case(1536, 768, 512, torch.float16, seed=block_n)
    y = ops.gemm_layernorm(*_cuda(a, w, gamma, beta), bias=b.cuda(), residual=r.cuda(), block_n=block_n)
    check_close(y, _ref(a, w, b, r, gamma, beta), torch.float16, f"slice {block_n}")


@pytest.mark.parametrize("num_ctas", [4, 8, 12])
def test_gemm_layernorm_many_blocks_per_cluster(num_ctas):
    """One to three 4-CTA clusters walk all 256 row blocks of a 32768-row problem
    (the 12-layer stack's M), so each statistics buffer is reused many times."""
    a, w, b, r, gamma, beta = _case(32768, 768, 256, torch.float16, seed=num_ctas)
    y = ops.gemm_layernorm(*_cuda(a, w, gamma, beta), bias=b.cuda(), residual=r.cuda(), num_ctas=num_ctas)
    check_close(y, _ref(a, w, b, r, gamma, beta), torch.float16, f"grid {num_ctas}")
    assert ops.device_error() == 0


def test_gemm_layernorm_equals_unfused_kernels():
    """Fused and unfused GPU paths round the same fp16 sum and normalise it in fp32:
    they agree to within one or two output ulps."""
    a, w, b, r, gamma, beta = _case(4096, 768, 768, torch.float16, seed=7)
    ac, wc, bc, rc, gc, bec = _cuda(a, w, b, r, gamma, beta)
    fused = ops.gemm_layernorm(ac, wc, gc, bec, bias=bc, residual=rc)
    h = ops.gemm(ac, wc, bias=bc, residual=rc, b_layout="nk")
    unfused = ops.layernorm(h, gc, bec, 1e-5)
    diff = (fused.float() - unfused.float()).abs().max().item()
    assert diff <= 8e-3, diff


def test_gemm_layernorm_unsupported_width_falls_back():
    """N = 100 fits no cluster split: the C ABI answers UNSUPPORTED without launching,
    and ops.gemm_layernorm runs the GEMM and LayerNorm kernels instead."""
    a, w, b, r, gamma, beta = _case(256, 100, 64, torch.float16, seed=5)
    ac, wc, bc, rc, gc, bec = _cuda(a, w, b, r, gamma, beta)
    y = torch.empty(256, 100, dtype=torch.float16, device="cuda")
    lib = _lib.load()
    rc_ = lib.lunara_gemm_layernorm(ac.data_ptr(), wc.data_ptr(), y.data_ptr(), bc.data_ptr(), rc.data_ptr(),
                                    gc.data_ptr(), bec.data_ptr(), 256, 100, 64, 64, 64, 100, 100, _lib.B_NK,
                                    _lib.F16, 1e-5, None, torch.cuda.current_stream().cuda_stream)
    assert rc_ == _lib.ERR_UNSUPPORTED
    out = ops.gemm_layernorm(ac, wc, gc, bec, bias=bc, residual=rc)
    check_close(out, _ref(a, w, b, r, gamma, beta), torch.float16, "fallback")
