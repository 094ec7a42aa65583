"""GPU parity of the bandwidth kernels (LayerNorm, Softmax, elementwise, index ops)
against the CPU oracle, through the C ABI. Sizes cover the benchmark shapes
(16384x768 LayerNorm, 16384x3072 bias+GELU) and the edge cases of each kernel:
rows that are not whole 16-byte vectors, rows longer than the warp path,
unaligned pointers (scalar paths), empty inputs, out-of-range gather indices."""
import pytest
import torch

from oracle import inputs, oracle
from tests._tol import check_close

pytestmark = pytest.mark.gpu

DT = [torch.float16, torch.bfloat16, torch.float32]


def _ops():
    from lunara_b200.runtime import ops
    return ops


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("M,N", [(37, 768), (5, 64), (3, 96), (7, 100), (2, 4096), (3, 5000), (1, 8)])
def test_layernorm_shapes(dtype, M, N):
    g = torch.Generator().manual_seed(M * 1000 + N)
    x = (torch.randn(M, N, generator=g) * 2 + 0.3).to(dtype)
    w = (1 + 0.1 * torch.randn(N, generator=g)).to(dtype)
    b = (0.1 * torch.randn(N, generator=g)).to(dtype)
    y = _ops().layernorm(x.cuda(), w.cuda(), b.cuda(), 1e-5)
    check_close(y, oracle.layernorm(x, w, b, 1e-5), dtype, f"layernorm {M}x{N}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_layernorm_benchmark_shape(dtype):
    x, w, b = inputs.layernorm_inputs()
    x, w, b = x.to(dtype), w.to(dtype), b.to(dtype)
    y = _ops().layernorm(x.cuda(), w.cuda(), b.cuda(), 1e-5)
    check_close(y, oracle.layernorm(x, w, b, 1e-5), dtype, "layernorm 16384x768")


def test_layernorm_3d_and_empty():
    ops = _ops()
    x = torch.randn(2, 3, 256).half()
    w, b = torch.ones(256).half(), torch.zeros(256).half()
    y = ops.layernorm(x.cuda(), w.cuda(), b.cuda())
    assert y.shape == x.shape
    check_close(y, oracle.layernorm(x, w, b), torch.float16, "layernorm 3-d")
    e = ops.layernorm(torch.empty(0, 256, dtype=torch.float16, device="cuda"), w.cuda(), b.cuda())
    assert e.shape == (0, 256)


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("M,N", [(33, 512), (6, 100), (4, 64), (2, 4096), (3, 6000)])
def test_softmax(dtype, M, N):
    g = torch.Generator().manual_seed(N)
    x = (torch.randn(M, N, generator=g) * 3).to(dtype)
    y = _ops().softmax(x.cuda())
    check_close(y, oracle.softmax(x), dtype, f"softmax {M}x{N}")


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("act", ["relu", "gelu", "gelu_tanh", "sigmoid", "tanh", "identity"])
def test_unary(dtype, act):
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(10007, generator=g) * 3).to(dtype)
    y = _ops().unary(x.cuda(), act)
    check_close(y, oracle.unary(x, act), dtype, f"unary {act}")


def test_unary_unaligned_and_inplace():
    ops = _ops()
    x = torch.randn(4099).half().cuda()
    xs = x[1:]  # 2-byte offset: scalar path
    check_close(ops.unary(xs, "relu"), oracle.unary(xs.cpu(), "relu"), torch.float16, "unaligned")
    z = torch.randn(4096).half().cuda()
    ref = oracle.unary(z.cpu(), "sigmoid")
    ops.unary(z, "sigmoid", out=z)
    check_close(z, ref, torch.float16, "in place")


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("op", ["add", "mul"])
def test_binary(dtype, op):
    g = torch.Generator().manual_seed(8)
    x = torch.randn(3, 1001, generator=g).to(dtype)
    y = torch.randn(3, 1001, generator=g).to(dtype)
    out = _ops().binary(x.cuda(), y.cuda(), op)
    check_close(out, oracle.binary(x, y, op), dtype, f"binary {op}")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_bias_gelu_benchmark_shape(dtype):
    x, bias = inputs.bias_gelu_inputs()
    x, bias = x.to(dtype), bias.to(dtype)
    y = _ops().bias_act(x.cuda(), bias.cuda(), "gelu_tanh")
    check_close(y, oracle.bias_act(x, bias, "gelu_tanh"), dtype, "bias+gelu 16384x3072")


@pytest.mark.parametrize("act", ["relu", "gelu", "gelu_tanh", "sigmoid", "tanh", "identity"])
@pytest.mark.parametrize("cols", [3072, 100, 7])
def test_bias_act_shapes(act, cols):
    g = torch.Generator().manual_seed(cols)
    x = torch.randn(33, cols, generator=g).half()
    bias = (0.1 * torch.randn(cols, generator=g)).half()
    y = _ops().bias_act(x.cuda(), bias.cuda(), act)
    check_close(y, oracle.bias_act(x, bias, act), torch.float16, f"bias_act {act} cols={cols}")


# ───────────────────────────────────────────────────────────── index ops ──

@pytest.mark.parametrize("dtype,row", [(torch.float16, 768), (torch.float32, 5), (torch.uint8, 3), (torch.int64, 4)])
def test_gather_bit_exact(dtype, row):
    ops = _ops()
    g = torch.Generator().manual_seed(9)
    src = (torch.randn(300, row, generator=g) * 100).to(dtype)
    idx = torch.randint(0, 300, (517,), generator=g)
    out = ops.gather(src.cuda(), idx.cuda())
    assert torch.equal(out.cpu(), oracle.gather(src, idx))


def test_gather_out_of_range_sets_device_error():
    ops = _ops()
    ops.device_error(clear=True)
    src = torch.randn(10, 16).half().cuda()
    idx = torch.tensor([0, 3, 10, 2], dtype=torch.int64).cuda()
    out = ops.gather(src, idx)
    code = ops.device_error(clear=True)
    assert code == 0x301
    assert torch.equal(out[2].cpu(), torch.zeros(16, dtype=torch.float16))
    assert torch.equal(out[[0, 1, 3]].cpu(), src.cpu()[[0, 3, 2]])
    assert ops.device_error(clear=True) == 0


@pytest.mark.parametrize("perm", [(0, 2, 1, 3), (3, 2, 1, 0), (1, 0, 2, 3)])
def test_transpose_copy_bit_exact(perm):
    ops = _ops()
    x = torch.randn(4, 6, 10, 16).half()
    v = x.cuda().permute(*perm)
    out = ops.contiguous_copy(v)
    assert torch.equal(out.cpu(), x.permute(*perm).contiguous())


@pytest.mark.parametrize("starts,ends,steps", [
    ([0, 2, 0], [4, 9, 64], [1, 1, 1]),
    ([1, 0, 3], [4, 10, 64], [2, 3, 5]),
    ([-3, -8, 0], [4, 10, 16], [1, 2, 1]),
])
def test_slice_bit_exact(starts, ends, steps):
    ops = _ops()
    x = torch.arange(4 * 10 * 64, dtype=torch.int32).view(4, 10, 64).to(torch.float16)
    out = ops.slice(x.cuda(), starts, ends, steps)
    norm = [s + n if s < 0 else s for s, n in zip(starts, x.shape)]
    assert torch.equal(out.cpu(), oracle.slice_(x, norm, ends, steps))


def test_qkv_split_and_reshape_bit_exact():
    ops = _ops()
    B, S, H, D = 2, 37, 12, 64
    qkv = torch.randn(B, S, 3 * H * D).half()
    q, k, v = ops.qkv_split(qkv.cuda(), H)
    rq, rk, rv = oracle.qkv_split(qkv, H)
    assert torch.equal(q.cpu(), rq) and torch.equal(k.cpu(), rk) and torch.equal(v.cpu(), rv)
    r = ops.reshape(q.transpose(1, 2), (B, S, H * D))
    assert torch.equal(r.cpu(), rq.transpose(1, 2).reshape(B, S, H * D))


@pytest.mark.parametrize("B,S,H,D,dtype", [(8, 512, 12, 64, torch.float16), (3, 5, 2, 8, torch.bfloat16),
                                           (2, 33, 4, 60, torch.float16), (1, 7, 3, 12, torch.float32)])
def test_qkv_split_shapes_bit_exact(B, S, H, D, dtype):
    """One-launch 16-byte path (head rows a multiple of 16 bytes) and the strided-copy fallback (D=60 fp16,
    D=12 fp32 = 48 bytes: still 16-byte units)."""
    ops = _ops()
    qkv = torch.randn(B, S, 3 * H * D).to(dtype)
    q, k, v = ops.qkv_split(qkv.cuda(), H)
    rq, rk, rv = oracle.qkv_split(qkv, H)
    assert torch.equal(q.cpu(), rq) and torch.equal(k.cpu(), rk) and torch.equal(v.cpu(), rv)
    assert ops.device_error() == 0


def test_library_rejects_bad_arguments_on_gpu():
    from lunara_b200.runtime import _lib
    ops = _ops()
    x = torch.randn(4, 8).half().cuda()
    with pytest.raises(ValueError):
        ops.layernorm(x, torch.ones(8).half().cuda(), torch.zeros(8).half().cuda(), eps=-1.0)
    lib = _lib.load()
    rc = lib.lunara_softmax(x.data_ptr(), x.data_ptr(), 4, 8, 7, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.ERR_INVALID_ARG
    assert b"dtype" in lib.lunara_last_error_string()
