"""ONNX graph -> kernel specs (lunara_b200.frontend.onnx_graph), on CPU.

The onnx package is not available, so the test writes ONNX files itself with
a minimal protobuf encoder (the field numbers of the public ONNX schema), then
checks the kernel list the driver derives from them.
"""
import struct

import pytest

from lunara_b200.codegen.kernel_emitter import KernelKind
from lunara_b200.frontend.onnx_graph import OnnxFormatError, graph_kernel_specs, parse_onnx


# ─────────────────────────────────────────────── minimal protobuf writer ──

def _varint(v: int) -> bytes:
    if v < 0:
        v += 1 << 64
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(num: int, wt: int) -> bytes:
    return _varint((num << 3) | wt)


def _len(num: int, payload: bytes) -> bytes:
    return _key(num, 2) + _varint(len(payload)) + payload


def _s(num: int, text: str) -> bytes:
    return _len(num, text.encode())


def _i(num: int, v: int) -> bytes:
    return _key(num, 0) + _varint(v)


def attr_int(name, v):
    return _s(1, name) + _i(3, v) + _i(20, 2)


def attr_str(name, v):
    return _s(1, name) + _len(4, v.encode()) + _i(20, 3)


def attr_ints(name, vals):
    return _s(1, name) + b"".join(_i(8, v) for v in vals) + _i(20, 7)


def node(op, inputs, outputs, name="", attrs=()):
    b = b"".join(_s(1, t) for t in inputs) + b"".join(_s(2, t) for t in outputs)
    if name:
        b += _s(3, name)
    b += _s(4, op)
    b += b"".join(_len(5, a) for a in attrs)
    return b


def tensor(name, dims, packed=True):
    if packed:
        d = _len(1, b"".join(_varint(x) for x in dims))
    else:
        d = b"".join(_i(1, x) for x in dims)
    return d + _i(2, 10) + _s(8, name)


def value_info(name, dims):
    shape = b"".join(_len(1, _i(1, d)) for d in dims)
    ttype = _i(1, 10) + _len(2, shape)
    return _s(1, name) + _len(2, _len(1, ttype))


def model(nodes, inits, inputs, outputs, name="g"):
    g = b"".join(_len(1, n) for n in nodes) + _s(2, name)
    g += b"".join(_len(5, t) for t in inits)
    g += b"".join(_len(11, v) for v in inputs)
    g += b"".join(_len(12, v) for v in outputs)
    return _i(1, 8) + _len(7, g)


def bert_block(causal=False, hidden=768, heads=12, ffn=3072, act_attrs=(), packed=True):
    """A post-LN encoder block as exporters write it (fused QKV, scale Div, optional mask Add)."""
    hd = hidden // heads
    n = [
        node("MatMul", ["x", "w_qkv"], ["qkv_mm"]),
        node("Add", ["qkv_mm", "b_qkv"], ["qkv"]),
        node("Split", ["qkv"], ["q2", "k2", "v2"], attrs=[attr_int("axis", 2)]),
        node("Reshape", ["q2"], ["q4"], attrs=[attr_ints("shape", [8, 512, heads, hd])]),
        node("Transpose", ["q4"], ["q"]),
        node("Reshape", ["k2"], ["k4"], attrs=[attr_ints("shape", [8, 512, heads, hd])]),
        node("Transpose", ["k4"], ["kt"]),
        node("Reshape", ["v2"], ["v4"], attrs=[attr_ints("shape", [8, 512, heads, hd])]),
        node("Transpose", ["v4"], ["v"]),
        node("MatMul", ["q", "kt"], ["s"]),
        node("Div", ["s", "scale"], ["s_scaled"]),
    ]
    att_in = "s_scaled"
    if causal:
        n.append(node("Add", ["s_scaled", "causal_mask"], ["s_masked"]))
        att_in = "s_masked"
    n += [
        node("Softmax", [att_in], ["p"], attrs=[attr_int("axis", -1)]),
        node("MatMul", ["p", "v"], ["o4"]),
        node("Transpose", ["o4"], ["o3"]),
        node("Reshape", ["o3"], ["o"]),
        node("MatMul", ["o", "w_o"], ["h_mm"]),
        node("Add", ["h_mm", "b_o"], ["h_b"]),
        node("Add", ["h_b", "x"], ["h"]),
        node("LayerNormalization", ["h", "ln1_w", "ln1_b"], ["x1"], attrs=[attr_int("axis", -1)]),
        node("MatMul", ["x1", "w_1"], ["f_mm"]),
        node("Add", ["f_mm", "b_1"], ["f_b"]),
        node("Gelu", ["f_b"], ["f"], attrs=list(act_attrs)),
        node("MatMul", ["f", "w_2"], ["g_mm"]),
        node("Add", ["g_mm", "b_2"], ["g_b"]),
        node("Add", ["g_b", "x1"], ["g"]),
        node("LayerNormalization", ["g", "ln2_w", "ln2_b"], ["y"], attrs=[attr_int("axis", -1)]),
    ]
    inits = [tensor("w_qkv", [hidden, 3 * hidden], packed), tensor("b_qkv", [3 * hidden], packed),
             tensor("w_o", [hidden, hidden], packed), tensor("b_o", [hidden], packed),
             tensor("w_1", [hidden, ffn], packed), tensor("b_1", [ffn], packed),
             tensor("w_2", [ffn, hidden], packed), tensor("b_2", [hidden], packed),
             tensor("ln1_w", [hidden]), tensor("ln1_b", [hidden]), tensor("ln2_w", [hidden]),
             tensor("ln2_b", [hidden]), tensor("scale", [])]
    return model(n, inits, [value_info("x", [8, 512, hidden])], [value_info("y", [8, 512, hidden])])


def test_parse_reads_nodes_initializers_and_shapes():
    g = parse_onnx(bert_block())
    assert [n.op_type for n in g.nodes][:3] == ["MatMul", "Add", "Split"]
    assert g.initializers["w_qkv"] == [768, 2304] and g.initializers["b_1"] == [3072]
    assert g.inputs == {"x": [8, 512, 768]} and g.outputs == ["y"]
    ln = [n for n in g.nodes if n.op_type == "LayerNormalization"][0]
    assert ln.attrs["axis"] == -1
    rs = [n for n in g.nodes if n.op_type == "Reshape"][0]
    assert rs.attrs["shape"] == [8, 512, 12, 64]


def test_unpacked_dims_parse_like_packed():
    assert parse_onnx(bert_block(packed=False)).initializers == parse_onnx(bert_block()).initializers


def test_bert_block_gives_the_seven_block_kernels():
    specs = graph_kernel_specs(parse_onnx(bert_block()))
    kinds = [s.kind for s in specs]
    assert kinds == [KernelKind.GEMM, KernelKind.ATTENTION, KernelKind.GEMM, KernelKind.LAYERNORM,
                     KernelKind.GEMM, KernelKind.GEMM, KernelKind.LAYERNORM]
    qkv, attn, out, ln1, ffn1, ffn2, ln2 = specs
    assert qkv.has_bias and qkv.activation is None and qkv.epilogue_ops == []
    assert attn.num_heads == 12 and not attn.is_causal
    assert out.has_bias and out.epilogue_ops == ["residual"]
    assert ffn1.has_bias and ffn1.activation == "gelu"
    assert ffn2.has_bias and ffn2.epilogue_ops == ["residual"]
    assert len({s.name for s in specs}) == 7


def test_tanh_gelu_and_causal_mask():
    specs = graph_kernel_specs(parse_onnx(bert_block(causal=True, act_attrs=[attr_str("approximate", "tanh")])))
    attn = [s for s in specs if s.kind == KernelKind.ATTENTION][0]
    assert attn.is_causal
    assert [s.activation for s in specs if s.kind == KernelKind.GEMM] == [None, None, "gelu_tanh", None]


def test_gemm_op_bias_and_standalone_ops():
    n = [node("Gemm", ["a", "w", "b"], ["c"], attrs=[attr_int("transB", 1)]),
         node("Relu", ["c"], ["r"]),
         node("Softmax", ["r"], ["sm"]),
         node("Conv", ["sm", "k"], ["cv"])]
    inits = [tensor("w", [256, 128]), tensor("b", [256]), tensor("k", [8, 4, 3, 3])]
    specs = graph_kernel_specs(parse_onnx(model(n, inits, [value_info("a", [64, 128])], [value_info("cv", [1])])))
    assert [s.kind for s in specs] == [KernelKind.GEMM, KernelKind.SOFTMAX, KernelKind.CONV2D]
    assert specs[0].has_bias and specs[0].activation == "relu"


def test_elementwise_ops_without_gemm():
    n = [node("Add", ["a", "b"], ["c"]), node("Tanh", ["c"], ["d"])]
    specs = graph_kernel_specs(parse_onnx(model(n, [], [], [])))
    assert [s.kind for s in specs] == [KernelKind.ELEMENTWISE, KernelKind.ELEMENTWISE]
    assert specs[1].activation == "tanh"


@pytest.mark.parametrize("data", [b"", b"\x07\x07\x07", b"not a protobuf at all \xff\xff", _i(1, 8)])
def test_non_onnx_bytes_raise(data):
    with pytest.raises(OnnxFormatError):
        parse_onnx(data)


def test_compiler_uses_the_graph_and_falls_back(tmp_path):
    from lunara_b200.driver import Compiler
    path = tmp_path / "block.onnx"
    path.write_bytes(bert_block(causal=True))
    cm = Compiler(dtype="float16").compile(str(path), output_dir=str(tmp_path / "out"))
    assert [s.kind for s in cm.kernel_specs].count(KernelKind.GEMM) == 4
    assert any(s.kind == KernelKind.ATTENTION and s.is_causal for s in cm.kernel_specs)
    for s in cm.kernel_specs:
        assert callable(cm.get_launch_fn(s.name))
    bad = tmp_path / "bad.onnx"
    bad.write_bytes(b"\x07\x07\x07")
    cm2 = Compiler(dtype="float16").compile(str(bad), output_dir=str(tmp_path / "out2"))
    assert [s.name for s in cm2.kernel_specs] == ["qkv_proj", "flash_attn", "out_proj", "layernorm_attn",
                                                  "ffn1", "ffn2", "layernorm_ffn"]
