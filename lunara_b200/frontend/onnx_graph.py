"""ONNX model -> the block's kernel specs, without the onnx package.

The reference's ``Compiler.compile`` lowers an ONNX file through its MLIR
tool and then, in ``_extract_kernel_specs`` (lunara/driver.py:208-216),
ignores the lowered graph and returns the canonical encoder-block kernel
list. This module reads the ONNX file itself and derives the kernel list
from its graph, so a model whose layers differ from BERT-base (sizes, number
of layers, activation, causal mask) gets the kernels it actually needs.

ONNX files are protocol-buffer messages. Only the fields used here are read,
with their numbers from the public ONNX schema (onnx.proto):

  ModelProto      graph = 7
  GraphProto      node = 1, name = 2, initializer = 5, input = 11, output = 12
  NodeProto       input = 1, output = 2, name = 3, op_type = 4, attribute = 5
  AttributeProto  name = 1, f = 2, i = 3, s = 4, ints = 8
  TensorProto     dims = 1, data_type = 2, name = 8
  ValueInfoProto  name = 1, type = 2 -> TypeProto.tensor_type = 1 ->
                  elem_type = 1, shape = 2 -> dim = 1 -> dim_value = 1

Pattern matching over the node list (in graph order; ONNX graphs are stored
topologically sorted):

  MatMul / Gemm with a 2-D initializer weight       -> GEMM
      + Add of a 1-D initializer                    -> has_bias
      + Relu / Gelu / Tanh / Sigmoid                -> activation
      + Add of a non-initializer tensor             -> "residual" epilogue op
  MatMul(Q, K^T) [Mul/Div scale] [Add mask] Softmax MatMul(., V)
                                                    -> ATTENTION (causal when a
                                                       mask or Trilu feeds it)
  Softmax (outside the pattern above)               -> SOFTMAX
  LayerNormalization                                -> LAYERNORM
  Relu / Gelu / Tanh / Sigmoid / Add / Mul left     -> ELEMENTWISE
  Conv                                              -> CONV2D (no emitter, as in
                                                       the reference)

Reshape / Transpose / Split / Gather / Slice / Squeeze / Unsqueeze / Concat
are layout operations: the kernels take strided views (the attention reads
Q, K and V in place from the fused QKV buffer), so they produce no kernel.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, List, Optional, Tuple

from lunara_b200.codegen.kernel_emitter import KernelKind, KernelSpec, TileConfig

# ───────────────────────────────────────────────── protobuf wire format ──


class OnnxFormatError(ValueError):
    """The bytes are not a protobuf message of the expected shape."""


def _varint(buf: bytes, pos: int) -> Tuple[int, int]:
    result = 0
    shift = 0
    while True:
        if pos >= len(buf):
            raise OnnxFormatError("truncated varint")
        b = buf[pos]
        pos += 1
        result |= (b & 0x7F) << shift
        if not b & 0x80:
            return result, pos
        shift += 7
        if shift > 63:
            raise OnnxFormatError("varint longer than 64 bits")


def _fields(buf: bytes) -> List[Tuple[int, int, object]]:
    """(field number, wire type, value) for every field of one message.

    Varints and fixed-width values are returned as ints, length-delimited
    fields as bytes.
    """
    out = []
    pos = 0
    n = len(buf)
    while pos < n:
        key, pos = _varint(buf, pos)
        num, wt = key >> 3, key & 7
        if num == 0:
            raise OnnxFormatError("field number 0")
        if wt == 0:
            v, pos = _varint(buf, pos)
        elif wt == 1:
            if pos + 8 > n:
                raise OnnxFormatError("truncated 64-bit field")
            v = struct.unpack_from("<Q", buf, pos)[0]
            pos += 8
        elif wt == 2:
            ln, pos = _varint(buf, pos)
            if pos + ln > n:
                raise OnnxFormatError("truncated length-delimited field")
            v = buf[pos:pos + ln]
            pos += ln
        elif wt == 5:
            if pos + 4 > n:
                raise OnnxFormatError("truncated 32-bit field")
            v = struct.unpack_from("<I", buf, pos)[0]
            pos += 4
        else:
            raise OnnxFormatError(f"unsupported wire type {wt}")
        out.append((num, wt, v))
    return out


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= (1 << 63) else v


def _ints(entries: List[Tuple[int, int, object]], num: int) -> List[int]:
    """A repeated int64 field, packed or not."""
    vals: List[int] = []
    for n, wt, v in entries:
        if n != num:
            continue
        if wt == 0:
            vals.append(_signed(v))
        elif wt == 2:
            p = 0
            while p < len(v):
                x, p = _varint(v, p)
                vals.append(_signed(x))
    return vals


def _str(entries, num: int, default: str = "") -> str:
    for n, wt, v in entries:
        if n == num and wt == 2:
            return v.decode("utf-8", "replace")
    return default


def _strs(entries, num: int) -> List[str]:
    return [v.decode("utf-8", "replace") for n, wt, v in entries if n == num and wt == 2]


def _msgs(entries, num: int) -> List[bytes]:
    return [v for n, wt, v in entries if n == num and wt == 2]


# ──────────────────────────────────────────────────────────── graph model ──

@dataclass
class OnnxNode:
    op_type: str
    name: str
    inputs: List[str]
    outputs: List[str]
    attrs: Dict[str, object] = field(default_factory=dict)


@dataclass
class OnnxGraph:
    name: str
    nodes: List[OnnxNode]
    initializers: Dict[str, List[int]]        # name -> dims
    inputs: Dict[str, List[int]]              # graph input name -> dims (-1 = symbolic)
    outputs: List[str]


def _attribute(buf: bytes) -> Tuple[str, object]:
    e = _fields(buf)
    name = _str(e, 1)
    for n, wt, v in e:
        if n == 2 and wt == 5:
            return name, struct.unpack("<f", struct.pack("<I", v))[0]
        if n == 3 and wt == 0:
            return name, _signed(v)
        if n == 4 and wt == 2:
            return name, v.decode("utf-8", "replace")
    ints = _ints(e, 8)
    return name, ints if ints else None


def _value_info_dims(buf: bytes) -> Tuple[str, List[int]]:
    e = _fields(buf)
    name = _str(e, 1)
    dims: List[int] = []
    for tbuf in _msgs(e, 2):                         # TypeProto
        for ttbuf in _msgs(_fields(tbuf), 1):        # TypeProto.Tensor
            for sbuf in _msgs(_fields(ttbuf), 2):    # TensorShapeProto
                for dbuf in _msgs(_fields(sbuf), 1):  # Dimension
                    de = _fields(dbuf)
                    vals = [_signed(v) for n, wt, v in de if n == 1 and wt == 0]
                    dims.append(vals[0] if vals else -1)
    return name, dims


def parse_onnx(data: bytes) -> OnnxGraph:
    """Parse the graph of a serialized ONNX ModelProto."""
    model = _fields(data)
    graphs = _msgs(model, 7)
    if not graphs:
        raise OnnxFormatError("no graph in the model")
    g = _fields(graphs[0])
    nodes = []
    for nbuf in _msgs(g, 1):
        ne = _fields(nbuf)
        attrs = dict(_attribute(a) for a in _msgs(ne, 5))
        nodes.append(OnnxNode(op_type=_str(ne, 4), name=_str(ne, 3), inputs=_strs(ne, 1),
                              outputs=_strs(ne, 2), attrs=attrs))
    inits = {}
    for tbuf in _msgs(g, 5):
        te = _fields(tbuf)
        inits[_str(te, 8)] = _ints(te, 1)
    ins = dict(_value_info_dims(v) for v in _msgs(g, 11))
    outs = [_value_info_dims(v)[0] for v in _msgs(g, 12)]
    if not nodes:
        raise OnnxFormatError("the graph has no nodes")
    return OnnxGraph(name=_str(g, 2), nodes=nodes, initializers=inits, inputs=ins, outputs=outs)


def load_onnx(path) -> OnnxGraph:
    return parse_onnx(Path(path).read_bytes())


# ─────────────────────────────────────────────────── graph -> kernel specs ──

_ACTS = {"Relu": "relu", "Gelu": "gelu", "Tanh": "tanh", "Sigmoid": "sigmoid"}
_LAYOUT_OPS = {"Reshape", "Transpose", "Split", "Gather", "Slice", "Squeeze", "Unsqueeze", "Concat",
               "Identity", "Shape", "Constant", "Cast", "Flatten"}


def _consumers(g: OnnxGraph) -> Dict[str, List[int]]:
    cons: Dict[str, List[int]] = {}
    for i, n in enumerate(g.nodes):
        for t in n.inputs:
            cons.setdefault(t, []).append(i)
    return cons


def _is_weight(g: OnnxGraph, t: str) -> bool:
    return t in g.initializers and len(g.initializers[t]) == 2


def _is_bias(g: OnnxGraph, t: str) -> bool:
    return t in g.initializers and len(g.initializers[t]) == 1


def graph_kernel_specs(g: OnnxGraph, dtype: str = "float16", num_heads: int = 0) -> List[KernelSpec]:
    """The kernel list of an ONNX graph (see the module docstring for the patterns)."""
    cons = _consumers(g)
    producer = {o: i for i, n in enumerate(g.nodes) for o in n.outputs}
    used = [False] * len(g.nodes)
    specs: List[KernelSpec] = []
    count: Dict[str, int] = {}
    t_gemm = TileConfig(BLOCK_M=128, BLOCK_N=128, BLOCK_K=32, num_stages=4, num_warps=4)

    def name_of(base: str) -> str:
        k = count.get(base, 0)
        count[base] = k + 1
        return f"{base}_{k}"

    def single_consumer(i: int) -> Optional[int]:
        outs = g.nodes[i].outputs
        c = cons.get(outs[0], []) if outs else []
        return c[0] if len(c) == 1 else None

    def head_count_for(i: int) -> int:
        # Heads: the Reshape feeding attention splits the hidden size into [heads, head_dim];
        # take the largest of its shape attributes' second-to-last entries when present.
        if num_heads:
            return num_heads
        seen = []
        for n in g.nodes:
            if n.op_type == "Reshape" and isinstance(n.attrs.get("shape"), list) and len(n.attrs["shape"]) == 4:
                seen.append(n.attrs["shape"][2])
        return max(seen) if seen else 1

    # Attention: MatMul(Q, K^T) -> [Mul|Div] -> [Add mask | Where] -> Softmax -> MatMul(P, V)
    for i, n in enumerate(g.nodes):
        if used[i] or n.op_type != "Softmax":
            continue
        chain = [i]
        causal = False
        j = producer.get(n.inputs[0])
        while j is not None and g.nodes[j].op_type in ("Add", "Where", "Mul", "Div"):
            op = g.nodes[j]
            if op.op_type in ("Add", "Where"):
                causal = causal or any(
                    (producer.get(t) is not None and g.nodes[producer[t]].op_type == "Trilu") or
                    ("mask" in t.lower()) for t in op.inputs)
            chain.append(j)
            j = producer.get(op.inputs[0])
        if j is None or g.nodes[j].op_type != "MatMul" or _is_weight(g, g.nodes[j].inputs[1]):
            continue
        chain.append(j)
        k = single_consumer(i)
        if k is None or g.nodes[k].op_type != "MatMul" or _is_weight(g, g.nodes[k].inputs[1]):
            continue
        chain.append(k)
        for c in chain:
            used[c] = True
        heads = head_count_for(i)
        specs.append((j, KernelSpec(kind=KernelKind.ATTENTION, name=name_of("attention"),
                                    tile=TileConfig(BLOCK_SEQ=64, HEAD_DIM=64, num_stages=2, num_warps=4),
                                    dtype=dtype, is_causal=causal, num_heads=heads)))

    for i, n in enumerate(g.nodes):
        if used[i]:
            continue
        op = n.op_type
        if op in ("MatMul", "Gemm") and len(n.inputs) >= 2 and _is_weight(g, n.inputs[1]):
            used[i] = True
            has_bias = op == "Gemm" and len(n.inputs) > 2 and _is_bias(g, n.inputs[2])
            act: Optional[str] = None
            epi: List[str] = []
            cur = i
            nxt = single_consumer(cur)
            if nxt is not None and not used[nxt] and g.nodes[nxt].op_type == "Add" and not has_bias and \
                    any(_is_bias(g, t) for t in g.nodes[nxt].inputs):
                has_bias = True
                used[nxt] = True
                cur = nxt
                nxt = single_consumer(cur)
            if nxt is not None and not used[nxt] and g.nodes[nxt].op_type in _ACTS:
                act = _ACTS[g.nodes[nxt].op_type]
                if act == "gelu" and g.nodes[nxt].attrs.get("approximate") == "tanh":
                    act = "gelu_tanh"
                used[nxt] = True
                cur = nxt
                nxt = single_consumer(cur)
            if act is None and nxt is not None and not used[nxt] and g.nodes[nxt].op_type == "Add" and \
                    not any(t in g.initializers for t in g.nodes[nxt].inputs):
                epi.append("residual")
                used[nxt] = True
            specs.append((i, KernelSpec(kind=KernelKind.GEMM, name=name_of("gemm"), tile=t_gemm, dtype=dtype,
                                        has_bias=has_bias, activation=act, epilogue_ops=epi)))
        elif op == "LayerNormalization":
            used[i] = True
            specs.append((i, KernelSpec(kind=KernelKind.LAYERNORM, name=name_of("layernorm"),
                                        tile=TileConfig(num_warps=4), dtype=dtype)))
        elif op == "Softmax":
            used[i] = True
            specs.append((i, KernelSpec(kind=KernelKind.SOFTMAX, name=name_of("softmax"), dtype=dtype)))
        elif op in _ACTS or op in ("Add", "Mul"):
            used[i] = True
            specs.append((i, KernelSpec(kind=KernelKind.ELEMENTWISE, name=name_of(op.lower()), dtype=dtype,
                                        activation=_ACTS.get(op))))
        elif op == "Conv":
            used[i] = True
            specs.append((i, KernelSpec(kind=KernelKind.CONV2D, name=name_of("conv2d"), dtype=dtype)))
    specs.sort(key=lambda p: p[0])
    return [s for _, s in specs]
