"""Minimal protobuf wire-format writer for ONNX ModelProto (IR 10, opset 21).

The reference framework serialises its concrete graphs with protobuf-net from the
generated ONNX IR types (src/Shorokoo/Core/Factory/IR/onnx_IR10.cs) in
FastOnnxModelBuilder.BuildInternalOnnxModel (src/Shorokoo/Core/Factory/FastOnnxModelBuilder.cs:165-300).
Neither the `onnx` package nor `torch.onnx` is usable here, so this module writes the
same wire format directly.  Field numbers are the public onnx.proto ones.

Only encoding lives here; the graph builders that decide *what* is emitted are in
``shorokoo_b200.emit.graphs``.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence, Union

import numpy as np

# ONNX TensorProto.DataType numbering (also ShorokooTensorElementType,
# src/Shorokoo/Core/Inference/Abstractions/ShorokooTensorElementType.cs:6-31).
FLOAT, UINT8, INT8, UINT16, INT16, INT32, INT64, STRING, BOOL = 1, 2, 3, 4, 5, 6, 7, 8, 9
FLOAT16, DOUBLE, UINT32, UINT64, BFLOAT16 = 10, 11, 12, 13, 16

NP_TO_ONNX = {
    np.dtype(np.float32): FLOAT, np.dtype(np.uint8): UINT8, np.dtype(np.int8): INT8,
    np.dtype(np.uint16): UINT16, np.dtype(np.int16): INT16, np.dtype(np.int32): INT32,
    np.dtype(np.int64): INT64, np.dtype(np.bool_): BOOL, np.dtype(np.float16): FLOAT16,
    np.dtype(np.float64): DOUBLE, np.dtype(np.uint32): UINT32, np.dtype(np.uint64): UINT64,
}

# AttributeProto.AttributeType
A_FLOAT, A_INT, A_STRING, A_TENSOR, A_GRAPH, A_FLOATS, A_INTS, A_STRINGS = 1, 2, 3, 4, 5, 6, 7, 8


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


def _key(field_no: int, wire: int) -> bytes:
    return _varint((field_no << 3) | wire)


def f_varint(no: int, v: int) -> bytes:
    return _key(no, 0) + _varint(int(v))


def f_bytes(no: int, b: Union[bytes, bytearray, memoryview]) -> bytes:
    b = bytes(b)
    return _key(no, 2) + _varint(len(b)) + b


def f_str(no: int, s: str) -> bytes:
    return f_bytes(no, s.encode("utf-8"))


def f_float(no: int, v: float) -> bytes:
    return _key(no, 5) + struct.pack("<f", float(v))


def f_packed_varints(no: int, vals: Sequence[int]) -> bytes:
    body = b"".join(_varint(int(v)) for v in vals)
    return f_bytes(no, body)


@dataclass
class Tensor:
    """A TensorProto. ``encoding`` picks raw_data (the reference's choice for
    initializers, FastOnnxProtoFactory.cs:120-159) or the typed repeated fields."""
    name: str
    array: np.ndarray
    encoding: str = "raw"      # "raw" | "typed"
    doc: str = ""

    def encode(self) -> bytes:
        a = np.asarray(self.array)
        dt = NP_TO_ONNX[a.dtype]
        out = bytearray()
        if a.ndim:
            out += f_packed_varints(1, a.shape)
        out += f_varint(2, dt)
        if self.name:
            out += f_str(8, self.name)
        if self.doc:
            out += f_str(12, self.doc)
        flat = np.ascontiguousarray(a).reshape(-1)
        if self.encoding == "raw" or dt not in (FLOAT, INT64, INT32, DOUBLE, BOOL):
            out += f_bytes(9, flat.astype(a.dtype.newbyteorder("<"), copy=False).tobytes())
        elif dt == FLOAT:
            out += f_bytes(4, flat.astype("<f4").tobytes())
        elif dt == DOUBLE:
            out += f_bytes(10, flat.astype("<f8").tobytes())
        elif dt == INT64:
            out += f_packed_varints(7, flat.tolist())
        else:  # INT32 / BOOL travel in int32_data
            out += f_packed_varints(5, flat.astype(np.int64).tolist())
        return bytes(out)


@dataclass
class Attr:
    name: str
    value: Any
    kind: Optional[int] = None

    def encode(self) -> bytes:
        v, k = self.value, self.kind
        if k is None:
            if isinstance(v, Graph):
                k = A_GRAPH
            elif isinstance(v, Tensor):
                k = A_TENSOR
            elif isinstance(v, (bool, int, np.integer)):
                k = A_INT
            elif isinstance(v, (float, np.floating)):
                k = A_FLOAT
            elif isinstance(v, str):
                k = A_STRING
            elif isinstance(v, (list, tuple)) and all(isinstance(x, (int, np.integer)) for x in v):
                k = A_INTS
            elif isinstance(v, (list, tuple)):
                k = A_FLOATS
            else:
                raise TypeError(f"cannot infer attribute type for {self.name}={v!r}")
        out = bytearray(f_str(1, self.name))
        out += f_varint(20, k)
        if k == A_INT:
            out += f_varint(3, int(v))
        elif k == A_FLOAT:
            out += f_float(2, v)
        elif k == A_STRING:
            out += f_bytes(4, v.encode() if isinstance(v, str) else v)
        elif k == A_TENSOR:
            out += f_bytes(5, v.encode())
        elif k == A_GRAPH:
            out += f_bytes(6, v.encode())
        elif k == A_INTS:
            out += f_packed_varints(8, v)
        elif k == A_FLOATS:
            out += f_bytes(7, struct.pack(f"<{len(v)}f", *v))
        else:
            raise ValueError(k)
        return bytes(out)


@dataclass
class Node:
    op_type: str
    inputs: List[str]
    outputs: List[str]
    name: str = ""
    attrs: List[Attr] = field(default_factory=list)
    domain: str = ""

    def encode(self) -> bytes:
        out = bytearray()
        for i in self.inputs:
            out += f_str(1, i)
        for o in self.outputs:
            out += f_str(2, o)
        if self.name:
            out += f_str(3, self.name)
        out += f_str(4, self.op_type)
        for a in self.attrs:
            out += f_bytes(5, a.encode())
        if self.domain:
            out += f_str(7, self.domain)
        return bytes(out)


@dataclass
class ValueInfo:
    """Graph inputs carry elem type + rank-only symbolic dims named ``<name>_dim<i>``
    (FastOnnxProtoFactory.CreateGraphInputInfo, FastOnnxProtoFactory.cs:65-96); graph
    outputs are name-only (CreateGraphOutputInfo, :107-113)."""
    name: str
    elem_type: Optional[int] = None
    rank: Optional[int] = None
    dims: Optional[Sequence[Union[int, str]]] = None
    metadata: Dict[str, str] = field(default_factory=dict)

    def encode(self) -> bytes:
        out = bytearray(f_str(1, self.name))
        tp = bytearray()
        if self.elem_type is not None:
            tt = bytearray(f_varint(1, self.elem_type))
            dims = self.dims
            if dims is None and self.rank is not None:
                dims = [f"{self.name}_dim{i}" for i in range(self.rank)]
            if dims is not None:
                shp = bytearray()
                for d in dims:
                    if isinstance(d, str):
                        shp += f_bytes(1, f_str(2, d))
                    else:
                        shp += f_bytes(1, f_varint(1, d))
                tt += f_bytes(2, bytes(shp))
            tp += f_bytes(1, bytes(tt))
        out += f_bytes(2, bytes(tp))
        for k, v in self.metadata.items():
            out += f_bytes(4, f_str(1, k) + f_str(2, v))
        return bytes(out)


@dataclass
class Graph:
    name: str
    nodes: List[Node] = field(default_factory=list)
    initializers: List[Tensor] = field(default_factory=list)
    inputs: List[ValueInfo] = field(default_factory=list)
    outputs: List[ValueInfo] = field(default_factory=list)

    def encode(self) -> bytes:
        parts = [f_bytes(1, n.encode()) for n in self.nodes]
        parts.append(f_str(2, self.name))
        parts += [f_bytes(5, t.encode()) for t in self.initializers]
        parts += [f_bytes(11, v.encode()) for v in self.inputs]
        parts += [f_bytes(12, v.encode()) for v in self.outputs]
        return b"".join(parts)


@dataclass
class Function:
    name: str
    domain: str
    inputs: List[str]
    outputs: List[str]
    nodes: List[Node]
    opsets: Dict[str, int] = field(default_factory=lambda: {"": 21})

    def encode(self) -> bytes:
        out = bytearray(f_str(1, self.name))
        for i in self.inputs:
            out += f_str(4, i)
        for o in self.outputs:
            out += f_str(5, o)
        for n in self.nodes:
            out += f_bytes(7, n.encode())
        for d, v in self.opsets.items():
            out += f_bytes(9, f_str(1, d) + f_varint(2, v))
        out += f_str(10, self.domain)
        return bytes(out)


@dataclass
class Model:
    graph: Graph
    opsets: Dict[str, int] = field(default_factory=lambda: {"": 21})
    functions: List[Function] = field(default_factory=list)
    ir_version: int = 10
    producer: str = "OnnxNet"

    def encode(self) -> bytes:
        parts = [f_varint(1, self.ir_version), f_str(2, self.producer), f_str(3, "0.0.1")]
        parts.append(f_bytes(7, self.graph.encode()))
        for d, v in self.opsets.items():
            parts.append(f_bytes(8, f_str(1, d) + f_varint(2, v)))
        for fn in self.functions:
            parts.append(f_bytes(25, fn.encode()))
        return b"".join(parts)
