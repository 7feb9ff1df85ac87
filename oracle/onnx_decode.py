"""ORACLE (test infrastructure only): an independent protobuf decoder for ONNX ModelProto.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use anything
under oracle/.  The product library parses ONNX in its own C++ reader; this file is a
separate implementation so that a parser bug cannot hide in both.

Decodes the subset of onnx.proto the reference emits (src/Shorokoo/Core/Factory/IR/onnx_IR10.cs):
ModelProto, GraphProto, NodeProto, AttributeProto, TensorProto, ValueInfoProto, FunctionProto.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

import numpy as np

ONNX_TO_NP = {1: np.float32, 2: np.uint8, 3: np.int8, 4: np.uint16, 5: np.int16, 6: np.int32,
              7: np.int64, 9: np.bool_, 10: np.float16, 11: np.float64, 12: np.uint32, 13: np.uint64}


def _read_varint(buf: memoryview, pos: int) -> Tuple[int, int]:
    result = 0
    shift = 0
    while True:
        b = buf[pos]
        pos += 1
        result |= (b & 0x7F) << shift
        if not b & 0x80:
            return result, pos
        shift += 7
        if shift > 70:
            raise ValueError("varint too long")


def _fields(buf: memoryview):
    """Yields (field_no, wire_type, value) where value is int for varint/fixed and memoryview for bytes."""
    pos, n = 0, len(buf)
    while pos < n:
        key, pos = _read_varint(buf, pos)
        no, wt = key >> 3, key & 7
        if wt == 0:
            v, pos = _read_varint(buf, pos)
        elif wt == 1:
            v = buf[pos:pos + 8]
            pos += 8
        elif wt == 2:
            ln, pos = _read_varint(buf, pos)
            if pos + ln > n:
                raise ValueError("truncated length-delimited field")
            v = buf[pos:pos + ln]
            pos += ln
        elif wt == 5:
            v = buf[pos:pos + 4]
            pos += 4
        else:
            raise ValueError(f"unsupported wire type {wt}")
        if pos > n:
            raise ValueError("truncated message")
        yield no, wt, v


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= (1 << 63) else v


def _packed_ints(wt, v) -> List[int]:
    if wt == 0:
        return [_signed(v)]
    out, pos = [], 0
    while pos < len(v):
        x, pos = _read_varint(v, pos)
        out.append(_signed(x))
    return out


@dataclass
class TensorP:
    name: str = ""
    dims: List[int] = field(default_factory=list)
    data_type: int = 0
    raw: Optional[bytes] = None
    floats: List[float] = field(default_factory=list)
    doubles: List[float] = field(default_factory=list)
    int32s: List[int] = field(default_factory=list)
    int64s: List[int] = field(default_factory=list)

    def to_numpy(self) -> np.ndarray:
        dt = ONNX_TO_NP.get(self.data_type)
        if dt is None:
            raise NotImplementedError(f"tensor dtype {self.data_type}")
        shape = tuple(self.dims)
        if self.raw is not None:
            a = np.frombuffer(self.raw, dtype=np.dtype(dt).newbyteorder("<")).astype(dt)
        elif self.data_type == 1:
            a = np.array(self.floats, np.float32)
        elif self.data_type == 11:
            a = np.array(self.doubles, np.float64)
        elif self.data_type == 7:
            a = np.array(self.int64s, np.int64)
        else:
            a = np.array(self.int32s, np.int64).astype(dt)
        return a.reshape(shape).copy()


def decode_tensor(buf) -> TensorP:
    t = TensorP()
    for no, wt, v in _fields(memoryview(buf)):
        if no == 1:
            t.dims += _packed_ints(wt, v)
        elif no == 2:
            t.data_type = v
        elif no == 8:
            t.name = bytes(v).decode()
        elif no == 9:
            t.raw = bytes(v)
        elif no == 4:
            t.floats += list(struct.unpack(f"<{len(v) // 4}f", v)) if wt == 2 else [struct.unpack("<f", v)[0]]
        elif no == 10:
            t.doubles += list(struct.unpack(f"<{len(v) // 8}d", v)) if wt == 2 else [struct.unpack("<d", v)[0]]
        elif no == 5:
            t.int32s += _packed_ints(wt, v)
        elif no == 7:
            t.int64s += _packed_ints(wt, v)
    return t


@dataclass
class AttrP:
    name: str = ""
    type: int = 0
    f: float = 0.0
    i: int = 0
    s: bytes = b""
    t: Optional[TensorP] = None
    g: Optional["GraphP"] = None
    floats: List[float] = field(default_factory=list)
    ints: List[int] = field(default_factory=list)

    def value(self) -> Any:
        return {1: self.f, 2: self.i, 3: self.s, 4: self.t, 5: self.g, 6: self.floats, 7: self.ints}.get(self.type)


def decode_attr(buf) -> AttrP:
    a = AttrP()
    for no, wt, v in _fields(memoryview(buf)):
        if no == 1:
            a.name = bytes(v).decode()
        elif no == 20:
            a.type = v
        elif no == 2:
            a.f = struct.unpack("<f", v)[0]
        elif no == 3:
            a.i = _signed(v)
        elif no == 4:
            a.s = bytes(v)
        elif no == 5:
            a.t = decode_tensor(v)
        elif no == 6:
            a.g = decode_graph(v)
        elif no == 7:
            a.floats += list(struct.unpack(f"<{len(v) // 4}f", v)) if wt == 2 else [struct.unpack("<f", v)[0]]
        elif no == 8:
            a.ints += _packed_ints(wt, v)
    return a


@dataclass
class NodeP:
    op_type: str = ""
    domain: str = ""
    name: str = ""
    inputs: List[str] = field(default_factory=list)
    outputs: List[str] = field(default_factory=list)
    attrs: Dict[str, AttrP] = field(default_factory=dict)

    def attr(self, name, default=None):
        a = self.attrs.get(name)
        return default if a is None else a.value()


def decode_node(buf) -> NodeP:
    n = NodeP()
    for no, wt, v in _fields(memoryview(buf)):
        if no == 1:
            n.inputs.append(bytes(v).decode())
        elif no == 2:
            n.outputs.append(bytes(v).decode())
        elif no == 3:
            n.name = bytes(v).decode()
        elif no == 4:
            n.op_type = bytes(v).decode()
        elif no == 7:
            n.domain = bytes(v).decode()
        elif no == 5:
            a = decode_attr(v)
            n.attrs[a.name] = a
    return n


@dataclass
class ValueInfoP:
    name: str = ""
    elem_type: int = 0
    dims: Optional[List[Any]] = None


def decode_value_info(buf) -> ValueInfoP:
    vi = ValueInfoP()
    for no, wt, v in _fields(memoryview(buf)):
        if no == 1:
            vi.name = bytes(v).decode()
        elif no == 2:
            for no2, _, v2 in _fields(v):
                if no2 == 1:    # tensor_type
                    for no3, _, v3 in _fields(v2):
                        if no3 == 1:
                            vi.elem_type = v3
                        elif no3 == 2:
                            vi.dims = []
                            for no4, _, v4 in _fields(v3):
                                if no4 == 1:
                                    d: Any = None
                                    for no5, _, v5 in _fields(v4):
                                        d = v5 if no5 == 1 else bytes(v5).decode()
                                    vi.dims.append(d)
    return vi


@dataclass
class GraphP:
    name: str = ""
    nodes: List[NodeP] = field(default_factory=list)
    initializers: List[TensorP] = field(default_factory=list)
    inputs: List[ValueInfoP] = field(default_factory=list)
    outputs: List[ValueInfoP] = field(default_factory=list)


def decode_graph(buf) -> GraphP:
    g = GraphP()
    for no, wt, v in _fields(memoryview(buf)):
        if no == 1:
            g.nodes.append(decode_node(v))
        elif no == 2:
            g.name = bytes(v).decode()
        elif no == 5:
            g.initializers.append(decode_tensor(v))
        elif no == 11:
            g.inputs.append(decode_value_info(v))
        elif no == 12:
            g.outputs.append(decode_value_info(v))
    return g


@dataclass
class FunctionP:
    name: str = ""
    domain: str = ""
    inputs: List[str] = field(default_factory=list)
    outputs: List[str] = field(default_factory=list)
    nodes: List[NodeP] = field(default_factory=list)


@dataclass
class ModelP:
    ir_version: int = 0
    opsets: Dict[str, int] = field(default_factory=dict)
    graph: Optional[GraphP] = None
    functions: List[FunctionP] = field(default_factory=list)


def decode_model(buf: bytes) -> ModelP:
    m = ModelP()
    for no, wt, v in _fields(memoryview(buf)):
        if no == 1:
            m.ir_version = v
        elif no == 7:
            m.graph = decode_graph(v)
        elif no == 8:
            d, ver = "", 0
            for no2, _, v2 in _fields(v):
                if no2 == 1:
                    d = bytes(v2).decode()
                elif no2 == 2:
                    ver = v2
            m.opsets[d] = ver
        elif no == 25:
            f = FunctionP()
            for no2, _, v2 in _fields(v):
                if no2 == 1:
                    f.name = bytes(v2).decode()
                elif no2 == 10:
                    f.domain = bytes(v2).decode()
                elif no2 == 4:
                    f.inputs.append(bytes(v2).decode())
                elif no2 == 5:
                    f.outputs.append(bytes(v2).decode())
                elif no2 == 7:
                    f.nodes.append(decode_node(v2))
            m.functions.append(f)
    if m.graph is None:
        raise ValueError("ModelProto has no graph")
    return m
