"""Writes ONNX models (protobuf wire format) without the onnx package.

The plans this package generates are ordinary ONNX ModelProto messages: the
fields written here are the subset the reference reads
(src/frontend/onnx_to_ir.cc:86-140) and `inferc optimize` writes
(src/cli/main.cpp:200-227): graph nodes with attributes, initializers as
raw_data, graph inputs / outputs with element type and shape, and opset
imports (the default domain plus "inferc" v1 for the fused ops). Field numbers
follow onnx.proto.
"""
from __future__ import annotations

import struct

import numpy as np

FLOAT, UINT8, INT32, INT64, BOOL = 1, 2, 6, 7, 9
_NP = {FLOAT: np.float32, UINT8: np.uint8, INT32: np.int32, INT64: np.int64, BOOL: np.bool_}
_CODE = {np.dtype(np.float32): FLOAT, np.dtype(np.uint8): UINT8, np.dtype(np.int32): INT32,
         np.dtype(np.int64): INT64, np.dtype(np.bool_): BOOL}

# AttributeProto.AttributeType
A_FLOAT, A_INT, A_STRING, A_TENSOR, A_FLOATS, A_INTS = 1, 2, 3, 4, 6, 7


def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1  # negative int64 values take ten bytes
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wire: int) -> bytes:
    return _varint((field << 3) | wire)


def _len(field: int, payload: bytes) -> bytes:
    return _key(field, 2) + _varint(len(payload)) + payload


def _str(field: int, s: str) -> bytes:
    return _len(field, s.encode())


def _int(field: int, v: int) -> bytes:
    return _key(field, 0) + _varint(int(v))


def _packed_ints(field: int, vals) -> bytes:
    return _len(field, b"".join(_varint(int(v)) for v in vals))


def tensor(name: str, array: np.ndarray) -> bytes:
    """TensorProto {dims 1, data_type 2, name 8, raw_data 9}."""
    a = np.asarray(array)  # (ascontiguousarray would turn a scalar into shape [1])
    code = _CODE[a.dtype]
    body = b""
    if a.ndim:
        body += _packed_ints(1, a.shape)
    body += _int(2, code) + _str(8, name)
    raw = a.astype(_NP[code]).tobytes() if code != BOOL else a.astype(np.uint8).tobytes()
    return body + _len(9, raw)


def attr(name: str, value) -> bytes:
    """AttributeProto {name 1, f 2, i 3, s 4, t 5, floats 7, ints 8, type 20}."""
    body = _str(1, name)
    if isinstance(value, float):
        body += _key(2, 5) + struct.pack("<f", value) + _int(20, A_FLOAT)
    elif isinstance(value, (bool, int, np.integer)):
        body += _int(3, int(value)) + _int(20, A_INT)
    elif isinstance(value, str):
        body += _len(4, value.encode()) + _int(20, A_STRING)
    elif isinstance(value, np.ndarray):
        body += _len(5, tensor("", value)) + _int(20, A_TENSOR)
    elif isinstance(value, (list, tuple)) and all(isinstance(v, float) for v in value):
        body += _len(7, b"".join(struct.pack("<f", v) for v in value)) + _int(20, A_FLOATS)
    elif isinstance(value, (list, tuple)):
        body += _packed_ints(8, value) + _int(20, A_INTS)
    else:
        raise TypeError(f"attribute {name}: unsupported value {value!r}")
    return body


def node(op: str, inputs, outputs, name: str = "", domain: str = "", **attrs) -> bytes:
    """NodeProto {input 1, output 2, name 3, op_type 4, attribute 5, domain 7}."""
    body = b"".join(_str(1, i) for i in inputs) + b"".join(_str(2, o) for o in outputs)
    if name:
        body += _str(3, name)
    body += _str(4, op)
    body += b"".join(_len(5, attr(k, v)) for k, v in attrs.items())
    if domain:
        body += _str(7, domain)
    return body


def value_info(name: str, elem_type: int, dims) -> bytes:
    """ValueInfoProto {name 1, type 2 {tensor_type 1 {elem_type 1, shape 2}}};
    a str dim is symbolic (dim_param), an int a fixed dim_value."""
    shape = b""
    for d in dims:
        shape += _len(1, _str(2, d) if isinstance(d, str) else _int(1, d))
    ttype = _int(1, elem_type) + _len(2, shape)
    return _str(1, name) + _len(2, _len(1, ttype))


class GraphBuilder:
    """Accumulates nodes / initializers and serialises a ModelProto."""

    def __init__(self, name: str):
        self.name = name
        self.nodes: list[bytes] = []
        self.inits: list[bytes] = []
        self.inputs: list[bytes] = []
        self.outputs: list[bytes] = []
        self.op_counts: dict[str, int] = {}
        self._n = 0
        self._consts: dict[tuple, str] = {}

    def fresh(self, stem: str) -> str:
        self._n += 1
        return f"{stem}_{self._n}"

    def init(self, name: str, array: np.ndarray) -> str:
        self.inits.append(tensor(name, array))
        return name

    def const_i64(self, values) -> str:
        """A small int64 initializer (shape operands: Reshape targets, axes)."""
        key = ("i64", tuple(int(v) for v in np.atleast_1d(values)), np.ndim(values))
        if key not in self._consts:
            self._consts[key] = self.init(self.fresh("const"), np.asarray(values, np.int64))
        return self._consts[key]

    def const_f32(self, value: float) -> str:
        key = ("f32", float(value))
        if key not in self._consts:
            self._consts[key] = self.init(self.fresh("constf"), np.asarray(value, np.float32))
        return self._consts[key]

    def add(self, op: str, inputs, n_out: int = 1, domain: str = "", outputs=None,
            **attrs) -> list[str]:
        outs = list(outputs) if outputs is not None else [self.fresh(op.lower())
                                                           for _ in range(n_out)]
        self.nodes.append(node(op, inputs, outs, name=self.fresh(op), domain=domain, **attrs))
        self.op_counts[op] = self.op_counts.get(op, 0) + 1
        return outs

    def one(self, op: str, inputs, domain: str = "", **attrs) -> str:
        return self.add(op, inputs, 1, domain, **attrs)[0]

    def input(self, name: str, elem_type: int, dims) -> str:
        self.inputs.append(value_info(name, elem_type, dims))
        return name

    def output(self, name: str, elem_type: int, dims) -> str:
        self.outputs.append(value_info(name, elem_type, dims))
        return name

    def model(self, opsets=(("", 17), ("inferc", 1)), producer="inferc_b200") -> bytes:
        graph = (b"".join(_len(1, n) for n in self.nodes) + _str(2, self.name) +
                 b"".join(_len(5, t) for t in self.inits) +
                 b"".join(_len(11, v) for v in self.inputs) +
                 b"".join(_len(12, v) for v in self.outputs))
        ops = b"".join(_len(8, (_str(1, d) if d else b"") + _int(2, v)) for d, v in opsets)
        return _int(1, 8) + _str(2, producer) + _len(7, graph) + ops
