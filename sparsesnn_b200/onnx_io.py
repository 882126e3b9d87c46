"""Plugin-mode ONNX files without the ``onnx`` package: a reader and a writer
of the protobuf wire format for the subset of ``onnx.proto`` that SNN
graphs use (model, graph, nodes with attributes, initializer tensors, value
infos with static shapes).

The reader returns objects with the field names of the ``onnx`` Python API
(``model.graph.node[i].op_type``, ``.input``, ``.attribute[j].f`` /
``.i`` / ``.ints`` / ``.t``, ``graph.initializer``,
``vi.type.tensor_type.shape.dim[k].dim_value``, ``HasField``), so code
written against ``onnx.load`` -- the reference's ``sengine/parser.py`` --
reads these files unchanged; ``to_array`` is ``numpy_helper.to_array``.

Field numbers follow the public ``onnx.proto`` (ModelProto.graph = 7,
GraphProto.node = 1 / initializer = 5 / input = 11 / output = 12 /
value_info = 13, NodeProto.input = 1 / output = 2 / name = 3 / op_type = 4 /
attribute = 5 / domain = 7, AttributeProto.name = 1 / f = 2 / i = 3 / s = 4 /
t = 5 / floats = 7 / ints = 8 / type = 20, TensorProto.dims = 1 /
data_type = 2 / float_data = 4 / int64_data = 7 / name = 8 / raw_data = 9).
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

# AttributeProto.AttributeType
A_FLOAT, A_INT, A_STRING, A_TENSOR, A_GRAPH, A_FLOATS, A_INTS, A_STRINGS = 1, 2, 3, 4, 5, 6, 7, 8
# TensorProto.DataType
T_FLOAT, T_UINT8, T_INT8, T_INT32, T_INT64, T_FLOAT16, T_DOUBLE = 1, 2, 3, 6, 7, 10, 11
_NP = {T_FLOAT: np.float32, T_UINT8: np.uint8, T_INT8: np.int8, T_INT32: np.int32,
       T_INT64: np.int64, T_FLOAT16: np.float16, T_DOUBLE: np.float64}


# ------------------------------------------------------------------ wire format
def _varint(buf, pos):
    x = shift = 0
    while True:
        b = buf[pos]
        pos += 1
        x |= (b & 0x7F) << shift
        if b < 0x80:
            return x, pos
        shift += 7
        if shift > 70:
            raise ValueError("malformed varint")


def _fields(buf):
    """Yield (field number, wire type, value) of one message; value is an int
    (varint / fixed) or a memoryview (length-delimited)."""
    pos, n = 0, len(buf)
    while pos < n:
        key, pos = _varint(buf, pos)
        fno, wt = key >> 3, key & 7
        if wt == 0:
            v, pos = _varint(buf, pos)
        elif wt == 1:
            v = struct.unpack_from("<Q", buf, pos)[0]
            pos += 8
        elif wt == 2:
            ln, pos = _varint(buf, pos)
            if pos + ln > n:
                raise ValueError("truncated field")
            v = buf[pos:pos + ln]
            pos += ln
        elif wt == 5:
            v = struct.unpack_from("<I", buf, pos)[0]
            pos += 4
        else:
            raise ValueError(f"unsupported wire type {wt}")
        yield fno, wt, v


def _signed64(v):
    return v - (1 << 64) if v >= 1 << 63 else v


def _packed_varints(v):
    out, pos = [], 0
    while pos < len(v):
        x, pos = _varint(v, pos)
        out.append(_signed64(x))
    return out


class _Msg:
    _repeated: tuple = ()

    def __init__(self):
        for name in self._repeated:
            setattr(self, name, [])

    def HasField(self, name):  # noqa: N802 - onnx API name
        return getattr(self, name, None) is not None


class Dimension(_Msg):
    def __init__(self, buf=b""):
        self.dim_value, self.dim_param = 0, ""
        for f, wt, v in _fields(buf):
            if f == 1:
                self.dim_value = _signed64(v)
            elif f == 2:
                self.dim_param = bytes(v).decode()


class TensorShape(_Msg):
    _repeated = ("dim",)

    def __init__(self, buf=b""):
        super().__init__()
        for f, wt, v in _fields(buf):
            if f == 1:
                self.dim.append(Dimension(v))


class TensorType(_Msg):
    def __init__(self, buf=b""):
        self.elem_type, self.shape = 0, None
        for f, wt, v in _fields(buf):
            if f == 1:
                self.elem_type = v
            elif f == 2:
                self.shape = TensorShape(v)


class TypeProto(_Msg):
    def __init__(self, buf=b""):
        self.tensor_type = None
        for f, wt, v in _fields(buf):
            if f == 1:
                self.tensor_type = TensorType(v)
        if self.tensor_type is None:
            self.tensor_type = TensorType()


class ValueInfo(_Msg):
    def __init__(self, buf=b""):
        self.name, self.type = "", TypeProto()
        for f, wt, v in _fields(buf):
            if f == 1:
                self.name = bytes(v).decode()
            elif f == 2:
                self.type = TypeProto(v)


class Tensor(_Msg):
    _repeated = ("dims", "float_data", "int64_data", "int32_data")

    def __init__(self, buf=b""):
        super().__init__()
        self.data_type, self.name, self.raw_data = 0, "", b""
        for f, wt, v in _fields(buf):
            if f == 1:
                self.dims.extend(_packed_varints(v) if wt == 2 else [_signed64(v)])
            elif f == 2:
                self.data_type = v
            elif f == 4:
                self.float_data.extend(np.frombuffer(bytes(v), "<f4").tolist() if wt == 2
                                       else [struct.unpack("<f", struct.pack("<I", v))[0]])
            elif f == 5:
                self.int32_data.extend(_packed_varints(v) if wt == 2 else [_signed64(v)])
            elif f == 7:
                self.int64_data.extend(_packed_varints(v) if wt == 2 else [_signed64(v)])
            elif f == 8:
                self.name = bytes(v).decode()
            elif f == 9:
                self.raw_data = bytes(v)


class Attribute(_Msg):
    _repeated = ("floats", "ints", "strings")

    def __init__(self, buf=b""):
        super().__init__()
        self.name, self.type, self.f, self.i, self.s, self.t = "", 0, 0.0, 0, b"", None
        for f, wt, v in _fields(buf):
            if f == 1:
                self.name = bytes(v).decode()
            elif f == 2:
                self.f = struct.unpack("<f", struct.pack("<I", v))[0]
            elif f == 3:
                self.i = _signed64(v)
            elif f == 4:
                self.s = bytes(v)
            elif f == 5:
                self.t = Tensor(v)
            elif f == 7:
                self.floats.extend(np.frombuffer(bytes(v), "<f4").tolist() if wt == 2
                                   else [struct.unpack("<f", struct.pack("<I", v))[0]])
            elif f == 8:
                self.ints.extend(_packed_varints(v) if wt == 2 else [_signed64(v)])
            elif f == 9:
                self.strings.append(bytes(v))
            elif f == 20:
                self.type = v


class Node(_Msg):
    _repeated = ("input", "output", "attribute")

    def __init__(self, buf=b""):
        super().__init__()
        self.name, self.op_type, self.domain = "", "", ""
        for f, wt, v in _fields(buf):
            if f == 1:
                self.input.append(bytes(v).decode())
            elif f == 2:
                self.output.append(bytes(v).decode())
            elif f == 3:
                self.name = bytes(v).decode()
            elif f == 4:
                self.op_type = bytes(v).decode()
            elif f == 5:
                self.attribute.append(Attribute(v))
            elif f == 7:
                self.domain = bytes(v).decode()


class Graph(_Msg):
    _repeated = ("node", "initializer", "input", "output", "value_info")

    def __init__(self, buf=b""):
        super().__init__()
        self.name = ""
        for f, wt, v in _fields(buf):
            if f == 1:
                self.node.append(Node(v))
            elif f == 2:
                self.name = bytes(v).decode()
            elif f == 5:
                self.initializer.append(Tensor(v))
            elif f == 11:
                self.input.append(ValueInfo(v))
            elif f == 12:
                self.output.append(ValueInfo(v))
            elif f == 13:
                self.value_info.append(ValueInfo(v))


class Model(_Msg):
    def __init__(self, buf=b""):
        self.ir_version, self.producer_name, self.graph, self.opset = 0, "", Graph(), {}
        for f, wt, v in _fields(buf):
            if f == 1:
                self.ir_version = v
            elif f == 2:
                self.producer_name = bytes(v).decode()
            elif f == 7:
                self.graph = Graph(v)
            elif f == 8:
                dom, ver = "", 0
                for f2, _, v2 in _fields(v):
                    if f2 == 1:
                        dom = bytes(v2).decode()
                    elif f2 == 2:
                        ver = v2
                self.opset[dom] = ver


def load(path) -> Model:
    """Read an ONNX file (``onnx.load`` for the supported subset)."""
    return Model(memoryview(Path(path).read_bytes()))


def to_array(t: Tensor) -> np.ndarray:
    """``numpy_helper.to_array`` for the supported data types."""
    if t.data_type not in _NP:
        raise ValueError(f"tensor {t.name}: unsupported data type {t.data_type}")
    dt = _NP[t.data_type]
    shape = tuple(int(d) for d in t.dims)
    if t.raw_data:
        a = np.frombuffer(t.raw_data, dtype=np.dtype(dt).newbyteorder("<")).astype(dt)
    elif t.data_type == T_FLOAT:
        a = np.asarray(t.float_data, np.float32)
    elif t.data_type == T_INT64:
        a = np.asarray(t.int64_data, np.int64)
    else:
        a = np.asarray(t.int32_data, dt)
    return a.reshape(shape) if shape else a.reshape(())


# ------------------------------------------------------------------ writer
def _enc_varint(x):
    if x < 0:
        x += 1 << 64
    out = bytearray()
    while True:
        b = x & 0x7F
        x >>= 7
        if x:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(fno, wt):
    return _enc_varint((fno << 3) | wt)


def _ld(fno, payload):
    return _key(fno, 2) + _enc_varint(len(payload)) + payload


def _str(fno, s):
    return _ld(fno, s.encode() if isinstance(s, str) else s)


def _int(fno, v):
    return _key(fno, 0) + _enc_varint(int(v))


def _float(fno, v):
    return _key(fno, 5) + struct.pack("<f", float(v))


def tensor_bytes(name, arr) -> bytes:
    arr = np.ascontiguousarray(arr)
    code = {np.dtype(np.float32): T_FLOAT, np.dtype(np.int64): T_INT64, np.dtype(np.float16): T_FLOAT16,
            np.dtype(np.int32): T_INT32, np.dtype(np.uint8): T_UINT8}[arr.dtype]
    out = b"".join(_int(1, d) for d in arr.shape) + _int(2, code) + _str(8, name)
    return out + _ld(9, arr.astype(arr.dtype.newbyteorder("<")).tobytes())


def attr_bytes(name, value) -> bytes:
    """An attribute from a Python value: float, int, list of ints / floats,
    numpy array (tensor)."""
    out = _str(1, name)
    if isinstance(value, float):
        return out + _float(2, value) + _int(20, A_FLOAT)
    if isinstance(value, (bool, int, np.integer)):
        return out + _int(3, int(value)) + _int(20, A_INT)
    if isinstance(value, np.ndarray):
        return out + _ld(5, tensor_bytes("", value)) + _int(20, A_TENSOR)
    if isinstance(value, (list, tuple)) and all(isinstance(v, (int, np.integer)) for v in value):
        return out + _ld(8, b"".join(_enc_varint(int(v)) for v in value)) + _int(20, A_INTS)
    if isinstance(value, (list, tuple)):
        return out + _ld(7, struct.pack(f"<{len(value)}f", *value)) + _int(20, A_FLOATS)
    raise TypeError(f"attribute {name}: unsupported value {value!r}")


def node_bytes(op_type, inputs, outputs, name="", domain="", **attrs) -> bytes:
    out = b"".join(_str(1, i) for i in inputs) + b"".join(_str(2, o) for o in outputs)
    if name:
        out += _str(3, name)
    out += _str(4, op_type)
    out += b"".join(_ld(5, attr_bytes(k, v)) for k, v in attrs.items())
    if domain:
        out += _str(7, domain)
    return out


def value_info_bytes(name, shape, elem_type=T_FLOAT) -> bytes:
    dims = b"".join(_ld(1, _int(1, d)) for d in shape)
    ttype = _int(1, elem_type) + _ld(2, dims)
    return _str(1, name) + _ld(2, _ld(1, ttype))


class GraphWriter:
    """Collects nodes, initializers and value infos, then writes a model."""

    def __init__(self, name="snn"):
        self.name = name
        self.nodes, self.inits, self.inputs, self.outputs, self.infos = [], [], [], [], []

    def node(self, op_type, inputs, outputs, name="", domain="", **attrs):
        self.nodes.append(node_bytes(op_type, inputs, outputs, name, domain, **attrs))

    def init(self, name, arr):
        self.inits.append(tensor_bytes(name, arr))
        return name

    def input(self, name, shape):
        self.inputs.append(value_info_bytes(name, shape))

    def output(self, name, shape):
        self.outputs.append(value_info_bytes(name, shape))

    def info(self, name, shape):
        self.infos.append(value_info_bytes(name, shape))

    def save(self, path, opset=17, custom_domains=("",)):
        g = b"".join(_ld(1, n) for n in self.nodes) + _str(2, self.name)
        g += b"".join(_ld(5, t) for t in self.inits)
        g += b"".join(_ld(11, v) for v in self.inputs) + b"".join(_ld(12, v) for v in self.outputs)
        g += b"".join(_ld(13, v) for v in self.infos)
        m = _int(1, 8) + _str(2, "sparsesnn_b200") + _ld(7, g)
        for dom in custom_domains:
            m += _ld(8, _str(1, dom) + _int(2, opset if dom == "" else 1))
        Path(path).write_bytes(m)
        return path
