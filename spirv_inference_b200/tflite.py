"""TFLite FlatBuffer front-end: `.tflite` bytes <-> the `nets.Model` graph the
executors run.

Reader: restates the reference loader (source/tflite_loader/src/model.rs:
260-529 and op_decoder.rs:124-211).  A FlatBuffer table is located by its
root offset; a field is found through the table's vtable (signed offset at
the table start, vtable = [vtable size, table size, field offsets...]) and
is absent when its slot is beyond the vtable or zero.  Model fields: 0
version, 1 operator_codes, 2 subgraphs, 3 description, 4 buffers; SubGraph:
0 tensors, 1 inputs, 2 outputs, 3 operators; Tensor: 0 shape, 1 type,
2 buffer, 3 name; Operator: 0 opcode_index, 1 inputs, 2 outputs,
3 builtin_options_type, 4 builtin_options; OperatorCode: 0 deprecated
builtin code (i8), 1 custom code, 3 builtin code (i32; preferred); Buffer:
0 data.  Options tables are decoded with the reference's field ids and
defaults (Conv2D: padding, stride_w, stride_h, activation, dilation_w,
dilation_h; DepthwiseConv2D adds depth_multiplier at 3; Pool2D: padding,
stride_w, stride_h, filter_w, filter_h, activation; Add/Mul/Sub/Div and
FullyConnected: activation at 0; Softmax: beta; Reshape: new_shape).

Writer: emits the same schema subset (a minimal FlatBuffer builder), so the
seeded graphs in `nets` can be saved as real `.tflite` files and read back;
it is how the reader is tested here, since the reference vendors no models.
"""
from __future__ import annotations

import struct

import numpy as np

from .nets import Model, Op

# TFLite builtin codes (model.rs:94-150 BuiltinOp::from_code, the subset the
# CNN executors run).
BUILTIN = {0: "ADD", 1: "AVERAGE_POOL_2D", 3: "CONV_2D", 4: "DEPTHWISE_CONV_2D",
           9: "FULLY_CONNECTED", 17: "MAX_POOL_2D", 18: "MUL", 22: "RESHAPE", 25: "SOFTMAX",
           41: "SUB", 42: "DIV"}
CODE = {v: k for k, v in BUILTIN.items()}
# BuiltinOptions union tags of the schema for those ops.
OPTIONS_TYPE = {"CONV_2D": 1, "DEPTHWISE_CONV_2D": 2, "AVERAGE_POOL_2D": 5, "MAX_POOL_2D": 5,
                "FULLY_CONNECTED": 8, "SOFTMAX": 9, "ADD": 11, "RESHAPE": 17, "MUL": 21,
                "SUB": 28, "DIV": 29}
PADDING = {0: "SAME", 1: "VALID"}


class TFLiteError(ValueError):
    pass


# ---------------------------------------------------------------------------
# reader
class _Table:
    def __init__(self, buf: bytes, pos: int):
        self.b, self.pos = buf, pos

    def _u16(self, p):
        return struct.unpack_from("<H", self.b, p)[0]

    def field(self, fid: int):
        vt = self.pos - struct.unpack_from("<i", self.b, self.pos)[0]
        if vt < 0 or vt + 4 > len(self.b):
            raise TFLiteError("invalid vtable offset")
        vtsize = self._u16(vt)
        slot = 4 + 2 * fid
        if slot + 2 > vtsize:
            return None
        off = self._u16(vt + slot)
        return self.pos + off if off else None

    def scalar(self, fid, fmt, default=None):
        p = self.field(fid)
        return default if p is None else struct.unpack_from("<" + fmt, self.b, p)[0]

    def _indirect(self, fid):
        p = self.field(fid)
        return None if p is None else p + struct.unpack_from("<I", self.b, p)[0]

    def table(self, fid):
        p = self._indirect(fid)
        return None if p is None else _Table(self.b, p)

    def vector(self, fid):
        """(start, length) of a vector field, or None."""
        p = self._indirect(fid)
        return None if p is None else (p + 4, struct.unpack_from("<I", self.b, p)[0])

    def string(self, fid):
        v = self.vector(fid)
        return None if v is None else self.b[v[0]:v[0] + v[1]].decode("utf-8", "replace")

    def ints(self, fid, fmt="i"):
        v = self.vector(fid)
        if v is None:
            return None
        return list(struct.unpack_from("<%d%s" % (v[1], fmt), self.b, v[0]))

    def tables(self, fid):
        v = self.vector(fid)
        if v is None:
            return []
        out = []
        for i in range(v[1]):
            p = v[0] + 4 * i
            out.append(_Table(self.b, p + struct.unpack_from("<I", self.b, p)[0]))
        return out


def _options(op_type: str, t: _Table | None) -> dict:
    g = (lambda fid, fmt, d: d) if t is None else t.scalar
    if op_type == "CONV_2D":
        return dict(padding=PADDING.get(g(0, "b", 0), "SAME"), stride=(g(2, "i", 1), g(1, "i", 1)),
                    activation=g(3, "b", 0), dilation=(g(5, "i", 1), g(4, "i", 1)))
    if op_type == "DEPTHWISE_CONV_2D":
        return dict(padding=PADDING.get(g(0, "b", 0), "SAME"), stride=(g(2, "i", 1), g(1, "i", 1)),
                    depth_multiplier=g(3, "i", 1), activation=g(4, "b", 0),
                    dilation=(g(6, "i", 1), g(5, "i", 1)))
    if op_type in ("AVERAGE_POOL_2D", "MAX_POOL_2D"):
        return dict(padding=PADDING.get(g(0, "b", 0), "SAME"), stride=(g(2, "i", 1), g(1, "i", 1)),
                    filter=(g(4, "i", 1), g(3, "i", 1)), activation=g(5, "b", 0))
    if op_type in ("ADD", "MUL", "SUB", "DIV", "FULLY_CONNECTED"):
        return dict(activation=g(0, "b", 0))
    if op_type == "SOFTMAX":
        return dict(beta=g(0, "f", 1.0))
    return {}


def read_tflite(buf: bytes, name: str = "tflite") -> Model:
    """Parses a TFLite FlatBuffer into a `nets.Model` (first subgraph, float32
    weights from the buffers, batch dimension dropped from the shapes)."""
    if len(buf) < 8:
        raise TFLiteError("too small to be a TFLite FlatBuffer")
    if buf[4:8] != b"TFL3":
        raise TFLiteError("missing TFL3 FlatBuffer identifier")
    model = _Table(buf, struct.unpack_from("<I", buf, 0)[0])
    codes = []
    for oc in model.tables(1):
        new, old = oc.scalar(3, "i", None), oc.scalar(0, "b", None)
        codes.append(new if new is not None else (old if old is not None else 0))
    subgraphs = model.tables(2)
    if not subgraphs:
        raise TFLiteError("model has no subgraphs")
    buffers = []
    for b in model.tables(4):
        v = b.vector(0)
        buffers.append(b"" if v is None else buf[v[0]:v[0] + v[1]])
    sg = subgraphs[0]
    tensors = []
    for i, t in enumerate(sg.tables(0)):
        ttype = t.scalar(1, "b", 0)
        tensors.append(dict(shape=tuple(t.ints(0) or ()), type=ttype, buffer=t.scalar(2, "I", 0),
                            name=t.string(3) or f"tensor_{i}"))
    names = [t["name"] for t in tensors]
    weights: dict[str, np.ndarray] = {}
    for t in tensors:
        data = buffers[t["buffer"]] if t["buffer"] < len(buffers) else b""
        if data:
            if t["type"] != 0:
                raise TFLiteError(f"tensor {t['name']}: only float32 constants are supported")
            weights[t["name"]] = np.frombuffer(data, np.float32).reshape(t["shape"]).copy()
    ops = []
    for o in sg.tables(3):
        idx = o.scalar(0, "I", 0)
        if idx >= len(codes):
            raise TFLiteError("opcode index out of range")
        code = codes[idx]
        if code not in BUILTIN:
            raise TFLiteError(f"unsupported builtin operator code {code}")
        op_type = BUILTIN[code]
        ins = [names[i] for i in (o.ints(1) or []) if i >= 0]
        outs = [names[i] for i in (o.ints(2) or [])]
        ops.append(Op(op_type, ins, outs[0], _options(op_type, o.table(4))))
    inputs = [names[i] for i in (sg.ints(1) or [])]
    outputs = [names[i] for i in (sg.ints(2) or [])]
    if len(inputs) != 1 or len(outputs) != 1:
        raise TFLiteError("one input and one output tensor are supported")
    shapes = {t["name"]: tuple(t["shape"][1:]) for t in tensors if t["name"] not in weights}
    return Model(name, inputs[0], outputs[0], shapes, ops, weights)


# ---------------------------------------------------------------------------
# writer (minimal FlatBuffer builder, back to front)
class _Builder:
    def __init__(self):
        self.buf = bytearray()

    def _pad(self, align, extra=0):
        while (len(self.buf) + extra) % align:
            self.buf[0:0] = b"\0"

    def _prepend(self, data: bytes, align: int):
        self._pad(align, len(data))
        self.buf[0:0] = data
        return len(self.buf)  # offset from the end

    def vector(self, fmt: str, items, elem_align=4) -> int:
        body = struct.pack("<%d%s" % (len(items), fmt), *items) if items else b""
        self._pad(max(4, elem_align), len(body) + 4)
        self.buf[0:0] = struct.pack("<I", len(items)) + body
        return len(self.buf)

    def bytes_vector(self, data: bytes) -> int:
        self._pad(16, len(data))  # 16-byte aligned data
        self.buf[0:0] = data
        self._pad(4, 4)
        self.buf[0:0] = struct.pack("<I", len(data))
        return len(self.buf)

    def string(self, s: str) -> int:
        data = s.encode() + b"\0"
        self._pad(4, len(data) + 4)
        self.buf[0:0] = struct.pack("<I", len(data) - 1) + data
        return len(self.buf)

    def offsets_vector(self, offs) -> int:
        self._pad(4, 4 * len(offs) + 4)
        n = len(offs)
        body = bytearray()
        for i, o in enumerate(offs):
            here = len(self.buf) + 4 * (n - i)  # offset-from-end of this slot
            body += struct.pack("<I", here - o)
        self.buf[0:0] = struct.pack("<I", n) + bytes(body)
        return len(self.buf)

    def table(self, fields: list) -> int:
        """fields[i] = None | ('b'|'i'|'I'|'f', value) | ('o', offset-from-end)."""
        # layout: [soffset][fields...], largest first for alignment simplicity
        items = [(i, f) for i, f in enumerate(fields) if f is not None]
        body = b""
        layout = {}
        ordered = sorted(items, key=lambda x: -struct.calcsize(x[1][0] if x[1][0] != "o" else "I"))
        rel = []
        for fid, (fmt, val) in ordered:
            size = 4 if fmt == "o" else struct.calcsize(fmt)
            while (4 + len(body)) % size:
                body += b"\0"
            layout[fid] = 4 + len(body)
            rel.append((fid, fmt, val, 4 + len(body)))
            body += b"\0" * size
        while (4 + len(body)) % 4:
            body += b"\0"
        tsize = 4 + len(body)
        self._pad(4, tsize)
        start_end = len(self.buf) + tsize  # offset-from-end of the table start
        body = bytearray(body)
        for fid, fmt, val, off in rel:
            if fmt == "o":
                slot_end = start_end - off  # offset-from-end of this field
                struct.pack_into("<I", body, off - 4, slot_end - val)
            else:
                struct.pack_into("<" + fmt, body, off - 4, val)
        # vtable right before the table: [vtsize, tsize, offsets...]
        nf = len(fields)
        vt = struct.pack("<HH", 4 + 2 * nf, tsize) + b"".join(
            struct.pack("<H", layout.get(i, 0)) for i in range(nf))
        table = bytearray(4) + body
        self.buf[0:0] = table
        table_end = len(self.buf)
        self._pad(2, len(vt))
        self.buf[0:0] = vt
        vt_end = len(self.buf)
        # soffset: table_pos - vtable_pos (positions from the start)
        struct.pack_into("<i", self.buf, vt_end - table_end, vt_end - table_end)
        return table_end

    def finish(self, root: int, ident: bytes = b"TFL3") -> bytes:
        # Alignment was taken from the end: make the total a multiple of 16
        # so it holds from the start too.
        self._pad(16, 8)
        self.buf[0:0] = ident
        self.buf[0:0] = struct.pack("<I", len(self.buf) + 4 - root)
        return bytes(self.buf)


def write_tflite(model: Model, batch: int = 1) -> bytes:
    """Serialises a `nets.Model` as a TFLite FlatBuffer (float32, batch dim
    `batch` on activation tensors)."""
    b = _Builder()
    names: list[str] = []
    shapes: list[tuple] = []
    for name in [model.input] + [o.output for o in model.ops]:
        if name not in names:
            names.append(name)
            shapes.append((batch,) + tuple(model.shapes[name]))
    wnames = [n for n in model.weights if n not in names]
    names += wnames
    shapes += [tuple(model.weights[n].shape) for n in wnames]
    index = {n: i for i, n in enumerate(names)}
    # buffers: 0 = empty (TFLite convention), then one per weight
    buf_offs = []
    for n in reversed(wnames):
        data = np.ascontiguousarray(model.weights[n], np.float32).tobytes()
        buf_offs.append(b.table([("o", b.bytes_vector(data))]))
    buf_offs.reverse()
    empty = b.table([None])
    buffers = b.offsets_vector([empty] + buf_offs)
    tensors = []
    for i in reversed(range(len(names))):
        name_off = b.string(names[i])
        shape_off = b.vector("i", list(shapes[i]))
        bufi = 1 + wnames.index(names[i]) if names[i] in model.weights else 0
        tensors.append(b.table([("o", shape_off), ("b", 0), ("I", bufi), ("o", name_off)]))
    tensors.reverse()
    tensors_v = b.offsets_vector(tensors)
    types = sorted({op.type for op in model.ops}, key=lambda t: CODE[t])
    op_index = {t: i for i, t in enumerate(types)}
    ops = []
    for op in reversed(model.ops):
        a = op.attrs
        ot = OPTIONS_TYPE.get(op.type)
        opt = None
        pad = 1 if a.get("padding") == "VALID" else 0
        if op.type == "CONV_2D":
            opt = b.table([("b", pad), ("i", a["stride"][1]), ("i", a["stride"][0]),
                           ("b", a.get("activation", 0)), ("i", a.get("dilation", (1, 1))[1]),
                           ("i", a.get("dilation", (1, 1))[0])])
        elif op.type == "DEPTHWISE_CONV_2D":
            opt = b.table([("b", pad), ("i", a["stride"][1]), ("i", a["stride"][0]),
                           ("i", a.get("depth_multiplier", 1)), ("b", a.get("activation", 0)),
                           ("i", a.get("dilation", (1, 1))[1]),
                           ("i", a.get("dilation", (1, 1))[0])])
        elif op.type in ("AVERAGE_POOL_2D", "MAX_POOL_2D"):
            opt = b.table([("b", pad), ("i", a["stride"][1]), ("i", a["stride"][0]),
                           ("i", a["filter"][1]), ("i", a["filter"][0]),
                           ("b", a.get("activation", 0))])
        elif op.type in ("ADD", "MUL", "SUB", "DIV", "FULLY_CONNECTED"):
            opt = b.table([("b", a.get("activation", 0))])
        elif op.type == "SOFTMAX":
            opt = b.table([("f", float(a.get("beta", 1.0)))])
        ins = b.vector("i", [index[n] for n in op.inputs])
        outs = b.vector("i", [index[op.output]])
        ops.append(b.table([("I", op_index[op.type]), ("o", ins), ("o", outs),
                            ("b", ot) if opt is not None else None,
                            ("o", opt) if opt is not None else None]))
    ops.reverse()
    ops_v = b.offsets_vector(ops)
    sg_in = b.vector("i", [index[model.input]])
    sg_out = b.vector("i", [index[model.output]])
    sg = b.table([("o", tensors_v), ("o", sg_in), ("o", sg_out), ("o", ops_v)])
    sgs = b.offsets_vector([sg])
    codes = [b.table([("b", min(CODE[t], 127)), None, None, ("i", CODE[t])])
             for t in reversed(types)]
    codes.reverse()
    codes_v = b.offsets_vector(codes)
    desc = b.string(f"{model.name} (spirv_inference_b200)")
    root = b.table([("i", 3), ("o", codes_v), ("o", sgs), ("o", desc), ("o", buffers)])
    return b.finish(root)
