"""ONNX export / import without the onnx package: a hand-written protobuf
encoder/decoder for the subset of onnx.proto (ModelProto, GraphProto,
NodeProto, AttributeProto, TensorProto, ValueInfoProto) that an inference
graph of a Sequential model needs, plus a small evaluator (`run`) used to
check an exported graph against the model.

Reference: ONNXExporter writes a text pseudo-graph with no weights
(src/export/model_export.cpp:51-147).  This writes a binary ModelProto
(IR version 8, opset 17) with every weight as an initializer and the
model's architecture in `metadata_props["dlvk.architecture"]` so that
`import_model` can rebuild the Sequential.

Layer mapping: Dense -> MatMul (+Add) (+Relu/Gelu); Conv2D -> Conv (+Relu);
pools -> MaxPool / AveragePool(count_include_pad=0); BatchNorm ->
BatchNormalization (running stats); LayerNorm -> LayerNormalization;
Dropout -> (nothing, inference); Flatten -> Flatten; activations -> Relu /
Sigmoid / Tanh / Softmax(axis=-1) / erf-GELU; Embedding -> Gather;
PositionalEncoding -> Add of the table sliced to the export sequence
length; MultiHeadAttention / TransformerEncoder -> MatMul / Reshape /
Transpose / Softmax / LayerNormalization / Add subgraphs; RNN / LSTM /
GRU -> the ONNX RNN / LSTM / GRU operators (layout=1, gates reordered to
ONNX's i,o,f,c and z,r,h orders, linear_before_reset=1 for GRU).
"""
from __future__ import annotations

import json
import math
import struct
from typing import Dict, List, Optional, Sequence, Tuple

import torch

# ----------------------------------------------------------------- protobuf wire format
_VARINT, _I64, _LEN, _I32 = 0, 1, 2, 5


def _varint(n: int) -> bytes:
    n &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = n & 0x7F
        n >>= 7
        if n:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field: int, wt: int) -> bytes:
    return _varint((field << 3) | wt)


def _f_varint(field: int, v: int) -> bytes:
    return _key(field, _VARINT) + _varint(v)


def _f_bytes(field: int, b: bytes) -> bytes:
    return _key(field, _LEN) + _varint(len(b)) + b


def _f_str(field: int, s: str) -> bytes:
    return _f_bytes(field, s.encode())


def _f_float(field: int, f: float) -> bytes:
    return _key(field, _I32) + struct.pack("<f", f)


def _parse(buf: bytes) -> Dict[int, list]:
    """Decode one message into {field: [raw values]} (varints as int,
    length-delimited as bytes, fixed32/64 as bytes)."""
    out: Dict[int, list] = {}
    i, n = 0, len(buf)
    while i < n:
        k, i = _read_varint(buf, i)
        field, wt = k >> 3, k & 7
        if wt == _VARINT:
            v, i = _read_varint(buf, i)
        elif wt == _LEN:
            ln, i = _read_varint(buf, i)
            v = buf[i:i + ln]
            i += ln
        elif wt == _I32:
            v = buf[i:i + 4]
            i += 4
        elif wt == _I64:
            v = buf[i:i + 8]
            i += 8
        else:
            raise ValueError(f"protobuf wire type {wt} not supported")
        out.setdefault(field, []).append(v)
    return out


def _read_varint(buf: bytes, i: int) -> Tuple[int, int]:
    shift = v = 0
    while True:
        b = buf[i]
        i += 1
        v |= (b & 0x7F) << shift
        if not b & 0x80:
            return v, i
        shift += 7


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= 1 << 63 else v


# ----------------------------------------------------------------- ONNX messages
FLOAT, INT32, INT64, FLOAT16, BFLOAT16 = 1, 6, 7, 10, 16
_DT = {torch.float32: FLOAT, torch.int32: INT32, torch.int64: INT64, torch.float16: FLOAT16,
       torch.bfloat16: BFLOAT16}
_DT_INV = {v: k for k, v in _DT.items()}


def tensor_proto(name: str, t: torch.Tensor) -> bytes:
    t = t.detach().cpu().contiguous()
    b = b"".join(_f_varint(1, int(d)) for d in t.shape)
    b += _f_varint(2, _DT[t.dtype]) + _f_str(8, name)
    raw = t.view(torch.uint8).numpy().tobytes() if t.dtype == torch.bfloat16 else t.numpy().tobytes()
    return b + _f_bytes(9, raw)


def parse_tensor(buf: bytes) -> Tuple[str, torch.Tensor]:
    f = _parse(buf)
    dims = [_signed(d) for d in f.get(1, [])]
    dt = _DT_INV[f[2][0]]
    name = f[8][0].decode()
    raw = f.get(9, [b""])[0]
    if dt == torch.bfloat16:
        t = torch.frombuffer(bytearray(raw), dtype=torch.uint8).view(torch.bfloat16)
    else:
        t = torch.frombuffer(bytearray(raw), dtype=dt) if raw else torch.empty(0, dtype=dt)
    return name, t.reshape(dims).clone()


def attr(name: str, v) -> bytes:
    b = _f_str(1, name)
    if isinstance(v, float):
        return b + _f_float(2, v) + _f_varint(20, 1)
    if isinstance(v, bool) or isinstance(v, int):
        return b + _f_varint(3, int(v)) + _f_varint(20, 2)
    if isinstance(v, str):
        return b + _f_bytes(4, v.encode()) + _f_varint(20, 3)
    if isinstance(v, (list, tuple)) and all(isinstance(x, int) for x in v):
        return b + b"".join(_f_varint(8, int(x)) for x in v) + _f_varint(20, 7)
    if isinstance(v, (list, tuple)):
        return b + b"".join(_f_float(7, float(x)) for x in v) + _f_varint(20, 6)
    raise TypeError(f"attribute {name}: {type(v)}")


def parse_attr(buf: bytes):
    f = _parse(buf)
    name = f[1][0].decode()
    kind = f[20][0]
    if kind == 1:
        return name, struct.unpack("<f", f[2][0])[0]
    if kind == 2:
        return name, _signed(f[3][0])
    if kind == 3:
        return name, f[4][0].decode()
    if kind == 7:
        vals = []
        for v in f.get(8, []):
            if isinstance(v, bytes):  # packed
                i = 0
                while i < len(v):
                    x, i = _read_varint(v, i)
                    vals.append(_signed(x))
            else:
                vals.append(_signed(v))
        return name, vals
    if kind == 6:
        return name, [struct.unpack("<f", x)[0] for x in f.get(7, [])]
    raise ValueError(f"attribute type {kind}")


def node(op: str, inputs: Sequence[str], outputs: Sequence[str], name: str = "", **attrs) -> bytes:
    b = b"".join(_f_str(1, i) for i in inputs) + b"".join(_f_str(2, o) for o in outputs)
    b += _f_str(3, name or outputs[0]) + _f_str(4, op)
    for k, v in attrs.items():
        b += _f_bytes(5, attr(k, v))
    return b


def value_info(name: str, elem: int, shape: Optional[Sequence] = None) -> bytes:
    tt = _f_varint(1, elem)
    if shape is not None:
        dims = b""
        for d in shape:
            dims += _f_bytes(1, _f_varint(1, d) if isinstance(d, int) else _f_str(2, str(d)))
        tt += _f_bytes(2, dims)
    return _f_str(1, name) + _f_bytes(2, _f_bytes(1, tt))


def model_proto(nodes: List[bytes], inits: List[bytes], inputs: List[bytes], outputs: List[bytes], graph_name: str,
                metadata: Dict[str, str], opset: int = 17, producer: str = "dlvk_b200") -> bytes:
    g = b"".join(_f_bytes(1, n) for n in nodes) + _f_str(2, graph_name)
    g += b"".join(_f_bytes(5, t) for t in inits)
    g += b"".join(_f_bytes(11, v) for v in inputs) + b"".join(_f_bytes(12, v) for v in outputs)
    m = _f_varint(1, 8) + _f_str(2, producer) + _f_str(3, "1.0") + _f_varint(5, 1)
    m += _f_bytes(7, g) + _f_bytes(8, _f_str(1, "") + _f_varint(2, opset))
    for k, v in metadata.items():
        m += _f_bytes(14, _f_str(1, k) + _f_str(2, v))
    return m


def parse_model(buf: bytes) -> dict:
    m = _parse(buf)
    g = _parse(m[7][0])
    nodes = []
    for nb in g.get(1, []):
        f = _parse(nb)
        nodes.append({"inputs": [x.decode() for x in f.get(1, [])], "outputs": [x.decode() for x in f.get(2, [])],
                      "op": f[4][0].decode(), "attrs": dict(parse_attr(a) for a in f.get(5, []))})
    inits = dict(parse_tensor(t) for t in g.get(5, []))
    ins = [_parse(v)[1][0].decode() for v in g.get(11, [])]
    outs = [_parse(v)[1][0].decode() for v in g.get(12, [])]
    meta = {}
    for e in m.get(14, []):
        f = _parse(e)
        meta[f[1][0].decode()] = f[2][0].decode()
    opset = _parse(m[8][0])[2][0]
    return {"ir_version": m[1][0], "opset": opset, "nodes": nodes, "initializers": inits, "inputs": ins,
            "outputs": outs, "metadata": meta, "producer": m[2][0].decode()}


# ----------------------------------------------------------------- graph builder
class _G:
    def __init__(self, params=()):
        self.nodes: List[bytes] = []
        self.inits: List[bytes] = []
        self.n = 0
        self.pidx = {id(p): i for i, p in enumerate(params)}
        self.done = set()

    def param(self, p) -> str:
        """Initializer of a model parameter, named `param.<index>`."""
        nm = f"param.{self.pidx[id(p)]}"
        if nm not in self.done:
            self.done.add(nm)
            self.inits.append(tensor_proto(nm, _f32(p)))
        return nm

    def named(self, nm: str, t: torch.Tensor) -> str:
        self.inits.append(tensor_proto(nm, t))
        return nm

    def name(self, base: str) -> str:
        self.n += 1
        return f"{base}_{self.n}"

    def init(self, base: str, t: torch.Tensor) -> str:
        nm = self.name(base)
        self.inits.append(tensor_proto(nm, t))
        return nm

    def op(self, op: str, inputs, **attrs) -> str:
        out = self.name(op.lower())
        self.nodes.append(node(op, inputs, [out], **attrs))
        return out


def _f32(p) -> torch.Tensor:
    return p.master.detach().float().cpu()


def _gelu(g: _G, x: str) -> str:
    s = g.op("Div", [x, g.init("sqrt2", torch.tensor(math.sqrt(2.0)))])
    e = g.op("Erf", [s])
    one = g.op("Add", [e, g.init("one", torch.tensor(1.0))])
    h = g.op("Mul", [x, one])
    return g.op("Mul", [h, g.init("half", torch.tensor(0.5))])


def _act(g: _G, x: str, act) -> str:
    if act in (None, "none", "linear"):
        return x
    if act == "relu":
        return g.op("Relu", [x])
    if act == "gelu":
        return _gelu(g, x)
    raise ValueError(f"activation {act}")


def _dense(g: _G, x: str, w, b, act=None) -> str:
    y = g.op("MatMul", [x, g.param(w)])
    if b is not None:
        y = g.op("Add", [y, g.param(b)])
    return _act(g, y, act)


def _layernorm(g: _G, x: str, layer) -> str:
    return g.op("LayerNormalization", [x, g.param(layer.gamma), g.param(layer.beta)],
                axis=-1, epsilon=float(layer.eps))


def _mha(g: _G, x: str, layer, S: int, residual: Optional[str] = None) -> str:
    E, Hh = layer.embed_dim, layer.num_heads
    D = E // Hh
    qkv = g.op("MatMul", [x, g.param(layer.w_qkv)])                   # [B, S, 3E]
    r = g.op("Reshape", [qkv, g.init("shape", torch.tensor([0, S, 3, Hh, D], dtype=torch.int64))])
    t = g.op("Transpose", [r], perm=[2, 0, 3, 1, 4])                              # [3, B, H, S, D]
    q = g.op("Gather", [t, g.init("i0", torch.tensor(0, dtype=torch.int64))], axis=0)
    k = g.op("Gather", [t, g.init("i1", torch.tensor(1, dtype=torch.int64))], axis=0)
    v = g.op("Gather", [t, g.init("i2", torch.tensor(2, dtype=torch.int64))], axis=0)
    kt = g.op("Transpose", [k], perm=[0, 1, 3, 2])
    s = g.op("MatMul", [q, kt])
    s = g.op("Mul", [s, g.init("scale", torch.tensor(1.0 / math.sqrt(D)))])
    p = g.op("Softmax", [s], axis=-1)
    a = g.op("MatMul", [p, v])                                                    # [B, H, S, D]
    a = g.op("Transpose", [a], perm=[0, 2, 1, 3])
    a = g.op("Reshape", [a, g.init("shape", torch.tensor([0, S, E], dtype=torch.int64))])
    o = g.op("MatMul", [a, g.param(layer.w_o)])
    if residual is not None:
        o = g.op("Add", [o, residual])
    return o


def _recurrent(g: _G, x: str, cells, H: int, li: int) -> str:
    """ONNX RNN/LSTM/GRU with layout=1 ([B, T, ...]); returns [B, T, D*H]."""
    kind = cells[0].kind
    D = len(cells)
    Ws, Rs, Bs = [], [], []
    for c in cells:
        w, r = _f32(c.w_ih), _f32(c.w_hh)
        bi = _f32(c.b_ih) if c.b_ih is not None else torch.zeros(w.shape[0])
        bh = _f32(c.b_hh) if c.b_hh is not None else torch.zeros(w.shape[0])
        if kind == 1:      # ours i,f,g,o -> ONNX i,o,f,c
            perm = [0, 3, 1, 2]
        elif kind == 2:    # ours r,z,n -> ONNX z,r,h
            perm = [1, 0, 2]
        else:
            perm = [0]
        def re(t):
            return torch.cat([t.reshape(len(perm), H, *t.shape[1:])[j] for j in perm], 0)
        Ws.append(re(w))
        Rs.append(re(r))
        Bs.append(torch.cat([re(bi), re(bh)], 0))
    op = {0: "RNN", 1: "LSTM", 2: "GRU"}[kind]
    attrs = dict(hidden_size=H, layout=1, direction="bidirectional" if D == 2 else "forward")
    if kind == 2:
        attrs["linear_before_reset"] = 1
    ins = [x, g.named(f"rec.{li}.W", torch.stack(Ws)), g.named(f"rec.{li}.R", torch.stack(Rs)),
           g.named(f"rec.{li}.B", torch.stack(Bs))]
    y = g.name(op.lower())
    g.nodes.append(node(op, ins, [y], **attrs))                                 # [B, T, D, H]
    return g.op("Reshape", [y, g.init("shape", torch.tensor([0, 0, D * H], dtype=torch.int64))])


def build_graph(model, input_shape: Sequence[int]) -> Tuple[List[bytes], List[bytes], List[bytes], List[bytes]]:
    from ..models import layers as L

    g = _G(model.parameters())
    int_input = isinstance(model.m_layers[0], L.EmbeddingLayer)
    x = "input"
    shape = list(input_shape)
    S = shape[1] if len(shape) > 1 else 1
    for li, layer in enumerate(model.m_layers):
        if isinstance(layer, L.DenseLayer):
            x = _dense(g, x, layer.weight, layer.bias, layer.activation)
        elif isinstance(layer, L.Conv2DLayer):
            ins = [x, g.param(layer.weight)] + ([g.param(layer.bias)] if layer.bias is not None else [])
            p = layer.padding
            x = g.op("Conv", ins, kernel_shape=[layer.kernel_size] * 2, strides=[layer.stride] * 2, pads=[p] * 4)
            if layer.relu:
                x = g.op("Relu", [x])
        elif isinstance(layer, L.MaxPool2DLayer):
            k = layer.pool_size
            x = g.op("MaxPool", [x], kernel_shape=[k, k], strides=[layer.stride or k] * 2)
        elif isinstance(layer, L.AvgPool2DLayer):
            k = layer.pool_size
            x = g.op("AveragePool", [x], kernel_shape=[k, k], strides=[layer.stride or k] * 2,
                     pads=[getattr(layer, "padding", 0)] * 4, count_include_pad=0)
        elif isinstance(layer, L._BatchNormBase):
            C = layer.num_features
            gam = g.param(layer.gamma) if layer.gamma is not None else g.init("ones", torch.ones(C))
            bet = g.param(layer.beta) if layer.beta is not None else g.init("zeros", torch.zeros(C))
            x = g.op("BatchNormalization", [x, gam, bet,
                                            g.named(f"buf.{li}.mean", layer.running_mean.detach().float().cpu()),
                                            g.named(f"buf.{li}.var", layer.running_var.detach().float().cpu())],
                     epsilon=float(layer.eps))
        elif isinstance(layer, L.DropoutLayer):
            continue
        elif isinstance(layer, L.FlattenLayer):
            x = g.op("Flatten", [x], axis=1)
        elif isinstance(layer, L.ActivationLayer):
            a = layer.activation.value
            if a == "softmax":
                x = g.op("Softmax", [x], axis=-1)
            elif a == "gelu":
                x = _gelu(g, x)
            elif a != "linear":
                x = g.op({"relu": "Relu", "sigmoid": "Sigmoid", "tanh": "Tanh"}[a], [x])
        elif isinstance(layer, L.EmbeddingLayer):
            x = g.op("Gather", [g.param(layer.weight), x], axis=0)
        elif isinstance(layer, L.LayerNormLayer):
            x = _layernorm(g, x, layer)
        elif isinstance(layer, L.PositionalEncodingLayer):
            x = g.op("Add", [x, g.init("pe", layer.table[:S].float())])
        elif isinstance(layer, L.MultiHeadAttentionLayer):
            x = _mha(g, x, layer, S, residual=x if layer.residual else None)
        elif isinstance(layer, L.TransformerEncoderLayer):
            h = _mha(g, _layernorm(g, x, layer.ln1), layer.attn, S, residual=x)
            f = _dense(g, _layernorm(g, h, layer.ln2), layer.ff1.weight, layer.ff1.bias, "relu")
            f = _dense(g, f, layer.ff2.weight, layer.ff2.bias)
            x = g.op("Add", [f, h])
        elif isinstance(layer, L.GlobalAvgPoolLayer):
            x = g.op("Flatten", [g.op("GlobalAveragePool", [x])], axis=1)
        elif isinstance(layer, L.ResidualLayer) and isinstance(layer.inner, L.DenseLayer):
            inner = layer.inner
            x = g.op("Add", [x, _dense(g, x, inner.weight, inner.bias, inner.activation)])
        elif isinstance(layer, (L.RNNLayer, L.LSTMLayer, L.GRULayer)):
            if layer.reverse:
                raise NotImplementedError("ONNX export of a stand-alone reversed recurrent layer")
            y = _recurrent(g, x, [layer], layer.hidden_size, li)
            x = y if layer.return_sequences else g.op(
                "Squeeze", [g.op("Slice", [y, g.init("st", torch.tensor([-1])), g.init("en", torch.tensor([2 ** 62])),
                                           g.init("ax", torch.tensor([1]))]), g.init("ax", torch.tensor([1]))])
        elif isinstance(layer, L.BidirectionalRNN):
            if not layer.return_sequences:
                raise NotImplementedError("ONNX export of a bidirectional layer without return_sequences")
            x = _recurrent(g, x, [layer.fwd, layer.bwd], layer.hidden_size, li)
        else:
            raise NotImplementedError(f"ONNX export of {layer.type_name}")
    if x == "input":
        x = g.op("Identity", [x])
    dims = ["N"] + [int(d) for d in shape[1:]]
    inputs = [value_info("input", INT64 if int_input else FLOAT, dims)]
    outputs = [value_info(x, FLOAT)]
    return g.nodes, g.inits, inputs, outputs


def export_model(model, path: str, input_shape: Sequence[int], metadata: Optional[Dict[str, str]] = None) -> None:
    model.build()
    nodes, inits, ins, outs = build_graph(model, input_shape)
    meta = {"dlvk.architecture": json.dumps(model.architecture()), "dlvk.input_shape": json.dumps(list(input_shape))}
    meta.update(metadata or {})
    blob = model_proto(nodes, inits, ins, outs, "dlvk_b200_model", meta)
    with open(path, "wb") as f:
        f.write(blob)


# ----------------------------------------------------------------- reference evaluator
def run(parsed: dict, x: torch.Tensor) -> torch.Tensor:
    """Evaluate a parsed graph with torch on the CPU (checks an export)."""
    import torch.nn.functional as F

    env = dict(parsed["initializers"])
    env[parsed["inputs"][0]] = x
    for nd in parsed["nodes"]:
        a = nd["attrs"]
        i = [env[n] if n else None for n in nd["inputs"]]
        op = nd["op"]
        if op == "MatMul":
            y = torch.matmul(i[0].float(), i[1].float())
        elif op in ("Add", "Mul", "Div"):
            y = {"Add": torch.add, "Mul": torch.mul, "Div": torch.div}[op](i[0], i[1])
        elif op == "Relu":
            y = torch.relu(i[0])
        elif op == "Sigmoid":
            y = torch.sigmoid(i[0])
        elif op == "Tanh":
            y = torch.tanh(i[0])
        elif op == "Erf":
            y = torch.erf(i[0])
        elif op == "Softmax":
            y = torch.softmax(i[0], a.get("axis", -1))
        elif op == "Identity":
            y = i[0]
        elif op == "Flatten":
            y = i[0].reshape(i[0].shape[0], -1)
        elif op == "Conv":
            p = a.get("pads", [0, 0, 0, 0])
            y = F.conv2d(i[0], i[1], i[2] if len(i) > 2 else None, stride=a["strides"], padding=(p[0], p[1]))
        elif op == "MaxPool":
            y = F.max_pool2d(i[0], a["kernel_shape"], a["strides"])
        elif op == "AveragePool":
            p = a.get("pads", [0, 0, 0, 0])
            y = F.avg_pool2d(i[0], a["kernel_shape"], a["strides"], padding=p[0], count_include_pad=False)
        elif op == "GlobalAveragePool":
            y = i[0].mean((2, 3), keepdim=True)
        elif op == "BatchNormalization":
            y = F.batch_norm(i[0], i[3], i[4], i[1], i[2], False, 0.0, a.get("epsilon", 1e-5))
        elif op == "LayerNormalization":
            y = F.layer_norm(i[0], i[0].shape[-1:], i[1], i[2], a.get("epsilon", 1e-5))
        elif op == "Gather":
            y = torch.index_select(i[0], a.get("axis", 0), i[1].reshape(-1).long()).reshape(
                *i[0].shape[:a.get("axis", 0)], *i[1].shape, *i[0].shape[a.get("axis", 0) + 1:])
        elif op == "Reshape":
            shp = [int(s) if int(s) != 0 else i[0].shape[k] for k, s in enumerate(i[1].tolist())]
            y = i[0].reshape(shp)
        elif op == "Transpose":
            y = i[0].permute(a["perm"])
        elif op == "Slice":
            st, en, ax = int(i[1][0]), int(i[2][0]), int(i[3][0])
            y = i[0].narrow(ax, st % i[0].shape[ax], 1) if st < 0 else i[0].narrow(ax, st, min(en, i[0].shape[ax]) - st)
        elif op == "Squeeze":
            y = i[0].squeeze(int(i[1][0]))
        elif op in ("RNN", "LSTM", "GRU"):
            y = _run_recurrent(op, a, i)
        else:
            raise NotImplementedError(op)
        env[nd["outputs"][0]] = y
    return env[parsed["outputs"][0]]


def _run_recurrent(op, a, i):
    x, W, R, Bv = i[0].float(), i[1], i[2], i[3]
    H = a["hidden_size"]
    D, B_, T = W.shape[0], x.shape[0], x.shape[1]
    ys = torch.zeros(B_, T, D, H)
    G = W.shape[1] // H
    for d in range(D):
        h = torch.zeros(B_, H)
        c = torch.zeros(B_, H)
        wb, rb = Bv[d][:G * H], Bv[d][G * H:]
        steps = range(T) if d == 0 else range(T - 1, -1, -1)
        for t in steps:
            xw = x[:, t] @ W[d].t() + wb
            hr = h @ R[d].t() + rb
            if op == "RNN":
                h = torch.tanh(xw + hr)
            elif op == "LSTM":
                z = xw + hr
                ii, oo, ff, cc = (z[:, k * H:(k + 1) * H] for k in range(4))
                c = torch.sigmoid(ff) * c + torch.sigmoid(ii) * torch.tanh(cc)
                h = torch.sigmoid(oo) * torch.tanh(c)
            else:
                zz = torch.sigmoid(xw[:, :H] + hr[:, :H])
                rr = torch.sigmoid(xw[:, H:2 * H] + hr[:, H:2 * H])
                nn_ = torch.tanh(xw[:, 2 * H:] + rr * hr[:, 2 * H:])
                h = (1 - zz) * nn_ + zz * h
            ys[:, t, d] = h
    return ys
