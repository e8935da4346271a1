"""ONNX export of the Llama decoder, written without the `onnx` package.

`export_onnx(sd, cfg, path)` encodes an ONNX ModelProto (IR version 8, default
opset 17) directly in protobuf wire format from the reference-named state dict
([in, out] matrices): input `input_ids` int64 [batch, seq], output `logits`
float32 [batch, seq, vocab], both with symbolic batch and sequence sizes (up to
`max_seq_len` positions: the RoPE tables and the causal mask are initializers
sliced to the sequence length).  The graph uses standard operators only:

    Gather (embedding), MatMul (projections, attention), Mul / Add / Sub / Div /
    Sqrt / ReduceMean (RMSNorm), Slice / Unsqueeze / Concat / Reshape (RoPE on
    the interleaved pairs (2i, 2i+1), head split), Transpose, Softmax (causal
    attention with an additive mask; grouped-query heads by broadcasting the
    K/V heads over their query group), Sigmoid (SwiGLU)

`load_onnx(path)` parses a file back (nodes, attributes, initializers, inputs,
outputs) and `run_onnx(model, feeds)` evaluates it with numpy following the
operator definitions, so an export can be checked against the fp32 oracle
where no ONNX runtime is installed.

The message and field numbers are those of the public onnx.proto (they are the
file format, so they have to be the same).

Reference: ExportSuite::export_onnx (include/io/export_suite.hpp:7-13, a
print-only stub) and OnnxBackend (include/serving/onnx_backend.hpp:13-104).
"""
from __future__ import annotations

import struct
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from ..config import TransformerConfig

IR_VERSION, OPSET = 8, 17
T_FLOAT, T_INT64 = 1, 7                      # TensorProto.DataType
A_FLOAT, A_INT, A_INTS = 1, 2, 7             # AttributeProto.AttributeType
_NP = {T_FLOAT: np.float32, T_INT64: np.int64}


# ------------------------------------------------------------ wire format
def _varint(v: int) -> bytes:
    v &= (1 << 64) - 1
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


def _f_int(field: int, v: int) -> bytes:
    return _key(field, 0) + _varint(v)


def _f_bytes(field: int, b: bytes) -> bytes:
    return _key(field, 2) + _varint(len(b)) + b


def _f_str(field: int, s: str) -> bytes:
    return _f_bytes(field, s.encode())


def _f_float(field: int, v: float) -> bytes:
    return _key(field, 5) + struct.pack("<f", v)


def _tensor(name: str, a: np.ndarray) -> bytes:
    dt = T_INT64 if a.dtype == np.int64 else T_FLOAT
    a = np.ascontiguousarray(a.astype(_NP[dt]))
    out = b"".join(_f_int(1, d) for d in a.shape) + _f_int(2, dt) + _f_str(8, name)
    return out + _f_bytes(9, a.tobytes())


def _value_info(name: str, elem: int, dims: List) -> bytes:
    dim = b"".join(_f_bytes(1, _f_str(2, d) if isinstance(d, str) else _f_int(1, d)) for d in dims)
    tensor_type = _f_int(1, elem) + _f_bytes(2, dim)
    return _f_str(1, name) + _f_bytes(2, _f_bytes(1, tensor_type))


def _attr(name: str, v) -> bytes:
    if isinstance(v, float):
        return _f_str(1, name) + _f_float(2, v) + _f_int(20, A_FLOAT)
    if isinstance(v, int):
        return _f_str(1, name) + _f_int(3, v) + _f_int(20, A_INT)
    return _f_str(1, name) + b"".join(_f_int(8, x) for x in v) + _f_int(20, A_INTS)


class _Graph:
    def __init__(self):
        self.nodes: List[bytes] = []
        self.inits: List[bytes] = []
        self.n = 0

    def init(self, name: str, a) -> str:
        a = a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a)
        if a.dtype not in (np.int64,):
            a = a.astype(np.float32)
        self.inits.append(_tensor(name, a))
        return name

    def const_i(self, vals) -> str:
        self.n += 1
        return self.init(f"c{self.n}", np.asarray(vals, dtype=np.int64))

    def const_f(self, v: float) -> str:
        self.n += 1
        return self.init(f"c{self.n}", np.asarray(v, dtype=np.float32))

    def op(self, op_type: str, *inputs: str, **attrs) -> str:
        self.n += 1
        out = f"t{self.n}"
        body = b"".join(_f_str(1, i) for i in inputs) + _f_str(2, out) + _f_str(3, f"n{self.n}")
        body += _f_str(4, op_type) + b"".join(_f_bytes(5, _attr(k, v)) for k, v in attrs.items())
        self.nodes.append(body)
        return out


# ------------------------------------------------------------------ export
def export_onnx(sd: Dict[str, torch.Tensor], cfg: TransformerConfig, path: str,
                max_seq_len: Optional[int] = None) -> None:
    """Write the decoder as an ONNX model (fp32 weights) to `path`."""
    H, KV, Dh, D = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.hidden_dim
    G = H // KV
    L = max_seq_len or cfg.max_seq_len
    g = _Graph()
    f32 = (lambda t: t.detach().float().cpu())
    emb = g.init("token_embedding.weight", f32(sd["token_embedding.weight"]))
    # RoPE tables and the causal mask, sliced to the sequence length at run time
    inv = cfg.rope_base ** (-torch.arange(0, Dh, 2, dtype=torch.float64) / Dh)
    ang = torch.arange(L, dtype=torch.float64)[:, None] * inv[None, :]
    cos = g.init("rope_cos", ang.cos().float())
    sin = g.init("rope_sin", ang.sin().float())
    mask = g.init("causal_mask", torch.full((L, L), -1e9).triu(1))
    eps, scale = g.const_f(cfg.norm_eps), g.const_f(1.0 / Dh ** 0.5)

    h = g.op("Gather", emb, "input_ids", axis=0)                              # [B, S, D]
    seq = g.op("Slice", g.op("Shape", "input_ids"), g.const_i([1]), g.const_i([2]), g.const_i([0]))
    cos_s = g.op("Unsqueeze", g.op("Slice", cos, g.const_i([0]), seq, g.const_i([0])), g.const_i([1]))
    sin_s = g.op("Unsqueeze", g.op("Slice", sin, g.const_i([0]), seq, g.const_i([0])), g.const_i([1]))
    mask_s = g.op("Slice", mask, g.const_i([0, 0]), g.op("Concat", seq, seq, axis=0), g.const_i([0, 1]))

    def rms(x: str, w: str) -> str:
        ms = g.op("ReduceMean", g.op("Mul", x, x), axes=[-1], keepdims=1)
        return g.op("Mul", g.op("Div", x, g.op("Sqrt", g.op("Add", ms, eps))), w)

    def rope(x4: str) -> str:        # [B, S, heads, Dh], pairs (2i, 2i+1)
        ev = g.op("Slice", x4, g.const_i([0]), g.const_i([Dh]), g.const_i([3]), g.const_i([2]))
        od = g.op("Slice", x4, g.const_i([1]), g.const_i([Dh]), g.const_i([3]), g.const_i([2]))
        e2 = g.op("Sub", g.op("Mul", ev, cos_s), g.op("Mul", od, sin_s))
        o2 = g.op("Add", g.op("Mul", ev, sin_s), g.op("Mul", od, cos_s))
        four = g.const_i([4])
        pair = g.op("Concat", g.op("Unsqueeze", e2, four), g.op("Unsqueeze", o2, four), axis=4)
        return g.op("Reshape", pair, g.const_i([0, 0, 0, Dh]))

    for i in range(cfg.num_layers):
        r = f"blocks.{i}."
        w = {k: g.init(r + k, f32(sd[r + k])) for k in
             ("rms_norm_attn.weight", "attn.Wq.weight", "attn.Wk.weight", "attn.Wv.weight", "attn.Wo.weight",
              "rms_norm_ffn.weight", "ffn.Wgate.weight", "ffn.Wup.weight", "ffn.Wdown.weight")}
        x = rms(h, w["rms_norm_attn.weight"])
        q = rope(g.op("Reshape", g.op("MatMul", x, w["attn.Wq.weight"]), g.const_i([0, 0, H, Dh])))
        k = rope(g.op("Reshape", g.op("MatMul", x, w["attn.Wk.weight"]), g.const_i([0, 0, KV, Dh])))
        v = g.op("Reshape", g.op("MatMul", x, w["attn.Wv.weight"]), g.const_i([0, 0, KV, Dh]))
        qg = g.op("Transpose", g.op("Reshape", q, g.const_i([0, 0, KV, G, Dh])), perm=[0, 2, 3, 1, 4])
        kt = g.op("Unsqueeze", g.op("Transpose", k, perm=[0, 2, 3, 1]), g.const_i([2]))   # [B, KV, 1, Dh, S]
        vt = g.op("Unsqueeze", g.op("Transpose", v, perm=[0, 2, 1, 3]), g.const_i([2]))   # [B, KV, 1, S, Dh]
        s = g.op("Add", g.op("Mul", g.op("MatMul", qg, kt), scale), mask_s)              # [B, KV, G, S, S]
        o = g.op("MatMul", g.op("Softmax", s, axis=-1), vt)                               # [B, KV, G, S, Dh]
        o = g.op("Reshape", g.op("Transpose", o, perm=[0, 3, 1, 2, 4]), g.const_i([0, 0, -1]))
        h = g.op("Add", h, g.op("MatMul", o, w["attn.Wo.weight"]))
        x = rms(h, w["rms_norm_ffn.weight"])
        gate = g.op("MatMul", x, w["ffn.Wgate.weight"])
        act = g.op("Mul", g.op("Mul", gate, g.op("Sigmoid", gate)), g.op("MatMul", x, w["ffn.Wup.weight"]))
        h = g.op("Add", h, g.op("MatMul", act, w["ffn.Wdown.weight"]))
    xf = rms(h, g.init("final_norm.weight", f32(sd["final_norm.weight"])))
    head = (g.init("lm_head.weight", f32(sd["token_embedding.weight"]).t().contiguous()) if cfg.tie_embeddings
            else g.init("lm_head.weight", f32(sd["lm_head.weight"])))
    logits = g.op("MatMul", xf, head)
    # rename the last output to "logits"
    g.nodes[-1] = g.nodes[-1].replace(_f_str(2, logits), _f_str(2, "logits"), 1)
    graph = b"".join(_f_bytes(1, n) for n in g.nodes) + _f_str(2, "lora_kernel_b200_llama")
    graph += b"".join(_f_bytes(5, t) for t in g.inits)
    graph += _f_bytes(11, _value_info("input_ids", T_INT64, ["batch", "seq"]))
    graph += _f_bytes(12, _value_info("logits", T_FLOAT, ["batch", "seq", cfg.vocab_size]))
    model = _f_int(1, IR_VERSION) + _f_str(2, "lora_kernel_b200") + _f_str(3, "0.1")
    model += _f_bytes(8, _f_str(1, "") + _f_int(2, OPSET)) + _f_bytes(7, graph)
    with open(path, "wb") as f:
        f.write(model)


# ------------------------------------------------------------------ reading
def _fields(buf: bytes) -> List[Tuple[int, int, object]]:
    """(field, wire type, value) of one message; length-delimited values as bytes."""
    out, i = [], 0
    while i < len(buf):
        k, i = _read_varint(buf, i)
        f, wt = k >> 3, k & 7
        if wt == 0:
            v, i = _read_varint(buf, i)
        elif wt == 2:
            n, i = _read_varint(buf, i)
            v, i = buf[i:i + n], i + n
        elif wt == 5:
            v, i = struct.unpack("<f", buf[i:i + 4])[0], i + 4
        elif wt == 1:
            v, i = struct.unpack("<d", buf[i:i + 8])[0], i + 8
        else:
            raise ValueError(f"unsupported wire type {wt}")
        out.append((f, wt, v))
    return out


def _read_varint(buf: bytes, i: int) -> Tuple[int, int]:
    v, s = 0, 0
    while True:
        b = buf[i]
        i += 1
        v |= (b & 0x7F) << s
        s += 7
        if not b & 0x80:
            return v, i


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= 1 << 63 else v


def _read_tensor(buf: bytes) -> Tuple[str, np.ndarray]:
    dims, dt, name, raw = [], T_FLOAT, "", b""
    for f, wt, v in _fields(buf):
        if f == 1:
            dims.append(_signed(v))
        elif f == 2:
            dt = v
        elif f == 8:
            name = v.decode()
        elif f == 9:
            raw = v
    return name, np.frombuffer(raw, dtype=_NP[dt]).reshape(dims).copy()


def load_onnx(path: str) -> dict:
    """{"opset", "nodes": [(op, inputs, outputs, attrs)], "inits": {name: array},
    "inputs": [names], "outputs": [names]} of a file written by export_onnx."""
    with open(path, "rb") as f:
        buf = f.read()
    model = {"opset": None, "nodes": [], "inits": {}, "inputs": [], "outputs": []}
    for f, _, v in _fields(buf):
        if f == 8:
            model["opset"] = dict((ff, vv) for ff, _, vv in _fields(v)).get(2)
        elif f == 7:
            for gf, _, gv in _fields(v):
                if gf == 1:
                    ins, outs, op, attrs = [], [], "", {}
                    for nf, _, nv in _fields(gv):
                        if nf == 1:
                            ins.append(nv.decode())
                        elif nf == 2:
                            outs.append(nv.decode())
                        elif nf == 4:
                            op = nv.decode()
                        elif nf == 5:
                            name, val, ints = "", None, []
                            for af, _, av in _fields(nv):
                                if af == 1:
                                    name = av.decode()
                                elif af == 2:
                                    val = av
                                elif af == 3:
                                    val = _signed(av)
                                elif af == 8:
                                    ints.append(_signed(av))
                            attrs[name] = ints if val is None else val
                    model["nodes"].append((op, ins, outs, attrs))
                elif gf == 5:
                    name, arr = _read_tensor(gv)
                    model["inits"][name] = arr
                elif gf in (11, 12):
                    name = next(vv.decode() for ff, _, vv in _fields(gv) if ff == 1)
                    model["inputs" if gf == 11 else "outputs"].append(name)
    return model


def _slice(x, starts, ends, axes=None, steps=None):
    axes = range(len(starts)) if axes is None else axes
    steps = [1] * len(starts) if steps is None else steps
    idx = [slice(None)] * x.ndim
    for s, e, a, st in zip(starts, ends, axes, steps):
        idx[int(a)] = slice(int(s), int(min(e, x.shape[int(a)])), int(st))
    return x[tuple(idx)]


def _reshape(x, shape):
    shape = [x.shape[i] if d == 0 else int(d) for i, d in enumerate(shape)]
    return x.reshape(shape)


def _softmax(x, axis):
    e = np.exp(x - x.max(axis=axis, keepdims=True))
    return e / e.sum(axis=axis, keepdims=True)


_OPS = {
    "Gather": lambda a, i, axis=0: np.take(a[0], a[1], axis=axis),
    "Shape": lambda a, i: np.asarray(a[0].shape, dtype=np.int64),
    "Slice": lambda a, i: _slice(*a),
    "Concat": lambda a, i, axis=0: np.concatenate(a, axis=axis),
    "Unsqueeze": lambda a, i: np.expand_dims(a[0], tuple(int(x) for x in a[1])),
    "Reshape": lambda a, i: _reshape(a[0], a[1]),
    "Transpose": lambda a, i, perm=None: np.transpose(a[0], perm),
    "MatMul": lambda a, i: np.matmul(a[0], a[1]),
    "Add": lambda a, i: a[0] + a[1],
    "Sub": lambda a, i: a[0] - a[1],
    "Mul": lambda a, i: a[0] * a[1],
    "Div": lambda a, i: a[0] / a[1],
    "Sqrt": lambda a, i: np.sqrt(a[0]),
    "Sigmoid": lambda a, i: 1.0 / (1.0 + np.exp(-a[0])),
    "ReduceMean": lambda a, i, axes=None, keepdims=1: a[0].mean(axis=tuple(axes), keepdims=bool(keepdims)),
    "Softmax": lambda a, i, axis=-1: _softmax(a[0], axis),
}


def run_onnx(model: dict, feeds: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
    """Evaluate a loaded model with numpy (float32), node by node in file order."""
    env: Dict[str, np.ndarray] = dict(model["inits"])
    env.update(feeds)
    for op, ins, outs, attrs in model["nodes"]:
        fn = _OPS.get(op)
        if fn is None:
            raise NotImplementedError(f"operator {op}")
        env[outs[0]] = fn([env[x] for x in ins], ins, **attrs)
    return {k: env[k] for k in model["outputs"]}
