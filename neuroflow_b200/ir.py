"""NeuroIR v0 binary (.nneuroir) + NIRQ quantisation block: Python reader/writer.

The byte layout is the reference's (writer: neuroflow/ir/export.py:518-643, reader:
cpp/include/neuroflow/ir_loader.h:61-653) so that files written here load in the
reference runtime and reference-written files load here.  The product's loader is the
C++ one in csrc/nfx_ir.cpp; this module exists so that tests and bench.py can create
synthetic models and check the C++ loader.

Layout (little-endian):
  "NIR0", u16 version, u8 op_code, u8 0, i32 x (7 | 8) config, u8 activation, 3 pad,
  u32 n_weights, then per weight: u8 name_len, name, u8 ndim, i32 dims, f32 data.
  Optional trailer: "NIRQ", u8 1, u32 n, then per entry: u8 kind, u8 name_len, name,
  kind 0: f32 scale, i32 zp | kind 1: u32 n, u8 axis, f32[n], i32[n]
  kind 2: u32 n, u32 width, f32[n], i32[n] | kind 3: f32 scale.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Dict, List, Tuple

import numpy as np

# op name -> (op_code, version, config length); export.py:128-160 and :330-379.
OPS = {
    "FNO1d": (0x01, 2, 7),
    "FNO2d": (0x02, 2, 7),
    "FNO3d": (0x03, 3, 8),
    "DeepONet": (0x04, 3, 7),
    "TokenMixer": (0x05, 3, 8),
    "GraphOp": (0x06, 3, 8),
    "TokenMixer2D": (0x07, 3, 8),
    "GraphOp2D": (0x08, 3, 8),
}
OP_BY_CODE = {v[0]: k for k, v in OPS.items()}

# config key order per op (ir_loader.h:15-29)
CONFIG_KEYS = {
    "FNO1d": ["in_channels", "out_channels", "width", "modes", "n_layers", "pad_factor", "_"],
    "FNO2d": ["in_channels", "out_channels", "width", "modes_h", "modes_w", "n_layers",
              "pad_factor"],
    "FNO3d": ["in_channels", "out_channels", "width", "modes_h", "modes_w", "modes_d",
              "n_layers", "pad_factor"],
    "TokenMixer2D": ["in_dim", "out_dim", "latent_dim", "h", "w", "n_patches", "n_heads",
                     "n_layers"],
    "DeepONet": ["in_branch", "in_trunk", "latent_dim", "out_channels", "n_layers_branch",
                 "n_layers_trunk", "_"],
    "TokenMixer": ["in_dim", "out_dim", "latent_dim", "n_points", "n_patches", "n_heads",
                   "n_layers", "_"],
    "GraphOp": ["in_dim", "out_dim", "n_nodes", "hidden_dim", "n_layers", "_", "_", "_"],
    "GraphOp2D": ["in_dim", "out_dim", "h", "w", "hidden_dim", "n_layers", "_", "_"],
}


@dataclass
class PerTensor:
    scale: float
    zero_point: int


@dataclass
class PerChannel:
    scales: np.ndarray
    zero_points: np.ndarray
    channel_axis: int = 0


@dataclass
class PerToken:
    scales: np.ndarray
    zero_points: np.ndarray
    width: int


@dataclass
class FP8:
    scale: float


@dataclass
class Model:
    op: str
    config: Dict[str, int]
    activation: str = "gelu"
    weights: "Dict[str, np.ndarray]" = field(default_factory=dict)  # insertion-ordered
    qparams: "Dict[str, object]" = field(default_factory=dict)      # insertion-ordered
    quant_enabled: bool = False


def expected_weight_names(op: str, cfg: Dict[str, int]) -> List[str]:
    """Weight order the reference loader insists on (ir_loader.h:273-432)."""
    if op in ("FNO1d", "FNO2d", "FNO3d"):
        names = ["lift.weight", "lift.bias"]
        for i in range(cfg["n_layers"]):
            names += [f"specs.{i}.weights_real", f"specs.{i}.weights_imag",
                      f"locs.{i}.weight", f"locs.{i}.bias"]
        names += ["proj_q.weight", "proj_q.bias", "proj_out.weight", "proj_out.bias"]
        return names
    if op in ("TokenMixer", "TokenMixer2D"):
        names = ["slice_embed.proj.weight", "slice_embed.proj.bias"]
        for i in range(cfg["n_layers"]):
            p = f"blocks.{i}."
            for part in ("ln1", "q_proj", "k_proj", "v_proj", "o_proj", "ln2", "ffn0", "ffn1"):
                names += [p + part + ".weight", p + part + ".bias"]
        names += ["unslice.proj.weight", "unslice.proj.bias", "head.weight", "head.bias"]
        return names
    if op in ("GraphOp", "GraphOp2D"):
        names = ["lift.weight", "lift.bias"]
        for i in range(cfg["n_layers"]):
            p = f"blocks.{i}."
            names += [p + "lin_self.weight", p + "lin_self.bias", p + "lin_neigh.weight",
                      p + "lin_neigh.bias"]
        return names + ["head.weight", "head.bias", "graph.adj_offsets", "graph.adj_indices",
                        "graph.deg_inv"]
    if op == "DeepONet":
        names = []
        for net, n in (("branch", cfg["n_layers_branch"]), ("trunk", cfg["n_layers_trunk"])):
            for i in range(n):
                names += [f"{net}.layers.{i}.weight", f"{net}.layers.{i}.bias"]
        return names + ["bias.weight"]
    raise ValueError(f"unsupported op for the writer: {op}")


def write_bytes(m: Model) -> bytes:
    code, version, clen = OPS[m.op]
    keys = CONFIG_KEYS[m.op]
    cfg_block = [0 if k == "_" else int(m.config.get(k, 0)) for k in keys]
    assert len(cfg_block) == clen
    out = bytearray()
    out += b"NIR0"
    out += struct.pack("<HBB", version, code, 0)
    out += struct.pack(f"<{clen}i", *cfg_block)
    out += struct.pack("<B", 1 if m.activation == "relu" else 0) + b"\x00\x00\x00"
    out += struct.pack("<I", len(m.weights))
    for name, arr in m.weights.items():
        a = np.ascontiguousarray(arr, dtype=np.float32)
        nb = name.encode()
        out += struct.pack("<B", len(nb)) + nb
        out += struct.pack("<B", a.ndim) + struct.pack(f"<{a.ndim}i", *a.shape)
        out += a.tobytes()
    if m.quant_enabled:
        out += b"NIRQ" + struct.pack("<B", 1) + struct.pack("<I", len(m.qparams))
        for name, qp in m.qparams.items():
            nb = name.encode()
            if isinstance(qp, PerToken):
                n = len(qp.scales)
                out += struct.pack("<BB", 2, len(nb)) + nb + struct.pack("<II", n, qp.width)
                out += np.asarray(qp.scales, np.float32).tobytes()
                out += np.asarray(qp.zero_points, np.int32).tobytes()
            elif isinstance(qp, PerChannel):
                n = len(qp.scales)
                out += struct.pack("<BB", 1, len(nb)) + nb + struct.pack("<IB", n, qp.channel_axis)
                out += np.asarray(qp.scales, np.float32).tobytes()
                out += np.asarray(qp.zero_points, np.int32).tobytes()
            elif isinstance(qp, FP8):
                out += struct.pack("<BB", 3, len(nb)) + nb + struct.pack("<f", qp.scale)
            else:
                out += struct.pack("<BB", 0, len(nb)) + nb
                out += struct.pack("<fi", float(qp.scale), int(qp.zero_point))
    return bytes(out)


def write(path: str, m: Model) -> None:
    with open(path, "wb") as f:
        f.write(write_bytes(m))


class _Reader:
    def __init__(self, buf: bytes):
        self.b = buf
        self.o = 0

    def take(self, fmt: str) -> Tuple:
        n = struct.calcsize(fmt)
        if self.o + n > len(self.b):
            raise ValueError("truncated")
        v = struct.unpack_from(fmt, self.b, self.o)
        self.o += n
        return v

    def raw(self, n: int) -> bytes:
        if self.o + n > len(self.b):
            raise ValueError("truncated")
        v = self.b[self.o:self.o + n]
        self.o += n
        return v


def read_bytes(buf: bytes) -> Model:
    r = _Reader(buf)
    if r.raw(4) != b"NIR0":
        raise ValueError("bad magic")
    version, code, _ = r.take("<HBB")
    if version not in (1, 2, 3):
        raise ValueError("unsupported version")
    op = OP_BY_CODE[code]
    clen = OPS[op][2]
    cfg_vals = r.take(f"<{clen}i")
    keys = CONFIG_KEYS[op]
    cfg = {k: v for k, v in zip(keys, cfg_vals) if k != "_"}
    (act,) = r.take("<B")
    r.raw(3)
    (nw,) = r.take("<I")
    weights = {}
    for _ in range(nw):
        (ln,) = r.take("<B")
        name = r.raw(ln).decode()
        (nd,) = r.take("<B")
        dims = r.take(f"<{nd}i") if nd else ()
        cnt = int(np.prod(dims)) if nd else 1
        weights[name] = np.frombuffer(r.raw(4 * cnt), np.float32).reshape(dims).copy()
    m = Model(op=op, config=cfg, activation="relu" if act == 1 else "gelu", weights=weights)
    if r.o + 4 <= len(buf) and buf[r.o:r.o + 4] == b"NIRQ":
        r.raw(4)
        (flag,) = r.take("<B")
        if flag != 1:
            raise ValueError("unsupported quant_flag")
        m.quant_enabled = True
        (nq,) = r.take("<I")
        for _ in range(nq):
            kind, ln = r.take("<BB")
            name = r.raw(ln).decode()
            if kind == 0:
                s, z = r.take("<fi")
                m.qparams[name] = PerTensor(s, z)
            elif kind == 1:
                n, axis = r.take("<IB")
                sc = np.frombuffer(r.raw(4 * n), np.float32).copy()
                zp = np.frombuffer(r.raw(4 * n), np.int32).copy()
                m.qparams[name] = PerChannel(sc, zp, axis)
            elif kind == 2:
                n, width = r.take("<II")
                sc = np.frombuffer(r.raw(4 * n), np.float32).copy()
                zp = np.frombuffer(r.raw(4 * n), np.int32).copy()
                m.qparams[name] = PerToken(sc, zp, width)
            elif kind == 3:
                (s,) = r.take("<f")
                m.qparams[name] = FP8(s)
            else:
                raise ValueError("unsupported qparam kind")
    return m


def read(path: str) -> Model:
    with open(path, "rb") as f:
        return read_bytes(f.read())
