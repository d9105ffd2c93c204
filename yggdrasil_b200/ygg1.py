"""The YGG1 int8 model container: header, array table and per-expert records (host side, NumPy).

The product's loader is native (``ygg_load`` in ``csrc/ygg_load.cu`` parses the same bytes); this module writes files
(synthetic models for the tests and the benchmark) and reads headers for the Python API. The byte layout has to be the
reference's, so that files written by either side load in both:

* container (reference ``cpu/export.py:444-458``, ``cpu/ygg.cpp:78-86``): ``b"YGG1"``, 11 header int32s, the array
  count, then ``(name[32], offset int64, bytes int64)`` per array, zero padding to 64, then the arrays, each padded to
  64 bytes. Offsets count from the first array.
* per layer ``l`` the arrays are named ``l<l>_<tag>`` (``cpu/export.py:382-441``, ``cpu/ygg.cpp:173-202``); routed
  layers hold ``thr``, ``w``, optional ``r2b mulv vt mT vl mv``; every layer holds ``meta``, ``rec``, ``Q``, ``scal``
  and optional ``sqv mzl``.
* expert records (``cpu/export.py:321-350,410-430``): transition int16 ``[n/16][b/2][16][2]``, projections u8
  ``[rank/4][n][4]`` (stored +128), readout u8 (R = 8: ``[n/8][16][4]``, R >= 16: ``[R/16][n/4][16][4]``),
  table int16 rows, each record padded to 64 bytes.

One extension, written only when asked (``write_model(..., extended=True)``) and read only by this repository's
loader and oracle: ``d_state = 96`` (the 200M DNA benchmark shape) with its readout rank ``n/8 = 12``. Every packing
above holds at n = 96 (n/16, n/8 and n/4 are whole). A readout of rank 12 is stored in the R >= 16 layout as one group
of 16 rows whose rows 12-15 are zero weights; its group scales (``mzl``) stay 12 per expert. The reference's writer
and ``ygg`` refuse such files (``cpu/export.py:47``, ``cpu/ygg.cpp:141-146``).
"""
from __future__ import annotations

import dataclasses
import struct
from pathlib import Path

import numpy as np

MAGIC = b"YGG1"
HEADER_FIELDS = ("n_layers", "d_state", "block_size", "vocab", "router_depth", "readout_rank", "layer_input_rank",
                 "reserved", "router_token_dim", "input_rank", "shift")
RECORD_PARTS = ("transition", "layer_input_proj", "readout", "table", "input_proj", "bias", "input_scale")
SCALAR_NAMES = ("readout_scale", "unembed_scale", "rms_eps", "layer_input_scale")
OUTPUT_BIAS = "head_b"
SHIFT = 14
STATE_GROUP = 16
CLASS_PAD = 32
ALIGN = 64
RANK_MULTIPLE = 4
LIMITS = dict(d_state=(64, 128, 256), block_size=(8, 16), readout_rank=(8, 16, 32), max_layer_input_rank=64,
              max_input_rank=64, max_vocab=256, max_layers=8, max_router_depth=16)
EXTENDED_LIMITS = dict(LIMITS, d_state=(64, 96, 128, 256), readout_rank=(8, 12, 16, 32))
f32 = np.float32


def round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclasses.dataclass
class FactoredInput:
    """Factored input of a routed layer: T_r[x] = rint(f32(U_r v[x]) f32(su_r token_scale)) + c_r."""
    input_proj: np.ndarray     # (E, n, k) int8 values
    input_scale: np.ndarray    # (E,) f32 su_r
    bias: np.ndarray           # (E, n) int16 c_r
    token_code: np.ndarray     # (V, k) int8 values
    token_scale: np.ndarray    # (n,) f32


@dataclasses.dataclass
class IntLayer:
    """One int8 layer as integers and f32 scales (the fields of the reference's QuantLayer, cpu/export.py:184-205).

    A scale is one f32 (per tensor) or an f32 array (group scales)."""
    token_layer: bool
    n: int
    block: int
    depth: int
    transition: np.ndarray                 # (E, n/b, b, b) A16
    readout: np.ndarray                    # (E, R, n)
    readout_scale: object                  # f32 or (E, R)
    unembed: np.ndarray                    # (V, R)
    unembed_scale: object                  # f32 or (V,)
    table: np.ndarray = None               # (E, V, n) int16; token layer (V, 1, n)
    factored: FactoredInput = None
    router_weight: np.ndarray = None       # (2^D - 1, n) heap order from node 1
    router_threshold: np.ndarray = None    # (V, 2^D - 1) f32
    rms_eps: np.float32 = f32(0)
    state_r2: np.ndarray = None            # (n/16,) f32
    layer_input_down: np.ndarray = None    # (R2, n)
    layer_input_down_scale: np.ndarray = None  # (R2,) f32
    layer_input_proj: np.ndarray = None    # (E, n, R2)
    layer_input_scale: object = None       # f32 or (n,)


# ------------------------------------------------------------------------------------------------------ packing

def _pack_transition(a16: np.ndarray) -> np.ndarray:
    """(E, n/b, b, b) -> per expert int16 [n/16 row groups][b/2 column pairs][16 rows][2], as bytes (E, 2nb)."""
    e, g, b, _ = a16.shape
    n = g * b
    t = a16.reshape(e, n // 16, 16, b // 2, 2).transpose(0, 1, 3, 2, 4).astype(np.int16)
    return np.ascontiguousarray(t).reshape(e, -1).view(np.uint8)


def _pack_projection(u: np.ndarray) -> np.ndarray:
    """(E, n, rank) int8 values -> per expert u8 (u + 128) [rank/4][n][4]."""
    e, n, k = u.shape
    t = (u + 128).astype(np.uint8).reshape(e, n, k // 4, 4).transpose(0, 2, 1, 3)
    return np.ascontiguousarray(t).reshape(e, -1)


def _pack_readout(p: np.ndarray) -> np.ndarray:
    """(E, R, n) -> per expert u8 (p + 128): R = 8 as [n/8][16 lanes][4], R >= 16 as [R/16][n/4][16][4]; the
    extension's R = 12 as the R = 16 layout with zero rows 12-15."""
    e, r, n = p.shape
    if r == 12:
        p = np.concatenate([p, np.zeros((e, 4, n), p.dtype)], axis=1)
        r = 16
    if r >= 16:
        t = p.reshape(e, r // 16, 16, n // 4, 4).transpose(0, 1, 3, 2, 4)
    else:
        t = p.reshape(e, 8, n // 8, 2, 4).transpose(0, 2, 1, 3, 4)
    return np.ascontiguousarray((t + 128).astype(np.uint8)).reshape(e, -1)


def _pack_unembed(q: np.ndarray, vp: int) -> np.ndarray:
    """(V, R) -> u8 (q + 128) [R/4][VP][4], padded classes weight 0."""
    v, r = q.shape
    full = np.zeros((vp, r), np.int64)
    full[:v] = q
    return np.ascontiguousarray((full + 128).reshape(vp, r // 4, 4).transpose(1, 0, 2).astype(np.uint8))


def header_of(layers, vocab: int, router_token_dim: int = 0, input_rank: int = 0, extended: bool = False) -> dict:
    """Header values of layers, checked against LIMITS (EXTENDED_LIMITS if extended); ValueError names the failing
    field."""
    limits = EXTENDED_LIMITS if extended else LIMITS
    first, routed = layers[0], layers[1:]
    r2 = routed[0].layer_input_proj.shape[2] if routed and routed[0].layer_input_proj is not None else 0
    fac = [q.factored for q in layers if q.factored is not None]
    hdr = dict(n_layers=len(layers), d_state=first.n, block_size=first.block, vocab=vocab,
               router_depth=routed[0].depth if routed else 0, readout_rank=first.readout.shape[1],
               layer_input_rank=r2, reserved=0, router_token_dim=router_token_dim,
               input_rank=fac[0].input_proj.shape[2] if fac else input_rank, shift=SHIFT)

    def need(ok, field):
        if not ok:
            raise ValueError(f"YGG1 cannot hold {field} = {hdr.get(field)} (limits {limits})")
    for k in ("d_state", "block_size", "readout_rank"):
        need(hdr[k] in limits[k], k)
    need(r2 % RANK_MULTIPLE == 0 and r2 <= limits["max_layer_input_rank"], "layer_input_rank")
    need(vocab <= limits["max_vocab"], "vocab")
    need(1 <= len(layers) <= limits["max_layers"], "n_layers")
    need(not routed or 1 <= hdr["router_depth"] <= limits["max_router_depth"], "router_depth")
    need(not fac or (hdr["input_rank"] % RANK_MULTIPLE == 0
                     and RANK_MULTIPLE <= hdr["input_rank"] <= limits["max_input_rank"]), "input_rank")
    for q in routed:
        need(q.depth == hdr["router_depth"], "router_depth")
        need(q.readout.shape[1] == hdr["readout_rank"], "readout_rank")
        need((q.layer_input_proj is not None) == bool(r2)
             and (not r2 or q.layer_input_proj.shape[2] == r2), "layer_input_rank")
    return hdr


def _layer_arrays(l: int, q: IntLayer, hdr: dict):
    """(name, array) of layer l in file order."""
    n, v, r, r2 = hdr["d_state"], hdr["vocab"], hdr["readout_rank"], hdr["layer_input_rank"]
    vp, out = round_up(v, CLASS_PAD), []

    def add(name, a):
        out.append((f"l{l}_{name}", np.ascontiguousarray(a)))
    if not q.token_layer:
        e = 2 ** q.depth
        thr = np.zeros((v, e), f32)          # heap order from node 1, slot 0 unused
        thr[:, 1:] = q.router_threshold
        add("thr", thr)
        if q.state_r2 is not None:
            add("r2b", np.asarray(q.state_r2, f32))
        if np.ndim(q.layer_input_scale):
            add("mulv", np.asarray(q.layer_input_scale, f32))
        if q.factored is not None:
            add("vt", np.asarray(q.factored.token_code).astype(np.int8))
            add("mT", np.asarray(q.factored.token_scale, f32))
        w = np.zeros((e, n), np.int64)
        w[1:] = q.router_weight
        add("w", (w + 128).astype(np.uint8))
        if r2:
            groups = round_up(r2, 16) // 16
            vv = np.zeros((16 * groups, n), np.int64)
            vv[:r2] = q.layer_input_down
            add("vl", (vv + 128).reshape(groups, 16, n // 4, 4).transpose(0, 2, 1, 3).astype(np.uint8))
            mv = np.zeros(16 * groups, f32)
            mv[:r2] = q.layer_input_down_scale
            add("mv", mv)
    parts = {"transition": _pack_transition(q.transition)}
    if not q.token_layer and r2:
        parts["layer_input_proj"] = _pack_projection(q.layer_input_proj)
    parts["readout"] = _pack_readout(q.readout)
    if q.factored is not None:
        parts["input_proj"] = _pack_projection(q.factored.input_proj)
        parts["bias"] = np.ascontiguousarray(np.asarray(q.factored.bias, np.int16)).view(np.uint8)
        parts["input_scale"] = np.ascontiguousarray(np.asarray(q.factored.input_scale, f32)[:, None]).view(np.uint8)
    else:
        parts["table"] = np.ascontiguousarray(np.asarray(q.table, np.int16)).reshape(len(q.table), -1).view(np.uint8)
    offsets, off = {k: -1 for k in RECORD_PARTS}, 0
    for k, a in parts.items():
        offsets[k] = off
        off += a.shape[1]
    record = np.zeros((len(parts["transition"]), round_up(off, ALIGN)), np.uint8)
    for k, a in parts.items():
        record[:, offsets[k]:offsets[k] + a.shape[1]] = a
    del parts
    meta = [record.shape[1]] + [offsets[k] for k in RECORD_PARTS]
    add("meta", np.array(meta if q.factored is not None else meta[:5], np.int32))
    add("rec", record)
    add("Q", _pack_unembed(np.asarray(q.unembed), vp))
    if np.ndim(q.unembed_scale):
        sv = np.zeros(vp, f32)
        sv[:v] = q.unembed_scale
        add("sqv", sv)
    if np.ndim(q.readout_scale):             # R = 8: kernel lane i of the reference holds row i / 2
        rs = np.asarray(q.readout_scale, f32)
        add("mzl", np.repeat(rs, 2, axis=1) if r == 8 else rs)
    scal = dict(readout_scale=q.readout_scale, unembed_scale=q.unembed_scale, rms_eps=q.rms_eps,
                layer_input_scale=q.layer_input_scale)
    add("scal", np.array([0 if scal[k] is None or np.ndim(scal[k]) else scal[k] for k in SCALAR_NAMES], f32))
    return out


def write_model(layers, output_bias, path, router_token_dim: int = 0, input_rank: int = 0, extended: bool = False):
    """IntLayers -> a YGG1 file at path; returns (header dict, array bytes). extended: admit the d_state = 96
    extension (module docstring)."""
    v = len(output_bias)
    hdr = header_of(layers, v, router_token_dim, input_rank, extended)
    ob = np.zeros(round_up(v, CLASS_PAD), f32)
    ob[:v] = output_bias
    arrays = [(OUTPUT_BIAS, ob)] + [a for l, q in enumerate(layers) for a in _layer_arrays(l, q, hdr)]
    with open(path, "wb") as f:
        f.write(struct.pack(f"<4s{len(HEADER_FIELDS) + 1}i", MAGIC, *(hdr[k] for k in HEADER_FIELDS), len(arrays)))
        off, table = 0, []
        for name, a in arrays:
            if len(name.encode()) >= 32:
                raise ValueError(f"array name {name!r} longer than 31 bytes")
            table.append((name, off, a.nbytes))
            off += round_up(a.nbytes, ALIGN)
        for name, o, nb in table:
            f.write(struct.pack("<32sqq", name.encode(), o, nb))
        f.write(b"\0" * ((-f.tell()) % ALIGN))
        for (name, a), (_, o, nb) in zip(arrays, table):
            f.write(a.tobytes())
            f.write(b"\0" * (round_up(nb, ALIGN) - nb))
    return hdr, off


# ------------------------------------------------------------------------------------------------------ reading

def read_header(data) -> dict:
    """Header fields of a YGG1 file (path or bytes) -> dict; ValueError if it is not one."""
    if isinstance(data, (str, Path)):
        with open(data, "rb") as f:
            data = f.read(4 + 4 * (len(HEADER_FIELDS) + 1))
    data = bytes(data[:4 + 4 * (len(HEADER_FIELDS) + 1)])
    if len(data) < 4 + 4 * (len(HEADER_FIELDS) + 1) or data[:4] != MAGIC:
        raise ValueError("not a YGG1 model file")
    vals = struct.unpack(f"<{len(HEADER_FIELDS) + 1}i", data[4:])
    hdr = dict(zip(HEADER_FIELDS, vals[:-1]))
    hdr["n_arrays"] = vals[-1]
    return hdr


def array_table(data) -> dict:
    """name -> (offset from the array start, bytes), and the array start, of a YGG1 file given as bytes."""
    hdr = read_header(data)
    pos = 4 + 4 * (len(HEADER_FIELDS) + 1)
    table = {}
    for i in range(hdr["n_arrays"]):
        name, off, nb = struct.unpack_from("<32sqq", data, pos + 48 * i)
        table[name.rstrip(b"\0").decode()] = (off, nb)
    start = round_up(pos + 48 * hdr["n_arrays"], ALIGN)
    return table, start
