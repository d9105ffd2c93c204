"""Float checkpoints (.npz) to the int8 YGG1 model on the host, without JAX: read, hard layers, quantise, write.

The reference builds the int8 file in its exporter (cpu/export.py:548-573):
- `inference.read` loads the checkpoint (yggdrasil/inference.py:129-139, key aliases from yggdrasil/config.py:80-111);
- `hard_layers` precomputes the transitions and tables in float64 (cpu/export.py:99-116; the transitions are
  yggdrasil/experts.py:8-11, the tables yggdrasil/inference.py:150);
- `calibrate` measures the state ranges on training data (needs JAX and the datasets);
- `quantize` turns the float layers and the measured ranges into int8 (cpu/export.py:158-265).
The export also writes `model.bin.json`, holding the measured ranges (`stats`) and the chosen `quantize` arguments.
From a checkpoint and that record, the int8 model can be rebuilt without calibrating again, as cpu/check.py:43-47
does. This module does that rebuild with numpy and torch.

Transitions: blockdiag expm((G - G^T) / 2) uses torch.linalg.matrix_exp in float64 (the reference's Triton backend
computes the same matrix the same way, yggdrasil/inference_triton.py:109-114). The reference's exporter uses JAX's
expm; the two agree to ~1e-15, so a transition coefficient rint(2^14 A) could differ only where A lies within ~1e-11
of a half step.
"""
from __future__ import annotations

import dataclasses
import json
import os
import tempfile
from pathlib import Path

import numpy as np

from .ygg1 import SHIFT, STATE_GROUP, FactoredInput, IntLayer, write_model

f32 = np.float32
INT8_MAX = 127
SCALE_FLOOR = 1e-12
GROUP_SCALE_FLOOR = 1e-3
EXPERT_CHUNK = 256
RMS_EPS = 1e-6
LAYER_KEYS = {"token_embed", "input_proj", "bias", "rotation", "decay", "readout", "unembed", "router_embed",
              "router_weight", "router_bias", "layer_input_down", "layer_input_proj"}
# old checkpoint keys -> new (the released checkpoints use the old ones)
KEY_ALIASES = {
    "root": "token_layer", "branches": "routed_layers", "head_b": "output_bias", "levels": "hre_levels",
    "v_tok": "token_embed", "u_in": "input_proj", "c": "bias", "p_out": "readout", "q_out": "unembed",
    "skew": "rotation", "d_raw": "decay", "tok": "router_embed", "w_node": "router_weight", "b_node": "router_bias",
    "v_low": "layer_input_down", "u_low": "layer_input_proj",
}


# ------------------------------------------------------------------------------------------------------ read

def read_checkpoint(path):
    """.npz (new or old keys) -> (layers [token layer, routed layers...] as dicts of float32 arrays, output bias)."""
    with np.load(path) as z:
        flat = {"/".join(KEY_ALIASES.get(p, p) for p in name.split("/")): z[name].astype(np.float32)
                for name in z.files}
    token, routed, output_bias = {}, [], None
    for name, value in flat.items():
        top, *rest = name.split("/")
        if top == "token_layer":
            token[rest[0]] = value
        elif top == "routed_layers":
            i = int(rest[0])
            routed += [{} for _ in range(i + 1 - len(routed))]
            routed[i][rest[1]] = value
        elif top == "output_bias":
            output_bias = value
        else:
            raise ValueError(f"{path}: unknown checkpoint key {name!r}")
    layers = [token, *routed]
    for p in layers:
        if bad := set(p) - LAYER_KEYS:
            raise NotImplementedError(f"{path}: unsupported layer arrays {sorted(bad)}")
        if len(p["readout"]) != len(p["bias"]):
            raise NotImplementedError(f"{path}: the readout needs one matrix per expert")
    if output_bias is None:
        raise ValueError(f"{path}: no output_bias")
    return layers, output_bias


# ------------------------------------------------------------------------------------------------------ float layers

@dataclasses.dataclass
class FloatLayer:
    """One layer of the float64 inference model (the fields of the reference's FloatLayer, cpu/export.py:68-96)."""
    token_layer: bool
    transition: np.ndarray            # (E, n/b, b, b)
    table: np.ndarray                 # (E, V, n) T_r[x] = U_r v(x) + c_r
    input_proj: np.ndarray            # (E, n, input_rank)
    token_embed: np.ndarray           # (V, input_rank)
    bias: np.ndarray                  # (E, n)
    readout: np.ndarray               # (E, R, n)
    unembed: np.ndarray               # (V, R)
    router_embed: np.ndarray = None
    router_weight: np.ndarray = None
    router_bias: np.ndarray = None
    layer_input_down: np.ndarray = None
    layer_input_proj: np.ndarray = None
    depth: int = 0

    @property
    def n(self):
        return self.bias.shape[1]

    @property
    def block(self):
        return self.transition.shape[-1]

    @property
    def router_token_dim(self):
        return 0 if self.token_layer else self.router_embed.shape[1]


def transitions64(rotation, decay):
    """diag(clip(decay, -1, 1)) blockdiag(expm((G - G^T) / 2)) in float64 -> (E, n/b, b, b)."""
    import torch
    g = torch.as_tensor(np.asarray(rotation, np.float64))
    g = 0.5 * (g - g.transpose(-1, -2))
    d = torch.as_tensor(np.asarray(decay, np.float64)).clamp(-1.0, 1.0).reshape(g.shape[:-1])
    return (d[..., None] * torch.linalg.matrix_exp(g)).numpy()


def float_layers(layers, output_bias):
    """read_checkpoint() layers -> FloatLayers in float64 (the hard-routing inference model)."""
    out = []
    routed_depth = 0
    for i, p in enumerate(layers):
        p = {k: np.asarray(v, np.float64) for k, v in p.items()}
        if "rotation" not in p:
            raise NotImplementedError("experts without transitions (expert_type output) have no int8 export")
        if i and p["router_weight"].shape[1] == p["router_embed"].shape[1]:
            raise NotImplementedError("routing on the token only (router_input token) has no int8 export")
        if i:
            routed_depth = (p["router_weight"].shape[0] + 1).bit_length() - 1
        table = np.einsum("lkr,vr->lvk", p["input_proj"], p["token_embed"]) + p["bias"][:, None]
        kw = {k: p[k] for k in ("router_embed", "router_weight", "router_bias", "layer_input_down",
                                "layer_input_proj") if k in p}
        out.append(FloatLayer(token_layer=i == 0, transition=transitions64(p["rotation"], p["decay"]), table=table,
                              input_proj=p["input_proj"], token_embed=p["token_embed"], bias=p["bias"],
                              readout=p["readout"], unembed=p["unembed"], depth=routed_depth if i else 0, **kw))
    return out


# ------------------------------------------------------------------------------------------------------ quantise

@dataclasses.dataclass
class LayerStats:
    """Calibration maxima of one layer (the `stats` entries of the export record)."""
    state_max: float
    layer_input_max: float
    readout_max: float
    state_group_max: np.ndarray
    readout_row_max: np.ndarray


def _qrow(w):
    s = np.maximum(np.abs(w).max(-1, keepdims=True), SCALE_FLOOR) / INT8_MAX
    return np.rint(w / s).astype(np.int64), s[..., 0]


def _qten(w):
    s = max(np.abs(w).max(), SCALE_FLOOR) / INT8_MAX
    return np.rint(w / s).astype(np.int64), s


def _sat16(x):
    return np.clip(np.rint(x), -32768, 32767)


def _factor(fl, sc):
    vt, s_vt = _qten(fl.token_embed)
    su = np.maximum(np.abs(fl.input_proj).reshape(len(fl.input_proj), -1).max(-1), SCALE_FLOOR) / INT8_MAX
    return FactoredInput(input_proj=np.rint(fl.input_proj / su[:, None, None]).astype(np.int64),
                         input_scale=su.astype(f32), bias=_sat16(fl.bias / sc).astype(np.int16), token_code=vt,
                         token_scale=(s_vt / sc).astype(f32))


def quantize(layers, stats, hmargin=1.0, group=False, factored=False):
    """Int8 layers from float layers and calibration maxima, one state scale per layer or per 16 coordinates
    (group). The steps of cpu/export.py:216-265, so that a file rebuilt here equals the reference's export."""
    out, rel_prev, s_prev = [], None, 1.0
    for fl, st in zip(layers, stats):
        if group:
            g = np.maximum(np.asarray(st.state_group_max, np.float64),
                           GROUP_SCALE_FLOOR * max(np.max(st.state_group_max), SCALE_FLOOR))
            sg = g * hmargin / INT8_MAX
            sc, s_ref = np.repeat(sg, STATE_GROUP), float(sg.max())
        else:
            s_ref = st.state_max * hmargin / INT8_MAX
            sc = np.full(fl.n, s_ref)
        s_z = max(st.readout_max, SCALE_FLOOR) / INT8_MAX
        if group:
            readout, s_p = _qrow(fl.readout * sc[None, None, :])
            readout_scale = (s_p / s_z).astype(f32)
        else:
            readout, s_p = _qten(fl.readout)
            readout_scale = f32(s_p * s_ref / s_z)
        unembed, s_q = (_qrow if group else _qten)(fl.unembed)
        q = IntLayer(token_layer=fl.token_layer, n=fl.n, block=fl.block, depth=fl.depth,
                     transition=np.rint(fl.transition * 2.0 ** SHIFT).astype(np.int64), readout=readout,
                     readout_scale=readout_scale, unembed=unembed, unembed_scale=f32(s_q * s_z))
        if fl.token_layer:
            ar = np.arange(fl.table.shape[1])
            q.table = _sat16(fl.table[ar, ar] / sc).astype(np.int16)[:, None]
        elif factored:
            q.factored = _factor(fl, sc)
        else:
            q.table = np.empty(fl.table.shape, np.int16)
            for j in range(0, len(fl.table), EXPERT_CHUNK):
                q.table[j:j + EXPERT_CHUNK] = _sat16(fl.table[j:j + EXPERT_CHUNK] / sc)
        if not fl.token_layer:
            F = fl.router_token_dim
            token_part = fl.router_embed @ fl.router_weight[:, :F].T + fl.router_bias[None, :]
            q.router_weight, sw = _qrow(fl.router_weight[:, F:] * rel_prev[None, :])
            q.router_threshold = (-token_part / sw[None, :]).astype(f32)
            q.rms_eps = f32(RMS_EPS / s_prev ** 2)
            if group:
                q.state_r2 = (rel_prev[::STATE_GROUP] ** 2).astype(f32)
            if fl.layer_input_down is not None:
                q.layer_input_down, sv = _qrow(fl.layer_input_down * rel_prev[None, :])
                s_v = max(st.layer_input_max, SCALE_FLOOR) / INT8_MAX
                q.layer_input_down_scale = (sv / s_v).astype(f32)
                q.layer_input_proj, s_u = _qten(fl.layer_input_proj)
                scale = s_u * s_v / sc
                q.layer_input_scale = scale.astype(f32) if group else f32(scale[0])
        rel_prev, s_prev = sc / s_ref, s_ref
        out.append(q)
    return out


def stats_from_record(record) -> list:
    return [LayerStats(**{k: (np.asarray(v, np.float64) if isinstance(v, list) else v) for k, v in s.items()})
            for s in record["stats"]]


def export_bytes(npz, record) -> bytes:
    """The YGG1 bytes of checkpoint npz quantised with the export record (path or dict: its `stats` and
    `quantize` arguments, as cpu/export.py:563-572 writes them)."""
    if not isinstance(record, dict):
        record = json.loads(Path(record).read_text())
    layers, output_bias = read_checkpoint(npz)
    fl = float_layers(layers, output_bias)
    q = quantize(fl, stats_from_record(record), **record["quantize"])
    fd, tmp = tempfile.mkstemp(suffix=".bin")
    os.close(fd)
    try:
        write_model(q, output_bias, tmp, router_token_dim=fl[-1].router_token_dim,
                    input_rank=fl[0].token_embed.shape[1])
        return Path(tmp).read_bytes()
    finally:
        os.unlink(tmp)
