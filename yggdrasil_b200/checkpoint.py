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
computes the same matrix with torch, yggdrasil/inference_triton.py:109-114; its exporter uses JAX's expm). Two float64
expm implementations agree to ~1e-15, so a transition coefficient rint(2^14 A) could differ only where A lies within
~1e-11 of a half step; the tests compare transitions64 with scipy's float64 expm.

Quantisation (`quantize`) is organised as a scale plan per layer (`scale_plans`: every state, reference and readout
scale, decided from the calibration maxima before any weight is touched), then one function per kind of weight
(readout and head, token input, router, layer input) that folds the planned scales in and rounds. The rounding
steps themselves are the reference's (cpu/export.py:158-265), since the rebuilt file must equal its export.
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


@dataclasses.dataclass
class ScalePlan:
    """The quantisation scales of one layer, fixed before any tensor is quantised.

    state: the f64 scale of each state coordinate (n,): one value for the layer (tensor mode) or one per group of 16
    coordinates; ref: the layer's reference scale (the largest group scale); readout: the scale of the readout codes
    zq; below, below_ref: the state scales of the layer underneath relative to its reference scale, and that reference
    (None, 1.0 for the token layer). A layer's state is stored in units of `state`, so every weight that reads or
    writes a state has the state scales folded into it."""
    state: np.ndarray
    ref: float
    readout: float
    below: np.ndarray | None
    below_ref: float


def scale_plans(layers, stats, hmargin=1.0, group=False) -> list:
    """The ScalePlan of every layer, from the calibration maxima: state range x hmargin over 127, per layer or per
    group of 16 coordinates (a group's maximum is floored at 1e-3 of the layer's), and the readout range over 127."""
    plans = []
    below, below_ref = None, 1.0
    for fl, st in zip(layers, stats):
        if group:
            gmax = np.asarray(st.state_group_max, np.float64)
            floor = GROUP_SCALE_FLOOR * max(np.max(gmax), SCALE_FLOOR)
            per_group = np.maximum(gmax, floor) * hmargin / INT8_MAX
            state, ref = np.repeat(per_group, STATE_GROUP), float(per_group.max())
        else:
            ref = st.state_max * hmargin / INT8_MAX
            state = np.full(fl.n, ref)
        plans.append(ScalePlan(state=state, ref=ref, readout=max(st.readout_max, SCALE_FLOOR) / INT8_MAX,
                               below=below, below_ref=below_ref))
        below, below_ref = state / ref, ref
    return plans


def int8_codes(w, per_row: bool):
    """Symmetric int8 codes of w and their scale: one per row (over the last axis; an array) or one for the tensor (a
    float). scale = max(|w|, 1e-12) / 127 and code = rint(w / scale), in float64."""
    w = np.asarray(w, np.float64)
    if per_row:
        scale = np.maximum(np.abs(w).max(-1), SCALE_FLOOR) / INT8_MAX
        return np.rint(w / scale[..., None]).astype(np.int64), scale
    scale = max(np.abs(w).max(), SCALE_FLOOR) / INT8_MAX
    return np.rint(w / scale).astype(np.int64), scale


def int16_saturated(x, rows_per_pass: int = EXPERT_CHUNK):
    """rint(x) saturated to int16, computed `rows_per_pass` leading rows at a time (the tables are large)."""
    out = np.empty(x.shape, np.int16)
    for a in range(0, len(x), rows_per_pass):
        out[a:a + rows_per_pass] = np.clip(np.rint(x[a:a + rows_per_pass]), -32768, 32767)
    return out


def _readout_and_head(fl, plan, group):
    """Readout codes P and the scale of zq = rint(f32(P q) * scale); unembedding codes Q and their scale. With group
    scales the state scales go into the readout rows (one scale per expert and row), and Q has one scale per class."""
    if group:
        codes, row_scale = int8_codes(fl.readout * plan.state[None, None, :], per_row=True)
        readout_scale = (row_scale / plan.readout).astype(f32)
    else:
        codes, s = int8_codes(fl.readout, per_row=False)
        readout_scale = f32(s * plan.ref / plan.readout)
    head, head_scale = int8_codes(fl.unembed, per_row=group)
    return codes, readout_scale, head, f32(head_scale * plan.readout)


def _input_part(fl, plan, factored):
    """The token input in state units: the token layer keeps T_x[x] only; a routed layer keeps T_r[x] as int16 tables
    or, factored, int8 U_r (one scale per expert) and token codes v[x] (one scale) plus an int16 bias c_r."""
    if fl.token_layer:
        diag = fl.table[np.arange(fl.table.shape[1]), np.arange(fl.table.shape[1])]
        return {"table": int16_saturated(diag / plan.state)[:, None]}
    if not factored:
        return {"table": int16_saturated(fl.table / plan.state)}
    codes, code_scale = int8_codes(fl.token_embed, per_row=False)
    expert_scale = np.maximum(np.abs(fl.input_proj).reshape(len(fl.input_proj), -1).max(-1), SCALE_FLOOR) / INT8_MAX
    return {"factored": FactoredInput(
        input_proj=np.rint(fl.input_proj / expert_scale[:, None, None]).astype(np.int64),
        input_scale=expert_scale.astype(f32), bias=int16_saturated(fl.bias / plan.state), token_code=codes,
        token_scale=(code_scale / plan.state).astype(f32))}


def _router_part(fl, plan, group):
    """Router rows on the layer below's stored state (its relative scales folded in, one int8 scale per node), the
    token part of each node test folded into per-(token, node) thresholds in those units, and rho's epsilon in the
    units of the layer below."""
    F = fl.router_token_dim
    token_part = fl.router_embed @ fl.router_weight[:, :F].T + fl.router_bias[None, :]
    rows, node_scale = int8_codes(fl.router_weight[:, F:] * plan.below[None, :], per_row=True)
    out = {"router_weight": rows, "router_threshold": (-token_part / node_scale[None, :]).astype(f32),
           "rms_eps": f32(RMS_EPS / plan.below_ref ** 2)}
    if group:
        out["state_r2"] = (plan.below[::STATE_GROUP] ** 2).astype(f32)
    return out


def _layer_input_part(fl, plan, st, group):
    """The low-rank input from the layer below: V' rows on its stored state (per-row scales, over the layer-input
    range), and U'_r (one scale) mapped into this layer's state units, per coordinate with group scales."""
    down, row_scale = int8_codes(fl.layer_input_down * plan.below[None, :], per_row=True)
    code_scale = max(st.layer_input_max, SCALE_FLOOR) / INT8_MAX
    proj, proj_scale = int8_codes(fl.layer_input_proj, per_row=False)
    to_state = proj_scale * code_scale / plan.state
    return {"layer_input_down": down, "layer_input_down_scale": (row_scale / code_scale).astype(f32),
            "layer_input_proj": proj, "layer_input_scale": to_state.astype(f32) if group else f32(to_state[0])}


def quantize(layers, stats, hmargin=1.0, group=False, factored=False):
    """Int8 layers from float layers and calibration maxima: the scales of every layer first (scale_plans), then
    each part of each layer quantised on its own. Every rounding is the reference's (cpu/export.py:158-265: the same
    float64 quotients, rint, int8 and int16 saturation, and the f32 casts of the stored scales), so that a file
    rebuilt here equals the reference's export byte for byte."""
    plans = scale_plans(layers, stats, hmargin, group)
    out = []
    for fl, st, plan in zip(layers, stats, plans):
        readout, readout_scale, head, head_scale = _readout_and_head(fl, plan, group)
        kw = _input_part(fl, plan, factored)
        if not fl.token_layer:
            kw.update(_router_part(fl, plan, group))
            if fl.layer_input_down is not None:
                kw.update(_layer_input_part(fl, plan, st, group))
        out.append(IntLayer(token_layer=fl.token_layer, n=fl.n, block=fl.block, depth=fl.depth,
                            transition=np.rint(fl.transition * 2.0 ** SHIFT).astype(np.int64), readout=readout,
                            readout_scale=readout_scale, unembed=head, unembed_scale=head_scale, **kw))
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
