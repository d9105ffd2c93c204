"""Calibration and int8 export on the GPU: the reference's exporter (cpu/export.py:129-153 `calibrate`, :548-573
`export`) with its float64 JAX scan replaced by the B200 fp32 float step.

    from yggdrasil_b200.calibration import export
    record = export("run.npz", "model.bin", windows)      # windows: (S, T) int tokens, the calibration text

`calibrate(float_model, windows)` runs the float model (backend "b200f") over the windows from a zero state and keeps,
per layer, the maxima the reference's `LayerStats` holds (cpu/export.py:120-126): |h| per group of 16 state
coordinates, |V' rms(h_below)| and |P_r h| per readout row (the kernel accumulates them, `ygg_fstep_stats`).
`export` then does what the reference's export does with them: for each state-scale mode and each range margin of
its grid (HMARGIN_GRID) it quantises the float layers (`checkpoint.quantize`), scores the windows with the int8 model
on the GPU (backend "b200", the bit-exact int8 step), keeps the setting with the fewest bits, and writes the YGG1 file
and its export record (`<out>.json`: the stats and the `quantize` arguments, from which `checkpoint.export_bytes`
rebuilds the file). The datasets the reference calibrates on are not part of this library: the caller passes the
windows.

The reference calibrates in float64; this calibration runs in fp32, so its maxima agree with the reference's to about
1e-6 relative, and a file exported here can differ from the reference's in codes that sit on a rounding boundary.
"""
from __future__ import annotations

import json
import os
import tempfile
from pathlib import Path

import numpy as np

from . import checkpoint as ck
from ._native import check

HMARGIN_GRID = (1.0, 0.85, 0.7, 0.6)     # the reference's range margins (cpu/export.py:32)


def _torch():
    import torch
    return torch


def calibrate(model, windows, batch: int = 4096) -> list:
    """LayerStats (yggdrasil_b200.checkpoint) of every layer over windows (S, T), the float model `model`
    (B200FloatYggdrasil) stepping each batch of rows from a zero state."""
    torch = _torch()
    from ._native import flib
    x = np.atleast_2d(np.asarray(windows))
    if x.size and (x.min() < 0 or x.max() >= model.vocab):
        raise ValueError(f"windows: tokens out of range [0, {model.vocab})")
    L, n = model.layers, model.n
    R = model.readout_rank
    width = n // 16 + 1 + R
    dev = model.device
    stats = torch.zeros(L, width, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev), torch.no_grad():
        for i in range(0, len(x), batch):
            xb = torch.as_tensor(np.ascontiguousarray(x[i:i + batch], np.int32), device=dev)
            st = model.init_state(len(xb))
            lg = torch.empty(len(xb), model.classes, dtype=torch.float32, device=dev)
            for t in range(xb.shape[1]):
                tok = xb[:, t].contiguous()
                check(flib().ygg_fstep_stats(model._h, len(xb), tok.data_ptr(), st.data_ptr(), st.data_ptr(),
                                             lg.data_ptr(), None, stats.data_ptr(), stream), "ygg_fstep_stats")
        s = stats.cpu().numpy().astype(np.float64)
    model.status()
    out = []
    for l in range(L):
        groups, v, rows = s[l, :n // 16], float(s[l, n // 16]), s[l, n // 16 + 1:]
        out.append(ck.LayerStats(state_max=float(groups.max()), layer_input_max=v, readout_max=float(rows.max()),
                                 state_group_max=groups, readout_row_max=rows))
    return out


def _stats_record(stats) -> list:
    return [{"state_max": s.state_max, "layer_input_max": s.layer_input_max, "readout_max": s.readout_max,
             "state_group_max": np.asarray(s.state_group_max).tolist(),
             "readout_row_max": np.asarray(s.readout_row_max).tolist()} for s in stats]


def export(npz, out, windows, hmargin: float = 0.0, storage: str = "table", state_scale: str = "auto",
           device="cuda", batch: int = 4096) -> dict:
    """Calibrate checkpoint `npz` on `windows` (S, T + 1) int tokens, quantise, write the YGG1 file `out` and its
    export record `<out>.json`; returns the record (cpu/export.py:548-573). The first T tokens of each row calibrate
    the float model; the int8 candidates score the T next-token predictions of each row (bits per token, as the
    reference's bpc of int_forward logits against the shifted targets). hmargin 0: pick the range margin from
    HMARGIN_GRID by those bits; storage "table" or "factored"; state_scale "auto" (tensor and group scales tried),
    "tensor" or "group"."""
    from .float_backend import B200FloatYggdrasil
    from .inference import B200Yggdrasil
    from .ygg1 import write_model
    if storage not in ("table", "factored") or state_scale not in ("auto", "tensor", "group"):
        raise ValueError(f"storage {storage!r} / state_scale {state_scale!r}")
    w = np.atleast_2d(np.asarray(windows))
    if w.shape[1] < 2:
        raise ValueError("windows need at least two tokens per row (calibration tokens and their next tokens)")
    raw, output_bias = ck.read_checkpoint(npz)
    layers = ck.float_layers(raw, output_bias)             # float64, and the variants the int8 format cannot hold
    fmodel = B200FloatYggdrasil(raw, output_bias, device=device)
    stats = calibrate(fmodel, w[:, :-1], batch=batch)
    del fmodel
    fac = storage == "factored"
    kw = dict(router_token_dim=layers[-1].router_token_dim, input_rank=layers[0].token_embed.shape[1])
    modes = {"auto": ("tensor", "group"), "tensor": ("tensor",), "group": ("group",)}[state_scale]
    fd, tmp = tempfile.mkstemp(suffix=".bin")
    os.close(fd)
    cal = {}
    try:
        for mode in modes:
            for hm in ((hmargin,) if hmargin else HMARGIN_GRID):
                write_model(ck.quantize(layers, stats, hm, mode == "group", fac), output_bias, tmp, **kw)
                m8 = B200Yggdrasil(tmp, device=device)
                cal[(mode, hm)] = float(m8.score(w, batch=batch).sum() / (w.shape[0] * (w.shape[1] - 1)))
                del m8
    finally:
        os.unlink(tmp)
    mode, hm = min(cal, key=cal.get)
    args = dict(hmargin=hm, group=mode == "group", factored=fac)
    hdr, nbytes = write_model(ck.quantize(layers, stats, **args), output_bias, out, **kw)
    rec = dict(header=hdr, bytes=nbytes, quantize=args, state_scale=mode, storage=storage,
               calib_seq_len=int(w.shape[1] - 1), calib_windows=int(w.shape[0]),
               calib_bpc={f"{k[0]}_{k[1]}": v for k, v in cal.items()}, stats=_stats_record(stats),
               calibrated_on="b200f fp32 step")
    Path(str(out) + ".json").write_text(json.dumps(rec))
    return rec
