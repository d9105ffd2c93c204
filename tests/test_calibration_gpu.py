"""Calibration and int8 export on the GPU (yggdrasil_b200.calibration) against the reference's definitions (GPU).

The calibration maxima (cpu/export.py:120-153: |h| per group of 16 coordinates, |V' rms(h_below)|, |P_r h| per
readout row) from the fp32 float step must equal the same maxima of the reference's own fp32 Triton step on the
fixture's windows (tests/golden/float_cases.npz) and of the float64 oracle, within 1e-5 relative. The export must
pick the setting with the fewest calibration bits, write a file that its own record rebuilds byte for byte through
checkpoint.export_bytes (the rebuild of cpu/check.py:43-47), and that file must run bit-exactly against the int8
oracle.
"""
import json

import numpy as np
import pytest
from test_float_oracle import FLOAT, float_case

import checkpoints as C
from oracle import oracle as O
from oracle.float_oracle import FloatOracle

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def stats_arrays(stats):
    return (np.stack([s.state_group_max for s in stats]), np.array([s.layer_input_max for s in stats]),
            np.stack([s.readout_row_max for s in stats]))


@pytest.mark.parametrize("rec", FLOAT, ids=[r["name"] for r in FLOAT])
def test_calibration_matches_reference_maxima(rec, tmp_path):
    from yggdrasil_b200.calibration import calibrate
    from yggdrasil_b200.float_backend import B200FloatYggdrasil
    npz, ref = float_case(rec, tmp_path)
    g, v, r = stats_arrays(calibrate(B200FloatYggdrasil.from_checkpoint(npz), ref["tokens"]))
    np.testing.assert_allclose(g, ref["stats_groups"], rtol=RTOL)
    np.testing.assert_allclose(v, ref["stats_layer_input"], rtol=RTOL)
    np.testing.assert_allclose(r, ref["stats_rows"], rtol=RTOL)


def test_calibration_matches_oracle_over_batches(tmp_path):
    """More windows than one launch batch (batch=40 over 100 rows): the maxima run across calls."""
    from yggdrasil_b200.calibration import calibrate
    from yggdrasil_b200.checkpoint import read_checkpoint
    from yggdrasil_b200.float_backend import B200FloatYggdrasil
    npz = tmp_path / "ck.npz"
    C.synthetic_checkpoint(npz, seed=8)
    x = np.random.default_rng(3).integers(0, 27, (100, 24))
    got = stats_arrays(calibrate(B200FloatYggdrasil.from_checkpoint(npz), x, batch=40))
    want = FloatOracle(*read_checkpoint(npz)).calibrate(x)
    np.testing.assert_allclose(got[0], np.stack([s[0] for s in want]), rtol=RTOL)
    np.testing.assert_allclose(got[1], np.array([s[1] for s in want]), rtol=RTOL)
    np.testing.assert_allclose(got[2], np.stack([s[2] for s in want]), rtol=RTOL)


@pytest.mark.parametrize("storage,scale,hmargin", [("table", "auto", 0.0), ("factored", "group", 0.85)])
def test_export_picks_fewest_bits_and_rebuilds(storage, scale, hmargin, tmp_path):
    from yggdrasil_b200 import Yggdrasil
    from yggdrasil_b200.calibration import export
    from yggdrasil_b200.checkpoint import export_bytes
    npz, out = tmp_path / "ck.npz", tmp_path / "model.bin"
    C.synthetic_checkpoint(npz, seed=9)
    w = np.random.default_rng(4).integers(0, 27, (48, 33))
    rec = export(npz, out, w, hmargin=hmargin, storage=storage, state_scale=scale)
    assert json.loads((tmp_path / "model.bin.json").read_text())["quantize"] == rec["quantize"]
    assert rec["quantize"]["factored"] == (storage == "factored")
    best = min(rec["calib_bpc"], key=rec["calib_bpc"].get)
    assert best == f"{rec['state_scale']}_{rec['quantize']['hmargin']}"
    assert len(rec["calib_bpc"]) == (8 if scale == "auto" and not hmargin else 1)
    data = out.read_bytes()
    assert export_bytes(npz, rec) == data                      # the record rebuilds the file
    model, om = Yggdrasil.load(out, backend="b200"), O.OracleModel(data)
    x = w[:16, :12]
    st, ost = model.init_state(16), om.init_state(16)
    for t in range(x.shape[1]):
        lg, st = model.step(x[:, t], st)
        np.testing.assert_array_equal(lg.cpu().numpy(), om.step(x[:, t], ost))
    bits = model.score(w).sum() / (w.shape[0] * (w.shape[1] - 1))
    assert abs(bits - rec["calib_bpc"][best]) < 1e-9
