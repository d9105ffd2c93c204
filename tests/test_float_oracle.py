"""The float oracle (oracle/float_oracle.py, float64) against the reference's own fp32 GPU step (the Triton kernel of
yggdrasil/inference_triton.py, run by Triton's interpreter in tests/golden/make_golden.py) on seeded synthetic float
checkpoints (CPU).

Each step starts from the reference's state of the step before (as the reference's own Triton-vs-JAX test does,
cpu/tests/test_triton.py:49-61), so that a routing flip at a node score within rounding of 0 changes one stream step
only. Tolerances are the reference's: log-probabilities within 1e-4 for all but 1e-3 of the stream steps, the score
bits within rtol 1e-4 (cpu/tests/test_triton.py:29-30,67).
"""
import json

import numpy as np
import pytest

from conftest import GOLDEN

import checkpoints as C
from oracle.float_oracle import FloatOracle, log_softmax

FLOAT = json.loads((GOLDEN / "float_cases.json").read_text())
ATOL, FLIPS, BITS_RTOL = 1e-4, 1e-3, 1e-4


def float_case(rec, tmp_path):
    """(checkpoint path, fixture arrays) of a float case."""
    npz = tmp_path / f"f{rec['name']}.npz"
    kw = {} if rec["shape"] is None else {"shape": rec["shape"]}
    C.synthetic_checkpoint(npz, seed=rec["seed"], old_keys=rec["old_keys"], **kw)
    with np.load(GOLDEN / "float_cases.npz") as z:
        arrays = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(rec["name"] + "/")}
    return npz, arrays


@pytest.mark.parametrize("rec", FLOAT, ids=[r["name"] for r in FLOAT])
def test_float_oracle_matches_reference_triton_step(rec, tmp_path):
    from yggdrasil_b200.checkpoint import read_checkpoint
    npz, ref = float_case(rec, tmp_path)
    om = FloatOracle(*read_checkpoint(npz))
    x = ref["tokens"]
    st, off, total = om.init_state(x.shape[0]), 0, 0
    for t in range(x.shape[1]):
        lg, new, experts = om.step(x[:, t], st)
        np.testing.assert_array_equal(experts, ref["experts"][:, t])
        d = np.abs(log_softmax(lg) - log_softmax(ref["logits"][:, t])).max(-1)
        off, total = off + int((d > ATOL).sum()), total + len(d)
        np.testing.assert_allclose(new, ref["states"][:, t], rtol=1e-5, atol=1e-5 * np.abs(ref["states"]).max())
        st = ref["states"][:, t].astype(np.float64)
    assert off <= FLIPS * total
    np.testing.assert_allclose(om.score(x), ref["bits"], rtol=BITS_RTOL)


@pytest.mark.parametrize("rec", FLOAT, ids=[r["name"] for r in FLOAT])
def test_float_oracle_calibration_matches_reference(rec, tmp_path):
    """The calibration maxima of cpu/export.py:129-153 (|h| per group of 16, |V' rms(h_below)|, |P_r h| per row), from
    the float oracle's float64 steps, against the same maxima of the reference's fp32 Triton steps on the same
    windows: within 1e-5 relative (fp32 against float64)."""
    from yggdrasil_b200.checkpoint import read_checkpoint
    npz, ref = float_case(rec, tmp_path)
    stats = FloatOracle(*read_checkpoint(npz)).calibrate(ref["tokens"])
    np.testing.assert_allclose(np.stack([s[0] for s in stats]), ref["stats_groups"], rtol=1e-5)
    np.testing.assert_allclose(np.array([s[1] for s in stats]), ref["stats_layer_input"], rtol=1e-5)
    np.testing.assert_allclose(np.stack([s[2] for s in stats]), ref["stats_rows"], rtol=1e-5)
