"""The oracle and the synthetic-model generator against the reference's golden digests (CPU only).

Pins: the model files this repository writes equal the reference's (sha256) on every shape of the reference's kernel
test, and the C oracle's logits equal the reference's int_forward / ygg logits bit for bit (sha256 of the f32 bytes).
"""
import os

import numpy as np
import pytest

from conftest import ROOT, case_tokens, golden, sha, shape_of

from oracle import oracle as O

CASES = golden("kernel_cases.json")
LONG = golden("long_cases.json")
WORKLOADS = golden("workloads.json")
EXTENDED = golden("extended_cases.json")
EXT_CASES = [r for r in EXTENDED if "shape" in r]
EXT_WORKLOADS = [r for r in EXTENDED if "workload" in r]


def _ids(cases):
    return ["-".join(f"{k[0]}{int(v)}" for k, v in c["shape"].items()) for c in cases]


@pytest.mark.parametrize("rec", CASES, ids=_ids(CASES))
def test_generator_bytes_match_reference(rec, case_model):
    data = case_model(rec).read_bytes()
    assert len(data) == rec["model_bytes"]
    assert sha(data) == rec["model_sha256"]


@pytest.mark.parametrize("rec", CASES + LONG, ids=_ids(CASES) + [f"long-{i}" for i in _ids(LONG)])
def test_oracle_logits_match_reference(rec, case_model):
    """Logits, and the int32 accumulators before saturation (the reference int_forward's `drive`, which cpu/ygg.cpp
    narrows with cvtsepi32_epi8): the oracle's equal the reference's bit for bit."""
    om = O.OracleModel(case_model(rec))
    x = case_tokens(rec)
    lg, acc = om.logits(x, acc=True)
    assert lg.dtype == np.float32 and lg.shape == (rec["streams"], rec["steps"], rec["shape"]["vocab"])
    if sha(np.ascontiguousarray(lg).tobytes()) != rec["logits_sha256"]:
        np.testing.assert_array_equal(lg[0, :4, :8], np.asarray(rec["logits_head"], np.float32))
        pytest.fail("oracle logits differ from the reference's")
    assert [int(acc.min()), int(acc.max())] == rec["acc_range"]
    assert sha(acc.tobytes()) == rec["acc_sha256"], "oracle accumulators differ from the reference's"


def test_accumulators_leave_the_int8_range():
    """The accumulator pins mean something only if they are not already int8: most shapes saturate."""
    wide = [r["acc_range"][0] < -128 or r["acc_range"][1] > 127 for r in CASES + LONG]
    assert sum(wide) >= 0.75 * len(wide) and any(wide[len(CASES):])


@pytest.mark.parametrize("rec", CASES[:6], ids=_ids(CASES[:6]))
def test_oracle_score_matches_reference_bits(rec, case_model):
    om = O.OracleModel(case_model(rec))
    bits = om.score(case_tokens(rec))
    np.testing.assert_allclose(bits, rec["bits"], rtol=1e-12)


@pytest.mark.parametrize("rec", CASES[:4], ids=_ids(CASES[:4]))
def test_oracle_step_equals_windows(rec, case_model):
    """step() over B streams, state carried, equals the zero-state windows of logits()."""
    om = O.OracleModel(case_model(rec))
    x = case_tokens(rec)
    ref = om.logits(x)
    st = om.init_state(x.shape[0])
    for t in range(x.shape[1]):
        np.testing.assert_array_equal(om.step(x[:, t], st), ref[:, t])


def test_oracle_rejects_bad_tokens(case_model):
    om = O.OracleModel(case_model(CASES[3]))
    with pytest.raises(ValueError):
        om.logits(np.full((1, 3), om.vocab, np.int32))
    with pytest.raises(ValueError):
        om.step(np.array([-1], np.int32), om.init_state(1))


@pytest.mark.skipif(not O.ref_available(), reason="reference binary not built (make -C oracle)")
@pytest.mark.parametrize("rec", CASES[::4], ids=_ids(CASES[::4]))
def test_reference_binary_matches_oracle(rec, case_model, tmp_path):
    x = case_tokens(rec)
    np.testing.assert_array_equal(O.ref_logits(case_model(rec), x, str(tmp_path)),
                                  O.OracleModel(case_model(rec)).logits(x))


@pytest.mark.parametrize("rec", WORKLOADS, ids=[w["workload"] for w in WORKLOADS])
def test_workload_models_match_reference_writer(rec, workload_model):
    """The benchmark models (c4 and c4f with their Zipf-calibrated thresholds from tests/golden/zipf_thresholds.npz):
    this repository's writer equals the reference's writer on the same layers, and the oracle's logits and
    accumulators equal the reference's int_forward on them."""
    from yggdrasil_b200 import synth
    w = synth.WORKLOADS[rec["workload"]]
    p = workload_model(rec["workload"])
    assert p.stat().st_size == rec["model_bytes"]
    assert sha(p.read_bytes()) == rec["model_sha256"]
    x = synth.workload_tokens(w, rec["streams"], rec["steps"], seed=rec["token_seed"])
    lg, acc = O.OracleModel(p).logits(x, acc=True)
    assert sha(np.ascontiguousarray(lg).tobytes()) == rec["logits_sha256"]
    assert sha(acc.tobytes()) == rec["acc_sha256"]


def test_zipf_fixture_shapes():
    """The calibrated thresholds: one row per routed layer, one per tree node, finite, not all equal."""
    from yggdrasil_b200 import synth
    for key in ("c4", "c4f"):
        w = synth.WORKLOADS[key]
        thr = synth.zipf_thresholds_of(w, ROOT)
        assert thr.shape == (w.shape.n_layers - 1, 2 ** w.shape.router_depth - 1) and thr.dtype == np.float32
        assert np.isfinite(thr).all() and len(np.unique(thr)) > 1000
    assert synth.zipf_thresholds_of(synth.WORKLOADS["c5"], ROOT).shape == synth.zipf_thresholds_of(
        synth.WORKLOADS["c4"], ROOT).shape


@pytest.mark.parametrize("rec", EXT_CASES, ids=_ids(EXT_CASES))
def test_extension_oracle_matches_reference_int_forward(rec, case_model):
    """The d_state 96 extension, which the reference's writer and ygg refuse: the oracle over this repository's file
    equals the reference's int_forward on the same random model, bit for bit."""
    p = case_model(rec)
    assert sha(p.read_bytes()) == rec["model_sha256"] and p.stat().st_size == rec["model_bytes"]
    lg, acc = O.OracleModel(p).logits(case_tokens(rec), acc=True)
    if sha(np.ascontiguousarray(lg).tobytes()) != rec["logits_sha256"]:
        np.testing.assert_array_equal(lg[0, :4, :8], np.asarray(rec["logits_head"], np.float32))
        pytest.fail("oracle logits differ from the reference's int_forward")
    assert sha(acc.tobytes()) == rec["acc_sha256"]
    np.testing.assert_allclose(O.OracleModel(p).score(case_tokens(rec)), rec["bits"], rtol=1e-12)


@pytest.mark.parametrize("rec", EXT_WORKLOADS, ids=[w["workload"] for w in EXT_WORKLOADS])
def test_extension_workload_matches_reference_int_forward(rec, tmp_path):
    from yggdrasil_b200 import synth
    from yggdrasil_b200.ygg1 import write_model
    w = synth.WORKLOADS[rec["workload"]]
    p = tmp_path / "w.bin"
    write_model(synth.workload_layers(w, seed=7), np.linspace(-1, 1, w.shape.vocab), p, extended=w.extended)
    assert sha(p.read_bytes()) == rec["model_sha256"]
    x = synth.workload_tokens(w, rec["streams"], rec["steps"], seed=rec["token_seed"])
    lg, acc = O.OracleModel(p).logits(x, acc=True)
    assert sha(np.ascontiguousarray(lg).tobytes()) == rec["logits_sha256"]
    assert sha(acc.tobytes()) == rec["acc_sha256"]
