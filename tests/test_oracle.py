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
    om = O.OracleModel(case_model(rec))
    x = case_tokens(rec)
    lg = om.logits(x)
    assert lg.dtype == np.float32 and lg.shape == (rec["streams"], rec["steps"], rec["shape"]["vocab"])
    if sha(np.ascontiguousarray(lg).tobytes()) != rec["logits_sha256"]:
        np.testing.assert_array_equal(lg[0, :4, :8], np.asarray(rec["logits_head"], np.float32))
        pytest.fail("oracle logits differ from the reference's")


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
def test_workload_models_match_reference_writer(rec, tmp_path):
    """The benchmark models: this repository's writer equals the reference's writer on the same layers, and the
    oracle's logits equal the reference's int_forward on them."""
    from yggdrasil_b200 import synth
    w = synth.WORKLOADS[rec["workload"]]
    p = tmp_path / "w.bin"
    layers = synth.workload_layers(w, seed=7)
    from yggdrasil_b200.ygg1 import write_model
    write_model(layers, np.linspace(-1, 1, w.shape.vocab), p)
    assert sha(p.read_bytes()) == rec["model_sha256"]
    x = synth.workload_tokens(w, rec["streams"], rec["steps"], seed=rec["token_seed"])
    lg = O.OracleModel(p).logits(x)
    assert sha(np.ascontiguousarray(lg).tobytes()) == rec["logits_sha256"]


@pytest.mark.parametrize("rec", EXT_CASES, ids=_ids(EXT_CASES))
def test_extension_oracle_matches_reference_int_forward(rec, case_model):
    """The d_state 96 extension, which the reference's writer and ygg refuse: the oracle over this repository's file
    equals the reference's int_forward on the same random model, bit for bit."""
    p = case_model(rec)
    assert sha(p.read_bytes()) == rec["model_sha256"] and p.stat().st_size == rec["model_bytes"]
    lg = O.OracleModel(p).logits(case_tokens(rec))
    if sha(np.ascontiguousarray(lg).tobytes()) != rec["logits_sha256"]:
        np.testing.assert_array_equal(lg[0, :4, :8], np.asarray(rec["logits_head"], np.float32))
        pytest.fail("oracle logits differ from the reference's int_forward")
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
    assert sha(np.ascontiguousarray(O.OracleModel(p).logits(x)).tobytes()) == rec["logits_sha256"]
