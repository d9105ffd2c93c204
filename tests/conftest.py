"""Shared fixtures and adapters for the tests.

Markers: gpu (needs a CUDA device and the built libygg_b200.so; the parity tests proper). Tests without the marker
run on the CPU: the oracle against the reference's golden digests, the file format, the host logic, and that the
C-ABI library loads and exports what include/ygg_b200.h declares.

The adapters follow the reference's backend-conformance hooks (tests/conftest.py:165-207 of the reference):
``ygg_step_logp`` works for any backend whose step returns (logits (1, V), state).
"""
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (sm_100) and the built libygg_b200.so")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        return False


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden(name):
    return json.loads((GOLDEN / name).read_text())


def sha(b) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


def shape_of(rec):
    from yggdrasil_b200.synth import ModelShape
    return ModelShape(**rec["shape"])


def case_tokens(rec):
    """The reference kernel test's tokens: default_rng(0).integers(0, V, (streams, steps)) (cpu/tests/test_kernel.py)."""
    v = rec["shape"]["vocab"]
    return np.random.default_rng(rec["token_seed"]).integers(0, v, (rec["streams"], rec["steps"])).astype(np.int32)


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("models")


@pytest.fixture(scope="session")
def case_model(model_dir):
    """path of the random model of a kernel-test case (written once per session)."""
    from yggdrasil_b200 import synth
    cache = {}

    def get(rec):
        key = json.dumps(rec["shape"], sort_keys=True)
        if key not in cache:
            p = model_dir / f"case{len(cache)}.bin"
            shape = shape_of(rec)
            synth.write_random_model(shape, p, seed=rec["seed"], extended=shape.extended)
            cache[key] = p
        return cache[key]
    return get


@pytest.fixture(scope="session")
def workload_model(model_dir):
    """path of a benchmark workload's model (synth.WORKLOADS key; the Zipf-calibrated ones with their fixture
    thresholds), written once per session: c4's table-storage file is 1.9 GB."""
    from yggdrasil_b200 import synth
    from yggdrasil_b200.ygg1 import write_model
    cache = {}

    def get(key):
        w = synth.WORKLOADS[key]
        name = w.model or key
        if name not in cache:
            p = model_dir / f"workload_{name}.bin"
            layers = synth.workload_layers(w, seed=7, thresholds=synth.zipf_thresholds_of(w, ROOT))
            write_model(layers, np.linspace(-1, 1, w.shape.vocab), p, extended=w.extended)
            cache[name] = p
        return cache[name]
    return get


@pytest.fixture(scope="session")
def oracle_of():
    """The C oracle of a model path, loaded once per session (a c4 oracle holds the 1.9 GB file)."""
    from oracle import oracle as O
    cache = {}

    def get(path):
        key = str(path)
        if key not in cache:
            cache[key] = O.OracleModel(path)
        return cache[key]
    return get


def ygg_step_logp(ygg, tokens):
    """Feed tokens (T,) one at a time through ygg.step (one stream, from ygg.init_state(1)) -> log-probabilities
    (T, classes) of the next token."""
    state, out = ygg.init_state(1), []
    for t in tokens:
        logits, state = ygg.step(np.array([t], np.int32), state)
        out.append(_numpy(logits)[0])
    z = np.asarray(out, np.float64)
    return z - (np.log(np.exp(z - z.max(-1, keepdims=True)).sum(-1, keepdims=True)) + z.max(-1, keepdims=True))


def ygg_score(ygg, tokens):
    """score on one stream tokens (n + 1,) -> bits per token of tokens[1:]."""
    tokens = np.asarray(tokens, np.int32)
    return float(_numpy(ygg.score(tokens[None])).sum() / (len(tokens) - 1))


def _numpy(a):
    return a.detach().cpu().numpy() if hasattr(a, "detach") else np.asarray(a)
