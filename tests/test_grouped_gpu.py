"""The leaf-grouped scoring path (tensor-core GEMMs for leaves shared by many streams) against the fused score kernel
and the oracle (GPU). Everything in the step is integer-exact or the reference's single-rounded f32 ops, and the
float64 NLL is summed by the same code, so the bits must be identical to the fused kernel's (np.array_equal), and
the final states too; against the oracle the bits agree to rtol 1e-10 (the oracle sums its f64 exps in another
order).
"""
import numpy as np
import pytest

from conftest import golden, shape_of

from oracle import oracle as O

pytestmark = pytest.mark.gpu

CASES = golden("kernel_cases.json")
EXT_CASES = [r for r in golden("extended_cases.json") if "shape" in r]   # d_state 96 (device layout padded to 128)
BITS_RTOL = 1e-10


def _ids(cases):
    return ["-".join(f"{k[0]}{int(v)}" for k, v in c["shape"].items()) for c in cases]


def load(path):
    from yggdrasil_b200 import Yggdrasil
    return Yggdrasil.load(path, backend="b200")


def run_both(model, x, min_group, torch, state=None):
    t = torch.as_tensor(x, device=model.device)
    st1 = state.clone() if state is not None else model.init_state(x.shape[0])
    st2 = st1.clone()
    b1 = torch.empty(x.shape[0], dtype=torch.float64, device=model.device)
    b2 = torch.empty_like(b1)
    model.score_into(t, st1, b1)
    model.score_grouped_into(t, st2, b2, min_group=min_group)
    torch.cuda.synchronize()
    return b1.cpu().numpy(), b2.cpu().numpy(), st1, st2


@pytest.fixture(scope="module")
def torch():
    import torch
    return torch


@pytest.mark.parametrize("min_group", [1, 3, 1 << 30])
@pytest.mark.parametrize("rec", CASES + EXT_CASES, ids=_ids(CASES) + [f"ext-{i}" for i in _ids(EXT_CASES)])
def test_grouped_equals_fused(rec, min_group, case_model, torch):
    """min_group 1: every leaf through the tensor cores; 3: mixed; 2^30: every stream on the per-stream path."""
    path = case_model(rec)
    model = load(path)
    v = rec["shape"]["vocab"]
    x = np.random.default_rng(11).integers(0, v, (384, 12)).astype(np.int32)
    b1, b2, s1, s2 = run_both(model, x, min_group, torch)
    np.testing.assert_array_equal(b2, b1)
    assert torch.equal(s1, s2)
    model.status()


@pytest.mark.parametrize("rec", CASES[::3], ids=_ids(CASES[::3]))
def test_grouped_matches_oracle(rec, case_model, torch):
    path = case_model(rec)
    model, om = load(path), O.OracleModel(path)
    v = rec["shape"]["vocab"]
    x = np.random.default_rng(5).integers(0, v, (64, 20)).astype(np.int32)
    bits = model.score(x, grouped=True, min_group=2)
    np.testing.assert_allclose(bits, om.score(x), rtol=BITS_RTOL)


@pytest.mark.parametrize("rec", [CASES[0], EXT_CASES[0]], ids=["n128", "ext-n96"])
def test_grouped_from_state(rec, case_model, torch):
    model = load(case_model(rec))
    x = np.random.default_rng(3).integers(0, rec["shape"]["vocab"], (200, 10)).astype(np.int32)
    st = model.init_state(200)
    for i in range(5):
        _, st = model.step(x[:, i], st)
    b1, b2, s1, s2 = run_both(model, x[:, 5:], 2, torch, state=st)
    np.testing.assert_array_equal(b2, b1)
    assert torch.equal(s1, s2)


@pytest.mark.parametrize("key", ["c3", "c3n96", "c4", "c4f"])
def test_grouped_benchmark_shape(key, workload_model, torch):
    """The benchmark shapes at 4096 streams: c3 (n128 b16 R16 R2=32, 4 layers, V = 5; and the d 96 extension, padded
    to n 128 on the device), where DNA tokens make the token layer's five leaves and the hot routed leaves heavy, and
    c4 / c4f (V = 256, table and factored storage), whose Zipf-calibrated routers concentrate the routed layers on a
    few hundred leaves."""
    from yggdrasil_b200 import synth
    w = synth.WORKLOADS[key]
    model = load(workload_model(key))
    x = synth.workload_tokens(w, 4096, 16, seed=2)
    for g in (1, 32):
        b1, b2, s1, s2 = run_both(model, x, g, torch)
        np.testing.assert_array_equal(b2, b1)
        assert torch.equal(s1, s2)


def test_grouped_bad_rows_score_nan(case_model, torch):
    rec = CASES[3]
    model = load(case_model(rec))
    v = rec["shape"]["vocab"]
    x = np.random.default_rng(1).integers(0, v, (40, 6)).astype(np.int32)
    x[7, 3] = v + 2
    t = torch.as_tensor(x, device=model.device)
    bits = torch.empty(40, dtype=torch.float64, device=model.device)
    model.score_grouped_into(t, None, bits, min_group=1)
    b = bits.cpu().numpy()
    assert np.isnan(b[7]) and not np.isnan(np.delete(b, 7)).any()
    with pytest.raises(ValueError):
        model.status()
    ref = model.score(np.delete(x, 7, axis=0))
    np.testing.assert_array_equal(np.delete(b, 7), ref)
