"""The fp32 B200 float step (backend "b200f", csrc/ygg_float.cu) against the reference's own fp32 GPU step and the
float oracle (GPU).

The reference's float step is its Triton backend (yggdrasil/inference_triton.py), whose outputs on seeded synthetic
checkpoints are the fixture tests/golden/float_cases.npz (its kernel run by Triton's interpreter). As in the
reference's own Triton-vs-JAX test (cpu/tests/test_triton.py:40-67), each step starts from the reference's state of
the step before, so that a routing flip at a node score within rounding of 0 changes one stream step only, and the
tolerances are the reference's: log-probabilities within ATOL = 1e-4 for all but FLIPS = 1e-3 of the stream steps,
the score bits within rtol 1e-4. Experts must be equal (a flip would show as a log-probability beyond ATOL too).
"""
import numpy as np
import pytest
from test_float_oracle import ATOL, BITS_RTOL, FLIPS, FLOAT, float_case

import checkpoints as C
from oracle.float_oracle import FloatOracle, log_softmax

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch
    return torch


def load(npz, **kw):
    from yggdrasil_b200 import Yggdrasil
    return Yggdrasil.load(npz, backend="b200f", **kw)


def teacher_forced(model, x, states, logits_ref, experts_ref, torch):
    """Step the model from the reference states (S, T, L, n); returns (stream steps beyond ATOL, total, worst logp
    difference of the others, expert mismatches)."""
    s = x.shape[0]
    st = model.init_state(s)
    off = total = mism = 0
    worst = 0.0
    for t in range(x.shape[1]):
        lg, new, ex = model.step_experts(x[:, t], st)
        mism += int((ex.cpu().numpy() != experts_ref[:, t]).sum())
        d = np.abs(log_softmax(lg.cpu().numpy()) - log_softmax(logits_ref[:, t])).max(-1)
        off, total = off + int((d > ATOL).sum()), total + len(d)
        worst = max(worst, float(d[d <= ATOL].max(initial=0.0)))
        np.testing.assert_allclose(new.cpu().numpy(), states[:, t], rtol=1e-4,
                                   atol=1e-5 * np.abs(states).max())
        st = torch.as_tensor(np.ascontiguousarray(states[:, t], np.float32), device=model.device)
    return off, total, worst, mism


@pytest.mark.parametrize("rec", FLOAT, ids=[r["name"] for r in FLOAT])
def test_float_step_matches_reference_triton_step(rec, tmp_path, torch):
    npz, ref = float_case(rec, tmp_path)
    model = load(npz)
    off, total, worst, mism = teacher_forced(model, ref["tokens"], ref["states"], ref["logits"], ref["experts"], torch)
    assert mism == 0 and off <= FLIPS * total, (off, total, mism)
    np.testing.assert_allclose(model.score(ref["tokens"]), ref["bits"], rtol=BITS_RTOL)


@pytest.mark.parametrize("rec", FLOAT, ids=[r["name"] for r in FLOAT])
def test_float_step_matches_oracle_on_many_streams(rec, tmp_path, torch):
    """300 streams (a ragged count) x 20 steps against the float64 oracle, each step from the oracle's state; then
    the score from zero and from a carried state."""
    from yggdrasil_b200.checkpoint import read_checkpoint
    npz, _ = float_case(rec, tmp_path)
    model, om = load(npz), FloatOracle(*read_checkpoint(npz))
    rng = np.random.default_rng(7)
    x = rng.integers(0, model.vocab, (300, 20))
    st = om.init_state(300)
    off = total = mism = 0
    for t in range(x.shape[1]):
        lg, new, ex = model.step_experts(x[:, t], torch.as_tensor(st, dtype=torch.float32, device=model.device))
        olg, ost, oex = om.step(x[:, t], st)
        mism += int((ex.cpu().numpy() != oex).sum())
        d = np.abs(log_softmax(lg.cpu().numpy()) - log_softmax(olg)).max(-1)
        off, total = off + int((d > ATOL).sum()), total + len(d)
        st = ost
    assert off <= FLIPS * total and mism <= FLIPS * total * model.layers, (off, mism, total)
    np.testing.assert_allclose(model.score(x[:64]), om.score(x[:64]), rtol=BITS_RTOL)
    h = torch.as_tensor(st[:64], dtype=torch.float32, device=model.device)
    np.testing.assert_allclose(model.score(x[:64, :8], state=h), om.score(x[:64, :8], st[:64]), rtol=BITS_RTOL)


SMALL_BATCH_SHAPES = [
    dict(vocab=256, n=256, block=16, depth=3, readout=32, layer_input=128, input_rank=64, router_token=16, routed=2),
    dict(vocab=200, n=128, block=16, depth=9, readout=16, layer_input=32, input_rank=32, router_token=16, routed=2),
    dict(vocab=40, n=64, block=8, depth=7, readout=8, layer_input=16, input_rank=16, router_token=8, routed=3),
]


@pytest.mark.parametrize("shape", SMALL_BATCH_SHAPES, ids=["n256-R2128-D3", "n128-V200-D9", "n64-D7"])
def test_float_small_batch_branches_match_oracle(shape, torch):
    """The small-batch step (at most two streams per SM, four threads per coordinate) on random float models whose
    shapes take its other branches: V' too large to stage in shared memory (n 256, R2 128) with the layer input
    summed before the router, a single router round (depth 3), more classes than coordinates (the head after the last
    layer), a last round of one level (depth 9) and of three (depth 7). Six streams, 12 steps, each from the oracle's
    state, against the float64 oracle with the reference's tolerances."""
    from yggdrasil_b200 import synth
    from yggdrasil_b200.float_backend import B200FloatYggdrasil
    layers, ob = synth.random_float_layers(shape, seed=11)
    model, om = B200FloatYggdrasil(layers, ob), FloatOracle(layers, ob)
    x = np.random.default_rng(3).integers(0, model.vocab, (6, 12))
    st = om.init_state(6)
    off = total = mism = 0
    for t in range(x.shape[1]):
        lg, new, ex = model.step_experts(x[:, t], torch.as_tensor(st, dtype=torch.float32, device=model.device))
        olg, ost, oex = om.step(x[:, t], st)
        mism += int((ex.cpu().numpy() != oex).sum())
        d = np.abs(log_softmax(lg.cpu().numpy()) - log_softmax(olg)).max(-1)
        off, total = off + int((d > ATOL).sum()), total + len(d)
        np.testing.assert_allclose(new.cpu().numpy(), ost, rtol=1e-4, atol=1e-5 * np.abs(ost).max())
        st = ost
    assert off <= FLIPS * total and mism <= FLIPS * total * model.layers, (off, mism, total)
    model.status()


def test_float_cuda_graph_and_in_place(tmp_path, torch):
    """The CUDA-graph step equals the plain step exactly; an in-place step_into equals a step."""
    npz = tmp_path / "ck.npz"
    C.synthetic_checkpoint(npz, seed=4)
    plain, graph = load(npz), load(npz, cuda_graph=True)
    x = np.random.default_rng(1).integers(0, plain.vocab, (33, 6))
    s1, s2 = plain.init_state(33), graph.init_state(33)
    for t in range(6):
        l1, s1 = plain.step(x[:, t], s1)
        l2, s2 = graph.step(x[:, t], s2)
        assert torch.equal(l1, l2) and torch.equal(s1, s2)
    st = plain.init_state(33)
    lg = torch.empty(33, plain.classes, device=plain.device)
    ref_state = plain.init_state(33)
    for t in range(6):
        plain.step_into(torch.as_tensor(x[:, t], dtype=torch.int32, device=plain.device), st, st, lg)
        ref_lg, ref_state = plain.step(x[:, t], ref_state)
        assert torch.equal(lg, ref_lg) and torch.equal(st, ref_state)


def test_float_tokens_out_of_range(tmp_path, torch):
    npz = tmp_path / "ck.npz"
    C.synthetic_checkpoint(npz, seed=5)
    model = load(npz)
    with pytest.raises(ValueError):
        model.step(np.array([model.vocab], np.int32), model.init_state(1))
    with pytest.raises(ValueError):
        model.score(np.array([[0, 1, -1]]))
    st = model.init_state(3)
    lg, new = model.step(torch.as_tensor([2, model.vocab + 3, 4], dtype=torch.int32, device=model.device), st)
    assert torch.isnan(lg[1]).all() and torch.equal(new[1], st[1]) and not torch.isnan(lg[0]).any()
    with pytest.raises(ValueError):
        model.status()
    model.status()   # cleared


def test_float_generate_greedy_matches_oracle(tmp_path, torch):
    from yggdrasil_b200.checkpoint import read_checkpoint
    npz = tmp_path / "ck.npz"
    C.synthetic_checkpoint(npz, seed=6)
    model, om = load(npz), FloatOracle(*read_checkpoint(npz))
    prompt = np.array([[1, 2, 3], [4, 5, 6]])
    out = model.generate(prompt, 6, temperature=0)
    st, toks = om.init_state(2), [prompt[:, i] for i in range(3)]
    for t in range(3):
        lg, st, _ = om.step(prompt[:, t], st)
    for _ in range(6):
        nxt = lg.argmax(-1)
        toks.append(nxt)
        lg, st, _ = om.step(nxt, st)
    np.testing.assert_array_equal(out, np.stack(toks, 1))
    sampled = model.generate(np.array([1, 2]), 5, temperature=0.7, top_k=4, seed=3)
    assert sampled.shape == (7,) and sampled.min() >= 0 and sampled.max() < model.classes


def test_float_backend_refuses_unsupported(tmp_path, torch):
    from yggdrasil_b200.checkpoint import read_checkpoint
    from yggdrasil_b200.float_backend import B200FloatYggdrasil
    npz = tmp_path / "ck.npz"
    C.synthetic_checkpoint(npz, seed=0)
    layers, ob = read_checkpoint(npz)
    with pytest.raises(NotImplementedError):
        B200FloatYggdrasil(layers[:1], ob)          # no routed layer
