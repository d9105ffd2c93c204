"""The CUDA path against the oracle and the reference's golden digests, through the C-ABI (GPU).

The bar is bit-exact: routes (the leaf of every layer), the raw int32 accumulators before saturation (compared
unclamped: most shapes carry values far outside the int8 range), the int8 states and the f32 logits must equal the
oracle's (the C restatement pinned to cpu/ygg.cpp / cpu/export.py:int_forward by tests/test_oracle.py, accumulators
included) on every shape of the reference's kernel test and on every benchmark workload (c1-c4f, c4 and c4f with their
Zipf-calibrated thresholds), and the digests of the logits and of the accumulators must equal the reference's. Score
bits are float64 sums in another order than the oracle's: rtol 1e-10 (the north-star bar is 1e-4).
"""
import numpy as np
import pytest

from conftest import case_tokens, golden, sha, ygg_score, ygg_step_logp

from oracle import oracle as O

pytestmark = pytest.mark.gpu

CASES = golden("kernel_cases.json")
LONG = golden("long_cases.json")
WORKLOADS = golden("workloads.json")
EXTENDED = golden("extended_cases.json")      # the d_state 96 extension, pinned to the reference's int_forward
EXT_CASES = [r for r in EXTENDED if "shape" in r]
EXT_WORKLOADS = [r for r in EXTENDED if "workload" in r]
BITS_RTOL = 1e-10


def _ids(cases):
    return ["-".join(f"{k[0]}{int(v)}" for k, v in c["shape"].items()) for c in cases]


@pytest.fixture(scope="module")
def torch():
    import torch
    return torch


def load(path, **kw):
    from yggdrasil_b200 import Yggdrasil
    return Yggdrasil.load(path, backend="b200", **kw)


def run_windows(model, om, x, torch, with_acc=False):
    """Step the GPU model and the oracle over windows x (S, T) from zero; compare routes, raw accumulators, states
    and logits at every step. Returns the GPU logits (S, T, V) [and accumulators (S, T, L, n)]."""
    s, t = x.shape
    st = model.init_state(s)
    ost = om.init_state(s)
    out = np.empty((s, t, model.vocab), np.float32)
    accs = np.empty((s, t, model.layers, model.n), np.int32)
    for i in range(t):
        lg, nst, rt, acc = model.step_debug(x[:, i], st)
        olg, ort, oacc = om.step(x[:, i], ost, routes=True, acc=True)
        np.testing.assert_array_equal(rt.cpu().numpy(), ort, err_msg=f"routes at step {i}")
        np.testing.assert_array_equal(acc.cpu().numpy(), oacc, err_msg=f"raw accumulators at step {i}")
        np.testing.assert_array_equal(nst.cpu().numpy(), ost, err_msg=f"states at step {i}")
        np.testing.assert_array_equal(lg.cpu().numpy(), olg, err_msg=f"logits at step {i}")
        out[:, i] = lg.cpu().numpy()
        accs[:, i] = acc.cpu().numpy()
        st = nst
    return (out, accs) if with_acc else out


@pytest.mark.parametrize("rec", CASES + EXT_CASES, ids=_ids(CASES) + [f"ext-{i}" for i in _ids(EXT_CASES)])
def test_step_bit_exact(rec, case_model, torch):
    path = case_model(rec)
    model, om = load(path), O.OracleModel(path)
    x = case_tokens(rec)
    lg, acc = run_windows(model, om, x, torch, with_acc=True)
    assert sha(np.ascontiguousarray(lg).tobytes()) == rec["logits_sha256"]
    assert sha(acc.tobytes()) == rec["acc_sha256"], "accumulators differ from the reference int_forward's"
    model.status()


@pytest.mark.parametrize("rec", LONG, ids=_ids(LONG))
def test_long_sequences_bit_exact(rec, case_model, torch):
    """512 steps (deep state dynamics, long runs of saturation): the logits and the raw accumulators of every step
    against the reference's digests."""
    path = case_model(rec)
    model = load(path)
    x = case_tokens(rec)
    st = model.init_state(x.shape[0])
    out, accs = [], []
    for i in range(x.shape[1]):
        lg, st, _, acc = model.step_debug(x[:, i], st)
        out.append(lg.cpu().numpy())
        accs.append(acc.cpu().numpy())
    lg = np.stack(out, 1)
    acc = np.stack(accs, 1)
    assert sha(np.ascontiguousarray(lg).tobytes()) == rec["logits_sha256"]
    assert [int(acc.min()), int(acc.max())] == rec["acc_range"]
    assert sha(np.ascontiguousarray(acc).tobytes()) == rec["acc_sha256"]


@pytest.mark.parametrize("rec", CASES[::2] + EXT_CASES,
                         ids=_ids(CASES[::2]) + [f"ext-{i}" for i in _ids(EXT_CASES)])
def test_score_matches_reference_bits(rec, case_model, torch):
    model = load(case_model(rec))
    bits = model.score(case_tokens(rec))
    np.testing.assert_allclose(bits, rec["bits"], rtol=BITS_RTOL)


@pytest.mark.parametrize("rec", CASES[:4], ids=_ids(CASES[:4]))
def test_score_from_state_and_state_out(rec, case_model, torch):
    """score continues from a given state (yggdrasil/inference.py:179-188) and leaves the caller's state alone."""
    path = case_model(rec)
    model, om = load(path), O.OracleModel(path)
    x = case_tokens(rec)
    pre, rest = x[:, :16], x[:, 15:]
    st = model.init_state(x.shape[0])
    for i in range(15):
        _, st = model.step(pre[:, i], st)
    keep = st.clone()
    bits = model.score(rest, state=st)
    assert torch.equal(st, keep)
    ost = om.init_state(x.shape[0])
    for i in range(15):
        om.step(pre[:, i], ost)
    np.testing.assert_allclose(bits, om.score(rest, ost), rtol=BITS_RTOL)


@pytest.mark.parametrize("batch", [1, 2, 31, 33, 257, 1000])
def test_ragged_batches(batch, case_model, torch):
    rec = CASES[0]
    path = case_model(rec)
    model, om = load(path), O.OracleModel(path)
    rng = np.random.default_rng(batch)
    x = rng.integers(0, model.vocab, (batch, 5)).astype(np.int32)
    st, ost = model.init_state(batch), om.init_state(batch)
    for i in range(x.shape[1]):
        lg, st = model.step(x[:, i], st)
        np.testing.assert_array_equal(lg.cpu().numpy(), om.step(x[:, i], ost))
    np.testing.assert_array_equal(st.cpu().numpy(), ost)


def test_empty_batch(case_model, torch):
    model = load(case_model(CASES[0]))
    lg, st = model.step(np.zeros(0, np.int32), model.init_state(0))
    assert tuple(lg.shape) == (0, model.vocab) and tuple(st.shape) == (0, model.layers, model.n)
    assert model.score(np.zeros((0, 4), np.int32)).shape == (0,)


def test_in_place_state(case_model, torch):
    rec = CASES[1]
    path = case_model(rec)
    model, om = load(path), O.OracleModel(path)
    x = case_tokens(rec)
    st, ost = model.init_state(x.shape[0]), om.init_state(x.shape[0])
    logits = torch.empty(x.shape[0], model.vocab, dtype=torch.float32, device=model.device)
    for i in range(8):
        tok = torch.as_tensor(x[:, i], device=model.device)
        model.step_into(tok, st, st, logits)
        np.testing.assert_array_equal(logits.cpu().numpy(), om.step(x[:, i], ost))
    np.testing.assert_array_equal(st.cpu().numpy(), ost)


def test_cuda_graph_step(case_model, torch):
    rec = CASES[2]
    path = case_model(rec)
    plain, graph = load(path), load(path, cuda_graph=True)
    x = case_tokens(rec)
    s1, s2 = plain.init_state(x.shape[0]), graph.init_state(x.shape[0])
    for i in range(6):
        l1, s1 = plain.step(x[:, i], s1)
        l2, s2 = graph.step(x[:, i], s2)
        assert torch.equal(l1, l2) and torch.equal(s1, s2)


def test_host_token_out_of_range_raises(case_model, torch):
    model = load(case_model(CASES[3]))
    with pytest.raises(ValueError):
        model.step(np.array([model.vocab], np.int32), model.init_state(1))
    with pytest.raises(ValueError):
        model.score(np.array([[0, 1, -1]], np.int32))


def test_device_token_out_of_range_is_flagged(case_model, torch):
    """A bad token on the device skips its stream (NaN logits, state unchanged) and sets the status word; the other
    streams are exact."""
    rec = CASES[0]
    path = case_model(rec)
    model, om = load(path), O.OracleModel(path)
    x = np.array([3, model.vocab + 7, 5], np.int32)
    st = model.init_state(3)
    lg, nst = model.step(torch.as_tensor(x, device=model.device), st)
    with pytest.raises(ValueError):
        model.status()
    model.status()   # cleared
    ost = om.init_state(1)
    np.testing.assert_array_equal(lg[0].cpu().numpy(), om.step(x[:1], ost)[0])
    assert torch.isnan(lg[1]).all() and torch.equal(nst[1], st[1])


def test_conformance_adapters(case_model, torch):
    """The reference's backend hooks: step log-probabilities and the streamed score agree."""
    rec = CASES[5]
    model = load(case_model(rec))
    x = case_tokens(rec)[0, :20]
    logp = ygg_step_logp(model, x)
    manual = -logp[np.arange(len(x) - 1), x[1:]].sum() / np.log(2) / (len(x) - 1)
    np.testing.assert_allclose(ygg_score(model, x), manual, rtol=1e-9)


def test_generate_greedy_matches_oracle(case_model, torch):
    rec = CASES[0]
    path = case_model(rec)
    model, om = load(path), O.OracleModel(path)
    prompt = np.array([1, 2, 3], np.int32)
    out = model.generate(prompt, 5, temperature=0)
    st, toks = om.init_state(1), list(prompt)
    for t in prompt:
        lg = om.step(np.array([t], np.int32), st)
    for _ in range(5):
        nxt = int(lg[0].argmax())
        toks.append(nxt)
        lg = om.step(np.array([nxt], np.int32), st)
    np.testing.assert_array_equal(out, toks)
    sampled = model.generate(np.array([[1, 2], [3, 4]]), 4, temperature=0.8, top_k=5, seed=1)
    assert sampled.shape == (2, 6) and sampled.min() >= 0 and sampled.max() < model.vocab


@pytest.mark.parametrize("rec", WORKLOADS + EXT_WORKLOADS, ids=[w["workload"] for w in WORKLOADS + EXT_WORKLOADS])
def test_benchmark_workloads_bit_exact(rec, workload_model, oracle_of, torch):
    """Every benchmark model, c4 (the north-star 730M shape, table storage, Zipf-calibrated) and c4f (factored)
    included: routes, raw accumulators, states and logits at every step against the oracle, and the digests of the
    logits and accumulators and the score bits against the reference's int_forward."""
    from yggdrasil_b200 import synth
    w = synth.WORKLOADS[rec["workload"]]
    p = workload_model(rec["workload"])
    model, om = load(p), oracle_of(p)
    x = synth.workload_tokens(w, rec["streams"], rec["steps"], seed=rec["token_seed"])
    lg, acc = run_windows(model, om, x, torch, with_acc=True)
    assert sha(np.ascontiguousarray(lg).tobytes()) == rec["logits_sha256"]
    assert sha(acc.tobytes()) == rec["acc_sha256"]
    np.testing.assert_allclose(model.score(x), rec["bits"], rtol=BITS_RTOL)


@pytest.mark.parametrize("key", ["c3", "c3n96", "c4", "c4f"])
def test_large_batch_sampled_streams(key, workload_model, oracle_of, torch):
    """At the benchmark batch (65536 streams of the c3 shape at d 128 and d 96, and of the c4 and c4f shapes with
    their Zipf-calibrated routers), a checksum over all streams' states and logits is reproducible, and a sample of
    streams equals the oracle exactly after 3 steps."""
    from yggdrasil_b200 import synth
    w = synth.WORKLOADS[key]
    p = workload_model(key)
    model, om = load(p), oracle_of(p)
    B = 65536
    x = synth.workload_tokens(w, B, 3, seed=0)
    st = model.init_state(B)
    for i in range(3):
        lg, st = model.step(x[:, i], st)
    st2 = model.init_state(B)
    for i in range(3):
        lg2, st2 = model.step(x[:, i], st2)
    assert torch.equal(st, st2) and torch.equal(lg, lg2)
    idx = np.random.default_rng(5).choice(B, 256, replace=False)
    ost = om.init_state(len(idx))
    for i in range(3):
        olg = om.step(x[idx, i], ost)
    np.testing.assert_array_equal(lg.cpu().numpy()[idx], olg)
    np.testing.assert_array_equal(st.cpu().numpy()[idx], ost)


@pytest.mark.parametrize("rec", EXT_CASES[:3], ids=_ids(EXT_CASES[:3]))
def test_extension_state_layout(rec, case_model, torch):
    """A d_state 96 model keeps the caller's (B, L, 96) state: in-place steps, score from a state and the state it
    leaves equal the oracle's."""
    path = case_model(rec)
    model, om = load(path), O.OracleModel(path)
    assert model.n == 96
    x = case_tokens(rec)
    st, ost = model.init_state(x.shape[0]), om.init_state(x.shape[0])
    assert tuple(st.shape) == (x.shape[0], model.layers, 96)
    logits = torch.empty(x.shape[0], model.vocab, dtype=torch.float32, device=model.device)
    for i in range(10):
        model.step_into(torch.as_tensor(x[:, i], device=model.device), st, st, logits)
        np.testing.assert_array_equal(logits.cpu().numpy(), om.step(x[:, i], ost))
    np.testing.assert_array_equal(st.cpu().numpy(), ost)
    bits = model.score(x[:, 9:], state=st)
    np.testing.assert_allclose(bits, om.score(x[:, 9:], ost), rtol=BITS_RTOL)


# the launch configurations the library chooses between by batch, each forced for every batch
LAUNCH_CONFIGS = {
    "pipe": {"YGG_PIPE": "1000000"},                       # scoring as a layer wavefront, router and update groups
    "pipe-whole": {"YGG_PIPE": "1000000", "YGG_PIPE_SPLIT": "0"},   # the wavefront with one group per layer
    "coop": {"YGG_COOP": "1000000", "YGG_PIPE": "0"},      # 4 warps per stream (n = 128; others keep the policy)
    "warp-staged": {"YGG_LANES": "32", "YGG_DIRECT": "0"},  # a warp per stream, records staged in shared memory
    "warp-direct": {"YGG_LANES": "32", "YGG_DIRECT": "1"},  # a warp per stream, records read from global memory
    "half-staged": {"YGG_LANES": "16", "YGG_DIRECT": "0"},  # two streams per warp (shapes that allow it)
    "half-direct": {"YGG_LANES": "16", "YGG_DIRECT": "1"},
    # the layer-phased step (one launch per layer over all streams), a warp and half a warp per stream
    "phased": {"YGG_PHASED": "1", "YGG_LANES": "32", "YGG_DIRECT": "1"},
    "phased-half": {"YGG_PHASED": "1", "YGG_LANES": "16", "YGG_DIRECT": "1"},
}


@pytest.mark.parametrize("cfg", list(LAUNCH_CONFIGS))
@pytest.mark.parametrize("rec", CASES[:6] + CASES[11:14] + EXT_CASES[:2],
                         ids=_ids(CASES[:6] + CASES[11:14]) + [f"ext-{i}" for i in _ids(EXT_CASES[:2])])
def test_every_launch_configuration_bit_exact(cfg, rec, case_model, torch, monkeypatch):
    """Every launch configuration, forced for every batch (LAUNCH_CONFIGS): each gives the oracle's routes,
    accumulators, states and logits, with ragged batches (an odd count leaves a warp's second stream unseen) and the
    score path."""
    for k, v in LAUNCH_CONFIGS[cfg].items():
        monkeypatch.setenv(k, v)
    path = case_model(rec)
    model, om = load(path), O.OracleModel(path)
    x = case_tokens(rec)[:7, :12]
    run_windows(model, om, x, torch)
    np.testing.assert_allclose(model.score(x), om.score(x), rtol=BITS_RTOL)


@pytest.mark.parametrize("cfg", list(LAUNCH_CONFIGS))
@pytest.mark.parametrize("rec", WORKLOADS + EXT_WORKLOADS, ids=[w["workload"] for w in WORKLOADS + EXT_WORKLOADS])
def test_fast_instances_bit_exact(cfg, rec, workload_model, oracle_of, torch, monkeypatch):
    """The benchmark shapes run the fast instances (shape fixed at compile time; c4 and c4f are the n128 L4 R2=32
    V256 instances, the north-star target): every launch configuration against the oracle and the reference's
    digests, with 7 streams (ragged) in the score path."""
    from yggdrasil_b200 import synth
    for k, v in LAUNCH_CONFIGS[cfg].items():
        monkeypatch.setenv(k, v)
    w = synth.WORKLOADS[rec["workload"]]
    p = workload_model(rec["workload"])
    model, om = load(p), oracle_of(p)
    x = synth.workload_tokens(w, rec["streams"], rec["steps"], seed=rec["token_seed"])
    lg, acc = run_windows(model, om, x, torch, with_acc=True)
    assert sha(np.ascontiguousarray(lg).tobytes()) == rec["logits_sha256"]
    assert sha(acc.tobytes()) == rec["acc_sha256"]
    x7 = synth.workload_tokens(w, 7, 20, seed=3)
    np.testing.assert_allclose(model.score(x7), om.score(x7), rtol=BITS_RTOL)


N128 = [c for c in CASES if c["shape"]["d_state"] == 128]


@pytest.mark.parametrize("rec", N128, ids=_ids(N128))
def test_pipe_score_rows_short_sequences_and_state(rec, case_model, torch, monkeypatch):
    """The layer wavefront (one row per block; a router and an update group per layer for L <= 4, else one group per
    layer): more rows than blocks (a block takes a second row), sequences shorter than the pipeline's depth (T = 1, 2,
    3), and a carried state in and out. Its bits must equal the sequential latency kernel's and the one-group-per-layer
    wavefront's exactly (same operations, same order) and the oracle's within rtol."""
    path = case_model(rec)
    om = O.OracleModel(path)
    rng = np.random.default_rng(5)
    monkeypatch.setenv("YGG_PIPE", "1000000")
    pipe = load(path)
    monkeypatch.setenv("YGG_PIPE_SPLIT", "0")
    whole = load(path)
    monkeypatch.setenv("YGG_PIPE", "0")
    monkeypatch.setenv("YGG_COOP", "1000000")
    coop = load(path)
    rows = 150
    warm = rng.integers(0, pipe.vocab, (rows, 6)).astype(np.int32)
    st0 = pipe.init_state(rows)
    ost0 = om.init_state(rows)
    for i in range(warm.shape[1]):
        _, st0 = pipe.step(warm[:, i], st0)
        om.step(warm[:, i], ost0)
    np.testing.assert_array_equal(st0.cpu().numpy(), ost0)
    for t in (1, 2, 3, 9):
        x = rng.integers(0, pipe.vocab, (rows, t)).astype(np.int32)
        xd = torch.as_tensor(x).cuda()
        sp, sc = st0.clone(), st0.clone()
        bp = torch.empty(rows, dtype=torch.float64, device="cuda")
        bc = torch.empty_like(bp)
        pipe.score_into(xd, sp, bp)
        coop.score_into(xd, sc, bc)
        sw, bw = st0.clone(), torch.empty_like(bp)
        whole.score_into(xd, sw, bw)
        np.testing.assert_array_equal(bp.cpu().numpy(), bw.cpu().numpy(), err_msg=f"split vs whole bits, T={t}")
        np.testing.assert_array_equal(sp.cpu().numpy(), sw.cpu().numpy(), err_msg=f"split vs whole state, T={t}")
        ost = ost0.copy()
        ob = om.score(x, ost)
        np.testing.assert_array_equal(bp.cpu().numpy(), bc.cpu().numpy(), err_msg=f"pipe vs coop bits, T={t}")
        np.testing.assert_allclose(bp.cpu().numpy(), ob, rtol=BITS_RTOL)
        np.testing.assert_array_equal(sp.cpu().numpy(), ost, err_msg=f"state after T={t}")
        bz = torch.empty_like(bp)
        pipe.score_into(xd, None, bz)
        np.testing.assert_allclose(bz.cpu().numpy(), om.score(x), rtol=BITS_RTOL)
