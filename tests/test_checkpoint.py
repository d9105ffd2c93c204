"""Float checkpoint (.npz) + export record -> int8 YGG1 on the host (CPU), pinned to the reference's read / quantize /
write by golden digests (tests/golden/make_golden.py); and the loaded model against the oracle (GPU)."""
import json

import numpy as np
import pytest

from conftest import golden, sha

import checkpoints as C

CKPTS = golden("checkpoints.json")


def _make(tmp_path, rec):
    npz = tmp_path / f"ck{rec['seed']}.npz"
    C.synthetic_checkpoint(npz, seed=rec["seed"], old_keys=rec["old_keys"])
    q = rec["quantize"]
    record = C.synthetic_record(seed=rec["record_seed"], hmargin=q["hmargin"], group=q["group"],
                                factored=q["factored"])
    return npz, record


@pytest.mark.parametrize("rec", CKPTS, ids=[f"s{c['seed']}-old{int(c['old_keys'])}-r{c['record_seed']}" for c in CKPTS])
def test_export_equals_reference(rec, tmp_path):
    from yggdrasil_b200.checkpoint import export_bytes
    npz, record = _make(tmp_path, rec)
    data = export_bytes(npz, record)
    assert len(data) == rec["model_bytes"]
    assert sha(data) == rec["model_sha256"]


@pytest.mark.parametrize("seed", [0, 1])
def test_transitions_match_scipy_expm(seed, tmp_path):
    """transitions64 (torch's float64 matrix_exp) against scipy's float64 expm of the same skew blocks, clipped decays
    on the rows: the int8 export rounds 2^14 A, so the two must agree far below half a step (2^-15)."""
    from scipy.linalg import expm

    from yggdrasil_b200.checkpoint import read_checkpoint, transitions64
    npz = tmp_path / "ck.npz"
    C.synthetic_checkpoint(npz, seed=seed)
    layers, _ = read_checkpoint(npz)
    for p in layers:
        rot = np.asarray(p["rotation"], np.float64)
        got = transitions64(rot, p["decay"])
        skew = 0.5 * (rot - np.swapaxes(rot, -1, -2))
        d = np.clip(np.asarray(p["decay"], np.float64), -1, 1).reshape(skew.shape[:-1])
        want = d[..., None] * np.stack([expm(b) for b in skew.reshape(-1, *skew.shape[-2:])]).reshape(skew.shape)
        assert np.abs(got - want).max() < 1e-12
        assert np.array_equal(np.rint(got * 2.0 ** 14), np.rint(want * 2.0 ** 14))


def test_record_from_file(tmp_path):
    from yggdrasil_b200.checkpoint import export_bytes
    rec = CKPTS[0]
    npz, record = _make(tmp_path, rec)
    p = tmp_path / "model.bin.json"
    p.write_text(json.dumps(record))
    assert sha(export_bytes(npz, p)) == rec["model_sha256"]


def test_unsupported_checkpoints(tmp_path):
    from yggdrasil_b200.checkpoint import read_checkpoint
    npz = tmp_path / "bad.npz"
    C.synthetic_checkpoint(npz, seed=3)
    z = dict(np.load(npz))
    z["token_layer/mystery"] = np.zeros(3, np.float32)
    np.savez(npz, **z)
    with pytest.raises(NotImplementedError):
        read_checkpoint(npz)
    z = {k: v for k, v in dict(np.load(npz)).items() if k != "token_layer/mystery"}
    z["something_else"] = np.zeros(1, np.float32)
    np.savez(npz, **z)
    with pytest.raises(ValueError):
        read_checkpoint(npz)


@pytest.mark.gpu
@pytest.mark.parametrize("rec", CKPTS[:2], ids=["tensor", "group-factored"])
def test_npz_backend_matches_oracle(rec, tmp_path):
    from oracle import oracle as O
    from yggdrasil_b200 import Yggdrasil
    from yggdrasil_b200.checkpoint import export_bytes
    npz, record = _make(tmp_path, rec)
    model = Yggdrasil.load(npz, backend="b200", record=record)
    om = O.OracleModel(export_bytes(npz, record))
    x = np.random.default_rng(0).integers(0, model.vocab, (16, 24)).astype(np.int32)
    st, ost = model.init_state(16), om.init_state(16)
    for t in range(x.shape[1]):
        lg, st, routes, _ = model.step_debug(x[:, t], st)
        olg, ort = om.step(x[:, t], ost, routes=True)
        np.testing.assert_array_equal(routes.cpu().numpy(), ort)
        np.testing.assert_array_equal(lg.cpu().numpy(), olg)
    np.testing.assert_allclose(model.score(x), om.score(x), rtol=1e-10)


def test_npz_without_record_is_refused(tmp_path):
    from yggdrasil_b200 import Yggdrasil
    npz = tmp_path / "ck.npz"
    C.synthetic_checkpoint(npz, seed=0)
    with pytest.raises(NotImplementedError):
        Yggdrasil.load(npz, backend="b200")
