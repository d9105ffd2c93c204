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
    assert rec["transitions_match_reference_triton_backend"]


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
