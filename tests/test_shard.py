"""Stream sharding host logic on the CPU: world_size-2 gloo ranks, the final gather, and a failing rank surfacing as
an error on the others (failure made on the host: a rank that raises, or that never joins the gather)."""
import os
import socket
import traceback

import numpy as np
import pytest
import torch.multiprocessing as mp

from yggdrasil_b200.shard import ShardedScorer, shard_rows


def test_shard_rows_cover_and_balance():
    for n in (0, 1, 7, 8, 65536, 65537):
        for world in (1, 2, 3, 8):
            spans = [shard_rows(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_rows(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def fake_bits(rows):
    """stand-in for B200Yggdrasil.score: a deterministic function of each row"""
    rows = np.asarray(rows, np.float64)
    return rows.sum(-1) * 0.5 + rows[:, 0]


def _worker(rank, world, port, mode, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        tokens = np.random.default_rng(0).integers(0, 5, (13, 6))
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 failed before the gather")
        bits = ShardedScorer(fake_bits).score(tokens)
        q.put((rank, "ok", bits.tolist()))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-300:]}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, status, payload = q.get(timeout=120)
        out[r] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_two_ranks_gather_all_rows():
    out = _run("ok")
    tokens = np.random.default_rng(0).integers(0, 5, (13, 6))
    for r in (0, 1):
        assert out[r][0] == "ok", out[r][1]
        np.testing.assert_allclose(out[r][1], fake_bits(tokens))


def test_failed_rank_is_an_error_on_the_other():
    out = _run("fail")
    assert out[1][0] == "error" and "rank 1 failed" in out[1][1]
    assert out[0][0] == "error", "rank 0 must not hang or return a partial result"
