"""Regenerate tests/golden/*.json from the reference implementation (run in a container that has the reference tree).

    python tests/golden/make_golden.py [--ref /path/to/yggdrasil] [--only cases,zipf,workloads,ext,checkpoints]

The fixtures pin this repository's generator and oracle to the reference:
  kernel_cases.json  for every shape of the reference's kernel test (cpu/tests/test_kernel.py:22-33): the sha256 of
                     the model file the reference writes (cpu/export.py random_model + write, seed 7), and the sha256
                     of the reference's logits (cpu/export.py:int_forward, equal to cpu/ygg.cpp's `logits` command) on
                     the test's tokens (default_rng(0), 8 streams x 64 steps), the per-row bits derived from them in
                     float64, and a few logits in clear for reading a failure;
  long_cases.json    two shapes run for 512 steps (deep state dynamics, saturation);
  workloads.json     the benchmark shapes (yggdrasil_b200.synth WORKLOADS c1-c4f) written by the reference's writer,
                     with int_forward logits on a few streams;
  zipf_thresholds.npz  the router thresholds of the Zipf(1.1)-calibrated models (c4, c4f; c5 scores the c4 model):
                     layer by layer, the C oracle (itself pinned to the reference here) runs 16 384 streams of uniform
                     bytes for 64 steps, and each node's threshold is set at the quantile of the sampled scores that
                     sends the Zipf share of its subtree to the right (synth.zipf_thresholds). The calibrated models
                     are then written by the reference's writer and run by its int_forward like the other workloads.
  extended_cases.json  shapes of this repository's d_state 96 format extension, which the reference's writer and ygg
                     refuse: the reference's random_model (seed 7) and int_forward logits on the kernel test's tokens,
                     and the c3n96 benchmark shape's int_forward logits on a few streams. The model digests here are
                     this repository's writer's (a regression check, not a pin); the logits are the pin.
  checkpoints.json   digests of the files the reference's quantize + write make from seeded synthetic checkpoints.
  float_cases.json/.npz  the reference's own fp32 GPU step (yggdrasil/inference_triton.py: its Triton kernel _ygg_step
                     and its torch.addmm head, run on the CPU by Triton's interpreter, TRITON_INTERPRET=1) on seeded
                     synthetic float checkpoints of three shapes: per step the logits, the experts and the new state,
                     from a zero state, and the score bits of the windows (TritonYggdrasil.score); and the calibration
                     maxima of cpu/export.py:129-153 (LayerStats: |h| per group of 16, |V' rms(h_below)|, |P_r h| per
                     row) over those steps; the pin of the float oracle (oracle/float_oracle.py), of the B200 float step
                     (backend "b200f") and of its calibration (yggdrasil_b200/calibration.py).
Every record of the first four also carries acc_sha256: the digest of the int32 accumulators before saturation,
(S, T, L, n), taken from int_forward's own `drive` array (cpu/export.py:300-310; the value cpu/ygg.cpp:388 narrows with
cvtsepi32_epi8) by watching its saturating np.clip(drive, -128, 127) calls.
The reference sources are read in place and never copied; only digests and a few numbers land here.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def bits_from_logits(lg: np.ndarray, x: np.ndarray) -> np.ndarray:
    """bits of x[:, 1:] given the logits after x[:, t], per row, float64 (the score of yggdrasil/inference.py)."""
    z = lg[:, :-1].astype(np.float64)
    mx = z.max(-1, keepdims=True)
    lse = np.log(np.exp(z - mx).sum(-1)) + mx[..., 0]
    tgt = np.take_along_axis(z, x[:, 1:, None].astype(np.int64), -1)[..., 0]
    return (lse - tgt).sum(-1) / np.log(2.0)


class AccCapture:
    """Records the array of every np.clip(a, -128, 127) call while active: in the reference's int_forward that is
    the saturation of each layer's accumulator `drive` into the new int8 state, once per (step, layer), in order."""

    def __enter__(self):
        self.arrays, self._clip = [], np.clip

        def clip(a, lo=None, hi=None, *args, **kw):
            if isinstance(lo, int) and isinstance(hi, int) and (lo, hi) == (-128, 127):
                self.arrays.append(np.array(a, copy=True))
            return self._clip(a, lo, hi, *args, **kw)
        np.clip = clip
        return self

    def __exit__(self, *exc):
        np.clip = self._clip

    def acc(self, S, T, L):
        """The accumulators as int32 (S, T, L, n); checks that no value left the int32 range of cpu/ygg.cpp."""
        a = np.stack(self.arrays).reshape(T, L, S, -1)
        assert np.abs(a).max() < 2 ** 31
        return np.ascontiguousarray(a.transpose(2, 0, 1, 3).astype(np.int32))


def forward_with_acc(E, layers, ob, x):
    """int_forward's logits and its accumulators before saturation."""
    with AccCapture() as cap:
        lg = E.int_forward(layers, ob, x)
    return lg, cap.acc(x.shape[0], x.shape[1], len(layers))


def oracle_layer_states(path, w, streams, snapshots, layer, procs=8):
    """States of `layer` (int8, (streams * len(snapshots), n)) after each step in snapshots, running the C oracle on
    `streams` streams of the workload's tokens (seed 77) from zero, split over processes."""
    from multiprocessing import get_context

    from yggdrasil_b200 import synth
    x = synth.workload_tokens(w, streams, max(snapshots), seed=77)
    chunks = np.array_split(np.arange(streams), procs)
    with get_context("spawn").Pool(procs) as pool:
        parts = pool.starmap(_oracle_chunk, [(str(path), x[c], tuple(snapshots), layer) for c in chunks])
    return np.concatenate([np.concatenate(p) for p in zip(*parts)])


def _oracle_chunk(path, x, snapshots, layer):
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    om = O.OracleModel(path)
    st = om.init_state(x.shape[0])
    out = []
    for t in range(max(snapshots)):
        om.step(x[:, t], st)
        if t + 1 in snapshots:
            out.append(st[:, layer].copy())
    return out


def calibrate_zipf(key, tmp, streams=16384, snapshots=(48, 56, 64), s=1.1, seed=7):
    """Per-node router thresholds (L - 1, 2^D - 1) of workload `key` for Zipf(s) leaf usage over a seeded leaf order
    (synth.zipf_leaf_probs, seed + 100 + l), layer by layer on the states the layers below produce."""
    from yggdrasil_b200 import synth
    from yggdrasil_b200.ygg1 import write_model
    w = synth.WORKLOADS[key]
    layers = synth.workload_layers(w, seed=seed)
    ob = np.linspace(-1, 1, w.shape.vocab)
    E = 2 ** w.shape.router_depth
    thr = np.zeros((len(layers) - 1, E - 1), np.float32)
    path = os.path.join(tmp, f"{key}_cal.bin")
    for l in range(1, len(layers)):
        write_model(layers, ob, path)
        qb = oracle_layer_states(path, w, streams, snapshots, l - 1)
        q = layers[l]
        rho = synth.rho_f32(qb, q.rms_eps, q.state_r2)
        thr[l - 1] = synth.zipf_thresholds(q.router_weight, qb, rho, synth.zipf_leaf_probs(E, s, seed + 100 + l))
        synth.apply_thresholds(layers, thr, only=l)
        print(f"calibrated {key} layer {l}", flush=True)
    os.remove(path)
    return thr


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("YGG_REFERENCE", "/root/reference"))
    ap.add_argument("--only", default="cases,workloads,zipf,ext,checkpoints",
                    help="comma-separated parts to regenerate (zipf recalibrates c4/c4f; workloads reads the .npz; "
                         "float runs the reference's Triton step under the interpreter)")
    a = ap.parse_args()
    parts = set(a.only.split(","))
    if "float" in parts:
        os.environ["TRITON_INTERPRET"] = "1"      # before anything imports triton: the kernel runs on the CPU
    ref = Path(a.ref)
    sys.path.insert(0, str(ref / "cpu"))
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ROOT))
    import export as E  # the reference's cpu/export.py
    from yggdrasil_b200 import synth
    ygg = ROOT / "oracle" / "_ref" / "ygg"
    sys.path.insert(0, str(ref / "cpu" / "tests"))
    from test_kernel import CASES, STEPS, STREAMS

    fields = [f for f in ("d_state", "block_size", "router_depth", "vocab", "n_layers", "readout_rank",
                          "layer_input_rank", "input_rank", "group")]

    def run_case(cfg, streams, steps, tmp):
        layers = E.random_model(cfg, seed=7)
        ob = np.linspace(-1, 1, cfg.vocab)
        path = os.path.join(tmp, "m.bin")
        E.write(layers, ob, path)
        x = np.random.default_rng(0).integers(0, cfg.vocab, (streams, steps)).astype(np.int32)
        lg, acc = forward_with_acc(E, layers, ob, x)
        rec = dict(shape={k: getattr(cfg, k) for k in fields}, seed=7, streams=streams, steps=steps, token_seed=0,
                   model_sha256=sha(Path(path).read_bytes()), model_bytes=os.path.getsize(path),
                   logits_sha256=sha(np.ascontiguousarray(lg, np.float32).tobytes()), acc_sha256=sha(acc.tobytes()),
                   acc_range=[int(acc.min()), int(acc.max())],
                   bits=[float(v) for v in bits_from_logits(lg, x)],
                   logits_head=np.asarray(lg[0, :4, :8], np.float64).tolist())
        if ygg.exists():   # the reference binary agrees with int_forward (the reference test's own assertion)
            xf, of = os.path.join(tmp, "x.i32"), os.path.join(tmp, "o.f32")
            x.tofile(xf)
            subprocess.run([str(ygg), "logits", path, xf, str(streams), str(steps), of], check=True,
                           stdout=subprocess.DEVNULL)
            rec["ygg_equal"] = bool(np.array_equal(np.fromfile(of, np.float32).reshape(lg.shape), lg))
        return rec

    with tempfile.TemporaryDirectory(dir=os.environ.get("YGG_GOLDEN_TMP")) as tmp:
        if "cases" in parts:
            cases = [run_case(c, STREAMS, STEPS, tmp) for c in CASES]
            (HERE / "kernel_cases.json").write_text(json.dumps(cases, indent=1) + "\n")
            longs = [run_case(CASES[i], 4, 512, tmp) for i in (1, 12)]
            (HERE / "long_cases.json").write_text(json.dumps(longs, indent=1) + "\n")
        if "zipf" in parts:
            thr = {key: calibrate_zipf(key, tmp) for key in ("c4", "c4f")}
            np.savez(HERE / "zipf_thresholds.npz", **thr)
        if "workloads" in parts:
            works = []
            for key in ("c1", "c2", "c3", "c4", "c4f"):
                w = synth.WORKLOADS[key]
                layers = synth.workload_layers(w, seed=7, thresholds=synth.zipf_thresholds_of(w, ROOT))
                ob = np.linspace(-1, 1, w.shape.vocab)
                path = os.path.join(tmp, "w.bin")
                E.write(layers, ob, path)            # the reference's writer on this repository's layers
                x = synth.workload_tokens(w, 4, 32, seed=0)
                lg, acc = forward_with_acc(E, layers, ob, x)
                works.append(dict(workload=key, model_sha256=sha(Path(path).read_bytes()),
                                  model_bytes=os.path.getsize(path), streams=4, steps=32, token_seed=0,
                                  logits_sha256=sha(np.ascontiguousarray(lg, np.float32).tobytes()),
                                  acc_sha256=sha(acc.tobytes()), acc_range=[int(acc.min()), int(acc.max())],
                                  bits=[float(v) for v in bits_from_logits(lg, x)]))
                os.remove(path)
                del layers
            (HERE / "workloads.json").write_text(json.dumps(works, indent=1) + "\n")
        if "ext" in parts:
            make_extended(E, synth, fields, tmp, STREAMS, STEPS)
        if "checkpoints" in parts:
            make_checkpoints(E, tmp)
        if "float" in parts:
            make_float(tmp)
    print("wrote", [p.name for p in HERE.glob("*.json")])


# shapes of the float cases: the synthetic checkpoint's (n 64, b 16), a DNA-like one (V 5, n 128, b 8, 3 routed
# layers, old keys) and one of the enwik8 large family (V 256, n 256, b 16, R 32, R2 64, k 64) at depth 6; the larger
# two draw smaller readouts and unembeddings so that their logits stay in the range of a trained model's (|logit| of
# order 10), where the reference's fp32 tolerance on log-probabilities (1e-4) is meant to hold
FLOAT_CASES = [
    dict(name="n64", seed=0, old_keys=False, streams=8, steps=12, shape=None),
    dict(name="n128-b8", seed=1, old_keys=True, streams=6, steps=8,
         shape=dict(vocab=5, n=128, block=8, depth=5, readout=16, layer_input=32, input_rank=32, router_token=16,
                    routed=3, readout_std=0.07, unembed_std=0.15)),
    dict(name="n256", seed=2, old_keys=False, streams=4, steps=6,
         shape=dict(vocab=256, n=256, block=16, depth=6, readout=32, layer_input=64, input_rank=64, router_token=16,
                    routed=2, readout_std=0.04, unembed_std=0.1)),
]


def make_float(tmp):
    """The reference's Triton float step on the CPU (see the module docstring)."""
    import torch
    sys.path.insert(0, str(HERE.parent))
    import checkpoints as C
    from yggdrasil import inference as I
    from yggdrasil import inference_triton as IT
    arrays, recs = {}, []
    for case in FLOAT_CASES:
        npz = os.path.join(tmp, f"f{case['name']}.npz")
        kw = {} if case["shape"] is None else {"shape": case["shape"]}
        C.synthetic_checkpoint(npz, seed=case["seed"], old_keys=case["old_keys"], **kw)
        layers, ob = I.read(npz)
        m = IT.TritonYggdrasil(layers, ob, device="cpu")
        S, T = case["streams"], case["steps"]
        x = np.random.default_rng(case["seed"]).integers(0, m.vocab, (S, T))
        h = m.init_state(S)
        logits, experts, states = [], [], []
        L, n = m.layers, m.n
        groups, rows, vmax = np.zeros((L, n // 16)), np.zeros((L, m.ro)), np.zeros(L)
        for t in range(T):
            xt = torch.as_tensor(np.ascontiguousarray(x[:, t]))   # the kernel reads the tokens flat
            h_out, z = torch.empty_like(h), torch.empty(S, m.layers, m.ro)
            ex = torch.empty(S, m.layers, dtype=torch.int32)
            m._launch(xt, h, h_out, z, ex, 1, 3)           # the reference's _step, less its GPU-timed tuning
            logits.append(torch.addmm(m.output_bias, z.view(S, -1), m.unembed).numpy())
            experts.append(ex.numpy())
            states.append(h_out.numpy())
            # the calibration maxima of cpu/export.py:129-153 (LayerStats) over this step's states and readouts
            hs, zs = h_out.numpy().astype(np.float64), z.numpy().astype(np.float64)
            groups = np.maximum(groups, np.abs(hs).reshape(S, L, n // 16, 16).max((0, 3)))
            rows = np.maximum(rows, np.abs(zs).max(0))
            for l in range(1, L):
                if "layer_input_down" in layers[l]:
                    below = hs[:, l - 1] / np.sqrt((hs[:, l - 1] ** 2).mean(-1, keepdims=True) + 1e-6)
                    v = below @ np.asarray(layers[l]["layer_input_down"], np.float64).T
                    vmax[l] = max(vmax[l], np.abs(v).max())
            h = h_out
        m._config[S] = (1, 3)                               # score() steps through _step without tuning
        bits = m.score(x)
        p = case["name"]
        arrays.update({f"{p}/tokens": x.astype(np.int32), f"{p}/logits": np.stack(logits, 1).astype(np.float32),
                       f"{p}/experts": np.stack(experts, 1).astype(np.int16),
                       f"{p}/states": np.stack(states, 1).astype(np.float32), f"{p}/bits": np.asarray(bits),
                       f"{p}/stats_groups": groups, f"{p}/stats_rows": rows, f"{p}/stats_layer_input": vmax})
        recs.append({k: v for k, v in case.items()} | {"classes": int(m.classes), "layers": int(m.layers)})
        print(f"float case {p}: done", flush=True)
    np.savez_compressed(HERE / "float_cases.npz", **arrays)
    (HERE / "float_cases.json").write_text(json.dumps(recs, indent=1) + "\n")


def make_extended(E, synth, fields, tmp, STREAMS, STEPS):
    """The d_state 96 extension: int_forward works at any shape; the file is this repository's writer's."""
    from yggdrasil_b200.synth import ModelShape, write_random_model
    from yggdrasil_b200.ygg1 import write_model
    ext_cfgs = [E.KernelConfig(96, 16, 8, 256, 2, 12, 24), E.KernelConfig(96, 8, 6, 5, 3, 12, 24, group=True),
                E.KernelConfig(96, 16, 7, 27, 3, 12, 24, input_rank=24, group=True),
                E.KernelConfig(96, 16, 6, 256, 2, 16, 32), E.KernelConfig(96, 8, 5, 5, 2, 8, 0)]
    ext = []
    for cfg in ext_cfgs:
        layers = E.random_model(cfg, seed=7)
        ob = np.linspace(-1, 1, cfg.vocab)
        path = os.path.join(tmp, "x.bin")
        shape = ModelShape(**{k: getattr(cfg, k) for k in fields})
        write_random_model(shape, path, seed=7, extended=True)
        x = np.random.default_rng(0).integers(0, cfg.vocab, (STREAMS, STEPS)).astype(np.int32)
        lg, acc = forward_with_acc(E, layers, ob, x)
        ext.append(dict(shape={k: getattr(cfg, k) for k in fields}, seed=7, streams=STREAMS, steps=STEPS,
                        token_seed=0, extended=True, model_sha256=sha(Path(path).read_bytes()),
                        model_bytes=os.path.getsize(path),
                        logits_sha256=sha(np.ascontiguousarray(lg, np.float32).tobytes()),
                        acc_sha256=sha(acc.tobytes()), acc_range=[int(acc.min()), int(acc.max())],
                        bits=[float(v) for v in bits_from_logits(lg, x)],
                        logits_head=np.asarray(lg[0, :4, :8], np.float64).tolist()))
    w = synth.WORKLOADS["c3n96"]
    layers = synth.workload_layers(w, seed=7)
    ob = np.linspace(-1, 1, w.shape.vocab)
    path = os.path.join(tmp, "w.bin")
    write_model(layers, ob, path, extended=True)
    x = synth.workload_tokens(w, 4, 32, seed=0)
    lg, acc = forward_with_acc(E, layers, ob, x)
    ext.append(dict(workload="c3n96", extended=True, model_sha256=sha(Path(path).read_bytes()),
                    model_bytes=os.path.getsize(path), streams=4, steps=32, token_seed=0,
                    logits_sha256=sha(np.ascontiguousarray(lg, np.float32).tobytes()),
                    acc_sha256=sha(acc.tobytes()), acc_range=[int(acc.min()), int(acc.max())],
                    bits=[float(v) for v in bits_from_logits(lg, x)]))
    (HERE / "extended_cases.json").write_text(json.dumps(ext, indent=1) + "\n")


def make_checkpoints(E, tmp):
    """Checkpoints: the reference's read (yggdrasil/inference.py:129-139), FloatLayer, quantize and write
    (cpu/export.py:68-96,216-265,461-468) on seeded synthetic checkpoints and export records. The float64
    transitions come from this repository's transitions64 (the reference's exporter uses JAX, absent here);
    tests/test_checkpoint.py checks them against scipy's float64 expm at test time."""
    sys.path.insert(0, str(HERE.parent))
    import checkpoints as C
    from yggdrasil import inference as I
    from yggdrasil_b200.checkpoint import transitions64
    ckpts = []
    for seed, old in ((0, False), (1, True)):
        npz = os.path.join(tmp, f"ck{seed}.npz")
        C.synthetic_checkpoint(npz, seed=seed, old_keys=old)
        raw, ob = I.read(npz)
        raw = [{k: v.astype(np.float64) for k, v in p.items()} for p in raw]
        depth = I.router_depth(raw[1])
        fl = []
        for i, p in enumerate(raw):
            table = np.einsum("lkr,vr->lvk", p["input_proj"], p["token_embed"]) + p["bias"][:, None]
            kw = {k: p[k] for k in ("router_embed", "router_weight", "router_bias", "layer_input_down",
                                    "layer_input_proj") if k in p}
            fl.append(E.FloatLayer(token_layer=i == 0, depth=depth if i else 0,
                                   transition=transitions64(p["rotation"], p["decay"]), table=table,
                                   input_proj=p["input_proj"], token_embed=p["token_embed"], bias=p["bias"],
                                   readout=p["readout"], unembed=p["unembed"], **kw))
        for rs, (hm, group, fac) in enumerate(((0.85, False, False), (1.0, True, True))):
            rec = C.synthetic_record(seed=rs, hmargin=hm, group=group, factored=fac)
            stats = [E.LayerStats(**{k: (np.asarray(v) if isinstance(v, list) else v) for k, v in s.items()})
                     for s in rec["stats"]]
            q = E.quantize(fl, stats, **rec["quantize"])
            out = os.path.join(tmp, "ck.bin")
            E.write(q, ob, out, router_token_dim=fl[-1].router_token_dim, input_rank=fl[0].token_embed.shape[1])
            ckpts.append(dict(seed=seed, old_keys=old, record_seed=rs, quantize=rec["quantize"],
                              model_sha256=sha(Path(out).read_bytes()), model_bytes=os.path.getsize(out)))
    (HERE / "checkpoints.json").write_text(json.dumps(ckpts, indent=1) + "\n")


if __name__ == "__main__":
    main()
