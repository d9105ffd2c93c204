"""Synthetic int8 models and token streams for the tests and the benchmark (no checkpoints or datasets needed).

``random_layers(shape, seed)`` draws the same integers, in the same order from ``np.random.default_rng(seed)``, as the
reference's random-model generator (``cpu/export.py:473-532``): orthogonal b x b blocks times decays U[0.6, 1] in Q14,
int16 tables U[-24, 24], uniform int8 projections and readouts, thresholds 300 N(0, 1). Keeping the draw order lets
a file written here equal, byte for byte, the file the reference writes for the same shape and seed, which is what
pins this generator (and, through it, the parity fixtures) to the reference.

``WORKLOADS`` are the benchmark shapes. The router rows of those are redrawn as N(0, 0.02) quantised symmetrically
per row to int8, the scheme the benchmark configuration names; everything else is the generator above.
"""
from __future__ import annotations

import dataclasses

import numpy as np

from .ygg1 import LIMITS, SHIFT, STATE_GROUP, FactoredInput, IntLayer, write_model

f32 = np.float32


@dataclasses.dataclass(frozen=True)
class ModelShape:
    """Shape of a random int8 model (the reference's KernelConfig fields, cpu/export.py:473-484)."""
    d_state: int
    block_size: int
    router_depth: int
    vocab: int
    n_layers: int = 2
    readout_rank: int = 8
    layer_input_rank: int = 16
    input_rank: int = 0          # > 0: factored input storage of this rank
    group: bool = False          # group scales

    @property
    def extended(self) -> bool:
        """Outside the reference's YGG1 limits: a file of this shape needs the d_state 96 extension (ygg1 module)."""
        return self.d_state not in LIMITS["d_state"] or self.readout_rank not in LIMITS["readout_rank"]


def random_layers(shape: ModelShape, seed: int = 1):
    """Random IntLayers of the given shape (draw order of cpu/export.py:487-532)."""
    rng = np.random.default_rng(seed)
    n, b, depth, vocab = shape.d_state, shape.block_size, shape.router_depth, shape.vocab
    r, r2 = shape.readout_rank, shape.layer_input_rank
    blocks = np.linalg.qr(rng.standard_normal((64, b, b)))[0]   # 64 distinct orthogonal blocks
    layers = []
    for l in range(shape.n_layers):
        experts = vocab if l == 0 else 2 ** depth
        a16 = np.empty((experts, n // b, b, b), np.int64)
        for j in range(0, experts, 4096):
            m = min(4096, experts - j)
            decay = rng.uniform(0.6, 1.0, (m, n // b, b, 1))
            a16[j:j + m] = np.rint(2.0 ** SHIFT * decay * blocks[rng.integers(0, 64, (m, n // b))])
        kw = dict(token_layer=l == 0, n=n, block=b, depth=0 if l == 0 else depth, transition=a16)
        if l == 0:
            kw["table"] = rng.integers(-24, 25, (vocab, 1, n), dtype=np.int16)
        else:
            if shape.input_rank:
                k = shape.input_rank
                proj = rng.integers(-127, 128, (experts, n, k), dtype=np.int8).astype(np.int64)
                su = rng.uniform(0.5, 1.5, experts).astype(f32)
                bias = rng.integers(-24, 25, (experts, n), dtype=np.int16)
                code = rng.integers(-127, 128, (vocab, k))
                ts = rng.uniform(0.0002, 0.001, n).astype(f32)
                kw["factored"] = FactoredInput(input_proj=proj, input_scale=su, bias=bias, token_code=code,
                                               token_scale=ts)
            else:
                kw["table"] = rng.integers(-24, 25, (experts, vocab, n), dtype=np.int16)
            kw["router_weight"] = rng.integers(-127, 128, (experts - 1, n))
            kw["router_threshold"] = (300 * rng.standard_normal((vocab, experts - 1))).astype(f32)
            kw["rms_eps"] = f32(1e-4)
            if r2:
                kw["layer_input_down"] = rng.integers(-127, 128, (r2, n))
                kw["layer_input_down_scale"] = np.full(r2, 0.05, f32)
                kw["layer_input_proj"] = rng.integers(-127, 128, (experts, n, r2), dtype=np.int8).astype(np.int64)
                kw["layer_input_scale"] = f32(0.002)
        kw["readout_scale"], kw["unembed_scale"] = f32(0.002), f32(0.001)
        if shape.group:
            kw["readout_scale"] = rng.uniform(0.0005, 0.004, (experts, r)).astype(f32)
            kw["unembed_scale"] = rng.uniform(0.0005, 0.002, vocab).astype(f32)
            if l > 0:
                kw["state_r2"] = (rng.uniform(0.05, 1.0, n // STATE_GROUP) ** 2).astype(f32)
                if r2:
                    kw["layer_input_scale"] = rng.uniform(0.0005, 0.004, n).astype(f32)
        kw["readout"] = rng.integers(-127, 128, (experts, r, n))
        kw["unembed"] = rng.integers(-127, 128, (vocab, r))
        layers.append(IntLayer(**kw))
    return layers


def write_random_model(shape: ModelShape, path, seed: int = 7, output_bias=None, extended: bool = False):
    """Random model of shape written to path; output bias linspace(-1, 1, V) by default (as the reference's kernel
    test uses, cpu/tests/test_kernel.py:39). extended: admit the d_state 96 extension. Returns the layers."""
    layers = random_layers(shape, seed)
    ob = np.linspace(-1, 1, shape.vocab) if output_bias is None else output_bias
    write_model(layers, ob, path, extended=extended)
    return layers


def gaussian_router_rows(layers, seed: int, std: float = 0.02):
    """Replace each routed layer's router rows by N(0, std) draws quantised symmetrically per row to int8."""
    rng = np.random.default_rng(seed)
    for q in layers[1:]:
        w = rng.normal(0.0, std, q.router_weight.shape)
        s = np.maximum(np.abs(w).max(-1, keepdims=True), 1e-12) / 127
        q.router_weight = np.rint(w / s).astype(np.int64)
    return layers


# ------------------------------------------------------------------------------------------------------ workloads

DNA_P = np.array([0.295, 0.205, 0.205, 0.295, 0.0001])
DNA_P = DNA_P / DNA_P.sum()


@dataclasses.dataclass(frozen=True)
class Workload:
    name: str
    shape: ModelShape
    streams: int
    steps: int
    tokens: str                  # "uniform" or "dna"
    note: str = ""
    leaves: str = "random"       # "random": the generator's thresholds; "zipf": calibrated to Zipf(1.1) leaf usage
    model: str = ""              # the workload whose model file this one shares ("": its own)

    @property
    def extended(self) -> bool:
        return self.shape.extended


WORKLOADS = {
    # V256 L2 d64 D10: batch 1, 4096 uniform bytes
    "c1": Workload("c1-5M-enwik8", ModelShape(64, 16, 10, 256, 2, 8, 16), 1, 4096, "uniform"),
    # V256 L4 d64 D12, factored k=16 (73.1 MB) is the file closest to the named 65 MB
    "c2": Workload("c2-65MB-enwik8", ModelShape(64, 16, 12, 256, 4, 8, 16, input_rank=16), 4096, 1024, "uniform"),
    # V5 L4 D13 with R = n/8, R2 = n/4 at d = 128 (287 MB): the nearest shape inside the reference's YGG1 limits
    # (d_state 64/128/256, readout rank 8/16/32), so that the reference's ygg runs the same file as the CPU baseline
    "c3": Workload("c3-200M-dna-d128", ModelShape(128, 16, 13, 5, 4, 16, 32), 65536, 512, "dna",
                   "d_state 128 in place of 96 (the reference's YGG1 allows 64/128/256)"),
    # the named d = 96 (186.9 MB, R = 12, R2 = 24) through this repository's d_state 96 extension, which the
    # reference's ygg refuses; its oracle is the reference's int_forward
    "c3n96": Workload("c3-200M-dna-d96", ModelShape(96, 16, 13, 5, 4, 12, 24), 65536, 512, "dna",
                      "d_state 96 through the format extension (the reference's ygg refuses the file)"),
    # V256 L4 d128 D13 R16 R2=32, table storage (1892 MB)
    "c4": Workload("c4-730M-enwik8", ModelShape(128, 16, 13, 256, 4, 16, 32), 262144, 256, "uniform",
                   "table storage, 1892 MB; thresholds calibrated to Zipf(1.1) leaf usage", leaves="zipf"),
    # the same model with factored input storage k=32 (390 MB)
    "c4f": Workload("c4-730M-enwik8-factored", ModelShape(128, 16, 13, 256, 4, 16, 32, input_rank=32), 262144, 256,
                    "uniform", "factored storage k=32, 390 MB; Zipf(1.1) leaf usage", leaves="zipf"),
    # the scoring configuration: 512 rows of 8192 uniform bytes on the c4 model
    "c5": Workload("c5-score-730M", ModelShape(128, 16, 13, 256, 4, 16, 32), 512, 8192, "uniform",
                   "whole rows scored on the c4 model", leaves="zipf", model="c4"),
}


def workload_layers(w: Workload, seed: int = 7, thresholds=None):
    """Layers of a benchmark workload: the random generator plus N(0, 0.02) int8 router rows. thresholds: the
    per-node router thresholds of the routed layers, (L - 1, 2^D - 1) f32, shared by every token (the Zipf-calibrated
    workloads c4, c4f and c5 take them from their fixture, ZIPF_FIXTURE); None keeps the generator's."""
    layers = gaussian_router_rows(random_layers(w.shape, seed), seed + 1)
    if thresholds is not None:
        apply_thresholds(layers, thresholds)
    return layers


def apply_thresholds(layers, thresholds, only: int = 0):
    """Set the router thresholds of the routed layers to per-node values shared by every token: thresholds (L - 1,
    2^D - 1) f32, row l - 1 for layer l; only > 0 sets that layer alone."""
    thr = np.asarray(thresholds, f32)
    for l in range(1, len(layers)):
        if only and l != only:
            continue
        q = layers[l]
        q.router_threshold = np.ascontiguousarray(np.broadcast_to(thr[l - 1], (q_vocab(layers), thr.shape[1])),
                                                  dtype=f32)
    return layers


def q_vocab(layers) -> int:
    """Vocabulary of a model's layers (the token layer has one expert per token)."""
    return int(layers[0].transition.shape[0])


# Router thresholds of the Zipf-calibrated workloads (tests/golden/make_golden.py computes them with the C oracle and
# pins the resulting models to the reference's writer and int_forward): an .npz with one (L - 1, 2^D - 1) f32 array
# per model key (c4, c4f). c5 scores the c4 model.
ZIPF_FIXTURE = "tests/golden/zipf_thresholds.npz"


def zipf_thresholds_of(w: Workload, root) -> np.ndarray | None:
    """The fixture thresholds of a Zipf-calibrated workload (None for the others); root: the repository root."""
    if w.leaves != "zipf":
        return None
    from pathlib import Path
    key = w.model or next(k for k, v in WORKLOADS.items() if v is w)
    with np.load(Path(root) / ZIPF_FIXTURE) as z:
        return z[key]


def workload_tokens(w: Workload, streams: int, steps: int, seed: int = 0) -> np.ndarray:
    """(streams, steps) int32 tokens: uniform over the vocabulary, or i.i.d. DNA bases with DNA_P."""
    rng = np.random.default_rng(seed)
    if w.tokens == "dna":
        return rng.choice(len(DNA_P), size=(streams, steps), p=DNA_P).astype(np.int32)
    return rng.integers(0, w.shape.vocab, (streams, steps)).astype(np.int32)


def zipf_leaf_probs(n_leaves: int, s: float, seed: int) -> np.ndarray:
    """Zipf(s) probabilities over the leaves in a seeded random order: leaf perm[i] gets rank i + 1."""
    p = 1.0 / np.arange(1, n_leaves + 1, dtype=np.float64) ** s
    out = np.empty(n_leaves)
    out[np.random.default_rng(seed).permutation(n_leaves)] = p / p.sum()
    return out


def effective_leaves(p: np.ndarray) -> float:
    """exp of the entropy of a leaf distribution (the number of equally used leaves with the same entropy)."""
    p = p[p > 0] / p.sum()
    return float(np.exp(-(p * np.log(p)).sum()))


def rho_f32(qb: np.ndarray, eps, r2b=None) -> np.ndarray:
    """The router's f32 rho of int8 states qb (S, n), as the reference computes it (cpu/ygg.cpp:248-266)."""
    n = qb.shape[1]
    q = qb.astype(np.int64)
    if r2b is None:
        ss = (q * q).sum(1).astype(f32)
    else:
        g = (q * q).reshape(len(q), -1, STATE_GROUP).sum(-1)
        ss = np.zeros(len(q), f32)
        for j in range(g.shape[1]):
            ss = (ss + f32(r2b[j]) * g[:, j].astype(f32)).astype(f32)
    return (f32(1) / np.sqrt(ss * f32(1.0 / n) + f32(eps))).astype(f32)


def zipf_thresholds(router_weight: np.ndarray, qb: np.ndarray, rho: np.ndarray, leaf_p: np.ndarray) -> np.ndarray:
    """Per-node thresholds (2^D - 1,) that route the sample states qb (S, n) with rho (S,) to leaf frequencies leaf_p
    (2^D,): top-down, node ix sends the share mass(right subtree) / mass(subtree) of the samples reaching it to the
    right, the threshold being that quantile of their f32 scores f32(w_ix . qb) * rho. Nodes no sample reaches get 0."""
    E = len(leaf_p)
    depth = E.bit_length() - 1
    mass = np.zeros(2 * E)
    mass[E:] = leaf_p
    for ix in range(E - 1, 0, -1):
        mass[ix] = mass[2 * ix] + mass[2 * ix + 1]
    thr = np.zeros(E, f32)                                   # heap slots 1 .. E-1
    w = np.zeros((E, router_weight.shape[1]), np.int64)
    w[1:] = router_weight
    node = np.ones(len(qb), np.int64)
    q = qb.astype(np.int64)
    for _ in range(depth):
        score = (np.einsum("sn,sn->s", w[node], q).astype(f32) * rho).astype(f32)
        order = np.lexsort((score, node))
        ns, sc = node[order], score[order]
        starts = np.flatnonzero(np.r_[True, ns[1:] != ns[:-1]])
        ends = np.r_[starts[1:], len(ns)]
        for a, b in zip(starts, ends):
            ix = ns[a]
            p_right = mass[2 * ix + 1] / mass[ix] if mass[ix] > 0 else 0.5
            k = int(np.clip(round((b - a) * (1.0 - p_right)), 0, b - a))  # k samples stay left
            if k <= 0:
                thr[ix] = np.nextafter(sc[a], f32(-np.inf))
            elif k >= b - a:
                thr[ix] = sc[b - 1]
            else:
                thr[ix] = sc[a + k - 1]                      # right iff score > thr: the top (b - a - k) go right
        node = 2 * node + (score > thr[node])
    return thr[1:]


def gathered_bytes_per_token(shape: ModelShape, with_io: bool = True) -> int:
    """Algorithmic bytes gathered per token of one decode step (per-stream weights and state/logit traffic; shared
    per-launch weights excluded): G = G_tok + (L-1) G_rt (+ IO = 2 L n + 4 V + 4)."""
    n, b, d, v = shape.d_state, shape.block_size, shape.router_depth, shape.vocab
    r, r2, k, L = shape.readout_rank, shape.layer_input_rank, shape.input_rank, shape.n_layers
    g_tok = 2 * n * b + r * n + 2 * n
    s = (n * k + 2 * n + 4) if k else 2 * n
    g_rt = d * n + 4 * d + 2 * n * b + n * r2 + r * n + s
    io = 2 * L * n + 4 * v + 4 if with_io else 0
    return g_tok + (L - 1) * g_rt + io


# ------------------------------------------------------------------------------------------------- float models

# The float model of the reference's enwik8 large configuration (configs/enwik8/large.yaml: 5 layers, d_state 256,
# blocks of 16, router depth 10, router token dim 16, input rank 64, readout rank 32, layer-input rank 64, V 256), the
# model its published fp32 GPU time is quoted on (80.1 us/token at batch 1, README.md:43).
FLOAT_ENWIK8_LARGE = dict(vocab=256, n=256, block=16, depth=10, readout=32, layer_input=64, input_rank=64,
                          router_token=16, routed=4)


def random_float_layers(shape: dict, seed: int = 0):
    """Random parameters of a float model with the checkpoint's keys and shapes (yggdrasil/config.py PARAMS):
    (layers [token layer, routed layers...] as dicts of float32 arrays, output bias), as read_checkpoint returns them.
    Scales keep the state and the logits in a trained model's range: decays U[0.6, 1], rotation generators N(0, 0.4),
    the readout and unembedding scaled by 1/sqrt of their fan-in."""
    rng = np.random.default_rng(seed)
    V, n, b, D = shape["vocab"], shape["n"], shape["block"], shape["depth"]
    R, R2, k, F = shape["readout"], shape["layer_input"], shape["input_rank"], shape["router_token"]

    def layer(E, routed):
        p = {"token_embed": rng.standard_normal((V, k), dtype=f32),
             "input_proj": (rng.standard_normal((E, n, k), dtype=f32) * f32(0.3 / np.sqrt(k / 16))),
             "bias": rng.standard_normal((E, n), dtype=f32) * f32(0.5),
             "rotation": rng.standard_normal((E, n // b, b, b), dtype=f32) * f32(0.4),
             "decay": rng.uniform(0.6, 1.0, (E, n)).astype(f32),
             "readout": rng.standard_normal((E, R, n), dtype=f32) * f32(1.0 / n),
             "unembed": rng.standard_normal((V, R), dtype=f32) * f32(2.0 / np.sqrt(R))}
        if routed:
            p.update(router_embed=rng.standard_normal((V, F), dtype=f32),
                     router_weight=rng.standard_normal((E - 1, F + n), dtype=f32) * f32(0.3),
                     router_bias=rng.standard_normal(E - 1, dtype=f32) * f32(0.1),
                     layer_input_down=rng.standard_normal((R2, n), dtype=f32) * f32(1.0 / np.sqrt(n)),
                     layer_input_proj=rng.standard_normal((E, n, R2), dtype=f32) * f32(0.2 / np.sqrt(R2 / 16)))
        return p

    layers = [layer(V, False)] + [layer(2 ** D, True) for _ in range(shape["routed"])]
    return layers, rng.standard_normal(V, dtype=f32) * f32(0.5)
