"""TEST INFRASTRUCTURE ONLY: a float64 NumPy restatement of the reference's float streaming step, the checker of the
fp32 B200 float step (backend "b200f").

It follows yggdrasil/inference.py of the reference:
  route   :42-52  f = [router_embed(x); rms(h_below)] (the state part only when the router reads it), down the heap
                  from node 0, right iff f . W_node + b_node > 0, expert = node - (2^D - 1);
  update  :55-63  h <- T_r[x] + U'_r (V' rms(h_below)) + A_r h, z = P_r h;
  step    :66-75  the token layer takes expert x, no input from below; logits = output_bias + sum_l z_l Q_l^T;
  Yggdrasil.__init__ :142-152  T_r[x] = U_r v(x) + c_r and A_r = diag(clip(decay, -1, 1)) blockdiag(expm((G - G^T)/2))
                  (yggdrasil/experts.py:8-11), here with scipy's float64 expm;
  rms     yggdrasil/model.py:92-93, eps 1e-6 (yggdrasil/config.py:8);
  score   :179-188  bits of tokens[:, 1:] per row, float64;
  calibrate  cpu/export.py:120-153  the maxima over windows of |h| per group of 16 coordinates, |V' rms(h_below)| and
                  |P_r h| per readout row, per layer (LayerStats), from a zero state.
Only the tests use this module (and tests/golden/make_golden.py, which pins it to the reference's own Triton step);
the product never imports it.
"""
from __future__ import annotations

import numpy as np

RMS_EPS = 1e-6


def _transitions(rotation, decay):
    from scipy.linalg import expm
    g = np.asarray(rotation, np.float64)
    g = 0.5 * (g - np.swapaxes(g, -1, -2))
    e = np.stack([expm(b) for b in g.reshape(-1, *g.shape[-2:])]).reshape(g.shape)
    d = np.clip(np.asarray(decay, np.float64), -1.0, 1.0).reshape(g.shape[:-1])
    return d[..., None] * e


def rms(h):
    return h / np.sqrt(np.mean(h * h, -1, keepdims=True) + RMS_EPS)


class FloatOracle:
    """layers, output_bias as the reference's inference.read returns them (dicts of arrays per layer)."""

    def __init__(self, layers, output_bias):
        self.layers = []
        for p in layers:
            p = {k: np.asarray(v, np.float64) for k, v in p.items()}
            q = {k: v for k, v in p.items() if k not in ("input_proj", "token_embed", "bias", "rotation", "decay")}
            q["table"] = np.einsum("lkr,vr->lvk", p["input_proj"], p["token_embed"]) + p["bias"][:, None]
            if "rotation" in p:
                q["transition"] = _transitions(p["rotation"], p["decay"])
            self.layers.append(q)
        self.output_bias = np.asarray(output_bias, np.float64)
        self.n = self.layers[0]["table"].shape[-1]
        self.vocab = self.layers[0]["table"].shape[1]
        self.classes = len(self.output_bias)
        self.n_layers = len(self.layers)

    def init_state(self, batch):
        return np.zeros((batch, self.n_layers, self.n), np.float64)

    def _route(self, p, x, below):
        f = p["router_embed"][x]
        if p["router_weight"].shape[1] > f.shape[1]:
            f = np.concatenate([f, below], -1)
        depth = (p["router_weight"].shape[0] + 1).bit_length() - 1
        node = np.zeros(len(x), np.int64)
        for _ in range(depth):
            s = np.einsum("bf,bf->b", f, p["router_weight"][node]) + p["router_bias"][node]
            node = 2 * node + 1 + (s > 0)
        return node - (2 ** depth - 1)

    def calibrate(self, windows):
        """Per layer (group maxima of |h| (n/16,), max |V' rms(h_below)|, row maxima of |P_r h| (R,)) over the steps
        of windows (S, T) run from a zero state (cpu/export.py:129-153)."""
        x = np.atleast_2d(np.asarray(windows, np.int64))
        st = self.init_state(len(x))
        L, n = self.n_layers, self.n
        groups = np.zeros((L, n // 16))
        rows = [np.zeros(p["readout"].shape[1]) for p in self.layers]
        vmax = np.zeros(L)
        for t in range(x.shape[1]):
            _, st, _, extra = self.step(x[:, t], st, with_readout=True)
            groups = np.maximum(groups, np.abs(st).reshape(len(x), L, n // 16, 16).max((0, 3)))
            for l in range(L):
                rows[l] = np.maximum(rows[l], np.abs(extra["z"][l]).max(0))
                if extra["v"][l] is not None:
                    vmax[l] = max(vmax[l], np.abs(extra["v"][l]).max())
        return [(groups[l], vmax[l], rows[l]) for l in range(L)]

    def step(self, tokens, state, with_readout=False):
        """tokens (B,), state (B, L, n) -> logits (B, classes), new state (B, L, n), experts (B, L) [, the readouts z
        and the layer inputs V' rms(h_below) of every layer]."""
        x = np.asarray(tokens, np.int64)
        logits = np.broadcast_to(self.output_bias, (len(x), self.classes)).copy()
        new = np.empty_like(state, dtype=np.float64)
        experts = np.empty((len(x), self.n_layers), np.int64)
        below = None
        zs, vs = [], []
        for i, p in enumerate(self.layers):
            r = x if i == 0 else self._route(p, x, below)
            h = p["table"][r, x]
            v = None
            if "layer_input_down" in p and below is not None:
                v = below @ p["layer_input_down"].T
                h = h + np.einsum("bkr,br->bk", p["layer_input_proj"][r], v)
            vs.append(v)
            if "transition" in p:
                a = p["transition"][r]
                h = h + np.einsum("bgij,bgj->bgi", a, state[:, i].reshape(a.shape[:-1])).reshape(h.shape)
            new[:, i] = h
            experts[:, i] = r
            z = np.einsum("brk,bk->br", p["readout"][r], h)
            zs.append(z)
            logits = logits + z @ p["unembed"].T
            below = rms(h)
        if with_readout:
            return logits, new, experts, {"z": zs, "v": vs}
        return logits, new, experts

    def score(self, tokens, state=None):
        """Bits of tokens[:, 1:] per row, float64; state (B, L, n) or None (zero)."""
        tok = np.atleast_2d(np.asarray(tokens, np.int64))
        st = self.init_state(len(tok)) if state is None else np.asarray(state, np.float64)
        nll = np.zeros(len(tok))
        for t in range(tok.shape[1] - 1):
            lg, st, _ = self.step(tok[:, t], st)
            mx = lg.max(-1, keepdims=True)
            lp = lg - (np.log(np.exp(lg - mx).sum(-1, keepdims=True)) + mx)
            nll -= lp[np.arange(len(tok)), tok[:, t + 1]]
        return nll / np.log(2.0)


def log_softmax(z):
    z = np.asarray(z, np.float64)
    mx = z.max(-1, keepdims=True)
    return z - (np.log(np.exp(z - mx).sum(-1, keepdims=True)) + mx)
