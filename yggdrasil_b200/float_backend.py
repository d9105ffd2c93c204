"""The fp32 float step on B200, backend "b200f": the reference's float inference model (yggdrasil/inference.py) run by
the sm_100a kernel of libygg_b200.so (csrc/ygg_float.cu) through its C-ABI (ygg_fload / ygg_fstep).

    from yggdrasil_b200 import Yggdrasil
    model = Yggdrasil.load("results/<run>.npz", backend="b200f")   # a training checkpoint, as the reference reads it
    state = model.init_state(B)                                   # (B, layers, n) float32 on the GPU
    logits, state = model.step(tokens, state)                     # (B,) -> (B, classes) float32
    bits = model.score(windows)                                   # (B, L) -> bits of windows[:, 1:] per row

The interface and behaviour are those of the reference's Triton backend (yggdrasil/inference_triton.py:123-248): the
same tables T_r[x] = U_r v(x) + c_r and transitions A_r formed in float64 and rounded to float32
(inference_triton.py:109-120), the same state layout, step, score (float64 sums of fp32 log-softmax values) and
generate; and the reference's errors: NotImplementedError for a model without a routed layer or with routed layers of
mixed kinds (inference_triton.py:126-128), ValueError for a token out of range.
"""
from __future__ import annotations

import ctypes
import math
from pathlib import Path

import numpy as np

from . import _native
from ._native import check, flib as lib

LN2 = math.log(2.0)


def _torch():
    import torch
    return torch


class YggFShape(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in (
        "n_layers", "d_state", "block_size", "vocab", "classes", "router_depth", "router_token_dim", "readout_rank",
        "layer_input_rank", "route_on_state", "token_transition", "routed_transition")]


ARRAYS_PER_LAYER = 9


def _transitions(p):
    """A_r = diag(clip(decay, -1, 1)) blockdiag(expm((G - G^T) / 2)) in float64, rounded to float32."""
    from .checkpoint import transitions64
    return transitions64(p["rotation"], p["decay"]).astype(np.float32)


def _table(p, own_rows: bool):
    """T_r[x] = U_r v(x) + c_r in float64, rounded to float32: (E, V, n), or the token layer's own rows (V, n)."""
    torch = _torch()
    u, v, c = (torch.as_tensor(np.asarray(p[k]), dtype=torch.float64) for k in ("input_proj", "token_embed", "bias"))
    if own_rows:   # expert x of the token layer only ever reads its own row x
        return (torch.einsum("vkr,vr->vk", u, v) + c).float().numpy()
    return (torch.einsum("lkr,vr->lvk", u, v) + c[:, None, :]).float().numpy()


class B200FloatYggdrasil:
    """layers, output_bias as yggdrasil_b200.checkpoint.read_checkpoint (or the reference's inference.read) returns
    them. device: a CUDA device; cuda_graph: replay one captured step per batch size."""

    def __init__(self, layers, output_bias, device="cuda", cuda_graph=False):
        torch = _torch()
        tk, rt = layers[0], layers[1:]
        if not rt or len({"rotation" in p for p in rt}) > 1:
            raise NotImplementedError("the fused step needs at least one routed layer, all of one kind")
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError(f"device {device!r}: the b200f backend runs on a CUDA device")
        self.device = torch.device("cuda", dev.index if dev.index is not None else torch.cuda.current_device())
        r0 = rt[0]
        self.layers, self.n = len(layers), np.asarray(tk["bias"]).shape[1]
        self.vocab, self.classes = np.asarray(tk["token_embed"]).shape[0], len(output_bias)
        self.readout_rank = np.asarray(tk["readout"]).shape[1]
        F = np.asarray(r0["router_embed"]).shape[1]
        fin = np.asarray(r0["router_weight"]).shape[1]
        self.depth = (np.asarray(r0["router_weight"]).shape[0] + 1).bit_length() - 1
        token_a, routed_a = "rotation" in tk, "rotation" in r0
        block = np.asarray((tk if token_a else r0)["rotation"]).shape[-1] if token_a or routed_a else 2
        r2 = np.asarray(r0["layer_input_down"]).shape[0] if "layer_input_down" in r0 else 0
        shape = YggFShape(self.layers, self.n, block, self.vocab, self.classes, self.depth, F,
                          np.asarray(tk["readout"]).shape[1], r2, int(fin != F), int(token_a), int(routed_a))
        keep, ptrs = [], []

        def arr(a):
            if a is None:
                ptrs.append(None)
                return
            a = np.ascontiguousarray(a, np.float32)
            keep.append(a)
            ptrs.append(a.ctypes.data_as(ctypes.c_void_p))

        for i, p in enumerate(layers):
            arr(_table(p, own_rows=i == 0))
            arr(_transitions(p) if "rotation" in p else None)
            arr(p["readout"])
            arr(p["unembed"])
            if i == 0:
                ptrs.extend([None] * 5)
            else:
                arr(p["router_embed"])
                arr(p["router_weight"])
                arr(p["router_bias"])
                arr(p.get("layer_input_down") if r2 else None)
                arr(p.get("layer_input_proj") if r2 else None)
        arr(output_bias)
        table = (ctypes.c_void_p * len(ptrs))(*[p.value if p is not None else None for p in ptrs])
        self._h = ctypes.c_void_p()
        code = lib().ygg_fload(ctypes.byref(shape), table, self.device.index, ctypes.byref(self._h))
        if code == _native.YGG_E_UNSUPPORTED:
            raise NotImplementedError("float model outside the limits of the b200f step (include/ygg_b200.h)")
        check(code, "ygg_fload")
        self.cuda_graph, self._graphs = cuda_graph, {}

    @classmethod
    def from_checkpoint(cls, path, **kw):
        from .checkpoint import read_checkpoint
        return cls(*read_checkpoint(path), **kw)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                lib().ygg_ffree(h)
            except Exception:  # noqa: BLE001 (interpreter shutdown)
                pass
            self._h = None

    def init_state(self, batch_size):
        """Zero state of batch_size streams, (B, layers, n) float32."""
        torch = _torch()
        return torch.zeros(batch_size, self.layers, self.n, dtype=torch.float32, device=self.device)

    def _tokens(self, tokens):
        torch = _torch()
        if isinstance(tokens, torch.Tensor) and tokens.is_cuda:
            return tokens.to(device=self.device, dtype=torch.int32).contiguous()
        a = np.asarray(tokens.cpu() if isinstance(tokens, torch.Tensor) else tokens)
        if a.size and (a.min() < 0 or a.max() >= self.vocab):
            bad = a[(a < 0) | (a >= self.vocab)].flat[0]
            raise ValueError(f"tokens: token {int(bad)} out of range [0, {self.vocab})")
        return torch.as_tensor(np.ascontiguousarray(a, np.int32)).to(self.device)

    def status(self):
        """Raise ValueError if a step since the last call met a device token out of range, RuntimeError if one of its
        bounded waits for an asynchronous copy gave up (its results are still exact)."""
        torch = _torch()
        out = ctypes.c_int(0)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(lib().ygg_fstatus(self._h, ctypes.c_void_p(stream), ctypes.byref(out)), "ygg_fstatus")
        if out.value == _native.YGG_E_TOKEN:
            raise ValueError("a device token was out of range (those streams were skipped)")
        if out.value == _native.YGG_E_TIMEOUT:
            raise RuntimeError("a step's bounded wait for an asynchronous copy gave up (it read global memory instead)")

    def step_into(self, tokens, state_in, state_out, logits, experts=None):
        """One step into caller buffers (state_out may be state_in). tokens: an int32 device tensor."""
        torch = _torch()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(lib().ygg_fstep(self._h, tokens.shape[0], tokens.data_ptr(), state_in.data_ptr(), state_out.data_ptr(),
                              logits.data_ptr(), experts.data_ptr() if experts is not None else None, stream),
              "ygg_fstep")

    def _step(self, x, h):
        torch = _torch()
        out = torch.empty_like(h)
        logits = torch.empty((x.shape[0], self.classes), dtype=torch.float32, device=self.device)
        self.step_into(x, h, out, logits)
        return logits, out

    def _check_state(self, state, batch):
        torch = _torch()
        if not isinstance(state, torch.Tensor) or state.dtype != torch.float32 or tuple(state.shape) != (
                batch, self.layers, self.n) or state.device != self.device:
            raise ValueError(f"state must be a float32 tensor ({batch}, {self.layers}, {self.n}) on {self.device}")
        return state.contiguous()

    def step(self, tokens, state):
        """One token per stream: tokens (B,) -> logits (B, classes) of the next token, state."""
        torch = _torch()
        if not self.cuda_graph and type(tokens) is torch.Tensor and tokens.is_cuda and tokens.dtype == torch.int32 \
                and tokens.device == self.device and tokens.is_contiguous() and type(state) is torch.Tensor \
                and state.dtype == torch.float32 and state.device == self.device and state.is_contiguous() \
                and state.shape == (tokens.shape[0], self.layers, self.n):
            return self._step(tokens, state)   # device tokens and state as they are: no device switch, no copies
        with torch.cuda.device(self.device):
            x = self._tokens(tokens)
            state = self._check_state(state, x.shape[0])
            if not self.cuda_graph:
                return self._step(x, state)
            b = x.shape[0]
            if b not in self._graphs:
                sx, sh = torch.zeros(b, dtype=torch.int32, device=self.device), self.init_state(b)
                self._step(sx, sh)
                torch.cuda.synchronize(self.device)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    out = self._step(sx, sh)
                self._graphs[b] = g, sx, sh, out
            g, sx, sh, (logits, h) = self._graphs[b]
            sx.copy_(x)
            sh.copy_(state)
            g.replay()
            return logits.clone(), h.clone()

    def step_experts(self, tokens, state):
        """step that also returns the expert of every layer (B, layers) int32."""
        torch = _torch()
        with torch.cuda.device(self.device):
            x = self._tokens(tokens)
            state = self._check_state(state, x.shape[0])
            out = torch.empty_like(state)
            logits = torch.empty(x.shape[0], self.classes, dtype=torch.float32, device=self.device)
            experts = torch.empty(x.shape[0], self.layers, dtype=torch.int32, device=self.device)
            self.step_into(x, state, out, logits, experts)
            return logits, out, experts

    def score(self, tokens, state=None, batch=1024):
        """Bits of tokens[:, 1:] given the tokens before them, per row of tokens (B, L), as float64 (B,)
        (inference_triton.py:214-227: fp32 log-softmax of each step's logits, summed in float64)."""
        torch = _torch()
        tokens = np.atleast_2d(np.asarray(tokens.cpu() if isinstance(tokens, torch.Tensor) else tokens))
        if tokens.size and (tokens.min() < 0 or tokens.max() >= self.vocab):
            raise ValueError(f"tokens out of range [0, {self.vocab})")
        out = []
        with torch.cuda.device(self.device), torch.no_grad():
            for i in range(0, len(tokens), batch):
                x = torch.as_tensor(np.ascontiguousarray(tokens[i:i + batch], np.int32), device=self.device)
                st = self.init_state(len(x)) if state is None else self._check_state(state[i:i + batch], len(x)).clone()
                logits = torch.empty(len(x), self.classes, dtype=torch.float32, device=self.device)
                nll = torch.zeros(len(x), dtype=torch.float64, device=self.device)
                for t in range(x.shape[1] - 1):
                    self.step_into(x[:, t].contiguous(), st, st, logits)
                    nll -= torch.log_softmax(logits, -1).gather(1, x[:, t + 1, None].long())[:, 0].double()
                out.append((nll / LN2).cpu().numpy())
        self.status()
        return np.concatenate(out) if out else np.zeros(0, np.float64)

    def generate(self, prompt, n, temperature=1.0, top_k=0, seed=0):
        """Prompt (L,) or (B, L), L >= 1, followed by n sampled tokens. temperature 0: greedy
        (inference_triton.py:229-248; sampling draws from torch's generator, as the Triton backend's does)."""
        torch = _torch()
        prompt = np.asarray(prompt, np.int64)
        x = np.atleast_2d(prompt)
        with torch.cuda.device(self.device), torch.no_grad():
            state = self.init_state(len(x))
            gen = torch.Generator(self.device).manual_seed(seed)
            out = [torch.as_tensor(x, device=self.device)]
            logits = None
            for t in range(x.shape[1]):
                logits, state = self.step(x[:, t], state)
            for i in range(n):
                if temperature == 0:
                    tok = logits.argmax(-1)
                else:
                    lg = logits
                    if top_k:
                        lg = lg.masked_fill(lg < lg.topk(top_k, -1).values[:, -1:], -float("inf"))
                    tok = torch.multinomial(torch.softmax(lg / temperature, -1), 1, generator=gen)[:, 0]
                out.append(tok[:, None])
                if i + 1 < n:
                    logits, state = self.step(tok.to(torch.int32), state)
            res = torch.cat(out, 1).cpu().numpy()
        return res[0] if prompt.ndim == 1 else res
