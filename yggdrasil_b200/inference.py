"""The int8 B200 backend behind the reference's inference API (yggdrasil/inference.py:142-202).

    from yggdrasil_b200 import Yggdrasil
    model = Yggdrasil.load("model.bin", backend="b200")     # a YGG1 int8 file (cpu/export.py writes them)
    state = model.init_state(batch_size)                    # (B, layers, n) int8 on the GPU
    logits, state = model.step(tokens, state)               # tokens (B,) -> logits (B, V) float32, new state
    bits = model.score(windows)                             # (B, L) -> bits of windows[:, 1:] per row, float64
    text = model.generate(prompt, 200, temperature=0.8, top_k=20)

Same calls, argument meaning and errors as the reference's backends: ``ValueError`` for an unknown backend or a
token outside the vocabulary, ``ImportError`` when the backend's native library is missing,
``NotImplementedError`` for model variants this backend does not run. The step is one launch of the hand-written
sm_100a kernel in libygg_b200.so through its C-ABI; PyTorch only holds device memory and the current stream.
The int8 state is the reference kernel's (cpu/ygg.cpp:439, one int8 vector per layer), so ``step`` and ``score``
equal cpu/ygg.cpp / cpu/export.py:int_forward bit for bit on the logits.
"""
from __future__ import annotations

import ctypes
import math
from pathlib import Path

import numpy as np

from . import _native
from ._native import YggInfo, check, lib

LN2 = math.log(2.0)


def _torch():
    import torch
    return torch


def _raw_stream(index: int) -> int:
    """The current CUDA stream of device `index` as a raw pointer (torch's own accessor, which step() calls once per
    token; torch.cuda.current_stream builds a Stream object around the same pointer)."""
    torch = _torch()
    get = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    return get(index) if get is not None else torch.cuda.current_stream(index).cuda_stream


class Yggdrasil:
    """Backend dispatch of the reference's ``Yggdrasil.load`` (yggdrasil/inference.py:158-169)."""

    @classmethod
    def load(cls, path, backend="b200", **kw):
        """backend "b200": the sm_100a int8 step of a YGG1 file (or of an .npz with its export record); "b200f": the
        sm_100a fp32 step of a training checkpoint (.npz), the float model of the reference's jax and triton
        backends. kw device="cuda", cuda_graph=False."""
        if backend == "b200":
            return B200Yggdrasil(path, **kw)
        if backend == "b200f":
            from .float_backend import B200FloatYggdrasil
            return B200FloatYggdrasil.from_checkpoint(path, **kw)
        if backend in ("jax", "triton"):
            raise ValueError(f"backend {backend!r} is a backend of the reference package; yggdrasil_b200 provides "
                             "backend='b200' (the int8 step) and backend='b200f' (the fp32 step)")
        raise ValueError(f"backend {backend!r}: b200 or b200f")


class B200Yggdrasil:
    def __init__(self, model, device="cuda", cuda_graph=False, record=None):
        """model: path of a YGG1 file, or its bytes, or a float checkpoint (.npz) with `record`, the export record
        (model.bin.json, or its dict) whose calibration stats and quantize arguments rebuild the int8 model
        (yggdrasil_b200.checkpoint). device: a CUDA device. cuda_graph: replay one captured step per batch size (as
        the reference's Triton backend, inference_triton.py:196-212)."""
        torch = _torch()
        if isinstance(model, (str, Path)):
            p = Path(model)
            if p.suffix == ".npz":
                if record is None:
                    raise NotImplementedError(
                        f"{p}: a float checkpoint needs its calibration before it runs in int8: pass record= (the "
                        "model.bin.json the reference's cpu/export.py writes), or export a YGG1 file first")
                from .checkpoint import export_bytes
                data = export_bytes(p, record)
            else:
                data = p.read_bytes()
        else:
            data = bytes(model)
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError(f"device {device!r}: the b200 backend runs on a CUDA device")
        self.device = torch.device("cuda", dev.index if dev.index is not None else torch.cuda.current_device())
        self._h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(data, len(data))
        code = lib().ygg_load(buf, len(data), self.device.index, ctypes.byref(self._h))
        if code == _native.YGG_E_FORMAT:
            raise ValueError("not a YGG1 model file")
        if code == _native.YGG_E_UNSUPPORTED:
            raise NotImplementedError("model outside the YGG1 limits (cpu/export.py LIMITS)")
        check(code, "ygg_load")
        info = YggInfo()
        check(lib().ygg_info(self._h, ctypes.byref(info)), "ygg_info")
        self.info = {k: getattr(info, k) for k, _ in YggInfo._fields_}
        self.layers, self.n, self.vocab = info.n_layers, info.d_state, info.vocab
        self.classes, self.depth = info.vocab, info.router_depth
        self.cuda_graph, self._graphs = cuda_graph, {}
        self._dix, self._state_shape = self.device.index, (self.layers, self.n)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                lib().ygg_free(h)
            except Exception:  # noqa: BLE001 (interpreter shutdown)
                pass
            self._h = None

    # ------------------------------------------------------------------------------------------------ state

    def init_state(self, batch_size):
        """Zero state of batch_size streams, (B, layers, n) int8 on the device."""
        torch = _torch()
        return torch.zeros(batch_size, self.layers, self.n, dtype=torch.int8, device=self.device)

    def _tokens(self, tokens, what="tokens"):
        """tokens -> int32 contiguous device tensor; host tokens are range-checked here (cpu/ygg.cpp:493-495)."""
        torch = _torch()
        if isinstance(tokens, torch.Tensor):
            if tokens.is_cuda:
                return tokens.to(device=self.device, dtype=torch.int32).contiguous()
            t = tokens.to(torch.int32).contiguous()   # a pinned int32 tensor is copied asynchronously as it is
            if t.numel():
                lo, hi = int(t.min()), int(t.max())
                if lo < 0 or hi >= self.vocab:
                    raise ValueError(f"{what}: token {lo if lo < 0 else hi} out of range [0, {self.vocab})")
            return t.to(self.device, non_blocking=True)
        a = np.asarray(tokens)
        if a.size and (a.min() < 0 or a.max() >= self.vocab):
            bad = a[(a < 0) | (a >= self.vocab)].flat[0]
            raise ValueError(f"{what}: token {int(bad)} out of range [0, {self.vocab})")
        return torch.as_tensor(np.ascontiguousarray(a, np.int32)).to(self.device)

    def _check_state(self, state, batch):
        torch = _torch()
        if not isinstance(state, torch.Tensor) or state.dtype != torch.int8 or tuple(state.shape) != (
                batch, self.layers, self.n) or state.device != self.device:
            raise ValueError(f"state must be an int8 tensor ({batch}, {self.layers}, {self.n}) on {self.device}")
        return state.contiguous()

    def status(self, clear=True):
        """Raise if a kernel since the last call met a bad device token or a bounded wait that gave up."""
        torch = _torch()
        out = ctypes.c_int(0)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(lib().ygg_status(self._h, ctypes.c_void_p(stream), int(clear), ctypes.byref(out)), "ygg_status")
        if out.value == _native.YGG_E_TOKEN:
            raise ValueError("a device token was out of range (those streams were skipped)")
        check(out.value, "device status")

    # ------------------------------------------------------------------------------------------------ step

    def step_into(self, tokens, state_in, state_out, logits=None, routes=None, acc=None):
        """One step into caller buffers (state_out may be state_in: in place). tokens: an int32 device tensor."""
        torch = _torch()
        b = tokens.shape[0]
        stream = _raw_stream(self._dix)
        if routes is None and acc is None:
            # pointers as plain ints (the bound argtypes convert them): the per-token path of step()
            code = lib().ygg_step(self._h, b, tokens.data_ptr(), state_in.data_ptr(), state_out.data_ptr(),
                                  logits.data_ptr() if logits is not None else None, stream)
        else:
            p = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
            code = lib().ygg_step_debug(self._h, b, p(tokens), p(state_in), p(state_out), p(logits), p(routes),
                                        p(acc), stream)
        check(code, "ygg_step")

    def _step(self, x, h):
        torch = _torch()
        out = torch.empty_like(h)
        logits = torch.empty((x.shape[0], self.vocab), dtype=torch.float32, device=h.device)
        code = lib().ygg_step(self._h, x.shape[0], x.data_ptr(), h.data_ptr(), out.data_ptr(), logits.data_ptr(),
                              _raw_stream(self._dix))
        if code:
            check(code, "ygg_step")
        return logits, out

    def step(self, tokens, state):
        """One token per stream: tokens (B,) -> logits (B, classes) of the next token, and the new state."""
        torch = _torch()
        if not self.cuda_graph and type(tokens) is torch.Tensor and type(state) is torch.Tensor \
                and tokens.dtype is torch.int32 and state.dtype is torch.int8 and tokens.get_device() == self._dix \
                and state.get_device() == self._dix and tokens.dim() == 1 and tokens.is_contiguous() \
                and state.is_contiguous() and state.shape[0] == tokens.shape[0] and state.shape[1:] == self._state_shape:
            return self._step(tokens, state)   # device tokens and state as they are: no device switch, no copies
        with torch.cuda.device(self.device):
            x = self._tokens(tokens)
            state = self._check_state(state, x.shape[0])
            if not self.cuda_graph:
                return self._step(x, state)
            b = x.shape[0]
            if b not in self._graphs:
                sx, sh = torch.zeros(b, dtype=torch.int32, device=self.device), self.init_state(b)
                self._step(sx, sh)   # warm the launch path before the capture
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

    def step_debug(self, tokens, state):
        """step that also returns the leaf of every layer (B, layers) and the int32 accumulators before saturation
        (B, layers, n), for bit-exact checks against the reference kernel."""
        torch = _torch()
        with torch.cuda.device(self.device):
            x = self._tokens(tokens)
            state = self._check_state(state, x.shape[0])
            b = x.shape[0]
            out = torch.empty_like(state)
            logits = torch.empty(b, self.vocab, dtype=torch.float32, device=self.device)
            routes = torch.empty(b, self.layers, dtype=torch.int32, device=self.device)
            acc = torch.empty(b, self.layers, self.n, dtype=torch.int32, device=self.device)
            self.step_into(x, state, out, logits, routes, acc)
            return logits, out, routes, acc

    # ------------------------------------------------------------------------------------------------ score

    def score_into(self, tokens, state, bits):
        """One fused score launch into caller buffers: tokens int32 (B, T) device tensor, state int8 (B, L, n) or
        None (zero, not written back), bits float64 (B,)."""
        torch = _torch()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(lib().ygg_score(self._h, tokens.shape[0], tokens.shape[1], ctypes.c_void_p(tokens.data_ptr()),
                              ctypes.c_void_p(state.data_ptr()) if state is not None else None,
                              ctypes.c_void_p(bits.data_ptr()), ctypes.c_void_p(stream)), "ygg_score")

    def score_grouped_into(self, tokens, state, bits, min_group=32):
        """score_into through the grouped path: per step and layer the streams are bucketed by leaf and leaves with
        at least min_group streams run as int8 tensor-core GEMMs. Allocates the workspace with torch."""
        torch = _torch()
        b = tokens.shape[0]
        nbytes = lib().ygg_score_grouped_workspace(self._h, b)
        ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=self.device)
        base = ws.data_ptr()
        base += (-base) % 256
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(lib().ygg_score_grouped(self._h, b, tokens.shape[1], ctypes.c_void_p(tokens.data_ptr()),
                                      ctypes.c_void_p(state.data_ptr()) if state is not None else None,
                                      ctypes.c_void_p(bits.data_ptr()), int(min_group), ctypes.c_void_p(base),
                                      nbytes, ctypes.c_void_p(stream)), "ygg_score_grouped")

    def score(self, tokens, state=None, batch=1024, grouped=False, min_group=32):
        """Bits of tokens[:, 1:] given the tokens before them, per row of tokens (B, L), as float64 (B,).
        Rows start from state, or from zero; bits per token = score(tokens).sum() / (B (L - 1)).
        One fused launch per batch of rows: the state and the logits stay on chip across the whole row.
        grouped=True: the leaf-grouped path instead (tensor-core GEMMs for leaves shared by >= min_group streams);
        same bits."""
        torch = _torch()
        with torch.cuda.device(self.device):
            if isinstance(tokens, torch.Tensor) and tokens.is_cuda:
                tok = tokens.to(torch.int32)
                tok = tok[None] if tok.dim() == 1 else tok
            else:
                tok = self._tokens(np.atleast_2d(np.asarray(tokens.cpu() if isinstance(tokens, torch.Tensor)
                                                            else tokens)))
            tok = tok.contiguous()
            rows, steps = tok.shape
            out = []
            stream = torch.cuda.current_stream(self.device).cuda_stream
            for i in range(0, rows, batch):
                x = tok[i:i + batch].contiguous()
                st = None if state is None else self._check_state(state[i:i + batch], x.shape[0]).clone()
                bits = torch.empty(x.shape[0], dtype=torch.float64, device=self.device)
                if grouped:
                    self.score_grouped_into(x, st, bits, min_group)
                else:
                    check(lib().ygg_score(self._h, x.shape[0], steps, ctypes.c_void_p(x.data_ptr()),
                                          ctypes.c_void_p(st.data_ptr()) if st is not None else None,
                                          ctypes.c_void_p(bits.data_ptr()), ctypes.c_void_p(stream)), "ygg_score")
                out.append(bits)
            res = torch.cat(out).cpu().numpy() if out else np.zeros(0, np.float64)
            self.status()
            return res

    # ------------------------------------------------------------------------------------------------ generate

    def generate(self, prompt, n, temperature=1.0, top_k=0, seed=0):
        """Prompt (L,) or (B, L), L >= 1, followed by n sampled tokens. temperature 0: greedy
        (yggdrasil/inference_triton.py:229-248). Sampling draws from torch's generator seeded with `seed`, as the
        reference's Triton backend does; the reference's JAX backend draws from a JAX PRNG key instead
        (yggdrasil/inference.py:190-202), so for the same seed the sampled tokens differ from that backend's. Greedy
        decoding (temperature 0) equals the reference's on the same model."""
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
