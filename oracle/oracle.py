"""TEST INFRASTRUCTURE ONLY: ctypes wrapper of the C restatement of the reference int8 step (oracle/ygg_oracle.c)
and a runner for the reference's own binary (oracle/_ref/ygg, built by oracle/Makefile from cpu/ygg.cpp).

Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` use this module, as the checker
of the CUDA path. The product (``yggdrasil_b200``) never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_YGG = HERE / "_ref" / "ygg"

_lib = None


def build(quiet: bool = True) -> None:
    """Compile liboracle.so (and _ref/ygg when the reference tree is mounted)."""
    out = subprocess.run(["make", "-C", str(HERE), "all"], capture_output=True, text=True)
    if out.returncode:
        raise RuntimeError(f"oracle build failed:\n{out.stdout}\n{out.stderr}")
    if not quiet:
        print(out.stdout)


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        l = ctypes.CDLL(str(LIB))
        l.orc_load.restype = ctypes.c_void_p
        l.orc_load.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_int]
        l.orc_free.argtypes = [ctypes.c_void_p]
        l.orc_info.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        l.orc_step.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                               ctypes.c_void_p, ctypes.c_void_p]
        l.orc_logits.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                 ctypes.c_void_p, ctypes.c_void_p]
        l.orc_score.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                ctypes.c_void_p]
        for f in (l.orc_step, l.orc_logits, l.orc_score):
            f.restype = ctypes.c_int
        _lib = l
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


class OracleModel:
    """The C oracle over one YGG1 file (path or bytes)."""

    def __init__(self, model):
        data = Path(model).read_bytes() if isinstance(model, (str, Path)) else bytes(model)
        err = ctypes.create_string_buffer(256)
        self._h = lib().orc_load(data, len(data), err, 256)
        if not self._h:
            raise ValueError(f"oracle: {err.value.decode()}")
        info = np.zeros(12, np.int32)
        lib().orc_info(self._h, _ptr(info))
        (self.n_layers, self.n, self.block, self.vocab, self.depth, self.readout_rank, self.layer_input_rank,
         self.input_rank, self.shift, self.n_experts, self.vocab_pad, factored) = (int(v) for v in info)
        self.factored = bool(factored)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_free(self._h)
            self._h = None

    def init_state(self, batch: int) -> np.ndarray:
        return np.zeros((batch, self.n_layers, self.n), np.int8)

    def step(self, tokens, state, routes: bool = False, acc: bool = False):
        """tokens (B,), state (B, L, n) int8 (updated in place) -> logits (B, V) f32 [, routes (B, L)] [, acc (B, L, n)
        int32: the accumulators before saturation to the new state]."""
        tok = np.ascontiguousarray(tokens, np.int32)
        assert state.dtype == np.int8 and state.flags.c_contiguous and state.shape == (len(tok), self.n_layers, self.n)
        lg = np.empty((len(tok), self.vocab), np.float32)
        rt = np.empty((len(tok), self.n_layers), np.int32) if routes else None
        ac = np.empty((len(tok), self.n_layers, self.n), np.int32) if acc else None
        if lib().orc_step(self._h, len(tok), _ptr(tok), _ptr(state), _ptr(lg), _ptr(rt), _ptr(ac)):
            raise ValueError("token out of range")
        out = (lg,) + ((rt,) if routes else ()) + ((ac,) if acc else ())
        return out if len(out) > 1 else lg

    def logits(self, tokens, routes: bool = False, acc: bool = False):
        """windows (S, T), zero state per window -> logits (S, T, V) f32 [, routes (S, T, L)] [, acc (S, T, L, n) int32
        before saturation]."""
        tok = np.ascontiguousarray(tokens, np.int32)
        s, t = tok.shape
        lg = np.empty((s, t, self.vocab), np.float32)
        rt = np.empty((s, t, self.n_layers), np.int32) if routes else None
        ac = np.empty((s, t, self.n_layers, self.n), np.int32) if acc else None
        if lib().orc_logits(self._h, s, t, _ptr(tok), _ptr(lg), _ptr(rt), _ptr(ac)):
            raise ValueError("token out of range")
        out = (lg,) + ((rt,) if routes else ()) + ((ac,) if acc else ())
        return out if len(out) > 1 else lg

    def score(self, tokens, state=None):
        """bits of tokens[:, 1:] per row (f64); state (S, L, n) int8 updated in place, or None (zero)."""
        tok = np.ascontiguousarray(np.atleast_2d(tokens), np.int32)
        s, t = tok.shape
        bits = np.empty(s, np.float64)
        if lib().orc_score(self._h, s, t, _ptr(tok), _ptr(state), _ptr(bits)):
            raise ValueError("token out of range")
        return bits


def ref_available() -> bool:
    return REF_YGG.exists() and os.access(REF_YGG, os.X_OK)


def ref_logits(model_path, tokens, tmpdir) -> np.ndarray:
    """The reference binary's logits command (cpu/ygg.cpp:500-525) on windows tokens (S, T)."""
    tok = np.ascontiguousarray(tokens, np.int32)
    xf, of = os.path.join(tmpdir, "x.i32"), os.path.join(tmpdir, "o.f32")
    tok.tofile(xf)
    subprocess.run([str(REF_YGG), "logits", str(model_path), xf, str(tok.shape[0]), str(tok.shape[1]), of],
                   check=True, stdout=subprocess.DEVNULL)
    return np.fromfile(of, np.float32).reshape(tok.shape[0], tok.shape[1], -1)
