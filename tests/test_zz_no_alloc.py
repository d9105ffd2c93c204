"""The allocation-free grouped score (ygg_score_grouped_noalloc), called through the C-ABI (GPU).

Some callers cannot allocate device memory while they run: a host whose own pool owns the GPU's memory, a serving
loop that forbids allocation on its hot path, a binding with no CUDA allocator. The entry point serves them with a
fixed scratch array that the library holds on each GPU, instead of a workspace the caller passes. Its results must
equal those of the workspace entry point (ygg_score_grouped): the bits within the tolerance of the other score tests
(rtol 1e-10; they are in fact identical) and the final states exactly. Two calls in a row with different tokens check
that each call starts from a clean scratch, since the array keeps the last call's contents. The file is named to be
collected last, and it needs nothing from the tests before it.
"""
import ctypes

import numpy as np
import pytest

from conftest import golden

pytestmark = pytest.mark.gpu

BITS_RTOL = 1e-10
CAPACITY = 16 << 20


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


NO_ALLOC_CASES = [golden("kernel_cases.json")[0], [r for r in golden("extended_cases.json") if "shape" in r][0]]


@pytest.mark.parametrize("rec", NO_ALLOC_CASES, ids=["n128", "ext-n96"])
def test_no_alloc_equals_workspace_entry_on_two_calls(rec, case_model):
    """n128, and a d_state 96 model, whose padded state copy (the grouped path pads the caller's 96 coordinates to
    the device layout's 128) also lives in the fixed scratch: with a carried state and with a zero start state."""
    import torch

    from yggdrasil_b200 import Yggdrasil, _native
    lib = _native.lib()
    model = Yggdrasil.load(case_model(rec), backend="b200")
    dev, v = model.device, rec["shape"]["vocab"]
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for call, (rows, steps, min_group) in enumerate([(300, 10, 2), (257, 7, 1)]):
        x = torch.as_tensor(np.random.default_rng(100 + call).integers(0, v, (rows, steps)).astype(np.int32),
                            device=dev)
        start = torch.as_tensor(np.random.default_rng(200 + call).integers(-60, 61, (rows, model.layers, model.n)),
                                dtype=torch.int8, device=dev)
        ref_bits = torch.empty(rows, dtype=torch.float64, device=dev)
        ref_state = start.clone()
        model.score_grouped_into(x, ref_state, ref_bits, min_group=min_group)
        bits = torch.full((rows,), -1.0, dtype=torch.float64, device=dev)
        state = start.clone()
        rc = lib.ygg_score_grouped_noalloc(model._h, rows, steps, _ptr(x), _ptr(state), _ptr(bits), min_group,
                                           stream)
        assert rc == _native.YGG_OK, _native.strerror(rc)
        torch.cuda.synchronize(dev)
        np.testing.assert_allclose(bits.cpu().numpy(), ref_bits.cpu().numpy(), rtol=BITS_RTOL)
        assert torch.equal(state, ref_state), f"call {call}: final states differ"
        # the same with the zero start state the call makes for itself
        bits0 = torch.empty(rows, dtype=torch.float64, device=dev)
        rc = lib.ygg_score_grouped_noalloc(model._h, rows, steps, _ptr(x), None, _ptr(bits0), min_group, stream)
        assert rc == _native.YGG_OK, _native.strerror(rc)
        ref0 = torch.empty_like(bits0)
        model.score_grouped_into(x, None, ref0, min_group=min_group)
        torch.cuda.synchronize(dev)
        np.testing.assert_allclose(bits0.cpu().numpy(), ref0.cpu().numpy(), rtol=BITS_RTOL)
    model.status()


def test_no_alloc_refuses_a_batch_beyond_its_scratch(case_model):
    import torch

    from yggdrasil_b200 import Yggdrasil, _native
    lib = _native.lib()
    rec = golden("kernel_cases.json")[0]
    model = Yggdrasil.load(case_model(rec), backend="b200")
    rows = 1024
    while lib.ygg_score_grouped_workspace(model._h, rows) <= CAPACITY:
        rows *= 2
    x = torch.zeros((rows, 2), dtype=torch.int32, device=model.device)
    bits = torch.empty(rows, dtype=torch.float64, device=model.device)
    rc = lib.ygg_score_grouped_noalloc(model._h, rows, 2, _ptr(x), None, _ptr(bits), 4,
                                       ctypes.c_void_p(torch.cuda.current_stream(model.device).cuda_stream))
    assert rc == _native.YGG_E_CAPACITY
    assert "scratch" in _native.strerror(rc)
