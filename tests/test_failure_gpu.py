"""Failure detection on the GPU without a GPU fault (GPU).

Every device wait of the kernels is bounded; one that runs out makes the kernel return with an error status that the
host reads, and the context stays usable. Here the library's wait self test makes such a wait run out (an mbarrier
that nothing completes, a limit of a few milliseconds); afterwards a model still loads and steps exactly.
"""
import ctypes

import numpy as np
import pytest

from conftest import case_tokens, golden

from oracle import oracle as O

pytestmark = pytest.mark.gpu

CASES = golden("kernel_cases.json")


def test_a_wait_that_runs_out_reports_and_the_context_survives(case_model):
    import torch

    from yggdrasil_b200 import Yggdrasil, _native
    lib = _native.lib()
    status = ctypes.c_int(99)
    stream = torch.cuda.current_stream().cuda_stream
    # ~5 ms at 2 GHz: the wait on an mbarrier nothing completes gives up and reports a timeout
    assert lib.ygg_selftest_wait(0, 10_000_000, ctypes.c_void_p(stream), ctypes.byref(status)) == _native.YGG_OK
    assert status.value == _native.YGG_E_TIMEOUT
    # the context is intact: a model loads and steps bit-exact against the oracle
    rec = CASES[0]
    path = case_model(rec)
    model, om = Yggdrasil.load(path, backend="b200"), O.OracleModel(path)
    x = case_tokens(rec)
    st, ost = model.init_state(x.shape[0]), om.init_state(x.shape[0])
    for t in range(4):
        lg, st = model.step(x[:, t], st)
        np.testing.assert_array_equal(lg.cpu().numpy(), om.step(x[:, t], ost))
    model.status()
