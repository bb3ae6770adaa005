"""Failure detection without a GPU fault: every spin-wait of the persistent
kernels is bounded and reports through an error word. Here a wait that nothing
satisfies (an mbarrier with no arrival, a grid counter nobody increments) runs
out after a short limit, the status comes back, and the same context then runs
a normal kernel correctly."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from gpu_util import dev, empty, host, ptr, rel_l2, sync  # noqa: E402
from xpose_b200._lib import check, lib  # noqa: E402

TK_ERR_GRID_BAR, TK_ERR_MBAR = 2, 4


def test_waits_time_out_into_a_status():
    err = C.c_uint32(0)
    check(lib().xp_selftest_wait_timeout(2000, C.byref(err)))
    assert err.value & TK_ERR_MBAR
    assert err.value & TK_ERR_GRID_BAR
    # the context is still usable
    rows, cols = 1152, 256
    w = O.gen_normal(4, 1, rows * cols, 0.02)
    x = O.gen_normal(4, 2, rows, 1.0)
    words, scales = O.pack(w, rows, cols)
    out = empty(cols)
    check(lib().xp_mv_km4_bs(None, ptr(out), ptr(dev(x)), ptr(dev(words)), ptr(dev(scales)), rows, cols))
    sync()
    assert rel_l2(host(out), O.mv(x, words, scales, rows, cols)) < 1e-5


def test_session_error_word_is_clear_after_decoding():
    from xpose_b200.decode import DecodeConfig, DecodeSession, Sampling
    s = DecodeSession.random(DecodeConfig(n_layers=2, vocab=32768, max_seq=64), Sampling(greedy=True), seed=1)
    s.prefill(np.arange(4, dtype=np.uint32))
    s.generate(4)
    assert s.error_word() == 0
