"""GPU parity of the sm_100a kernels against the CPU oracle (oracle/xp_oracle.c),
called through the C ABI (include/xp_cuda.h). Tolerances follow BASELINE's bar:
bit-exact for integer/packing work, <= 1e-3 relative L2 for fp32 outputs
(measured values are ~1e-6), plus the reference matvec selftest's error
relative to the output RMS (examples/llm/decode.cpp:2543-2561)."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from gpu_util import dev, empty, host, ptr, rel_l2, sync  # noqa: E402
from xpose_b200._lib import check, lib  # noqa: E402

# examples/llm/decode.cpp:2461-2464: the real per-token shapes plus the LM head
SHAPES = [(1152, 1024), (1152, 256), (1024, 1152), (1152, 6912), (6912, 1152), (1152, 8192)]


def test_gen_normal_bitexact():
    n = 1 << 20
    t = empty(n)
    check(lib().xp_gen_normal(None, ptr(t), n, 123, 7, 99, 0.02))
    sync()
    want = O.gen_normal(7, 99, n, 0.02, offset=123)
    assert np.array_equal(host(t).view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("rows,cols", [(1152, 6912), (128, 64), (6912, 1152)])
def test_pack_bitexact(rows, cols):
    w = O.gen_normal(3, 11, rows * cols, 0.02)
    w[:32] = 0.0          # an all-zero block (scale 0)
    w[64:96] *= 1e4       # a block with a large range
    words, scales = O.pack(w, rows, cols)
    dw, ds = empty(rows * cols // 8, torch.int32), empty(rows * cols // 64, torch.int32)
    check(lib().xp_pack_km4bf16(None, ptr(dev(w)), rows, cols, ptr(dw), ptr(ds)))
    sync()
    assert np.array_equal(host(dw, np.uint32), words)
    assert np.array_equal(host(ds, np.uint32), scales)


def _mv_case(rows, cols, seed=0):
    w = O.gen_normal(seed, 1, rows * cols, 0.02)
    x = O.gen_normal(seed, 2, rows, 1.0)
    words, scales = O.pack(w, rows, cols)
    return x, words, scales, O.mv(x, words, scales, rows, cols)


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_mv_km4_bs(rows, cols):
    x, words, scales, want = _mv_case(rows, cols)
    out = torch.full((cols,), -1e30, device="cuda")  # sentinel: every output must be written
    check(lib().xp_mv_km4_bs(None, ptr(out), ptr(dev(x)), ptr(dev(words)), ptr(dev(scales)), rows, cols))
    sync()
    got = host(out)
    assert np.all(got != -1e30)
    rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
    assert np.max(np.abs(got - want)) / rms < 1e-4
    assert rel_l2(got, want) < 1e-5


def test_mv_km4_bs_split_reduce():
    rows, cols, split = 1152, 1024, 4
    x, words, scales, want = _mv_case(rows, cols, seed=5)
    part = empty(split * cols)
    out = empty(cols)
    check(lib().xp_mv_km4_bs_split(None, ptr(part), ptr(dev(x)), ptr(dev(words)), ptr(dev(scales)), rows, cols,
                                   split))
    check(lib().xp_mv_reduce(None, ptr(out), ptr(part), cols, split))
    sync()
    # partition p covers quads [3p, 3p+3) (9 quads over 4 splits: 3/3/3/0)
    p = host(part).reshape(split, cols)
    assert np.all(p[3] == 0.0)
    assert rel_l2(host(out), want) < 1e-5


def test_mv_special_values():
    """Zero blocks, huge and tiny activations, all-zero input."""
    rows, cols = 1152, 256
    w = O.gen_normal(9, 1, rows * cols, 0.02)
    w[: rows * 3] = 0.0
    words, scales = O.pack(w, rows, cols)
    for x in (np.zeros(rows, np.float32), O.gen_normal(9, 2, rows, 1e-20), O.gen_normal(9, 3, rows, 1e20)):
        want = O.mv(x, words, scales, rows, cols)
        out = empty(cols)
        check(lib().xp_mv_km4_bs(None, ptr(out), ptr(dev(x)), ptr(dev(words)), ptr(dev(scales)), rows, cols))
        sync()
        got = host(out)
        if not np.any(want):
            assert not np.any(got)
        else:
            assert rel_l2(got, want) < 1e-5
