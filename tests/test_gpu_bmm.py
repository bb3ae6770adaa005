"""Batched int4 matvec on tcgen05 (xp_mv_km4_bs_batch): every sequence's row
must match the oracle restatement of kernels/llm_matvec.cl:422-434 for that
sequence, and xp_mv_km4_bs on the same planes, within the fp32 bar (the
activation enters as two fp16 halves, ~22 bits; measured error ~1e-6 relative
L2; bound 1e-5). Covers K split across CTAs (rows 6912), one K range (rows
1152 over many tiles), 1..64 sequences (padding to 32/64) and a second call
on the same scratch."""
import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from gpu_util import dev, empty, host, ptr, rel_l2, sync  # noqa: E402
from xpose_b200._lib import XpError, check, lib  # noqa: E402


def _run(rows, cols, n, seed):
    w = O.gen_normal(seed, 1, rows * cols, 0.02)
    words, scales = O.pack(w, rows, cols)
    xs = np.stack([O.gen_normal(seed, 100 + s, rows, 1.0 + 3.0 * (s % 3)) for s in range(n)])
    dw, ds, dx = dev(words), dev(scales), dev(xs.reshape(-1))
    nbytes = lib().xp_mv_km4_bs_batch_scratch_bytes(rows, cols, n)
    assert nbytes > 0
    scratch = torch.zeros(nbytes // 4 + 64, dtype=torch.int32, device="cuda")
    out = torch.full((n * cols,), -1e30, device="cuda")
    for rep in range(2):
        out.fill_(-1e30)
        check(lib().xp_mv_km4_bs_batch(None, ptr(out), ptr(dx), ptr(dw), ptr(ds), rows, cols, n, ptr(scratch)))
        sync()
        assert int(host(scratch, np.uint32)[64]) == 0, "pipeline wait ran out"
        got = host(out).reshape(n, cols)
        for s in (0, n // 2, n - 1):
            want = O.mv(xs[s], words, scales, rows, cols)
            assert rel_l2(got[s], want) < 1e-5, (rows, cols, n, s, rel_l2(got[s], want))
        one = empty(cols)
        check(lib().xp_mv_km4_bs(None, ptr(one), ptr(dev(xs[n - 1])), ptr(dw), ptr(ds), rows, cols))
        sync()
        assert rel_l2(got[n - 1], host(one)) < 1e-5


@pytest.mark.parametrize("rows,cols,n", [(1152, 1024, 64), (6912, 1152, 64), (1152, 6912, 40), (1024, 1152, 1),
                                         (1152, 256, 17)])
def test_batch_matches_oracle(rows, cols, n):
    _run(rows, cols, n, seed=7 + n)


def test_batch_rejects_bad_shapes():
    t = empty(1024)
    with pytest.raises(XpError):
        check(lib().xp_mv_km4_bs_batch(None, ptr(t), ptr(t), ptr(t), ptr(t), 1152, 1000, 4, ptr(t)))
    with pytest.raises(XpError):
        check(lib().xp_mv_km4_bs_batch(None, ptr(t), ptr(t), ptr(t), ptr(t), 1152, 1024, 65, ptr(t)))
    assert lib().xp_mv_km4_bs_batch_scratch_bytes(1152, 1024, 0) == 0


def test_batch_scratch_shared_across_shapes():
    """One scratch, zeroed once, used by a K-split shape, another K-split shape
    whose activations land where the first keeps its sums, then the first
    again: every call must still match the oracle (the library clears the
    sums when a scratch changes shape)."""
    shapes = [(6912, 1152, 64), (1152, 1024, 64), (6912, 1152, 64), (1152, 6912, 40)]
    need = max(lib().xp_mv_km4_bs_batch_scratch_bytes(r, c, n) for r, c, n in shapes)
    scratch = torch.zeros(need // 4 + 64, dtype=torch.int32, device="cuda")
    for i, (rows, cols, n) in enumerate(shapes):
        w = O.gen_normal(40 + i, 1, rows * cols, 0.02)
        words, scales = O.pack(w, rows, cols)
        xs = np.stack([O.gen_normal(40 + i, 100 + s, rows, 1.0) for s in range(n)])
        out = torch.full((n * cols,), -1e30, device="cuda")
        check(lib().xp_mv_km4_bs_batch(None, ptr(out), ptr(dev(xs.reshape(-1))), ptr(dev(words)), ptr(dev(scales)),
                                       rows, cols, n, ptr(scratch)))
        sync()
        got = host(out).reshape(n, cols)
        for s in (0, n - 1):
            want = O.mv(xs[s], words, scales, rows, cols)
            assert rel_l2(got[s], want) < 1e-5, (i, rows, cols, s, rel_l2(got[s], want))


@pytest.mark.parametrize("tiny", [False, True])
def test_batch_operand_modes(tiny):
    """Scaled operand mode (every bf16 scale in [2^-14, 8160]: the dequantised
    weight is an exact fp16) and the integer mode the kernel falls back to when
    one block's scale is below 2^-14 (here one 32-row block of weights near
    1e-7): both must match the oracle at the same bar."""
    rows, cols, n = 1152, 1024, 64
    w = O.gen_normal(91, 1, rows * cols, 0.02).reshape(cols, rows)  # [cols][rows]
    if tiny:
        w[5, 32:64] *= 5e-6
    words, scales = O.pack(w.reshape(-1), rows, cols)
    xs = np.stack([O.gen_normal(91, 100 + s, rows, 1.0) for s in range(n)])
    nbytes = lib().xp_mv_km4_bs_batch_scratch_bytes(rows, cols, n)
    scratch = torch.zeros(nbytes // 4 + 64, dtype=torch.int32, device="cuda")
    out = torch.full((n * cols,), -1e30, device="cuda")
    check(lib().xp_mv_km4_bs_batch(None, ptr(out), ptr(dev(xs.reshape(-1))), ptr(dev(words)), ptr(dev(scales)),
                                   rows, cols, n, ptr(scratch)))
    sync()
    sc = host(scratch, np.uint32)
    assert int(sc[64]) == 0, "pipeline wait ran out"
    assert int(sc[96]) == (1 if tiny else 0), "scale-range flag of the call"
    got = host(out).reshape(n, cols)
    for s in (0, 31, n - 1):
        want = O.mv(xs[s], words, scales, rows, cols)
        assert rel_l2(got[s], want) < 1e-5, (tiny, s, rel_l2(got[s], want))
