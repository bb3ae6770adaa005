"""Many matvecs in one launch (xp_mv_plan_*): every job's output must match
the oracle restatement of kernels/llm_matvec.cl:422-434 and the single-matvec
entry point xp_mv_km4_bs on the same planes, within the fp32 bar (<= 1e-5
relative L2, measured ~1e-6), with shared and distinct inputs, mixed K (1152 and
6912), and on a second run of the same plan."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from gpu_util import dev, empty, host, ptr, rel_l2, sync  # noqa: E402
from xpose_b200._lib import XpError, check, lib  # noqa: E402


class Job(C.Structure):
    _fields_ = [("out", C.c_void_p), ("inp", C.c_void_p), ("wq", C.c_void_p), ("sc", C.c_void_p),
                ("rows", C.c_uint32), ("cols", C.c_uint32)]


def _case(rows, cols, seed):
    w = O.gen_normal(seed, 1, rows * cols, 0.02)
    words, scales = O.pack(w, rows, cols)
    return words, scales


def test_plan_matches_oracle_and_single_matvec():
    xa = O.gen_normal(3, 2, 1152, 1.0)
    xb = O.gen_normal(3, 3, 6912, 1.0)
    xc = O.gen_normal(3, 4, 1152, 1e-3)
    shapes = [(1152, 1024, xa), (1152, 256, xa), (6912, 1152, xb), (1152, 6912, xc), (1152, 64, xa)]
    dx = {id(x): dev(x) for x in (xa, xb, xc)}
    jobs, outs, wants, planes = [], [], [], []
    for i, (rows, cols, x) in enumerate(shapes):
        words, scales = _case(rows, cols, 10 + i)
        dw, ds = dev(words), dev(scales)
        out = torch.full((cols,), -1e30, device="cuda")
        jobs.append(Job(ptr(out), ptr(dx[id(x)]), ptr(dw), ptr(ds), rows, cols))
        outs.append(out)
        planes.append((dw, ds))
        wants.append(O.mv(x, words, scales, rows, cols))
    arr = (Job * len(jobs))(*jobs)
    plan = C.c_void_p()
    check(lib().xp_mv_plan_create(C.cast(arr, C.c_void_p), len(jobs), C.byref(plan)))
    try:
        nbytes = C.c_uint64()
        check(lib().xp_mv_plan_bytes(plan, C.byref(nbytes)))
        assert nbytes.value == sum(r * c // 2 + r * c // 16 + 4 * r + 4 * c for r, c, _ in shapes)
        for rep in range(2):
            if rep:
                for o in outs:
                    o.fill_(-1e30)
            check(lib().xp_mv_plan_run(plan, None))
            sync()
            for (rows, cols, x), out, want, (dw, ds) in zip(shapes, outs, wants, planes):
                got = host(out)
                assert np.all(got != -1e30)
                assert rel_l2(got, want) < 1e-5, (rows, cols)
                single = empty(cols)
                check(lib().xp_mv_km4_bs(None, ptr(single), ptr(dx[id(x)]), ptr(dw), ptr(ds), rows, cols))
                sync()
                assert rel_l2(got, host(single)) < 1e-5
    finally:
        lib().xp_mv_plan_destroy(plan)


def test_plan_rejects_bad_shapes():
    t = empty(128)
    bad = (Job * 1)(Job(ptr(t), ptr(t), ptr(t), ptr(t), 100, 64))
    plan = C.c_void_p()
    with pytest.raises(XpError) as e:
        check(lib().xp_mv_plan_create(C.cast(bad, C.c_void_p), 1, C.byref(plan)))
    assert e.value.name == "XP_ERR_INVALID"
    assert not plan.value
