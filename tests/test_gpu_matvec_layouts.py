"""The layout-study matvecs the reference keeps beside its shipped kernel
(kernels/llm_matvec.cl:79-366: mv_ref, mv_ref_split, mv_kmn, mv_km, mv_km4 and
its work-group / column-blocking / split-k variants) and the first matvec
module (kernels/llm.cl: matvec_f32, matvec_q4, matvec_q4_split, matvec_reduce,
stream_read), launched through the registry and compared with the
reference's own kernels compiled for the host (oracle/_ref) on random packed
planes. The per-block sums are formed in the same order; blocks are summed in
another order here, so outputs agree to fp32 rounding (rtol 1e-5 of the
output scale); the integer probe is exact. matvec_bench.cpp, the reference's
harness for these kernels, runs unchanged on the drop-in."""
import os
import subprocess

import numpy as np
import pytest

import oracle_lib as O

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(O.ref() is None, reason="oracle/_ref not built")]
pytest.importorskip("torch")
from xpose_b200.vulkore import Context, Grid, Program, launch  # noqa: E402

ROWS, COLS = 1152, 1024
MV, LLM = "kernels/llm_matvec.spv", "kernels/llm.spv"
CASES = [  # (module, name, split, reference grid)
    (MV, "mv_ref", 0, COLS), (MV, "mv_ref_split", 4, COLS * 4), (MV, "mv_kmn", 0, COLS), (MV, "mv_km", 0, COLS),
    (MV, "mv_km4", 0, COLS), (MV, "mv_km4_wg32", 0, COLS), (MV, "mv_km4_wg128", 0, COLS),
    (MV, "mv_km4_wg256", 0, COLS), (MV, "mv_km4_c2", 0, COLS // 2), (MV, "mv_km4_c2_wg32", 0, COLS // 2),
    (MV, "mv_km4_c4", 0, COLS // 4), (MV, "mv_km4_split", 8, COLS * 8), (LLM, "matvec_q4", 0, COLS),
    (LLM, "matvec_q4_split", 3, COLS * 3),
]


@pytest.fixture(scope="module")
def ctx():
    return Context()


def buf(ctx, a):
    b = ctx.alloc(len(a), a.dtype)
    b.upload(a)
    return b


@pytest.mark.parametrize("module,name,split,grid", CASES)
def test_layout_matvec_matches_reference(ctx, module, name, split, grid):
    rng = np.random.default_rng(len(name) * 31 + split)
    words = rng.integers(0, 2**32, ROWS * COLS // 8, dtype=np.uint32)
    scales = rng.uniform(0.001, 0.02, (ROWS // 32) * COLS).astype(np.float32)
    x = rng.uniform(-1, 1, ROWS).astype(np.float32)
    n_out = COLS * (split or 1)
    want = np.zeros(n_out, np.float32)
    args = (x, words, scales, ROWS, COLS) + ((split,) if split else ())
    O.ref_launch(name, grid, want, *args, module=module)
    out = ctx.alloc(n_out)
    launch(Program.from_file(ctx, module).kernel(name), Grid(grid), out, buf(ctx, x), buf(ctx, words),
           buf(ctx, scales), ROWS, COLS, *((split,) if split else ()), stream=ctx.stream)
    ctx.wait_idle()
    got = out.download()
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-5 * np.abs(want).max())


def test_llm_module_f32_matvec_reduce_and_probe(ctx):
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.02, ROWS * COLS).astype(np.float32)
    x = rng.uniform(-1, 1, ROWS).astype(np.float32)
    want = np.zeros(COLS, np.float32)
    O.ref_launch("matvec_f32", COLS, want, x, w, ROWS, COLS, module=LLM)
    prog = Program.from_file(ctx, LLM)
    out = ctx.alloc(COLS)
    launch(prog.kernel("matvec_f32"), Grid(COLS), out, buf(ctx, x), buf(ctx, w), ROWS, COLS, stream=ctx.stream)
    ctx.wait_idle()
    np.testing.assert_allclose(out.download(), want, rtol=0, atol=1e-5 * np.abs(want).max())
    part = rng.normal(0, 1, 3 * COLS).astype(np.float32)
    red_want = np.zeros(COLS, np.float32)
    O.ref_launch("matvec_reduce", COLS, red_want, part, COLS, 3, module=LLM)
    launch(prog.kernel("matvec_reduce"), Grid(COLS), out, buf(ctx, part), COLS, 3, stream=ctx.stream)
    ctx.wait_idle()
    assert np.array_equal(out.download(), red_want)
    src = rng.integers(0, 2**20, 1 << 20, dtype=np.uint32)
    probe_want = np.zeros(1, np.float32)
    O.ref_launch("stream_read", 65536, probe_want, src, len(src), module=LLM)
    launch(prog.kernel("stream_read"), Grid(65536), out, buf(ctx, src), len(src), stream=ctx.stream)
    ctx.wait_idle()
    assert out.download()[0] == probe_want[0]


def test_matvec_bench_harness_runs():
    exe = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                       "matvec_bench_gpu")
    if not os.path.exists(exe):
        pytest.skip("matvec_bench_gpu not built")
    p = subprocess.run(["stdbuf", "-oL", exe, "kernels/llm.spv", "kernels/llm_matvec.spv", "--quick"],
                       capture_output=True, text=True, timeout=600, cwd=os.path.dirname(exe))
    assert p.returncode == 0, (p.stdout + p.stderr)[-3000:]
    assert "FAIL" not in p.stdout, p.stdout[-3000:]
