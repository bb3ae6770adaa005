"""The reference's prefill-shape entry points (kernels/llm_sampling.cl:495-736)
through the kernel registry (Program::kernel by name + launch / Batch), on the
cases of the reference's own harness examples/llm/sampling_test.cpp:725-1020:
T = 37 rows (not a multiple of 64), 4 q-heads / 1 kv-head of 256, hidden 1152.
Outputs are compared with the pinned oracle under the harness's own
numpy-allclose rule (|gpu - cpu| <= 1e-6 + 1e-4 |cpu|, masked -inf entries
equal), outputs start as a -1e30 sentinel that must be overwritten, and the
two equivalences the harness checks hold here exactly: prefill scores at one
query equal the decode `attention_scores`, and `rope_prefill` equals the
decode `rope` row by row."""
import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu
pytest.importorskip("torch")
from xpose_b200.vulkore import Batch, Context, Grid, Program, launch  # noqa: E402

T, NH, KVH, HD, H = 37, 4, 1, 256, 1152
SENT = np.float32(-1.0e30)
RNG = np.random.default_rng(20260719)
SCALE = float(np.float32(1.0 / 16))
EPS = float(np.float32(1e-6))


def rand(n):
    return RNG.uniform(-1.5, 1.5, n).astype(np.float32)


def allclose(gpu, cpu, live=True):
    gpu, cpu = np.asarray(gpu), np.asarray(cpu)
    fin = np.isfinite(cpu)
    assert np.array_equal(gpu[~fin], cpu[~fin]), "masked entries differ"
    assert np.isfinite(gpu[fin]).all(), "non-finite output where the oracle is finite"
    if live:
        assert not (gpu == SENT).any(), "an output was never written"
    bad = np.abs(gpu[fin] - cpu[fin]) > 1e-6 + 1e-4 * np.abs(cpu[fin])
    assert not bad.any(), f"{bad.sum()} of {fin.sum()} outside 1e-6 + 1e-4|cpu|"


@pytest.fixture(scope="module")
def env():
    ctx = Context()
    return ctx, Program.from_file(ctx, "kernels/llm_sampling.spv"), Program.from_file(ctx, "kernels/llm_transformer.spv")


def run(ctx, kernel, grid, *args):
    """vulkore::launch(...).wait() on the context's stream."""
    launch(kernel, grid, *args, stream=ctx.stream)
    ctx.wait_idle()


def buf(ctx, a, dtype=np.float32):
    b = ctx.alloc(len(a), dtype)
    b.upload(np.asarray(a, dtype))
    return b


def test_softmax_many_rows(env):
    ctx, prog, _ = env
    rows, cols = NH * T, T
    x = rand(rows * cols)
    dx, ds = buf(ctx, x), buf(ctx, np.full(2 * rows, SENT))
    b = Batch(ctx)
    b.add(prog.kernel("softmax_rows_stats"), Grid(rows), ds, dx, rows, cols)
    b.add(prog.kernel("softmax_rows_apply"), Grid(rows * cols), dx, ds, rows, cols)
    b.submit().wait()
    got = dx.download()
    st = np.zeros(2 * rows, np.float32)
    want = x.copy()
    O.oracle().xo_softmax_rows_stats(st, want, rows, cols)
    O.oracle().xo_softmax_rows_apply(want, st, rows, cols)
    allclose(got, want, live=False)
    assert np.abs(got.reshape(rows, cols).sum(1, dtype=np.float64) - 1.0).max() < 1e-4


@pytest.mark.parametrize("window", [0, 8])
def test_attention_scores_prefill_masks(env, window):
    ctx, prog, _ = env
    nq, nsc, ncache = NH * T * HD, NH * T * T, T * KVH * HD
    q, kc = rand(nq), rand(ncache)
    dq, dk, ds = buf(ctx, q), buf(ctx, kc), buf(ctx, np.full(nsc, SENT))
    run(ctx, prog.kernel("attention_scores_prefill"), Grid(nsc), ds, dq, dk, NH, KVH, HD, T, T, 0, window, SCALE)
    want = np.zeros(nsc, np.float32)
    O.oracle().xo_attention_scores_prefill(want, q, kc, NH, KVH, HD, T, T, 0, window, SCALE)
    allclose(ds.download(), want)
    assert np.isneginf(want).sum() > 0


def test_prefill_attention_block_causal(env):
    """scores -> stats -> apply -> attention_apply_prefill in one Batch, with a
    chunk offset (queries at positions 20..56 over 57 cached rows)."""
    ctx, prog, _ = env
    q_off = 20
    seq = q_off + T
    nq, nsc = NH * T * HD, NH * T * seq
    q, kc, vc = rand(nq), rand(seq * KVH * HD), rand(seq * KVH * HD)
    dq, dk, dv = buf(ctx, q), buf(ctx, kc), buf(ctx, vc)
    ds, dst, do = buf(ctx, np.zeros(nsc)), buf(ctx, np.zeros(2 * NH * T)), buf(ctx, np.full(nq, SENT))
    b = Batch(ctx)
    b.add(prog.kernel("attention_scores_prefill"), Grid(nsc), ds, dq, dk, NH, KVH, HD, T, seq, q_off, 0, SCALE)
    b.add(prog.kernel("softmax_rows_stats"), Grid(NH * T), dst, ds, NH * T, seq)
    b.add(prog.kernel("softmax_rows_apply"), Grid(nsc), ds, dst, NH * T, seq)
    b.add(prog.kernel("attention_apply_prefill"), Grid(nq), do, ds, dv, NH, KVH, HD, T, seq)
    b.submit().wait()
    sc = np.zeros(nsc, np.float32)
    O.oracle().xo_attention_scores_prefill(sc, q, kc, NH, KVH, HD, T, seq, q_off, 0, SCALE)
    st = np.zeros(2 * NH * T, np.float32)
    O.oracle().xo_softmax_rows_stats(st, sc, NH * T, seq)
    O.oracle().xo_softmax_rows_apply(sc, st, NH * T, seq)
    want = np.zeros(nq, np.float32)
    O.oracle().xo_attention_apply_prefill(want, sc, vc, NH, KVH, HD, T, seq)
    allclose(do.download(), want)


def test_prefill_scores_equal_decode_scores(env):
    ctx, prog, tprog = env
    pos = T - 1
    q1, kc = rand(NH * HD), rand(T * KVH * HD)
    dq, dk = buf(ctx, q1), buf(ctx, kc)
    d1, d2 = buf(ctx, np.zeros(NH * T)), buf(ctx, np.zeros(NH * T))
    run(ctx, prog.kernel("attention_scores_prefill"), Grid(NH * T), d1, dq, dk, NH, KVH, HD, 1, T, pos, 0, SCALE)
    run(ctx, tprog.kernel("attention_scores"), Grid(NH * T), d2, dq, dk, NH, KVH, HD, T, SCALE, 0)
    assert np.array_equal(d1.download(), d2.download())


def test_prefill_rmsnorm_rows(env):
    ctx, prog, _ = env
    n = T * H
    x, w = rand(n), rand(H)
    dx, dw, dss, do = buf(ctx, x), buf(ctx, w), buf(ctx, np.zeros(T)), buf(ctx, np.full(n, SENT))
    b = Batch(ctx)
    b.add(prog.kernel("rmsnorm_rows_sumsq"), Grid(T), dss, dx, T, H)
    b.add(prog.kernel("rmsnorm_rows_apply_gemma"), Grid(n), do, dx, dw, dss, T, H, EPS)
    b.submit().wait()
    ss = np.zeros(T, np.float32)
    want = np.zeros(n, np.float32)
    O.oracle().xo_rmsnorm_rows_sumsq(ss, x, T, H)
    O.oracle().xo_rmsnorm_rows_apply_gemma(want, x, w, ss, T, H, 1e-6)
    allclose(do.download(), want)
    nh = T * NH * HD
    x2, w2 = rand(nh), rand(HD)
    d2, dw2, do2 = buf(ctx, x2), buf(ctx, w2), buf(ctx, np.full(nh, SENT))
    run(ctx, prog.kernel("rmsnorm_heads_rows_gemma"), Grid(nh), do2, d2, dw2, T, NH, HD, EPS)
    want2 = np.zeros(nh, np.float32)
    O.oracle().xo_rmsnorm_heads_rows_gemma(want2, x2, w2, T, NH, HD, 1e-6)
    allclose(do2.download(), want2)


@pytest.mark.parametrize("pos0,theta", [(5, 1e6), (8100, 1e4)])
def test_rope_prefill_equals_decode_rope(env, pos0, theta):
    ctx, prog, tprog = env
    per = NH * HD
    x = rand(T * per)
    dx = buf(ctx, x)
    run(ctx, prog.kernel("rope_prefill"), Grid(T * NH * HD // 2), dx, T, NH, HD, pos0, float(theta))
    got = dx.download()
    rows = []
    drow = ctx.alloc(per)
    for t in range(T):
        drow.upload(x[t * per:(t + 1) * per])
        run(ctx, tprog.kernel("rope"), Grid(NH * HD // 2), drow, NH, HD, pos0 + t, float(theta))
        rows.append(drow.download())
    assert np.array_equal(got, np.concatenate(rows))
    assert (got != x).sum() > 0.9 * x.size
    want = x.copy()
    O.oracle().xo_rope_prefill(want, T, NH, HD, pos0, theta)
    np.testing.assert_allclose(got, want, rtol=0, atol=2e-5 if pos0 < 1000 else 2e-3)


def test_prefill_plumbing(env):
    ctx, prog, _ = env
    row, cap, pos0 = KVH * HD, 64, 11
    cache = np.full(row * cap, 7.0, np.float32)
    src = rand(row * T)
    dc, dsrc = buf(ctx, cache), buf(ctx, src)
    run(ctx, prog.kernel("kv_append_rows"), Grid(T * row), dc, dsrc, T, row, pos0)
    want = cache.copy()
    O.oracle().xo_kv_append_rows(want, src, T, row, pos0)
    assert np.array_equal(dc.download(), want)
    vocab = 4096
    table = (np.arange(vocab * H) % 977).astype(np.float32) * np.float32(0.01)
    toks = ((np.arange(T) * 251 + 13) % vocab).astype(np.uint32)
    dt, dtok, do = buf(ctx, table), buf(ctx, toks, np.uint32), buf(ctx, np.full(T * H, SENT))
    run(ctx, prog.kernel("embed_lookup_rows"), Grid(T * H), do, dt, dtok, T, H)
    want = np.zeros(T * H, np.float32)
    O.oracle().xo_embed_lookup_rows(want, table, toks, T, H)
    assert np.array_equal(do.download(), want)


def test_registry_lists_every_prefill_entry_point(env):
    _, prog, _ = env
    names = set(prog.kernel_names())
    for n in ("softmax_rows_stats", "softmax_rows_apply", "attention_scores_prefill", "attention_apply_prefill",
              "rmsnorm_rows_sumsq", "rmsnorm_rows_apply_gemma", "rmsnorm_heads_rows_gemma", "rope_prefill",
              "kv_append_rows", "embed_lookup_rows"):
        assert n in names
