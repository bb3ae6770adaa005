"""Benchmark: random-init Gemma-3-1B int4 decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one decoded token. The workload is BASELINE.json's config 3: 26
layers, hidden 1152, 4 q / 1 kv heads of 256, FFN 6912 GeGLU, vocab 262144,
N(0, 0.02) weights packed to int4 (KM4 nibbles + bf16 block scales), fp16 KV
cache, greedy decode, batch 1, a prompt of 128 uniform-random ids, then
decoding toward position 4096 (default K = 3965 timed after W = 3 warm-up
tokens, so the timed tokens cover positions 131..4095). Every token streams
562 MB of weights (> the 126 MB L2), so no L2 flush is needed between steps.

value : tokens/s of the device-resident loop (DecodeSession.generate(): the
        greedy token kernel decodes up to 512 positions per launch, each
        position's input token picked on the device), timed with CUDA events.
e2e   : the same tokens through the public API DecodeSession.decode_step()
        (C ABI xp_session_decode_step): per token a 4-byte host->device copy
        of the input id and a 4-byte device->host read of the sampled id.
roofline : the persistent token kernel (the only kernel of a decode step):
        algorithmic bytes per position = int4 nibbles + bf16 scales of every
        matrix + the fp16 KV rows attended + embedding row and logits, over the
        average device time per position.
cpu_baseline : the CPU restatement of the same decode (oracle/, "port"),
        timed on this host's cores over a bounded sample.
batched : BASELINE config 4's batched decode: 64 independent sequences per
        GPU (prompts of 128 uniform-random ids, then 256 sampled tokens with
        top-k 64 / top-p 0.95 / T 1.0), every int4 matvec one tensor-core
        launch for all sequences (xp_bdec_*); tokens/s over the 256 decode
        steps (device time), all ranks' sequences / the slowest rank under
        torchrun (data-parallel replicas, no collective).
long_context : BASELINE config 5: single-query GQA attention (4 q / 1 kv x 256)
        over fp16 K/V caches of 8192 positions ~N(0, 1), 26 layers in the
        5 local (window 512) : 1 global pattern, 26 distinct caches (208 MB >
        L2), RoPE at position 8191, then top-k 64 / top-p 0.95 / T 1.0
        sampling on 262,144 logits ~N(0, 3); device time per step and the K/V
        bytes it reads.
matvec : BASELINE configs 1 and 2 on the streaming int4 matvec
        (xp_mv_plan_*: many matvecs in one persistent launch), timed with CUDA
        events over whole plan runs (limb prep included): config 1 = W
        6912x1152 N(0, 0.02) packed by the reference packer, x N(0, 1), seed 0,
        64 distinct copies of W per run (289 MB > L2); config 2 = the session's
        own per-token sweep (26 x q, k, v, o, gate, up, down + LM head, 567 MB).

Under torchrun (N > 1) each rank decodes its own independent sequence on its
own GPU (data-parallel replicas, weak scaling); value = all ranks' tokens /
the slowest rank's device time. The `tp` object then reports one sequence
decoded by all N GPUs together with the LM head's rows split over them (the
argmax exchanged over NVLink inside the token kernel): tokens/s of that one
sequence, the slowest rank's device time.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Gemma-3-1B-shape int4 decode tok/s (matvec HBM GB/s, % of peak)"
PROMPT = 128
TARGET_POS = 4096


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-matvec", action="store_true")
    ap.add_argument("--no-batched", action="store_true")
    ap.add_argument("--no-tp", action="store_true")
    ap.add_argument("--no-long", action="store_true")
    ap.add_argument("--ncu-case", choices=["full", "small", "multi", "matvec", "bmm", "batched", "long", "prefill"],
                    default=None,
                    help="run only a short untimed decode as an ncu capture target: 'full' = the bench model "
                         "(4 prompt tokens, 2 decode tokens), 'small' = 4 layers and a 32K vocab, 'multi' = the "
                         "five-kernel graph path on the bench model, 'matvec' = three runs of the config-1 "
                         "matvec plan, 'bmm' = three tensor-core batched matvecs of the LM head for 64 sequences")
    return ap.parse_args()


class MvJob(__import__("ctypes").Structure):
    import ctypes as _C
    _fields_ = [("out", _C.c_void_p), ("inp", _C.c_void_p), ("wq", _C.c_void_p), ("sc", _C.c_void_p),
                ("rows", _C.c_uint32), ("cols", _C.c_uint32)]


def config1_plan(copies=64, rows=1152, cols=6912):
    """W (cols x rows) N(0, 0.02) packed by the reference
    packer (device port, bit-exact), x N(0, 1), seed 0; `copies` distinct copies
    of the packed planes in one matvec plan. Returns (plan, keep-alive list)."""
    import ctypes as C
    import torch
    from xpose_b200._lib import check, lib
    w = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    x = torch.empty(rows, dtype=torch.float32, device="cuda")
    check(lib().xp_gen_normal(None, w.data_ptr(), rows * cols, 0, 0, 1, 0.02))
    check(lib().xp_gen_normal(None, x.data_ptr(), rows, 0, 0, 2, 1.0))
    wq = torch.empty(rows * cols // 8, dtype=torch.int32, device="cuda")
    sc = torch.empty(rows * cols // 64, dtype=torch.int32, device="cuda")
    check(lib().xp_pack_km4bf16(None, w.data_ptr(), rows, cols, wq.data_ptr(), sc.data_ptr()))
    del w
    keep = [x]
    jobs = []
    for _ in range(copies):
        cw, cs, out = wq.clone(), sc.clone(), torch.empty(cols, device="cuda")
        keep += [cw, cs, out]
        jobs.append(MvJob(out.data_ptr(), x.data_ptr(), cw.data_ptr(), cs.data_ptr(), rows, cols))
    arr = (MvJob * len(jobs))(*jobs)
    plan = C.c_void_p()
    check(lib().xp_mv_plan_create(C.cast(arr, C.c_void_p), len(jobs), C.byref(plan)))
    return plan, keep


def batched_bench(sess, cfg, rank, world, max_over_ranks, barrier, nseq=64, prompt=128, new=256):
    """BASELINE config 4 (batched part) on this rank's GPU."""
    from xpose_b200.decode import BatchDecode, Sampling
    bd = BatchDecode(sess, nseq, prompt + new + 1,
                     Sampling(greedy=False, temperature=1.0, top_k=64, top_p=0.95, seed=4242), seq0=rank * nseq)
    try:
        prompts = np.random.default_rng(500 + rank).integers(0, cfg.vocab, (nseq, prompt), dtype=np.uint32)
        bd.prefill(prompts)
        toks = bd.step()  # the first decode step (untimed warm-up)
        barrier()
        ms = bd.generate(new - 1)
        ms = max_over_ranks(ms)
        return {"workload": f"{nseq} sequences per GPU, prompt {prompt}, {new} new tokens, top-k 64 / top-p 0.95 / "
                            "T 1.0 (BASELINE config 4, batched part)",
                "value": round(world * nseq * (new - 1) / (ms / 1000.0), 1), "unit": "tok/s",
                "ms_per_step": round(ms / (new - 1), 3), "sequences": world * nseq,
                "kernel": "bmm_kernel (tcgen05.mma kind::f16, TMEM accumulators) for every int4 matvec",
                "first_tokens": [int(t) for t in toks[:4]]}
    finally:
        bd.close()


def long_context_bench(peak, iters=20):
    """BASELINE config 5 through the C ABI (xp_attention_decode, xp_sample_topk)."""
    import torch
    from xpose_b200._lib import check, lib
    L, S, pos, vocab = 26, 8192, 8191, 262144
    g = torch.Generator(device="cuda").manual_seed(5)
    kc = [torch.randn(S * 256, generator=g, device="cuda").half() for _ in range(L)]
    vc = [torch.randn(S * 256, generator=g, device="cuda").half() for _ in range(L)]
    q = torch.randn(1024, generator=g, device="cuda")
    k = torch.randn(256, generator=g, device="cuda")
    v = torch.randn(256, generator=g, device="cuda")
    qn = torch.randn(256, generator=g, device="cuda") * 0.02
    kn = torch.randn(256, generator=g, device="cuda") * 0.02
    logits = torch.randn(vocab, generator=g, device="cuda") * 3.0
    out = torch.empty(1024, device="cuda")
    posd = torch.tensor([pos], dtype=torch.int32, device="cuda")
    tok = torch.empty(1, dtype=torch.int32, device="cuda")
    ns_g, ns_l = 64, 8
    scr = torch.zeros(lib().xp_attention_scratch_bytes(ns_g) // 4 + 64, dtype=torch.int32, device="cuda")
    sscr = torch.zeros(lib().xp_sample_scratch_bytes(vocab) // 4 + 64, dtype=torch.int32, device="cuda")
    layers = [(l, (l + 1) % 6 == 0) for l in range(L)]
    stream = torch.cuda.Stream()

    def step():
        st = stream.cuda_stream
        for l, glob in layers:
            check(lib().xp_attention_decode(st, out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                            qn.data_ptr(), kn.data_ptr(), kc[l].data_ptr(), vc[l].data_ptr(),
                                            posd.data_ptr(), 0 if glob else 512, 1e6 if glob else 1e4, 1e-6,
                                            1.0 / 16, ns_g if glob else ns_l, S, scr.data_ptr()))
        check(lib().xp_sample_topk(st, tok.data_ptr(), None, None, logits.data_ptr(), vocab, 64, 1.0, 0.95, 7, 0,
                                   posd.data_ptr(), sscr.data_ptr()))
    with torch.cuda.stream(stream):
        for _ in range(3):
            step()
    torch.cuda.synchronize()
    # one step as a CUDA graph: the device time, not Python's submission rate
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        graph.replay()
        e0.record(stream)
        for _ in range(iters):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    nglob = sum(1 for _, gl in layers if gl)
    kv_bytes = (nglob * S + (L - nglob) * 512) * 256 * 2 * 2
    return {"workload": "26 x single-query GQA attention over 8192-position fp16 caches (5 local w512 : 1 global) + "
                        "top-k 64 / top-p 0.95 sampling on 262144 logits",
            "us_per_step": round(ms * 1000.0, 1), "kv_bytes": kv_bytes,
            "kv_GB/s": round(kv_bytes / ms / 1e6, 1), "frac": round(kv_bytes / ms / 1e6 / peak, 4),
            "launches_per_step": 2 * L + 2}


def matvec_bench(sess, peak):
    """BASELINE configs 1 and 2 on the streaming matvec (GB/s of algorithmic bytes)."""
    import ctypes as C
    import torch
    from xpose_b200._lib import check, lib
    ms2, b2, _ = sess.profile_matvec(iters=20)
    plan, keep = config1_plan()
    try:
        b1 = C.c_uint64()
        check(lib().xp_mv_plan_bytes(plan, C.byref(b1)))
        for _ in range(3):
            check(lib().xp_mv_plan_run(plan, None))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 20
        torch.cuda.synchronize()
        e0.record()
        for _ in range(n):
            check(lib().xp_mv_plan_run(plan, None))
        e1.record()
        torch.cuda.synchronize()
        ms1 = e0.elapsed_time(e1) / n
    finally:
        lib().xp_mv_plan_destroy(plan)
        del keep

    def entry(workload, nbytes, ms):
        gbs = nbytes / ms / 1e6
        return {"workload": workload, "bytes": int(nbytes), "us": round(ms * 1000.0, 2), "GB/s": round(gbs, 1),
                "frac": round(gbs / peak, 4)}
    return {"kernel": "mv_stream_kernel (xp_mv_plan_run: limb prep + one persistent streaming launch)",
            "peak": peak, "unit": "GB/s",
            "config1": entry("W 6912x1152 int4 matvec, 64 distinct weight copies per run", b1.value, ms1),
            "config2": entry("per-token matvec sweep: 26 x (q, k, v, o, gate, up, down) + LM head", b2, ms2)}


def ncu_case(which):
    """A short, untimed run used as the target of the ncu captures in profiles/."""
    if which == "bmm":
        import torch
        from xpose_b200._lib import check, lib
        rows, cols, n = 1152, 262144, 64
        w = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
        check(lib().xp_gen_normal(None, w.data_ptr(), rows * cols, 0, 0, 1, 0.02))
        wq = torch.empty(rows * cols // 8, dtype=torch.int32, device="cuda")
        sc = torch.empty(rows * cols // 64, dtype=torch.int32, device="cuda")
        check(lib().xp_pack_km4bf16(None, w.data_ptr(), rows, cols, wq.data_ptr(), sc.data_ptr()))
        del w
        x = torch.randn(n * rows, device="cuda")
        out = torch.empty(n * cols, device="cuda")
        nb = lib().xp_mv_km4_bs_batch_scratch_bytes(rows, cols, n)
        scr = torch.zeros(nb // 4 + 64, dtype=torch.int32, device="cuda")
        for _ in range(3):
            check(lib().xp_mv_km4_bs_batch(None, out.data_ptr(), x.data_ptr(), wq.data_ptr(), sc.data_ptr(), rows, cols,
                                           n, scr.data_ptr()))
        torch.cuda.synchronize()
        print("ncu case bmm: 3 batched LM-head matvecs, 64 sequences")
        return 0
    if which == "matvec":
        import torch
        from xpose_b200._lib import check, lib
        plan, keep = config1_plan()
        for _ in range(3):
            check(lib().xp_mv_plan_run(plan, None))
        torch.cuda.synchronize()
        lib().xp_mv_plan_destroy(plan)
        print("ncu case matvec: 3 runs of the config-1 plan")
        return 0
    if which == "long":
        r = long_context_bench(1.0, iters=2)
        print("ncu case long:", r["us_per_step"], "us per step (graph replays of 26 attention calls + sampling)")
        return 0
    from xpose_b200.decode import DecodeConfig, DecodeSession, Sampling
    if which == "prefill":
        s = DecodeSession.random(DecodeConfig(max_seq=4096), Sampling(), seed=0)
        prompt = np.random.default_rng(0).integers(0, s.cfg.vocab, size=PROMPT).astype(np.uint32)
        s.prefill(prompt)  # creates the chunked-prefill engine
        s.reset()
        print("ncu case prefill: second prefill of", PROMPT, "tokens follows")
        s.prefill(prompt)
        return 0
    if which == "batched":
        from xpose_b200.decode import BatchDecode
        cfg = DecodeConfig(max_seq=512)
        s = DecodeSession.random(cfg, Sampling(), seed=1)
        bd = BatchDecode(s, 64, 512, Sampling(greedy=False, temperature=1.0, top_k=64, top_p=0.95, seed=5))
        try:
            bd.prefill(np.random.default_rng(0).integers(0, cfg.vocab, size=(64, 1)).astype(np.uint32))
            bd.step()
            bd.step()
        finally:
            bd.close()
        print("ncu case batched: 64 sequences, one prompt position, two decode steps")
        return 0
    if which == "multi":
        os.environ["XP_ENGINE_MULTI"] = "1"
    cfg = DecodeConfig(max_seq=4096) if which in ("full", "multi") else DecodeConfig(n_layers=4, vocab=32768,
                                                                                       max_seq=512)
    s = DecodeSession.random(cfg, Sampling(), seed=0)
    s.prefill(np.arange(4, dtype=np.uint32))
    toks, ms = s.generate(2)
    print("ncu case", which, "tokens", list(toks), "kernels/token", s.stats()["kernels_per_token"])
    return 0


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def token_bytes(cfg, p0, p1):
    """Average algorithmic HBM bytes of one decode token over positions [p0, p1)."""
    H, V = cfg.hidden, cfg.vocab
    w = cfg.weight_bytes()
    kv_row = 2 * cfg.n_kv_heads * cfg.head_dim * 2  # K + V, fp16
    n = max(1, p1 - p0)
    tot = 0
    for p in range(p0, p0 + n):
        seq = p + 1
        tot += sum(seq if cfg.layer_is_global(l) else min(seq, cfg.sliding_window) for l in range(cfg.n_layers))
    return int(w + tot * kv_row / n + H * 4 + V * 4)


def steps_default(warmup):
    return TARGET_POS - PROMPT - warmup


# ---------------------------------------------------------------------------
# CPU baseline (oracle restatement, test infrastructure used only as the checker arm)
# ---------------------------------------------------------------------------
def cpu_decode(n_tokens, warm=1, prompt_len=8):
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O
    from xpose_b200.decode import DecodeConfig

    cfg = DecodeConfig(max_seq=prompt_len + warm + n_tokens + 1)
    t0 = time.time()
    om = O.OracleModel(cfg, seed=0)
    build_s = time.time() - t0
    # A short prompt fills the KV rows (time excluded); a decode token's CPU
    # cost is the 562 MB weight stream, which does not depend on the position.
    prompt = O.gen_tokens(0, 0x777, prompt_len, cfg.vocab)
    logits = None
    for p, t in enumerate(prompt):
        logits = om.forward(int(t), p, want_logits=(p == prompt_len - 1))
    pos = prompt_len
    tok = int(np.argmax(logits))
    for _ in range(warm):
        logits = om.forward(tok, pos)
        tok = int(np.argmax(logits))
        pos += 1
    t0 = time.perf_counter()
    for _ in range(n_tokens):
        logits = om.forward(tok, pos)
        tok = int(np.argmax(logits))
        pos += 1
    dt = time.perf_counter() - t0
    return n_tokens / dt, build_s, os.cpu_count()


def ref_engine_decode(n_tokens, warm=1, prompt_len=8):
    """The reference's own DecodeSession (examples/llm/decode.cpp) and kernels,
    built from the reference sources into oracle/_ref/libxpref.so, on a
    full-size seeded GGUF. Returns None when that library was not built."""
    if not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libxpref.so")):
        return None
    import shutil
    import tempfile
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O
    from xpose_b200.decode import DecodeConfig

    cfg = DecodeConfig(max_seq=prompt_len + warm + n_tokens + 1)
    tmp = tempfile.mkdtemp(prefix="_refgguf", dir=ROOT)
    try:
        path = os.path.join(tmp, "model.gguf")
        O.write_random_gguf(cfg, 0, path)
        sess = O.RefSession(path, cfg.max_seq, cfg.global_every)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    sess.prefill(O.gen_tokens(0, 0x777, prompt_len, cfg.vocab))
    for _ in range(warm):
        sess.decode_step()
    t0 = time.perf_counter()
    for _ in range(n_tokens):
        sess.decode_step()
    dt = time.perf_counter() - t0
    sess.close()
    return n_tokens / dt, os.cpu_count()


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    k = min(args.steps or 8, 8)
    w = min(args.warmup, 1)
    got = ref_engine_decode(k, warm=w)
    sample = (f"{k} full-size decode tokens at positions {8 + w}..{8 + w + k - 1} after an 8-token prompt "
              "(per-token cost is the weight stream, independent of position)")
    if got is not None:
        tps, cores = got
        kind = "reference"
        note = ("the reference's own DecodeSession and kernel sources (examples/llm/decode.cpp, kernels/*.cl) "
                "compiled for the host cores (oracle/_ref/libxpref.so), OpenMP over each dispatch's work items; "
                "its Vulkan runtime and llvmpipe path are unavailable on this box")
    else:
        tps, _, cores = cpu_decode(k, warm=w)
        kind = "port"
        note = "CPU restatement of the reference decode path (oracle/xp_oracle.c); oracle/_ref was not built"
    line = {
        "metric": METRIC, "impl": "reference", "value": round(tps, 4), "unit": "tok/s", "n_gpus": 1,
        "steps": k, "warmup": w, "ms_per_step": round(1000.0 / tps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights, fp32 compute, fp16 KV",
        "data": "synthetic (seeded N(0,0.02) random-init weights, uniform-random prompt ids)",
        "config": {"workload": "Gemma-3-1B-shape greedy decode, batch 1 (BASELINE config 3)", "sample": sample},
        "cpu_baseline": {"value": round(tps, 4), "unit": "tok/s", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": round(tps, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": note,
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
def main():
    args = parse()
    rank, world, local = dist_env()
    if args.ncu_case:
        return ncu_case(args.ncu_case)
    if args.impl == "reference":
        return run_reference(args)

    import torch

    W = max(3, args.warmup)
    K = args.steps if args.steps is not None else steps_default(W)
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = local if world > 1 else 0

    from xpose_b200.decode import DecodeConfig, DecodeSession, Sampling

    max_seq = max(TARGET_POS, PROMPT + W + K + 1)
    max_seq = (max_seq + 63) // 64 * 64
    cfg = DecodeConfig(max_seq=max_seq)
    sess = DecodeSession.random(cfg, Sampling(greedy=True), seed=0, device=dev)
    rng = np.random.default_rng(1000 + rank)
    prompt = rng.integers(0, cfg.vocab, PROMPT, dtype=np.uint32)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{dev}")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident decode (value) ----
    # prefill of the 128-token prompt (chunked: 64 positions per tensor-core
    # pass), host wall clock around the synchronous call, after one untimed
    # prefill that creates the chunked-prefill engine
    sess.reset()
    sess.prefill(prompt)  # warm: creates the chunked-prefill engine once
    sess.reset()
    t_pf = time.perf_counter()
    sess.prefill(prompt)
    pf_ms = (time.perf_counter() - t_pf) * 1000.0
    prefill = {"tokens": len(prompt), "ms": round(pf_ms, 3), "tok/s": round(len(prompt) / pf_ms * 1000.0, 1),
               "path": "chunked: 64 prompt positions per pass on the tensor-core batched engine (host wall clock)"}
    sess.generate(W, want_tokens=False)
    gpu_index = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(dev)).split(",")[dev]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else dev
    clocks = ClockSampler(gpu_index)
    barrier()
    clocks.start()
    _, ms = sess.generate(K, want_tokens=False)
    clock_info = clocks.stop()
    barrier()
    ms_max = max_over_ranks(ms)
    value = world * K / (ms_max / 1000.0)
    kpt = sess.stats()["kernels_per_token"]
    assert sess.error_word() == 0

    # ---- roofline of the dominant kernel ----
    # One launch of the persistent token kernel decodes one position, so its
    # average duration is the device time per token. Algorithmic bytes per
    # launch = int4 nibbles + bf16 scales of every matrix (562,360,320 B) + the
    # fp16 K and V rows the layers attend at that position (local layers a
    # 512 window, global layers the whole prefix) + the embedding row and the
    # logits, averaged over the timed positions.
    peak, peak_kind = measured_peak()
    tok_bytes = token_bytes(cfg, PROMPT + W, PROMPT + W + K)
    achieved = tok_bytes / (ms_max / K / 1000.0) / 1e9

    # ---- e2e through the public API ----
    e2e = None
    if not args.no_e2e:
        sess.reset()
        sess.prefill(prompt)
        for _ in range(W):
            sess.decode_step()
        barrier()
        sess.timer_start()
        for _ in range(K):
            sess.decode_step()
        e_ms = sess.timer_stop()
        e_ms = max_over_ranks(e_ms)
        e2e = {"value": round(world * K / (e_ms / 1000.0), 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
               "d2h_bytes_per_step": 4}

    traffic = None
    tpath = os.path.join(ROOT, "profiles", "token_kernel_traffic.json")
    if os.path.exists(tpath):
        try:
            with open(tpath) as f:
                tr = json.load(f)
            traffic = tr.get("dram_bytes_per_token")
        except Exception:
            traffic = None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            tps, build_s, cores = cpu_decode(4, warm=1)
            cpu = {"value": round(tps, 4), "unit": "tok/s", "cores": cores, "kind": "port",
                   "sample": "4 full-size decode tokens at positions 9-12 after an 8-token prompt "
                             "(OpenMP over all host cores)"}
        except Exception as e:  # the checker arm must not hide the GPU result
            cpu = {"value": None, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port", "sample": f"failed: {e}"}

    tp = None
    if world > 1 and not args.no_tp:
        try:
            from xpose_b200.tp import shard_lm_head
            shard_lm_head(sess)
            sess.reset()
            tprompt = np.random.default_rng(77).integers(0, cfg.vocab, PROMPT, dtype=np.uint32)
            sess.prefill(tprompt)
            sess.generate(W, want_tokens=False)
            kt = min(K, 1000)
            barrier()
            _, tms = sess.generate(kt, want_tokens=False)
            tms = max_over_ranks(tms)
            assert sess.error_word() == 0
            tp = {"workload": f"one sequence, LM head rows split over {world} GPUs (NVLink argmax exchange)",
                  "value": round(kt / (tms / 1000.0), 2), "unit": "tok/s", "ms_per_step": round(tms / kt, 4),
                  "steps": kt, "scaling": "strong"}
        except Exception as e:
            tp = {"error": str(e)}

    bat = None
    if not args.no_batched:
        try:
            bat = batched_bench(sess, cfg, rank, world, max_over_ranks, barrier)
        except Exception as e:  # a failure here must not hide the decode result
            bat = {"error": str(e)}

    lc = None
    if rank == 0 and not args.no_long:
        try:
            lc = long_context_bench(peak)
        except Exception as e:
            lc = {"error": str(e)}

    mv = None
    if rank == 0 and not args.no_matvec:
        try:
            mv = matvec_bench(sess, peak)
        except Exception as e:  # a failure here must not hide the decode result
            mv = {"error": str(e)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(ms_max / K, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int4 weights (KM4 + bf16 scales), fp32 accumulation, fp16 KV",
            "data": "synthetic (seeded N(0,0.02) random-init weights, uniform-random prompt ids)",
            "config": {"workload": "BASELINE config 3: Gemma-3-1B-shape greedy decode, batch 1, prompt 128, "
                                   f"positions {PROMPT + W}..{PROMPT + W + K - 1}",
                       "parallelism": f"dp{world} (independent sequences)" if world > 1 else "single GPU",
                       "l2": "weights 562 MB/token > 126 MB L2; no flush needed"},
            "e2e": e2e,
            # generate() runs the greedy token kernel over up to 512 positions
            # per cooperative launch (xp_session_generate)
            "gpu_launches": (K + 511) // 512 if kpt == 1 else kpt * K,
            "kernels_per_token": kpt,
            "tokens_per_launch": 512 if kpt == 1 else 1,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": "token_kernel (persistent; each position one pass: all int4 matvecs, attention, "
                                   "norms, LM head, argmax; up to 512 positions per launch)",
                         "algorithmic_bytes_per_token": tok_bytes,
                         "avg_token_us": round(ms_max / K * 1000.0, 2), "peak_kind": peak_kind},
            "clocks": clock_info,
            "cpu_baseline": cpu,
            "matvec": mv,
            "prefill": prefill,
            "batched": bat,
            "tp": tp,
            "long_context": lc,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
