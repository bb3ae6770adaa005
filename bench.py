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
    ap.add_argument("--attn-layer-cost", action="store_true",
                    help="print the in-graph cost of one xp_attention_decode layer (slope of 1 vs 26 launches) "
                         "for local and global layers at several split counts, then exit")
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


def measured_tflops():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops_sustained"]), "measured (sustained)"
    except Exception:
        return 1400.0, "fallback (sustained)"


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
        # per step: every int4 weight byte once (all sequences share it) and
        # 2 flops per weight per sequence on the tensor cores
        step_s = ms / (new - 1) / 1000.0
        wb = cfg.weight_bytes()
        nweights = wb * 16 // 9  # 4.5 bits per weight (nibble + 1/16 bf16 scale per 32)
        gbs = wb / step_s / 1e9
        tfs = 2.0 * nseq * nweights / step_s / 1e12
        hbm_peak, _ = measured_peak()
        tc_peak, tc_kind = measured_tflops()
        hb, tb = gbs / hbm_peak, tfs / tc_peak
        roof = {"bound": "hbm" if hb >= tb else "tensor", "achieved": round(gbs if hb >= tb else tfs, 1),
                "peak": hbm_peak if hb >= tb else tc_peak, "unit": "GB/s" if hb >= tb else "TFLOP/s",
                "frac": round(max(hb, tb), 4), "traffic": None,
                "hbm": {"achieved_GBps": round(gbs, 1), "frac": round(hb, 4)},
                "tensor": {"achieved_TFLOPs": round(tfs, 2), "frac": round(tb, 4), "peak_kind": tc_kind},
                "kernel": "whole batched step (bmm_kernel for every int4 matvec + per-sequence kernels)"}
        return {"roofline": roof, "workload": f"{nseq} sequences per GPU, prompt {prompt}, {new} new tokens, top-k 64 / top-p 0.95 / "
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
    ns_g, ns_l = 64, 16
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
    step_bytes = kv_bytes + vocab * 4  # + the logits the sampler reads
    gbs = step_bytes / ms / 1e6
    return {"roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "traffic": None, "algorithmic_bytes_per_step": step_bytes,
                         "kernel": "attn_decode_kernel x 26 + topk_cand_kernel + topk_draw_kernel (one graph)"},
            "workload": "26 x single-query GQA attention over 8192-position fp16 caches (5 local w512 : 1 global) + "
                        "top-k 64 / top-p 0.95 sampling on 262144 logits",
            "us_per_step": round(ms * 1000.0, 1), "kv_bytes": kv_bytes,
            "kv_GB/s": round(kv_bytes / ms / 1e6, 1), "frac": round(kv_bytes / ms / 1e6 / peak, 4),
            "launches_per_step": 2 * L + 2}


def attn_layer_cost():
    """In-graph cost of one attention layer at position 8191: a CUDA graph of 1
    and of 26 xp_attention_decode launches (4 distinct 8192-position caches,
    so global layers are partly L2-resident), per layer = the slope."""
    import torch
    from xpose_b200._lib import check, lib
    S, pos = 8192, 8191
    g = torch.Generator(device="cuda").manual_seed(5)
    kc = [torch.randn(S * 256, generator=g, device="cuda").half() for _ in range(4)]
    vc = [torch.randn(S * 256, generator=g, device="cuda").half() for _ in range(4)]
    q, k, v = (torch.randn(n, generator=g, device="cuda") for n in (1024, 256, 256))
    qn, kn = (torch.randn(256, generator=g, device="cuda") * 0.02 for _ in range(2))
    out = torch.empty(1024, device="cuda")
    posd = torch.tensor([pos], dtype=torch.int32, device="cuda")
    scr = torch.zeros(lib().xp_attention_scratch_bytes(128) // 4 + 64, dtype=torch.int32, device="cuda")
    stream = torch.cuda.Stream()

    def run(n, glob, ns):
        for l in range(n):
            check(lib().xp_attention_decode(stream.cuda_stream, out.data_ptr(), q.data_ptr(), k.data_ptr(),
                                            v.data_ptr(), qn.data_ptr(), kn.data_ptr(), kc[l % 4].data_ptr(),
                                            vc[l % 4].data_ptr(), posd.data_ptr(), 0 if glob else 512,
                                            1e6 if glob else 1e4, 1e-6, 1.0 / 16, ns, S, scr.data_ptr()))

    def us(n, glob, ns, iters=50):
        with torch.cuda.stream(stream):
            run(n, glob, ns)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            run(n, glob, ns)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            gr.replay()
            e0.record(stream)
            for _ in range(iters):
                gr.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters * 1000.0

    for glob, splits in ((False, (1, 2, 4, 8, 16, 32)), (True, (16, 32, 64, 128))):
        for ns in splits:
            t1, t26 = us(1, glob, ns), us(26, glob, ns)
            print(json.dumps({"layer": "global" if glob else "local", "splits": ns, "us_1": round(t1, 2),
                              "us_26": round(t26, 2), "us_per_layer": round((t26 - t1) / 25, 2)}))
    return 0


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
                "frac": round(gbs / peak, 4),
                "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(gbs / peak, 4), "traffic": None,
                             "kernel": "mv_stream_kernel (one launch per plan run)"}}
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


def depth_buckets(K, W, nb=4):
    """Where the K timed tokens sit: `nb` equal segments of the decode range
    [PROMPT + W, TARGET_POS) (positions 131..4095 at W = 3), K/nb tokens
    centred in each, so a short run still averages over attention depth. At
    the default K the segments are covered whole (one contiguous sweep).
    Returns [(first timed position, tokens)]."""
    lo, hi = PROMPT + W, TARGET_POS
    if K >= hi - lo:
        return [(lo, K)]
    nb = max(1, min(nb, K))
    out = []
    for b in range(nb):
        kb = K // nb + (1 if b < K % nb else 0)
        s0, s1 = lo + (hi - lo) * b // nb, lo + (hi - lo) * (b + 1) // nb
        out.append((s0 + max(0, (s1 - s0 - kb) // 2), kb))
    return out


def context_tokens(rank=0):
    """The token ids that fill the positions before a bucket: the 128-token
    uniform-random prompt, then uniform-random ids (teacher-forced context)."""
    rng = np.random.default_rng(1000 + rank)
    return rng.integers(0, 262144, TARGET_POS + 64, dtype=np.uint32)


# ---------------------------------------------------------------------------
# CPU baselines. The checker code under oracle/ (the reference's own kernel
# sources and DecodeSession compiled for the host, oracle/_ref/libxpref.so, or
# the C restatement oracle/liboracle.so) is timed here as the reported CPU
# arm; it is never part of the measured GPU path.
# ---------------------------------------------------------------------------
def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def _checkers():
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O
    have_ref = os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libxpref.so"))
    return O, have_ref


def _timed(fn, reps):
    fn()  # warm
    t0 = time.perf_counter()
    for _ in range(reps):
        fn()
    return (time.perf_counter() - t0) / reps


def cpu_decode_port(om, n_tokens, greedy=True, prompt_len=8):
    """Decode tokens/s of the C restatement (OpenMP over all host cores) on the
    full-size model, after a short prompt (a decode token's CPU cost is the
    562 MB weight stream; attention over a short prefix is negligible)."""
    O, _ = _checkers()
    prompt = O.gen_tokens(0, 0x777, prompt_len, om.cfg.vocab)
    logits = None
    for p, t in enumerate(prompt):
        logits = om.forward(int(t), p, want_logits=(p == prompt_len - 1))
    pos = prompt_len

    def pick(lg, p):
        if greedy:
            return int(np.argmax(lg))
        u = O.oracle().xo_uniform(4242, 0, p)
        return int(O.oracle().xo_sample(lg, om.cfg.vocab, 1.0, 64, 0.95, u))
    tok = pick(logits, pos - 1)
    logits = om.forward(tok, pos)  # warm
    tok = pick(logits, pos)
    pos += 1
    t0 = time.perf_counter()
    for _ in range(n_tokens):
        logits = om.forward(tok, pos)
        tok = pick(logits, pos)
        pos += 1
    return n_tokens / (time.perf_counter() - t0)


def cpu_matvec_baseline(om):
    """BASELINE configs 1 and 2 on the host: the reference's `mv_km4_bs`
    (kernels/llm_matvec.cl, compiled for the CPU, one work item per output
    column, OpenMP over all cores), else the restatement's xo_mv_km4_bs.
    Config 1 streams 64 distinct copies of the packed 6912x1152 W per pass
    (like the GPU case, more than the host's caches); config 2 the model's
    own 26 layers x 7 matrices + LM head once per pass."""
    O, have_ref = _checkers()
    cores = host_cores()
    kind = "reference" if have_ref else "port"

    def mv(out, x, words, scales, rows, cols):
        if have_ref:
            O.ref_launch("mv_km4_bs", cols, out, x, words, scales, rows, cols, threads=cores)
        else:
            O.oracle().xo_mv_km4_bs(out, x, words, scales, rows, cols)

    def nbytes(rows, cols):
        return rows * cols // 2 + rows * cols // 16 + 4 * rows + 4 * cols

    rows, cols = 1152, 6912
    w = O.gen_normal(0, 1, rows * cols, 0.02)
    x1 = O.gen_normal(0, 2, rows, 1.0)
    words, scales = O.pack(w, rows, cols)
    copies = [(words.copy(), scales.copy()) for _ in range(64)]
    out1 = np.zeros(cols, np.float32)

    def pass1():
        for wq, sc in copies:
            mv(out1, x1, wq, sc, rows, cols)
    t1 = _timed(pass1, 2)
    b1 = 64 * nbytes(rows, cols)
    mats = []
    for lw in om.layers_np:
        for m, (r, c) in enumerate(om.cfg.matrix_shapes()):
            mats.append((lw["words"][m], lw["scales"][m], r, c))
    mats.append((om.lm_words, om.lm_scales, om.cfg.hidden, om.cfg.vocab))
    xs = {r: O.gen_normal(0, 3 + r, r, 1.0) for r in {m[2] for m in mats}}
    outs = {c: np.zeros(c, np.float32) for c in {m[3] for m in mats}}

    def pass2():
        for wq, sc, r, c in mats:
            mv(outs[c], xs[r], wq, sc, r, c)
    t2 = _timed(pass2, 2)
    b2 = sum(nbytes(r, c) for _, _, r, c in mats)
    what = ("the reference's mv_km4_bs (kernels/llm_matvec.cl) compiled for the host" if have_ref
            else "the C restatement xo_mv_km4_bs")
    return ({"value": round(b1 / t1 / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": kind,
             "sample": f"2 passes over 64 copies of W 6912x1152 ({what})"},
            {"value": round(b2 / t2 / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": kind,
             "sample": f"2 sweeps of the 26 x 7 layer matrices + LM head ({what})"})


def _softmax_parts(span, min_span=128, max_parts=256):
    # examples/llm/decode.hpp softmax_parts_for
    if span < min_span:
        return 1
    p = 1
    while p * p < span and p < max_parts:
        p *= 2
    return min(p, span)


def cpu_long_context_baseline():
    """BASELINE config 5 on the host through the reference's own kernels
    (oracle/_ref): per layer QK-norm (rmsnorm_heads_gemma), rope, kv_append,
    attention_scores_mq4 + softmax_rows_{partial,finish,scale} +
    attention_apply_mq4 (split 16) + attention_apply_reduce over fp32 caches
    (the reference's KV type), the sequence of examples/llm/decode.cpp:1676-1731
    for spans >= 128; then topk4_partial (1024 chains) and the host draw over
    its 4096 candidates (decode.cpp:1873-1917, restated in oracle/). Without
    oracle/_ref: the restatement's xo_attention and xo_sample ("port")."""
    O, have_ref = _checkers()
    cores = host_cores()
    L, S, pos, vocab, hd = 26, 8192, 8191, 262144, 256
    rng = np.random.default_rng(5)
    kc = [rng.standard_normal(S * hd, dtype=np.float32) for _ in range(L)]
    vc = [rng.standard_normal(S * hd, dtype=np.float32) for _ in range(L)]
    q0 = rng.standard_normal(4 * hd, dtype=np.float32)
    k0 = rng.standard_normal(hd, dtype=np.float32)
    qn = (rng.standard_normal(hd, dtype=np.float32) * 0.02).astype(np.float32)
    logits = (rng.standard_normal(vocab, dtype=np.float32) * 3.0).astype(np.float32)
    glob = [(l + 1) % 6 == 0 for l in range(L)]
    q, k, att = np.zeros(4 * hd, np.float32), np.zeros(hd, np.float32), np.zeros(4 * hd, np.float32)
    scores = np.zeros(4 * S, np.float32)
    pmax, psum, stats = np.zeros(4 * 256, np.float32), np.zeros(4 * 256, np.float32), np.zeros(8, np.float32)
    part = np.zeros(16 * 4 * hd, np.float32)
    cval, cidx = np.zeros(4096, np.float32), np.zeros(4096, np.uint32)

    def step_ref():
        for l in range(L):
            seq = pos + 1
            kv_start = 0 if glob[l] or seq <= 512 else seq - 512
            span = seq - kv_start
            theta = 1e6 if glob[l] else 1e4
            O.ref_launch("rmsnorm_heads_gemma", 4 * hd, q, q0, qn, 4, hd, 1e-6, threads=cores)
            O.ref_launch("rmsnorm_heads_gemma", hd, k, k0, qn, 1, hd, 1e-6, threads=cores)
            O.ref_launch("rope", 2 * hd, q, 4, hd, pos, theta, threads=cores)
            O.ref_launch("rope", hd // 2, k, 1, hd, pos, theta, threads=cores)
            O.ref_launch("kv_append", hd, kc[l], k, hd, pos, threads=cores)
            O.ref_launch("kv_append", hd, vc[l], k0, hd, pos, threads=cores)
            O.ref_launch("attention_scores_mq4", span, scores, q, kc[l], hd, span, 1.0 / 16, kv_start, threads=cores)
            npt = _softmax_parts(span)
            O.ref_launch("softmax_rows_partial", 4 * npt, pmax, psum, scores, 4, span, npt, threads=cores)
            O.ref_launch("softmax_rows_finish", 4, stats, pmax, psum, 4, npt, threads=cores)
            O.ref_launch("softmax_rows_scale", 4 * span, scores, stats, 4, span, threads=cores)
            O.ref_launch("attention_apply_mq4", hd * 16, part, scores, vc[l], hd, span, kv_start, 16, threads=cores)
            O.ref_launch("attention_apply_reduce", 4 * hd, att, part, 4 * hd, 16, threads=cores)
        O.ref_launch("topk4_partial", 1024, cval, cidx, logits, vocab, 1024, threads=cores)
        u = O.oracle().xo_uniform(7, 0, pos)
        O.oracle().xo_sample(cval, 4096, 1.0, 64, 0.95, u)

    kc16 = [a.astype(np.float16).view(np.uint16) for a in kc] if not have_ref else None
    vc16 = [a.astype(np.float16).view(np.uint16) for a in vc] if not have_ref else None

    def step_port():
        for l in range(L):
            seq = pos + 1
            kv_start = 0 if glob[l] or seq <= 512 else seq - 512
            O.oracle().xo_attention(att, q0, kc16[l].ctypes.data, vc16[l].ctypes.data, 1, 4, 1, hd, kv_start,
                                    seq - kv_start, 1.0 / 16)
        u = O.oracle().xo_uniform(7, 0, pos)
        O.oracle().xo_sample(logits, vocab, 1.0, 64, 0.95, u)

    t = _timed(step_ref if have_ref else step_port, 5)
    return {"value": round(t * 1e6, 1), "unit": "us/step", "cores": cores,
            "kind": "reference" if have_ref else "port",
            "sample": "5 steps of 26 attention layers at position 8191 (4 global over 8192, 22 local over 512) + "
                      "sampling 262144 logits"}


def ref_engine_session(max_seq, greedy=True):
    """The reference's own DecodeSession (examples/llm/decode.cpp) and kernel
    sources, compiled for the host into oracle/_ref/libxpref.so, on the
    full-size seeded model written as a GGUF file. None when that library was
    not built."""
    if not os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libxpref.so")):
        return None
    import shutil
    import tempfile
    O, _ = _checkers()
    from xpose_b200.decode import DecodeConfig
    cfg = DecodeConfig(max_seq=max_seq)
    tmp = tempfile.mkdtemp(prefix="_refgguf", dir=ROOT)
    try:
        path = os.path.join(tmp, "model.gguf")
        O.write_random_gguf(cfg, 0, path)
        return O.RefSession(path, cfg.max_seq, cfg.global_every, greedy=greedy)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def config_block(W, K, buckets, world):
    return {"workload": "BASELINE config 3: Gemma-3-1B-shape greedy decode, batch 1, prompt 128, "
                        "decoding toward position 4096",
            "timed_positions": [[s, s + k - 1] for s, k in buckets],
            "parallelism": f"dp{world} (independent sequences)" if world > 1 else "single GPU",
            "l2": "weights 562 MB/token > 126 MB L2; no flush needed"}


def run_reference(args):
    """The reference arm: the reference's own CPU implementation of the decode
    path on this host's cores, at the same workload as ours: the 128-token
    prompt, then the same K timed positions in the same depth buckets, each
    after W untimed tokens (the positions between buckets are filled with the
    reference's own prefill). Rank 0 alone runs it under torchrun."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    W = max(3, args.warmup)
    K = args.steps if args.steps is not None else steps_default(W)
    buckets = depth_buckets(K, W)
    ctx = context_tokens(0)
    max_seq = max(TARGET_POS, buckets[-1][0] + buckets[-1][1] + 1)
    cores = host_cores()
    sess = ref_engine_session(max_seq)
    kind = "reference"
    total_s = 0.0
    if sess is not None:
        sess.prefill(ctx[:PROMPT])
        at = PROMPT
        for start, kb in buckets:
            if start - W > at:
                sess.prefill(ctx[at:start - W])
                at = start - W
            for _ in range(W):
                sess.decode_step()
            t0 = time.perf_counter()
            for _ in range(kb):
                sess.decode_step()
            total_s += time.perf_counter() - t0
            at = start + kb
        sess.close()
        note = ("the reference's own DecodeSession and kernel sources (examples/llm/decode.cpp, kernels/*.cl) "
                "compiled for the host cores (oracle/_ref/libxpref.so), OpenMP over each dispatch's work items; "
                "its Vulkan runtime and llvmpipe path are unavailable on this box")
    else:
        kind = "port"
        O, _ = _checkers()
        from xpose_b200.decode import DecodeConfig
        om = O.OracleModel(DecodeConfig(max_seq=max_seq), 0)
        for p in range(PROMPT):
            om.forward(int(ctx[p]), p, want_logits=False)
        at = PROMPT
        for start, kb in buckets:
            for p in range(at, start):
                om.forward(int(ctx[p]), p, want_logits=False)
            tok = int(ctx[start])
            t0 = time.perf_counter()
            for p in range(start, start + kb):
                tok = int(np.argmax(om.forward(tok, p)))
            total_s += time.perf_counter() - t0
            at = start + kb
        note = "CPU restatement of the reference decode path (oracle/xp_oracle.c); oracle/_ref was not built"
    tps = K / total_s
    positions = ", ".join(f"{s}..{s + k - 1}" for s, k in buckets)
    sample = f"{K} greedy decode tokens at positions {positions} after a 128-token prompt"
    line = {
        "metric": METRIC, "impl": "reference", "value": round(tps, 4), "unit": "tok/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": round(1000.0 / tps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights, fp32 compute, fp32 KV",
        "data": "synthetic (seeded N(0,0.02) random-init weights, uniform-random prompt ids)",
        "config": config_block(W, K, buckets, world),
        "cpu_baseline": {"value": round(tps, 4), "unit": "tok/s", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": round(tps, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": note + (f"; one process on all {cores} host cores serves every N (the whole host against the "
                        f"whole {world}-GPU job)" if world > 1 else ""),
    }
    print(json.dumps(line), flush=True)
    return 0


def tp_bench(sess, cfg, K, W, world, rank, barrier, max_over_ranks, shard_ffn=False):
    """One sequence decoded by all ranks with the LM head's rows (and with
    shard_ffn the FFN's gate|up columns and down-proj rows) split over them.
    First every rank decodes the same prompt unsharded, then sharded; the
    sharded tokens must equal the unsharded ones and each rank's logit rows
    must equal the same rows of the unsharded logits (bit-exact)."""
    import torch
    from xpose_b200.tp import shard_lm_head
    tprompt = np.random.default_rng(77).integers(0, cfg.vocab, PROMPT, dtype=np.uint32)
    n_check = 64
    sess.reset()
    # the same (tensor-parallel) kernel at one rank is the bit-exact reference
    sess.tp_attach(0, 1, [sess.tp_handle()], shard_ffn=True)
    sess.prefill(tprompt)
    ref_logits = sess.last_logits()
    ref_toks, _ = sess.generate(n_check)
    shard_lm_head(sess, shard_ffn=shard_ffn)
    sess.reset()
    sess.prefill(tprompt)
    logits = sess.last_logits()
    toks, _ = sess.generate(n_check)
    units = cfg.vocab // 64
    u0, u1 = units * rank // world, units * (rank + 1) // world
    shard_exact = bool(np.array_equal(logits[u0 * 64:u1 * 64], ref_logits[u0 * 64:u1 * 64]))
    match = bool(np.array_equal(np.asarray(toks), np.asarray(ref_toks)))
    flags = torch.tensor([int(match), int(shard_exact)], dtype=torch.int32, device="cuda")
    torch.distributed.all_reduce(flags, op=torch.distributed.ReduceOp.MIN)
    sess.reset()
    sess.prefill(tprompt)
    sess.generate(W, want_tokens=False)
    kt = min(K, 1000)
    barrier()
    _, tms = sess.generate(kt, want_tokens=False)
    tms = max_over_ranks(tms)
    assert sess.error_word() == 0
    what = "LM head rows and FFN gate|up columns / down-proj rows" if shard_ffn else "LM head rows"
    return {"workload": f"one sequence, {what} split over {world} GPUs (exchanges over NVLink inside the token kernel)",
            "value": round(kt / (tms / 1000.0), 2), "unit": "tok/s", "ms_per_step": round(tms / kt, 4),
            "steps": kt, "positions": [PROMPT + W, PROMPT + W + kt - 1], "scaling": "strong",
            "tokens_match": bool(flags[0].item()), "logit_shard_exact": bool(flags[1].item()),
            "checked_tokens": n_check}


# ---------------------------------------------------------------------------
def main():
    args = parse()
    rank, world, local = dist_env()
    if args.ncu_case:
        return ncu_case(args.ncu_case)
    if args.attn_layer_cost:
        return attn_layer_cost()
    if args.impl == "reference":
        # torchrun sets OMP_NUM_THREADS=1; the reference arm uses every host
        # core (set before any OpenMP runtime is loaded)
        os.environ["OMP_NUM_THREADS"] = str(host_cores())
        return run_reference(args)

    import torch

    W = max(3, args.warmup)
    K = args.steps if args.steps is not None else steps_default(W)
    buckets = depth_buckets(K, W)
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = local if world > 1 else 0

    from xpose_b200.decode import DecodeConfig, DecodeSession, Sampling

    max_seq = max(TARGET_POS, buckets[-1][0] + buckets[-1][1] + 1)
    max_seq = (max_seq + 63) // 64 * 64
    cfg = DecodeConfig(max_seq=max_seq)
    sess = DecodeSession.random(cfg, Sampling(greedy=True), seed=0, device=dev)
    ctx = context_tokens(rank)
    prompt = ctx[:PROMPT]

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

    # ---- prefill of the 128-token prompt (chunked: 64 positions per
    # tensor-core pass), host wall clock around the synchronous call, after
    # one untimed prefill that creates the chunked-prefill engine
    sess.reset()
    sess.prefill(prompt)
    sess.reset()
    t_pf = time.perf_counter()
    sess.prefill(prompt)
    pf_ms = (time.perf_counter() - t_pf) * 1000.0
    prefill = {"tokens": len(prompt), "ms": round(pf_ms, 3), "tok/s": round(len(prompt) / pf_ms * 1000.0, 1),
               "path": "chunked: 64 prompt positions per pass on the tensor-core batched engine (host wall clock)"}

    def to_bucket(start):
        # the context before the bucket (chunked prefill), then W untimed tokens
        sess.reset()
        sess.prefill(ctx[:start - W])

    # ---- device-resident decode (value): K tokens in depth buckets ----
    gpu_index = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(dev)).split(",")[dev]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else dev
    clocks = ClockSampler(gpu_index)
    clocks.start()
    ms = 0.0
    per_bucket = []
    for start, kb in buckets:
        to_bucket(start)
        sess.generate(W, want_tokens=False)
        barrier()
        _, bms = sess.generate(kb, want_tokens=False)
        barrier()
        ms += bms
        per_bucket.append({"positions": [start, start + kb - 1], "us_per_token": round(bms / kb * 1000.0, 2)})
    clock_info = clocks.stop()
    ms_max = max_over_ranks(ms)
    value = world * K / (ms_max / 1000.0)
    kpt = sess.stats()["kernels_per_token"]
    assert sess.error_word() == 0

    # ---- roofline of the dominant kernel ----
    # One pass of the persistent token kernel decodes one position, so its
    # average duration is the device time per token. Algorithmic bytes per
    # position = int4 nibbles + bf16 scales of every matrix (562,360,320 B) +
    # the fp16 K and V rows the layers attend at that position (local layers a
    # 512 window, global layers the whole prefix) + the embedding row and the
    # logits, averaged over the timed positions.
    peak, peak_kind = measured_peak()
    tok_bytes = int(sum(token_bytes(cfg, s, s + k) * k for s, k in buckets) / K)
    achieved = tok_bytes / (ms_max / K / 1000.0) / 1e9

    # ---- e2e through the public API: DecodeSession.decode_step() ----
    e2e = None
    if not args.no_e2e:
        e_ms = 0.0
        for start, kb in buckets:
            to_bucket(start)
            for _ in range(W):
                sess.decode_step()
            barrier()
            sess.timer_start()
            for _ in range(kb):
                sess.decode_step()
            e_ms += sess.timer_stop()
        e_ms = max_over_ranks(e_ms)
        e2e = {"value": round(world * K / (e_ms / 1000.0), 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
               "d2h_bytes_per_step": 4}

    traffic = None
    tpath = os.path.join(ROOT, "profiles", "token_kernel_traffic.json")
    if os.path.exists(tpath):
        try:
            with open(tpath) as f:
                traffic = json.load(f).get("dram_bytes_per_token")
        except Exception:
            traffic = None

    # ---- CPU baselines (rank 0 at N = 1 only) ----
    cpu = cpu_mv = cpu_bat = cpu_lc = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            O, _ = _checkers()
            om = O.OracleModel(DecodeConfig(max_seq=64), 0)
            cores = host_cores()
            tps = cpu_decode_port(om, 4)
            cpu = {"value": round(tps, 4), "unit": "tok/s", "cores": cores, "kind": "port",
                   "sample": "4 full-size greedy decode tokens at positions 9-12 after an 8-token prompt "
                             "(the C restatement, OpenMP over all host cores)"}
            tps_s = cpu_decode_port(om, 4, greedy=False)
            cpu_bat = {"value": round(tps_s, 4), "unit": "tok/s", "cores": cores, "kind": "port",
                       "sample": "4 sampled (top-k 64 / top-p 0.95 / T 1) decode tokens of one sequence: the "
                                 "reference decodes sequences one at a time, so its batched rate is its "
                                 "single-sequence rate"}
            cpu_mv = cpu_matvec_baseline(om)
            del om
            cpu_lc = cpu_long_context_baseline()
        except Exception as e:  # the checker arm must not hide the GPU result
            cpu = {"value": None, "unit": "tok/s", "cores": host_cores(), "kind": "port", "sample": f"failed: {e}"}

    tp = None
    if world > 1 and not args.no_tp:
        try:
            tp = tp_bench(sess, cfg, K, W, world, rank, barrier, max_over_ranks)
            tp["ffn_sharded"] = tp_bench(sess, cfg, K, W, world, rank, barrier, max_over_ranks, shard_ffn=True)
        except Exception as e:
            tp = {"error": str(e)}

    bat = None
    if not args.no_batched:
        try:
            bat = batched_bench(sess, cfg, rank, world, max_over_ranks, barrier)
            bat["cpu_baseline"] = cpu_bat
        except Exception as e:  # a failure here must not hide the decode result
            bat = {"error": str(e)}

    lc = None
    if rank == 0 and not args.no_long:
        try:
            lc = long_context_bench(peak)
            lc["cpu_baseline"] = cpu_lc
        except Exception as e:
            lc = {"error": str(e)}

    mv = None
    if rank == 0 and not args.no_matvec:
        try:
            mv = matvec_bench(sess, peak)
            if cpu_mv:
                mv["config1"]["cpu_baseline"], mv["config2"]["cpu_baseline"] = cpu_mv
        except Exception as e:  # a failure here must not hide the decode result
            mv = {"error": str(e)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(ms_max / K, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int4 weights (KM4 + bf16 scales), fp32 accumulation, fp16 KV",
            "data": "synthetic (seeded N(0,0.02) random-init weights, uniform-random prompt ids)",
            "config": config_block(W, K, buckets, world),
            "depth_buckets": per_bucket,
            "e2e": e2e,
            # generate() runs the greedy token kernel over up to 512 positions
            # per cooperative launch (xp_session_generate)
            "gpu_launches": sum((kb + 511) // 512 for _, kb in buckets) if kpt == 1 else kpt * K,
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
