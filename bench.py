"""Benchmark: batch-1 decode tok/s of the 36-layer VQ decoder on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--ctx C] [--impl ours|reference]

A step is one greedy decode token of the full model (36 layers, hidden 2560, GQA
16/4 x 256, FFN 10240, tied Q8_0 head over a 131072 vocabulary) at a 4096-token
context, f16 KV cache, random-init weights in the reference's formats (DQV3
4x4096x2 residual-VQ trunk). The prompt is seeded synthetic ids, run through the
model before timing. Weights (3.2 GB) are larger than L2, so every step streams
them from HBM; no flush is needed.

One JSON line on rank 0:
  value      tok/s of the device-resident decode loop (CUDA-graph replay per token);
             N>1: one sequence over N tensor-parallel ranks (strong scaling), the
             residual reduced over NVLink peer stores twice per layer
  e2e        tok/s through the C-ABI with host buffers (token up, next id down per step)
  roofline   the dominant kernel (the fused gate+up VQ GEMV), timed live with CUDA
             events over all 36 layers' weights, against the measured HBM peak
  cpu_baseline  the CPU restatement of model.rs::forward (oracle/) on a bounded sample
`--impl reference` times that CPU implementation alone (the reference's Rust runtime
cannot be built here; its restatement stands in for it).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import re
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "spark-x2.6-4b-q6k_b200"))

METRIC = "batch-1 decode tok/s (4B VQ) at 1/2/4/8 B200; GEMV HBM GB/s vs peak"
FALLBACK_HBM_GBS = 6650.0


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class Clocks:
    """nvidia-smi sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                for line in out.stdout.strip().splitlines():
                    self.rows.append([x.strip() for x in line.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in self.rows for k in range(4) if len(r) > 4 + k and r[4 + k] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def traffic_from_profiles(name: str):
    """traffic_bytes_per_launch recorded in profiles/<name>.md from an ncu capture."""
    p = os.path.join(ROOT, "profiles", name + ".md")
    try:
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(p).read())
        return float(m.group(1)) if m else None
    except OSError:
        return None


def cpu_baseline(ctx: int, tokens: int = 3, seed: int = 0) -> dict:
    """The CPU restatement of model.rs::forward (oracle/, f32 weights expanded at load as
    Weights::from_vq does), all host threads, on a bounded sample: a 4-layer slice of the
    config-2 model ([T,T,T,F]: 3 sliding + 1 full layer) plus the tied head, its KV cache
    filled with seeded values to `ctx` positions, timed over `tokens` decode steps at pos
    `ctx`; the head GEMV is timed alone, and tok/s = 1 / (9 * t_4layers + t_head)."""
    import oracle
    from spk.model import ModelConfig, synth_weights

    threads = os.cpu_count() or 1
    cfg = ModelConfig(layers=4, full=[False, False, False, True])
    W = synth_weights(cfg, seed=seed)
    layers = [{"in_norm": L["in_norm"], "post_norm": L["post_norm"],
               **{n: oracle.decode(L[n]) for n in ("qkv", "attn_gate", "out", "gate", "up", "down")}}
              for L in W["layers"]]
    embed = oracle.q80_dequant(W["embed"], cfg.vocab, cfg.hidden)
    m = oracle.Model(cfg.as_oracle(), layers, embed, W["norm"], ctx + tokens + 1, threads=threads)
    m.fill_kv(ctx, seed)
    m.forward(1, ctx)   # first touch
    t0 = time.perf_counter()
    for k in range(tokens):
        m.forward(2 + k, ctx + 1 + k)
    t4 = (time.perf_counter() - t0) / tokens
    x = np.random.default_rng(seed).normal(0, 1, cfg.hidden).astype(np.float32)
    oracle.matvec(embed, x, threads)
    t0 = time.perf_counter()
    for _ in range(tokens):
        oracle.matvec(embed, x, threads)
    th = (time.perf_counter() - t0) / tokens
    m.close()
    t_tok = 9.0 * max(t4 - th, 1e-9) + th
    return {"value": 1.0 / t_tok, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"model.rs forward restated in C (oracle/), 4 of 36 layers (3 sliding + 1 full) + tied "
                      f"head at ctx {ctx} with seeded KV, {tokens} tokens timed; scaled 9x layers + head; "
                      f"t_4layers+head {t4 * 1e3:.1f} ms, t_head {th * 1e3:.1f} ms"}


def len_embed(cfg) -> int:
    return cfg.vocab * cfg.hidden // 32 * 34


def dist_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def run_reference(args) -> None:
    """--impl reference: the reference's CPU implementation of the path (its Rust runtime is not
    buildable without cargo; the C restatement of model.rs::forward in oracle/ stands in), rank 0
    only. A step is one whole decode token: all 36 layers and the tied head over f32 weights
    expanded at load (as Weights::from_vq does), all host threads, at positions ctx, ctx + 1, ...
    over a KV cache holding ctx seeded positions (the prompt itself is not run on the CPU: the
    decode token reads the same cache bytes). W untimed tokens, then exactly K timed tokens."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import oracle
    from spk.model import ModelConfig, synth_weights

    threads = os.cpu_count() or 1
    cfg = ModelConfig()
    t_setup = time.perf_counter()
    W = synth_weights(cfg, seed=1234)
    layers = [{"in_norm": L["in_norm"], "post_norm": L["post_norm"],
               **{n: oracle.decode(L[n]) for n in ("qkv", "attn_gate", "out", "gate", "up", "down")}}
              for L in W["layers"]]
    embed = oracle.q80_dequant(W["embed"], cfg.vocab, cfg.hidden)
    m = oracle.Model(cfg.as_oracle(), layers, embed, W["norm"], args.ctx + args.warmup + args.steps + 1,
                     threads=threads)
    m.fill_kv(args.ctx, 7)
    del W
    t_setup = time.perf_counter() - t_setup
    tok, pos = 1, args.ctx
    for _ in range(args.warmup):
        tok = oracle.argmax(m.forward(tok, pos))
        pos += 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok = oracle.argmax(m.forward(tok, pos))
        pos += 1
    dt = time.perf_counter() - t0
    m.close()
    v = args.steps / dt
    sample = (f"model.rs forward restated in C (oracle/), all 36 layers + tied head, {threads} threads, "
              f"{args.steps} timed tokens at positions {args.ctx}..{pos - 1} after {args.warmup} untimed, "
              f"over a seeded {args.ctx}-position f32 KV cache; load + f32 expansion {t_setup:.0f} s untimed")
    cb = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample}
    line = {"metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights, seeded KV cache)",
            "impl": "reference", "config": {"workload": f"config2: 36-layer VQ decoder batch-1 greedy decode at ctx "
                                                        f"{args.ctx} (CPU, f32 KV)",
                                            "model": "spark-x2.6-4b geometry (random-init), f32 weights",
                                            "global_batch": 1, "seq_len": args.ctx, "parallelism": "cpu"},
            "cpu_baseline": cb, "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference_gemv(args) -> None:
    """--impl reference for configs 0 (`vq`) and the gate+up pair (`vq-pair`): the reference's CPU
    implementation of the GEMV (Stage::dot_row per stage, restated in C in oracle/, "port"), all
    host threads, K timed whole GEMVs over the same seeded matrices and x as our arm. When the
    reference's own GPU kernel file was built here for sm_100a (oracle/_ref/libvqg_ref.so, from
    tools/vq/gpu/decode-gpu.cu by `make -C oracle ref`), its GEMV is timed too, the way the
    reference's runtime runs it (vq-model-gpu.cu:651-660: y zeroed, then one vqg_gemv_launch per
    stage, the DQV3 block kernel chosen by variant 0), over 8 rotating copies with CUDA events,
    and reported as `reference_gpu` beside the CPU line."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import ctypes as C

    import oracle
    from spk import formats as F

    pair = args.workload == "vq-pair"
    ng = 2 if pair else 1
    rows, cols, ncopy = 10240, 2560, 8
    bufs = [F.random_rvq_fast(rows, cols, 4, 4096, 2, seed=g) for g in range(ng)]
    rng = np.random.default_rng(1)
    x = rng.normal(0, 1, cols).astype(np.float32)
    alg = sum(len(b) for b in bufs) + cols * 4 + rows * 4 + (cols * 4 if pair else 0)
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        for b in bufs:
            oracle.gemv_fused(b, x, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for b in bufs:
            oracle.gemv_fused(b, x, threads)
    dt = (time.perf_counter() - t0) / args.steps
    v = alg / dt / 1e9
    sample = (f"Stage::dot_row GEMV restated in C (oracle/), {ng} matrix(es) 10240x2560 DQV3 4x4096x2, {threads} "
              f"threads, {args.steps} timed GEMVs after {args.warmup} untimed")
    ref_gpu = None
    so = os.path.join(ROOT, "oracle", "_ref", "libvqg_ref.so")
    try:
        import torch

        if os.path.exists(so) and torch.cuda.is_available():
            R = C.CDLL(so)
            R.vqg_gemv_launch.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                          C.c_void_p, C.c_int]
            R.vqg_gemv_launch.restype = C.c_int
            dev = torch.device("cuda", 0)
            c = F.parse_container(bufs[0])
            copies = []
            for _ in range(ncopy):   # every stage its own buffer with the 8 zeroed slack bytes
                ts = []
                for b in bufs:
                    for q in range(2):
                        t = torch.zeros(c.stage_bytes + 8, dtype=torch.uint8, device=dev)
                        t[:c.stage_bytes].copy_(torch.frombuffer(bytearray(b[c.stage_offset(q):c.stage_offset(q) +
                                                                             c.stage_bytes]), dtype=torch.uint8))
                        ts.append(t)
                copies.append(ts)
            xd = torch.from_numpy(x).to(dev)
            ys = [torch.zeros(rows, device=dev) for _ in range(ng)]

            def step(k):
                ts = copies[k % ncopy]
                for gi in range(ng):
                    ys[gi].zero_()
                    for q in range(2):
                        if R.vqg_gemv_launch(ts[2 * gi + q].data_ptr(), 4, 4096, rows, cols, 1, xd.data_ptr(),
                                             ys[gi].data_ptr(), 0) != 0:
                            raise RuntimeError("reference vqg_gemv_launch failed")

            for k in range(max(args.warmup, ncopy)):
                step(k)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for k in range(args.steps):
                step(k)
            e1.record()
            e1.synchronize()
            tg = e0.elapsed_time(e1) / 1e3 / args.steps
            want = oracle.gemv_fused(bufs[0], x, threads)
            got = ys[0].cpu().numpy()   # every copy holds the same matrices
            ref_gpu = {"value": alg / tg / 1e9, "unit": "GB/s", "us_per_step": tg * 1e6,
                       "kernel": "the reference's gemv_v3blk_kernel (tools/vq/gpu/decode-gpu.cu:267-301) built for "
                                 "sm_100a, one launch per stage (+ a y memset per matrix), as vq-model-gpu.cu runs it",
                       "check_relL2_vs_oracle": float(np.linalg.norm(got - want) / np.linalg.norm(want))}
    except Exception as e:   # the comparison point is optional; the CPU line stands on its own
        ref_gpu = {"unavailable": f"{type(e).__name__}: {e}"}
    cb = {"value": v, "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample}
    line = {"metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded weights in the reference's formats, x ~ N(0,1))",
            "impl": "reference",
            "config": {"workload": ("decode-step FFN gate+up: two VQ 10240x2560 DQV3 4x4096x2 matrices" if pair else
                                    "config0: VQ decode-GEMV 10240x2560, DQV3 dim 4, K 4096, 2 stages, batch 1"),
                       "rows": rows, "cols": cols},
            "cpu_baseline": cb, "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "reference_gpu": ref_gpu}
    print(json.dumps(line), flush=True)


def run_ours(args) -> None:
    import ctypes as C

    import torch

    import spk
    from spk.model import MATS, DeviceModel, ModelConfig, synth_weights, tp_shard

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
        pg = dist
    cfg = ModelConfig()
    # one model; at N > 1 every rank holds its tensor-parallel shard of it
    W = tp_shard(cfg, synth_weights(cfg, seed=1234), rank, world)
    extra = 64
    m = DeviceModel(cfg, W, max_ctx=args.ctx + args.warmup + args.steps + extra + 2, kv_f16=args.kv == "f16",
                    kv_q8=args.kv == "q8", device=dev)
    del W
    if world > 1:
        m.tp_connect()
    # the synthetic prompt, fed through the host API (teacher-forced)
    prompt = np.random.default_rng(7).integers(0, cfg.vocab, args.ctx)
    prompt_s = None
    if args.fill_kv:
        m.advance_len(args.ctx)
    else:   # the prompt through the chunked tensor-core path (spk_model_prefill), wall clock with its syncs
        if pg:
            pg.barrier()
        t0 = time.perf_counter()
        m.prefill(prompt.tolist(), 0, want_logits=False)
        prompt_s = time.perf_counter() - t0
    ids = torch.zeros(args.warmup + args.steps, dtype=torch.int32, device=dev)
    m.begin(int(prompt[-1]), args.ctx, ids, args.warmup + args.steps)
    m.run(args.warmup)
    m.stream.synchronize()
    if pg:
        pg.barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        ev0.record(m.stream)
        m.run(args.steps)
        ev1.record(m.stream)
        ev1.synchronize()
    torch.cuda.synchronize(dev)
    dt = ev0.elapsed_time(ev1) / 1e3
    if pg:
        t = torch.tensor([dt], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        dt = float(t.item())
        pg.barrier()
    m.advance_len(args.warmup + args.steps)
    pos = m.len
    value = args.steps / dt
    # the greedy ids of the warm-up and timed steps: the same on every rank, and at every N
    # (tensor parallelism changes only the summation order of the logits)
    gen = ids.cpu().numpy().astype("<i4")
    greedy = {"n": int(gen.size), "sha1": hashlib.sha1(gen.tobytes()).hexdigest(), "first8": gen[:8].tolist()}
    if pg:
        h = torch.tensor(np.frombuffer(hashlib.sha1(gen.tobytes()).digest()[:8], dtype="<i8").copy(), device=dev)
        hmax, hmin = h.clone(), h.clone()
        pg.all_reduce(hmax, op=pg.ReduceOp.MAX)
        pg.all_reduce(hmin, op=pg.ReduceOp.MIN)
        greedy["ranks_agree"] = bool(hmax.item() == hmin.item())

    # the dominant kernel, timed live: the fused gate+up VQ GEMV over every layer's weights
    L = spk.lib()
    x = torch.randn(cfg.hidden, device=dev)
    rows_l = m.mats[0]["gate"].rows
    act = torch.zeros(rows_l, device=dev)
    launches = []
    # the model runs the pair through the bank-scheduled table kernel (vq_tab.cu) at >= 4096 rows,
    # when it takes the geometry: time that one, on index words re-laid here the way the model does
    tab_n = L.spk_vq_tab_bytes(4, 4096, rows_l, cfg.hidden, 1) if rows_l >= 4096 else 0
    tabs = []
    for li in range(cfg.layers):
        g, u = m.mats[li]["gate"], m.mats[li]["up"]
        stp = [g.stages[0], g.stages[1], u.stages[0], u.stages[1]]
        st = (C.c_void_p * 4)(*stp)
        lt = None
        if tab_n:
            ws = [torch.empty(tab_n, dtype=torch.uint8, device=dev) for _ in range(4)]
            for p_, w_ in zip(stp, ws):
                spk.check(L.spk_vq_tab_pack(C.c_void_p(p_), 4, 4096, rows_l, cfg.hidden, 1, w_.data_ptr(), None))
            tabs.append(ws)
            lt = (C.c_void_p * 4)(*[w_.data_ptr() for w_ in ws])
        launches.append((st, lt, m.norms[li][1]))
    scr = (torch.zeros(L.spk_vq_tab_scratch_bytes(2, 4, 4096, rows_l, cfg.hidden, 1), dtype=torch.uint8, device=dev)
           if tab_n else None)
    torch.cuda.synchronize(dev)
    sp = C.c_void_p(m.stream.cuda_stream)

    def gateup(k):
        st, lt, nw = launches[k % cfg.layers]
        if lt is not None:
            spk.check(L.spk_vq_tab_gemv(st, lt, 2, 2, 4, 4096, rows_l, cfg.hidden, 1, x.data_ptr(), nw.data_ptr(),
                                        cfg.eps, act.data_ptr(), 0, scr.data_ptr(), sp))
        else:
            spk.check(L.spk_vq_gemv(st, 2, 2, 4, 4096, rows_l, cfg.hidden, 1, x.data_ptr(), nw.data_ptr(), cfg.eps,
                                    act.data_ptr(), 0, sp))

    for k in range(cfg.layers):
        gateup(k)
    reps = 4 * cfg.layers
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record(m.stream)
    for k in range(reps):
        gateup(k)
    k1.record(m.stream)
    k1.synchronize()
    t_kernel = k0.elapsed_time(k1) / 1e3 / reps
    from spk.formats import StageGeom
    stage = StageGeom(4, 4096, rows_l, cfg.hidden, True).stage_bytes
    alg_bytes = 2 * 2 * stage + 2 * cfg.hidden * 4 + rows_l * 4
    peak, peak_kind = hbm_peak()
    achieved = alg_bytes / t_kernel / 1e9
    traffic = (traffic_from_profiles("vq_tab_gate_up_10240x2560x2" if tab_n else "vq_gate_up_gemv_10240x2560x2")
               if world == 1 else None)
    del tabs

    # end to end through the C-ABI with host buffers: token up, next id down, every step
    e2e_n = min(args.steps, 64)
    tok = int(ids[-1].item())
    t0 = time.perf_counter()
    for k in range(e2e_n):
        tok, _ = m.forward(tok, pos + k, want_logits=False)
    e2e = e2e_n / (time.perf_counter() - t0)
    if pg:
        t = torch.tensor([e2e_n / e2e], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e = e2e_n / float(t.item())

    # one more step with per-launch device times (every rank together), summed by kernel
    trace = {}
    for name, us in m.trace():
        trace.setdefault(name, []).append(us)
    trace = {k: {"sum_us": round(float(np.sum(v)), 1), "median_us": round(float(np.median(v)), 2), "n": len(v)}
             for k, v in trace.items()}
    bytes_per_token = m.weight_bytes   # this rank's shard (+ its vocabulary rows of the head below)
    if world > 1:
        bytes_per_token -= len_embed(cfg) - len_embed(cfg) // world
    kv_heads_l = max(cfg.kv_heads // world, 1)
    row = {"f32": cfg.head_dim * 4, "f16": cfg.head_dim * 2, "q8": cfg.head_dim + cfg.head_dim // 16}[args.kv]
    kv_bytes = sum((args.ctx if f else cfg.window) for f in cfg.full) * kv_heads_l * row * 2
    cb = cpu_baseline(args.ctx) if (rank == 0 and world == 1 and not args.no_cpu) else None
    step_launches = L.spk_model_step_launches(C.c_void_p(m.h))
    m.close()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights in DQV3/Q8_0 formats, seeded prompt ids)",
            "config": {"workload": (f"config4: long-context decode at ctx {args.ctx}, {args.kv} KV"
                                    if args.workload == "long" else
                                    f"config2: 36-layer VQ decoder batch-1 greedy decode at ctx {args.ctx}")
                                   + (" (zeroed KV, no prompt run)" if args.fill_kv else ""),
                       "model": f"spark-x2.6-4b geometry, VQ 4x4096x2 trunk, Q8_0 tied head, {args.kv} KV",
                       "global_batch": 1, "seq_len": args.ctx,
                       "parallelism": f"tp{world}" if world > 1 else "single", "l2": "weights 3.2 GB > L2, no flush",
                       "prompt_tok_s": args.ctx / prompt_s if prompt_s else None,
                       "step_bytes_per_gpu": bytes_per_token + kv_bytes,
                       "step_hbm_gbs_per_gpu": (bytes_per_token + kv_bytes) * args.steps / dt / 1e9,
                       "step_trace_rank0": trace},
            "roofline": {"bound": "hbm",
                         "kernel": (("vq_tab.cu vq_tab_kernel" if tab_n else "vq_fast_kernel") +
                                    f" gate+up pair {rows_l}x2560 x2 stages (RMSNorm, GELU), rank 0"),
                         "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "alg_bytes_per_launch": alg_bytes,
                         "us_per_launch": t_kernel * 1e6},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4},
            "gpu_launches": args.steps * step_launches,
            "greedy_ids": greedy,
            "clocks": clk.summary(),
        }
        if cb:
            line["cpu_baseline"] = cb
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()


def hot_replay(g, stream, seconds: float = 0.4) -> None:
    """Enqueue replays of graph `g` for about `seconds` of device time and return without
    waiting, so the timed replay that follows starts on a GPU already at load clocks
    (an idle B200 needs that long to raise its clocks; a short timed region right after
    host work would measure the ramp)."""
    import torch

    with torch.cuda.stream(stream):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        g.replay()
        b.record(stream)
        b.synchronize()
        n = int(seconds * 1e3 / max(a.elapsed_time(b), 1e-3)) + 1
        for _ in range(min(n, 100000)):
            g.replay()


def run_spec(args) -> None:
    """Config 3: speculative decode of the config-2 target at an 8192-token context with the
    5-layer BF16 DSpark draft (624 M parameters, random-init). A round is spec.rs:177-245's:
    the draft proposes a block of 7 at pos0 (spk_draft_block: anchor + 6 mask rows through
    the draft, the target's tied head, the Markov chain on device), the target verifies
    [anchor, 7 proposals] in one M = 8 batch (spk_model_verify), the cache rolls back to the
    accepted prefix, and the draft encodes the committed rows' layer-input captures
    (spk_draft_encode). Acceptance is synthetic: a random-init draft and target agree ~never,
    so a seeded Bernoulli(p) acceptor sets the accepted prefix length k; every kernel runs on
    the real proposals. value = committed tokens (k + 1 per round) per second of wall time
    for whole rounds (draft + verify + encode, host round trips included)."""
    import ctypes as C

    import torch

    import spk
    from spk.draft import DeviceDraft, DraftConfig, synth_draft
    from spk.model import DeviceModel, ModelConfig, synth_weights

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg, dcfg = ModelConfig(), DraftConfig()
    W = synth_weights(cfg, seed=1234)
    ctx, nd, p_acc = args.ctx, dcfg.draft_max(), args.accept
    max_ctx = ctx + (args.warmup + args.steps) * (nd + 1) + 16
    m = DeviceModel(cfg, W, max_ctx=max_ctx, kv_f16=True, device=dev)
    del W
    DW = synth_draft(dcfg, seed=4321)
    d = DeviceDraft(dcfg, DW, max_ctx=max_ctx, device=dev, stream=m.stream)
    del DW
    m.enable_capture(dcfg.target_layers)
    d.use_target_head(m)
    caps, stride = m.captures()
    m.advance_len(ctx)   # a zeroed KV cache at the context length (the attention reads the same bytes)
    d.encode_features(caps, stride, ctx - dcfg.swa_window - 1, ctx)   # the draft's window before pos0
    embed = m.embed_dev.data_ptr()
    rng = np.random.default_rng(11)
    pos, anchor, emitted = ctx, 5, 0
    t_draft = t_verify = t_enc = 0.0

    def round_(count):
        nonlocal pos, anchor, emitted, t_draft, t_verify, t_enc
        t0 = time.perf_counter()
        props, _, _ = d.decode_block(embed, cfg.vocab, anchor, pos, nd)
        t1 = time.perf_counter()
        ids, _ = m.verify([anchor] + props[dcfg.i_beg():], pos)
        t2 = time.perf_counter()
        acc = rng.random(nd) < p_acc
        k = int(np.argmin(acc)) if not acc.all() else nd   # the acceptor's prefix length
        m.rollback(pos + k + 1)
        d.encode_features(caps, stride, pos, pos + k + 1)
        m.stream.synchronize()
        t3 = time.perf_counter()
        pos, anchor = pos + k + 1, ids[k]
        if count:
            emitted += k + 1
            t_draft += t1 - t0
            t_verify += t2 - t1
            t_enc += t3 - t2

    for _ in range(args.warmup):
        round_(False)
    torch.cuda.synchronize(dev)
    rounds = args.steps
    with Clocks(0) as clk:
        t0 = time.perf_counter()
        for _ in range(rounds):
            round_(True)
        t = time.perf_counter() - t0
    # the verify forward alone, device-timed (one batch of 8 at the current position)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(m.stream)
    spk.check(spk.lib().spk_model_verify(m.h, (C.c_int * 8)(*([anchor] * 8)), 8, pos, None, None))
    e1.record(m.stream)
    e1.synchronize()
    m.rollback(pos)
    t_vdev = e0.elapsed_time(e1) / 1e3
    peak, peak_kind = hbm_peak()
    step_bytes = m.weight_bytes
    draft_bytes = d.weight_bytes
    d.close()
    m.close()
    value = emitted / t
    per = lambda x: x / rounds * 1e3
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": 1, "steps": rounds, "warmup": args.warmup,
            "ms_per_step": t / rounds * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded random-init target and draft, seeded Bernoulli acceptor)",
            "config": {"workload": f"config3: speculative rounds (DSpark 5-layer BF16 draft, block 7; M=1+7 verify) "
                                   f"of the config-2 target at ctx {ctx}, acceptance {p_acc}",
                       "model": "spark-x2.6-4b geometry, VQ 4x4096x2 trunk, Q8_0 tied head, f16 KV; draft 624M bf16",
                       "accepted_per_round": emitted / rounds, "draft_ms": per(t_draft), "verify_ms": per(t_verify),
                       "encode_ms": per(t_enc), "verify_ms_device": t_vdev * 1e3,
                       "verify_weight_gbs": step_bytes / t_vdev / 1e9, "draft_weight_bytes": draft_bytes},
            "roofline": {"bound": "hbm", "kernel": "verify forward (VQ mma.sync GEMMs, M=8)",
                         "achieved": step_bytes / t_vdev / 1e9, "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": step_bytes / t_vdev / 1e9 / peak, "traffic": None},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 4 * (2 + nd + 1),
                    "d2h_bytes_per_step": 4 * (2 * nd + 1 + nd + 1)},
            "gpu_launches": rounds * ((16 + 8 * cfg.layers) + (2 + 8 * dcfg.layers + 1 + nd) + (3 + 2 * dcfg.layers)),
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)


def _gemv_line(args, workload: str, value: float, alg: int, t_launch: float, kernel: str, traffic, extra: dict,
               e2e: float, h2d: int, d2h: int, cb, clk, launches: int) -> dict:
    peak, peak_kind = hbm_peak()
    ach = alg / t_launch / 1e9
    line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": alg / value / 1e6, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded weights in the reference's formats, x ~ N(0,1))",
            "config": {"workload": workload, **extra},
            "roofline": {"bound": "hbm", "kernel": kernel, "achieved": ach, "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": ach / peak, "traffic": traffic, "alg_bytes_per_launch": alg,
                         "us_per_launch": t_launch * 1e6},
            "e2e": {"value": e2e, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches, "clocks": clk.summary()}
    if cb:
        line["cpu_baseline"] = cb
    return line


def run_vq_gemv(args) -> None:
    """Config 0: one VQ decode-GEMV, W 10240x2560 as DQV3 4x4096x2 (seeded codebooks and
    indices), x ~ N(0,1) seed 1, y fp32 [10240]. A step is the whole GEMV (both stages, one
    launch) through the bank-scheduled table kernel (spk_vq_tab_gemv, the decode step's kernel
    for matrices of 8192 rows and more; its index words re-laid once at load by
    spk_vq_tab_pack, outside the timed region). Eight copies of the container (158 MB > L2)
    rotate, so every step reads HBM. `--workload vq-pair` runs the decode step's dominant
    launch instead: the FFN gate and up matrices (two such containers) in one launch with the
    RMSNorm prologue and the gelu(gate)*up epilogue."""
    import ctypes as C

    import torch

    import spk
    from spk import formats as F

    pair = args.workload == "vq-pair"
    ng = 2 if pair else 1
    rows, cols, ncopy = 10240, 2560, 8
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = spk.lib()
    bufs = [F.random_rvq_fast(rows, cols, 4, 4096, 2, seed=g) for g in range(ng)]
    c = F.parse_container(bufs[0])
    nw_bytes = L.spk_vq_tab_bytes(4, 4096, rows, cols, 1)
    copies = []
    for _ in range(ncopy):
        ts = [spk.dev_bytes(b[c.stage_offset(s):c.stage_offset(s) + c.stage_bytes], dev) for b in bufs for s in range(2)]
        ws = [torch.empty(nw_bytes, dtype=torch.uint8, device=dev) for _ in ts]
        for t, w in zip(ts, ws):
            spk.check(L.spk_vq_tab_pack(t.data_ptr(), 4, 4096, rows, cols, 1, w.data_ptr(), None))
        copies.append(((C.c_void_p * len(ts))(*[t.data_ptr() for t in ts]), ts,
                       (C.c_void_p * len(ws))(*[w.data_ptr() for w in ws]), ws))
    scr = torch.zeros(L.spk_vq_tab_scratch_bytes(ng, 4, 4096, rows, cols, 1), dtype=torch.uint8, device=dev)
    rng = np.random.default_rng(1)
    x_host = rng.normal(0, 1, cols).astype(np.float32)
    x = torch.from_numpy(x_host).to(dev)
    nw = torch.from_numpy((1.0 + 0.1 * rng.normal(0, 1, cols)).astype(np.float32)).to(dev) if pair else None
    y = torch.zeros(rows, device=dev)
    torch.cuda.synchronize(dev)
    s = torch.cuda.Stream(dev)
    sp = C.c_void_p(s.cuda_stream)
    alg = sum(len(b) for b in bufs) + cols * 4 + rows * 4 + (cols * 4 if pair else 0)

    def step(k, stream):
        cp = copies[k % ncopy]
        spk.check(L.spk_vq_tab_gemv(cp[0], cp[2], 2, ng, 4, 4096, rows, cols, 1, x.data_ptr(),
                                    nw.data_ptr() if pair else None, 1e-6, y.data_ptr(), 0, scr.data_ptr(), stream))

    for k in range(args.warmup):
        step(k, sp)
    s.synchronize()
    # the K timed launches as one CUDA graph, so host launch cost stays out of the kernel time
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for k in range(args.steps):
            step(k, C.c_void_p(s.cuda_stream))
    g.replay()
    s.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(0) as clk:
        hot_replay(g, s)
        with torch.cuda.stream(s):
            e0.record(s)
            g.replay()
            e1.record(s)
        e1.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / args.steps
    del g
    # end to end: x from pinned host memory up, the GEMV, y down, every step
    xh = torch.from_numpy(x_host).pin_memory()
    yh = torch.empty(rows, dtype=torch.float32).pin_memory()
    n = min(args.steps, 64)
    t0 = time.perf_counter()
    with torch.cuda.stream(s):
        for k in range(n):
            x.copy_(xh, non_blocking=True)
            step(k, sp)
            yh.copy_(y, non_blocking=True)
            s.synchronize()
    e2e = alg * n / (time.perf_counter() - t0) / 1e9
    cb = None
    if not args.no_cpu:
        import oracle

        thr = os.cpu_count() or 1
        for b in bufs:
            oracle.gemv_fused(b, x_host, thr)
        reps = 5
        t0 = time.perf_counter()
        for _ in range(reps):
            for b in bufs:
                oracle.gemv_fused(b, x_host, thr)
        tc = (time.perf_counter() - t0) / reps
        cb = {"value": alg / tc / 1e9, "unit": "GB/s", "cores": thr, "kind": "port",
              "sample": f"Stage::dot_row fused GEMV restated in C (oracle/), the full {ng}-matrix workload, "
                        f"{reps} reps, {tc * 1e3:.1f} ms each"}
    if pair:
        workload = "decode-step FFN gate+up: two VQ 10240x2560 DQV3 4x4096x2 matrices, RMSNorm in, gelu(g)*u out"
        kernel, prof = "vq_tab_kernel gate+up 10240x2560 x2 stages", "vq_tab_gate_up_10240x2560x2"
    else:
        workload = "config0: VQ decode-GEMV 10240x2560, DQV3 dim 4, K 4096, 2 stages, batch 1"
        kernel, prof = "vq_tab_kernel 10240x2560 x2 stages", "vq_tab_10240x2560x2"
    line = _gemv_line(args, workload, alg / t / 1e9, alg, t, kernel, traffic_from_profiles(prof),
                      {"rows": rows, "cols": cols, "container_bytes": [len(b) for b in bufs],
                       "l2": f"{ncopy} rotating copies, {ncopy * alg / 1e6:.0f} MB > L2"},
                      e2e, cols * 4, rows * 4, cb, clk, args.steps)
    print(json.dumps(line), flush=True)


GGML_SHAPES = [("q6k", "q", 4096, 2560), ("q6k", "k", 1024, 2560), ("q6k", "v", 1024, 2560),
               ("q6k", "o", 2560, 4096), ("q6k", "gate", 10240, 2560), ("q6k", "up", 10240, 2560),
               ("q6k", "down", 2560, 10240), ("q80", "head", 131072, 2560)]


def run_ggml(args) -> None:
    """Config 1: the Q6_K dequant-GEMV over every trunk shape and the Q8_0 GEMV over the
    131072x2560 tied head (the tensor-core head the decode step runs, with its argmax), batch 1, W ~ N(0, 0.02^2) quantized with the block rules (Q6_K by
    the package's encoder, Q8_0 by ggml's d = max|w|/127 statistics), x ~ N(0,1). A step is
    one pass over the eight matrices; value = their bytes over the sum of their per-launch times."""
    import ctypes as C

    import torch

    import spk
    from spk import formats as F

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = spk.lib()
    rng = np.random.default_rng(0)
    mats = []
    for fmt, name, rows, cols in GGML_SHAPES:
        if fmt == "q6k":
            blob = F.quantize_q6_k(rng.normal(0, 0.02, (rows, cols)).astype(np.float32))
        else:
            blob = F.synth_q8_0(rows, cols, seed=1)
        x_host = rng.normal(0, 1, cols).astype(np.float32)
        mats.append({"fmt": fmt, "name": name, "rows": rows, "cols": cols, "blob": blob,
                     "w": spk.dev_bytes(blob, dev), "x_host": x_host, "x": torch.from_numpy(x_host).to(dev),
                     "y": torch.zeros(rows, device=dev), "alg": len(blob) + 4 * cols + 4 * rows})
    # each matrix rotates over copies totalling > 2x L2, so back-to-back launches read HBM. The Q8_0
    # head runs as the decode step runs it: its blocks re-laid once (outside the timed region) into
    # the tensor-core tile layout (spk_q80_tile), then spk_q80_tile_head over those tiles.
    for m in mats:
        if m["fmt"] == "q80":
            t = torch.zeros(L.spk_q80_tile_bytes(m["rows"], m["cols"]), dtype=torch.uint8, device=dev)
            spk.check(L.spk_q80_tile(m["w"].data_ptr(), m["rows"], m["cols"], t.data_ptr(), None))
            m["w"] = t
            m["scratch"] = torch.zeros(L.spk_q80_tile_scratch_bytes(), dtype=torch.uint8, device=dev)
            m["amax"] = torch.zeros(1, dtype=torch.int32, device=dev)
        m["copies"] = [m["w"]] + [m["w"].clone() for _ in range(-(-256_000_000 // m["w"].numel()) - 1)]
    torch.cuda.synchronize(dev)
    s = torch.cuda.Stream(dev)
    sp = C.c_void_p(s.cuda_stream)

    def launch(m, k=0, stream=sp):
        w = m["copies"][k % len(m["copies"])]
        if m["fmt"] == "q6k":
            spk.check(L.spk_q6k_gemv(w.data_ptr(), m["rows"], m["cols"], m["x"].data_ptr(), None, 0.0,
                                     m["y"].data_ptr(), 0, stream))
        else:
            spk.check(L.spk_q80_tile_head(w.data_ptr(), m["rows"], m["cols"], 1, m["x"].data_ptr(), m["cols"], None,
                                          0.0, m["y"].data_ptr(), m["rows"], m["amax"].data_ptr(),
                                          m["scratch"].data_ptr(), stream))

    for k in range(args.warmup):
        for m in mats:
            launch(m, k)
    s.synchronize()
    # per matrix: its `steps` launches captured as one CUDA graph, timed with events around the replay
    per = np.zeros(len(mats))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(0) as clk:
        for i, m in enumerate(mats):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for k in range(args.steps):
                    launch(m, k, C.c_void_p(s.cuda_stream))
            hot_replay(g, s, 0.2)
            with torch.cuda.stream(s):
                e0.record(s)
                g.replay()
                e1.record(s)
            e1.synchronize()
            per[i] = e0.elapsed_time(e1) / 1e3 / args.steps
            del g
    alg = sum(m["alg"] for m in mats)
    t = float(per.sum())
    xh = [torch.from_numpy(m["x_host"]).pin_memory() for m in mats]
    yh = [torch.empty(m["rows"], dtype=torch.float32).pin_memory() for m in mats]
    n = min(args.steps, 16)
    t0 = time.perf_counter()
    with torch.cuda.stream(s):
        for _ in range(n):
            for i, m in enumerate(mats):
                m["x"].copy_(xh[i], non_blocking=True)
                launch(m)
                yh[i].copy_(m["y"], non_blocking=True)
            s.synchronize()
    e2e = alg * n / (time.perf_counter() - t0) / 1e9
    cb = None
    if not args.no_cpu:
        import oracle

        thr = os.cpu_count() or 1
        tc = 0.0
        for m in mats:
            fn = oracle.q6k_gemv if m["fmt"] == "q6k" else oracle.q80_gemv
            fn(m["blob"], m["rows"], m["cols"], m["x_host"], thr)
            t0 = time.perf_counter()
            fn(m["blob"], m["rows"], m["cols"], m["x_host"], thr)
            tc += time.perf_counter() - t0
        cb = {"value": alg / tc / 1e9, "unit": "GB/s", "cores": thr, "kind": "port",
              "sample": f"ggml dequantize_row_q6_K / q8_0 order GEMV restated in C (oracle/), one pass over the "
                        f"eight matrices, {tc * 1e3:.1f} ms"}
    peak, _ = hbm_peak()
    detail = {f"{m['fmt']}_{m['name']}_{m['rows']}x{m['cols']}": {"us": per[i] * 1e6,
                                                                   "gbs": m["alg"] / per[i] / 1e9,
                                                                   "frac": m["alg"] / per[i] / 1e9 / peak}
              for i, m in enumerate(mats)}
    head = len(mats) - 1
    line = _gemv_line(args, "config1: Q6_K trunk shapes + Q8_0 131072x2560 head, batch 1", alg / t / 1e9,
                      mats[head]["alg"], per[head], "q8t_head_kernel Q8_0 131072x2560 (tensor-core tile layout, fused argmax)",
                      traffic_from_profiles("q8t_head_131072x2560"),
                      {"matrices": detail, "l2": "each matrix rotates over copies totalling > 256 MB"},
                      e2e, sum(4 * m["cols"] for m in mats), sum(4 * m["rows"] for m in mats), cb, clk,
                      args.steps * len(mats))
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "long", "spec", "vq", "vq-pair", "ggml"],
                    help="decode: config 2 (default); long: config 4 (ctx 131072, q8_0 KV, zeroed KV cache); "
                         "spec: config 3 speculative rounds, draft + verify (ctx 8192, synthetic acceptance); "
                         "vq: config 0 GEMV; vq-pair: the FFN gate+up launch; ggml: config 1 Q6_K/Q8_0 sweep")
    ap.add_argument("--kv", default=None, choices=["f32", "f16", "q8"],
                    help="decode KV cache type (default f16; long: q8)")
    ap.add_argument("--fill-kv", action="store_true",
                    help="decode: start at ctx over a zeroed KV cache instead of running the prompt "
                         "(the same attention bytes per step; for profiler captures)")
    ap.add_argument("--accept", type=float, default=0.25, help="spec: acceptance probability per proposal")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline sample")
    args = ap.parse_args()
    if args.workload == "long":
        # a 131072-token prompt through decode steps would take ~10 minutes: the cache
        # starts zeroed at the context length (the attention reads the same bytes)
        args.fill_kv = True
        args.no_cpu = True
        if args.ctx == 4096:
            args.ctx = 131072
        args.kv = args.kv or "q8"
    args.kv = args.kv or "f16"
    if args.workload == "spec" and args.ctx == 4096:
        args.ctx = 8192
    if args.warmup < 3:
        ap.error("at least 3 warm-up steps")
    if args.impl == "reference" and args.workload in ("vq", "vq-pair"):
        run_reference_gemv(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload in ("vq", "vq-pair"):
        run_vq_gemv(args)
    elif args.workload == "ggml":
        run_ggml(args)
    elif args.workload == "spec":
        run_spec(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
