"""The B200 tuner: measure this build's GEMV kernels per matrix geometry of an artifact and
write the VQPROF 1 profile the model reads (spk.vqprof, DeviceModel.use_profile).

Mirrors tools/vq-tune/src/main.rs: for every distinct geometry of the artifact's matrices
(manifest order), every kernel that can run it is timed on that matrix's own payload and gated
on agreement (relative L2 <= 1e-4, the tuner's gate, main.rs:107-108) with the reference
ABI's generic warp-per-row kernel (vqg_gemv variant 1, stage by stage); the fastest kernel
that passes becomes the geometry's `gemv` entry. The candidates are this build's own: the
code-word kernel (variant 3 as vqg_gemv numbers it; spk_vq_gemv over all stages in one pass)
and the shared-memory table kernel over re-laid words (SPK_VARIANT_TABLE; spk_vq_tab_*).
The profile is bound to the artifact's fingerprint, the device name and the driver version,
and is written through a temporary file; a profile of another artifact at the path is kept
unless `force` (main.rs:366-373).

Usage: python -m spk.tune DIR [--profile PATH] [--iters N] [--force]
"""
from __future__ import annotations

import argparse
import ctypes as C
import os

import numpy as np

from . import SpkError, check, dev_bytes, lib
from . import formats as F
from . import vqprof as P

GATE_REL = 1e-4


def _rel(a: np.ndarray, b: np.ndarray) -> float:
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _time(fn, iters: int, warmup: int) -> float:
    """Mean device time of one call in microseconds (CUDA events on the current stream)."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / iters


def tune_geometry(buf: bytes, iters: int = 50, warmup: int = 5, device="cuda:0") -> list[dict]:
    """Every runnable candidate for one RQVQ container: [{variant, threads, us, gbs, rel}] with
    the gate applied (rel <= GATE_REL), fastest first."""
    import torch

    L = lib()
    c = F.parse_container(buf)
    g = c.geom
    dim, nc, rows, cols, v3, ns = g.dim, g.nc, c.rows, c.cols, int(g.v3), c.nstages
    stages = [dev_bytes(buf[c.stage_offset(s):c.stage_offset(s) + c.stage_bytes], device) for s in range(ns)]
    ptrs = (C.c_void_p * ns)(*[t.data_ptr() for t in stages])
    x = torch.from_numpy(np.random.default_rng(rows * 7 + cols).normal(0, 1, cols).astype(np.float32)).to(device)
    y = torch.zeros(rows, device=device)

    ref = torch.zeros(rows, device=device)   # the generic kernel, stage by stage (+=)
    for t in stages:
        check(L.vqg_gemv_launch_t(t.data_ptr(), dim, nc, rows, cols, v3, x.data_ptr(), ref.data_ptr(), 1, 256))
    torch.cuda.synchronize()
    want = ref.cpu().numpy()
    payload = ns * c.stage_bytes
    out = []

    def add(variant: int, threads: int, fn) -> None:
        fn()
        torch.cuda.synchronize()
        rel = _rel(y.cpu().numpy(), want)
        if rel > GATE_REL:
            return
        us = _time(fn, iters, warmup)
        out.append({"variant": variant, "threads": threads, "us": us, "gbs": payload / us / 1e3, "rel": rel})

    if L.spk_vq_gemv_fast_ok(ns, 1, dim, nc, rows, cols, v3):
        add(3, 512, lambda: check(L.spk_vq_gemv(ptrs, ns, 1, dim, nc, rows, cols, v3, x.data_ptr(), None, 0.0,
                                                y.data_ptr(), 0, None)))
    nb = L.spk_vq_tab_bytes(dim, nc, rows, cols, v3)
    if nb:
        words = [torch.zeros(nb, dtype=torch.uint8, device=device) for _ in range(ns)]
        for t, w in zip(stages, words):
            check(L.spk_vq_tab_pack(t.data_ptr(), dim, nc, rows, cols, v3, w.data_ptr(), None))
        wptrs = (C.c_void_p * ns)(*[w.data_ptr() for w in words])
        scr = torch.zeros(L.spk_vq_tab_scratch_bytes(1, dim, nc, rows, cols, v3), dtype=torch.uint8, device=device)
        add(P.VARIANT_TABLE, 512, lambda: check(L.spk_vq_tab_gemv(ptrs, wptrs, ns, 1, dim, nc, rows, cols, v3,
                                                                  x.data_ptr(), None, 0.0, y.data_ptr(), 0,
                                                                  scr.data_ptr(), None)))
    if not out:   # neither fast kernel takes it: the generic kernel is the answer
        def generic():
            y.zero_()
            for t in stages:
                check(L.vqg_gemv_launch_t(t.data_ptr(), dim, nc, rows, cols, v3, x.data_ptr(), y.data_ptr(), 1, 256))
        add(1, 256, generic)
    return sorted(out, key=lambda r: r["us"])


def tune(dir: str, profile: str | None = None, iters: int = 50, warmup: int = 5, force: bool = False,
         device="cuda:0", log=print) -> str:
    """Measure every geometry of the artifact in `dir` and write its profile (default
    dir/vq-tune.profile). Returns the path written."""
    fp = P.fingerprint(dir)
    path = profile or os.path.join(dir, "vq-tune.profile")
    if os.path.exists(path) and not force:
        try:
            old = P.load(path)
        except SpkError:
            old = None
        if old is not None and old.artifact != fp:
            raise SpkError(f"{path} belongs to artifact {old.artifact:016x}, this one is {fp:016x}; use force")
    drv = lib().vqg_driver_version()
    prof = P.new(fp, P.device_name(), str(drv))
    seen = set()
    for name, rows, cols, stages, _ in P.read_manifest(dir):
        if stages <= 0:
            continue
        buf = P.read_container(dir, name)
        c = F.parse_container(buf)
        key = (c.geom.dim, c.geom.nc, c.rows, c.cols, int(c.geom.v3))
        if key in seen:
            continue
        seen.add(key)
        res = tune_geometry(buf, iters, warmup, device)
        if not res:
            log(f"{name}: no kernel passed the gate; no entry")
            continue
        best = res[0]
        prof.add_gemv(*key, best["variant"], best["threads"], best["gbs"])
        log(f"{name} {c.rows}x{c.cols}: " + ", ".join(f"v{r['variant']} {r['us']:.1f} us" for r in res))
    P.write(path, prof)
    log(f"profile     {path} ({prof.n} entries)")
    return path


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("dir")
    ap.add_argument("--profile", default=None)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args(argv)
    tune(a.dir, a.profile, a.iters, force=a.force)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
