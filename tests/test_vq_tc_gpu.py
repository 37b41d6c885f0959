"""The VQ GEMM of a token batch on the tcgen05 tensor cores (vq_tc.cu, spk_vq_lut_gemm) against
the CPU oracle: Y[n] = sum_s gain_s W_s RMSNorm?(X[n]) for the verify batch (ntok <= 8) and
prompt chunks (up to 128 tokens), at the decode step's matrix shapes and small ragged ones.
Tolerance: relative L2 <= 1e-5 per token row (activations as f16 hi/lo pairs, ~22 bits, products
exact in f32; the north-star bound on GEMM outputs is 1e-3)."""
import ctypes as C

import numpy as np
import pytest

import oracle
from spk import formats as F

pytestmark = pytest.mark.gpu
TOL = 1e-5


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def rms(x, w, eps=1e-6):
    x = x.astype(np.float64)
    return (x / np.sqrt(np.mean(x * x) + eps) * w).astype(np.float32)


def _setup(cuda, rows, cols, ns, seed, fast=True):
    import torch

    import spk

    L = spk.lib()
    buf = (F.random_rvq_fast(rows, cols, 4, 4096, ns, seed=seed) if fast else
           F.random_rvq(rows, cols, 4, 4096, ns, seed=seed, unit_gains=False))
    c = F.parse_container(buf)
    st = [spk.dev_bytes(buf[c.stage_offset(s):c.stage_offset(s) + c.stage_bytes], cuda) for s in range(ns)]
    n = L.spk_vq_lut_bytes(4, 4096, rows, cols, 1)
    lt = [torch.zeros(n, dtype=torch.uint8, device=cuda) for _ in range(ns)]
    for a, w in zip(st, lt):
        spk.check(L.spk_vq_lut_pack(C.c_void_p(a.data_ptr()), 4, 4096, rows, cols, 1, w.data_ptr(), None))
    return buf, st, lt


def _run(cuda, lt, rows, cols, X, nw, y0, acc):
    import torch

    import spk

    L = spk.lib()
    ntok = X.shape[0]
    scr = torch.zeros(L.spk_vq_lut_gemm_scratch_bytes(rows, cols, ntok), dtype=torch.uint8, device=cuda)
    ptrs = (C.c_void_p * len(lt))(*[t.data_ptr() for t in lt])
    xd = torch.from_numpy(X).to(cuda)
    wd = torch.from_numpy(nw).to(cuda) if nw is not None else None
    outs = []
    for _ in range(2):   # twice: the second call reuses the scratch the first left behind
        yd = torch.from_numpy(y0.copy()).to(cuda)
        spk.check(L.spk_vq_lut_gemm(ptrs, len(lt), 4, 4096, rows, cols, 1, ntok, xd.data_ptr(), cols,
                                    wd.data_ptr() if wd is not None else None, 1e-6, yd.data_ptr(), rows, acc,
                                    scr.data_ptr(), None))
        torch.cuda.synchronize()
        spk.check(L.spk_check_device_error(), "device error")
        outs.append(yd.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    return outs[0]


@pytest.mark.parametrize("rows,cols", [(6144, 2560), (2560, 4096), (10240, 2560), (2560, 10240)])
@pytest.mark.parametrize("ntok", [1, 3, 8])
def test_batched_gemm_decode_shapes(cuda, rows, cols, ntok):
    buf, st, lt = _setup(cuda, rows, cols, 2, seed=rows + cols)
    W = oracle.decode(buf).astype(np.float64)
    rng = np.random.default_rng(ntok)
    X = rng.normal(0, 1, (ntok, cols)).astype(np.float32)
    got = _run(cuda, lt, rows, cols, X, None, np.zeros((ntok, rows), np.float32), 0)
    want = X.astype(np.float64) @ W.T
    for n in range(ntok):
        assert rel(got[n], want[n]) < TOL, (rows, cols, ntok, n, rel(got[n], want[n]))


@pytest.mark.parametrize("ntok", [16, 64, 128])
def test_batched_gemm_prompt_chunks(cuda, ntok):
    rows, cols = 2048, 2560
    buf, st, lt = _setup(cuda, rows, cols, 2, seed=ntok)
    W = oracle.decode(buf).astype(np.float64)
    rng = np.random.default_rng(ntok + 1)
    X = rng.normal(0, 1, (ntok, cols)).astype(np.float32)
    nw = (1 + 0.1 * rng.normal(0, 1, cols)).astype(np.float32)
    y0 = rng.normal(0, 1, (ntok, rows)).astype(np.float32)
    got = _run(cuda, lt, rows, cols, X, nw, y0, 1)
    for n in range(ntok):
        want = y0[n] + W @ rms(X[n], nw).astype(np.float64)
        assert rel(got[n], want) < TOL, (ntok, n, rel(got[n], want))


@pytest.mark.parametrize("rows,cols,ns", [(200, 512, 2), (33, 256, 2), (1000, 2560, 1), (136, 4096, 2)])
def test_batched_gemm_ragged(cuda, rows, cols, ns):
    buf, st, lt = _setup(cuda, rows, cols, ns, seed=rows, fast=False)
    W = oracle.decode(buf).astype(np.float64)
    rng = np.random.default_rng(rows)
    X = rng.normal(0, 1, (5, cols)).astype(np.float32)
    got = _run(cuda, lt, rows, cols, X, None, np.zeros((5, rows), np.float32), 0)
    for n in range(5):
        assert rel(got[n], W @ X[n].astype(np.float64)) < TOL


def test_batched_gemm_refuses(cuda):
    import spk

    L = spk.lib()
    p = (C.c_void_p * 2)(None, None)
    assert L.spk_vq_lut_gemm(p, 2, 4, 4096, 64, 256, 1, 129, None, 256, None, 0.0, None, 64, 0, None, None) == -1
    assert L.spk_vq_lut_gemm_scratch_bytes(64, 250, 4) == 0
