"""Q6_K / Q8_0 kernels on the GPU, through the C-ABI, against the CPU oracle
and the gguf-py golden fixtures. Dequant is bit-exact; GEMVs are gated at
relative L2 <= 1e-5 (the north-star bound is 1e-3)."""
import os

import numpy as np
import pytest

import oracle
import spk
from spk import formats as F

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
TOL = 1e-5


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def weights(rows, cols, seed):
    return np.random.default_rng(seed).normal(0, 0.02, (rows, cols)).astype(np.float32)


def test_q6k_dequant_bitexact_golden(cuda):
    import torch

    z = np.load(os.path.join(GOLDEN, "q6k.npz"))
    rows, cols = int(z["rows"]), int(z["cols"])
    w = spk.dev_bytes(z["blocks"].tobytes(), cuda)
    out = torch.empty(rows * cols, device=cuda)
    spk.check(spk.lib().spk_q6k_dequant(w.data_ptr(), rows * cols // 256, spk.ptr(out), None))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), z["gguf_dequant"].reshape(-1).view(np.uint32))


def test_q80_dequant_bitexact_golden(cuda):
    import torch

    z = np.load(os.path.join(GOLDEN, "q80.npz"))
    rows, cols = int(z["rows"]), int(z["cols"])
    w = spk.dev_bytes(z["blocks"].tobytes(), cuda)
    out = torch.empty(rows * cols, device=cuda)
    spk.check(spk.lib().spk_q80_dequant(w.data_ptr(), rows * cols // 32, spk.ptr(out), None))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), z["gguf_dequant"].reshape(-1).view(np.uint32))


Q6K_SHAPES = [(4096, 2560), (1024, 2560), (2560, 4096), (10240, 2560), (2560, 10240), (6144, 2560), (16, 2560),
              (7, 256), (33, 768)]


@pytest.mark.parametrize("rows,cols", Q6K_SHAPES)
def test_q6k_gemv_vs_oracle(cuda, rows, cols):
    import torch

    blocks = F.quantize_q6_k(weights(rows, cols, rows + cols))
    x = np.random.default_rng(1).normal(0, 1, cols).astype(np.float32)
    want = oracle.q6k_gemv(blocks, rows, cols, x)
    w = spk.dev_bytes(blocks, cuda)
    xd = torch.from_numpy(x).to(cuda)
    y0 = np.random.default_rng(2).normal(0, 1, rows).astype(np.float32)
    for acc in (0, 1):
        yd = torch.from_numpy(y0).to(cuda)
        spk.check(spk.lib().spk_q6k_gemv(w.data_ptr(), rows, cols, spk.ptr(xd), None, 0.0, spk.ptr(yd), acc, None))
        torch.cuda.synchronize()
        assert rel(yd.cpu().numpy(), want + (y0 if acc else 0)) < TOL


@pytest.mark.parametrize("rows,cols", [(131072 // 8, 2560), (100, 2560), (5, 64)])
def test_q80_gemv_vs_oracle(cuda, rows, cols):
    import torch

    blocks = F.quantize_q8_0(weights(rows, cols, rows))
    x = np.random.default_rng(1).normal(0, 1, cols).astype(np.float32)
    want = oracle.q80_gemv(blocks, rows, cols, x)
    w = spk.dev_bytes(blocks, cuda)
    xd = torch.from_numpy(x).to(cuda)
    yd = torch.zeros(rows, device=cuda)
    spk.check(spk.lib().spk_q80_gemv(w.data_ptr(), rows, cols, spk.ptr(xd), None, 0.0, spk.ptr(yd), 0, None))
    torch.cuda.synchronize()
    assert rel(yd.cpu().numpy(), want) < TOL


def test_q6k_gemv_rmsnorm(cuda):
    import torch

    rows, cols = 1024, 2560
    blocks = F.quantize_q6_k(weights(rows, cols, 3))
    rng = np.random.default_rng(3)
    x = rng.normal(0, 2, cols).astype(np.float32)
    nw = rng.normal(1, 0.1, cols).astype(np.float32)
    want = oracle.q6k_gemv(blocks, rows, cols, oracle.rms_norm(x, nw, 1e-6))
    w = spk.dev_bytes(blocks, cuda)
    yd = torch.zeros(rows, device=cuda)
    xd, nwd = torch.from_numpy(x).to(cuda), torch.from_numpy(nw).to(cuda)   # keep alive until the launch ran
    spk.check(spk.lib().spk_q6k_gemv(w.data_ptr(), rows, cols, spk.ptr(xd), spk.ptr(nwd), 1e-6, spk.ptr(yd), 0, None))
    torch.cuda.synchronize()
    assert rel(yd.cpu().numpy(), want) < TOL


@pytest.mark.parametrize("rows", [131072, 4099])
def test_q80_head_logits_and_argmax(cuda, rows):
    import torch

    cols = 2560
    Wt = weights(rows, cols, 11)
    blocks = F.quantize_q8_0(Wt)
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, cols).astype(np.float32)
    nw = rng.normal(1, 0.1, cols).astype(np.float32)
    xn = oracle.rms_norm(x, nw, 1e-6)
    want = oracle.q80_gemv(blocks, rows, cols, xn)
    w = spk.dev_bytes(blocks, cuda)
    logits = torch.zeros(rows, device=cuda)
    am = torch.full((1,), -1, dtype=torch.int32, device=cuda)
    xd, nwd = torch.from_numpy(x).to(cuda), torch.from_numpy(nw).to(cuda)
    for _ in range(2):   # the finishing counter must reset itself
        spk.check(spk.lib().spk_q80_head(w.data_ptr(), rows, cols, spk.ptr(xd), spk.ptr(nwd), 1e-6, spk.ptr(logits),
                                         spk.ptr(am), None))
        torch.cuda.synchronize()
        got = logits.cpu().numpy()
        assert rel(got, want) < TOL
        assert int(am.item()) == oracle.argmax(got)
    top2 = np.sort(want)[-2:]
    if top2[1] - top2[0] > 1e-4 * abs(top2[1]):
        assert int(am.item()) == oracle.argmax(want)


def test_q80_head_ties_pick_first(cuda):
    import torch

    rows, cols = 4096, 64
    W = np.zeros((rows, cols), np.float32)
    W[[17, 1000, 4000], :] = 0.5          # three identical maximal rows
    blocks = F.quantize_q8_0(W)
    w = spk.dev_bytes(blocks, cuda)
    x = torch.ones(cols, device=cuda)
    logits = torch.zeros(rows, device=cuda)
    am = torch.full((1,), -1, dtype=torch.int32, device=cuda)
    spk.check(spk.lib().spk_q80_head(w.data_ptr(), rows, cols, spk.ptr(x), None, 0.0, spk.ptr(logits), spk.ptr(am),
                                     None))
    torch.cuda.synchronize()
    assert int(am.item()) == 17


def test_q80_row_gather(cuda):
    import torch

    rows, cols = 1000, 2560
    blocks = F.quantize_q8_0(weights(rows, cols, 8))
    D = oracle.q80_dequant(blocks, rows, cols)
    w = spk.dev_bytes(blocks, cuda)
    out = torch.zeros(cols, device=cuda)
    spk.check(spk.lib().spk_q80_row(w.data_ptr(), rows, cols, 123, None, spk.ptr(out), None))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), D[123].view(np.uint32))
    tok = torch.tensor([999], dtype=torch.int32, device=cuda)
    spk.check(spk.lib().spk_q80_row(w.data_ptr(), rows, cols, 0, spk.ptr(tok), spk.ptr(out), None))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), D[999].view(np.uint32))
