"""The Q8_0 head that allocates nothing (spk_q80_head_noalloc), through the C-ABI.

It exists for callers that cannot call cudaMalloc — code inside a CUDA-graph capture,
real-time loops that must not stall on an allocation, host frameworks that own all
device memory — and keeps its scratch in a fixed array inside the library. Its output
must equal the allocating entry point's (spk_q80_head) on the same inputs, within the
GEMV tolerance these tests use, on two calls in a row (the second call reuses the
array the first one left behind), and match the CPU oracle's GEMV and first-max argmax. This file sorts last so a stop-at-first-failure run
has already run every other test; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

import oracle
import spk
from spk import formats as F

pytestmark = pytest.mark.gpu
TOL = 1e-5


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("rows,cols", [(131072, 2560), (4099, 64)], ids=["head-fast-path", "head-generic-path"])
def test_noalloc_head_matches_allocating_head_twice(cuda, rows, cols):
    import torch

    rng = np.random.default_rng(rows + cols)
    blocks = F.quantize_q8_0(rng.normal(0, 0.02, (rows, cols)).astype(np.float32))
    w = spk.dev_bytes(blocks, cuda)
    x = torch.from_numpy(rng.normal(0, 1, cols).astype(np.float32)).to(cuda)
    nw = torch.from_numpy(rng.normal(1, 0.1, cols).astype(np.float32)).to(cuda)
    L = spk.lib()

    ref_logits = torch.zeros(rows, device=cuda)
    ref_arg = torch.full((1,), -1, dtype=torch.int32, device=cuda)
    spk.check(L.spk_q80_head(w.data_ptr(), rows, cols, x.data_ptr(), nw.data_ptr(), 1e-6, ref_logits.data_ptr(),
                             ref_arg.data_ptr(), None), "allocating head")
    torch.cuda.synchronize()
    want, want_arg = ref_logits.cpu().numpy(), int(ref_arg.item())
    # the CPU oracle's GEMV (ggml's dequantize_row_q8_0 restated) and first-max argmax, directly
    xn = oracle.rms_norm(x.cpu().numpy(), nw.cpu().numpy(), 1e-6)
    o_logits = oracle.q80_gemv(blocks, rows, cols, xn)

    for call in range(2):
        logits = torch.zeros(rows, device=cuda)
        arg = torch.full((1,), -1, dtype=torch.int32, device=cuda)
        spk.check(L.spk_q80_head_noalloc(w.data_ptr(), rows, cols, x.data_ptr(), nw.data_ptr(), 1e-6,
                                         logits.data_ptr(), arg.data_ptr(), None), f"no-alloc head, call {call}")
        torch.cuda.synchronize()
        spk.check(L.spk_check_device_error(), "device error")
        got = logits.cpu().numpy()
        assert rel(got, want) < TOL, call
        assert int(arg.item()) == want_arg, call
        assert rel(got, o_logits) < TOL, call
        assert int(arg.item()) == oracle.argmax(got), call
        if np.sort(o_logits)[-2] < o_logits.max() - 1e-3 * max(1.0, abs(float(o_logits.max()))):
            assert int(arg.item()) == oracle.argmax(o_logits), call


def test_noalloc_head_rejects_bad_arguments(cuda):
    import torch

    L = spk.lib()
    w = spk.dev_bytes(F.quantize_q8_0(np.zeros((64, 64), np.float32)), cuda)
    x = torch.zeros(64, device=cuda)
    y = torch.zeros(64, device=cuda)
    assert L.spk_q80_head_noalloc(w.data_ptr(), 64, 64, x.data_ptr(), None, 0.0, y.data_ptr(), None, None) == -1
    assert L.spk_q80_head_noalloc(w.data_ptr(), 64, 60, x.data_ptr(), None, 0.0, y.data_ptr(), None, None) == -1


@pytest.mark.parametrize("rows,cols", [(131072, 2560), (4099, 64)], ids=["head-fast-path", "head-generic-path"])
def test_noalloc_head_inside_a_graph_capture(cuda, rows, cols):
    """Its stated use: called once eagerly, then inside a CUDA-graph capture on a caller
    stream; two replays give the allocating head's logits and argmax."""
    import torch

    rng = np.random.default_rng(rows + 3 * cols)
    blocks = F.quantize_q8_0(rng.normal(0, 0.02, (rows, cols)).astype(np.float32))
    w = spk.dev_bytes(blocks, cuda)
    x = torch.from_numpy(rng.normal(0, 1, cols).astype(np.float32)).to(cuda)
    nw = torch.from_numpy(rng.normal(1, 0.1, cols).astype(np.float32)).to(cuda)
    L = spk.lib()
    ref_logits = torch.zeros(rows, device=cuda)
    ref_arg = torch.full((1,), -1, dtype=torch.int32, device=cuda)
    spk.check(L.spk_q80_head(w.data_ptr(), rows, cols, x.data_ptr(), nw.data_ptr(), 1e-6, ref_logits.data_ptr(),
                             ref_arg.data_ptr(), None), "allocating head")
    torch.cuda.synchronize()
    want, want_arg = ref_logits.cpu().numpy(), int(ref_arg.item())

    s = torch.cuda.Stream()
    logits = torch.zeros(rows, device=cuda)
    arg = torch.full((1,), -1, dtype=torch.int32, device=cuda)
    call = lambda: spk.check(L.spk_q80_head_noalloc(w.data_ptr(), rows, cols, x.data_ptr(), nw.data_ptr(), 1e-6,
                                                    logits.data_ptr(), arg.data_ptr(), s.cuda_stream), "no-alloc head")
    with torch.cuda.stream(s):
        call()   # eagerly first: the one-time set-up happens outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        call()
    for rep in range(2):
        logits.zero_()
        arg.fill_(-1)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        spk.check(L.spk_check_device_error(), "device error")
        assert rel(logits.cpu().numpy(), want) < TOL, rep
        assert int(arg.item()) == want_arg, rep
    del g
