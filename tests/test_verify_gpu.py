"""The speculative verify on the GPU: the M <= 8 batched VQ GEMM against the oracle,
and the verify forward against M sequential decode steps (spec.rs:197-249)."""
import ctypes as C

import numpy as np
import pytest

import oracle
from spk import formats as F
from spk.model import DeviceModel, small_config, synth_weights

pytestmark = pytest.mark.gpu
GEMM_TOL = 1e-5     # f16 hi/lo activations carry ~22 bits; north-star tolerance is 1e-3
LOGIT_TOL = 1e-4
EPS_MARGIN = 1e-3


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def rms(x, w, eps=1e-6):
    x = x.astype(np.float64)
    return (x / np.sqrt(np.mean(x * x) + eps) * w).astype(np.float32)


# rows, cols, nc, stages: tensor-core geometries (one pass, K passes, 13-bit plane) and fallbacks
GEMMS = [(1002, 2560, 4096, 2), (300, 4096, 4096, 2), (256, 10240, 4096, 2), (96, 1024, 8192, 2),
         (16, 2560, 4096, 1), (200, 1000, 4096, 2), (64, 512, 4096, 3)]


@pytest.mark.parametrize("geom", GEMMS)
@pytest.mark.parametrize("ntok", [1, 3, 4, 5, 8])
def test_verify_gemm_matches_oracle(cuda, geom, ntok):
    import torch

    import spk

    rows, cols, nc, stages = geom
    buf = F.random_rvq(rows, cols, 4, nc, stages, seed=rows + ntok)
    c = F.parse_container(buf)
    W = oracle.decode(buf).reshape(rows, cols)
    rng = np.random.default_rng(ntok)
    X = rng.normal(0, 1, (ntok, cols)).astype(np.float32)
    nw = (1 + 0.1 * rng.normal(0, 1, cols)).astype(np.float32)
    keep = [spk.dev_bytes(buf[c.stage_offset(s):c.stage_offset(s) + c.stage_bytes], cuda) for s in range(stages)]
    st = (C.c_void_p * stages)(*[t.data_ptr() for t in keep])
    x = torch.from_numpy(X).to(cuda)
    w = torch.from_numpy(nw).to(cuda)
    L = spk.lib()
    for norm in (False, True):
        Y0 = rng.normal(0, 1, (ntok, rows)).astype(np.float32)
        y = torch.from_numpy(Y0).to(cuda)
        torch.cuda.synchronize()
        spk.check(L.spk_verify_gemm(st, stages, 4, nc, rows, cols, 1, ntok, x.data_ptr(), cols,
                                    w.data_ptr() if norm else None, 1e-6, y.data_ptr(), rows, 1, None))
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        for n in range(ntok):
            xin = rms(X[n], nw) if norm else X[n]
            want = Y0[n] + W.astype(np.float64) @ xin.astype(np.float64)
            assert rel(got[n], want) < GEMM_TOL, (geom, ntok, norm, n, rel(got[n], want))


# the config-3 verify batch's matrices at their full size, M = 8 (qkv, out, gate/up, down)
FULL = [(6144, 2560), (2560, 4096), (10240, 2560), (2560, 10240)]


@pytest.mark.parametrize("rows,cols", FULL)
def test_verify_gemm_full_shapes_m8(cuda, rows, cols):
    import torch

    import spk

    buf = F.random_rvq_fast(rows, cols, 4, 4096, 2, seed=rows * 7 + cols)
    c = F.parse_container(buf)
    W = oracle.decode(buf).reshape(rows, cols).astype(np.float64)
    rng = np.random.default_rng(rows + cols)
    X = rng.normal(0, 1, (8, cols)).astype(np.float32)
    keep = [spk.dev_bytes(buf[c.stage_offset(s):c.stage_offset(s) + c.stage_bytes], cuda) for s in range(2)]
    st = (C.c_void_p * 2)(*[t.data_ptr() for t in keep])
    x = torch.from_numpy(X).to(cuda)
    y = torch.zeros(8, rows, device=cuda)
    L = spk.lib()
    spk.check(L.spk_verify_gemm(st, 2, 4, 4096, rows, cols, 1, 8, x.data_ptr(), cols, None, 0.0, y.data_ptr(), rows,
                                0, None))
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    want = X.astype(np.float64) @ W.T
    for n in range(8):
        assert rel(got[n], want[n]) < GEMM_TOL, (rows, cols, n, rel(got[n], want[n]))


def test_verify_gemm_rejects_bad_arguments(cuda):
    import spk

    L = spk.lib()
    st = (C.c_void_p * 2)(None, None)
    assert L.spk_verify_gemm(st, 2, 4, 4096, 64, 512, 1, 9, None, 512, None, 0.0, None, 64, 0, None) == -1
    assert b"tokens" in L.spk_last_error()
    assert L.spk_verify_gemm(st, 2, 4, 4096, 64, 512, 1, 2, None, 512, None, 0.0, None, 64, 0, None) == -1


@pytest.fixture(scope="module")
def small(cuda):
    cfg = small_config()
    return cfg, synth_weights(cfg, seed=3, exact_q80=True)


def test_verify_matches_sequential_steps(small):
    """Verify of 1+7 tokens == 8 decode steps: logits per row, greedy ids, and the cache it
    leaves (a rollback to the accepted prefix, then decode continues as sequentially)."""
    cfg, W = small
    prompt = [5, 17, 301, 42, 4000, 7]
    seq = DeviceModel(cfg, W, max_ctx=64)
    ids, logits, tok = [], [], prompt[0]
    for pos in range(len(prompt) + 10):
        nxt, lg = seq.forward(tok, pos)
        ids.append(nxt)
        logits.append(lg)
        tok = prompt[pos + 1] if pos + 1 < len(prompt) else nxt
    seq.close()
    p0 = len(prompt) - 1
    block = [prompt[-1]] + ids[p0:p0 + 7]   # anchor + 7 proposals: the target's own continuation
    dev = DeviceModel(cfg, W, max_ctx=64)
    for pos in range(p0):
        dev.forward(prompt[pos], pos, want_logits=False)
    for rnd in range(2):   # eager, then from the captured verify graph
        tgt, lg = dev.verify(block, p0, want_logits=True)
        for t in range(8):
            assert rel(lg[t], logits[p0 + t]) < LOGIT_TOL, (rnd, t)
            if tgt[t] != ids[p0 + t]:
                s = np.sort(logits[p0 + t])[-2:]
                assert s[1] - s[0] < EPS_MARGIN
        assert dev.len == p0 + 8
        dev.rollback(p0)
    # a wrong proposal at index 3: k = 3 accepted, the target's token after them, cache at p0 + 4
    bad = list(block[1:])
    bad[3] = (bad[3] + 1) % cfg.vocab
    k, nxt, tgt = dev.spec_round(block[0], bad, p0)
    assert k == 3 and nxt == tgt[3] and dev.len == p0 + 4
    # decoding resumes from the accepted prefix exactly as the sequential run
    for pos in range(p0 + 4, p0 + 8):
        feed = nxt if pos == p0 + 4 else nid
        nid, lg = dev.forward(feed, pos)
        assert rel(lg, logits[pos]) < LOGIT_TOL, pos
    dev.close()


def test_verify_rejects_bad_inputs(small):
    import spk

    cfg, W = small
    dev = DeviceModel(cfg, W, max_ctx=16)
    with pytest.raises(spk.SpkError):
        dev.verify([1] * 9, 0)
    with pytest.raises(spk.SpkError):
        dev.verify([cfg.vocab], 0)
    with pytest.raises(spk.SpkError):
        dev.verify([1, 2], 3)   # skips cached positions
    with pytest.raises(spk.SpkError):
        dev.verify([1] * 8, 12)  # past the cache
    dev.close()


@pytest.mark.parametrize("ntok", [1, 3, 8])
@pytest.mark.parametrize("rows,cols", [(131072, 2560), (1000, 512), (300, 992)])
def test_q80_head_batch_matches_per_row_head(cuda, ntok, rows, cols):
    """spk_q80_head_batch (one pass, tensor cores) against spk_q80_head run row by row:
    logits within GEMM_TOL and the same greedy ids (cols 992 takes the per-row path)."""
    import torch

    import spk

    L = spk.lib()
    w = spk.dev_bytes(F.synth_q8_0(rows, cols, seed=ntok), cuda)
    rng = np.random.default_rng(rows + ntok)
    x = torch.from_numpy(rng.normal(0, 1, (ntok, cols)).astype(np.float32)).to(cuda)
    nw = torch.from_numpy((1 + 0.1 * rng.normal(0, 1, cols)).astype(np.float32)).to(cuda)
    lg = torch.zeros(ntok, rows, device=cuda)
    am = torch.zeros(ntok, dtype=torch.int32, device=cuda)
    ref = torch.zeros(ntok, rows, device=cuda)
    ram = torch.zeros(ntok, dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    for n in range(ntok):
        spk.check(L.spk_q80_head(w.data_ptr(), rows, cols, x[n].data_ptr(), nw.data_ptr(), 1e-6, ref[n].data_ptr(),
                                 ram[n:].data_ptr(), None))
    for _ in range(2):   # the ticket is left reset for the next call
        spk.check(L.spk_q80_head_batch(w.data_ptr(), rows, cols, ntok, x.data_ptr(), cols, nw.data_ptr(), 1e-6,
                                       lg.data_ptr(), rows, am.data_ptr(), None))
        torch.cuda.synchronize()
        for n in range(ntok):
            assert rel(lg[n].cpu().numpy(), ref[n].cpu().numpy()) < GEMM_TOL
        a, b = am.cpu().numpy(), ram.cpu().numpy()
        for n in range(ntok):
            if a[n] != b[n]:   # only a near-tie may differ
                r = ref[n].cpu().numpy()
                assert abs(r[a[n]] - r[b[n]]) < 1e-5 * abs(r[b[n]]) + 1e-6
