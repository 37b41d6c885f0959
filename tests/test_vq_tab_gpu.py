"""The bank-scheduled table look-up VQ GEMV (vq_tab.cu, spk_vq_tab_*) against the CPU oracle.

* CPU: a numpy restatement of what the re-lay must hold — per (slice, row) 8 u16 byte offsets
  16384 (jj mod 4) + 4 idx_jj into a half table (u16 0-3: jj 0-3, u16 4-7: jj 4-7, each half
  in any order) of the row's indices at bytes [12 sl, 12 sl + 12) of its DQV3 stream — and of
  the look-up sum over those words gives oracle.gemv_fused's result.
* GPU: every re-laid word holds exactly its row's 8 (jj, idx) pairs (bit-exact, order free
  within a half),
  and the scheduled order spreads each warp's 8 load steps over the banks (mean per-step
  maximum bank load well below a random order's ~3.5); spk_vq_tab_gemv matches the oracle at
  relative L2 <= 1e-5 (fp32 sums in another order; the north-star bound is 1e-3) for the
  decode step's shapes and their tensor-parallel shards, one and two stages, store /
  accumulate, the RMSNorm prologue and the gelu_erf(gate) * up pair, on repeated calls with
  one scratch (the grid barrier's count carries over), and down to matrices with fewer work
  units than CTAs; geometries it does not take are refused.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from spk import formats as F

GEMV_TOL = 1e-5


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def np_indices(buf: bytes, c: F.Container, s: int) -> np.ndarray:
    """[nsl][rows][8] indices of stage s from its DQV3 row streams (12-bit little-endian)."""
    rows, nsl = c.rows, c.cols // 32
    o = c.stage_offset(s) + 24 + c.nc * 8 + rows * 2
    b = np.frombuffer(buf, np.uint8, rows * nsl * 12, o).reshape(rows, nsl, 4, 3).astype(np.uint32)
    trip = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16)
    return np.stack([trip & 0xFFF, trip >> 12], axis=-1).reshape(rows, nsl, 8).transpose(1, 0, 2)


def np_offsets(idx: np.ndarray) -> np.ndarray:
    """u16 byte offsets into the half tables, in jj order: 16384 (jj mod 4) + 4 idx."""
    return (16384 * (np.arange(8, dtype=np.uint32) % 4) + 4 * idx.astype(np.uint32)).astype(np.uint16)


def np_words(buf: bytes, c: F.Container, s: int, seed: int = 0) -> np.ndarray:
    """A valid re-lay in some order: [nsl][rows][8] u16 offsets, each half's four shuffled
    (any order within a half is a valid word)."""
    w = np_offsets(np_indices(buf, c, s))
    rng = np.random.default_rng(seed)
    perm = np.argsort(rng.random(w.shape[:-1] + (2, 4)), axis=-1) + np.array([0, 4])[:, None]
    return np.take_along_axis(w, perm.reshape(w.shape), axis=-1)


def np_tab_gemv(buf: bytes, c: F.Container, x: np.ndarray) -> np.ndarray:
    rows, nsl = c.rows, c.cols // 32
    y = np.zeros(rows, np.float64)
    for s in range(c.nstages):
        o = c.stage_offset(s) + 24
        cb = np.frombuffer(buf, np.float16, c.nc * 4, o).astype(np.float64).reshape(c.nc, 4)
        gain = np.frombuffer(buf, np.float16, rows, o + c.nc * 8).astype(np.float64)
        w = np_words(buf, c, s, seed=s).astype(np.int64)
        for sl in range(nsl):
            T = (cb @ x[32 * sl:32 * sl + 32].astype(np.float64).reshape(8, 4).T).T.reshape(2, -1)   # [half][jj][code]
            y += gain * (T[0][w[sl, :, :4] // 4].sum(axis=1) + T[1][w[sl, :, 4:] // 4].sum(axis=1))
    return y


def test_tab_restatement_matches_oracle():
    rows, cols = 96, 512
    buf = F.random_rvq(rows, cols, 4, 4096, 2, seed=3, unit_gains=False)
    c = F.parse_container(buf)
    x = np.random.default_rng(1).normal(0, 1, cols).astype(np.float32)
    assert rel(np_tab_gemv(buf, c, x), oracle.gemv_fused(buf, x)) < 1e-6


def _dev_stages(buf, c, cuda):
    import spk

    return [spk.dev_bytes(buf[c.stage_offset(s):c.stage_offset(s) + c.stage_bytes], cuda) for s in range(c.nstages)]


def _packed(bufs, c, cuda):
    import torch

    import spk

    L = spk.lib()
    n = L.spk_vq_tab_bytes(4, c.nc, c.rows, c.cols, 1)
    assert n == c.cols // 32 * c.rows * 16
    out = []
    for b in bufs:
        t = torch.zeros(n, dtype=torch.uint8, device=cuda)
        spk.check(L.spk_vq_tab_pack(b.data_ptr(), 4, c.nc, c.rows, c.cols, 1, t.data_ptr(), None))
        out.append(t)
    return out


@pytest.mark.gpu
def test_tab_pack_holds_each_rows_lookups_and_spreads_banks(cuda):
    import torch

    rows, cols = 1024, 2560
    buf = F.random_rvq(rows, cols, 4, 4096, 2, seed=5, unit_gains=False)
    c = F.parse_container(buf)
    bufs = _dev_stages(buf, c, cuda)
    packed = _packed(bufs, c, cuda)
    torch.cuda.synchronize()
    nsl = cols // 32
    for s in range(2):
        got = packed[s].cpu().numpy().view(np.uint16).reshape(nsl, rows, 8)
        want = np_offsets(np_indices(buf, c, s))
        for h in (slice(0, 4), slice(4, 8)):
            assert np.array_equal(np.sort(got[..., h], axis=-1), np.sort(want[..., h], axis=-1))
        # per warp (32 rows) and load step: the most-loaded bank's count
        banks = ((got >> 2) & 31).reshape(nsl, rows // 32, 32, 8)
        worst = []
        for step in range(8):
            b = banks[..., step]                                    # [nsl][chunk][lane]
            cnt = np.zeros(b.shape[:2] + (32,), np.int32)
            np.add.at(cnt, (np.arange(nsl)[:, None, None], np.arange(rows // 32)[None, :, None], b), 1)
            worst.append(cnt.max(axis=-1))
        sched = float(np.mean(worst))
        rnd = ((want >> 2) & 31).reshape(nsl, rows // 32, 32, 8)
        rworst = []
        for step in range(8):
            cnt = np.zeros(rnd.shape[:2] + (32,), np.int32)
            np.add.at(cnt, (np.arange(nsl)[:, None, None], np.arange(rows // 32)[None, :, None], rnd[..., step]), 1)
            rworst.append(cnt.max(axis=-1))
        natural = float(np.mean(rworst))
        assert sched < 2.45 and natural > 3.0, (sched, natural)


def _run(cuda, bufs, packed, ns, ng, rows, cols, x, w, y0, acc, calls=1, scr=None):
    import torch

    import spk

    L = spk.lib()
    st = (C.c_void_p * len(bufs))(*[b.data_ptr() for b in bufs])
    lt = (C.c_void_p * len(packed))(*[p.data_ptr() for p in packed])
    if scr is None:
        scr = torch.zeros(L.spk_vq_tab_scratch_bytes(ng, 4, 4096, rows, cols, 1), dtype=torch.uint8, device=cuda)
    xd = torch.from_numpy(x).to(cuda)
    wd = torch.from_numpy(w).to(cuda) if w is not None else None
    outs = []
    for _ in range(calls):
        yd = torch.from_numpy(y0.copy()).to(cuda)
        spk.check(L.spk_vq_tab_gemv(st, lt, ns, ng, 4, 4096, rows, cols, 1, xd.data_ptr(),
                                    wd.data_ptr() if wd is not None else None, 1e-6, yd.data_ptr(), acc,
                                    scr.data_ptr(), None))
        torch.cuda.synchronize()
        spk.check(L.spk_check_device_error(), "device error")
        outs.append(yd.cpu().numpy())
    return outs


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols,ns,acc", [(10240, 2560, 2, 0), (6144, 2560, 2, 0), (2560, 4096, 2, 1),
                                              (2560, 10240, 2, 1), (1280, 2560, 2, 0), (2560, 1280, 2, 1),
                                              (1024, 2560, 2, 0), (2560, 512, 2, 1), (4096, 2048, 1, 1),
                                              (32, 64, 2, 0), (96, 256, 1, 1)])
def test_tab_gemv_matches_oracle(cuda, rows, cols, ns, acc):
    buf = F.random_rvq(rows, cols, 4, 4096, ns, seed=rows + cols + ns, unit_gains=False)
    c = F.parse_container(buf)
    rng = np.random.default_rng(rows)
    x = rng.normal(0, 1, cols).astype(np.float32)
    y0 = rng.normal(0, 1, rows).astype(np.float32)
    bufs = _dev_stages(buf, c, cuda)
    got = _run(cuda, bufs, _packed(bufs, c, cuda), ns, 1, rows, cols, x, None, y0, acc, calls=2)
    want = oracle.gemv_fused(buf, x).astype(np.float64) + (y0 if acc else 0)
    for g in got:
        assert rel(g, want) < GEMV_TOL
    assert np.array_equal(got[0], got[1])   # the same summation order on every call


@pytest.mark.gpu
def test_tab_gemv_rmsnorm_prologue(cuda):
    rows, cols = 6144, 2560
    buf = F.random_rvq(rows, cols, 4, 4096, 2, seed=21, unit_gains=False)
    c = F.parse_container(buf)
    rng = np.random.default_rng(4)
    x = rng.normal(0, 3, cols).astype(np.float32)
    w = rng.normal(1, 0.2, cols).astype(np.float32)
    want = oracle.gemv_fused(buf, oracle.rms_norm(x, w, 1e-6))
    bufs = _dev_stages(buf, c, cuda)
    got = _run(cuda, bufs, _packed(bufs, c, cuda), 2, 1, rows, cols, x, w, np.zeros(rows, np.float32), 0)[0]
    assert rel(got, want) < GEMV_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(10240, 2560), (1280, 2560), (96, 512)])
def test_tab_gemv_gate_up_gelu(cuda, rows, cols):
    g_buf = F.random_rvq(rows, cols, 4, 4096, 2, seed=31, unit_gains=False)
    u_buf = F.random_rvq(rows, cols, 4, 4096, 2, seed=32, unit_gains=False)
    cg, cu = F.parse_container(g_buf), F.parse_container(u_buf)
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, cols).astype(np.float32)
    w = rng.normal(1, 0.1, cols).astype(np.float32)
    xn = oracle.rms_norm(x, w, 1e-6)
    g, u = oracle.gemv_fused(g_buf, xn), oracle.gemv_fused(u_buf, xn)
    want = np.array([oracle.lib().orc_gelu(float(a)) for a in g], np.float32) * u
    bufs = _dev_stages(g_buf, cg, cuda) + _dev_stages(u_buf, cu, cuda)
    packed = _packed(bufs[:2], cg, cuda) + _packed(bufs[2:], cu, cuda)
    got = _run(cuda, bufs, packed, 2, 2, rows, cols, x, w, np.zeros(rows, np.float32), 0, calls=2)
    for gv in got:
        assert rel(gv, want) < 1e-4


@pytest.mark.gpu
def test_tab_refuses_other_geometries(cuda):
    import spk

    L = spk.lib()
    assert L.spk_vq_tab_bytes(4, 8192, 334, 1024, 1) == 0    # 13-bit plane
    assert L.spk_vq_tab_bytes(8, 256, 40, 128, 1) == 0       # dim 8
    assert L.spk_vq_tab_bytes(4, 4096, 64, 200, 1) == 0      # 50 index groups: not whole slices
    assert L.spk_vq_tab_bytes(4, 4096, 40, 256, 1) == 0      # rows not a multiple of 32
    assert L.spk_vq_tab_bytes(4, 4096, 10272, 256, 1) == 0   # more rows than the kernel's warps own
    assert L.spk_vq_tab_bytes(4, 512, 64, 96, 0) == 0        # DQVQ
    assert L.spk_vq_tab_gemv(None, None, 2, 1, 4, 4096, 64, 256, 1, None, None, 0.0, None, 0, None, None) == -1
    st = (C.c_void_p * 4)(None, None, None, None)
    assert L.spk_vq_tab_gemv(st, st, 2, 2, 4, 4096, 64, 256, 1, None, None, 0.0, None, 1, None, None) == -1
