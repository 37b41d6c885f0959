"""The table look-up VQ GEMV (vq_lut.cu, spk_vq_lut_*) against the CPU oracle.

* CPU: a numpy restatement of the re-lay (code words, gains, then the 8 indices at bytes
  [12 sl, 12 sl + 12) of each DQV3 row stream as a 12-byte record at [sl][row]) and of the
  look-up sum
  (T[jj][c] = cb[c] . x[4(8 sl + jj) ..]) gives oracle.gemv_fused's result.
* GPU: spk_vq_lut_pack is bit-exact against that re-lay; spk_vq_lut_gemv matches the oracle
  at relative L2 <= 1e-5 (fp32 sums in another order; the north-star bound is 1e-3) for the
  decode step's shapes, one and two stages, store / accumulate, the RMSNorm prologue and
  the gelu_erf(gate) * up pair; geometries it does not take are refused.
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


def np_pack(buf: bytes, c: F.Container, s: int) -> np.ndarray:
    """Stage s re-laid for the table kernel: its code words (32 KB) in the table builder's order
    (u32 word (block, t, g) = the f16 pair (cb[16 block + g][t], cb[16 block + g + 8][t])), the
    code words in their own order (32 KB), its gains (rows padded to a multiple of 8 with zeros, then to 16 bytes), then the index stream
    slice-major: record [sl][row] = bytes [12 sl, 12 sl + 12) of the row's DQV3 stream (rows
    padded with zeros)."""
    rows, nidx = c.rows, c.cols // 4
    rows8, nsl, mrow = (rows + 7) // 8 * 8, nidx // 8, nidx * 3 // 2
    o = c.stage_offset(s) + 24
    cb = np.frombuffer(buf, np.uint16, c.nc * 4, o).reshape(c.nc // 16, 2, 8, 4)   # [block][half][g][t]
    cw = (cb[:, 0].astype(np.uint32) | (cb[:, 1].astype(np.uint32) << 16)).transpose(0, 2, 1)   # [block][t][g]
    gains = np.zeros((rows8 * 2 + 15) // 16 * 16, np.uint8)
    gains[:rows * 2] = np.frombuffer(buf, np.uint8, rows * 2, o + c.nc * 8)
    st = np.frombuffer(buf, np.uint8, rows * mrow, o + c.nc * 8 + rows * 2).reshape(rows, nsl, 12)
    rec = np.zeros((nsl, rows8, 12), np.uint8)
    rec[:, :rows] = st.transpose(1, 0, 2)
    cbn = np.frombuffer(buf, np.uint8, c.nc * 8, o)
    return np.concatenate([np.ascontiguousarray(cw).view(np.uint8).reshape(-1), cbn, gains, rec.reshape(-1)])


def np_indices(buf: bytes, c: F.Container, s: int) -> np.ndarray:
    """[nsl][rows][8] indices from the re-laid records (12-bit little-endian fields)."""
    rows, nsl = c.rows, c.cols // 32
    rows8 = (rows + 7) // 8 * 8
    w = np_pack(buf, c, s)
    off = 2 * c.nc * 8 + (rows8 * 2 + 15) // 16 * 16
    b = w[off:].reshape(nsl, rows8, 4, 3).astype(np.uint32)[:, :rows]
    trip = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16)            # two indices per 3 bytes
    return np.stack([trip & 0xFFF, trip >> 12], axis=-1).reshape(nsl, rows, 8)


def np_lut_gemv(buf: bytes, c: F.Container, x: np.ndarray) -> np.ndarray:
    rows, nsl = c.rows, c.cols // 32
    y = np.zeros(rows, np.float64)
    for s in range(c.nstages):
        o = c.stage_offset(s) + 24
        cb = np.frombuffer(buf, np.float16, c.nc * 4, o).astype(np.float64).reshape(c.nc, 4)
        gain = np.frombuffer(buf, np.float16, rows, o + c.nc * 8).astype(np.float64)
        W = np_indices(buf, c, s).astype(np.int64)
        for sl in range(nsl):
            T = cb @ x[32 * sl:32 * sl + 32].astype(np.float64).reshape(8, 4).T   # [code][jj]
            for jj in range(8):
                y += gain * T[W[sl, :, jj], jj]
    return y


def test_lut_restatement_matches_oracle():
    rows, cols = 96, 512
    buf = F.random_rvq(rows, cols, 4, 4096, 2, seed=3, unit_gains=False)
    c = F.parse_container(buf)
    x = np.random.default_rng(1).normal(0, 1, cols).astype(np.float32)
    assert rel(np_lut_gemv(buf, c, x), oracle.gemv_fused(buf, x)) < 1e-6


def _dev_stages(buf, c, cuda):
    import spk

    return [spk.dev_bytes(buf[c.stage_offset(s):c.stage_offset(s) + c.stage_bytes], cuda) for s in range(c.nstages)]


def _packed(bufs, c, cuda):
    import torch

    import spk

    L = spk.lib()
    n = L.spk_vq_lut_bytes(4, c.nc, c.rows, c.cols, 1)
    rows8 = (c.rows + 7) // 8 * 8
    assert n == 2 * c.nc * 8 + (rows8 * 2 + 15) // 16 * 16 + c.cols // 32 * rows8 * 12
    out = []
    for b in bufs:
        t = torch.zeros(n, dtype=torch.uint8, device=cuda)
        spk.check(L.spk_vq_lut_pack(b.data_ptr(), 4, c.nc, c.rows, c.cols, 1, t.data_ptr(), None))
        out.append(t)
    return out


@pytest.mark.gpu
def test_lut_pack_is_bit_exact(cuda):
    import torch

    rows, cols = 1000, 2560
    buf = F.random_rvq(rows, cols, 4, 4096, 2, seed=5, unit_gains=False)
    c = F.parse_container(buf)
    bufs = _dev_stages(buf, c, cuda)
    packed = _packed(bufs, c, cuda)
    torch.cuda.synchronize()
    for s in range(2):
        want = np_pack(buf, c, s)
        got = packed[s].cpu().numpy()
        assert got.size == want.size and np.array_equal(got, want)


def _run(cuda, bufs, packed, ns, ng, rows, cols, x, w, y0, acc):
    import torch

    import spk

    L = spk.lib()
    st = (C.c_void_p * len(bufs))(*[b.data_ptr() for b in bufs])
    lt = (C.c_void_p * len(packed))(*[p.data_ptr() for p in packed])
    scr = torch.zeros(L.spk_vq_lut_scratch_bytes(ng, 4, 4096, rows, cols, 1), dtype=torch.uint8, device=cuda)
    xd = torch.from_numpy(x).to(cuda)
    wd = torch.from_numpy(w).to(cuda) if w is not None else None
    yd = torch.from_numpy(y0.copy()).to(cuda)
    spk.check(L.spk_vq_lut_gemv(st, lt, ns, ng, 4, 4096, rows, cols, 1, xd.data_ptr(), wd.data_ptr() if wd is not None
                                else None, 1e-6, yd.data_ptr(), acc, scr.data_ptr(), None))
    torch.cuda.synchronize()
    return yd.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols,ns,acc", [(10240, 2560, 2, 0), (6144, 2560, 2, 0), (2560, 4096, 2, 1),
                                              (2560, 10240, 2, 1), (300, 512, 1, 0), (4096, 2048, 1, 1),
                                              (33, 256, 2, 0)])
def test_lut_gemv_matches_oracle(cuda, rows, cols, ns, acc):
    buf = F.random_rvq(rows, cols, 4, 4096, ns, seed=rows + cols + ns, unit_gains=False)
    c = F.parse_container(buf)
    rng = np.random.default_rng(rows)
    x = rng.normal(0, 1, cols).astype(np.float32)
    y0 = rng.normal(0, 1, rows).astype(np.float32)
    bufs = _dev_stages(buf, c, cuda)
    got = _run(cuda, bufs, _packed(bufs, c, cuda), ns, 1, rows, cols, x, None, y0, acc)
    want = oracle.gemv_fused(buf, x).astype(np.float64) + (y0 if acc else 0)
    assert rel(got, want) < GEMV_TOL


@pytest.mark.gpu
def test_lut_gemv_rmsnorm_prologue(cuda):
    rows, cols = 6144, 2560
    buf = F.random_rvq(rows, cols, 4, 4096, 2, seed=21, unit_gains=False)
    c = F.parse_container(buf)
    rng = np.random.default_rng(4)
    x = rng.normal(0, 3, cols).astype(np.float32)
    w = rng.normal(1, 0.2, cols).astype(np.float32)
    want = oracle.gemv_fused(buf, oracle.rms_norm(x, w, 1e-6))
    bufs = _dev_stages(buf, c, cuda)
    got = _run(cuda, bufs, _packed(bufs, c, cuda), 2, 1, rows, cols, x, w, np.zeros(rows, np.float32), 0)
    assert rel(got, want) < GEMV_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(10240, 2560), (300, 512)])
def test_lut_gemv_gate_up_gelu(cuda, rows, cols):
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
    got = _run(cuda, bufs, packed, 2, 2, rows, cols, x, w, np.zeros(rows, np.float32), 0)
    assert rel(got, want) < 1e-4


@pytest.mark.gpu
def test_lut_refuses_other_geometries(cuda):
    import spk

    L = spk.lib()
    assert L.spk_vq_lut_bytes(4, 8192, 334, 1024, 1) == 0    # 13-bit plane
    assert L.spk_vq_lut_bytes(8, 256, 40, 128, 1) == 0       # dim 8
    assert L.spk_vq_lut_bytes(4, 4096, 17, 200, 1) == 0      # 50 index groups: not whole slices
    assert L.spk_vq_lut_bytes(4, 512, 37, 96, 0) == 0        # DQVQ
    assert L.spk_vq_lut_gemv(None, None, 2, 1, 4, 4096, 64, 256, 1, None, None, 0.0, None, 0, None, None) == -1
    st = (C.c_void_p * 2)(None, None)
    assert L.spk_vq_lut_gemv_t(st, st, 2, 1, 4, 4096, 64, 256, 1, None, None, 0.0, None, 0, None, 1024, None) == -1


@pytest.mark.gpu
@pytest.mark.parametrize("threads", [0, 512])
def test_lut_gemv_block_sizes(cuda, threads):
    import torch

    import spk

    rows, cols = 10240, 2560
    buf = F.random_rvq(rows, cols, 4, 4096, 2, seed=77, unit_gains=False)
    c = F.parse_container(buf)
    x = np.random.default_rng(8).normal(0, 1, cols).astype(np.float32)
    bufs = _dev_stages(buf, c, cuda)
    packed = _packed(bufs, c, cuda)
    L = spk.lib()
    st = (C.c_void_p * 2)(*[b.data_ptr() for b in bufs])
    lt = (C.c_void_p * 2)(*[p.data_ptr() for p in packed])
    scr = torch.zeros(L.spk_vq_lut_scratch_bytes(1, 4, 4096, rows, cols, 1), dtype=torch.uint8, device=cuda)
    xd, yd = torch.from_numpy(x).to(cuda), torch.zeros(rows, device=cuda)
    spk.check(L.spk_vq_lut_gemv_t(st, lt, 2, 1, 4, 4096, rows, cols, 1, xd.data_ptr(), None, 0.0, yd.data_ptr(), 0,
                                  scr.data_ptr(), threads, None))
    torch.cuda.synchronize()
    assert rel(yd.cpu().numpy(), oracle.gemv_fused(buf, x)) < GEMV_TOL
    assert L.spk_vq_lut_gemv_t(st, lt, 2, 1, 4, 4096, rows, cols, 1, xd.data_ptr(), None, 0.0, yd.data_ptr(), 0,
                               scr.data_ptr(), 256, None) == -1
