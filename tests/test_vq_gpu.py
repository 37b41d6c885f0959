"""VQ kernels on the GPU, through the C-ABI, against the CPU oracle.

Tolerances: dequant is bit-exact (integer index work + one rounded f32 mul/add);
GEMV outputs are fp32 accumulations in a different order than the CPU's, gated
at relative L2 <= 1e-5 here (the north-star bound is 1e-3).
"""
import ctypes as C

import numpy as np
import pytest

import oracle
import spk
from spk import formats as F

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-5


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def stage_ptrs(dev_buf, c: F.Container):
    base = dev_buf.data_ptr()
    return [base + c.stage_offset(s) for s in range(c.nstages)]


def stage_bufs(buf: bytes, c: F.Container, device):
    """Each stage in its own device buffer with zeroed slack (the load_mat layout,
    vq-model-gpu.cu:278-288), returned with its device pointer."""
    out = []
    for s in range(c.nstages):
        o = c.stage_offset(s)
        out.append(spk.dev_bytes(buf[o:o + c.stage_bytes], device))
    return out


GEOMS = [
    # rows, cols, dim, nc, stages, v3   (fast path where dim 4 / 12-13 bit / cols/128 in {4,8,16,20}*k)
    (10240, 2560, 4, 4096, 2, True),    # config 0 (FFN up shape)
    (6144, 2560, 4, 4096, 2, True),     # qkv
    (2560, 4096, 4, 4096, 2, True),     # out_proj (k-split 2)
    (2560, 10240, 4, 4096, 2, True),    # down_proj (k-split 4)
    (16, 2560, 4, 4096, 2, True),       # g_proj
    (1002, 512, 4, 4096, 2, True),      # ragged tiles, F=4
    (1001, 512, 4, 4096, 2, True),      # odd rows: 2-aligned stream -> generic
    (334, 1024, 4, 8192, 2, True),      # 13-bit plane, F=8
    (64, 2048, 4, 8192, 1, True),       # plane, F=16
    (50, 256, 4, 1024, 2, True),        # 10-bit stream -> generic
    (40, 128, 8, 256, 2, True),         # dim 8 -> generic
    (37, 96, 4, 512, 2, False),         # DQVQ 9-bit -> generic
    (20, 64, 4, 256, 1, False),         # DQVQ 8-bit -> generic
    (17, 200, 4, 4096, 2, True),        # nidx_row 50: not whole 32-groups -> generic
    (64, 16384, 4, 4096, 2, True),      # F=16, k-split 8: x wider than one staging batch
]


@pytest.mark.parametrize("geom", GEOMS, ids=[f"{g[0]}x{g[1]}d{g[2]}k{g[3]}s{g[4]}{'v3' if g[5] else 'v2'}" for g in GEOMS])
def test_spk_vq_gemv_all_stages_vs_oracle(cuda, geom):
    import torch

    rows, cols, dim, nc, st, v3 = geom
    buf = F.random_rvq(rows, cols, dim, nc, st, seed=rows + cols, unit_gains=False, v3=v3)
    c = F.parse_container(buf)
    x = np.random.default_rng(1).normal(0, 1, cols).astype(np.float32)
    want = oracle.gemv_fused(buf, x)
    bufs = stage_bufs(buf, c, cuda)
    ptrs = (C.c_void_p * c.nstages)(*[b.data_ptr() for b in bufs])
    xd = torch.from_numpy(x).to(cuda)
    y0 = np.random.default_rng(2).normal(0, 1, rows).astype(np.float32)
    for accumulate in (0, 1):
        yd = torch.from_numpy(y0).to(cuda)
        spk.check(spk.lib().spk_vq_gemv(ptrs, c.nstages, 1, dim, nc, rows, cols, int(v3), spk.ptr(xd), None, 0.0,
                                        spk.ptr(yd), accumulate, None))
        torch.cuda.synchronize()
        spk.check(spk.lib().spk_check_device_error())
        got = yd.cpu().numpy()
        ref = want + (y0 if accumulate else 0)
        assert rel(got, ref) < GEMV_TOL, (accumulate, rel(got, ref))


@pytest.mark.parametrize("geom", GEOMS[:6] + GEOMS[7:9], ids=[f"{g[0]}x{g[1]}" for g in GEOMS[:6] + GEOMS[7:9]])
def test_fast_path_is_taken(cuda, geom):
    rows, cols, dim, nc, st, v3 = geom
    assert spk.lib().spk_vq_gemv_fast_ok(st, 1, dim, nc, rows, cols, int(v3)) == 1


@pytest.mark.parametrize("variant", [0, 1, 2, 3])
@pytest.mark.parametrize("geom", [GEOMS[0], GEOMS[7], GEOMS[9], GEOMS[11]], ids=["cfg0", "plane", "10bit", "v2"])
def test_vqg_gemv_per_stage_variants(cuda, geom, variant):
    """The reference ABI: one stage per call, y accumulates; caller loops stages."""
    import torch

    rows, cols, dim, nc, st, v3 = geom
    L = spk.lib()
    buf = F.random_rvq(rows, cols, dim, nc, st, seed=5, unit_gains=False, v3=v3)
    c = F.parse_container(buf)
    x = np.random.default_rng(3).normal(0, 1, cols).astype(np.float32)
    bufs = stage_bufs(buf, c, cuda)
    xd = torch.from_numpy(x).to(cuda)
    yd = torch.zeros(rows, device=cuda)
    if not L.vqg_gemv_ready(dim, nc, rows, cols, int(v3), variant):
        # an illegal variant is an error, never a silent fallback (decode-gpu.cu:814-818)
        rc = L.vqg_gemv_launch(bufs[0].data_ptr(), dim, nc, rows, cols, int(v3), spk.ptr(xd), spk.ptr(yd), variant)
        assert rc == -1 and b"does not take" in L.vqg_decode_error()
        return
    want = oracle.gemv_fused(buf, x)
    ms = C.c_double()
    for b in bufs:
        spk.check(L.vqg_gemv(b.data_ptr(), dim, nc, rows, cols, int(v3), spk.ptr(xd), spk.ptr(yd), variant, 1,
                             C.byref(ms)))
    torch.cuda.synchronize()
    assert rel(yd.cpu().numpy(), want) < GEMV_TOL
    # launch form, same result
    yd2 = torch.zeros(rows, device=cuda)
    for b in bufs:
        spk.check(L.vqg_gemv_launch_t(b.data_ptr(), dim, nc, rows, cols, int(v3), spk.ptr(xd), spk.ptr(yd2), variant,
                                      128))
    torch.cuda.synchronize()
    assert rel(yd2.cpu().numpy(), want) < GEMV_TOL


@pytest.mark.parametrize("geom", GEOMS[:1] + GEOMS[5:], ids=lambda g: f"{g[0]}x{g[1]}d{g[2]}k{g[3]}")
def test_vqg_dequant_bitexact(cuda, geom):
    import torch

    rows, cols, dim, nc, st, v3 = geom
    buf = F.random_rvq(rows, cols, dim, nc, st, seed=9, unit_gains=False, v3=v3)
    c = F.parse_container(buf)
    want = oracle.decode(buf)
    bufs = stage_bufs(buf, c, cuda)
    out = torch.zeros(rows * cols, device=cuda)
    ms = C.c_double()
    for b in bufs:
        spk.check(spk.lib().vqg_dequant(b.data_ptr(), dim, nc, rows, cols, int(v3), spk.ptr(out), 1, C.byref(ms)))
    torch.cuda.synchronize()
    got = out.cpu().numpy().reshape(rows, cols)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # row dequant: a few rows, bit-exact
    for r in (0, rows // 2, rows - 1):
        o = torch.zeros(cols, device=cuda)
        for b in bufs:
            spk.check(spk.lib().vqg_row_dequant(b.data_ptr(), dim, nc, rows, cols, int(v3), r, spk.ptr(o)))
        torch.cuda.synchronize()
        assert np.array_equal(o.cpu().numpy().view(np.uint32), want[r].view(np.uint32))


@pytest.mark.parametrize("rows,cols", [(2048, 2560), (64, 16384)])
def test_spk_vq_gemv_rmsnorm_prologue(cuda, rows, cols):
    """The RMSNorm prologue; 16384 columns take the staging loop for x wider than one batch."""
    import torch

    buf = F.random_rvq(rows, cols, 4, 4096, 2, seed=21, unit_gains=False)
    c = F.parse_container(buf)
    rng = np.random.default_rng(4)
    x = rng.normal(0, 3, cols).astype(np.float32)
    w = rng.normal(1, 0.2, cols).astype(np.float32)
    xn = oracle.rms_norm(x, w, 1e-6)
    want = oracle.gemv_fused(buf, xn)
    bufs = stage_bufs(buf, c, cuda)
    ptrs = (C.c_void_p * 2)(*[b.data_ptr() for b in bufs])
    xd, wd = torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda)
    yd = torch.zeros(rows, device=cuda)
    spk.check(spk.lib().spk_vq_gemv(ptrs, 2, 1, 4, 4096, rows, cols, 1, spk.ptr(xd), spk.ptr(wd), 1e-6, spk.ptr(yd), 0,
                                    None))
    torch.cuda.synchronize()
    assert rel(yd.cpu().numpy(), want) < GEMV_TOL


@pytest.mark.parametrize("rows,cols", [(10240, 2560), (300, 512)])
def test_spk_vq_gemv_gate_up_gelu(cuda, rows, cols):
    import torch

    g_buf = F.random_rvq(rows, cols, 4, 4096, 2, seed=31, unit_gains=False)
    u_buf = F.random_rvq(rows, cols, 4, 4096, 2, seed=32, unit_gains=False)
    cg, cu = F.parse_container(g_buf), F.parse_container(u_buf)
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, cols).astype(np.float32)
    w = rng.normal(1, 0.1, cols).astype(np.float32)
    xn = oracle.rms_norm(x, w, 1e-6)
    g = oracle.gemv_fused(g_buf, xn)
    u = oracle.gemv_fused(u_buf, xn)
    want = np.array([oracle.lib().orc_gelu(float(a)) for a in g], np.float32) * u
    bufs = stage_bufs(g_buf, cg, cuda) + stage_bufs(u_buf, cu, cuda)
    ptrs = (C.c_void_p * 4)(*[b.data_ptr() for b in bufs])
    xd, wd = torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda)
    yd = torch.zeros(rows, device=cuda)
    spk.check(spk.lib().spk_vq_gemv(ptrs, 2, 2, 4, 4096, rows, cols, 1, spk.ptr(xd), spk.ptr(wd), 1e-6, spk.ptr(yd), 0,
                                    None))
    torch.cuda.synchronize()
    assert rel(yd.cpu().numpy(), want) < 1e-4


@pytest.mark.parametrize("ntok", [1, 7, 8, 9, 64])
def test_vqg_prefill_vs_oracle(cuda, ntok):
    import torch

    rows, cols = 512, 2560
    buf = F.random_rvq(rows, cols, 4, 4096, 2, seed=41, unit_gains=False)
    c = F.parse_container(buf)
    X = np.random.default_rng(6).normal(0, 1, (ntok, cols)).astype(np.float32)
    want = np.stack([oracle.gemv_fused(buf, X[t]) for t in range(ntok)])
    bufs = stage_bufs(buf, c, cuda)
    xT = torch.from_numpy(np.ascontiguousarray(X.T)).to(cuda)
    yd = torch.zeros(ntok * rows, device=cuda)
    ms = C.c_double()
    for b in bufs:
        spk.check(spk.lib().vqg_prefill(b.data_ptr(), 4, 4096, rows, cols, 1, spk.ptr(xT), ntok, spk.ptr(yd), 1,
                                        C.byref(ms), 0))
    torch.cuda.synchronize()
    assert rel(yd.cpu().numpy().reshape(ntok, rows), want) < GEMV_TOL


def test_vqg_gemv_f32(cuda):
    import torch

    rng = np.random.default_rng(7)
    W = rng.normal(0, 1, (300, 1000)).astype(np.float32)
    x = rng.normal(0, 1, 1000).astype(np.float32)
    Wd, xd = torch.from_numpy(W).to(cuda), torch.from_numpy(x).to(cuda)
    yd = torch.zeros(300, device=cuda)
    ms = C.c_double()
    spk.check(spk.lib().vqg_gemv_f32(spk.ptr(Wd), spk.ptr(xd), spk.ptr(yd), 300, 1000, 1, C.byref(ms)))
    torch.cuda.synchronize()
    assert rel(yd.cpu().numpy(), oracle.matvec(W, x)) < GEMV_TOL


def test_error_paths(cuda):
    L = spk.lib()
    b = spk.dev_bytes(b"\0" * 64, cuda)
    assert L.vqg_gemv_launch(b.data_ptr(), 4, 16384, 8, 64, 1, None, None, 0) == -1
    assert b"13 index bits" in L.vqg_decode_error()
    assert L.vqg_gemv_launch(b.data_ptr(), 4, 4096, 0, 64, 1, None, None, 0) == -1
    assert L.vqg_gemv_launch_t(b.data_ptr(), 4, 4096, 8, 64, 1, None, None, 0, 48) == -1
    assert L.vqg_row_dequant(b.data_ptr(), 4, 4096, 8, 64, 1, 8, None) == -1
    assert L.vqg_prefill_launch(b.data_ptr(), 4, 4096, 8, 64, 1, None, 0, None, 0) == -1
    name = C.create_string_buffer(128)
    assert L.vqg_device_name(name, 128) == 0 and b"B200" in name.value
    assert L.vqg_driver_version() > 0
