"""The CPU oracle pinned to implementations it did not write (no GPU needed).

* VQ decode: bit-exact against the reference's own tools/vq/decode.c output
  stored in tests/golden (and, when oracle/_ref/decode was built here, live).
* Q6_K / Q8_0 dequant: bit-exact against gguf-py's block decoders (fixtures).
* Q8_0 quantizer: byte-exact against gguf-py's (ggml's reference rule).
"""
import glob
import os
import struct
import tempfile

import numpy as np
import pytest

import oracle
from spk import formats as F

from conftest import GOLDEN

VQ_FIX = sorted(glob.glob(os.path.join(GOLDEN, "vq_*.npz")))


@pytest.mark.parametrize("path", VQ_FIX, ids=[os.path.basename(p) for p in VQ_FIX])
def test_vq_decode_bitexact_vs_reference_decode_c(path):
    z = np.load(path)
    W = oracle.decode(z["container"].tobytes())
    R = z["ref_decoded"]
    assert W.shape == R.shape
    assert np.array_equal(W.view(np.uint32), R.view(np.uint32))


@pytest.mark.parametrize("path", VQ_FIX, ids=[os.path.basename(p) for p in VQ_FIX])
def test_vq_matvec_checksum_vs_reference(path):
    """decode.c `matvec` prints sum and norm of y = W x (%.6f); the oracle's decode
    plus a serial row dot reproduces both to the printed precision."""
    z = np.load(path)
    W = oracle.decode(z["container"].tobytes())
    x = z["x"]
    y = np.empty(W.shape[0], np.float32)
    for r in range(W.shape[0]):
        acc = np.float32(0)
        for c in range(W.shape[1]):
            acc = np.float32(acc + np.float32(W[r, c] * x[c]))
        y[r] = acc
    s = float(np.sum(y.astype(np.float64)))
    n = float(np.sqrt(np.sum(y.astype(np.float64) ** 2)))
    assert abs(s - float(z["ref_matvec_sum"])) <= 2e-6 + 1e-6 * abs(s)
    assert abs(n - float(z["ref_matvec_norm"])) <= 2e-6 + 1e-6 * abs(n)


@pytest.mark.parametrize("path", VQ_FIX, ids=[os.path.basename(p) for p in VQ_FIX])
def test_fused_dot_row_matches_decoded_matvec(path):
    """Stage::dot_row (fused) and decode-then-dot differ only in summation order."""
    z = np.load(path)
    buf = z["container"].tobytes()
    W = oracle.decode(buf).astype(np.float64)
    y = oracle.gemv_fused(buf, z["x"])
    ref = W @ z["x"].astype(np.float64)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-5


def test_q6k_dequant_bitexact_vs_gguf():
    z = np.load(os.path.join(GOLDEN, "q6k.npz"))
    rows, cols = int(z["rows"]), int(z["cols"])
    W = oracle.q6k_dequant(z["blocks"], rows, cols)
    assert np.array_equal(W.view(np.uint32), z["gguf_dequant"].view(np.uint32))


def test_q80_dequant_bitexact_vs_gguf():
    z = np.load(os.path.join(GOLDEN, "q80.npz"))
    rows, cols = int(z["rows"]), int(z["cols"])
    W = oracle.q80_dequant(z["blocks"], rows, cols)
    assert np.array_equal(W.view(np.uint32), z["gguf_dequant"].view(np.uint32))


def test_q80_quantizer_matches_gguf():
    z = np.load(os.path.join(GOLDEN, "q80.npz"))
    assert np.array_equal(np.frombuffer(F.quantize_q8_0(z["weights"]), np.uint8), z["gguf_quant"])


def test_q6k_quantizer_roundtrip_quality():
    rng = np.random.default_rng(3)
    W = rng.normal(0, 0.02, (32, 512)).astype(np.float32)
    D = oracle.q6k_dequant(F.quantize_q6_k(W), 32, 512)
    rel = np.linalg.norm(D - W) / np.linalg.norm(W)
    assert rel < 0.03   # the reference reports 1.79% on a real matrix


@pytest.mark.skipif(not os.path.exists(oracle.REF_DECODE), reason="oracle/_ref/decode not built here")
@pytest.mark.parametrize("geom", [(32, 512, 4, 4096, 2, True), (16, 256, 4, 8192, 2, True),
                                  (8, 96, 4, 512, 3, False), (8, 64, 8, 256, 1, True)])
def test_vq_decode_live_vs_reference(geom):
    rows, cols, dim, nc, st, v3 = geom
    buf = F.random_rvq(rows, cols, dim, nc, st, seed=rows * 7 + nc, unit_gains=False, v3=v3)
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "c.bin")
        with open(p, "wb") as f:
            f.write(buf)
        R = oracle.ref_decode_dump(p, os.path.join(d, "o.f32")).reshape(rows, cols)
    W = oracle.decode(buf)
    assert np.array_equal(W.view(np.uint32), R.view(np.uint32))


def test_container_layout_matches_reference_formula():
    """Stage sizes follow build-vq-gpu.c:56-64 (DQV3) and vq_qc_bytes.h:14-22 (DQVQ)."""
    for (rows, cols, dim, nc, v3) in [(10240, 2560, 4, 4096, True), (2560, 10240, 4, 4096, True),
                                       (6144, 2560, 4, 8192, True), (100, 40, 4, 1024, True),
                                       (100, 40, 4, 512, False), (100, 40, 4, 256, False)]:
        g = F.StageGeom(dim, nc, rows, cols, v3)
        nidx_row = cols // dim
        bits = F.index_bits(nc)
        if v3:
            mb = min(bits, 12)
            want = 24 + nc * dim * 2 + rows * 2 + rows * ((nidx_row * mb + 7) // 8) + \
                (rows * ((nidx_row + 7) // 8) if bits > 12 else 0)
        else:
            nidx = rows * nidx_row
            want = 16 + nc * dim * 2 + rows * 2 + (nidx if bits == 8 else (nidx * bits + 7) // 8 + 1)
        assert g.stage_bytes == want
    # config 0: 19,767,376 bytes (2 stages + 32-byte header, 6.03 bpw)
    assert 32 + 2 * F.StageGeom(4, 4096, 10240, 2560, True).stage_bytes == 19767376


def test_container_rejections():
    buf = bytearray(F.random_rvq(8, 64, 4, 4096, 2, seed=1))
    with pytest.raises(ValueError):
        oracle.decode(bytes(buf[:-1]))                 # truncated
    bad = bytearray(buf)
    bad[0:4] = b"XXXX"
    with pytest.raises(ValueError):
        oracle.decode(bytes(bad))                      # magic
    bad = bytearray(buf)
    struct.pack_into("<Q", bad, 24, 12345)
    with pytest.raises(ValueError):
        oracle.decode(bytes(bad))                      # payload count
    with pytest.raises(ValueError):
        F.v3_pack(np.zeros(4 * 16384, np.uint16), np.zeros(8, np.uint16), np.zeros((8, 16), np.int64),
                  8, 64, 4, 16384)                     # DQV3 is at most 13 bits


def test_rms_norm_f64_sum():
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, 2560).astype(np.float32)
    w = rng.normal(1, 0.1, 2560).astype(np.float32)
    out = oracle.rms_norm(x, w, 1e-6)
    inv = np.float32(1.0 / np.sqrt(np.sum(x.astype(np.float64) ** 2) / 2560 + np.float64(np.float32(1e-6))))
    assert np.array_equal(out, (x * inv) * w)


def test_argmax_first_max():
    v = np.array([1, 3, 3, -np.inf, np.nan, 2], np.float32)
    assert oracle.argmax(v) == 1
    assert oracle.argmax(np.full(5, -np.inf, np.float32)) == 0
