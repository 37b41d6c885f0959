"""Generate the golden fixtures under tests/golden/ (run here, where the reference exists).

Every fixture pins the CPU oracle (oracle/) to an implementation it did not write:

* ``vq_*.npz`` — seeded RQVQ containers in every payload geometry the reference
  decodes (DQV3 12-bit, 13-bit plane, 10-bit, 8-bit dim 8; DQVQ v2 12-, 9- and
  8-bit), each with the decoded f32 matrix that the reference's own
  ``tools/vq/decode.c`` ``dump`` writes (oracle/_ref/decode, compiled from the
  reference sources) and the ``matvec`` checksum line it prints for x.
* ``q6k.npz`` / ``q80.npz`` — Q6_K and Q8_0 blocks with gguf-py's numpy block
  decoders' output (``gguf.quants.dequantize``; gguf-py 0.19.0 restates
  ggml's dequantize_row_q6_K / dequantize_row_q8_0), and for Q8_0 gguf-py's
  quantizer output for the same weights.

Usage: python tests/golden/make_golden.py   (needs oracle/_ref/decode: make -C oracle ref)
"""
from __future__ import annotations

import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "spark-x2.6-4b-q6k_b200"))

import oracle  # noqa: E402
from spk import formats as F  # noqa: E402

VQ_CASES = [
    # name, rows, cols, dim, nc, stages, v3
    ("v3_12bit", 24, 256, 4, 4096, 2, True),
    ("v3_13bit", 16, 128, 4, 8192, 2, True),
    ("v3_10bit", 12, 160, 4, 1024, 1, True),
    ("v3_8bit_dim8", 8, 128, 8, 256, 2, True),
    ("v2_12bit", 12, 128, 4, 4096, 2, False),
    ("v2_9bit", 10, 96, 4, 512, 2, False),
    ("v2_8bit", 8, 64, 4, 256, 1, False),
]


def make_vq():
    for i, (name, rows, cols, dim, nc, st, v3) in enumerate(VQ_CASES):
        buf = F.random_rvq(rows, cols, dim, nc, st, seed=100 + i, unit_gains=False, v3=v3)
        x = np.sin(0.001 * np.arange(cols, dtype=np.float64)).astype(np.float32) + \
            np.random.default_rng(7 + i).normal(0, 1, cols).astype(np.float32)
        with tempfile.TemporaryDirectory() as d:
            cp, vp = os.path.join(d, "c.bin"), os.path.join(d, "x.f32")
            with open(cp, "wb") as f:
                f.write(buf)
            x.tofile(vp)
            W = oracle.ref_decode_dump(cp, os.path.join(d, "w.f32")).reshape(rows, cols)
            csum, cnorm = oracle.ref_decode_matvec(cp, vp)
        np.savez_compressed(os.path.join(HERE, f"vq_{name}.npz"), container=np.frombuffer(buf, np.uint8),
                            x=x, ref_decoded=W, ref_matvec_sum=csum, ref_matvec_norm=cnorm)
        print("wrote", name, W.shape)


def make_ggml():
    import gguf.quants as GQ
    from gguf import GGMLQuantizationType as T

    rng = np.random.default_rng(11)
    rows, cols = 16, 512
    W = rng.normal(0, 0.02, size=(rows, cols)).astype(np.float32)
    W[2, :256] = 0.0                        # an all-zero super-block
    W[5, 256:] = rng.normal(0, 3.0, 256)    # a wide-range block
    W[7, :32] = 1e-6                        # tiny values (f16 scale near subnormal)
    x = rng.normal(0, 1, cols).astype(np.float32)
    b6 = F.quantize_q6_k(W)
    g6 = GQ.dequantize(np.frombuffer(b6, np.uint8).reshape(rows, -1), T.Q6_K).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "q6k.npz"), blocks=np.frombuffer(b6, np.uint8), rows=rows,
                        cols=cols, x=x, gguf_dequant=g6)
    b8 = F.quantize_q8_0(W)
    g8 = GQ.dequantize(np.frombuffer(b8, np.uint8).reshape(rows, -1), T.Q8_0).astype(np.float32)
    q8g = GQ.quantize(W, T.Q8_0).reshape(-1)
    np.savez_compressed(os.path.join(HERE, "q80.npz"), blocks=np.frombuffer(b8, np.uint8), rows=rows,
                        cols=cols, x=x, weights=W, gguf_dequant=g8, gguf_quant=q8g)
    print("wrote q6k, q80")


if __name__ == "__main__":
    make_vq()
    make_ggml()
