"""The tensor-core Q8_0 head over the tile layout (q8t.cu) against float64: the re-lay is
byte-exact against a numpy restatement of the tile layout, logits within relL2 1e-5 of
float64 on the dequantized table, and the first-max argmax identical wherever the top-2
margin exceeds 1e-3."""
import numpy as np
import pytest

import oracle
from spk import formats as F

EPS_MARGIN = 1e-3


def tile_layout(q80: bytes, rows: int, cols: int) -> bytes:
    """The tile-block layout restated in numpy (q8t.cu header comment)."""
    blk = np.frombuffer(q80, np.uint8).reshape(rows, cols // 32, 34)
    R, nb = (rows + 15) // 16, cols // 32
    pad = np.zeros((R * 16, nb, 34), np.uint8)
    pad[:rows] = blk
    q = pad[:, :, 2:].reshape(R, 16, nb, 32)     # [R][row][B][col]
    d = pad[:, :, :2].reshape(R, 16, nb, 2)
    out = np.zeros((R, nb, 544), np.uint8)
    for L in range(32):
        g, t = L >> 2, L & 3
        parts = [q[:, g, :, 4 * t:4 * t + 4], q[:, g + 8, :, 4 * t:4 * t + 4],
                 q[:, g, :, 16 + 4 * t:16 + 4 * t + 4], q[:, g + 8, :, 16 + 4 * t:16 + 4 * t + 4]]
        out[:, :, 16 * L:16 * L + 16] = np.concatenate(parts, axis=-1)
    out[:, :, 512:] = d.transpose(0, 2, 1, 3).reshape(R, nb, 32)
    return out.tobytes()


def test_tile_layout_restatement_is_a_permutation():
    rows, cols = 48, 256
    q80 = F.quantize_q8_0(np.random.default_rng(0).standard_normal((rows, cols)).astype(np.float32))
    t = tile_layout(q80, rows, cols)
    assert len(t) == len(q80)
    assert sorted(t) == sorted(q80)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(131072, 2560), (4096, 512), (1040, 1024)])
def test_tiled_head_matches_reference(cuda, rows, cols):
    import torch

    import spk

    L = spk.lib()
    rng = np.random.default_rng(rows + cols)
    q80 = F.synth_q8_0(rows, cols, seed=3) if rows > 8192 else F.quantize_q8_0(
        (0.02 * rng.standard_normal((rows, cols))).astype(np.float32))
    w = spk.dev_bytes(q80, cuda)
    wt = torch.zeros(L.spk_q80_tile_bytes(rows, cols), dtype=torch.uint8, device=cuda)
    spk.check(L.spk_q80_tile(w.data_ptr(), rows, cols, wt.data_ptr(), None))
    torch.cuda.synchronize()
    if rows <= 8192:
        assert wt.cpu().numpy().tobytes() == tile_layout(q80, rows, cols)
    W = oracle.q80_dequant(q80, rows, cols).reshape(rows, cols).astype(np.float64)
    scratch = torch.zeros(L.spk_q80_tile_scratch_bytes(), dtype=torch.uint8, device=cuda)
    nw = (1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    tnw = torch.from_numpy(nw).to(cuda)
    for ntok in (1, 3, 8):
        x = rng.standard_normal((ntok, cols)).astype(np.float32)
        xn = x.astype(np.float64)
        xn = xn / np.sqrt(np.mean(xn * xn, axis=1, keepdims=True) + 1e-6) * nw
        want = xn @ W.T
        tx = torch.from_numpy(x).to(cuda)
        lg = torch.zeros(ntok, rows, device=cuda)
        am = torch.zeros(ntok, dtype=torch.int32, device=cuda)
        for _ in range(2):   # the scratch is left ready
            spk.check(L.spk_q80_tile_head(wt.data_ptr(), rows, cols, ntok, tx.data_ptr(), cols, tnw.data_ptr(), 1e-6,
                                          lg.data_ptr(), rows, am.data_ptr(), scratch.data_ptr(), None))
            torch.cuda.synchronize()
            got = lg.cpu().numpy()
            err = np.linalg.norm(got - want) / np.linalg.norm(want)
            assert err < 1e-5, (ntok, err)
            for n in range(ntok):
                top = np.sort(want[n])[-2:]
                assert int(am[n]) == int(np.argmax(want[n])) or top[1] - top[0] < EPS_MARGIN
    assert scratch.cpu().numpy()[:4].tolist() == [0, 0, 0, 0]   # the ticket is reset


@pytest.mark.gpu
def test_tiled_head_rejects_untiled_geometry(cuda):
    import spk

    L = spk.lib()
    assert L.spk_q80_tile_head(None, 16, 256, 1, None, 256, None, 1e-6, None, 16, None, None, None) == -1
    assert L.spk_q80_tile_bytes(16, 100) == 0
