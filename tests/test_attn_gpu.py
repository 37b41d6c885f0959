"""spk_attn_decode / spk_attn_store (GQA decode attention, model.rs:508-557) against a
float64 numpy restatement: one token with the in-kernel K/V store, and verify batches."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 2e-5


class AttnArgs(C.Structure):
    _fields_ = [("qkv", C.c_void_p), ("ldqkv", C.c_int), ("k_cache", C.c_void_p), ("v_cache", C.c_void_p),
                ("kv_type", C.c_int), ("slots", C.c_int), ("full", C.c_int), ("window", C.c_int),
                ("freq", C.c_void_p), ("pdim", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("pos_dev", C.c_void_p), ("ntok", C.c_int), ("store", C.c_int),
                ("nsplit", C.c_int), ("gate", C.c_void_p), ("ldgate", C.c_int), ("out", C.c_void_p),
                ("ldout", C.c_int), ("workspace", C.c_void_p)]


def rope(x, pos, freq, pdim):
    half = pdim // 2
    ang = np.float32(pos) * freq[:half].astype(np.float32)
    c, s = np.cos(ang.astype(np.float64)), np.sin(ang.astype(np.float64))
    a, b = x[..., :half].copy(), x[..., half:pdim].copy()
    x[..., :half], x[..., half:pdim] = a * c - b * s, b * c + a * s
    return x


def q8_rows(x):
    """ggml's q8_0 rule per 32 values in f32 arithmetic (d = max|x|/127, q = roundf(x * (1/d))),
    in the cache's planar row layout [hd int8][hd/32 f16 d]; returns (bytes rows, dequantized)."""
    x = np.asarray(x, np.float32)
    hd = x.shape[-1]
    blk = x.reshape(*x.shape[:-1], hd // 32, 32)
    d = (np.abs(blk).max(axis=-1) / np.float32(127)).astype(np.float32)
    idv = np.where(d != 0, np.float32(1) / np.where(d != 0, d, 1), 0).astype(np.float32)
    v = blk * idv[..., None]
    q = (np.sign(v) * np.floor(np.abs(v) + np.float32(0.5))).astype(np.int8)
    d16 = d.astype(np.float16)
    rows = np.concatenate([q.reshape(*x.shape[:-1], hd).view(np.uint8), d16.view(np.uint8).reshape(*x.shape[:-1], -1)],
                          axis=-1)
    deq = (q.astype(np.float64) * d16.astype(np.float64)[..., None]).reshape(x.shape)
    return rows, deq


def to_cache(x, kv_type):
    """Cache rows of type 0 f32 / 1 f16 / 2 q8_0 and their values as the kernel reads them."""
    if kv_type == 2:
        return q8_rows(x)
    dt = np.float16 if kv_type == 1 else np.float32
    c = np.asarray(x, np.float32).astype(dt)
    return c, c.astype(np.float64)


def reference(qkv, K, V, own, pos0, ntok, heads, kvh, hd, full, window, freq, pdim, gate):
    """K/V [kvh][slots][hd] holding the batch rows as the cache stores them (roped K);
    own[t] = token t's unrounded (k, v), which the kernel uses for its own position."""
    G = heads // kvh
    out = np.zeros((ntok, heads * hd))
    for t in range(ntok):
        pos = pos0 + t
        start = 0 if full else max(0, pos + 1 - window)
        q = rope(qkv[t, :heads * hd].reshape(heads, hd).astype(np.float64), pos, freq, pdim)
        Kt, Vt = K.copy(), V.copy()
        Kt[:, pos], Vt[:, pos] = own[t]
        for h in range(heads):
            k = Kt[h // G, start:pos + 1]
            v = Vt[h // G, start:pos + 1]
            sc = k @ q[h] / np.sqrt(hd)
            p = np.exp(sc - sc.max())
            out[t, h * hd:(h + 1) * hd] = (p / p.sum()) @ v / (1 + np.exp(-gate[t, h]))
    return out


@pytest.mark.parametrize("hd,heads,kvh", [(256, 16, 4), (128, 4, 1)])
@pytest.mark.parametrize("full", [1, 0])
@pytest.mark.parametrize("ntok,f16", [(1, 0), (1, 1), (8, 0), (5, 1), (1, 2), (8, 2)])
def test_attention_matches_reference(cuda, hd, heads, kvh, full, ntok, f16):
    """f16 is the cache type: 0 f32, 1 f16, 2 q8_0."""
    import torch

    import spk

    L = spk.lib()
    rng = np.random.default_rng(hd + 7 * ntok + full)
    slots, window, pos0, nsplit = 640, 64, 300, 37
    pdim = hd // 4 if full else hd
    freq = np.zeros(hd, np.float32)
    theta = 5e6 if full else 1e4
    freq[:pdim // 2] = (1.0 / np.power(np.float32(theta), np.arange(pdim // 2, dtype=np.float32) * 2 / pdim)).astype(np.float32)
    ld = (heads + 2 * kvh) * hd
    qkv = rng.normal(0, 1, (ntok, ld)).astype(np.float32)
    gate = rng.normal(0, 1, (ntok, heads)).astype(np.float32)
    K, Kref = to_cache(rng.normal(0, 1, (kvh, slots, hd)), f16)
    V, Vref = to_cache(rng.normal(0, 1, (kvh, slots, hd)), f16)
    own = []
    for t in range(ntok):   # the rows the kernel writes: roped k, v (rounded to the cache type)
        k = rope(qkv[t, heads * hd:(heads + kvh) * hd].reshape(kvh, hd).astype(np.float64), pos0 + t, freq, pdim)
        v = qkv[t, (heads + kvh) * hd:].reshape(kvh, hd).astype(np.float64)
        own.append((k, v))
        Kref[:, pos0 + t] = to_cache(k.astype(np.float32), f16)[1]
        Vref[:, pos0 + t] = to_cache(v.astype(np.float32), f16)[1]
    want = reference(qkv, Kref, Vref, own, pos0, ntok, heads, kvh, hd, full, window, freq, pdim, gate)

    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    t_qkv, t_gate, t_freq = dev(qkv), dev(gate), dev(freq)
    t_k, t_v = dev(K), dev(V)
    t_pos = torch.tensor([pos0], dtype=torch.int32, device=cuda)
    t_out = torch.zeros(ntok, heads * hd, device=cuda)
    ws = torch.zeros(L.spk_attn_workspace_bytes(ntok, heads, kvh, hd, nsplit), dtype=torch.uint8, device=cuda)
    a = AttnArgs(t_qkv.data_ptr(), ld, t_k.data_ptr(), t_v.data_ptr(), f16, slots, full, window, t_freq.data_ptr(),
                 pdim, heads, kvh, hd, t_pos.data_ptr(), ntok, 1 if ntok == 1 else 0, nsplit, t_gate.data_ptr(),
                 heads, t_out.data_ptr(), heads * hd, ws.data_ptr())
    torch.cuda.synchronize()
    if ntok > 1:
        spk.check(L.spk_attn_store(C.byref(a), None))
    for _ in range(2):   # the workspace is left ready for the next call
        spk.check(L.spk_attn_decode(C.byref(a), None))
        torch.cuda.synchronize()
        got = t_out.cpu().numpy()
        err = np.linalg.norm(got - want) / np.linalg.norm(want)
        # q8_0 batch rows: the reference ropes in f64, so a quant can land one step apart
        assert err < (1e-4 if f16 == 2 else TOL), err
    # the stored rows (in-kernel for one token, the batch store otherwise) are the cache type's
    # rounding of the roped k and of v: bit-exact for q8_0 (same f32 rule), close for f16/f32
    for t in range(ntok):
        kw = to_cache(own[t][0].astype(np.float32), f16)[0]
        kc = t_k.cpu().numpy()[:, pos0 + t]
        if f16 == 2:
            assert (np.abs(kc.view(np.int8)[:, :hd].astype(int) - kw.view(np.int8)[:, :hd].astype(int)) <= 1).all()
            assert np.array_equal(kc[:, hd:], kw[:, hd:]) or np.allclose(
                kc[:, hd:].copy().view(np.float16), kw[:, hd:].copy().view(np.float16), rtol=1e-3)
        else:
            assert np.allclose(kc.astype(np.float64), kw.astype(np.float64), rtol=1e-3, atol=1e-3)
    assert ws.cpu().numpy()[:1024].max() == 0   # tickets reset


@pytest.mark.parametrize("ntok,kv_type", [(1, 1), (8, 1), (1, 0), (3, 2)])
@pytest.mark.parametrize("nsplit", [1, 2, 3, 4, 8, 37])
def test_attention_long_splits(cuda, ntok, kv_type, nsplit):
    """Splits of 16-600 positions (several 64-position stages of the tensor-core kernel,
    a partial last stage, the own row inside a stage) at head_dim 256, full attention.
    1, 2, 4 and 8 splits merge inside one thread-block cluster; 3 and 37 through the
    workspace and the last split's ticket."""
    import torch

    import spk

    L = spk.lib()
    hd, heads, kvh = 256, 16, 4
    rng = np.random.default_rng(31 + ntok + 7 * kv_type + nsplit)
    slots, pos0, pdim = 640, 601 - ntok, hd // 4
    freq = np.zeros(hd, np.float32)
    freq[:pdim // 2] = (1.0 / np.power(np.float32(5e6), np.arange(pdim // 2, dtype=np.float32) * 2 / pdim)).astype(np.float32)
    ld = (heads + 2 * kvh) * hd
    qkv = rng.normal(0, 1, (ntok, ld)).astype(np.float32)
    gate = rng.normal(0, 1, (ntok, heads)).astype(np.float32)
    K, Kref = to_cache(rng.normal(0, 1, (kvh, slots, hd)), kv_type)
    V, Vref = to_cache(rng.normal(0, 1, (kvh, slots, hd)), kv_type)
    own = []
    for t in range(ntok):
        k = rope(qkv[t, heads * hd:(heads + kvh) * hd].reshape(kvh, hd).astype(np.float64), pos0 + t, freq, pdim)
        v = qkv[t, (heads + kvh) * hd:].reshape(kvh, hd).astype(np.float64)
        own.append((k, v))
        Kref[:, pos0 + t] = to_cache(k.astype(np.float32), kv_type)[1]
        Vref[:, pos0 + t] = to_cache(v.astype(np.float32), kv_type)[1]
    want = reference(qkv, Kref, Vref, own, pos0, ntok, heads, kvh, hd, 1, 64, freq, pdim, gate)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    t_qkv, t_gate, t_freq, t_k, t_v = dev(qkv), dev(gate), dev(freq), dev(K), dev(V)
    t_pos = torch.tensor([pos0], dtype=torch.int32, device=cuda)
    t_out = torch.zeros(ntok, heads * hd, device=cuda)
    ws = torch.zeros(L.spk_attn_workspace_bytes(ntok, heads, kvh, hd, nsplit), dtype=torch.uint8, device=cuda)
    a = AttnArgs(t_qkv.data_ptr(), ld, t_k.data_ptr(), t_v.data_ptr(), kv_type, slots, 1, 64, t_freq.data_ptr(),
                 pdim, heads, kvh, hd, t_pos.data_ptr(), ntok, 1 if ntok == 1 else 0, nsplit, t_gate.data_ptr(),
                 heads, t_out.data_ptr(), heads * hd, ws.data_ptr())
    torch.cuda.synchronize()
    if ntok > 1:
        spk.check(L.spk_attn_store(C.byref(a), None))
    for _ in range(2):
        spk.check(L.spk_attn_decode(C.byref(a), None))
        torch.cuda.synchronize()
        got = t_out.cpu().numpy()
        err = np.linalg.norm(got - want) / np.linalg.norm(want)
        assert err < (1e-4 if kv_type == 2 else TOL), err


def test_attention_rejects_bad_args(cuda):
    import spk

    L = spk.lib()
    a = AttnArgs()
    assert L.spk_attn_decode(C.byref(a), None) == -1
    assert L.spk_attn_workspace_bytes(0, 16, 4, 256, 37) == 0
