"""Tensor-parallel host logic on the CPU: the layout, the exact DQV3 re-cuts, the
sharded forward's algebra, and the handle exchange over gloo (world size 2).

The sharded forward is restated in numpy (float64) as libspk's tensor-parallel step
runs it (per rank: its q/KV heads, intermediate rows and vocabulary rows; the two
residual reductions per layer; the argmax over the vocabulary shards) and checked
against the unsharded restatement and against the oracle (model.rs::forward in C).
"""
import math
import os

import numpy as np
import pytest

import oracle
from spk import formats as F
from spk.model import ModelConfig, exchange_handles, mat_shapes, small_config, synth_weights, tp_layout, tp_shard


_erf = np.vectorize(math.erf)


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_layout_covers_every_head_once(world):
    cfg = ModelConfig()
    G = cfg.heads // cfg.kv_heads
    seen_q, seen_i, seen_v = [], [], []
    for r in range(world):
        lay = tp_layout(cfg, r, world)
        seen_q += list(range(lay["h0"], lay["h0"] + lay["hl"]))
        seen_i += list(range(lay["i0"], lay["i0"] + lay["il"]))
        seen_v += list(range(lay["v0"], lay["v0"] + lay["vl"]))
        # every local q head reads a local KV head, in order (GQA group of the kernel)
        for j in range(lay["hl"]):
            kvh = (lay["h0"] + j) // G
            assert lay["k0"] <= kvh < lay["k0"] + lay["kl"]
            assert kvh - lay["k0"] == j // (lay["hl"] // lay["kl"])
    assert seen_q == list(range(cfg.heads))
    assert seen_i == list(range(cfg.inter))
    assert seen_v == list(range(cfg.vocab))


def test_layout_rejects_indivisible():
    with pytest.raises(ValueError):
        tp_layout(ModelConfig(), 0, 3)


def _cfg():
    # kv_heads 2: world 2 splits the KV heads, world 4 replicates them
    return small_config(layers=4, hidden=256, heads=8, kv_heads=2, head_dim=128, inter=512, vocab=1024, window=8)


@pytest.fixture(scope="module")
def model():
    cfg = _cfg()
    return cfg, synth_weights(cfg, seed=11, nc=256, exact_q80=True)


@pytest.mark.parametrize("world", [2, 4])
def test_shards_are_exact_recuts(model, world):
    cfg, W = model
    shapes = mat_shapes(cfg)
    hd = cfg.head_dim
    for r in range(world):
        S = tp_shard(cfg, W, r, world)
        lay = tp_layout(cfg, r, world)
        for li in (0, cfg.layers - 1):
            full = {n: oracle.decode(W["layers"][li][n]).reshape(shapes[n]) for n in shapes}
            sh = {n: oracle.decode(S["layers"][li][n]) for n in shapes}
            q = np.arange(lay["h0"] * hd, (lay["h0"] + lay["hl"]) * hd)
            kv = np.arange(lay["k0"] * hd, (lay["k0"] + lay["kl"]) * hd)
            rows = np.concatenate([q, cfg.q_dim + kv, cfg.q_dim + cfg.kv_dim + kv])
            i0, i1 = lay["i0"], lay["i0"] + lay["il"]
            want = {"qkv": full["qkv"][rows], "attn_gate": full["attn_gate"][lay["h0"]:lay["h0"] + lay["hl"]],
                    "out": full["out"][:, q], "gate": full["gate"][i0:i1], "up": full["up"][i0:i1],
                    "down": full["down"][:, i0:i1]}
            for n in shapes:
                assert np.array_equal(sh[n].reshape(-1).view(np.uint32), want[n].reshape(-1).view(np.uint32)), (r, li, n)


# --------------------------------------------- the sharded forward, numpy ---
class NpTP:
    """model.rs:442-591 over `world` simulated ranks holding tp_shard's shards."""

    def __init__(self, cfg, W, world, max_ctx):
        self.cfg, self.world = cfg, world
        shapes = mat_shapes(cfg)
        self.ranks = []
        for r in range(world):
            S = tp_shard(cfg, W, r, world)
            lay = tp_layout(cfg, r, world)
            mats = []
            for L in S["layers"]:
                d = {}
                for n in shapes:
                    c = F.parse_container(L[n])
                    d[n] = oracle.decode(L[n]).reshape(c.rows, c.cols).astype(np.float64)
                d["in_norm"], d["post_norm"] = L["in_norm"].astype(np.float64), L["post_norm"].astype(np.float64)
                mats.append(d)
            kc = [np.zeros((max_ctx, lay["kl"], cfg.head_dim)) for _ in range(cfg.layers)]
            vc = [np.zeros((max_ctx, lay["kl"], cfg.head_dim)) for _ in range(cfg.layers)]
            self.ranks.append({"lay": lay, "mats": mats, "kc": kc, "vc": vc})
        self.embed = oracle.q80_dequant(W["embed"], cfg.vocab, cfg.hidden).reshape(cfg.vocab, cfg.hidden).astype(np.float64)
        self.norm = W["norm"].astype(np.float64)

    def _rms(self, x, w):
        return x / np.sqrt(np.mean(x * x) + self.cfg.eps) * w

    def _rope(self, x, pos, full):
        cfg = self.cfg
        part, theta = (cfg.rope_partial_full, cfg.rope_theta_full) if full else (cfg.rope_partial_slide, cfg.rope_theta_slide)
        pd = min(int(cfg.head_dim * part), cfg.head_dim)
        half = pd // 2
        f = 1.0 / np.power(theta, np.arange(half) * 2.0 / pd)
        c, s = np.cos(pos * f), np.sin(pos * f)
        a, b = x[..., :half].copy(), x[..., half:pd].copy()
        x[..., :half], x[..., half:pd] = a * c - b * s, b * c + a * s
        return x

    def forward(self, tok, pos):
        cfg, hd = self.cfg, self.cfg.head_dim
        G = cfg.heads // cfg.kv_heads
        h = self.embed[tok].copy()
        for li in range(cfg.layers):
            full = bool(cfg.full[li])
            start = 0 if full else max(0, pos + 1 - cfg.window)
            parts = []
            for R in self.ranks:
                lay, M = R["lay"], R["mats"][li]
                xn = self._rms(h, M["in_norm"])
                qkv, g = M["qkv"] @ xn, M["attn_gate"] @ xn
                q = self._rope(qkv[:lay["hl"] * hd].reshape(lay["hl"], hd), pos, full)
                k = self._rope(qkv[lay["hl"] * hd:(lay["hl"] + lay["kl"]) * hd].reshape(lay["kl"], hd), pos, full)
                v = qkv[(lay["hl"] + lay["kl"]) * hd:].reshape(lay["kl"], hd)
                R["kc"][li][pos], R["vc"][li][pos] = k, v
                att = np.empty((lay["hl"], hd))
                for j in range(lay["hl"]):
                    kv = (lay["h0"] + j) // G - lay["k0"]
                    K, V = R["kc"][li][start:pos + 1, kv], R["vc"][li][start:pos + 1, kv]
                    sc = K @ q[j] / np.sqrt(hd)
                    p = np.exp(sc - sc.max())
                    att[j] = (p / p.sum()) @ V / (1.0 + np.exp(-g[j]))
                parts.append(M["out"] @ att.reshape(-1))
            h = h + sum(parts)   # tp_sum: rank order
            parts = []
            for R in self.ranks:
                M = R["mats"][li]
                xn = self._rms(h, M["post_norm"])
                gt, up = M["gate"] @ xn, M["up"] @ xn
                gelu = 0.5 * gt * (1.0 + _erf(gt / np.sqrt(2.0)))
                parts.append(M["down"] @ (gelu * up))
            h = h + sum(parts)
        xn = self._rms(h, self.norm)
        logits = np.concatenate([self.embed[R["lay"]["v0"]:R["lay"]["v0"] + R["lay"]["vl"]] @ xn for R in self.ranks])
        return logits


def test_sharded_forward_matches_unsharded_and_oracle(model):
    cfg, W = model
    steps = 12
    one, two, four = NpTP(cfg, W, 1, steps), NpTP(cfg, W, 2, steps), NpTP(cfg, W, 4, steps)
    layers = [{"in_norm": L["in_norm"], "post_norm": L["post_norm"],
               **{n: oracle.decode(L[n]) for n in ("qkv", "attn_gate", "out", "gate", "up", "down")}}
              for L in W["layers"]]
    ref = oracle.Model(cfg.as_oracle(), layers, oracle.q80_dequant(W["embed"], cfg.vocab, cfg.hidden), W["norm"], steps)
    tok = 3
    for pos in range(steps):
        a, b, c = one.forward(tok, pos), two.forward(tok, pos), four.forward(tok, pos)
        o = ref.forward(tok, pos)
        assert rel(b, a) < 1e-12 and rel(c, a) < 1e-12, pos
        assert rel(a, o) < 1e-4, pos
        tok = int(np.argmax(a))
    ref.close()


# ------------------------------------------------ handle exchange, gloo x2 ---
def _exchange_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        got = exchange_handles(bytes([rank + 1]) * 64)
        q.put((rank, [g[:1] for g in got], [len(g) for g in got]))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_gloo_world2():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, firsts, lens in res:
        assert firsts == [b"\x01", b"\x02"] and lens == [64, 64], rank
