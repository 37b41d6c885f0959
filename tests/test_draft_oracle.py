"""The C restatement of the DSpark draft executor (oracle/draft.c) against an independent
float64 numpy restatement of tools/dspark/src/draft.rs (encode_features 567-628,
decode_block 641-901), on seeded small drafts in three shapes: the released checkpoint's
structure (attn_gate, tanh-GELU, non-causal block sampled from the anchor, Markov and
confidence heads), a variant with every optional tensor the reference reads (q/k norms,
post norms, layer_out_scale, SiLU, causal, bonus anchor row), and a draft without a Markov
head. No reference output exists for synthetic drafts (the Rust executor cannot be built
here), so this pins the C code against a second, independent transcription."""
import math

import numpy as np
import pytest

import oracle
from spk.draft import oracle_weights, small_draft_config, synth_draft

_tanh = np.tanh


def rms(x, w, eps):
    y = x / math.sqrt(float(np.mean(x * x)) + eps)
    return y * w if w is not None else y


def rope(v, heads, hd, pos, nrot, theta):
    dim = min(nrot, hd)
    half = dim // 2
    f = 1.0 / np.power(float(theta), np.arange(half) * 2.0 / dim)
    c, s = np.cos(pos * f), np.sin(pos * f)
    v = v.reshape(heads, hd).copy()
    lo, hi = v[:, :half].copy(), v[:, half:dim].copy()
    v[:, :half], v[:, half:dim] = lo * c - hi * s, hi * c + lo * s
    return v.reshape(-1)


def rope_for(cfg, li):
    return (cfg.rope_swa_dims, cfg.rope_swa_theta) if cfg.swa_pattern[li] else (cfg.rope_full_dims, cfg.rope_full_theta)


def np_encode(cfg, L, G, caps, positions):
    H, hd = cfg.hidden, cfg.head_dim
    inj = {}
    for p in positions:
        cat = np.concatenate([rms(caps[k, p].astype(np.float64), G["fc_norm"][k], cfg.eps) for k in range(cfg.n_target)])
        g = rms(G["fc"].astype(np.float64) @ cat, G["enc_norm"], cfg.eps)
        for li, Ld in enumerate(L):
            nrot, theta = rope_for(cfg, li)
            k = Ld["k"].astype(np.float64) @ g
            v = Ld["v"].astype(np.float64) @ g
            if Ld.get("k_norm") is not None:
                k = np.concatenate([rms(k[c * hd:(c + 1) * hd], Ld["k_norm"], cfg.eps) for c in range(cfg.kv_heads)])
            inj[(li, p)] = (rope(k, cfg.kv_heads, hd, p, nrot, theta), v)
    return inj


def np_decode(cfg, L, G, inj, embed, anchor, pos0, n_draft):
    hd, heads, kvh, H = cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.hidden
    markov = G.get("markov_w1") is not None
    nb = cfg.block_rows(n_draft)
    nswa = cfg.swa_window + 1 if markov else cfg.swa_window
    x = [embed[anchor if i == 0 else cfg.mask_token].astype(np.float64) for i in range(nb)]
    for li, Ld in enumerate(L):
        nrot, theta = rope_for(cfg, li)
        qs, ks, vs = [], [], []
        for i in range(nb):
            xn = rms(x[i], Ld["norm"], cfg.eps)
            q, k, v = (Ld[n].astype(np.float64) @ xn for n in ("q", "k", "v"))
            if Ld.get("q_norm") is not None and Ld.get("k_norm") is not None:
                q = np.concatenate([rms(q[c * hd:(c + 1) * hd], Ld["q_norm"], cfg.eps) for c in range(heads)])
                k = np.concatenate([rms(k[c * hd:(c + 1) * hd], Ld["k_norm"], cfg.eps) for c in range(kvh)])
            qs.append(rope(q, heads, hd, pos0 + i, nrot, theta))
            ks.append(rope(k, kvh, hd, pos0 + i, nrot, theta))
            vs.append(v)
        keys = [inj[(li, p)] for p in range(max(0, pos0 - nswa + 1), pos0)]
        keys += [(ks[i], vs[i]) for i in range(nb) if (not cfg.causal or i == 0)]
        K = np.stack([k for k, _ in keys])
        V = np.stack([v for _, v in keys])
        nx = []
        for i in range(nb):
            xn = rms(x[i], Ld["norm"], cfg.eps)
            g = Ld["gate"].astype(np.float64) @ xn if Ld.get("gate") is not None else None
            att = np.zeros(heads * hd)
            for h in range(heads):
                grp = h * kvh // heads
                sc = K[:, grp * hd:(grp + 1) * hd] @ qs[i][h * hd:(h + 1) * hd] / math.sqrt(hd)
                p = np.exp(sc - sc.max())
                o = (p / p.sum()) @ V[:, grp * hd:(grp + 1) * hd]
                if g is not None:
                    o = o / (1.0 + math.exp(-g[h]))
                att[h * hd:(h + 1) * hd] = o
            out = Ld["out"].astype(np.float64) @ att
            if Ld.get("attn_post") is not None:
                out = rms(out, Ld["attn_post"], cfg.eps)
            res = x[i] + out
            xn2 = rms(res, Ld["ffn_norm"], cfg.eps)
            up = Ld["ffn_up"].astype(np.float64) @ xn2
            gt = Ld["ffn_gate"].astype(np.float64) @ xn2
            if cfg.act == "silu":
                act = gt / (1.0 + np.exp(-gt)) * up
            else:
                act = 0.5 * gt * (1.0 + _tanh(0.7978846 * gt * (1.0 + 0.044715 * gt * gt))) * up
            res = res + Ld["ffn_down"].astype(np.float64) @ act
            if Ld.get("ffn_post") is not None:
                res = rms(res, Ld["ffn_post"], cfg.eps)
            if Ld.get("out_scale", 0.0) != 0.0:
                res = res * Ld["out_scale"]
            nx.append(res)
        x = nx
    hid = [rms(x[i], G["out_norm"], cfg.eps) for i in range(nb)]
    logits = np.stack([embed.astype(np.float64) @ hid[i] for i in range(nb)])
    conf = np.full(nb, np.nan)
    if markov:
        w1, w2 = G["markov_w1"].astype(np.float64), G["markov_w2"].astype(np.float64)
        prev = anchor
        if not cfg.sample_from_anchor and G.get("conf_proj") is not None:
            conf[0] = 1.0 / (1.0 + math.exp(-logits[0][0]))
        for i in range(cfg.i_beg(), nb):
            logits[i, :cfg.vocab] += w2 @ w1[prev]
            if G.get("conf_proj") is not None:
                c = float(G["conf_proj"] @ np.concatenate([hid[i], w1[prev]])) + G["conf_bias"]
                conf[i] = 1.0 / (1.0 + math.exp(-c))
            if i + 1 < nb:
                prev = int(np.argmax(logits[i]))
    return logits, conf, np.argmax(logits, axis=1)


CONFIGS = {
    "released": dict(),
    "variant": dict(gate=False, qk_norm=True, post_norms=True, out_scale=0.5, act="silu", causal=True,
                    sample_from_anchor=False, swa_pattern=[1, 0], rope_full_dims=64),
    "no_markov": dict(rank=0, conf=False),
}


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("name", list(CONFIGS))
def test_draft_oracle_matches_float64_restatement(name):
    cfg = small_draft_config(**CONFIGS[name])
    W = synth_draft(cfg, seed=7)
    L, G = oracle_weights(cfg, W)
    rng = np.random.default_rng(3)
    ctx, pos0, n_draft = 40, 29, cfg.draft_max()
    caps = rng.standard_normal((cfg.n_target, ctx, cfg.hidden)).astype(np.float32)
    embed = (0.02 * rng.standard_normal((cfg.vocab, cfg.hidden))).astype(np.float32)
    d = oracle.Draft(cfg.as_oracle(), L, G, ctx)
    d.encode(caps, 0, 20)
    d.encode(caps, 20, pos0)   # incremental encodes join
    lg, cf, am = d.decode_block(embed, 11, pos0, n_draft)
    inj = np_encode(cfg, L, G, caps, range(max(0, pos0 - cfg.swa_window - 1), pos0))
    wl, wc, wa = np_decode(cfg, L, G, inj, embed, 11, pos0, n_draft)
    assert lg.shape == wl.shape == (cfg.block_rows(n_draft), cfg.vocab)
    assert rel(lg, wl) < 1e-5, rel(lg, wl)
    np.testing.assert_allclose(cf, wc, rtol=1e-5, atol=1e-6, equal_nan=True)
    top2 = np.sort(wl, axis=1)[:, -2:]
    assert (top2[:, 1] - top2[:, 0] > 1e-3).all(), "near-tie in the float64 logits: pick another seed"
    assert am.tolist() == wa.tolist()
    d.close()


def test_draft_oracle_refuses_what_the_reference_refuses():
    cfg = small_draft_config()
    L, G = oracle_weights(cfg, synth_draft(cfg, seed=1))
    ctx = 32
    caps = np.zeros((cfg.n_target, ctx, cfg.hidden), np.float32)
    embed = np.zeros((cfg.vocab, cfg.hidden), np.float32)
    d = oracle.Draft(cfg.as_oracle(), L, G, ctx)
    d.encode(caps, 0, 10)
    with pytest.raises(ValueError):   # n_draft outside the trained block_size
        d.decode_block(embed, 1, 10, cfg.block_size + 1)
    with pytest.raises(ValueError):
        d.decode_block(embed, 1, 10, 0)
    with pytest.raises(ValueError):   # the window before pos0 is not encoded
        d.decode_block(embed, 1, 20, 3)
    with pytest.raises(ValueError):   # anchor outside the embedding
        d.decode_block(embed, cfg.vocab, 10, 3)
    d.decode_block(embed, 1, 10, 3)
    d.close()
