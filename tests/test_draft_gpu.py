"""The DSpark draft on the GPU against the CPU oracle (oracle/draft.c, the restatement of
tools/dspark/src/draft.rs), and the speculative loop (spec.rs::run) against the same loop
over the oracle target and draft.

* spk_bf16_gemm / spk_bf16_gemm_pair against float64 on the bf16-expanded weights
  (x enters the tensor cores as bf16 hi + lo, ~16 bits: relL2 <= 5e-5 here).
* spk_draft_encode + spk_draft_block on seeded small drafts of the three shapes the
  oracle test covers: biased logits relL2 <= 1e-4, confidence within 1e-4, greedy ids
  identical wherever the oracle's top-2 margin exceeds 1e-3.
* spk.spec.run on a small target + draft against the oracle loop: identical proposals,
  target ids and generated ids, round by round.
"""
import numpy as np
import pytest

import oracle
from spk import formats as F
from spk.draft import DeviceDraft, bf16_to_f32, oracle_weights, small_draft_config, synth_draft, to_bf16
from spk.model import DeviceModel, small_config, synth_weights

pytestmark = pytest.mark.gpu
GEMM_TOL = 5e-5
LOGIT_TOL = 1e-4
EPS_MARGIN = 1e-3

CONFIGS = {
    "released": dict(),
    "variant": dict(gate=False, qk_norm=True, post_norms=True, out_scale=0.5, act="silu", causal=True,
                    sample_from_anchor=False, swa_pattern=[1, 0], rope_full_dims=64),
    "no_markov": dict(rank=0, conf=False),
}


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("rows,cols,ntok,acc", [(6160, 2560, 7, 0), (1000, 512, 3, 1), (2560, 10240, 8, 1),
                                                (16, 12800, 1, 0), (33, 4096, 5, 0)])
def test_bf16_gemm_matches_float64(cuda, rows, cols, ntok, acc):
    import torch

    import spk

    rng = np.random.default_rng(rows + cols + ntok)
    W = to_bf16(0.02 * rng.standard_normal((rows, cols), dtype=np.float32))
    x = rng.standard_normal((ntok, cols)).astype(np.float32)
    y0 = rng.standard_normal((ntok, rows)).astype(np.float32)
    want = (acc * y0.astype(np.float64)) + x.astype(np.float64) @ bf16_to_f32(W).reshape(rows, cols).astype(np.float64).T
    tw = torch.from_numpy(W.view(np.int16)).to(cuda)
    tx, ty = torch.from_numpy(x).to(cuda), torch.from_numpy(y0).to(cuda)
    spk.check(spk.lib().spk_bf16_gemm(tw.data_ptr(), rows, cols, ntok, tx.data_ptr(), cols, ty.data_ptr(), rows, acc,
                                      None))
    torch.cuda.synchronize()
    assert rel(ty.cpu().numpy(), want) < GEMM_TOL


@pytest.mark.parametrize("act", [0, 1])
def test_bf16_gemm_pair_matches_float64(cuda, act):
    import torch

    import spk

    rows, cols, ntok = 1040, 2560, 7
    rng = np.random.default_rng(5 + act)
    G = to_bf16(0.02 * rng.standard_normal((rows, cols), dtype=np.float32))
    U = to_bf16(0.02 * rng.standard_normal((rows, cols), dtype=np.float32))
    x = rng.standard_normal((ntok, cols)).astype(np.float32)
    g = x.astype(np.float64) @ bf16_to_f32(G).reshape(rows, cols).astype(np.float64).T
    u = x.astype(np.float64) @ bf16_to_f32(U).reshape(rows, cols).astype(np.float64).T
    a = g / (1 + np.exp(-g)) if act else 0.5 * g * (1 + np.tanh(0.7978846 * g * (1 + 0.044715 * g * g)))
    want = a * u
    tg, tu = (torch.from_numpy(M.view(np.int16)).to(cuda) for M in (G, U))
    tx, ty = torch.from_numpy(x).to(cuda), torch.zeros(ntok, rows, device=cuda)
    spk.check(spk.lib().spk_bf16_gemm_pair(tg.data_ptr(), tu.data_ptr(), rows, cols, ntok, tx.data_ptr(), cols,
                                           ty.data_ptr(), rows, act, None))
    torch.cuda.synchronize()
    assert rel(ty.cpu().numpy(), want) < GEMM_TOL


def test_bf16_gemm_rejects_bad_arguments(cuda):
    import spk

    L = spk.lib()
    assert L.spk_bf16_gemm(None, 16, 512, 1, None, 512, None, 16, 0, None) == -1
    assert "bad arguments" in spk.last_error()


@pytest.mark.parametrize("name", list(CONFIGS))
def test_draft_block_matches_oracle(cuda, name):
    import torch

    cfg = small_draft_config(**CONFIGS[name])
    W = synth_draft(cfg, seed=7)
    L, G = oracle_weights(cfg, W)
    rng = np.random.default_rng(3)
    ctx, pos0, n_draft, anchor = 64, 41, cfg.draft_max(), 11
    caps = rng.standard_normal((cfg.n_target, ctx, cfg.hidden)).astype(np.float32)
    q80 = F.quantize_q8_0((0.02 * rng.standard_normal((cfg.vocab, cfg.hidden))).astype(np.float32))
    embed = oracle.q80_dequant(q80, cfg.vocab, cfg.hidden).reshape(cfg.vocab, cfg.hidden)

    ref = oracle.Draft(cfg.as_oracle(), L, G, ctx)
    ref.encode(caps, 0, pos0)
    wl, wc, wa = ref.decode_block(embed, anchor, pos0, n_draft)
    ref.close()

    import spk

    d = DeviceDraft(cfg, W, max_ctx=ctx, device=cuda)
    tcaps = torch.from_numpy(caps).to(cuda)
    temb = spk.dev_bytes(q80, cuda)
    d.encode_features(tcaps.data_ptr(), ctx * cfg.hidden, 0, 17)
    d.encode_features(tcaps.data_ptr(), ctx * cfg.hidden, 17, pos0)
    for _ in range(2):   # the Markov tickets and scratch are left ready for the next block
        ids, conf, logits = d.decode_block(temb.data_ptr(), cfg.vocab, anchor, pos0, n_draft, want_logits=True)
        assert logits.shape == wl.shape
        assert rel(logits, wl) < LOGIT_TOL, rel(logits, wl)
        np.testing.assert_allclose(conf, wc, rtol=1e-4, atol=1e-5, equal_nan=True)
        top2 = np.sort(wl, axis=1)[:, -2:]
        for i, (a, b) in enumerate(zip(ids, wa.tolist())):
            assert a == b or top2[i, 1] - top2[i, 0] < EPS_MARGIN, (i, a, b)
    d.close()


def test_draft_block_rejects_what_the_reference_refuses(cuda):
    import spk

    cfg = small_draft_config()
    d = DeviceDraft(cfg, synth_draft(cfg, seed=1), max_ctx=32, device=cuda)
    q80 = F.quantize_q8_0(np.zeros((cfg.vocab, cfg.hidden), np.float32))
    temb = spk.dev_bytes(q80, cuda)
    with pytest.raises(spk.SpkError, match="block_size"):
        d.decode_block(temb.data_ptr(), cfg.vocab, 1, 0, cfg.block_size + 1)
    with pytest.raises(spk.SpkError, match="not encoded"):
        d.decode_block(temb.data_ptr(), cfg.vocab, 1, 20, 3)
    with pytest.raises(spk.SpkError, match="outside"):
        d.decode_block(temb.data_ptr(), cfg.vocab, cfg.vocab, 0, 3)
    d.decode_block(temb.data_ptr(), cfg.vocab, 1, 0, 3)   # pos0 0: no window to encode
    d.close()


def _oracle_spec(tcfg, TW, dcfg, DW, ids, gen, max_ctx):
    layers = [{"in_norm": L["in_norm"], "post_norm": L["post_norm"],
               **{n: oracle.decode(L[n]) for n in ("qkv", "attn_gate", "out", "gate", "up", "down")}}
              for L in TW["layers"]]
    embed = oracle.q80_dequant(TW["embed"], tcfg.vocab, tcfg.hidden).reshape(tcfg.vocab, tcfg.hidden)
    m = oracle.Model(tcfg.as_oracle(), layers, embed, TW["norm"], max_ctx)
    cap = m.enable_capture(dcfg.target_layers)
    L, G = oracle_weights(dcfg, DW)
    d = oracle.Draft(dcfg.as_oracle(), L, G, max_ctx)
    n_draft, i_beg = dcfg.draft_max(), dcfg.i_beg()
    pos0 = len(ids) - 1
    for p, t in enumerate(ids[:pos0]):
        m.forward(t, p)
    d.encode(cap, 0, pos0)
    anchor, gen_ids, rounds = ids[pos0], [], []
    while len(gen_ids) < gen:
        _, _, am = d.decode_block(embed, anchor, pos0, n_draft)
        props = [int(v) for v in am[i_beg:]]
        tgt = [oracle.argmax(m.forward(anchor, pos0))] + [oracle.argmax(m.forward(p, pos0 + 1 + i))
                                                          for i, p in enumerate(props)]
        k = 0
        while k < n_draft and tgt[k] == props[k]:
            k += 1
        gen_ids += props[:k] + [tgt[k]]
        rounds.append((props, tgt))
        d.encode(cap, pos0, pos0 + k + 1)
        pos0 += k + 1
        anchor = tgt[k]
    m.close()
    d.close()
    return gen_ids[:gen], rounds


def test_spec_loop_matches_oracle(cuda):
    from spk import spec

    tcfg = small_config(layers=4, hidden=512, heads=4, kv_heads=1, head_dim=128, inter=1024, vocab=4096, window=16)
    TW = synth_weights(tcfg, seed=21, exact_q80=True)
    dcfg = small_draft_config(target_layers=[0, 1, 3])
    DW = synth_draft(dcfg, seed=22)
    prompt, gen, max_ctx = [5, 17, 301, 42, 4000, 7, 99, 1234, 8, 64], 24, 96
    want, want_rounds = _oracle_spec(tcfg, TW, dcfg, DW, prompt, gen, max_ctx)

    m = DeviceModel(tcfg, TW, max_ctx=max_ctx, device=cuda)
    d = DeviceDraft(dcfg, DW, max_ctx=max_ctx, device=cuda, stream=m.stream)
    spec.prepare(m, d)
    got = spec.run(m, d, prompt, gen)
    for r, ((wp, wt), gp, gt) in enumerate(zip(want_rounds, got.proposals, got.targets)):
        assert gp == wp, f"round {r}: draft proposals differ"
        assert gt == wt, f"round {r}: target ids differ"
    assert got.generated == want
    assert got.rounds == len(want_rounds)
    d.close()
    m.close()
