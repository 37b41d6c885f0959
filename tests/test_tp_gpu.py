"""Tensor-parallel decode on the GPU.

* 2, 4 and 8 ranks (one process per GPU, as many GPUs as ranks): the sharded small
  model's greedy tokens and gathered logits against the CPU oracle (model.rs::forward
  in C) and against each other; the device-resident loop against the host loop. At 4
  and 8 ranks the model's 2 KV heads are replicated over the ranks of each head.
* One GPU: a rank whose peer never arrives. Its exchange waits give up after the
  wait limit, the forward reports the peer timeout, and the context stays usable.
"""
import os
import socket

import numpy as np
import pytest

import oracle
from spk.model import DeviceModel, small_config, synth_weights, tp_shard

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-4
EPS_MARGIN = 1e-3
PROMPT = [5, 17, 301, 42, 4000, 7]
STEPS = 48


def _cfg():
    return small_config(layers=4, hidden=512, heads=8, kv_heads=2, head_dim=128, inter=1024, vocab=4096, window=16)


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _cfg()
        W = tp_shard(cfg, synth_weights(cfg, seed=3, exact_q80=True), rank, world)
        n = len(PROMPT) + STEPS
        m = DeviceModel(cfg, W, max_ctx=2 * n + 2, kv_f16=False, device=f"cuda:{rank}")
        m.tp_connect(wait_ms=10000)
        toks, logits = [], []
        tok = PROMPT[0]
        for pos in range(n):
            nxt, lg = m.forward(tok, pos)
            toks.append(nxt)
            logits.append(lg)
            tok = PROMPT[pos + 1] if pos + 1 < len(PROMPT) else nxt
        # the device loop from the same state, replayed from the prompt end
        m.rollback(len(PROMPT) - 1)
        ids = torch.zeros(STEPS, dtype=torch.int32, device=f"cuda:{rank}")
        m.begin(PROMPT[-1], len(PROMPT) - 1, ids, STEPS)
        m.run(STEPS)
        m.stream.synchronize()
        dev_ids = ids.cpu().numpy().tolist()
        # a verify batch (anchor + 7 proposals = the host loop's own ids): 8-row exchanges
        p0 = len(PROMPT) - 1
        m.rollback(p0)
        tgt, _ = m.verify([PROMPT[-1]] + toks[p0:p0 + 7], p0)
        m.close()
        q.put((rank, toks, np.stack(logits) if rank == 0 else None, (dev_ids, tgt), None))
    except Exception as e:   # report, do not hang the parent
        q.put((rank, None, None, None, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_matches_oracle(cuda, world):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        r = q.get(timeout=600)
        res[r[0]] = r
    for p in ps:
        p.join(timeout=120)
    for r in range(world):
        assert res[r][4] is None, res[r][4]
    toks0, logits, (dev0, tgt0) = res[0][1], res[0][2], res[0][3]
    for r in range(1, world):
        assert toks0 == res[r][1], f"rank {r} disagrees on the greedy ids"
        assert (dev0, tgt0) == res[r][3]
    p0 = len(PROMPT) - 1
    assert tgt0 == toks0[p0:p0 + 8], "the verify batch disagrees with the sequential steps"

    cfg = _cfg()
    W = synth_weights(cfg, seed=3, exact_q80=True)
    layers = [{"in_norm": L["in_norm"], "post_norm": L["post_norm"],
               **{n: oracle.decode(L[n]) for n in ("qkv", "attn_gate", "out", "gate", "up", "down")}}
              for L in W["layers"]]
    n = len(PROMPT) + STEPS
    ref = oracle.Model(cfg.as_oracle(), layers, oracle.q80_dequant(W["embed"], cfg.vocab, cfg.hidden), W["norm"], n + 1)
    tok, worst, mism = PROMPT[0], 0.0, 0
    for pos in range(n):
        want = ref.forward(tok, pos)
        worst = max(worst, rel(logits[pos], want))
        o_id = oracle.argmax(want)
        if toks0[pos] != o_id:
            t = np.sort(want)[-2:]
            assert t[1] - t[0] < EPS_MARGIN, f"pos {pos}: {toks0[pos]} vs oracle {o_id}"
            mism += 1
        tok = PROMPT[pos + 1] if pos + 1 < len(PROMPT) else toks0[pos]
    ref.close()
    assert worst < LOGIT_TOL, worst
    assert mism == 0
    # device loop: the id after position p is the host loop's id at p
    assert dev0 == toks0[len(PROMPT) - 1:len(PROMPT) - 1 + STEPS]


def test_tp_peer_timeout_reports_and_recovers(cuda):
    import spk

    cfg = _cfg()
    full = synth_weights(cfg, seed=5)
    m0 = DeviceModel(cfg, tp_shard(cfg, full, 0, 2), max_ctx=8, device=cuda)
    m1 = DeviceModel(cfg, tp_shard(cfg, full, 1, 2), max_ctx=8, device=cuda)   # never runs: its flags stay 0
    m0.tp_attach_ptrs([None, m1.tp_mailbox()], wait_ms=100)
    with pytest.raises(spk.SpkError, match="peer"):
        m0.forward(1, 0)
    m0.close()
    m1.close()
    # the context is still usable: a single-GPU model steps normally afterwards
    one = DeviceModel(cfg, full, max_ctx=4, device=cuda)
    nxt, logits = one.forward(1, 0)
    assert 0 <= nxt < cfg.vocab and np.isfinite(logits).all()
    one.close()
