"""Tuning profiles on the GPU: the model applies a profile per matrix geometry (the reference
runtime's substitution, vq-model-gpu.cu:301-324) with the decode step still matching the CPU
oracle, and the tuner (spk.tune, vq-tune's counterpart) writes a profile this device trusts."""
import os

import numpy as np
import pytest

import oracle
from spk import SpkError
from spk import formats as F
from spk import vqprof as P
from spk.model import DeviceModel, mat_shapes, small_config, synth_weights

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def oracle_model(cfg, W, max_ctx):
    layers = [{"in_norm": L["in_norm"], "post_norm": L["post_norm"],
               **{n: oracle.decode(L[n]) for n in ("qkv", "attn_gate", "out", "gate", "up", "down")}}
              for L in W["layers"]]
    return oracle.Model(cfg.as_oracle(), layers, oracle.q80_dequant(W["embed"], cfg.vocab, cfg.hidden), W["norm"],
                        max_ctx)


def run_greedy(dev, ref, prompt, steps):
    """Teacher-forced prompt then the oracle's greedy ids; returns (worst logits relL2,
    id mismatches outside near-ties)."""
    worst, mism, tok = 0.0, 0, prompt[0]
    for pos in range(len(prompt) + steps):
        want = ref.forward(tok, pos)
        nxt, got = dev.forward(tok, pos)
        worst = max(worst, rel(got, want))
        o_id = oracle.argmax(want)
        t = np.sort(want)[-2:]
        if nxt != o_id and float(t[1] - t[0]) > 1e-3 * max(1.0, abs(float(want.max()))):
            mism += 1
        tok = prompt[pos + 1] if pos + 1 < len(prompt) else o_id
    return worst, mism


def test_profile_moves_matrices_to_the_table_kernel_and_back(cuda):
    cfg = small_config()
    W = synth_weights(cfg, seed=5, exact_q80=True)
    prompt, steps = [3, 99, 1024, 7], 20
    dev = DeviceModel(cfg, W, max_ctx=len(prompt) + steps + 1, kv_f16=False)
    try:
        # the heuristic: every matrix of this small geometry on the code-word kernel
        assert all(dev.kernel_of(li, mi) == 3 for li in range(cfg.layers) for mi in range(6))
        shapes = mat_shapes(cfg)
        prof = P.new(0, "caller-trusted", "0")
        for n in ("qkv", "out", "gate", "down"):   # gate's entry covers up_proj (same geometry)
            r, c = shapes[n]
            prof.add_gemv(4, 4096, r, c, 1, P.VARIANT_TABLE, 512, 0.0)
        dev.use_profile(prof)
        for li in range(cfg.layers):
            assert [dev.kernel_of(li, mi) for mi in range(6)] == [4, 3, 4, 4, 4, 4]
        worst, mism = run_greedy(dev, oracle_model(cfg, W, len(prompt) + steps + 1), prompt, steps)
        assert worst < 1e-4 and mism == 0, (worst, mism)
        # an entry naming the code-word kernel, and no profile at all: back to the heuristic
        prof2 = P.new(0, "caller-trusted", "0")
        r, c = shapes["gate"]
        prof2.add_gemv(4, 4096, r, c, 1, 3, 512, 0.0)
        dev.use_profile(prof2)
        assert all(dev.kernel_of(li, 3) == 3 for li in range(cfg.layers))
        dev.use_profile(None)
        assert all(dev.kernel_of(li, mi) == 3 for li in range(cfg.layers) for mi in range(6))
        dev.reset()
        worst, mism = run_greedy(dev, oracle_model(cfg, W, len(prompt) + steps + 1), prompt, 4)
        assert worst < 1e-4 and mism == 0, (worst, mism)
    finally:
        dev.close()


def test_tuner_writes_a_profile_this_device_trusts(cuda, tmp_path):
    from spk import tune

    mats = {"blk.0.ffn_up": F.random_rvq_fast(1024, 512, seed=11), "blk.0.attn_output": F.random_rvq_fast(512, 1024, seed=12),
            "blk.1.ffn_up": F.random_rvq_fast(1024, 512, seed=13)}
    d = str(tmp_path / "art")
    P.write_artifact(d, mats, 4, 4096, 2)
    lines = []
    path = tune.tune(d, iters=5, warmup=2, log=lines.append)
    assert path == os.path.join(d, "vq-tune.profile")
    p = P.load(path)
    assert P.trust(p, P.fingerprint(d), P.device_name()) == 0
    assert p.n == 2   # one entry per geometry
    for (r, c) in ((1024, 512), (512, 1024)):
        e = P.find(p, 0, 4, 4096, r, c, 1)
        assert e is not None and e.variant in (3, P.VARIANT_TABLE) and e.rate > 0
    # another artifact's profile at the path is kept unless forced
    other = P.new(1, P.device_name(), "0")
    P.write(path, other)
    with pytest.raises(SpkError, match="belongs to artifact"):
        tune.tune(d, iters=2, warmup=1, log=lines.append)
    tune.tune(d, iters=2, warmup=1, force=True, log=lines.append)
    assert P.load(path).artifact == P.fingerprint(d)
