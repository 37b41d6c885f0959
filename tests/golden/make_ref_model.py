"""Golden outputs of the reference's own whole-model GPU runtime (tools/vq/gpu/vq-model-gpu.cu,
built for sm_100a from its sources by `make -C oracle ref` into oracle/_ref/vq-model-gpu), for
seeded synthetic models in the reference's artifact format. Run on a machine with a GPU:

    python tests/golden/make_ref_model.py [out_dir]      # writes ref_model_<name>.npz

For each model it writes an artifact directory as the reference reads it (vq-model-gpu.cu:
142-226 config.json; 230-361 `<tensor>.bin` RQVQ containers and RQVF f32 sidecars; the tied
embedding a container too, :742), runs

    vq-model-gpu --dir D --config D/config.json --ids <prompt> --gen G --ctx C --no-prefill --no-tune --logits L

(token-by-token prompt, f32 KV, every matrix through the reference's fused DQV3 GEMV), and keeps
the prompt, the logits after it and the generated ids. The weights are those of
spk.model.synth_weights(cfg, seed) except the tied embedding, which is built so that one and the
same f32 matrix is both a 1-stage DQV3 container (for the reference) and ggml Q8_0 blocks (for
this build): every weight is q * 2^-9 with q an int8, the VQ codebook holds such 4-vectors
(exact in f16, gains 1.0) and each Q8_0 block has d = 2^-9 (exact in f16). tests that use the
fixtures rebuild the weights from the seeds recorded in them.
"""
from __future__ import annotations

import json
import os
import re
import struct
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "spark-x2.6-4b-q6k_b200"))

from spk import formats as F  # noqa: E402
from spk.model import MATS, ModelConfig, small_config, synth_weights  # noqa: E402

REF_BIN = os.path.join(ROOT, "oracle", "_ref", "vq-model-gpu")

# name -> (config, weight seed, prompt length, generated tokens)
MODELS = {
    "small": (small_config(), 41, 40, 24),
    "wide4": (ModelConfig(layers=4, full=[False, False, False, True]), 43, 24, 8),
}

NAMES = {"qkv": "self_attn.q_k_v_proj.weight", "attn_gate": "self_attn.g_proj.weight", "out": "self_attn.out_proj.weight",
         "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight", "down": "mlp.down_proj.weight"}


def embedding_pair(vocab: int, hidden: int, seed: int) -> tuple[bytes, bytes]:
    """(RQVQ container, Q8_0 blocks) of one f32 matrix: a seeded 4096-entry codebook of int8
    4-vectors times 2^-9, uniform indices, gains 1.0 — and the same values as Q8_0 with d = 2^-9."""
    rng = np.random.default_rng(seed)
    q_cb = np.clip(np.rint(rng.normal(0, 12, (4096, 4))), -127, 127).astype(np.int8)
    cb16 = F._f16_bits((q_cb.astype(np.float32) * np.float32(2.0 ** -9)).reshape(-1))
    idx = rng.integers(0, 4096, (vocab, hidden // 4), dtype=np.int64)
    gains16 = F._f16_bits(np.ones(vocab, np.float32))
    payload = F.v3_pack(cb16, gains16, idx, vocab, hidden, 4, 4096)
    container = F.rqvq([payload], 4, 4096, vocab, hidden)
    q = q_cb[idx].reshape(vocab * hidden // 32, 32)
    blocks = np.empty((q.shape[0], 34), np.uint8)
    blocks[:, 0:2] = np.frombuffer(np.float16(2.0 ** -9).tobytes(), np.uint8)
    blocks[:, 2:] = q.view(np.uint8)
    return container, blocks.tobytes()


def model_weights(cfg: ModelConfig, seed: int) -> tuple[dict, bytes]:
    """This build's weights for a fixture model, and the embedding container the reference reads."""
    W = synth_weights(cfg, seed=seed)
    container, q80 = embedding_pair(cfg.vocab, cfg.hidden, seed + 5)
    W["embed"] = q80
    return W, container


def rqvf(v: np.ndarray) -> bytes:
    v = np.ascontiguousarray(v, np.float32).reshape(-1)
    return b"RQVF" + struct.pack("<II", 1, v.size) + v.tobytes()


def write_artifact(d: str, cfg: ModelConfig, W: dict, embed_container: bytes) -> None:
    layer_types = ["full_attention" if f else "sliding_attention" for f in cfg.full]
    conf = {"hidden_size": cfg.hidden, "num_hidden_layers": cfg.layers, "num_attention_heads": cfg.heads,
            "num_key_value_heads": cfg.kv_heads, "head_dim": cfg.head_dim, "intermediate_size": cfg.inter,
            "vocab_size": cfg.vocab, "sliding_window": cfg.window, "rms_norm_eps": cfg.eps, "layer_types": layer_types,
            "rope_parameters": {"full_attention": {"rope_theta": cfg.rope_theta_full,
                                                   "partial_rotary_factor": cfg.rope_partial_full},
                                "sliding_attention": {"rope_theta": cfg.rope_theta_slide,
                                                      "partial_rotary_factor": cfg.rope_partial_slide}}}
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(conf, f)
    with open(os.path.join(d, "model.embedding.weight.bin"), "wb") as f:
        f.write(embed_container)
    with open(os.path.join(d, "model.norm.weight.bin"), "wb") as f:
        f.write(rqvf(W["norm"]))
    for li, L in enumerate(W["layers"]):
        for k in MATS:
            with open(os.path.join(d, f"model.layers.{li}.{NAMES[k]}.bin"), "wb") as f:
                f.write(L[k])
        with open(os.path.join(d, f"model.layers.{li}.input_layernorm.weight.bin"), "wb") as f:
            f.write(rqvf(L["in_norm"]))
        with open(os.path.join(d, f"model.layers.{li}.post_attention_layernorm.weight.bin"), "wb") as f:
            f.write(rqvf(L["post_norm"]))


def run_reference(name: str, out_dir: str) -> str:
    cfg, seed, n_prompt, n_gen = MODELS[name]
    W, container = model_weights(cfg, seed)
    prompt = np.random.default_rng(seed + 9).integers(0, cfg.vocab, n_prompt).tolist()
    with tempfile.TemporaryDirectory() as d:
        write_artifact(d, cfg, W, container)
        lpath = os.path.join(d, "logits.f32")
        cmd = [REF_BIN, "--dir", d, "--config", os.path.join(d, "config.json"), "--ids", ",".join(map(str, prompt)),
               "--gen", str(n_gen), "--ctx", str(n_prompt + n_gen + 2), "--no-prefill", "--no-tune", "--logits", lpath]
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
        if r.returncode != 0:
            raise RuntimeError(f"reference runtime failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
        logits = np.fromfile(lpath, np.float32)
    m = re.search(r"generated\s+\[([0-9, ]*)\]", r.stdout)
    gen = [int(t) for t in m.group(1).split(",")] if m and m.group(1).strip() else []
    if logits.size != cfg.vocab or len(gen) != n_gen:
        raise RuntimeError(f"unexpected reference output:\n{r.stdout}")
    path = os.path.join(out_dir, f"ref_model_{name}.npz")
    np.savez_compressed(path, prompt=np.array(prompt, np.int32), logits=logits, generated=np.array(gen, np.int32),
                        seed=np.int64(seed), log=np.array(r.stdout))
    return path


if __name__ == "__main__":
    out = sys.argv[1] if len(sys.argv) > 1 else HERE
    for name in MODELS:
        print("wrote", run_reference(name, out), flush=True)
