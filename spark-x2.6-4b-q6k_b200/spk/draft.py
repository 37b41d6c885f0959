"""Host side of the DSpark draft: the dspark::draft API over libspk.

Mirrors tools/dspark/src/{manifest.rs Header, draft.rs Draft::open / encode_features /
decode_block}: ``DraftConfig`` is the manifest header (defaults are the released
Spark-X2.6-4B DSpark checkpoint's: 5 sliding-window layers, hidden 2560, 16/4 heads of
256, tanh-GELU, window 512, non-causal block of 7 sampled from the anchor, target layers
3, 11, 19, 26, 34, a rank-256 Markov head and a confidence head); ``DeviceDraft`` holds
the weights on device and runs spk_draft_encode / spk_draft_block.

``synth_draft`` builds seeded random-init BF16 weights of that architecture (the real
draft is not available here): matrices N(0, 0.02^2) rounded to bf16, norms 1 + N(0, 0.05^2).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import SpkError, check, lib

MAX_LAYERS = 32


@dataclass
class DraftConfig:
    hidden: int = 2560
    layers: int = 5
    ffn: int = 10240
    heads: int = 16
    kv_heads: int = 4
    head_dim: int = 256
    vocab: int = 131072
    mask_token: int = 2
    rope_full_dims: int = 64
    rope_swa_dims: int = 256
    rope_full_theta: float = 5e6
    rope_swa_theta: float = 1e4
    eps: float = 1e-6
    act: str = "gelu"              # "gelu" (ggml's tanh form) or "silu"
    swa_window: int = 512
    swa_pattern: list = field(default_factory=lambda: [1] * 5)
    causal: bool = False
    block_size: int = 7
    sample_from_anchor: bool = True
    target_layers: list = field(default_factory=lambda: [3, 11, 19, 26, 34])
    rank: int = 256                # Markov head rank (0: no Markov head)
    conf: bool = True              # confidence head (conf_proj, conf_bias)
    gate: bool = True              # attn_gate (excludes the q/k norms)
    qk_norm: bool = False
    post_norms: bool = False       # attn_post_norm and ffn_post_norm
    out_scale: float = 0.0         # layer_out_scale (0: none)

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def n_target(self) -> int:
        return len(self.target_layers)

    def block_rows(self, n_draft: int) -> int:
        """draft.rs:652-660."""
        if self.rank:
            return n_draft if self.sample_from_anchor else n_draft + 1
        return n_draft + 1

    def draft_max(self) -> int:
        """spec.rs:285-292: the proposals one block yields."""
        if self.rank and self.sample_from_anchor:
            return self.block_size
        return max(self.block_size - 1, 0)

    def i_beg(self) -> int:
        """spec.rs:130: the first block row that is a proposal."""
        return 0 if (self.rank and self.sample_from_anchor) else 1

    def as_oracle(self) -> dict:
        return {"hidden": self.hidden, "layers": self.layers, "heads": self.heads, "kv_heads": self.kv_heads,
                "head_dim": self.head_dim, "ffn": self.ffn, "vocab": self.vocab, "mask_token": self.mask_token,
                "rope_full_dims": self.rope_full_dims, "rope_swa_dims": self.rope_swa_dims,
                "rope_full_theta": self.rope_full_theta, "rope_swa_theta": self.rope_swa_theta, "eps": self.eps,
                "act": 1 if self.act == "silu" else 0, "swa_window": self.swa_window,
                "causal": int(self.causal), "block_size": self.block_size,
                "sample_from_anchor": int(self.sample_from_anchor), "n_target": self.n_target,
                "swa_pattern": list(self.swa_pattern)}


def small_draft_config(**kw) -> DraftConfig:
    """A CPU-oracle-sized draft with the released checkpoint's structure."""
    base = dict(hidden=512, layers=2, ffn=1024, heads=4, kv_heads=2, head_dim=128, vocab=4096, mask_token=2,
                swa_window=16, swa_pattern=[1, 1], block_size=7, target_layers=[0, 1, 3], rank=32)
    base.update(kw)
    return DraftConfig(**base)


# --------------------------------------------------------------- bf16 helpers ---
def to_bf16(a: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bits (round to nearest even), as torch and the converter store them."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    """bf16 bits -> f32 (exact)."""
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


MATS = ("q", "k", "v", "gate", "out", "ffn_gate", "ffn_up", "ffn_down")
VECS = ("norm", "q_norm", "k_norm", "ffn_norm", "attn_post", "ffn_post")


def mat_shapes(cfg: DraftConfig) -> dict:
    H = cfg.hidden
    return {"q": (cfg.q_dim, H), "k": (cfg.kv_dim, H), "v": (cfg.kv_dim, H), "gate": (cfg.heads, H),
            "out": (H, cfg.q_dim), "ffn_gate": (cfg.ffn, H), "ffn_up": (cfg.ffn, H), "ffn_down": (H, cfg.ffn)}


def synth_draft(cfg: DraftConfig, seed: int = 0, sigma: float = 0.02) -> dict:
    """Seeded random-init draft weights: bf16 matrices as uint16 arrays, f32 vectors."""
    rng = np.random.default_rng(seed)

    def mat(r, c):
        return to_bf16(rng.standard_normal((r, c), dtype=np.float32) * np.float32(sigma))

    def vec(n):
        return (1.0 + 0.05 * rng.standard_normal(n)).astype(np.float32)

    H = cfg.hidden
    layers = []
    for _ in range(cfg.layers):
        L = {n: mat(*s) for n, s in mat_shapes(cfg).items() if n != "gate" or cfg.gate}
        L["norm"], L["ffn_norm"] = vec(H), vec(H)
        if cfg.qk_norm and not cfg.gate:
            L["q_norm"], L["k_norm"] = vec(cfg.head_dim), vec(cfg.head_dim)
        if cfg.post_norms:
            L["attn_post"], L["ffn_post"] = vec(H), vec(H)
        L["out_scale"] = float(cfg.out_scale)
        layers.append(L)
    g = {"fc": mat(H, cfg.n_target * H), "fc_norm": vec(cfg.n_target * H).reshape(cfg.n_target, H),
         "enc_norm": vec(H), "out_norm": vec(H)}
    if cfg.rank:
        # the Markov bias at the scale of the head's logits, so it moves the argmax
        g["markov_w1"] = mat(cfg.vocab, cfg.rank)
        g["markov_w2"] = to_bf16(rng.standard_normal((cfg.vocab, cfg.rank), dtype=np.float32) * np.float32(1.0))
    if cfg.conf and cfg.rank:
        g["conf_proj"] = (sigma * rng.standard_normal(H + cfg.rank)).astype(np.float32)
        g["conf_bias"] = 0.1
    return {"layers": layers, "globals": g}


def oracle_weights(cfg: DraftConfig, W: dict):
    """The same weights as the oracle takes them (bf16 expanded to f32)."""
    layers = []
    for L in W["layers"]:
        d = {n: bf16_to_f32(L[n]).reshape(L[n].shape) for n in MATS if n in L}
        d.update({n: L[n] for n in VECS if n in L})
        d["out_scale"] = L.get("out_scale", 0.0)
        layers.append(d)
    g = dict(W["globals"])
    for n in ("fc", "markov_w1", "markov_w2"):
        if n in g:
            g[n] = bf16_to_f32(g[n]).reshape(g[n].shape)
    return layers, g


# ------------------------------------------------------------------- the ABI ---
class _DraftCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "layers", "heads", "kv_heads", "head_dim", "ffn", "vocab",
                                        "mask_token", "rope_full_dims", "rope_swa_dims")] + \
               [(n, C.c_float) for n in ("rope_full_theta", "rope_swa_theta", "eps")] + \
               [(n, C.c_int) for n in ("act", "swa_window", "causal", "block_size", "sample_from_anchor",
                                        "n_target", "rank", "max_ctx")] + \
               [("swa_pattern", C.c_int * MAX_LAYERS)]


class _DraftLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("q", "k", "v", "gate", "out", "ffn_gate", "ffn_up", "ffn_down",
                                          "norm", "q_norm", "k_norm", "ffn_norm", "attn_post", "ffn_post")] + \
               [("out_scale", C.c_float)]


class _DraftGlobals(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("fc", "fc_norm", "enc_norm", "out_norm", "markov_w1", "markov_w2",
                                          "conf_proj")] + [("conf_bias", C.c_float)]


class DeviceDraft:
    """dspark::draft::Draft on the GPU: Draft::open (weights to device), encode_features,
    decode_block. The target supplies its Q8_0 embedding and its layer-input captures."""

    def __init__(self, cfg: DraftConfig, weights: dict, max_ctx: int, device="cuda:0", stream=None):
        import torch

        self.cfg = cfg
        self.device = torch.device(device)
        self.stream = stream if stream is not None else torch.cuda.Stream(device=self.device)
        if len(cfg.swa_pattern) != cfg.layers or cfg.layers > MAX_LAYERS:
            raise SpkError("swa_pattern must have one entry per layer")
        pat = (C.c_int * MAX_LAYERS)(*([int(v) for v in cfg.swa_pattern] + [0] * (MAX_LAYERS - cfg.layers)))
        c = _DraftCfg(cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                      cfg.mask_token, cfg.rope_full_dims, cfg.rope_swa_dims, cfg.rope_full_theta,
                      cfg.rope_swa_theta, cfg.eps, 1 if cfg.act == "silu" else 0, cfg.swa_window, int(cfg.causal),
                      cfg.block_size, int(cfg.sample_from_anchor), cfg.n_target, cfg.rank, max_ctx, pat)
        L = lib()
        self.h = L.spk_draft_create(C.byref(c), C.c_void_p(self.stream.cuda_stream))
        if not self.h:
            raise SpkError(L.spk_last_error().decode())
        self.max_ctx = max_ctx
        self._keep = []
        self.weight_bytes = 0
        for li, Lw in enumerate(weights["layers"]):
            p = _DraftLayer()
            for n in MATS + VECS:
                if Lw.get(n) is not None:
                    setattr(p, n, self._dev(Lw[n]))
            p.out_scale = float(Lw.get("out_scale", 0.0))
            check(L.spk_draft_set_layer(self.h, li, C.byref(p)), f"draft layer {li}")
        gw = weights["globals"]
        g = _DraftGlobals()
        for n in ("fc", "fc_norm", "enc_norm", "out_norm", "markov_w1", "markov_w2", "conf_proj"):
            if gw.get(n) is not None:
                setattr(g, n, self._dev(gw[n]))
        g.conf_bias = float(gw.get("conf_bias", 0.0))
        check(L.spk_draft_set_globals(self.h, C.byref(g)), "draft globals")
        self._ids = np.zeros(8, np.int32)
        self._conf = np.zeros(8, np.float32)
        torch.cuda.synchronize(self.device)

    def _dev(self, a) -> int:
        import torch

        if isinstance(a, torch.Tensor):
            t = a.to(self.device).contiguous()
        else:
            a = np.ascontiguousarray(a)
            t = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).to(self.device)
        self._keep.append(t)
        if t.dtype in (torch.int16, torch.bfloat16):
            self.weight_bytes += t.numel() * 2
        return t.data_ptr()

    def use_target_head(self, target) -> bool:
        """Read the block's logits from the target's tiled head table when it has one (the
        same Q8_0 embedding, re-laid for the tensor-core head; one GPU only)."""
        p = lib().spk_model_head_tiled(target.h) if target.tp[1] == 1 else None
        check(lib().spk_draft_set_head_tiled(self.h, C.c_void_p(p) if p else None), "draft head")
        return bool(p)

    def encode_features(self, caps_ptr: int, slot_stride: int, p0: int, p1: int):
        """encode_features for the committed positions [p0, p1) (caps: the target's device
        captures, spk_model_captures)."""
        check(lib().spk_draft_encode(self.h, C.c_void_p(caps_ptr), slot_stride, p0, p1), f"encode [{p0}, {p1})")

    def decode_block(self, embed_ptr: int, vocab: int, anchor: int, pos0: int, n_draft: int, want_logits=False):
        """(argmax ids, conf, logits [n_block][vocab] or None) of one block-diffusion decode."""
        n = lib().spk_draft_block(self.h, C.c_void_p(embed_ptr), vocab, anchor, pos0, n_draft,
                                  self._ids.ctypes.data_as(C.c_void_p), self._conf.ctypes.data_as(C.c_void_p))
        if n < 0:
            raise SpkError(f"decode_block: {lib().spk_last_error().decode()}")
        logits = None
        if want_logits:
            import torch

            self.stream.synchronize()
            view = _DeviceView(lib().spk_draft_logits(self.h), (n, vocab))
            logits = torch.as_tensor(view, device=self.device).cpu().numpy().copy()
        return self._ids[:n].tolist(), self._conf[:n].copy(), logits

    def close(self):
        if self.h:
            lib().spk_draft_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()


class _DeviceView:
    """An f32 view of a library-owned device buffer (__cuda_array_interface__); copy it out."""

    def __init__(self, ptr: int, shape: tuple):
        if not ptr:
            raise SpkError("no device buffer")
        self.__cuda_array_interface__ = {"shape": shape, "typestr": "<f4", "data": (int(ptr), False), "version": 3,
                                         "strides": None}
