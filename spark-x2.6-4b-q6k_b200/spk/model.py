"""Host side of the decode step: the vq_runtime Model API over libspk.

Mirrors tools/vq-runtime/src/{config.rs, model.rs}: ``ModelConfig`` is
``Config`` (defaults are the Spark-X2.6-4B values), ``DeviceModel`` offers
``forward(token, pos) -> logits``, ``argmax``, ``rollback``, ``reset``. The
compute is libspk's (include/spk.h, spk_model_*); this module uploads weights
and marshals pointers.

``synth_weights`` builds a seeded random-init model in the reference's formats
(DQV3 residual-VQ containers for every projection, a Q8_0 tied embedding/head,
f32 norms), standing in for the absent real checkpoint.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import SpkError, check, dev_bytes, lib
from . import formats as F


@dataclass
class ModelConfig:
    """tools/vq-runtime/src/config.rs:16-30 (values from models/quantize.log:19-35)."""

    hidden: int = 2560
    layers: int = 36
    heads: int = 16
    kv_heads: int = 4
    head_dim: int = 256
    inter: int = 10240
    vocab: int = 131072
    window: int = 512
    eps: float = 1e-6
    rope_theta_full: float = 5_000_000.0
    rope_partial_full: float = 0.25
    rope_theta_slide: float = 10_000.0
    rope_partial_slide: float = 1.0
    full: list = field(default_factory=lambda: [(i % 4) == 3 for i in range(36)])   # [T,T,T,F] pattern

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def as_oracle(self) -> dict:
        d = {k: getattr(self, k) for k in ("hidden", "layers", "heads", "kv_heads", "head_dim", "inter", "vocab",
                                           "window", "eps", "rope_theta_full", "rope_partial_full",
                                           "rope_theta_slide", "rope_partial_slide")}
        d["full"] = [int(f) for f in self.full]
        return d


def small_config(layers: int = 4, hidden: int = 512, heads: int = 4, kv_heads: int = 1, head_dim: int = 128,
                 inter: int = 1024, vocab: int = 4096, window: int = 16) -> ModelConfig:
    """A reduced geometry with the same structure (GQA group 4, [T,T,T,F] layers), for
    parity runs the CPU oracle finishes in seconds."""
    return ModelConfig(hidden=hidden, layers=layers, heads=heads, kv_heads=kv_heads, head_dim=head_dim, inter=inter,
                       vocab=vocab, window=window, full=[(i % 4) == 3 for i in range(layers)])


MATS = ("qkv", "attn_gate", "out", "gate", "up", "down")


def mat_shapes(cfg: ModelConfig) -> dict:
    """model.rs:138-174: out x in of every projection."""
    return {"qkv": (cfg.q_dim + 2 * cfg.kv_dim, cfg.hidden), "attn_gate": (cfg.heads, cfg.hidden),
            "out": (cfg.hidden, cfg.q_dim), "gate": (cfg.inter, cfg.hidden), "up": (cfg.inter, cfg.hidden),
            "down": (cfg.hidden, cfg.inter)}


def synth_weights(cfg: ModelConfig, seed: int = 0, nc: int = 4096, stages: int = 2, exact_q80: bool = False) -> dict:
    """Seeded random-init weights: per layer a DQV3 container per projection (codebooks
    N(0, 0.02^2), residual stage scaled down, gains 1.0), norms N(1, 0.1^2); a Q8_0 tied
    embedding. exact_q80 quantizes an explicit N(0, 0.02^2) matrix (small vocab only)."""
    rng = np.random.default_rng(seed)
    shapes = mat_shapes(cfg)
    layers = []
    for li in range(cfg.layers):
        L = {}
        for k, n in enumerate(MATS):
            r, c = shapes[n]
            s = seed * 1000 + li * 16 + k
            L[n] = F.random_rvq_fast(r, c, 4, nc, stages, seed=s) if nc in (4096, 8192) else \
                F.random_rvq(r, c, 4, nc, stages, seed=s)
        L["in_norm"] = rng.normal(1.0, 0.1, cfg.hidden).astype(np.float32)
        L["post_norm"] = rng.normal(1.0, 0.1, cfg.hidden).astype(np.float32)
        layers.append(L)
    if exact_q80:
        embed = F.quantize_q8_0(rng.normal(0, 0.02, (cfg.vocab, cfg.hidden)).astype(np.float32))
    else:
        embed = F.synth_q8_0(cfg.vocab, cfg.hidden, seed=seed + 7)
    norm = rng.normal(1.0, 0.1, cfg.hidden).astype(np.float32)
    return {"layers": layers, "embed": embed, "norm": norm}


def tp_layout(cfg: ModelConfig, rank: int, world: int) -> dict:
    """What rank `rank` of `world` holds (the sharding libspk's tensor-parallel step runs):
    q heads [h0, h0+hl), KV heads [k0, k0+kl) (replicated when world > kv_heads),
    intermediate rows [i0, i0+il), vocabulary rows [v0, v0+vl)."""
    t = world
    if cfg.heads % t or (cfg.kv_heads % t and t % cfg.kv_heads) or cfg.inter % t or cfg.vocab % t:
        raise ValueError(f"{t}-way tensor parallelism does not divide this geometry")
    hl = cfg.heads // t
    kl = cfg.kv_heads // t if cfg.kv_heads >= t else 1
    k0 = rank * kl if cfg.kv_heads >= t else rank * cfg.kv_heads // t
    il, vl = cfg.inter // t, cfg.vocab // t
    return {"h0": rank * hl, "hl": hl, "k0": k0, "kl": kl, "i0": rank * il, "il": il, "v0": rank * vl, "vl": vl}


def tp_shard(cfg: ModelConfig, weights: dict, rank: int, world: int) -> dict:
    """Rank `rank`'s shard of full weights (exact re-cuts of the DQV3 containers,
    formats.shard_rows / shard_cols): q_k_v_proj rows of its q and KV heads, g_proj rows
    of its heads, out_proj input columns of its heads, gate/up rows and down input
    columns of its intermediate slice. The Q8_0 embedding (also the head) and the
    norms stay whole; the head GEMV reads the rank's vocabulary rows of it."""
    if world <= 1:
        return weights
    lay = tp_layout(cfg, rank, world)
    hd, qd = cfg.head_dim, cfg.q_dim
    q_rows = np.arange(lay["h0"] * hd, (lay["h0"] + lay["hl"]) * hd)
    kv = np.arange(lay["k0"] * hd, (lay["k0"] + lay["kl"]) * hd)
    qkv_rows = np.concatenate([q_rows, qd + kv, qd + cfg.kv_dim + kv])
    i0, i1 = lay["i0"], lay["i0"] + lay["il"]
    layers = []
    for Lw in weights["layers"]:
        layers.append({
            "qkv": F.shard_rows(Lw["qkv"], qkv_rows),
            "attn_gate": F.shard_rows(Lw["attn_gate"], np.arange(lay["h0"], lay["h0"] + lay["hl"])),
            "out": F.shard_cols(Lw["out"], lay["h0"] * hd, (lay["h0"] + lay["hl"]) * hd),
            "gate": F.shard_rows(Lw["gate"], np.arange(i0, i1)),
            "up": F.shard_rows(Lw["up"], np.arange(i0, i1)),
            "down": F.shard_cols(Lw["down"], i0, i1),
            "in_norm": Lw["in_norm"], "post_norm": Lw["post_norm"]})
    return {"layers": layers, "embed": weights["embed"], "norm": weights["norm"], "tp": (rank, world)}


def exchange_handles(handle: bytes, group=None) -> list:
    """Every rank's mailbox handle, in rank order, over torch.distributed (any backend)."""
    import torch.distributed as dist

    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


class _Cfg(C.Structure):
    _fields_ = [("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("inter", C.c_int), ("vocab", C.c_int), ("window", C.c_int),
                ("eps", C.c_float), ("rope_theta_full", C.c_float), ("rope_partial_full", C.c_float),
                ("rope_theta_slide", C.c_float), ("rope_partial_slide", C.c_float),
                ("full", C.POINTER(C.c_int)), ("max_ctx", C.c_int), ("kv_type", C.c_int),
                ("tp_rank", C.c_int), ("tp_world", C.c_int)]


class VqMatrix(C.Structure):
    """spk_vq_matrix: stage device pointers + geometry."""

    _fields_ = [("stages", C.c_void_p * 4), ("nstages", C.c_int), ("dim", C.c_int), ("nc", C.c_int),
                ("rows", C.c_int), ("cols", C.c_int), ("v3", C.c_int)]


def upload_container(buf: bytes, device) -> tuple[VqMatrix, list]:
    """Every stage in its own device buffer with zeroed slack (vq-model-gpu.cu:278-288)."""
    c = F.parse_container(buf)
    keep = []
    M = VqMatrix()
    for s in range(c.nstages):
        o = c.stage_offset(s)
        t = dev_bytes(buf[o:o + c.stage_bytes], device)
        keep.append(t)
        M.stages[s] = t.data_ptr()
    M.nstages, M.dim, M.nc, M.rows, M.cols, M.v3 = c.nstages, c.dim, c.nc, c.rows, c.cols, int(c.v3)
    return M, keep


class DeviceModel:
    """vq_runtime::model::Model on the GPU (model.rs:260-615)."""

    def __init__(self, cfg: ModelConfig, weights: dict, max_ctx: int, kv_f16: bool = False, device="cuda:0",
                 stream=None, kv_q8: bool = False):
        """``weights`` are full weights, or one rank's shard from ``tp_shard`` (then the model is
        that tensor-parallel rank and needs ``tp_connect`` before its first step)."""
        import torch

        self.cfg = cfg
        self.device = torch.device(device)
        self.stream = stream if stream is not None else torch.cuda.Stream(device=self.device)
        self._keep = []
        self._full = (C.c_int * cfg.layers)(*[int(f) for f in cfg.full])
        c = _Cfg(cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.inter, cfg.vocab, cfg.window,
                 cfg.eps, cfg.rope_theta_full, cfg.rope_partial_full, cfg.rope_theta_slide, cfg.rope_partial_slide,
                 self._full, max_ctx, 2 if kv_q8 else int(kv_f16), *weights.get("tp", (0, 1)))
        self.tp = weights.get("tp", (0, 1))
        L = lib()
        L.spk_model_create.restype = C.c_void_p
        self.h = L.spk_model_create(C.byref(c), C.c_void_p(self.stream.cuda_stream))
        if not self.h:
            raise SpkError(L.spk_last_error().decode())
        self.max_ctx = max_ctx
        self.weight_bytes = 0
        self.mats, self.norms = [], []   # per layer: {name: VqMatrix}, (in_norm, post_norm) device tensors
        for li, Lw in enumerate(weights["layers"]):
            mats = []
            for n in MATS:
                M, keep = upload_container(Lw[n], self.device)
                self._keep += keep
                mats.append(M)
                self.weight_bytes += len(Lw[n]) - 32
            nin = torch.from_numpy(np.ascontiguousarray(Lw["in_norm"])).to(self.device)
            npost = torch.from_numpy(np.ascontiguousarray(Lw["post_norm"])).to(self.device)
            self._keep += [nin, npost, mats]
            self.mats.append(dict(zip(MATS, mats)))
            self.norms.append((nin, npost))
            check(L.spk_model_set_layer(self.h, li, *[C.byref(M) for M in mats], nin.data_ptr(), npost.data_ptr()),
                  f"layer {li}")
        emb = dev_bytes(weights["embed"], self.device)
        norm = torch.from_numpy(np.ascontiguousarray(weights["norm"])).to(self.device)
        self._keep += [emb, norm]
        self.embed_dev = emb   # the tied Q8_0 embedding/head (the draft's TargetEmbed)
        self.weight_bytes += len(weights["embed"])
        check(L.spk_model_set_head(self.h, emb.data_ptr(), norm.data_ptr()), "head")
        self._logits = np.empty(cfg.vocab, np.float32)
        torch.cuda.synchronize(self.device)   # uploads ran on torch's stream; the model runs on its own

    def tp_handle(self) -> bytes:
        """This rank's mailbox as a cudaIpcMemHandle_t (64 bytes)."""
        buf = C.create_string_buffer(64)
        check(lib().spk_model_tp_handle(self.h, buf, 64), "tp_handle")
        return buf.raw

    def tp_attach(self, handles: list, wait_ms: int = 5000):
        blob = b"".join(handles)
        check(lib().spk_model_tp_attach(self.h, blob, len(blob), wait_ms), "tp_attach")

    def tp_connect(self, group=None, wait_ms: int = 5000):
        """Exchange mailbox handles with the other ranks (torch.distributed) and attach."""
        self.tp_attach(exchange_handles(self.tp_handle(), group), wait_ms)

    def tp_mailbox(self) -> int:
        return lib().spk_model_tp_mailbox(self.h) or 0

    def tp_attach_ptrs(self, mailboxes: list, wait_ms: int = 5000):
        """Mailboxes as pointers valid in this process (None for this rank's own)."""
        arr = (C.c_void_p * len(mailboxes))(*[m or None for m in mailboxes])
        check(lib().spk_model_tp_attach_ptrs(self.h, arr, len(mailboxes), wait_ms), "tp_attach_ptrs")

    def verify(self, tokens, pos: int, want_logits: bool = False):
        """Speculative verify (spec.rs:197-205): tokens (anchor + proposals, <= 8) at positions
        pos.. in one batched forward. Returns (greedy ids after each token, logits [n][vocab]
        or None); afterwards len = pos + len(tokens)."""
        n = len(tokens)
        tk = (C.c_int * n)(*[int(t) for t in tokens])
        nxt = (C.c_int * n)()
        lg = np.empty((n, self.cfg.vocab), np.float32) if want_logits else None
        check(lib().spk_model_verify(self.h, tk, n, pos, nxt, lg.ctypes.data_as(C.c_void_p) if lg is not None else None),
              f"verify({n} tokens at {pos})")
        return list(nxt), lg

    def prefill(self, tokens, pos: int = 0, want_logits: bool = True):
        """The prompt (forward_batch in chunks of up to 128 tokens on the tensor cores): tokens at
        positions pos.., every K/V row stored. Returns (the last token's greedy next id, its logits
        or None); afterwards len = pos + len(tokens)."""
        n = len(tokens)
        tk = (C.c_int * n)(*[int(t) for t in tokens])
        nxt = C.c_int()
        lg = np.empty(self.cfg.vocab, np.float32) if want_logits else None
        check(lib().spk_model_prefill(self.h, tk, n, pos, C.byref(nxt), lg.ctypes.data_as(C.c_void_p) if lg is not None
                                      else None), f"prefill({n} tokens at {pos})")
        return int(nxt.value), lg

    def spec_round(self, anchor: int, proposals, pos0: int):
        """One verify round of spec.rs:177-245: returns (accepted proposals k, the target's
        token after them, the ids) and leaves the cache at pos0 + k + 1 positions."""
        tgt, _ = self.verify([anchor] + list(proposals), pos0)
        k = 0
        while k < len(proposals) and tgt[k] == proposals[k]:
            k += 1
        self.rollback(pos0 + k + 1)
        return k, tgt[k], tgt

    def enable_capture(self, layers) -> None:
        """Model::enable_capture (model.rs:322-343): the residual entering each listed layer is
        kept on device at every position the step and the verify batch visit."""
        arr = (C.c_int * len(layers))(*[int(v) for v in layers])
        check(lib().spk_model_enable_capture(self.h, arr, len(layers)), "enable_capture")

    def captures(self) -> tuple[int, int]:
        """(device pointer, slot stride in floats) of the layer-input captures (Model::captured)."""
        st = C.c_size_t()
        p = lib().spk_model_captures(self.h, C.byref(st))
        if not p:
            raise SpkError("capture is not enabled")
        return p, st.value

    def trace(self) -> list:
        """One decode step (as run() does) with every launch's device time: [(name, us), ...]
        in enqueue order (spk_model_trace). All tensor-parallel ranks trace together. Under
        tensor parallelism out_proj and down_proj carry the residual exchange themselves where
        the code-word kernel takes the matrix; otherwise a tp_sum launch follows each."""
        tp = self.tp[1] > 1

        def names_for(fused: bool) -> list:
            ex = ["tp_sum"] if tp and not fused else []
            layer = ["qkv_g", "attention", "out"] + ex + ["gate_up", "down"] + ex
            return ["embed"] + layer * self.cfg.layers + ["head"] + (["tp_argmax"] if tp else []) + ["advance"]

        full = names_for(False)
        buf = (C.c_float * len(full))()
        n = lib().spk_model_trace(self.h, buf, len(full))
        if n < 0:
            raise SpkError(f"trace: {lib().spk_last_error().decode()}")
        for names in (names_for(True), full):
            if len(names) == n:
                return list(zip(names, [float(v) for v in buf[:n]]))
        raise SpkError(f"trace: {n} launches in a step, neither the fused nor the separate exchange layout")

    def use_profile(self, profile) -> None:
        """Apply a trusted VQPROF 1 profile (spk.vqprof.Profile) per matrix geometry, or None to
        return to the kernel heuristic (spk_model_use_profile). The caller checks trust first
        (spk.vqprof.trust, the reference runtime's gate, vq-model-gpu.cu:1094-1122)."""
        check(lib().spk_model_use_profile(self.h, C.byref(profile) if profile is not None else None), "use_profile")

    def kernel_of(self, layer: int, matrix: int) -> int:
        """The decode step's kernel for a layer matrix (0 qkv .. 5 down): 4 table, 3 code-word."""
        k = lib().spk_model_kernel_of(self.h, layer, matrix)
        if k < 0:
            raise SpkError(f"kernel_of: {lib().spk_last_error().decode()}")
        return k

    def forward(self, token: int, pos: int, want_logits: bool = True):
        """Model::forward: returns (next_id, logits or None) through host buffers."""
        nxt = C.c_int()
        lp = self._logits.ctypes.data_as(C.c_void_p) if want_logits else None
        check(lib().spk_model_forward(self.h, token, pos, lp, C.byref(nxt)), f"forward({token}, {pos})")
        return nxt.value, (self._logits.copy() if want_logits else None)

    def begin(self, token: int, pos: int, ids_dev=None, cap: int = 0):
        import torch

        torch.cuda.synchronize(self.device)   # ids_dev may have been written on torch's stream
        check(lib().spk_model_begin(self.h, token, pos, ids_dev.data_ptr() if ids_dev is not None else None, cap))

    def run(self, steps: int):
        check(lib().spk_model_run(self.h, steps), "run")

    def rollback(self, pos: int):
        check(lib().spk_model_rollback(self.h, pos), "rollback")

    def reset(self):
        check(lib().spk_model_reset(self.h), "reset")

    def advance_len(self, n: int):
        check(lib().spk_model_advance_len(self.h, n), "advance_len")

    def write_kv(self, layer: int, pos0: int, k, v):
        """Cache rows of `layer` at pos0.. from f32 device tensors k, v [n][kv_heads * head_dim]
        (keys already roped), stored in the cache's type; the host length is not changed."""
        n = int(k.shape[0])
        check(lib().spk_model_write_kv(self.h, layer, pos0, n, k.data_ptr(), v.data_ptr()), "write_kv")

    @property
    def len(self) -> int:
        return lib().spk_model_len(self.h)

    @staticmethod
    def argmax(logits: np.ndarray) -> int:
        """Model::argmax (model.rs:594-604): first index of the maximum."""
        return int(np.argmax(np.where(np.isnan(logits), -np.inf, logits)))

    def close(self):
        if self.h:
            self.stream.synchronize()
            lib().spk_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
