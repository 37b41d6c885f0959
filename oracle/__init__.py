"""ctypes face of the CPU oracle (liboracle.so, built from oracle.c / model.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg as the checker. The product never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_DECODE = os.path.join(HERE, "_ref", "decode")
REF_VQG = os.path.join(HERE, "_ref", "libvqg_ref.so")

_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.orc_f16.argtypes = [C.c_uint16]
        L.orc_f16.restype = C.c_float
        L.orc_container_decode.argtypes = [_u8p, C.c_size_t, _f32p, C.c_char_p, C.c_int]
        L.orc_container_gemv_fused.argtypes = [_u8p, C.c_size_t, _f32p, _f32p, C.c_int, C.c_char_p, C.c_int]
        L.orc_container_info.argtypes = [_u8p, C.c_size_t] + [C.POINTER(C.c_int)] * 6 + [C.c_char_p, C.c_int]
        L.orc_matvec.argtypes = [_f32p, C.c_size_t, C.c_size_t, _f32p, _f32p, C.c_int]
        L.orc_dot.argtypes = [_f32p, _f32p, C.c_size_t]
        L.orc_dot.restype = C.c_float
        for n in ("orc_q6k_dequant", "orc_q80_dequant"):
            getattr(L, n).argtypes = [_u8p, C.c_size_t, _f32p]
        for n in ("orc_q6k_gemv", "orc_q80_gemv"):
            getattr(L, n).argtypes = [_u8p, C.c_size_t, C.c_size_t, _f32p, _f32p, C.c_int]
        L.orc_rms_norm.argtypes = [_f32p, _f32p, C.c_float, C.c_size_t, _f32p]
        L.orc_gelu.argtypes = [C.c_float]
        L.orc_gelu.restype = C.c_float
        L.orc_sigmoid.argtypes = [C.c_float]
        L.orc_sigmoid.restype = C.c_float
        L.orc_argmax.argtypes = [_f32p, C.c_size_t]
        L.orc_argmax.restype = C.c_uint32
        L.orc_model_new.argtypes = [C.c_void_p, C.c_void_p, _f32p, _f32p, C.c_int, C.c_int]
        L.orc_model_new.restype = C.c_void_p
        L.orc_model_free.argtypes = [C.c_void_p]
        L.orc_model_forward.argtypes = [C.c_void_p, C.c_uint32, C.c_int, _f32p]
        L.orc_model_forward.restype = C.c_int
        L.orc_model_fill_kv.argtypes = [C.c_void_p, C.c_int, C.c_uint64]
        L.orc_model_kv.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        L.orc_model_kv.restype = C.c_int
        L.orc_model_capture.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.orc_model_capture.restype = C.c_int
        L.orc_draft_new.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int]
        L.orc_draft_new.restype = C.c_void_p
        L.orc_draft_free.argtypes = [C.c_void_p]
        L.orc_draft_encode.argtypes = [C.c_void_p, _f32p, C.c_size_t, C.c_int, C.c_int]
        L.orc_draft_encode.restype = C.c_int
        L.orc_draft_decode_block.argtypes = [C.c_void_p, _f32p, C.c_int, C.c_uint32, C.c_int, C.c_int, _f32p, _f32p,
                                             np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")]
        L.orc_draft_decode_block.restype = C.c_int
        L.orc_draft_block_rows.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.orc_draft_block_rows.restype = C.c_int
        _lib = L
    return _lib


def _u8(buf) -> np.ndarray:
    return np.frombuffer(buf, np.uint8) if not isinstance(buf, np.ndarray) else np.ascontiguousarray(buf, np.uint8)


def threads_default() -> int:
    return os.cpu_count() or 1


def container_info(buf) -> dict:
    b = _u8(buf)
    v = [C.c_int() for _ in range(6)]
    err = C.create_string_buffer(256)
    if lib().orc_container_info(b, b.size, *[C.byref(x) for x in v], err, 256):
        raise ValueError(err.value.decode())
    return dict(zip(("dim", "nc", "stages", "rows", "cols", "v3"), (x.value for x in v)))


def decode(buf) -> np.ndarray:
    """Container::decode (lib.rs:309-316): every stage summed into f32 rows x cols."""
    info = container_info(buf)
    b = _u8(buf)
    out = np.empty(info["rows"] * info["cols"], np.float32)
    err = C.create_string_buffer(256)
    if lib().orc_container_decode(b, b.size, out, err, 256):
        raise ValueError(err.value.decode())
    return out.reshape(info["rows"], info["cols"])


def gemv_fused(buf, x: np.ndarray, threads: int | None = None) -> np.ndarray:
    """dqvq gemv --fused: Stage::dot_row per stage per row (dqvq main.rs:131-143)."""
    info = container_info(buf)
    b = _u8(buf)
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(info["rows"], np.float32)
    err = C.create_string_buffer(256)
    if lib().orc_container_gemv_fused(b, b.size, x, y, threads or threads_default(), err, 256):
        raise ValueError(err.value.decode())
    return y


def matvec(W: np.ndarray, x: np.ndarray, threads: int | None = None) -> np.ndarray:
    """model.rs:229-234 over a decoded f32 matrix."""
    W = np.ascontiguousarray(W, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(W.shape[0], np.float32)
    lib().orc_matvec(W, W.shape[0], W.shape[1], x, y, threads or threads_default())
    return y


def q6k_dequant(blocks, rows: int, cols: int) -> np.ndarray:
    b = _u8(blocks)
    out = np.empty(rows * cols, np.float32)
    lib().orc_q6k_dequant(b, rows * cols // 256, out)
    return out.reshape(rows, cols)


def q80_dequant(blocks, rows: int, cols: int) -> np.ndarray:
    b = _u8(blocks)
    out = np.empty(rows * cols, np.float32)
    lib().orc_q80_dequant(b, rows * cols // 32, out)
    return out.reshape(rows, cols)


def q6k_gemv(blocks, rows: int, cols: int, x: np.ndarray, threads: int | None = None) -> np.ndarray:
    b = _u8(blocks)
    y = np.empty(rows, np.float32)
    lib().orc_q6k_gemv(b, rows, cols, np.ascontiguousarray(x, np.float32), y, threads or threads_default())
    return y


def q80_gemv(blocks, rows: int, cols: int, x: np.ndarray, threads: int | None = None) -> np.ndarray:
    b = _u8(blocks)
    y = np.empty(rows, np.float32)
    lib().orc_q80_gemv(b, rows, cols, np.ascontiguousarray(x, np.float32), y, threads or threads_default())
    return y


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().orc_rms_norm(x, np.ascontiguousarray(w, np.float32), eps, x.size, out)
    return out


def argmax(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, np.float32)
    return int(lib().orc_argmax(v, v.size))


def ref_decode_dump(container_path: str, out_path: str) -> np.ndarray:
    """Run the reference's own tools/vq/decode.c (built into _ref/decode) and read its f32 dump."""
    subprocess.run([REF_DECODE, "dump", container_path, out_path], check=True, capture_output=True)
    return np.fromfile(out_path, np.float32)


def ref_decode_matvec(container_path: str, vec_path: str) -> tuple[float, float]:
    """The reference decode.c `matvec` checksum line (sum, norm) over y = W x."""
    r = subprocess.run([REF_DECODE, "matvec", container_path, vec_path, "1"], check=True,
                       capture_output=True, text=True)
    for line in r.stdout.splitlines():
        if line.startswith("checksum"):
            parts = line.split()
            return float(parts[2].rstrip(",")), float(parts[4])
    raise RuntimeError("no checksum line in decode matvec output")


class _Cfg(C.Structure):
    _fields_ = [("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("inter", C.c_int), ("vocab", C.c_int), ("window", C.c_int),
                ("eps", C.c_float), ("rope_theta_full", C.c_float), ("rope_partial_full", C.c_float),
                ("rope_theta_slide", C.c_float), ("rope_partial_slide", C.c_float),
                ("full", C.POINTER(C.c_int))]


class _Layer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("in_norm", "post_norm", "qkv", "attn_gate", "out", "gate", "up", "down")]


class Model:
    """model.rs Model over decoded f32 weights. ``cfg`` is a dict with the config.rs fields;
    ``layers`` a list of dicts of f32 arrays (in_norm, post_norm, qkv, attn_gate, out, gate, up, down)."""

    def __init__(self, cfg: dict, layers: list[dict], embed: np.ndarray, norm: np.ndarray, max_ctx: int,
                 threads: int | None = None):
        self._keep = []
        full = (C.c_int * cfg["layers"])(*[int(f) for f in cfg["full"]])
        self._keep.append(full)
        c = _Cfg(cfg["hidden"], cfg["layers"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"], cfg["inter"],
                 cfg["vocab"], cfg["window"], cfg["eps"], cfg["rope_theta_full"], cfg["rope_partial_full"],
                 cfg["rope_theta_slide"], cfg["rope_partial_slide"], full)
        arr = (_Layer * cfg["layers"])()
        for i, L in enumerate(layers):
            for n, _ in _Layer._fields_:
                a = np.ascontiguousarray(L[n], np.float32)
                self._keep.append(a)
                setattr(arr[i], n, a.ctypes.data)
        self.embed = np.ascontiguousarray(embed, np.float32)
        self.norm = np.ascontiguousarray(norm, np.float32)
        self.vocab = cfg["vocab"]
        self.hidden, self.max_ctx = cfg["hidden"], max_ctx
        self.kv_dim = cfg["kv_heads"] * cfg["head_dim"]
        self._keep += [c, arr]
        self.h = lib().orc_model_new(C.byref(c), arr, self.embed, self.norm, max_ctx, threads or threads_default())
        if not self.h:
            raise MemoryError("oracle model allocation failed")

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.empty(self.vocab, np.float32)
        if lib().orc_model_forward(self.h, token, pos, out):
            raise ValueError(f"forward({token}, {pos}) rejected")
        return out

    def enable_capture(self, layers: list[int]) -> np.ndarray:
        """model.rs::enable_capture: the residual entering each listed layer is written, at
        every forward position, to the returned [len(layers)][max_ctx][hidden] array."""
        self.cap_layers = (C.c_int * len(layers))(*layers)
        self.cap = np.zeros((len(layers), self.max_ctx, self.hidden), np.float32)
        if lib().orc_model_capture(self.h, self.cap_layers, len(layers), self.cap.ctypes.data):
            raise ValueError(f"capture layers {layers} rejected")
        return self.cap

    def fill_kv(self, n: int, seed: int = 0):
        """Seeded K/V for the first n positions (CPU-baseline samples at long context)."""
        lib().orc_model_fill_kv(self.h, n, seed)

    def kv(self, layer: int) -> tuple[np.ndarray, np.ndarray]:
        """Views of layer's K and V caches, [max_ctx][kv_heads * head_dim] f32 (no copy)."""
        k, v = C.POINTER(C.c_float)(), C.POINTER(C.c_float)()
        if lib().orc_model_kv(self.h, layer, C.byref(k), C.byref(v)):
            raise ValueError(f"layer {layer} outside the model")
        n = self.max_ctx * self.kv_dim
        return (np.ctypeslib.as_array(k, (n,)).reshape(self.max_ctx, self.kv_dim),
                np.ctypeslib.as_array(v, (n,)).reshape(self.max_ctx, self.kv_dim))

    def close(self):
        if self.h:
            lib().orc_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


# ------------------------------------------------------------------ DSpark draft ---
class _DraftCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "layers", "heads", "kv_heads", "head_dim", "ffn", "vocab",
                                        "mask_token", "rope_full_dims", "rope_swa_dims")] + \
               [(n, C.c_float) for n in ("rope_full_theta", "rope_swa_theta", "eps")] + \
               [(n, C.c_int) for n in ("act", "swa_window", "causal", "block_size", "sample_from_anchor",
                                        "n_target")] + [("swa_pattern", C.c_void_p)]


_DRAFT_LAYER_F = ("norm", "q", "k", "v", "gate", "out", "q_norm", "k_norm", "ffn_norm", "ffn_gate", "ffn_up",
                  "ffn_down", "attn_post", "ffn_post")


class _DraftLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _DRAFT_LAYER_F] + [("out_scale", C.c_float)]


class _DraftGlobals(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("fc", "fc_norm", "enc_norm", "out_norm", "markov_w1", "markov_w2",
                                          "conf_proj")] + [("conf_bias", C.c_float), ("rank", C.c_int)]


class Draft:
    """draft.rs Draft over f32 weights (BF16 tensors expanded exactly). ``cfg`` holds the
    manifest header fields (oracle_draft.h); ``layers`` is a list of dicts keyed like
    DraftLayer (optional tensors absent or None); ``glob`` holds fc, fc_norm [n_target][hidden],
    enc_norm, out_norm and optionally markov_w1/markov_w2 [vocab][rank], conf_proj, conf_bias."""

    def __init__(self, cfg: dict, layers: list[dict], glob: dict, max_ctx: int, threads: int | None = None):
        self._keep = []
        self.cfg = dict(cfg)
        swa = (C.c_int * cfg["layers"])(*[int(v) for v in cfg["swa_pattern"]])
        c = _DraftCfg(*[int(cfg[n]) for n in ("hidden", "layers", "heads", "kv_heads", "head_dim", "ffn", "vocab",
                                              "mask_token", "rope_full_dims", "rope_swa_dims")],
                      *[float(cfg[n]) for n in ("rope_full_theta", "rope_swa_theta", "eps")],
                      *[int(cfg[n]) for n in ("act", "swa_window", "causal", "block_size", "sample_from_anchor",
                                              "n_target")], C.cast(swa, C.c_void_p))
        arr = (_DraftLayer * cfg["layers"])()
        for i, L in enumerate(layers):
            for n in _DRAFT_LAYER_F:
                setattr(arr[i], n, self._ptr(L.get(n)))
            arr[i].out_scale = float(L.get("out_scale", 0.0))
        g = _DraftGlobals(*[self._ptr(glob.get(n)) for n in ("fc", "fc_norm", "enc_norm", "out_norm", "markov_w1",
                                                              "markov_w2", "conf_proj")],
                          float(glob.get("conf_bias", 0.0)),
                          int(glob["markov_w1"].shape[1]) if glob.get("markov_w1") is not None else 0)
        self.has_markov = glob.get("markov_w1") is not None and glob.get("markov_w2") is not None
        self._keep += [swa, c, arr, g]
        self._c = c
        self.h = lib().orc_draft_new(C.byref(c), arr, C.byref(g), max_ctx, threads or threads_default())
        if not self.h:
            raise MemoryError("oracle draft allocation failed")

    def _ptr(self, a):
        if a is None:
            return None
        a = np.ascontiguousarray(a, np.float32)
        self._keep.append(a)
        return a.ctypes.data

    def block_rows(self, n_draft: int) -> int:
        return lib().orc_draft_block_rows(C.byref(self._c), int(self.has_markov), n_draft)

    def encode(self, caps: np.ndarray, p0: int, p1: int):
        """encode_features for positions [p0, p1) of caps [n_target][ctx][hidden]."""
        caps = np.ascontiguousarray(caps, np.float32)
        if lib().orc_draft_encode(self.h, caps.reshape(-1), caps.shape[1] * caps.shape[2], p0, p1):
            raise ValueError(f"encode [{p0}, {p1}) rejected")

    def decode_block(self, embed: np.ndarray, anchor: int, pos0: int, n_draft: int):
        """(logits [n_block][vocab], conf [n_block], argmax [n_block]) of decode_block."""
        vocab = embed.shape[0]
        nb = self.block_rows(n_draft)
        lg = np.zeros((max(nb, 1), vocab), np.float32)
        cf = np.zeros(max(nb, 1), np.float32)
        am = np.zeros(max(nb, 1), np.uint32)
        e = np.ascontiguousarray(embed, np.float32)
        rc = lib().orc_draft_decode_block(self.h, e.reshape(-1), vocab, anchor, pos0, n_draft, lg.reshape(-1), cf, am)
        if rc < 0:
            raise ValueError(f"decode_block(anchor {anchor}, pos0 {pos0}, n_draft {n_draft}) rejected")
        return lg[:rc], cf[:rc], am[:rc]

    def close(self):
        if self.h:
            lib().orc_draft_free(self.h)
            self.h = None

    def __del__(self):
        self.close()
