"""spk — Python face of libspk, the B200 decode hot path.

This module is what tools/vq-bench/src/cuda.rs is for the reference: a thin
binding of the C-ABI (include/spk.h) plus the device-buffer discipline the
kernels rely on (every stage buffer carries zeroed slack after its payload,
cuda.rs:139-160). The compute runs in libspk.so; this layer only marshals
pointers. If libspk.so is missing or a CUDA device is absent, calls fail
loudly — there is no CPU fallback.

Device memory comes from torch (allocation and streams only): a ``torch.Tensor``
on a CUDA device is passed to the library as its raw data pointer.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libspk.so")
SLACK = 64   # >= the 8 zeroed bytes the reference contract asks for

_lib = None


class SpkError(RuntimeError):
    pass


_vp, _i, _f, _d, _cp = C.c_void_p, C.c_int, C.c_float, C.c_double, C.c_char_p
_dp = C.POINTER(C.c_double)

_PROTOS = {
    "vqg_decode_error": ([], _cp),
    "spk_last_error": ([], _cp),
    "spk_check_device_error": ([], _i),
    "vqg_device_name": ([_cp, _i], _i),
    "vqg_driver_version": ([], _i),
    "vqg_gemv_ready": ([_i] * 6, _i),
    "vqg_gemv_t": ([_vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _i, _i, _dp], _i),
    "vqg_gemv": ([_vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _i, _dp], _i),
    "vqg_gemv_launch_t": ([_vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _i], _i),
    "vqg_gemv_launch": ([_vp, _i, _i, _i, _i, _i, _vp, _vp, _i], _i),
    "vqg_dequant": ([_vp, _i, _i, _i, _i, _i, _vp, _i, _dp], _i),
    "vqg_row_dequant": ([_vp, _i, _i, _i, _i, _i, _i, _vp], _i),
    "vqg_gemv_f32": ([_vp, _vp, _vp, _i, _i, _i, _dp], _i),
    "vqg_prefill_ready": ([_i] * 6, _i),
    "vqg_prefill_cfg_count": ([], _i),
    "vqg_prefill_cfg": ([_i, C.POINTER(_i), C.POINTER(_i)], _i),
    "vqg_prefill_cfg_ready": ([_i] * 8, _i),
    "vqg_prefill": ([_vp, _i, _i, _i, _i, _i, _vp, _i, _vp, _i, _dp, _i], _i),
    "vqg_prefill_tile": ([_vp, _i, _i, _i, _i, _i, _vp, _i, _vp, _i, _dp, _i, _i, _i], _i),
    "vqg_prefill_launch": ([_vp, _i, _i, _i, _i, _i, _vp, _i, _vp, _i], _i),
    "vqg_prefill_launch_tile": ([_vp, _i, _i, _i, _i, _i, _vp, _i, _vp, _i, _i, _i], _i),
    "spk_vq_gemv": ([_vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _f, _vp, _i, _vp], _i),
    "spk_vq_lut_bytes": ([_i, _i, _i, _i, _i], C.c_size_t),
    "spk_vq_lut_pack": ([_vp, _i, _i, _i, _i, _i, _vp, _vp], _i),
    "spk_vq_lut_scratch_bytes": ([_i, _i, _i, _i, _i, _i], C.c_size_t),
    "spk_vq_lut_gemv": ([_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _f, _vp, _i, _vp, _vp], _i),
    "spk_vq_lut_gemv_t": ([_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _f, _vp, _i, _vp, _i, _vp], _i),
    "spk_vq_tab_bytes": ([_i, _i, _i, _i, _i], C.c_size_t),
    "spk_vq_tab_pack": ([_vp, _i, _i, _i, _i, _i, _vp, _vp], _i),
    "spk_vq_tab_scratch_bytes": ([_i, _i, _i, _i, _i, _i], C.c_size_t),
    "spk_vq_tab_gemv": ([_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _f, _vp, _i, _vp, _vp], _i),
    "spk_vq_lut_gemm_scratch_bytes": ([_i, _i, _i], C.c_size_t),
    "spk_vq_lut_gemm": ([_vp, _i, _i, _i, _i, _i, _i, _i, _vp, _i, _vp, _f, _vp, _i, _i, _vp, _vp], _i),
    "spk_vq_gemv_fast_ok": ([_i] * 7, _i),
    "spk_vq_dequant": ([_vp, _i, _i, _i, _i, _i, _vp, _vp], _i),
    "spk_q6k_gemv": ([_vp, _i, _i, _vp, _vp, _f, _vp, _i, _vp], _i),
    "spk_q80_gemv": ([_vp, _i, _i, _vp, _vp, _f, _vp, _i, _vp], _i),
    "spk_q80_head": ([_vp, _i, _i, _vp, _vp, _f, _vp, _vp, _vp], _i),
    "spk_q80_head_noalloc": ([_vp, _i, _i, _vp, _vp, _f, _vp, _vp, _vp], _i),
    "spk_q6k_dequant": ([_vp, C.c_size_t, _vp, _vp], _i),
    "spk_q80_dequant": ([_vp, C.c_size_t, _vp, _vp], _i),
    "spk_q80_row": ([_vp, _i, _i, _i, _vp, _vp, _vp], _i),
    "spk_verify_gemm": ([_vp, _i, _i, _i, _i, _i, _i, _i, _vp, _i, _vp, _f, _vp, _i, _i, _vp], _i),
    "spk_attn_workspace_bytes": ([_i, _i, _i, _i, _i], C.c_size_t),
    "spk_attn_decode": ([_vp, _vp], _i),
    "spk_attn_store": ([_vp, _vp], _i),
    "spk_q80_head_batch": ([_vp, _i, _i, _i, _vp, _i, _vp, _f, _vp, _i, _vp, _vp], _i),
    "spk_model_create": ([_vp, _vp], _vp),
    "spk_model_destroy": ([_vp], None),
    "spk_model_set_layer": ([_vp, _i] + [_vp] * 8, _i),
    "spk_model_set_head": ([_vp, _vp, _vp], _i),
    "spk_model_forward": ([_vp, _i, _i, _vp, _vp], _i),
    "spk_model_begin": ([_vp, _i, _i, _vp, _i], _i),
    "spk_model_run": ([_vp, _i], _i),
    "spk_model_logits": ([_vp], _vp),
    "spk_model_rollback": ([_vp, _i], _i),
    "spk_model_reset": ([_vp], _i),
    "spk_model_len": ([_vp], _i),
    "spk_model_advance_len": ([_vp, _i], _i),
    "spk_model_write_kv": ([_vp, _i, _i, _i, _vp, _vp], _i),
    "spk_model_verify": ([_vp, _vp, _i, _i, _vp, _vp], _i),
    "spk_model_prefill": ([_vp, _vp, _i, _i, _vp, _vp], _i),
    "spk_model_trace": ([_vp, _vp, _i], _i),
    "spk_model_tp_handle": ([_vp, _vp, _i], _i),
    "spk_model_tp_attach": ([_vp, _vp, _i, _i], _i),
    "spk_model_tp_attach_ptrs": ([_vp, _vp, _i, _i], _i),
    "spk_model_tp_mailbox": ([_vp], _vp),
    "spk_model_enable_capture": ([_vp, _vp, _i], _i),
    "spk_model_captures": ([_vp, C.POINTER(C.c_size_t)], _vp),
    "spk_draft_create": ([_vp, _vp], _vp),
    "spk_draft_destroy": ([_vp], None),
    "spk_draft_set_layer": ([_vp, _i, _vp], _i),
    "spk_draft_set_globals": ([_vp, _vp], _i),
    "spk_draft_encode": ([_vp, _vp, C.c_size_t, _i, _i], _i),
    "spk_draft_block": ([_vp, _vp, _i, _i, _i, _i, _vp, _vp], _i),
    "spk_draft_logits": ([_vp], _vp),
    "spk_draft_set_head_tiled": ([_vp, _vp], _i),
    "spk_model_head_tiled": ([_vp], _vp),
    "spk_model_step_launches": ([_vp], _i),
    "spk_bf16_gemm": ([_vp, _i, _i, _i, _vp, _i, _vp, _i, _i, _vp], _i),
    "spk_q80_tile_bytes": ([_i, _i], C.c_size_t),
    "spk_q80_tile": ([_vp, _i, _i, _vp, _vp], _i),
    "spk_q80_tile_scratch_bytes": ([], C.c_size_t),
    "spk_q80_tile_head": ([_vp, _i, _i, _i, _vp, _i, _vp, _f, _vp, _i, _vp, _vp, _vp], _i),
    "spk_bf16_gemm_pair": ([_vp, _vp, _i, _i, _i, _vp, _i, _vp, _i, _i, _vp], _i),
    "spk_vqprof_fingerprint": ([_cp, C.POINTER(C.c_ulonglong)], _i),
    "spk_vqprof_load": ([_cp, _vp], _i),
    "spk_vqprof_find": ([_vp, _i, _i, _i, _i, _i, _i], _i),
    "spk_vqprof_trust": ([_vp, C.c_ulonglong, _cp], _i),
    "spk_vqprof_write": ([_cp, _vp], _i),
    "spk_model_use_profile": ([_vp, _vp], _i),
    "spk_model_kernel_of": ([_vp, _i, _i], _i),
}


def exported_symbols() -> list[str]:
    """Every entry point the header declares (the loader checks each one)."""
    return list(_PROTOS)


def lib():
    """Load libspk.so and bind every prototype. Raises if the library is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise SpkError(f"{LIB_PATH} is not built: run `python spark-x2.6-4b-q6k_b200/build.py`")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in _PROTOS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def last_error() -> str:
    p = lib().spk_last_error()
    return p.decode() if p else "unknown error"


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        raise SpkError(f"{what}: {last_error()}" if what else last_error())


def ptr(t) -> int | None:
    """Raw device pointer of a torch tensor (None stays NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise SpkError("libspk takes device buffers; got a host tensor")
    return t.data_ptr()


def stream_ptr(stream=None) -> int | None:
    if stream is None:
        return None
    return stream.cuda_stream


def dev_bytes(buf: bytes, device="cuda", slack: int = SLACK):
    """Upload bytes to a fresh device buffer with `slack` zeroed bytes after them
    (the DevBuf contract of tools/vq-bench/src/cuda.rs:139-160)."""
    import numpy as np
    import torch

    a = np.frombuffer(buf, np.uint8) if not isinstance(buf, np.ndarray) else buf.view(np.uint8).reshape(-1)
    t = torch.zeros(a.size + slack, dtype=torch.uint8, device=device)
    t[: a.size].copy_(torch.from_numpy(a.copy()))
    return t


from . import formats  # noqa: E402,F401
