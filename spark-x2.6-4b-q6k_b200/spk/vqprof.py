"""VQPROF 1 tuning profiles and artifact directories, over libspk's native reader and writer.

Mirrors tools/vq/gpu/vq-profile.h (``Profile`` is ``vqprof``, ``Entry`` is ``vqprof_entry``;
``fingerprint`` is ``vqprof_artifact``, ``load`` is ``vqprof_load``, ``find`` is
``vqprof_find``) and the writer of tools/vq-tune/src/profile.rs (``write``). ``trust``
applies the reference runtime's gate (vq-model-gpu.cu:1094-1122): version 1, the same
artifact fingerprint, the same device name. An artifact directory holds ``manifest.txt``
(``# encoding: dim=D nc=N stages=S`` then ``name rows cols stages file_bytes relL2`` per
matrix) and one RQVQ container ``name.bin`` per matrix (tools/vq-tune/src/artifact.rs:57-140).
"""
from __future__ import annotations

import ctypes as C
import os

from . import check, lib

VERSION = 1
MAX_ENTRIES = 512
VARIANT_TABLE = 4   # SPK_VARIANT_TABLE: the shared-memory table kernel (vq_tab.cu)
TRUST_REASONS = {0: "trusted", 1: "tuned on another artifact", 2: "tuned on another device", 3: "not version 1"}


class Entry(C.Structure):
    _fields_ = [("kind", C.c_int), ("dim", C.c_int), ("nc", C.c_int), ("rows", C.c_int), ("cols", C.c_int),
                ("v3", C.c_int), ("variant", C.c_int), ("threads", C.c_int), ("bn", C.c_int), ("bk", C.c_int),
                ("rate", C.c_double)]


class Profile(C.Structure):
    _fields_ = [("artifact", C.c_ulonglong), ("gpu", C.c_char * 128), ("driver", C.c_char * 64),
                ("version", C.c_int), ("n", C.c_int), ("e", Entry * MAX_ENTRIES)]

    def entries(self) -> list[Entry]:
        return [self.e[i] for i in range(min(self.n, MAX_ENTRIES))]

    def add_gemv(self, dim, nc, rows, cols, v3, variant, threads=256, rate=0.0) -> None:
        self._add(0, dim, nc, rows, cols, v3, variant, threads, 0, 0, rate)

    def add_prefill(self, dim, nc, rows, cols, v3, variant, bn, bk, rate=0.0) -> None:
        self._add(1, dim, nc, rows, cols, v3, variant, 0, bn, bk, rate)

    def _add(self, kind, dim, nc, rows, cols, v3, variant, threads, bn, bk, rate) -> None:
        if self.n >= MAX_ENTRIES:
            raise ValueError(f"a profile holds at most {MAX_ENTRIES} entries")
        self.e[self.n] = Entry(kind, dim, nc, rows, cols, int(bool(v3)), variant, threads, bn, bk, rate)
        self.n += 1


def new(artifact: int, gpu: str, driver: str) -> Profile:
    p = Profile()
    p.artifact = artifact
    p.gpu = gpu.encode()[:127]
    p.driver = driver.encode()[:63]
    p.version = VERSION
    return p


def fingerprint(dir: str) -> int:
    out = C.c_ulonglong(0)
    check(lib().spk_vqprof_fingerprint(dir.encode(), C.byref(out)))
    return out.value


def load(path: str) -> Profile:
    """The parsed profile; raises (spk.SpkError) when it is absent or not version 1."""
    p = Profile()
    check(lib().spk_vqprof_load(path.encode(), C.byref(p)))
    return p


def find(p: Profile, kind: int, dim: int, nc: int, rows: int, cols: int, v3: int) -> Entry | None:
    i = lib().spk_vqprof_find(C.byref(p), kind, dim, nc, rows, cols, int(bool(v3)))
    return p.e[i] if i >= 0 else None


def trust(p: Profile, artifact: int, device: str) -> int:
    """0 trusted; 1 another artifact; 2 another device; 3 not version 1 (TRUST_REASONS)."""
    return lib().spk_vqprof_trust(C.byref(p), artifact, device.encode())


def write(path: str, p: Profile) -> None:
    check(lib().spk_vqprof_write(path.encode(), C.byref(p)))


def device_name() -> str:
    """The current device's name (vqg_device_name), the string a profile is bound to."""
    buf = C.create_string_buffer(256)
    check(lib().vqg_device_name(buf, 256))
    return buf.value.decode()


def write_artifact(dir: str, mats: dict, dim: int, nc: int, stages: int) -> None:
    """An artifact directory from RQVQ containers {name: bytes}: the containers as name.bin and
    the manifest (the relL2 column is informational here and written as 0)."""
    from . import formats as F
    os.makedirs(dir, exist_ok=True)
    lines = [f"# encoding: dim={dim} nc={nc} stages={stages} (gpu)"]
    for name, buf in mats.items():
        c = F.parse_container(buf)
        with open(os.path.join(dir, f"{name}.bin"), "wb") as f:
            f.write(buf)
        lines.append(f"{name} {c.rows} {c.cols} {c.nstages} {len(buf)} 0.000000")
    with open(os.path.join(dir, "manifest.txt"), "w") as f:
        f.write("\n".join(lines) + "\n")


def read_manifest(dir: str) -> list[tuple[str, int, int, int, int]]:
    """(name, rows, cols, stages, file_bytes) for every matrix line with all six fields."""
    out = []
    with open(os.path.join(dir, "manifest.txt"), "rb") as f:
        for raw in f.read().split(b"\n"):
            line = raw.decode(errors="replace")
            if not line or line.startswith("#"):
                continue
            fs = line.split()
            if len(fs) < 6:
                continue
            try:
                out.append((fs[0], int(fs[1]), int(fs[2]), int(fs[3]), int(fs[4])))
                float(fs[5])
            except ValueError:
                continue
    return out


def read_container(dir: str, name: str) -> bytes:
    with open(os.path.join(dir, f"{name}.bin"), "rb") as f:
        return f.read()
