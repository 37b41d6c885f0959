"""Generate tests/golden/vqprof/: a small artifact directory and tuning profiles with what the
reference's own tools/vq/gpu/vq-profile.h computes for them (oracle/_ref/vqprof_ref, built from
the reference tree by `make -C oracle ref`).

The artifact covers every branch of the fingerprint: a container under 4096 bytes (its bytes
hashed twice), one of exactly 4096, one above, a comment line, a matrix line with stages 0 (not
hashed), a line with five fields (not a matrix line for the runtime's reader) and an empty
line. The profiles cover the reader: gemv and prefill entries with and without the trailing
rate, an unknown directive, CRLF line ends, trailing spaces, a device name longer than the
reader's buffer, a second entry for one geometry (the first one wins), a file that is not
version 1, more entries than the reader keeps and a line longer than its read buffer.

Usage: python tests/golden/make_vqprof.py
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "spark-x2.6-4b-q6k_b200"))

from spk import formats as F  # noqa: E402

OUT = os.path.join(HERE, "vqprof")
ART = os.path.join(OUT, "art")
REF = os.path.join(ROOT, "oracle", "_ref", "vqprof_ref")


def ref(*args) -> str:
    return subprocess.run([REF, *args], check=True, capture_output=True, text=True).stdout


def main() -> None:
    if not os.path.exists(REF):
        sys.exit(f"{REF} is missing: make -C oracle ref REF=<reference tree>")
    os.makedirs(ART, exist_ok=True)
    small = F.random_rvq(8, 64, 4, 256, 1, seed=1)        # ~2.2 KB: under one edge
    large = F.random_rvq(32, 256, 4, 256, 2, seed=2)      # ~8.5 KB: two distinct edges
    exact = bytes((7 * i + 3) & 0xFF for i in range(4096))   # exactly one edge
    files = {"blk.0.attn_qkv": small, "blk.0.ffn_up": large, "edge": exact}
    for name, buf in files.items():
        with open(os.path.join(ART, f"{name}.bin"), "wb") as f:
            f.write(buf)
    man = [
        "# encoding: dim=4 nc=256 stages=2 (gpu)",
        f"blk.0.attn_qkv 8 64 1 {len(small)} 0.012345",
        "# a comment between matrices",
        f"blk.0.ffn_up 32 256 2 {len(large)} 0.001000",
        "blk.0.norm 1 64 0 256 0.000000",
        f"edge 16 64 1 {len(exact)} 0.5",
        "five 1 2 3 4",
        "",
        "blk.1.gone 8 64 0 0 0",
    ]
    with open(os.path.join(ART, "manifest.txt"), "w") as f:
        f.write("\n".join(man) + "\n")
    rc, fp = ref("fp", ART).split()
    assert rc == "0", rc

    long_gpu = "NVIDIA B200 " + "x" * 140
    profiles = {
        "good.profile": "VQPROF 1\n"
                        f"artifact {fp}\n"
                        "gpu NVIDIA B200\n"
                        "driver 12090\n"
                        "gemv 4 4096 10240 2560 1 4 512 1346.2\n"
                        "gemv 4 4096 2560 4096 1 3 512\n"
                        "prefill 4 4096 6144 2560 1 2 128 64 5120.0\n"
                        "tune-note ignored by the reader\n"
                        "gemv 4 4096 10240 2560 1 3 256 900.0\n",
        "crlf.profile": "VQPROF 1\r\n"
                        f"artifact {fp}\r\n"
                        f"gpu {long_gpu}  \r\n"
                        "driver 12090 \r\n"
                        "gemv 4 256 8 64 1 1 128 10.0\r\n"
                        "prefill 4 256 32 256 1 1 64 64\r\n",
        "v2.profile": "VQPROF 2\n"
                      f"artifact {fp}\n"
                      "gpu NVIDIA B200\n"
                      "gemv 4 256 8 64 1 0 256 1.0\n",
        # more entries than the reader keeps (512), and a line longer than its 512-byte buffer
        # (the rest of that line is read as a line of its own)
        "many.profile": "VQPROF 1\n"
                        f"artifact {fp}\n"
                        "gpu NVIDIA B200\n"
                        "driver " + "d" * 80 + "\n"
                        + "".join(f"gemv 4 4096 {32 * (i + 1)} 2560 1 {i % 5} 512 {i}.5\n" for i in range(520)),
        "long.profile": "VQPROF 1\n"
                        f"artifact {fp}\n"
                        "gpu NVIDIA B200\n"
                        "gemv 4 4096 64 2560 1 3 512" + " " * 600 + "gemv 4 4096 96 2560 1 4 512 7.0\n"
                        "prefill 4 4096 64 2560 1 2 128 64\n",
    }
    expect = {"fingerprint": fp, "profiles": {}}
    for name, text in profiles.items():
        path = os.path.join(OUT, name)
        with open(path, "w", newline="") as f:
            f.write(text)
        lines = ref("load", path).splitlines()
        head = dict(line.split(" ", 1) if " " in line else (line, "") for line in lines if not line.startswith("entry"))
        entries = [[int(v) for v in line.split()[1:]] for line in lines if line.startswith("entry")]
        expect["profiles"][name] = {"rc": int(head["rc"]), "artifact": head["artifact"], "gpu": head["gpu"],
                                    "driver": head["driver"], "n": int(head["n"]), "entries": entries}
    with open(os.path.join(OUT, "expected.json"), "w") as f:
        json.dump(expect, f, indent=1)
    print(f"fingerprint {fp}; {len(profiles)} profiles")


if __name__ == "__main__":
    main()
