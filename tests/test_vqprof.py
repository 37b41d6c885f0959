"""VQPROF 1 tuning profiles (spk_vqprof_*), host code only: no GPU.

Pinned to the reference's own tools/vq/gpu/vq-profile.h: tests/golden/vqprof/expected.json
holds what its vqprof_artifact and vqprof_load return for the committed artifact directory
and profiles (tests/golden/make_vqprof.py, through oracle/_ref/vqprof_ref). Where that binary
exists (this container), the profiles this build writes are also read back by it.
"""
import ctypes
import json
import os
import shutil
import subprocess

import pytest

import spk
from spk import vqprof as P

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden", "vqprof")
ART = os.path.join(GOLD, "art")
REF = os.path.join(os.path.dirname(HERE), "oracle", "_ref", "vqprof_ref")
EXPECT = json.load(open(os.path.join(GOLD, "expected.json")))


def fnv_restatement(dir: str) -> int:
    """FNV-1a 64 over the artifact, restated from vq-profile.h:19-26 (the test's own copy),
    starting from the format's own value 1469598103934665603 (vq-profile.h:66)."""
    h = 1469598103934665603

    def eat(b: bytes):
        nonlocal h
        for x in b:
            h = ((h ^ x) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF

    man = open(os.path.join(dir, "manifest.txt"), "rb").read()
    eat(man)
    for line in man.split(b"\n"):
        if not line or line.startswith(b"#"):
            continue
        f = line.split()
        if len(f) < 6:
            continue
        if int(f[3]) <= 0:
            continue
        data = open(os.path.join(dir, f[0].decode() + ".bin"), "rb").read()
        eat(f[0])
        eat(len(data).to_bytes(8, "little"))
        eat(data[:4096])
        eat(data[-4096:] if len(data) > 4096 else data[:4096])
    return h


def entry_list(p: P.Profile) -> list:
    return [[e.kind, e.dim, e.nc, e.rows, e.cols, e.v3, e.variant, e.threads, e.bn, e.bk] for e in p.entries()]


def test_fingerprint_matches_the_reference():
    fp = int(EXPECT["fingerprint"], 16)
    assert P.fingerprint(ART) == fp
    assert fnv_restatement(ART) == fp


@pytest.mark.parametrize("name", sorted(EXPECT["profiles"]))
def test_load_matches_the_reference_reader(name):
    want = EXPECT["profiles"][name]
    p = P.Profile()
    rc = spk.lib().spk_vqprof_load(os.path.join(GOLD, name).encode(), ctypes.byref(p))
    assert rc == want["rc"]
    assert f"{p.artifact:016x}" == want["artifact"]
    assert p.gpu.decode() == want["gpu"]
    assert p.driver.decode() == want["driver"]
    assert p.n == want["n"]
    assert entry_list(p) == want["entries"]


def test_load_raises_on_other_versions_and_missing_files(tmp_path):
    with pytest.raises(spk.SpkError, match="version 2"):
        P.load(os.path.join(GOLD, "v2.profile"))
    with pytest.raises(spk.SpkError, match="cannot be opened"):
        P.load(str(tmp_path / "absent.profile"))


def test_find_takes_the_first_entry_of_a_geometry():
    p = P.load(os.path.join(GOLD, "good.profile"))
    e = P.find(p, 0, 4, 4096, 10240, 2560, 1)
    assert e is not None and e.variant == P.VARIANT_TABLE and e.threads == 512 and e.rate == pytest.approx(1346.2)
    assert P.find(p, 1, 4, 4096, 6144, 2560, 1).bn == 128
    assert P.find(p, 0, 4, 4096, 6144, 2560, 1) is None   # a prefill entry is not a gemv entry
    assert P.find(p, 0, 4, 4096, 10240, 2560, 0) is None  # DQVQ is another geometry


def test_trust_gate():
    fp = P.fingerprint(ART)
    p = P.load(os.path.join(GOLD, "good.profile"))
    assert P.trust(p, fp, "NVIDIA B200") == 0
    assert P.trust(p, fp ^ 1, "NVIDIA B200") == 1
    assert P.trust(p, fp, "NVIDIA B200 ") == 2           # names are matched literally
    assert P.trust(p, fp, "NVIDIA H100 80GB HBM3") == 2
    p.version = 2
    assert P.trust(p, fp, "NVIDIA B200") == 3


def test_fingerprint_follows_the_artifact(tmp_path):
    d = tmp_path / "art"
    shutil.copytree(ART, d)
    fp = P.fingerprint(str(d))
    assert fp == int(EXPECT["fingerprint"], 16)
    # a byte inside the first edge of a hashed container changes it
    with open(d / "blk.0.ffn_up.bin", "r+b") as f:
        f.seek(100)
        b = f.read(1)
        f.seek(100)
        f.write(bytes([b[0] ^ 0xFF]))
    assert P.fingerprint(str(d)) != fp
    # a manifest line that names a missing container is an error
    os.remove(d / "edge.bin")
    with pytest.raises(spk.SpkError, match="edge.bin"):
        P.fingerprint(str(d))
    with pytest.raises(spk.SpkError, match="manifest.txt"):
        P.fingerprint(str(tmp_path / "nowhere"))


def test_read_manifest_takes_six_field_lines():
    names = [m[0] for m in P.read_manifest(ART)]
    assert names == ["blk.0.attn_qkv", "blk.0.ffn_up", "blk.0.norm", "edge", "blk.1.gone"]


def test_write_round_trip(tmp_path):
    p = P.new(0x0123456789ABCDEF, "NVIDIA B200", "12090")
    p.add_gemv(4, 4096, 10240, 2560, 1, P.VARIANT_TABLE, 512, 1346.25)
    p.add_gemv(4, 4096, 2560, 10240, 1, 3, 512, 1020.0)
    p.add_prefill(4, 4096, 6144, 2560, 1, 2, 128, 64, 5120.0)
    path = str(tmp_path / "vq-tune.profile")
    P.write(path, p)
    assert not os.path.exists(path + ".tmp")
    text = open(path).read().splitlines()
    assert text[:4] == ["VQPROF 1", "artifact 0123456789abcdef", "gpu NVIDIA B200", "driver 12090"]
    assert text[4] == "gemv 4 4096 10240 2560 1 4 512 1346.2"   # the rate with one decimal, profile.rs's {:.1}
    q = P.load(path)
    assert q.artifact == p.artifact and q.n == 3 and entry_list(q) == entry_list(p)
    if os.path.exists(REF):   # the reference's reader reads what this build writes
        out = subprocess.run([REF, "load", path], check=True, capture_output=True, text=True).stdout.splitlines()
        assert out[0] == "rc 0" and out[1] == "artifact 0123456789abcdef" and out[4] == "n 3"
        assert [[int(v) for v in line.split()[1:]] for line in out if line.startswith("entry")] == entry_list(p)


def test_write_artifact_matches_manifest_format(tmp_path):
    from spk import formats as F

    bufs = {"a": F.random_rvq(8, 64, 4, 256, 1, seed=3), "b": F.random_rvq(16, 128, 4, 256, 2, seed=4)}
    P.write_artifact(str(tmp_path), bufs, 4, 256, 2)
    man = P.read_manifest(str(tmp_path))
    assert [(m[0], m[1], m[2], m[3], m[4]) for m in man] == [("a", 8, 64, 1, len(bufs["a"])),
                                                             ("b", 16, 128, 2, len(bufs["b"]))]
    assert P.fingerprint(str(tmp_path)) == fnv_restatement(str(tmp_path))
    if os.path.exists(REF):
        out = subprocess.run([REF, "fp", str(tmp_path)], check=True, capture_output=True, text=True).stdout.split()
        assert out == ["0", f"{P.fingerprint(str(tmp_path)):016x}"]


def test_tuner_bookkeeping_with_stubbed_measurements(tmp_path, monkeypatch):
    """spk.tune without a GPU: the measurement is stubbed, the rest is the tuner's own logic
    (one entry per geometry in manifest order, the fastest passing kernel, no entry when
    nothing passed, another artifact's profile kept unless forced)."""
    from spk import formats as F
    from spk import tune

    bufs = {"a": F.random_rvq(32, 256, 4, 256, 2, seed=5), "b": F.random_rvq(64, 128, 4, 256, 2, seed=6),
            "a2": F.random_rvq(32, 256, 4, 256, 2, seed=7), "c": F.random_rvq(16, 64, 4, 256, 1, seed=8)}
    d = str(tmp_path)
    P.write_artifact(d, bufs, 4, 256, 2)
    seen = []

    def fake(buf, iters, warmup, device):
        c = F.parse_container(buf)
        seen.append((c.rows, c.cols))
        if c.rows == 16:
            return []
        return [{"variant": P.VARIANT_TABLE if c.rows == 32 else 3, "threads": 512, "us": 5.0, "gbs": 12.5, "rel": 0.0}]

    monkeypatch.setattr(tune, "tune_geometry", fake)
    monkeypatch.setattr(P, "device_name", lambda: "NVIDIA B200")
    log = []
    path = tune.tune(d, log=log.append)
    assert seen == [(32, 256), (64, 128), (16, 64)]   # a2 shares a's geometry
    p = P.load(path)
    assert p.artifact == P.fingerprint(d) and p.gpu == b"NVIDIA B200" and p.n == 2
    assert [(e.rows, e.cols, e.variant) for e in p.entries()] == [(32, 256, P.VARIANT_TABLE), (64, 128, 3)]
    assert any("no kernel passed" in line for line in log)
    other = P.new(P.fingerprint(d) ^ 1, "NVIDIA B200", "0")
    P.write(path, other)
    with pytest.raises(spk.SpkError, match="belongs to artifact"):
        tune.tune(d, log=log.append)
    tune.tune(d, force=True, log=log.append)
    assert P.load(path).artifact == P.fingerprint(d)
