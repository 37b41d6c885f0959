"""Byte layouts of the weight formats on the decode path, and seeded writers for them.

The layouts are the reference's, byte for byte, because the kernels take the
reference's payloads unchanged:

* RQVQ container (tools/vq/gpu/build-vq-gpu.c:256-262, read by
  tools/vq-format/src/lib.rs:240-306): 32-byte header
  ``'RQVQ' u16 dim, u16 nc, u16 stages, u16 pad, u32 rows, u32 cols, u32 0,
  u64 payload_bytes`` then ``stages`` equal-sized stage payloads.
* DQV3 stage (``v3_pack``, build-vq-gpu.c:71-111): 24-byte header
  ``'DQV3' u16 dim, u16 nc, u32 rows, u32 cols, u32 flags, u32 pad``, f16
  codebook ``nc*dim``, f16 gain per row, then a row-local little-endian main
  stream of ``mb = min(nbit, 12)`` bits per index (``mrow`` bytes per row), then
  for ``nbit > 12`` a 1-bit plane of ``prow = ceil(nidx_row/8)`` bytes per row.
* DQVQ stage (``vq_pack``, tools/vq/vendor/vq_qc.h:241-264): 16-byte header, f16
  codebook, f16 gains, one global little-endian bitstream of ``nbit`` bits per
  index plus one trailing byte (one byte per index when ``nbit == 8``).
* ggml Q6_K block (210 B per 256 weights) and Q8_0 block (34 B per 32 weights),
  sizes as tools/kquant/stubs.c:23-52 prices them.

The seeded generators stand in for the reference's encoders (the real
checkpoint is not available): ``random_rvq`` draws codebooks and indices
directly; ``encode_rvq`` runs the reference's residual Lloyd recipe
(build-vq-gpu.c:224-253) and is meant for small matrices.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

RQVQ_HDR = 32
Q6K_BLOCK_BYTES, Q6K_BLOCK_WEIGHTS = 210, 256
Q80_BLOCK_BYTES, Q80_BLOCK_WEIGHTS = 34, 32


def index_bits(nc: int) -> int:
    """ceil(log2 nc), at least 1 (lib.rs:112-115)."""
    b = 1
    while (1 << b) < nc:
        b += 1
    return b


@dataclass(frozen=True)
class StageGeom:
    """Geometry of one stage payload, as the host parses it (decode-gpu.cu:40-56)."""

    dim: int
    nc: int
    rows: int
    cols: int
    v3: bool

    @property
    def nbit(self) -> int:
        return index_bits(self.nc)

    @property
    def nidx_row(self) -> int:
        return self.cols // self.dim

    @property
    def mb(self) -> int:
        return min(self.nbit, 12)

    @property
    def mrow(self) -> int:
        return (self.nidx_row * self.mb + 7) // 8 if self.v3 else 0

    @property
    def prow(self) -> int:
        return (self.nidx_row + 7) // 8 if (self.v3 and self.nbit > 12) else 0

    @property
    def header_bytes(self) -> int:
        return 24 if self.v3 else 16

    @property
    def index_bytes(self) -> int:
        if self.v3:
            return self.rows * (self.mrow + self.prow)
        nidx = self.rows * self.nidx_row
        return nidx if self.nbit == 8 else (nidx * self.nbit + 7) // 8 + 1

    @property
    def stage_bytes(self) -> int:
        return self.header_bytes + self.nc * self.dim * 2 + self.rows * 2 + self.index_bytes


def _pack_bits_rows(idx: np.ndarray, bits: int, row_bytes: int) -> np.ndarray:
    """Little-endian bit packing of each row of ``idx`` at ``bits`` bits per value."""
    rows, n = idx.shape
    idx = idx.astype(np.uint32)
    if bits == 12 and n % 2 == 0 and row_bytes == n * 12 // 8:
        a, b = idx[:, 0::2], idx[:, 1::2]
        w = a | (b << 12)
        out = np.empty((rows, n // 2, 3), np.uint8)
        out[..., 0] = w & 0xFF
        out[..., 1] = (w >> 8) & 0xFF
        out[..., 2] = (w >> 16) & 0xFF
        return out.reshape(rows, row_bytes)
    bitarr = ((idx[:, :, None] >> np.arange(bits, dtype=np.uint32)) & 1).astype(np.uint8)
    bitarr = bitarr.reshape(rows, n * bits)
    pad = row_bytes * 8 - n * bits
    if pad:
        bitarr = np.concatenate([bitarr, np.zeros((rows, pad), np.uint8)], axis=1)
    return np.packbits(bitarr, axis=1, bitorder="little")


def v3_pack(cb16: np.ndarray, gains16: np.ndarray, idx: np.ndarray, rows: int, cols: int,
            dim: int, nc: int) -> bytes:
    """One DQV3 stage payload (build-vq-gpu.c:71-111). ``cb16``/``gains16`` are f16 bit patterns."""
    g = StageGeom(dim, nc, rows, cols, True)
    if g.nbit > 13:
        raise ValueError(f"DQV3 carries 13 index bits, nc {nc} needs {g.nbit}")
    idx = np.asarray(idx).reshape(rows, g.nidx_row)
    hdr = b"DQV3" + struct.pack("<HHIIII", dim, nc, rows, cols, 1 if g.nbit > 12 else 0, 0)
    main = _pack_bits_rows(idx & ((1 << g.mb) - 1), g.mb, g.mrow)
    parts = [hdr, np.asarray(cb16, np.uint16).astype("<u2").tobytes(),
             np.asarray(gains16, np.uint16).astype("<u2").tobytes(), main.tobytes()]
    if g.prow:
        parts.append(_pack_bits_rows((idx >> 12) & 1, 1, g.prow).tobytes())
    out = b"".join(parts)
    assert len(out) == g.stage_bytes
    return out


def vq_pack(cb16: np.ndarray, gains16: np.ndarray, idx: np.ndarray, rows: int, cols: int,
            dim: int, nc: int) -> bytes:
    """One DQVQ (v2) stage payload (tools/vq/vendor/vq_qc.h:241-264)."""
    g = StageGeom(dim, nc, rows, cols, False)
    idx = np.asarray(idx).reshape(-1).astype(np.uint32)
    hdr = b"DQVQ" + struct.pack("<HHII", dim, nc, rows, cols)
    if g.nbit == 8:
        stream = idx.astype(np.uint8).tobytes()
    else:
        nb = (idx.size * g.nbit + 7) // 8 + 1
        packed = _pack_bits_rows(idx[None, :], g.nbit, nb)
        stream = packed.tobytes()
    out = b"".join([hdr, np.asarray(cb16, np.uint16).astype("<u2").tobytes(),
                    np.asarray(gains16, np.uint16).astype("<u2").tobytes(), stream])
    assert len(out) == g.stage_bytes
    return out


def rqvq(stages: list[bytes], dim: int, nc: int, rows: int, cols: int) -> bytes:
    """RQVQ container around equal-sized stage payloads (build-vq-gpu.c:256-262)."""
    per = len(stages[0])
    assert all(len(s) == per for s in stages)
    hdr = b"RQVQ" + struct.pack("<HHHHIIIQ", dim, nc, len(stages), 0, rows, cols, 0, per * len(stages))
    return hdr + b"".join(stages)


@dataclass(frozen=True)
class Container:
    """Parsed RQVQ header plus the byte range of every stage (lib.rs:240-306)."""

    dim: int
    nc: int
    nstages: int
    rows: int
    cols: int
    v3: bool
    stage_bytes: int

    def stage_offset(self, s: int) -> int:
        return RQVQ_HDR + s * self.stage_bytes

    @property
    def geom(self) -> StageGeom:
        return StageGeom(self.dim, self.nc, self.rows, self.cols, self.v3)


def parse_container(buf: bytes) -> Container:
    if len(buf) < RQVQ_HDR or buf[:4] != b"RQVQ":
        raise ValueError("not an RQVQ container")
    dim, nc, nst, _pad, rows, cols, _z, payload = struct.unpack_from("<HHHHIIIQ", buf, 4)
    if not (dim and nc and nst and rows and cols):
        raise ValueError("container header is inconsistent")
    v3 = len(buf) >= 36 and buf[32:36] == b"DQV3"
    g = StageGeom(dim, nc, rows, cols, v3)
    if v3 and g.nbit > 13:
        raise ValueError(f"DQV3 carries 13 index bits, nc {nc} needs {g.nbit}")
    if payload != nst * g.stage_bytes or len(buf) != RQVQ_HDR + payload:
        raise ValueError("payload byte count disagrees with the layout")
    return Container(dim, nc, nst, rows, cols, v3, g.stage_bytes)


def _f16_bits(a: np.ndarray) -> np.ndarray:
    return np.asarray(a, np.float32).astype(np.float16).view(np.uint16)


def random_rvq(rows: int, cols: int, dim: int = 4, nc: int = 4096, stages: int = 2, seed: int = 0,
               scale: float = 0.02, v3: bool = True, unit_gains: bool = True) -> bytes:
    """Seeded residual-VQ container: codebooks drawn N(0, s_k^2) with s_k shrinking per stage as a
    residual encoder's do, indices uniform. ``unit_gains`` matches the reference encoder's
    gains of 1.0 (build-vq-gpu.c:216-217); otherwise gains are drawn near 1."""
    rng = np.random.default_rng(seed)
    g = StageGeom(dim, nc, rows, cols, v3)
    payloads = []
    s_k = scale
    for _ in range(stages):
        cb = _f16_bits(rng.normal(0.0, s_k, size=nc * dim))
        gains = _f16_bits(np.ones(rows) if unit_gains else rng.uniform(0.5, 1.5, size=rows))
        idx = rng.integers(0, nc, size=(rows, g.nidx_row), dtype=np.int64)
        pack = v3_pack if v3 else vq_pack
        payloads.append(pack(cb, gains, idx, rows, cols, dim, nc))
        s_k *= 0.125
    return rqvq(payloads, dim, nc, rows, cols)


def random_rvq_fast(rows: int, cols: int, dim: int = 4, nc: int = 4096, stages: int = 2, seed: int = 0,
                    scale: float = 0.02) -> bytes:
    """random_rvq for a power-of-two codebook of 12 or 13 bits: every bit pattern of the row
    streams is a valid index there, so the streams are drawn as random bytes (fast enough for a
    whole 36-layer model). Codebooks N(0, s_k^2) per stage, gains 1.0."""
    g = StageGeom(dim, nc, rows, cols, True)
    if nc != (1 << g.nbit) or g.nbit not in (12, 13):
        raise ValueError("random_rvq_fast needs nc = 4096 or 8192")
    rng = np.random.default_rng(seed)
    hdr = b"DQV3" + struct.pack("<HHIIII", dim, nc, rows, cols, 1 if g.nbit > 12 else 0, 0)
    gains = _f16_bits(np.ones(rows)).astype("<u2").tobytes()
    payloads = []
    s_k = scale
    for _ in range(stages):
        cb = _f16_bits(rng.normal(0.0, s_k, size=nc * dim)).astype("<u2").tobytes()
        payloads.append(hdr + cb + gains + rng.bytes(g.index_bytes))
        s_k *= 0.125
    return rqvq(payloads, dim, nc, rows, cols)


def synth_q8_0(rows: int, cols: int, seed: int = 0, sigma: float = 0.02) -> bytes:
    """Q8_0 blocks with the statistics of quantize_q8_0(N(0, sigma^2)) without materialising the
    f32 matrix: q ~ round(N(0, (127/2.5)^2)) clipped to +-127, d ~ 2.5 sigma / 127 (the expected
    max |w| of 32 Gaussian draws over 127), jittered per block."""
    rng = np.random.default_rng(seed)
    nblk = rows * cols // Q80_BLOCK_WEIGHTS
    out = np.empty((nblk, Q80_BLOCK_BYTES), np.uint8)
    d = (2.5 * sigma / 127.0) * rng.uniform(0.8, 1.25, nblk)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    step = 1 << 22
    for i in range(0, nblk, step):
        n = min(step, nblk - i)
        q = np.clip(np.rint(rng.standard_normal((n, 32), dtype=np.float32) * (127.0 / 2.5)), -127, 127)
        out[i:i + n, 2:] = q.astype(np.int8).view(np.uint8)
    return out.tobytes()


def encode_rvq(W: np.ndarray, dim: int = 4, nc: int = 4096, stages: int = 2, iters: int = 8,
               v3: bool = True) -> bytes:
    """Residual Lloyd encoder following build-vq-gpu.c:224-253: per stage a strided subsample of
    at most 200k vectors, codebook initialised from every (nsub/nc)-th sample, ``iters`` Lloyd
    iterations, f16 round trip, nearest assignment of every vector, residual update."""
    W = np.asarray(W, np.float32)
    rows, cols = W.shape
    V = W.reshape(-1, dim).copy()
    nvec = V.shape[0]
    payloads = []
    for _ in range(stages):
        nsub = min(nvec, 200000)
        stride = nvec // nsub
        sub = V[np.arange(nsub) * stride]
        cst = max(1, nsub // nc)
        C = sub[np.minimum(np.arange(nc) * cst, nsub - 1)].copy()
        for _ in range(iters):
            a = _assign(sub, C)
            sums = np.zeros((nc, dim), np.float64)
            np.add.at(sums, a, sub.astype(np.float64))
            cnt = np.bincount(a, minlength=nc)
            nz = cnt > 0
            C[nz] = (sums[nz] / cnt[nz, None]).astype(np.float32)
        C = C.astype(np.float16).astype(np.float32)
        idx = _assign(V, C)
        V -= C[idx]
        pack = v3_pack if v3 else vq_pack
        payloads.append(pack(_f16_bits(C.reshape(-1)), _f16_bits(np.ones(rows)),
                             idx.reshape(rows, cols // dim), rows, cols, dim, nc))
    return rqvq(payloads, dim, nc, rows, cols)


def _assign(X: np.ndarray, C: np.ndarray, block: int = 16384) -> np.ndarray:
    c2 = (C.astype(np.float64) ** 2).sum(1)
    out = np.empty(X.shape[0], np.int64)
    for i in range(0, X.shape[0], block):
        x = X[i:i + block].astype(np.float64)
        d = c2[None, :] - 2.0 * (x @ C.T.astype(np.float64))
        out[i:i + block] = np.argmin(d, axis=1)
    return out


def _roundf(x: np.ndarray) -> np.ndarray:
    """C roundf: half away from zero."""
    return np.sign(x) * np.floor(np.abs(x) + 0.5)


def quantize_q8_0(W: np.ndarray) -> bytes:
    """ggml's reference Q8_0 rule: d = max|w|/127, q = roundf(w/d), d stored f16."""
    W = np.asarray(W, np.float32)
    rows, cols = W.shape
    assert cols % Q80_BLOCK_WEIGHTS == 0
    blk = W.reshape(-1, Q80_BLOCK_WEIGHTS)
    d = np.abs(blk).max(axis=1, keepdims=True) / np.float32(127)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    q = _roundf(blk * inv).astype(np.int8)
    out = np.empty((blk.shape[0], Q80_BLOCK_BYTES), np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


def quantize_q6_k(W: np.ndarray) -> bytes:
    """A valid Q6_K encoder (the graded contract is the decode, not this encoder): per 16-weight
    sub-block scale s = max|w|/31, super-block d = max s / 127 stored f16, int8 sub-scales
    round(s/d), q = clamp(round(w/(d*sc)), -32, 31) + 32 packed as ql (low 4) / qh (high 2)."""
    W = np.asarray(W, np.float32)
    rows, cols = W.shape
    assert cols % Q6K_BLOCK_WEIGHTS == 0
    blk = W.reshape(-1, 16, 16)                               # [nblk, sub-block, 16]
    nblk = blk.shape[0]
    s = np.abs(blk).max(axis=2) / np.float32(31)              # [nblk, 16]
    d = (s.max(axis=1) / np.float32(127)).astype(np.float16)  # [nblk]
    df = d.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(df[:, None] > 0, np.clip(_roundf(s / df[:, None]), -128, 127), 0).astype(np.int8)
        eff = (df[:, None] * sc.astype(np.float32))[:, :, None]
        q = np.where(eff > 0, np.clip(_roundf(blk / eff), -32, 31), 0).astype(np.int32) + 32
    q = q.reshape(nblk, 256).astype(np.uint8)                 # 0..63
    ql = np.zeros((nblk, 128), np.uint8)
    qh = np.zeros((nblk, 64), np.uint8)
    for h in range(2):
        qq = q[:, 128 * h:128 * (h + 1)].reshape(nblk, 4, 32)  # quadrant j, lane l
        lo = qq & 0x0F
        hi = (qq >> 4) & 0x03
        ql[:, 64 * h:64 * h + 32] = lo[:, 0] | (lo[:, 2] << 4)
        ql[:, 64 * h + 32:64 * h + 64] = lo[:, 1] | (lo[:, 3] << 4)
        qh[:, 32 * h:32 * h + 32] = hi[:, 0] | (hi[:, 1] << 2) | (hi[:, 2] << 4) | (hi[:, 3] << 6)
    out = np.empty((nblk, Q6K_BLOCK_BYTES), np.uint8)
    out[:, 0:128] = ql
    out[:, 128:192] = qh
    out[:, 192:208] = sc.view(np.uint8)
    out[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    return out.tobytes()


def q6k_row_bytes(cols: int) -> int:
    return cols // Q6K_BLOCK_WEIGHTS * Q6K_BLOCK_BYTES


def q80_row_bytes(cols: int) -> int:
    return cols // Q80_BLOCK_WEIGHTS * Q80_BLOCK_BYTES


# ------------------------------------------------- tensor-parallel re-cuts ---
# A DQV3 stream is row-local, so a shard of rows or of whole index columns is an
# exact re-cut of the payload: the same codebook, the same indices, the same gains.
# The decoded shard is bit-identical to the corresponding block of the decoded matrix.

def _unpack_bits_rows(raw: np.ndarray, bits: int, n: int) -> np.ndarray:
    """Inverse of _pack_bits_rows: ``raw`` [rows][row_bytes] -> uint32 [rows][n]."""
    rows = raw.shape[0]
    if bits == 12 and n % 2 == 0 and raw.shape[1] == n * 12 // 8:
        t = raw.reshape(rows, n // 2, 3).astype(np.uint32)
        w = t[..., 0] | (t[..., 1] << 8) | (t[..., 2] << 16)
        out = np.empty((rows, n), np.uint32)
        out[:, 0::2] = w & 0xFFF
        out[:, 1::2] = w >> 12
        return out
    bitarr = np.unpackbits(raw, axis=1, bitorder="little")[:, :n * bits].reshape(rows, n, bits).astype(np.uint32)
    return (bitarr << np.arange(bits, dtype=np.uint32)).sum(axis=2, dtype=np.uint32)


def v3_unpack(stage: bytes):
    """One DQV3 stage payload -> (geom, codebook f16 bits, gains f16 bits, indices [rows][nidx_row])."""
    if stage[:4] != b"DQV3":
        raise ValueError("not a DQV3 stage")
    dim, nc, rows, cols, _flags, _pad = struct.unpack_from("<HHIIII", stage, 4)
    g = StageGeom(dim, nc, rows, cols, True)
    a = np.frombuffer(stage, np.uint8)
    o = g.header_bytes
    cb = a[o:o + nc * dim * 2].view("<u2").copy()
    o += nc * dim * 2
    gains = a[o:o + rows * 2].view("<u2").copy()
    o += rows * 2
    idx = _unpack_bits_rows(a[o:o + rows * g.mrow].reshape(rows, g.mrow), g.mb, g.nidx_row)
    o += rows * g.mrow
    if g.prow:
        plane = _unpack_bits_rows(a[o:o + rows * g.prow].reshape(rows, g.prow), 1, g.nidx_row)
        idx |= plane << 12
    return g, cb, gains, idx


def _stages(buf: bytes):
    c = parse_container(buf)
    if not c.v3:
        raise ValueError("tensor-parallel re-cuts take DQV3 containers")
    return c, [buf[c.stage_offset(s):c.stage_offset(s) + c.stage_bytes] for s in range(c.nstages)]


def shard_rows(buf: bytes, rows) -> bytes:
    """The RQVQ container of the listed rows (in order) of a DQV3 container."""
    c, stages = _stages(buf)
    rows = np.asarray(rows, np.int64)
    out = []
    for st in stages:
        g, cb, gains, idx = v3_unpack(st)
        out.append(v3_pack(cb, gains[rows], idx[rows], len(rows), c.cols, c.dim, c.nc))
    return rqvq(out, c.dim, c.nc, len(rows), c.cols)


def shard_cols(buf: bytes, c0: int, c1: int) -> bytes:
    """The RQVQ container of input columns [c0, c1) of a DQV3 container (whole indices:
    c0 and c1 multiples of dim). The per-row gains are kept, so the shards' partial
    products sum to the full product."""
    c, stages = _stages(buf)
    if c0 % c.dim or c1 % c.dim or not 0 <= c0 < c1 <= c.cols:
        raise ValueError(f"columns [{c0}, {c1}) do not cut whole {c.dim}-wide indices of {c.cols}")
    out = []
    for st in stages:
        g, cb, gains, idx = v3_unpack(st)
        out.append(v3_pack(cb, gains, idx[:, c0 // c.dim:c1 // c.dim], c.rows, c1 - c0, c.dim, c.nc))
    return rqvq(out, c.dim, c.nc, c.rows, c1 - c0)


def shard_q80_rows(buf: bytes, cols: int, r0: int, r1: int) -> bytes:
    """Rows [r0, r1) of a row-major Q8_0 matrix (a contiguous byte range)."""
    rb = q80_row_bytes(cols)
    return buf[r0 * rb:r1 * rb]
