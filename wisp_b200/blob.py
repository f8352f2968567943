"""Expert blob format of the WISP engine (on disk, in the tier caches and in
VRAM): a 120-byte little-endian header, then per matrix (gate, up, down)
packed int4 | fp16 scales | fp16 zeros.

Layout (reference: wisp/converter/partitioner.py:10-24,
csrc/core/wisp_engine.h:214-251):

    0    u32 magic 0x57455850, u32 version 1, u32 layer, u32 expert,
         u32 group_size, u32 n_mats = 3
    24   3 x {u32 rows, u32 cols, u64 packed_bytes, u64 scales_bytes,
              u64 zeros_bytes}
    120  blobs

Because the header is 120 bytes, the packed data of a blob that starts on a
16-byte boundary sits 8 bytes off one; :func:`place_blob` puts a blob at an
address congruent to 8 mod 16 so every matrix inside it is 16-byte aligned.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

MAGIC = 0x57455850
VERSION = 1
HEADER = struct.Struct("<6I")
MAT_HEADER = struct.Struct("<2I3Q")
HEADER_BYTES = HEADER.size + 3 * MAT_HEADER.size
assert HEADER_BYTES == 120


@dataclass
class Int4Matrix:
    """One int4 matrix in the engine's packing (numpy arrays, host)."""
    packed: np.ndarray        # uint8 [rows * cols / 2], low nibble = even index
    scales: np.ndarray        # uint16 fp16 bits [rows * cols / gs]
    zeros: np.ndarray | None  # uint16 fp16 bits, or None (symmetric)
    rows: int
    cols: int


def pack_blob(gate: Int4Matrix, up: Int4Matrix, down: Int4Matrix, group_size: int,
              layer: int = 0, expert: int = 0, write_zeros: bool = True) -> bytes:
    """Serialise one expert. Symmetric matrices are written with all-zero
    zero points when ``write_zeros`` (the reference format always has them)."""
    mats = (gate, up, down)
    parts = [HEADER.pack(MAGIC, VERSION, layer, expert, group_size, 3)]
    body = []
    for m in mats:
        z = m.zeros
        if z is None and write_zeros:
            z = np.zeros_like(m.scales)
        zb = b"" if z is None else np.ascontiguousarray(z, dtype=np.uint16).tobytes()
        pb = np.ascontiguousarray(m.packed, dtype=np.uint8).tobytes()
        sb = np.ascontiguousarray(m.scales, dtype=np.uint16).tobytes()
        parts.append(MAT_HEADER.pack(m.rows, m.cols, len(pb), len(sb), len(zb)))
        body += [pb, sb, zb]
    return b"".join(parts + body)


@dataclass
class BlobMeta:
    packed_off: tuple
    scales_off: tuple
    zeros_off: tuple
    rows: tuple
    cols: tuple
    group_size: int
    total_bytes: int


def parse_blob(blob: bytes) -> BlobMeta:
    if len(blob) < HEADER_BYTES:
        raise ValueError(f"expert blob too small: {len(blob)} bytes")
    magic, ver, _l, _e, gs, nm = HEADER.unpack_from(blob)
    if magic != MAGIC or ver != VERSION or nm != 3:
        raise ValueError(f"expert blob corrupt: magic={magic:08x} version={ver} n_mats={nm}")
    off = HEADER_BYTES
    po, so, zo, rows, cols = [], [], [], [], []
    for i in range(3):
        r, c, pb, sb, zb = MAT_HEADER.unpack_from(blob, HEADER.size + i * MAT_HEADER.size)
        rows.append(r)
        cols.append(c)
        po.append(off)
        off += pb
        so.append(off)
        off += sb
        zo.append(off)
        off += zb
    if off > len(blob):
        raise ValueError(f"expert blob truncated: needs {off}, have {len(blob)}")
    return BlobMeta(tuple(po), tuple(so), tuple(zo), tuple(rows), tuple(cols), gs, off)


def place_blob(buf_base_addr: int, blob_len: int, align: int = 16) -> int:
    """Offset inside a buffer starting at ``buf_base_addr`` at which to put a
    blob so its payload (header + 120 bytes) is ``align``-byte aligned."""
    want = (-(buf_base_addr + HEADER_BYTES)) % align
    return want
