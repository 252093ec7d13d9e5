"""Q4_RDNA packed format and sidecar container, in numpy.

Byte layouts are the reference's, unchanged:
  * tile (source/q4rdna.cu:20-24, writer source/q4rdna_sidecar_pack.cpp:268-278):
    32 rows x 64 columns in 1088 bytes; bytes [0, 64) hold the 32 fp16 scales
    (row r at byte 2r, little endian); byte 64 + 32*i + r holds row r, columns
    2i (low nibble) and 2i+1 (high nibble), two's-complement int4;
    tile index = row_tile * groups + group.
  * sidecar (source/q4rdna.cu:26-50, writers source/pack_q4rdna_sidecar.py:16-23,
    128-146 and source/q4rdna_sidecar_pack.cpp:223-245): 48-byte header, 96-byte
    entries with absolute offsets, data at a 4096-aligned offset, every tensor
    256-aligned, zero padding in between.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

GROUP = 64
TILE_ROWS = 32
TILE_BYTES = 1088
MAGIC = b"Q4RDNA1\x00"
VERSION = 1
HEADER = struct.Struct("<8sIIIIIIQQ")
ENTRY = struct.Struct("<64sIIQQQ")
DATA_ALIGNMENT = 4096
TENSOR_ALIGNMENT = 256


def tensor_bytes(rows: int, cols: int) -> int:
    """Packed bytes of a rows x cols tensor: rows*cols*34/64 (source/q4rdna.cu:149)."""
    return rows * cols * 34 // GROUP


def align_up(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def pack_tiles(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Signed codes int [N, K] in [-8, 7] and fp16 scales [N, K/64] -> tile bytes."""
    codes = np.asarray(codes)
    N, K = codes.shape
    if N % TILE_ROWS or K % GROUP:
        raise ValueError(f"unsupported Q4_RDNA shape {codes.shape}")
    G = K // GROUP
    sc = np.ascontiguousarray(scales, dtype=np.float16).reshape(N // TILE_ROWS, TILE_ROWS, G)
    nib = (codes.astype(np.int16) & 15).astype(np.uint8).reshape(N // TILE_ROWS, TILE_ROWS, G, GROUP // 2, 2)
    byte = nib[..., 0] | (nib[..., 1] << 4)              # [RT, 32 rows, G, 32 pairs]
    tiles = np.empty((N // TILE_ROWS, G, TILE_BYTES), np.uint8)
    tiles[..., :64] = sc.transpose(0, 2, 1).copy().view(np.uint8).reshape(N // TILE_ROWS, G, 64)
    tiles[..., 64:] = byte.transpose(0, 2, 3, 1).reshape(N // TILE_ROWS, G, 1024)
    return tiles.reshape(-1)


def unpack_tiles(tiles: np.ndarray, N: int, K: int) -> tuple[np.ndarray, np.ndarray]:
    """Inverse of pack_tiles: (codes int8 [N, K], scales fp16 [N, K/64])."""
    G = K // GROUP
    t = np.asarray(tiles, np.uint8).reshape(N // TILE_ROWS, G, TILE_BYTES)
    scales = t[..., :64].copy().view(np.float16).reshape(N // TILE_ROWS, G, TILE_ROWS).transpose(0, 2, 1)
    b = t[..., 64:].reshape(N // TILE_ROWS, G, GROUP // 2, TILE_ROWS).transpose(0, 3, 1, 2)  # RT, r, G, i
    lo = (b & 15).astype(np.int8)
    hi = (b >> 4).astype(np.int8)
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    codes = np.stack([lo, hi], axis=-1).reshape(N, K).astype(np.int8)
    return codes, scales.reshape(N, G)


@dataclass
class SidecarEntry:
    name: str
    rows: int
    cols: int
    offset: int  # absolute file offset
    size: int


def layout(specs: list[tuple[str, int, int]]) -> tuple[int, list[SidecarEntry], int]:
    """Offsets the reference writers assign: (data_offset, entries, end)."""
    data_offset = align_up(HEADER.size + ENTRY.size * len(specs), DATA_ALIGNMENT)
    off = data_offset
    out = []
    for name, rows, cols in specs:
        size = tensor_bytes(rows, cols)
        out.append(SidecarEntry(name, rows, cols, off, size))
        off = align_up(off + size, TENSOR_ALIGNMENT)
    return data_offset, out, off


def write_sidecar(path: str, tensors: list[tuple[str, np.ndarray, int, int]]) -> list[SidecarEntry]:
    """Write (name, tile bytes, rows, cols) tensors as a sidecar file."""
    data_offset, entries, end = layout([(n, r, c) for n, _, r, c in tensors])
    with open(path, "wb") as f:
        f.write(HEADER.pack(MAGIC, VERSION, len(entries), GROUP, TILE_ROWS, TILE_BYTES, 0,
                            data_offset, end - data_offset))
        for e in entries:
            enc = e.name.encode("ascii")
            if len(enc) >= 64:
                raise ValueError(f"tensor name too long: {e.name}")
            f.write(ENTRY.pack(enc, e.rows, e.cols, e.offset, e.size, 0))
        f.write(bytes(data_offset - f.tell()))
        for e, (_, tiles, _, _) in zip(entries, tensors):
            if f.tell() != e.offset:
                f.write(bytes(e.offset - f.tell()))
            buf = np.ascontiguousarray(tiles, np.uint8).reshape(-1)
            if buf.size != e.size:
                raise ValueError(f"{e.name}: {buf.size} bytes, expected {e.size}")
            f.write(buf.tobytes())
        if f.tell() < end:
            f.write(bytes(end - f.tell()))
    return entries


def read_sidecar(path: str) -> tuple[dict, list[SidecarEntry]]:
    """Parse header and entries (no validation; the C loader validates)."""
    with open(path, "rb") as f:
        h = HEADER.unpack(f.read(HEADER.size))
        hdr = dict(magic=h[0], version=h[1], count=h[2], group=h[3], tile_rows=h[4], tile_bytes=h[5],
                   reserved=h[6], data_offset=h[7], data_bytes=h[8])
        es = []
        for _ in range(hdr["count"]):
            n, r, c, o, s, _ = ENTRY.unpack(f.read(ENTRY.size))
            es.append(SidecarEntry(n.split(b"\x00", 1)[0].decode("ascii"), r, c, o, s))
    return hdr, es
