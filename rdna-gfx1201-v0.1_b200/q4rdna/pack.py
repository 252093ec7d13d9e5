"""Sidecar packer command line, a drop-in for the reference's
``q4rdna_sidecar_pack MANIFEST OUTPUT`` (source/q4rdna_sidecar_pack.cpp:216-295)
with the quantisation on the GPU (q4rdna_pack_bf16).

The manifest has one tensor per line, tab-separated, as the reference reads it
(q4rdna_sidecar_pack.cpp:182-203): ``path  byte_offset  rows  columns  name``.
The weights are raw little-endian bf16 at ``byte_offset`` of ``path`` (a
safetensors data region, for example).  The output is the same file, byte for
byte, that the reference packer writes.

    python -m q4rdna.pack MANIFEST OUTPUT
"""
from __future__ import annotations

import os
import sys
import time
from dataclasses import dataclass

import numpy as np

from . import format as fmt


@dataclass
class ManifestEntry:
    path: str
    offset: int
    rows: int
    cols: int
    name: str


def read_manifest(path: str) -> list[ManifestEntry]:
    """Parses the manifest with the reference's rules: empty lines skipped,
    rows % 32 == 0, columns % 64 == 0, names shorter than 64 bytes."""
    out = []
    with open(path, encoding="utf-8") as f:
        for line in f.read().split("\n"):
            if not line:
                continue
            parts = line.split("\t", 4)
            if len(parts) != 5 or not parts[0]:
                raise ValueError("invalid manifest line")
            try:
                offset, rows, cols = int(parts[1]), int(parts[2]), int(parts[3])
            except ValueError:
                raise ValueError("invalid manifest line") from None
            if offset < 0 or rows <= 0 or cols <= 0:
                raise ValueError("invalid manifest line")
            name = parts[4]
            if rows % fmt.TILE_ROWS or cols % fmt.GROUP or len(name.encode()) >= 64:
                raise ValueError("unsupported tensor in manifest")
            out.append(ManifestEntry(parts[0], offset, rows, cols, name))
    return out


def read_bf16(e: ManifestEntry) -> np.ndarray:
    """The tensor's raw bf16 bit patterns [rows, cols] (uint16)."""
    count = e.rows * e.cols
    a = np.fromfile(e.path, dtype="<u2", count=count, offset=e.offset)
    if a.size != count:
        raise ValueError(f"failed to read {e.name}")
    return a.reshape(e.rows, e.cols)


def pack_manifest(manifest: str, output: str, device: int = 0, log=sys.stdout) -> int:
    """Packs every manifest tensor on the GPU and writes the sidecar; returns
    the file size."""
    import torch

    from . import pack_bf16

    entries = read_manifest(manifest)
    dev = torch.device("cuda", device)
    packed = []
    t0 = time.time()
    for i, e in enumerate(entries):
        t1 = time.time()
        w = torch.from_numpy(read_bf16(e).view(np.int16)).to(dev)
        tiles = pack_bf16(w).cpu().numpy()
        packed.append((e.name, tiles, e.rows, e.cols))
        if log is not None:
            print(f"[{i + 1:3d}/{len(entries)}] {e.name:<31s} {e.rows:5d}x{e.cols:5d} "
                  f"{time.time() - t1:.1f}s total {time.time() - t0:.1f}s", file=log, flush=True)
    fmt.write_sidecar(output, packed)
    size = os.path.getsize(output)
    if log is not None:
        print(f"wrote {output} ({size} bytes)", file=log, flush=True)
    return size


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) != 2:
        print("usage: python -m q4rdna.pack MANIFEST OUTPUT", file=sys.stderr)
        return 2
    try:
        pack_manifest(argv[0], argv[1])
    except (OSError, ValueError, RuntimeError) as err:
        print(f"error: {err}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
