"""Seeded synthetic Q4_RDNA tensors with the benchmark's value distributions.

Codes c are uniform in [0, 15] with value (c - 8) * scale, so the stored
two's-complement nibble is c ^ 8 and every code byte is a uniform byte; scales
are fp16(|N(0,1)| * 0.003) (round to nearest even, numpy's float16 cast);
activations are N(0,1) f32.  These stand in for Qwen3 weights, which are not
available offline.
"""
from __future__ import annotations

import numpy as np

from .format import GROUP, TILE_BYTES, TILE_ROWS

BASE_SEED = 20260816

# Qwen3-8B decoder linear tensors per layer as (ggml suffix, rows N, columns K);
# names follow source/pack_q4rdna_sidecar.py:25-33.
QWEN3_8B_LAYER = [
    ("attn_q.weight", 4096, 4096),
    ("attn_k.weight", 1024, 4096),
    ("attn_v.weight", 1024, 4096),
    ("attn_output.weight", 4096, 4096),
    ("ffn_gate.weight", 12288, 4096),
    ("ffn_up.weight", 12288, 4096),
    ("ffn_down.weight", 4096, 12288),
]
QWEN3_8B_LAYERS = 36

# Qwen3-32B: hidden 5120, 64 q heads / 8 kv heads x 128, intermediate 25600.
QWEN3_32B_LAYER = [
    ("attn_q.weight", 8192, 5120),
    ("attn_k.weight", 1024, 5120),
    ("attn_v.weight", 1024, 5120),
    ("attn_output.weight", 5120, 8192),
    ("ffn_gate.weight", 25600, 5120),
    ("ffn_up.weight", 25600, 5120),
    ("ffn_down.weight", 5120, 25600),
]
QWEN3_32B_LAYERS = 64


def model_tensors(model: str = "qwen3-8b") -> list[tuple[str, int, int]]:
    layer, n = (QWEN3_8B_LAYER, QWEN3_8B_LAYERS) if model == "qwen3-8b" else (QWEN3_32B_LAYER, QWEN3_32B_LAYERS)
    return [(f"blk.{L}.{suffix}", r, c) for L in range(n) for suffix, r, c in layer]


def tiles_np(N: int, K: int, seed: int) -> np.ndarray:
    """Packed tiles (uint8, N*K*34/64 bytes) drawn from PCG64(seed)."""
    if N % TILE_ROWS or K % GROUP:
        raise ValueError("N % 32 and K % 64 must be 0")
    rng = np.random.default_rng(seed)
    T = (N // TILE_ROWS) * (K // GROUP)
    t = np.empty((T, TILE_BYTES), np.uint8)
    t[:, 64:] = rng.integers(0, 256, (T, TILE_BYTES - 64), dtype=np.uint8)
    scales = (np.abs(rng.standard_normal((T, TILE_ROWS))) * 0.003).astype(np.float16)
    t[:, :64] = scales.view(np.uint8)
    return t.reshape(-1)


def x_np(K: int, B: int, seed: int) -> np.ndarray:
    """Activations f32 [B, K] ~ N(0, 1) from PCG64(seed)."""
    return np.random.default_rng(seed).standard_normal((B, K), dtype=np.float32)


def tiles_torch(N: int, K: int, seed: int, device):
    """Same distributions, drawn on the device with torch's generator (fast, for
    multi-GB benchmark streams; not bit-identical to tiles_np)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    T = (N // TILE_ROWS) * (K // GROUP)
    t = torch.empty((T, TILE_BYTES), dtype=torch.uint8, device=device)
    t[:, 64:] = torch.randint(0, 256, (T, TILE_BYTES - 64), generator=g, device=device, dtype=torch.uint8)
    sc = (torch.randn((T, TILE_ROWS), generator=g, device=device).abs_() * 0.003).to(torch.float16)
    t[:, :64] = sc.view(torch.uint8)
    return t.reshape(-1)


# ---- Q4_K (ggml block_q4_K) rows: the format of the Q/K/V tensors that the
# reference's qkv-fallback scope leaves on llama.cpp's stock path ----
Q4K_BLOCK = 256
Q4K_BLOCK_BYTES = 144


def q4k_bytes(N: int, K: int) -> int:
    if K % Q4K_BLOCK:
        raise ValueError("K % 256 must be 0")
    return N * (K // Q4K_BLOCK) * Q4K_BLOCK_BYTES


def q4k_np(N: int, K: int, seed: int) -> np.ndarray:
    """Q4_K rows (uint8, N*K/256*144 bytes) from PCG64(seed): uniform quant
    and 6-bit scale/min bytes; d and dmin = fp16((0.5 + |N(0,1)|) * 2e-4), so
    that a weight step d * scale spans the Q4_RDNA scales' range (fp16
    normal; subnormal d and dmin are edge cases of their own)."""
    nb = N * (K // Q4K_BLOCK) if K % Q4K_BLOCK == 0 else None
    if nb is None:
        raise ValueError("K % 256 must be 0")
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, (nb, Q4K_BLOCK_BYTES), dtype=np.uint8)
    dd = ((0.5 + np.abs(rng.standard_normal((nb, 2)))) * 2e-4).astype(np.float16)
    b[:, :4] = dd.view(np.uint8)
    return b.reshape(-1)


def q4k_torch(N: int, K: int, seed: int, device):
    """Same distributions drawn on the device (not bit-identical to q4k_np)."""
    import torch

    nb = N * (K // Q4K_BLOCK)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    b = torch.randint(0, 256, (nb, Q4K_BLOCK_BYTES), generator=g, device=device, dtype=torch.uint8)
    dd = ((torch.randn((nb, 2), generator=g, device=device).abs_() + 0.5) * 2e-4).to(torch.float16)
    b[:, :4] = dd.view(torch.uint8)
    return b.reshape(-1)
