"""Deterministic synthetic inputs for the attention configs.

Element i of a tensor drawn with (seed, stream) is
    z_i = sqrt(-2 ln u1) * cos(2 pi u2) * scale,  cast to bf16 (round to nearest even)
with u1 = (h(2i) >> 11 + 0.5) / 2^53, u2 = (h(2i+1) >> 11) / 2^53 and
h(n) = splitmix64(base + n), base = splitmix64(seed * 2^32 + stream).
Each element depends only on (seed, stream, i), so any (batch, head) shard of
a tensor can be regenerated independently and the CPU checker and the GPU see
identical bf16 arrays.  Box-Muller and splitmix64 are the published methods
(Box & Muller 1958; Steele, Lea & Flood 2014).
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)

# stream ids of the attention tensors
STREAM_Q, STREAM_K, STREAM_V, STREAM_DO, STREAM_X, STREAM_W = 1, 2, 3, 4, 5, 6


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x + _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    return (r >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def normal_bf16(n: int, seed: int, stream: int, scale: float = 1.0, offset: int = 0,
                chunk: int = 1 << 20, threads: int = 0) -> np.ndarray:
    """n bf16 bit patterns of N(0, scale^2) for elements offset .. offset+n-1.

    Chunks are generated on `threads` host threads (0: one per core; numpy
    releases the GIL inside its element-wise loops); every element depends
    only on its index, so the result does not depend on the thread count."""
    base = _splitmix64(np.array([(seed << 32) + stream], dtype=np.uint64))[0]
    out = np.empty(n, dtype=np.uint16)
    inv53 = 1.0 / float(1 << 53)

    def fill(s: int) -> None:
        e = min(n, s + chunk)
        idx = np.arange(offset + s, offset + e, dtype=np.uint64) * np.uint64(2)
        with np.errstate(over="ignore"):
            h1 = _splitmix64(idx + base)
            h2 = _splitmix64(idx + base + np.uint64(1))
        u1 = ((h1 >> np.uint64(11)).astype(np.float64) + 0.5) * inv53
        u2 = (h2 >> np.uint64(11)).astype(np.float64) * inv53
        z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2) * scale
        out[s:e] = f32_to_bf16_bits(z.astype(np.float32))

    starts = range(0, n, chunk)
    nthreads = threads or (os.cpu_count() or 1)
    if nthreads <= 1 or len(starts) <= 1:
        for s in starts:
            fill(s)
    else:
        with ThreadPoolExecutor(max_workers=min(nthreads, len(starts))) as ex:
            list(ex.map(fill, starts))
    return out


def attention_inputs(B: int, T: int, H: int, D: int, seed: int = 0, qkv_scale: float = 1.0,
                     do_scale: float = 1.0) -> dict[str, np.ndarray]:
    """Q, K, V, dO as bf16 bit arrays of shape [B, T, H*D] (the reference layout)."""
    n = B * T * H * D
    shape = (B, T, H * D)
    return {
        "q": normal_bf16(n, seed, STREAM_Q, qkv_scale).reshape(shape),
        "k": normal_bf16(n, seed, STREAM_K, qkv_scale).reshape(shape),
        "v": normal_bf16(n, seed, STREAM_V, qkv_scale).reshape(shape),
        "do": normal_bf16(n, seed, STREAM_DO, do_scale).reshape(shape),
    }


# The BASELINE configs (attention shape, input scales).
CONFIGS = {
    "c1": dict(B=16, T=256, H=6, D=64, qkv_scale=1.0, do_scale=1.0),
    "c2": dict(B=64, T=1024, H=12, D=64, qkv_scale=1.0, do_scale=1.0),
    "c3": dict(B=8, T=4096, H=16, D=128, qkv_scale=0.5, do_scale=1.0),
    "c4": dict(B=4, T=8192, H=32, D=64, qkv_scale=1.0, do_scale=1.0),
}


def causal_flops(B: int, T: int, H: int, D: int) -> tuple[float, float]:
    """Algorithmic causal FLOPs (fwd, bwd): 2*B*H*T^2*D and 5*B*H*T^2*D
    (T^2/2 causal pairs; 4 resp. 10 flops per pair per head dim)."""
    fwd = 2.0 * B * H * T * T * D
    return fwd, 2.5 * fwd
