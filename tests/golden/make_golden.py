"""Generates tests/golden/attn_golden.npz: small fixed cases of the attention
hot path computed by an independent fp64 numpy restatement of
attention.metal:56-299 (dense masked matrices, no tiling, no online softmax).

The reference itself cannot run here (Apple Metal only) and ships no vectors,
so these fixtures pin the CPU oracle and the CUDA kernels to a second,
structurally different restatement of the same math:
    S = Q K^T / sqrt(D), key > query masked       (attention.metal:113-121)
    O = softmax(S) V, l = max + ln(sum)           (attention.metal:125-161)
    D = rowsum(dO * O)                            (attention.metal:166-195)
    P = exp(S - l); dS = P (dO V^T - D) / sqrt(D) (attention.metal:274-284)
    dQ = dS K, dK = dS^T Q, dV = P^T dO           (attention.metal:288-296)
The backward uses l as stored (fp32) and D as stored (bf16), as the
reference's backward reads them.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from metalllm_b200.inputs import bf16_bits_to_f32, f32_to_bf16_bits, normal_bf16  # noqa: E402

CASES = [
    # name, B, T, H, D, qkv_scale, seed
    ("t64_h2_d64", 2, 64, 2, 64, 1.0, 11),
    ("t128_h2_d128", 1, 128, 2, 128, 0.5, 12),
    ("t192_h1_d64", 1, 192, 1, 64, 1.0, 13),
]


def heads(x, B, T, H, D):
    return x.reshape(B, T, H, D).transpose(0, 2, 1, 3)


def unheads(x, B, T, H, D):
    return x.transpose(0, 2, 1, 3).reshape(B, T, H * D)


def reference_fp64(qb, kb, vb, dob, B, T, H, D):
    f = lambda b: heads(bf16_bits_to_f32(b).astype(np.float64), B, T, H, D)
    q, k, v, do = f(qb), f(kb), f(vb), f(dob)
    scale = 1.0 / np.sqrt(D)
    s = q @ k.transpose(0, 1, 3, 2) * scale
    future = np.triu(np.ones((T, T), dtype=bool), 1)
    s = np.where(future, -np.inf, s)
    m = s.max(-1, keepdims=True)
    e = np.exp(s - m)
    lsum = e.sum(-1, keepdims=True)
    o = (e @ v) / lsum
    lse = (m + np.log(lsum))[..., 0]                       # [B,H,T]
    lse32 = lse.astype(np.float32)
    o_bits = f32_to_bf16_bits(unheads(o, B, T, H, D).astype(np.float32))
    # D from the stored bf16 O, summed in fp64, stored bf16
    o_st = heads(bf16_bits_to_f32(o_bits).astype(np.float64), B, T, H, D)
    dvec = (do * o_st).sum(-1)                             # [B,H,T]
    d_bits = f32_to_bf16_bits(dvec.transpose(0, 2, 1).astype(np.float32))  # [B,T,H]
    d_st = bf16_bits_to_f32(d_bits).astype(np.float64).transpose(0, 2, 1)
    p = np.where(future, 0.0, np.exp(s - lse32.astype(np.float64)[..., None]))
    dp = do @ v.transpose(0, 1, 3, 2)
    ds = p * (dp - d_st[..., None]) * scale
    dq = ds @ k
    dk = ds.transpose(0, 1, 3, 2) @ q
    dv = p.transpose(0, 1, 3, 2) @ do
    U = lambda x: unheads(x, B, T, H, D)
    return {
        "o": o_bits,
        "lse": lse32.transpose(0, 2, 1).copy(),
        "d32": dvec.transpose(0, 2, 1).astype(np.float32), "d": d_bits,
        "dq": U(dq).astype(np.float32), "dk32": U(dk).astype(np.float32),
        "dv32": U(dv).astype(np.float32),
    }


def main():
    out = {}
    for name, B, T, H, D, sc, seed in CASES:
        n = B * T * H * D
        qb = normal_bf16(n, seed, 1, sc).reshape(B, T, H * D)
        kb = normal_bf16(n, seed, 2, sc).reshape(B, T, H * D)
        vb = normal_bf16(n, seed, 3, sc).reshape(B, T, H * D)
        dob = normal_bf16(n, seed, 4, 1.0).reshape(B, T, H * D)
        ref = reference_fp64(qb, kb, vb, dob, B, T, H, D)
        out[f"{name}/shape"] = np.array([B, T, H, D], np.int64)
        for key, val in (("q", qb), ("k", kb), ("v", vb), ("do", dob), *ref.items()):
            out[f"{name}/{key}"] = val
    path = Path(__file__).resolve().parent / "attn_golden.npz"
    np.savez_compressed(path, **out)
    print(path, path.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
