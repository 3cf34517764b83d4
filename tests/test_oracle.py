"""CPU tests of the oracle (the checker) against the golden fixtures, the
reference's documented known answer and closed-form cases, plus an fp64
finite-difference check of its backward."""
from pathlib import Path

import numpy as np
import pytest

from metalllm_b200.inputs import bf16_bits_to_f32, f32_to_bf16_bits, normal_bf16

GOLDEN = Path(__file__).resolve().parent / "golden" / "attn_golden.npz"


def golden_cases():
    z = np.load(GOLDEN)
    names = sorted({k.split("/")[0] for k in z.files})
    return [(n, {k.split("/")[1]: z[k] for k in z.files if k.startswith(n + "/")}) for n in names]


def rand_bf16(shape, seed, stream, scale=1.0):
    n = int(np.prod(shape))
    return normal_bf16(n, seed, stream, scale).reshape(shape)


@pytest.mark.parametrize("name,case", golden_cases(), ids=[n for n, _ in golden_cases()])
def test_oracle_matches_golden(oracle_mod, name, case):
    o = oracle_mod
    B, T, H, D = (int(x) for x in case["shape"])
    out, lse, o32 = o.flash_forward(case["q"], case["k"], case["v"], H, want_f32=True)
    # exact-interface fp32 oracle vs the fp64 restatement
    assert np.abs(lse - case["lse"]).max() < 1e-4
    assert np.abs(bf16_bits_to_f32(out) - bf16_bits_to_f32(case["o"])).max() <= 2 ** -7
    Dv, d32 = o.compute_d(case["do"], case["o"], H, want_f32=True)
    assert np.abs(d32 - case["d32"]).max() < 1e-4
    # backward from the golden (stored) lse / D, as the reference reads them
    dQ, dK, dV, dk32, dv32 = o.flash_backward(case["do"], case["d"], case["lse"], case["q"],
                                              case["k"], case["v"], H, want_f32=True)
    for got, want in ((dQ, case["dq"]), (dk32, case["dk32"]), (dv32, case["dv32"])):
        scale = max(1.0, float(np.abs(want).max()))
        assert np.abs(got - want).max() < 1e-4 * scale
    # fp64 mode agrees even more tightly
    dQ64, _, _, dk64, dv64 = o.flash_backward(case["do"], case["d"], case["lse"], case["q"],
                                              case["k"], case["v"], H, mode=o.FP64, want_f32=True)
    assert np.abs(dQ64 - case["dq"]).max() < 1e-5 * max(1.0, float(np.abs(case["dq"]).max()))


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("T,D", [(64, 64), (192, 128)])
def test_row0_equals_v_row0(oracle_mod, mode, T, D):
    """README.md:132: row 0 of a causal head must equal V row 0 (bit-exact)."""
    B, H = 2, 3
    q = rand_bf16((B, T, H * D), 1, 1)
    k = rand_bf16((B, T, H * D), 1, 2)
    v = rand_bf16((B, T, H * D), 1, 3)
    out, lse = oracle_mod.flash_forward(q, k, v, H, mode=mode)
    assert np.array_equal(out[:, 0, :], v[:, 0, :])


def test_zero_query_gives_prefix_mean(oracle_mod):
    """Q = 0: every score is 0, so l[i] = ln(i+1) and O[i] = mean(V[0..i])."""
    B, T, H, D = 1, 128, 2, 64
    q = np.zeros((B, T, H * D), np.uint16)
    k = rand_bf16((B, T, H * D), 2, 2)
    v = rand_bf16((B, T, H * D), 2, 3)
    out, lse, o32 = oracle_mod.flash_forward(q, k, v, H, mode=2, want_f32=True)
    i = np.arange(T)
    assert np.allclose(lse[0], np.log(i + 1.0)[:, None], atol=1e-6)
    vf = bf16_bits_to_f32(v).astype(np.float64)
    prefix = np.cumsum(vf, axis=1) / (i + 1.0)[None, :, None]
    assert np.abs(o32 - prefix).max() < 1e-5


def test_constant_keys_give_prefix_mean(oracle_mod):
    """All keys equal: scores are equal along each row, O = prefix mean of V."""
    B, T, H, D = 1, 64, 1, 64
    q = rand_bf16((B, T, H * D), 3, 1)
    krow = rand_bf16((1, 1, H * D), 3, 2)
    k = np.broadcast_to(krow, (B, T, H * D)).copy()
    v = rand_bf16((B, T, H * D), 3, 3)
    out, lse, o32 = oracle_mod.flash_forward(q, k, v, H, mode=2, want_f32=True)
    vf = bf16_bits_to_f32(v).astype(np.float64)
    prefix = np.cumsum(vf, axis=1) / np.arange(1, T + 1)[None, :, None]
    assert np.abs(o32 - prefix).max() < 1e-5


def test_compute_d_matches_fp64(oracle_mod):
    B, T, H, D = 2, 64, 3, 128
    do = rand_bf16((B, T, H * D), 4, 4)
    o = rand_bf16((B, T, H * D), 4, 3, 0.3)
    Dv, d32 = oracle_mod.compute_d(do, o, H, want_f32=True)
    ref = (bf16_bits_to_f32(do).astype(np.float64) * bf16_bits_to_f32(o)).reshape(B, T, H, D).sum(-1)
    assert np.abs(d32 - ref).max() < 1e-4
    assert np.array_equal(Dv, f32_to_bf16_bits(d32))


def test_backward_finite_difference_fp64(oracle_mod):
    """The oracle backward (fp64 mode) matches central differences of the
    fp64 loss L = sum(dO * attention(Q, K, V)) on a tiny head."""
    o = oracle_mod
    T, D = 16, 64
    rng = np.random.default_rng(5)
    # bf16-representable inputs so the bf16 interface loses nothing
    mk = lambda s=1.0: f32_to_bf16_bits((rng.standard_normal((1, T, D)) * s).astype(np.float32))
    qb, kb, vb, dob = mk(), mk(), mk(), mk()
    out, lse, o32 = o.flash_forward(qb, kb, vb, 1, mode=2, want_f32=True)
    Dv, d32 = o.compute_d(dob, out, 1, mode=2, want_f32=True)
    # the backward reads D in bf16; compute it from the fp64 output instead for this check
    dd = (bf16_bits_to_f32(dob).astype(np.float64) * o32).sum(-1, keepdims=True)
    Dexact = f32_to_bf16_bits(dd.astype(np.float32)).reshape(1, T, 1)
    dQ, dK, dV, dk32, dv32 = o.flash_backward(dob, Dexact, lse, qb, kb, vb, 1, mode=2, want_f32=True)
    f = lambda b: bf16_bits_to_f32(b)[0].astype(np.float64)
    q, k, v, do = f(qb), f(kb), f(vb), f(dob)
    eps = 1e-4
    for which, grad in (("q", dQ[0]), ("k", dk32[0]), ("v", dv32[0])):
        num = np.zeros((T, D))
        for i in range(T):
            for c in range(0, D, 7):
                args = {"q": q.copy(), "k": k.copy(), "v": v.copy()}
                args[which][i, c] += eps
                lp = o.fp64_loss(args["q"], args["k"], args["v"], do)
                args[which][i, c] -= 2 * eps
                lm = o.fp64_loss(args["q"], args["k"], args["v"], do)
                num[i, c] = (lp - lm) / (2 * eps)
        sel = num != 0
        err = np.abs(num[sel] - grad[sel]).max()
        # D is stored in bf16 (2^-9 relative): allow that much slack on dQ/dK
        assert err < 2e-2 * max(1.0, np.abs(num[sel]).max()), (which, err)


def test_exact_and_faithful_modes_agree_loosely(oracle_mod):
    """The faithful mode (reference's bf16 intermediates) stays close to the
    exact-interface mode; informational bound, not the parity tolerance."""
    o = oracle_mod
    B, T, H, D = 1, 128, 2, 64
    q, k, v, do = (rand_bf16((B, T, H * D), 6, s) for s in (1, 2, 3, 4))
    oe, le = o.flash_forward(q, k, v, H, mode=0)
    of, lf = o.flash_forward(q, k, v, H, mode=1)
    ok, mae, rl2 = o.compare(bf16_bits_to_f32(of), bf16_bits_to_f32(oe), 0.1, 0.05)
    assert ok, (mae, rl2)
    assert np.abs(lf - le).max() < 0.05
    Dv = o.compute_d(do, oe, H)
    dqe, dke, dve = o.flash_backward(do, Dv, le, q, k, v, H, mode=0)
    dqf, dkf, dvf = o.flash_backward(do, Dv, le, q, k, v, H, mode=1)
    assert o.compare(dqf, dqe, 0.5, 0.1)[0]
    assert o.compare(bf16_bits_to_f32(dvf), bf16_bits_to_f32(dve), 0.5, 0.1)[0]


def test_thread_count_and_shards(oracle_mod):
    """Forward is bit-identical for any thread count; a shard range writes only
    its own (batch, head) slabs."""
    o = oracle_mod
    B, T, H, D = 2, 128, 3, 64
    q, k, v = (rand_bf16((B, T, H * D), 7, s) for s in (1, 2, 3))
    o1, l1 = o.flash_forward(q, k, v, H, nthreads=1)
    o8, l8 = o.flash_forward(q, k, v, H, nthreads=8)
    assert np.array_equal(o1, o8) and np.array_equal(l1, l8)
    sentinel = np.full_like(q, 0x7FC0)
    lsent = np.full((B, T, H), np.nan, np.float32)
    os_, ls_ = o.flash_forward(q, k, v, H, shard=(2, 5), out=sentinel, lse=lsent)
    for bh in range(B * H):
        b, h = divmod(bh, H)
        cols = slice(h * D, (h + 1) * D)
        if 2 <= bh < 5:
            assert np.array_equal(os_[b, :, cols], o1[b, :, cols])
            assert np.array_equal(ls_[b, :, h], l1[b, :, h])
        else:
            assert (os_[b, :, cols] == 0x7FC0).all()
            assert np.isnan(ls_[b, :, h]).all()


def test_compute_qkv_oracle(oracle_mod):
    B, M, N = 2, 64, 128
    X = rand_bf16((B, M, N), 8, 5)
    W = [rand_bf16((N, N), 8, 6 + i, 0.05) for i in range(3)]
    q, k, v, q32, k32, v32 = oracle_mod.compute_qkv(X, *W, want_f32=True)
    xf = bf16_bits_to_f32(X).astype(np.float64).reshape(B * M, N)
    for got, w in ((q32, W[0]), (k32, W[1]), (v32, W[2])):
        ref = xf @ bf16_bits_to_f32(w).astype(np.float64)
        assert np.abs(got.reshape(B * M, N) - ref).max() < 1e-4
    assert np.array_equal(q, f32_to_bf16_bits(q32))


def test_oracle_rejects_bad_shapes(oracle_mod):
    o = oracle_mod
    lib = o.load()
    q = np.zeros((1, 64, 64), np.uint16)
    lse = np.zeros((1, 64, 1), np.float32)
    # N != NH*D
    rc = lib.oracle_flash_forward(q.ctypes.data, q.ctypes.data, q.ctypes.data, q.ctypes.data,
                                  lse.ctypes.data, 64, 64, 32, 1, 1, 0, 1, 0, 1, None)
    assert rc != 0
    # shard range past the end
    rc = lib.oracle_flash_forward(q.ctypes.data, q.ctypes.data, q.ctypes.data, q.ctypes.data,
                                  lse.ctypes.data, 64, 64, 64, 1, 1, 0, 2, 0, 1, None)
    assert rc != 0


# ------------------------------------------------ GEMMs around attention
def test_oracle_gemms_match_numpy(oracle_mod):
    """The oracle's restatements of attention.metal:301-455 equal dense fp64
    numpy products of the same bf16/fp32 inputs to fp32 accuracy, and the
    row-sampled mode computes exactly the requested rows."""
    from metalllm_b200.inputs import bf16_bits_to_f32, normal_bf16
    o = oracle_mod
    B, M, N = 2, 50, 64
    R = B * M
    act = lambda s: normal_bf16(R * N, 7, s).reshape(B, M, N)
    w = lambda s: normal_bf16(N * N, 7, s, 0.02).reshape(N, N)
    f = bf16_bits_to_f32
    a, dz, x, dk, dv = act(1), act(2), act(3), act(4), act(5)
    wp, qw, kw, vw = w(6), w(7), w(8), w(9)
    dq = np.random.default_rng(0).standard_normal((B, M, N)).astype(np.float32)
    A64 = lambda t: f(t).reshape(R, N).astype(np.float64)
    tol = lambda got, want: np.abs(got - want).max() <= 1e-4 * max(1.0, np.abs(want).max())
    _, o32 = o.proj_forward(a, wp)
    assert tol(o32, A64(a) @ f(wp).astype(np.float64))
    _, d32 = o.proj_backward_dx(dz, wp)
    assert tol(d32, A64(dz) @ f(wp).astype(np.float64).T)
    _, w32 = o.proj_backward_dw(a, dz)
    assert tol(w32, A64(a).T @ A64(dz))
    dx = o.grad_dx(qw, kw, vw, dq, dk, dv)
    want = (dq.reshape(R, N).astype(np.float64) @ f(qw).astype(np.float64).T
            + A64(dk) @ f(kw).astype(np.float64).T + A64(dv) @ f(vw).astype(np.float64).T)
    assert tol(dx, want)
    dqw, _, _, k32, v32 = o.grad_dw(x, dq, dk, dv)
    assert tol(dqw, A64(x).T @ dq.reshape(R, N).astype(np.float64))
    assert tol(k32, A64(x).T @ A64(dk))
    assert tol(v32, A64(x).T @ A64(dv))
    rows = np.array([3, 17, 40])
    dx_s = o.grad_dx(qw, kw, vw, dq, dk, dv, rows=rows)
    assert np.array_equal(dx_s[rows], dx[rows])
    assert np.isnan(np.delete(dx_s, rows, axis=0)).all()


def test_train_oracle_gradients_match_finite_differences():
    """The training-step oracle's backward (oracle/train_oracle.py), with its
    bf16 rounding switched off and in float64, agrees with central finite
    differences of its own loss on a tiny model."""
    from oracle import train_oracle as O
    saved = O.r16, O.FLOAT
    O.r16 = lambda x: np.asarray(x, np.float64)
    O.FLOAT = np.float64
    try:
        B, T, E, NH, L, V, H = 2, 8, 16, 2, 1, 12, 32
        rng = np.random.default_rng(0)
        W = {"embed": rng.normal(0, 0.5, (V, E)), "pos": rng.normal(0, 0.5, (T, E)),
             "lnf_gamma": 1 + rng.normal(0, 0.1, E), "lnf_beta": rng.normal(0, 0.1, E),
             "linw": rng.normal(0, 0.3, (E, V))}
        for k, s in (("ln1_gamma", E), ("ln2_gamma", E)):
            W[f"layer0.{k}"] = 1 + rng.normal(0, 0.1, s)
        for k, s in (("ln1_beta", E), ("ln2_beta", E)):
            W[f"layer0.{k}"] = rng.normal(0, 0.1, s)
        for k, s in (("qw", (E, E)), ("kw", (E, E)), ("vw", (E, E)), ("projw", (E, E)),
                     ("up", (E, H)), ("dp", (H, E))):
            W[f"layer0.{k}"] = rng.normal(0, 0.3, s)
        tok = rng.integers(0, V, (B, T))
        tgt = rng.integers(0, V, (B, T))
        _, _, G = O.forward_backward(W, tok, tgt, B, T, NH, L)
        for name in ("layer0.qw", "layer0.up", "layer0.ln1_gamma", "linw", "embed", "pos",
                     "layer0.kw", "layer0.vw", "layer0.projw", "lnf_beta"):
            for _ in range(3):
                idx = tuple(rng.integers(0, d) for d in W[name].shape)
                if name == "embed":
                    idx = (int(tok[0, 0]),) + idx[1:]
                h = 1e-5
                W[name][idx] += h
                lp = O.forward_backward(W, tok, tgt, B, T, NH, L)[0]
                W[name][idx] -= 2 * h
                lm = O.forward_backward(W, tok, tgt, B, T, NH, L)[0]
                W[name][idx] += h
                fd = (lp - lm) / (2 * h)
                assert abs(fd - G[name][idx]) <= 1e-5 + 1e-4 * abs(fd), (name, idx, fd, G[name][idx])
    finally:
        O.r16, O.FLOAT = saved
