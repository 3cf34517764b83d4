"""GPU parity tests: every entry point of libmetalattn, called through the C
ABI, against the CPU oracle (exact-interface mode) and the golden fixtures.

Tolerances: O, dQ, dK, dV within max-abs 2e-2 and
relative-L2 1e-2 of the oracle's fp32 values; lse within 1e-3 absolute.
computeD is compared with the oracle's fp32 sum to 1 bf16 rounding step.
Configs 2, 3 and 4 are checked on every (batch, head) shard against the
oracle and, over the whole tensor, through size-independent identities."""
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from metalllm_b200.inputs import CONFIGS, bf16_bits_to_f32, normal_bf16  # noqa: E402

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2, LSE_ABS = 2e-2, 1e-2, 1e-3
GOLDEN = Path(__file__).resolve().parent / "golden" / "attn_golden.npz"


@pytest.fixture(scope="module")
def A():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from metalllm_b200.build import build_cuda
    build_cuda()
    from metalllm_b200 import attention
    return attention


def up(bits: np.ndarray) -> "torch.Tensor":
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def down(t: "torch.Tensor") -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def f32(t: "torch.Tensor") -> np.ndarray:
    return t.detach().cpu().float().numpy()


def bf(t) -> np.ndarray:
    return bf16_bits_to_f32(down(t)) if isinstance(t, torch.Tensor) else bf16_bits_to_f32(t)


def check(name, got, want, max_abs=MAX_ABS, rel_l2=REL_L2):
    from oracle.oracle import compare
    ok, mae, rl2 = compare(got, want, max_abs, rel_l2)
    assert ok, f"{name}: max_abs={mae:.3e} rel_l2={rl2:.3e}"


def inputs(B, T, H, D, seed=0, qkv_scale=1.0, do_scale=1.0):
    n = B * T * H * D
    shp = (B, T, H * D)
    return [normal_bf16(n, seed, s, sc).reshape(shp)
            for s, sc in ((1, qkv_scale), (2, qkv_scale), (3, qkv_scale), (4, do_scale))]


def gpu_chain(A, q, k, v, do, B, T, H, D):
    p = A.make_params(T, H, D)
    tq, tk, tv, tdo = up(q), up(k), up(v), up(do)
    out, l = A.flashAttentionForward(tq, tk, tv, p, B)
    Dv = A.computeD(tdo, out, p, B)
    dQ, dK, dV = A.flashAttentionBackward(tdo, Dv, l, tq, tk, tv, p, B)
    torch.cuda.synchronize()
    return out, l, Dv, dQ, dK, dV


# ------------------------------------------------------------------ golden
def _golden():
    z = np.load(GOLDEN)
    names = sorted({k.split("/")[0] for k in z.files})
    return [(n, {k.split("/")[1]: z[k] for k in z.files if k.startswith(n + "/")}) for n in names]


@pytest.mark.parametrize("name,case", _golden(), ids=[n for n, _ in _golden()])
def test_golden_vectors(A, name, case):
    B, T, H, D = (int(x) for x in case["shape"])
    p = A.make_params(T, H, D)
    tq, tk, tv, tdo = up(case["q"]), up(case["k"]), up(case["v"]), up(case["do"])
    out, l = A.flashAttentionForward(tq, tk, tv, p, B)
    check("O", bf(out), bf(case["o"]))
    assert np.abs(f32(l) - case["lse"]).max() <= LSE_ABS
    Dv = A.computeD(tdo, up(case["o"]), p, B)
    assert np.abs(bf(Dv) - case["d32"]).max() <= 2 ** -7 * max(1.0, np.abs(case["d32"]).max())
    dQ, dK, dV = A.flashAttentionBackward(tdo, up(case["d"]), torch.from_numpy(case["lse"]).cuda(),
                                          tq, tk, tv, p, B)
    check("dQ", f32(dQ), case["dq"])
    check("dK", bf(dK), case["dk32"])
    check("dV", bf(dV), case["dv32"])


# --------------------------------------------------- small and medium shapes
SHAPES = [
    (1, 64, 1, 64), (2, 128, 3, 64), (1, 192, 2, 128), (2, 256, 2, 64), (1, 320, 1, 128),
    (1, 1024, 2, 64), (1, 1024, 2, 128), (16, 256, 6, 64),  # the last one is config 1
    # sequence lengths that are not a multiple of the 64/128-row tiles (the
    # reference requires multiples of 64; here partial tiles are zero-filled
    # on load and clipped on store, per batch row)
    (1, 1, 1, 64), (2, 100, 2, 64), (3, 200, 3, 64), (2, 130, 2, 128), (1, 257, 2, 128),
    (2, 1000, 1, 64),
    # more than 16 tiles: both kernels deal their units by cluster launch
    # control (one CTA per unit) instead of static rounds
    (1, 2200, 2, 64), (1, 2113, 1, 128),
]


@pytest.mark.parametrize("B,T,H,D", SHAPES)
def test_parity_vs_oracle(A, oracle_mod, B, T, H, D):
    o = oracle_mod
    q, k, v, do = inputs(B, T, H, D, seed=T + D)
    out, l, Dv, dQ, dK, dV = gpu_chain(A, q, k, v, do, B, T, H, D)
    # forward against the oracle from the same inputs
    oo, ol, o32 = o.flash_forward(q, k, v, H, want_f32=True)
    check("O", bf(out), o32)
    assert np.abs(f32(l) - ol).max() <= LSE_ABS
    # computeD against the oracle from the GPU's O
    od, od32 = o.compute_d(do, down(out), H, want_f32=True)
    assert np.abs(bf(Dv) - od32).max() <= 2 ** -8 * max(1.0, np.abs(od32).max())
    # backward against the oracle fed the same l and D as the GPU
    rq, rk, rv, rk32, rv32 = o.flash_backward(do, down(Dv), f32(l), q, k, v, H, want_f32=True)
    check("dQ", f32(dQ), rq)
    check("dK", bf(dK), rk32)
    check("dV", bf(dV), rv32)


def test_row0_equals_v_row0(A):
    """README.md:132: row 0 of a causal head equals V row 0 (bit-exact)."""
    B, T, H, D = 3, 256, 4, 128
    q, k, v, _ = inputs(B, T, H, D, seed=3)
    p = A.make_params(T, H, D)
    out, l = A.flashAttentionForward(up(q), up(k), up(v), p, B)
    assert np.array_equal(down(out)[:, 0, :], v[:, 0, :])


@pytest.mark.parametrize("T", [256, 200])
def test_shard_entry_points(A, T):
    """Shard variants write exactly their (batch, head) slabs, bit-identical to
    the full call, and leave the rest untouched (also at a ragged length)."""
    B, H, D = 2, 3, 64
    q, k, v, do = inputs(B, T, H, D, seed=9)
    full = gpu_chain(A, q, k, v, do, B, T, H, D)
    p = A.make_params(T, H, D)
    tq, tk, tv, tdo = up(q), up(k), up(v), up(do)
    b0, b1 = 2, 5
    act = (B, T, H * D)
    out = torch.full(act, float("nan"), dtype=torch.bfloat16, device="cuda")
    l = torch.full((B, T, H), float("nan"), dtype=torch.float32, device="cuda")
    Dv = torch.full((B, T, H), float("nan"), dtype=torch.bfloat16, device="cuda")
    dQ = torch.full(act, float("nan"), dtype=torch.float32, device="cuda")
    dK = torch.full(act, float("nan"), dtype=torch.bfloat16, device="cuda")
    dV = torch.full(act, float("nan"), dtype=torch.bfloat16, device="cuda")
    A.flashAttentionForward(tq, tk, tv, p, B, out=out, l=l, shard=(b0, b1))
    A.computeD(tdo, full[0], p, B, D=Dv, shard=(b0, b1))
    A.flashAttentionBackward(tdo, full[2], full[1], tq, tk, tv, p, B, dQ=dQ, dK=dK, dV=dV,
                             shard=(b0, b1))
    torch.cuda.synchronize()
    for bh in range(B * H):
        b, h = divmod(bh, H)
        cols = slice(h * D, (h + 1) * D)
        inside = b0 <= bh < b1
        for got, ref in ((out, full[0]), (dK, full[4]), (dV, full[5])):
            g = down(got[b, :, cols])
            if inside:
                assert np.array_equal(g, down(ref[b, :, cols]))
            else:
                assert np.isnan(bf16_bits_to_f32(g)).all()
        for got, ref in ((l, full[1]), (Dv, full[2])):
            g = got[b, :, h].float().cpu().numpy()
            if inside:
                assert np.array_equal(g, ref[b, :, h].float().cpu().numpy())
            else:
                assert np.isnan(g).all()
        g = f32(dQ[b, :, cols])
        if inside:
            check("dQ shard", g, f32(full[3][b, :, cols]), 1e-5, 1e-6)
        else:
            assert np.isnan(g).all()


@pytest.mark.parametrize("B,T,H,D,shard", [(2, 100, 3, 64, None), (4, 256, 6, 64, None),
                                         (2, 1024, 2, 64, None), (3, 200, 2, 64, (1, 5)),
                                         (2, 130, 3, 128, None)])
def test_forward_with_fused_compute_d(A, B, T, H, D, shard):
    """ma_flashAttentionForwardComputeD: out and l bit-identical to the plain
    forward, D within one bf16 step of computeD on the same O (the fused fp32
    sum runs in another order); a shard touches only its (batch, head) slabs."""
    q, k, v, do = inputs(B, T, H, D, seed=27)
    p = A.make_params(T, H, D)
    tq, tk, tv, tdo = up(q), up(k), up(v), up(do)
    sentinel = lambda shp, dt: torch.full(shp, 7.0, dtype=dt, device="cuda")
    ref_out, ref_l = sentinel((B, T, H * D), torch.bfloat16), sentinel((B, T, H), torch.float32)
    A.flashAttentionForward(tq, tk, tv, p, B, out=ref_out, l=ref_l, shard=shard)
    ref_D = sentinel((B, T, H), torch.bfloat16)
    A.computeD(tdo, ref_out, p, B, D=ref_D, shard=shard)
    out, l, Dv = (sentinel((B, T, H * D), torch.bfloat16), sentinel((B, T, H), torch.float32),
                  sentinel((B, T, H), torch.bfloat16))
    A.flashAttentionForwardComputeD(tq, tk, tv, tdo, p, B, out=out, l=l, D=Dv, shard=shard)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    assert torch.equal(out, ref_out) and torch.equal(l, ref_l)
    got, want = Dv.float().cpu().numpy(), ref_D.float().cpu().numpy()
    assert np.abs(got - want).max() <= 2 ** -7 * max(1.0, np.abs(want).max())
    if shard is not None:  # untouched slabs keep the sentinel
        flat = Dv.float().cpu().numpy()
        for bh in list(range(0, shard[0])) + list(range(shard[1], B * H)):
            b, h = divmod(bh, H)
            assert np.all(flat[b, :, h] == 7.0)


def test_determinism(A):
    B, T, H, D = 2, 512, 2, 64
    q, k, v, do = inputs(B, T, H, D, seed=21)
    r1 = gpu_chain(A, q, k, v, do, B, T, H, D)
    r2 = gpu_chain(A, q, k, v, do, B, T, H, D)
    for i in (0, 1, 2, 4, 5):
        assert torch.equal(r1[i], r2[i]), i
    check("dQ rerun", f32(r1[3]), f32(r2[3]), 1e-5, 1e-6)


@pytest.mark.parametrize("B,T,H,D", [(2, 512, 2, 64), (1, 2304, 2, 64), (1, 1024, 2, 128)])
def test_replay_from_a_cuda_graph(A, B, T, H, D):
    """The attention step captured once into a CUDA graph and replayed twice
    gives the eager results: the plain chain (forward, computeD, backward) and
    the bench's two launches (forward with computeD and dQ's zeros, backward
    accumulating into dQ), under both schedules (static rounds at T=512;
    cluster launch control for both kernels at T=2304 and for the d=128
    backward)."""
    q, k, v, do = inputs(B, T, H, D, seed=41)
    ref = gpu_chain(A, q, k, v, do, B, T, H, D)
    p = A.make_params(T, H, D)
    tq, tk, tv, tdo = up(q), up(k), up(v), up(do)
    act, rows = (B, T, H * D), (B, T, H)
    new = lambda shp, dt: torch.full(shp, float("nan"), dtype=dt, device="cuda")
    bufs = [new(act, torch.bfloat16), new(rows, torch.float32), new(rows, torch.bfloat16),
            new(act, torch.float32), new(act, torch.bfloat16), new(act, torch.bfloat16)]
    fused = [new(act, torch.bfloat16), new(rows, torch.float32), new(rows, torch.bfloat16),
             new(act, torch.float32), new(act, torch.bfloat16), new(act, torch.bfloat16)]

    def step():
        out, l, Dv, dQ, dK, dV = bufs
        A.flashAttentionForward(tq, tk, tv, p, B, out=out, l=l)
        A.computeD(tdo, out, p, B, D=Dv)
        A.flashAttentionBackward(tdo, Dv, l, tq, tk, tv, p, B, dQ=dQ, dK=dK, dV=dV)
        out, l, Dv, dQ, dK, dV = fused
        A.flashAttentionForwardComputeD(tq, tk, tv, tdo, p, B, out=out, l=l, D=Dv, zero_dQ=dQ)
        A.flashAttentionBackward(tdo, Dv, l, tq, tk, tv, p, B, dQ=dQ, dK=dK, dV=dV, accumulate_dQ=True)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # eager warm-up outside the capture
        step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    # the eager results: the plain chain is the one gpu_chain runs (dQ to
    # fp32 rounding: its partial sums arrive in no fixed order); the fused
    # chain's D may differ from computeD's by one bf16 step, and dK, dQ with it
    for i in (0, 1, 2, 4, 5):
        assert torch.equal(bufs[i], ref[i]), i
    check("dQ plain", f32(bufs[3]), f32(ref[3]), 1e-4, 1e-5)
    eager = [[t.clone() for t in bufs], [t.clone() for t in fused]]
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(2):
        for b in bufs + fused:
            b.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert A.device_status() == 0
        for got, want in zip((bufs, fused), eager):
            for i in (0, 1, 2, 4, 5):
                assert torch.equal(got[i], want[i]), i
            check("dQ replay", f32(got[3]), f32(want[3]), 1e-4, 1e-5)


@pytest.mark.parametrize("B,M,H,D", [
    (2, 256, 6, 64),     # N = 384 (128-column tiles)
    (1, 64, 3, 64),      # N = 192 (64-column tiles), one partial row tile
    (3, 192, 2, 128),    # N = 256, rows not a multiple of 128
    (64, 256, 6, 64),    # config 5: rows = 16384, N = 384
    (3, 100, 3, 64),     # M not a multiple of 64: rows = 300
])
def test_compute_qkv(A, oracle_mod, B, M, H, D):
    N = H * D
    X = normal_bf16(B * M * N, 31, 5).reshape(B, M, N)
    W = [normal_bf16(N * N, 31, 6 + i, 0.02).reshape(N, N) for i in range(3)]
    p = A.make_params(M, H, D)
    q, k, v = A.computeQKV(up(X), up(W[0]), up(W[1]), up(W[2]), p, B)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    rq, rk, rv, rq32, rk32, rv32 = oracle_mod.compute_qkv(X, *W, want_f32=True)
    check("Q", bf(q), rq32, 1e-2, 5e-3)
    check("K", bf(k), rk32, 1e-2, 5e-3)
    check("V", bf(v), rv32, 1e-2, 5e-3)


def test_cuda_attention_class_and_stream(A, oracle_mod):
    B, T, H, D = 2, 256, 2, 128
    q, k, v, do = inputs(B, T, H, D, seed=41)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        att = A.CudaAttention(B, T, H, D)
        out, l = att.forward(up(q), up(k), up(v), stream=s)
        dQ, dK, dV = att.backward(up(do), stream=s)
    s.synchronize()
    ref = gpu_chain(A, q, k, v, do, B, T, H, D)
    assert torch.equal(out, ref[0]) and torch.equal(dK, ref[4])
    assert A.device_status() == 0


def test_bad_call_on_gpu_raises(A):
    p = A.make_params(96, 1, 32)  # head size 32
    x = torch.zeros(1, 96, 32, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(A.MetalAttnError, match="MA_ERR_SHAPE"):
        A.flashAttentionForward(x, x, x, p, 1)


# ------------------------------------------------ BASELINE configs 2, 3, 4
@pytest.mark.parametrize("cfg", ["c2", "c3", "c4"])
def test_full_config_every_shard(A, oracle_mod, cfg):
    """Every (batch, head) shard of configs 2, 3 and 4 (768, 128 and 128
    shards; attention.metal:74-76, 219-221 compute every head of every row)
    against the oracle: O and l against the oracle's forward, D against
    computeD of the oracle's own bf16 O, and dQ, dK, dV twice: against the
    oracle's backward fed the GPU's l and D (the backward kernel alone, at the
    north_star tolerance) and against the oracle's backward fed its own l and
    D, so that no GPU intermediate is in that chain (a convention shared by
    the GPU's forward and backward but not the reference's would show there).
    Plus, over the whole tensor, README.md:132 (row 0 of every causal head is
    V row 0, bit for bit) and sum_keys dV = sum_queries dO per head.  These
    cover every unit of the persistent forward's alternating rounds and both
    backward schedules (persistent at C2, one unit per CTA at C3/C4)."""
    c = CONFIGS[cfg]
    B, T, H, D = c["B"], c["T"], c["H"], c["D"]
    q, k, v, do = inputs(B, T, H, D, seed=0, qkv_scale=c["qkv_scale"], do_scale=c["do_scale"])
    out, l, Dv, dQ, dK, dV = gpu_chain(A, q, k, v, do, B, T, H, D)
    assert A.device_status() == 0
    assert np.array_equal(down(out[:, 0, :]), v[:, 0, :])
    sdv = dV.double().sum(1)
    sdo = torch.from_numpy(bf16_bits_to_f32(do)).cuda().double().sum(1)
    rel = ((sdv - sdo).norm() / sdo.norm()).item()
    assert rel < 1e-2, rel
    g_out, g_l, g_D = bf(out), f32(l), down(Dv)
    g_dQ, g_dK, g_dV = f32(dQ), bf(dK), bf(dV)
    del out, l, Dv, dQ, dK, dV
    # the oracle's own chain: O, l, D
    o_out, o_l, o_32 = oracle_mod.flash_forward(q, k, v, H, want_f32=True)
    check(f"{cfg} O", g_out, o_32)
    assert np.abs(g_l - o_l).max() <= LSE_ABS
    del o_32
    o_D, o_D32 = oracle_mod.compute_d(do, o_out, H, want_f32=True)
    gD = bf16_bits_to_f32(g_D)
    check(f"{cfg} D", gD, o_D32, 2 ** -6 * max(1.0, float(np.abs(o_D32).max())), REL_L2)
    del o_out, o_D32
    # the oracle's backward fed the GPU's l and D: the north_star tolerance
    fq, _, _, fk, fv = oracle_mod.flash_backward(do, g_D, g_l, q, k, v, H, want_f32=True)
    check(f"{cfg} dQ", g_dQ, fq)
    check(f"{cfg} dK", g_dK, fk)
    check(f"{cfg} dV", g_dV, fv)
    # the oracle's backward from its own l and D (no GPU value in the chain).
    # D is stored as bf16 (attention.metal:193), and where the two chains'
    # bf16 O differ by a rounding step their D can round one step apart; a
    # step of D moves dS = P (dP - D) / sqrt(d), hence dQ and dK, by up to
    # |dD| |K| / sqrt(d) per key.  The allowance is that effect as the oracle
    # itself shows it (its backward fed the GPU's D vs its own), on top of the
    # north_star max-abs; rel-L2 keeps the north_star bound.
    rq, _, _, rk, rv = oracle_mod.flash_backward(do, o_D, o_l, q, k, v, H, want_f32=True)
    for name, got, own, fed in (("dQ", g_dQ, rq, fq), ("dK", g_dK, rk, fk), ("dV", g_dV, rv, fv)):
        allowance = float(np.abs(own - fed).max())
        check(f"{cfg} {name} (oracle chain, allowance {allowance:.2e})", got, own, MAX_ABS + allowance, REL_L2)


@pytest.mark.parametrize("B,T,H,D,shard", [(2, 512, 3, 64, None), (3, 200, 2, 64, (1, 5)),
                                         (2, 130, 3, 128, None), (2, 256, 2, 128, (1, 3)),
                                         (2, 2200, 2, 64, (1, 3))])
def test_forward_zero_dq_and_accumulating_backward(A, B, T, H, D, shard):
    """ma_flashAttentionForwardComputeDZeroDQ writes out, l, D bit-identical
    to ma_flashAttentionForwardComputeD and exact zeros to dQ on the
    (batch, head) slabs it computes (rows < T), nothing elsewhere;
    ma_flashAttentionBackwardAccumulate then adds the backward's dQ into
    dQ (the reference's contract, attention.metal:292-296 with the host
    zeroing of model.h:549-551) and writes dK, dV bit-identical to
    ma_flashAttentionBackward."""
    q, k, v, do = inputs(B, T, H, D, seed=33)
    p = A.make_params(T, H, D)
    tq, tk, tv, tdo = up(q), up(k), up(v), up(do)
    act = (B, T, H * D)
    nan = lambda shp, dt: torch.full(shp, float("nan"), dtype=dt, device="cuda")
    r_out, r_l, r_D = nan(act, torch.bfloat16), nan((B, T, H), torch.float32), nan((B, T, H), torch.bfloat16)
    A.flashAttentionForwardComputeD(tq, tk, tv, tdo, p, B, out=r_out, l=r_l, D=r_D, shard=shard)
    r_dQ, r_dK, r_dV = nan(act, torch.float32), nan(act, torch.bfloat16), nan(act, torch.bfloat16)
    A.flashAttentionBackward(tdo, r_D, r_l, tq, tk, tv, p, B, dQ=r_dQ, dK=r_dK, dV=r_dV, shard=shard)
    out, l, Dv = nan(act, torch.bfloat16), nan((B, T, H), torch.float32), nan((B, T, H), torch.bfloat16)
    dQ = nan(act, torch.float32)
    A.flashAttentionForwardComputeD(tq, tk, tv, tdo, p, B, out=out, l=l, D=Dv, shard=shard, zero_dQ=dQ)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    same = lambda a, b: torch.equal(torch.nan_to_num(a.float(), nan=7.0), torch.nan_to_num(b.float(), nan=7.0))
    assert same(out, r_out) and same(l, r_l) and same(Dv, r_D)
    lo, hi = shard if shard is not None else (0, B * H)
    for bh in range(B * H):
        b, h = divmod(bh, H)
        slab = dQ[b, :, h * D:(h + 1) * D]
        if lo <= bh < hi:
            assert torch.equal(slab, torch.zeros_like(slab))
        else:
            assert torch.isnan(slab).all()
    # the accumulating backward on the zeros: dQ as the writing backward's
    dK, dV = nan(act, torch.bfloat16), nan(act, torch.bfloat16)
    A.flashAttentionBackward(tdo, Dv, l, tq, tk, tv, p, B, dQ=dQ, dK=dK, dV=dV, shard=shard,
                             accumulate_dQ=True)
    torch.cuda.synchronize()
    assert same(dK, r_dK) and same(dV, r_dV)
    for bh in range(lo, hi):
        b, h = divmod(bh, H)
        cols = slice(h * D, (h + 1) * D)
        check(f"dQ[{bh}]", f32(dQ[b, :, cols]), f32(r_dQ[b, :, cols]), 1e-5, 1e-6)
    # and onto earlier partial sums: dQ = X + the backward's dQ
    X = torch.randn(act, device="cuda")
    dQ2 = X.clone()
    A.flashAttentionBackward(tdo, Dv, l, tq, tk, tv, p, B, dQ=dQ2, shard=shard, accumulate_dQ=True)
    torch.cuda.synchronize()
    for bh in range(B * H):
        b, h = divmod(bh, H)
        cols = slice(h * D, (h + 1) * D)
        if lo <= bh < hi:
            check(f"X+dQ[{bh}]", f32(dQ2[b, :, cols]), f32(X[b, :, cols] + r_dQ[b, :, cols]), 1e-5, 1e-6)
        else:
            assert torch.equal(dQ2[b, :, cols], X[b, :, cols])
    assert A.device_status() == 0
