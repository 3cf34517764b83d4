"""GPU parity of the GEMMs around attention (attention.metal:301-455) against
the CPU oracle, through the C ABI: projForward, projBackwarddW,
projBackwarddX, computeGradDx, computeGradDw.

Tolerance: bf16 products of N(0,1) activations with N(0, 0.02) weights,
compared with the oracle's fp32 sums: max-abs error within 1e-2 of the
largest reference magnitude and relative-L2 within 5e-3 (the GPU rounds the
fp32 dQ operand to bf16 on entry; the outputs round once).  Config-5 shapes
(16384 activation rows) are checked on a sample of output rows."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from metalllm_b200.inputs import bf16_bits_to_f32, normal_bf16  # noqa: E402

pytestmark = pytest.mark.gpu

REL_MAX, REL_L2 = 1e-2, 5e-3
SHAPES = [(2, 100, 128), (4, 256, 384), (64, 256, 384)]  # (B, M, N); the last is config 5


@pytest.fixture(scope="module")
def A():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from metalllm_b200.build import build_cuda
    build_cuda()
    from metalllm_b200 import attention
    return attention


def up(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def bf(t):
    return bf16_bits_to_f32(t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16))


def rel_check(name, got, want, rows=None):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    if rows is not None:
        got, want = got[rows], want[rows]
    scale = max(np.abs(want).max(), 1e-30)
    mae = np.abs(got - want).max() / scale
    rl2 = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    assert mae <= REL_MAX and rl2 <= REL_L2, f"{name}: max_abs/scale={mae:.3e} rel_l2={rl2:.3e}"


def _data(B, M, N, seed):
    R = B * M
    act = lambda s, sc=1.0: normal_bf16(R * N, seed, s, sc).reshape(B, M, N)
    w = lambda s: normal_bf16(N * N, seed, s, 0.02).reshape(N, N)
    rng = np.random.default_rng(seed)
    dq = rng.standard_normal((B, M, N)).astype(np.float32)
    return act, w, dq


def _rows(R, big):
    if not big:
        return None
    rng = np.random.default_rng(5)
    return np.sort(rng.choice(R, size=96, replace=False))


@pytest.mark.parametrize("B,M,N", SHAPES)
def test_proj_forward_and_backward_dx(A, oracle_mod, B, M, N):
    act, w, _ = _data(B, M, N, 41)
    attn, wp = act(1), w(2)
    p = A.make_params(M, N // 64, 64)
    out = A.projForward(up(attn), up(wp), p, B)
    dz = act(3)
    dattn = A.projBackwarddX(up(dz), up(wp), p, B)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    R = B * M
    rows = _rows(R, R > 4096)
    _, o32 = oracle_mod.proj_forward(attn, wp, rows=rows)
    rel_check("projForward", bf(out).reshape(R, N), o32, rows)
    _, d32 = oracle_mod.proj_backward_dx(dz, wp, rows=rows)
    rel_check("projBackwarddX", bf(dattn).reshape(R, N), d32, rows)


@pytest.mark.parametrize("B,M,N", SHAPES)
def test_proj_backward_dw(A, oracle_mod, B, M, N):
    act, _, _ = _data(B, M, N, 43)
    attn, dz = act(1), act(2)
    p = A.make_params(M, N // 64, 64)
    dw = A.projBackwarddW(up(attn), up(dz), p, B)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    rows = np.arange(0, N, 7) if B * M > 4096 else None
    _, w32 = oracle_mod.proj_backward_dw(attn, dz, rows=rows)
    rel_check("projBackwarddW", bf(dw), w32, rows)


@pytest.mark.parametrize("B,M,N", SHAPES)
def test_compute_grad_dx(A, oracle_mod, B, M, N):
    act, w, dq = _data(B, M, N, 47)
    dk, dv = act(1), act(2)
    qw, kw, vw = w(3), w(4), w(5)
    p = A.make_params(M, N // 64, 64)
    dx = A.computeGradDx(up(qw), up(kw), up(vw), torch.from_numpy(dq).cuda(), up(dk), up(dv), p, B)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    R = B * M
    rows = _rows(R, R > 4096)
    ref = oracle_mod.grad_dx(qw, kw, vw, dq, dk, dv, rows=rows)
    rel_check("computeGradDx", dx.cpu().numpy().reshape(R, N), ref, rows)


@pytest.mark.parametrize("B,M,N", SHAPES)
def test_compute_grad_dw(A, oracle_mod, B, M, N):
    act, _, dq = _data(B, M, N, 53)
    x, dk, dv = act(1), act(2), act(3)
    p = A.make_params(M, N // 64, 64)
    dqw, dkw, dvw = A.computeGradDw(up(x), torch.from_numpy(dq).cuda(), up(dk), up(dv), p, B)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    rows = np.arange(0, N, 7) if B * M > 4096 else None
    rq, _, _, rk32, rv32 = oracle_mod.grad_dw(x, dq, dk, dv, rows=rows)
    rel_check("dQw", dqw.cpu().numpy(), rq, rows)
    rel_check("dKw", bf(dkw), rk32, rows)
    rel_check("dVw", bf(dvw), rv32, rows)


def test_gemm_outputs_written_not_accumulated(A):
    """Outputs are overwritten: NaN-filled output buffers give the same result
    as fresh ones (the reference's host zeroes them first, model.h:552-556)."""
    B, M, N = 2, 128, 128
    act, w, dq = _data(B, M, N, 59)
    x, dk, dv = up(act(1)), up(act(2)), up(act(3))
    tdq = torch.from_numpy(dq).cuda()
    p = A.make_params(M, N // 64, 64)
    ref = A.computeGradDw(x, tdq, dk, dv, p, B)
    bufs = [torch.full((N, N), float("nan"), dtype=t.dtype, device="cuda") for t in ref]
    got = A.computeGradDw(x, tdq, dk, dv, p, B, dQw=bufs[0], dKw=bufs[1], dVw=bufs[2])
    torch.cuda.synchronize()
    for g, r in zip(got, ref):
        assert torch.equal(g, r)


def test_gemm_rejects_bad_n(A):
    p = A.make_params(64, 1, 96)  # N = 96 is not a multiple of 64
    x = torch.zeros(1, 64, 96, dtype=torch.bfloat16, device="cuda")
    wt = torch.zeros(96, 96, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(A.MetalAttnError, match="MA_ERR_SHAPE"):
        A.projForward(x, wt, p, 1)


@pytest.mark.parametrize("B,M,H,D", [(2, 100, 2, 64), (4, 256, 6, 64), (2, 130, 3, 128)])
def test_proj_backward_dx_with_fused_compute_d(A, B, M, H, D):
    """projBackwarddX + computeD in one launch (D formed in the GEMM epilogue)
    equals the two separate entry points: dAttn bit for bit, D to one bf16
    rounding step (the fp32 sum runs in another order)."""
    N = H * D
    act, w, _ = _data(B, M, N, 61)
    dz, o, wp = up(act(1)), up(act(2)), up(w(3))
    p = A.make_params(M, H, D)
    dattn, Dv = A.projBackwarddXComputeD(dz, wp, o, p, B)
    ref_dattn = A.projBackwarddX(dz, wp, p, B)
    ref_D = A.computeD(ref_dattn, o, p, B)
    torch.cuda.synchronize()
    assert A.device_status() == 0
    assert torch.equal(dattn, ref_dattn)
    got, want = Dv.float().cpu().numpy(), ref_D.float().cpu().numpy()
    assert np.abs(got - want).max() <= 2 ** -7 * max(1.0, np.abs(want).max())
