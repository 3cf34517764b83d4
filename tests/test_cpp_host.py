"""The C++ host mirrors in include/metalattn.hpp: CudaAttention (the
reference's MetalAttention harness, main.cpp:955-1284) compiles and links as
a reference-side C++ host would (CPU test), and on a GPU its forward/backward
give the same bits as the same entry points called from Python, with dX and
dQw rounded to bf16 on the host as the reference does; Model (model.h's
Model) gives the same loss sequence as the Python TrainingModel."""
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
CUDA = Path("/usr/local/cuda")

HOST_SRC = r'''
#include "metalattn.hpp"
#include <cstdio>
#include <cstdlib>
#include <vector>
// usage: host m n d B in.bin out.bin
// in.bin: x[B*m*n], qw, kw, vw, projw [n*n], dRes[B*m*n] (bf16 bits)
// out.bin: out[B*m*n], dprojw, dX[B*m*n], dqw, dkw, dvw
int main(int argc, char** argv) {
  if (argc != 7) return 2;
  const int m = std::atoi(argv[1]), n = std::atoi(argv[2]), d = std::atoi(argv[3]), B = std::atoi(argv[4]);
  const size_t act = (size_t)B * m * n, w = (size_t)n * n;
  std::vector<uint16_t> x(act), qw(w), kw(w), vw(w), pw(w), dres(act);
  FILE* f = std::fopen(argv[5], "rb");
  if (!f) return 3;
  for (auto* v : {&x, &qw, &kw, &vw, &pw, &dres})
    if (std::fread(v->data(), 2, v->size(), f) != v->size()) return 4;
  std::fclose(f);
  std::vector<uint16_t> out(act), dpw(w), dx(act), dqw(w), dkw(w), dvw(w);
  try {
    metalattn::CudaAttention attn(m, n, d, B);
    attn.forward(x.data(), qw.data(), kw.data(), vw.data(), pw.data(), out.data());
    attn.backward(dres.data(), dpw.data(), dx.data(), dqw.data(), dkw.data(), dvw.data());
  } catch (const std::exception& e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 5;
  }
  FILE* g = std::fopen(argv[6], "wb");
  for (auto* v : {&out, &dpw, &dx, &dqw, &dkw, &dvw}) std::fwrite(v->data(), 2, v->size(), g);
  std::fclose(g);
  return 0;
}
'''


def _build(tmp_path):
    src = tmp_path / "host.cpp"
    src.write_text(HOST_SRC)
    exe = tmp_path / "host"
    libdir = ROOT / "metalllm_b200"
    subprocess.run(["g++", "-std=c++17", "-O2", "-I", str(ROOT / "include"), "-I", str(CUDA / "include"), str(src),
                    "-L", str(libdir), "-lmetalattn", "-L", str(CUDA / "lib64"), "-lcudart",
                    f"-Wl,-rpath,{libdir}", f"-Wl,-rpath,{CUDA / 'lib64'}", "-o", str(exe)], check=True)
    return exe


def test_cpp_mirror_compiles_and_links(tmp_path, cuda_lib):
    assert _build(tmp_path).exists()


def _rne(a):
    """fp32 -> bf16 bits, round to nearest even (as metalattn::to_bf16)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,d,B", [(128, 128, 64, 1), (200, 256, 128, 2)])
def test_cpp_mirror_matches_python_path(tmp_path, cuda_lib, m, n, d, B):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from metalllm_b200 import attention as A
    from metalllm_b200.inputs import normal_bf16
    act, w = B * m * n, n * n
    x, dres = normal_bf16(act, 11, 1), normal_bf16(act, 11, 2)
    qw, kw, vw, pw = (normal_bf16(w, 11, 3 + i, 0.05) for i in range(4))
    inp, outp = tmp_path / "in.bin", tmp_path / "out.bin"
    with open(inp, "wb") as f:
        for a in (x, qw, kw, vw, pw, dres):
            f.write(np.ascontiguousarray(a, np.uint16).tobytes())
    exe = _build(tmp_path)
    r = subprocess.run([str(exe), str(m), str(n), str(d), str(B), str(inp), str(outp)], capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(outp, np.uint16)
    sizes = [act, w, act, w, w, w]
    parts = np.split(got, np.cumsum(sizes)[:-1])
    # the same sequence through the Python operator interface
    up = lambda a, shp: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).reshape(shp).cuda()
    bits = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).ravel()
    p = A.make_params(m, n // d, d)
    X, dR = up(x, (B, m, n)), up(dres, (B, m, n))
    Wq, Wk, Wv, Wp = (up(a, (n, n)) for a in (qw, kw, vw, pw))
    q, k, v = A.computeQKV(X, Wq, Wk, Wv, p, B)
    o, l = A.flashAttentionForward(q, k, v, p, B)
    po = A.projForward(o, Wp, p, B)
    dpw = A.projBackwarddW(o, dR, p, B)
    dz = A.projBackwarddX(dR, Wp, p, B)
    Dv = A.computeD(dz, o, p, B)
    dQ, dK, dV = A.flashAttentionBackward(dz, Dv, l, q, k, v, p, B)
    dX = A.computeGradDx(Wq, Wk, Wv, dQ, dK, dV, p, B)
    dQw, dKw, dVw = A.computeGradDw(X, dQ, dK, dV, p, B)
    torch.cuda.synchronize()
    want = [bits(po), bits(dpw), _rne(dX.cpu().numpy()).ravel(), _rne(dQw.cpu().numpy()).ravel(), bits(dKw),
            bits(dVw)]
    for name, g_, w_ in zip(("out", "dprojw", "dX", "dqw", "dkw", "dvw"), parts, want):
        assert np.array_equal(g_, w_), name


MODEL_SRC = r'''
#include "metalattn.hpp"
#include <cstdio>
#include <cstdlib>
#include <vector>
// usage: model in.bin  (tokens[B*m], targets[B*m] uint32); prints one loss per step
int main(int argc, char** argv) {
  const int m = 64, v = 128, e = 128, s = 2, d = 64, layers = 2, B = 2;
  std::vector<uint32_t> tok(B * m), tgt(B * m);
  FILE* f = std::fopen(argv[1], "rb");
  if (!f || std::fread(tok.data(), 4, tok.size(), f) != tok.size() ||
      std::fread(tgt.data(), 4, tgt.size(), f) != tgt.size())
    return 3;
  std::fclose(f);
  try {
    metalattn::Model model(m, v, e, s, d, layers, B, 0.003f, 3);
    for (int i = 0; i < 4; ++i) {  // Model::forward returns the loss (model.h:414), then backward, step
      const float loss = model.forward(tok.data(), tgt.data());
      model.backward();
      model.step();
      std::printf("%.9g\n", loss);
    }
  } catch (const std::exception& ex) {
    std::fprintf(stderr, "%s\n", ex.what());
    return 5;
  }
  return 0;
}
'''


@pytest.mark.gpu
def test_cpp_model_mirror_matches_python_training_model(tmp_path, cuda_lib):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from metalllm_b200 import train as T
    src, exe, inp = tmp_path / "model.cpp", tmp_path / "model", tmp_path / "tok.bin"
    src.write_text(MODEL_SRC)
    libdir = ROOT / "metalllm_b200"
    subprocess.run(["g++", "-std=c++17", "-O2", "-I", str(ROOT / "include"), "-I", str(CUDA / "include"), str(src),
                    "-L", str(libdir), "-lmetalattn", "-L", str(CUDA / "lib64"), "-lcudart",
                    f"-Wl,-rpath,{libdir}", f"-Wl,-rpath,{CUDA / 'lib64'}", "-o", str(exe)], check=True)
    rng = np.random.default_rng(9)
    tok = rng.integers(0, 128, (2, 64)).astype(np.uint32)
    tgt = rng.integers(0, 128, (2, 64)).astype(np.uint32)
    with open(inp, "wb") as f:
        f.write(tok.tobytes())
        f.write(tgt.tobytes())
    r = subprocess.run([str(exe), str(inp)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    cpp_losses = [float(x) for x in r.stdout.split()]
    model = T.TrainingModel(B=2, T=64, E=128, NH=2, layers=2, mlp_scale=2, vocab=128, lr=0.003, seed=3)
    ttok = torch.from_numpy(tok.astype(np.int32)).cuda()
    ttgt = torch.from_numpy(tgt.astype(np.int32)).cuda()
    py_losses = []
    for _ in range(4):
        model.forward(ttok, ttgt)
        py_losses.append(model.loss())
        model.backward()
        model.step()
    model.close()
    assert np.array_equal(np.float32(cpp_losses), np.float32(py_losses)), (cpp_losses, py_losses)
    assert cpp_losses[-1] < cpp_losses[0]
