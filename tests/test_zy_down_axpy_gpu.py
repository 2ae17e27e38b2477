"""GPU parity of the engine's down projection in the reference's transposed
layout, ft::matmul_down_axpy (ft/src/cpu_backend.cpp:60-75): y[m] += x_m . W
over n_in rows of N weights, zero activations skipped, y accumulated.
Checked against the CPU oracle and, through the golden fixture, against the
reference's own outputs.  Tolerance as in the GEMV tests: max |y - ref| /
(|ref| + 1e-2 rms(ref)) <= 2e-3 (the GPU sums row slabs separately).  Also
runs the C++ adapter's down_project and moe_ffn checks
(tests/cpp/test_cuda_backend.cpp --down-project).  The file runs late in the suite, after the kernels this
path shares (dequant, GEMV, GEMM) are checked."""
import subprocess

import numpy as np
import pytest

from xwfes_b200 import formats as F, synth as S

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 2e-3
FLOOR = 1e-2


def rel_err(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(y - ref) / (np.abs(ref) + FLOOR * rms)))


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def ftc():
    assert torch.cuda.is_available(), "GPU test needs CUDA"
    from xwfes_b200 import ftc as mod
    mod.lib()
    return mod


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def weights(t, n_in, n, seed=0):
    """n_in rows of n weights in format t, as uint8 [n_in, row_bytes]."""
    if t in (F.Q8_0, F.Q4_K, F.Q6_K):
        return S.weight(t, n_in, n, seed=seed, name="axpy.w")
    g = np.random.default_rng(1000 + seed * 31 + t)
    if t == F.F32:
        return g.standard_normal((n_in, n), dtype=np.float32).view(np.uint8)
    if t == F.F16:
        return g.standard_normal((n_in, n)).astype(np.float16).view(np.uint8)
    if t == F.BF16:
        return S.f32_to_bf16_bits(g.standard_normal((n_in, n)).astype(np.float32)).view(np.uint8)
    eb, bb = F.BLOCK[t]
    w = g.integers(0, 256, size=(n_in, n // eb, bb), dtype=np.uint8)
    w[:, :, 0:2] = np.array([0x2E66], dtype=np.uint16).view(np.uint8)  # sane fp16 scales
    if t == F.Q4_1:
        w[:, :, 2:4] = np.array([0x2A66], dtype=np.uint16).view(np.uint8)
    return w.reshape(n_in, -1)


def inputs(m, n_in, n, seed=0):
    x = S.activations_f32(m, n_in, seed=seed, name="axpy.x")
    x[:, ::5] = 0.0  # rows the reference skips
    y0 = S.activations_f32(m, n, seed=seed + 1, name="axpy.y")
    return x, y0


def run(ftc, w, t, n_in, n, x, y0, offset=0):
    """The device entry; ``offset`` > 0 places the weight that many bytes
    into a buffer (misaligned rows take the element-by-element decoder)."""
    buf = np.zeros(w.size + 16, dtype=np.uint8)
    buf[offset:offset + w.size] = w.reshape(-1)
    d = dev(buf)
    y = dev(y0)
    ftc.matmul_down_axpy(d[offset:], t, n_in, n, dev(x), y, row_stride=w.shape[1])
    torch.cuda.synchronize()
    return y.cpu().numpy()


CASES = [
    (F.Q4_K, 14336, 4096, 1),  # Llama-3-8B dense down at one token: many row slabs
    (F.Q4_K, 4096, 14336, 2),
    (F.Q4_K, 37, 512, 3),      # ragged slabs
    (F.Q4_K, 1000, 256, 13),   # two token groups
    (F.Q6_K, 333, 1024, 2),
    (F.Q6_K, 2048, 4096, 8),
    (F.Q8_0, 96, 4096, 9),
    (F.Q8_0, 5, 32, 1),        # one block per row, one slab
    (F.F16, 100, 100, 4),      # N not a multiple of 8
    (F.BF16, 64, 72, 1),
    (F.F32, 50, 33, 2),
    (F.Q4_0, 72, 96, 5),
    (F.Q4_1, 40, 64, 3),
]


@pytest.mark.parametrize("t,n_in,n,m", CASES)
def test_matches_oracle(ftc, oracle, t, n_in, n, m):
    w = weights(t, n_in, n)
    x, y0 = inputs(m, n_in, n)
    y = run(ftc, w, t, n_in, n, x, y0)
    ref = oracle.matmul_down_axpy(x, w, t, n, y0.copy(), threads=8)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("name,t", [("q8_0", F.Q8_0), ("f16", F.F16), ("q4_0", F.Q4_0)])
def test_reference_golden(ftc, golden, name, t):
    g = golden("ref_down_axpy.npz")
    w, x, y0 = g[name + "_w"], g[name + "_x"], g[name + "_y0"]
    y = run(ftc, w, t, w.shape[0], y0.shape[1], x, y0)
    assert rel_err(y, g[name + "_y"]) <= TOL


@pytest.mark.parametrize("t,offset", [(F.Q4_K, 2), (F.Q4_K, 1), (F.Q6_K, 1), (F.Q8_0, 1)])
def test_vector_decoders_equal_element_decoder(ftc, t, offset):
    """Misaligned weights take the element-by-element decoder with the same
    plan and order of sums: the vector decoders must give the same bits."""
    n_in, n, m = 300, 2048, 3
    w = weights(t, n_in, n, seed=2)
    x, y0 = inputs(m, n_in, n, seed=2)
    a = run(ftc, w, t, n_in, n, x, y0)
    b = run(ftc, w, t, n_in, n, x, y0, offset=offset)
    assert np.array_equal(bits(a), bits(b))


def test_deterministic(ftc):
    t, n_in, n, m = F.Q4_K, 14336, 4096, 1
    w = weights(t, n_in, n, seed=3)
    x, y0 = inputs(m, n_in, n, seed=3)
    a = run(ftc, w, t, n_in, n, x, y0)
    b = run(ftc, w, t, n_in, n, x, y0)
    assert np.array_equal(bits(a), bits(b))


def test_zero_activation_skips_non_finite_weights(ftc, oracle):
    """The reference adds nothing for x == 0, so an inf weight in such a row
    leaves y finite."""
    n_in, n = 16, 64
    vals = np.random.default_rng(5).standard_normal((n_in, n)).astype(np.float16)
    vals[3, 10] = np.inf
    w = vals.view(np.uint8)
    x = S.activations_f32(2, n_in, seed=5)
    x[:, 3] = 0.0
    y0 = np.zeros((2, n), dtype=np.float32)
    y = run(ftc, w, F.F16, n_in, n, x, y0)
    ref = oracle.matmul_down_axpy(x, w, F.F16, n, y0.copy())
    assert np.isfinite(y).all() and np.isfinite(ref).all()
    assert rel_err(y, ref) <= TOL


def test_backend_entry(ftc, oracle):
    """ftc_backend_matmul_down_axpy: host buffers, weight through the cache."""
    t, n_in, n, m = F.Q4_K, 2048, 4096, 2
    w = weights(t, n_in, n, seed=4)
    x, y0 = inputs(m, n_in, n, seed=4)
    be = ftc.CudaBackend(0)
    try:
        W = ftc.HostTensor(w, t, (n, n_in))
        y = y0.copy()
        be.matmul_down_axpy(x, m, n_in, W, y)
        ref = oracle.matmul_down_axpy(x, w, t, n, y0.copy(), threads=8)
        assert rel_err(y, ref) <= TOL
        y2 = y0.copy()
        be.matmul_down_axpy(x, 0, n_in, W, y2)  # no rows: y unchanged
        assert np.array_equal(y2, y0)
        with pytest.raises(ValueError):
            be.matmul_down_axpy(x, m, n_in + 1, W, y2)
    finally:
        be.close()


def test_cpp_adapter_down_project(tmp_path):
    from tests.test_cpp_backend import compile_test
    exe = compile_test(str(tmp_path / "test_cuda_backend"))
    r = subprocess.run([exe, "--down-project"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "all tests passed" in r.stdout, r.stdout + r.stderr
