"""The small-batch Q4_K GEMV on the integer tensor path (gemv_imma.cu:
mma.sync m16n8k32 with the activations as exact 24-bit signed-digit planes),
which ftc_mul_mat_vec uses for 2..8 tokens: parity with the CPU oracle
(the reference's per-row dot_row_f32 arithmetic, ft/include/ft/quant.h:
86-103), exactness on one-hot activations, and the launch shapes whose
row-tiles are split over CTAs or k-groups (finished through the fix-up
slots)."""
import os

import numpy as np
import pytest

from xwfes_b200 import formats as F, synth as S

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 2e-3
FLOOR = 1e-2
THREADS = os.cpu_count() or 8


def rel_err(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(y - ref) / (np.abs(ref) + FLOOR * rms)))


@pytest.fixture(scope="module")
def ftc():
    assert torch.cuda.is_available(), "GPU test needs CUDA"
    from xwfes_b200 import ftc as mod
    mod.lib()
    return mod


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def gemv(ftc, w, n, k, x):
    y = ftc.mul_mat_vec(dev(w), F.Q4_K, n, k, dev(x))
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
    return y.cpu().numpy()


@pytest.mark.parametrize("m", [2, 3, 4, 5, 8])
@pytest.mark.parametrize("n,k", [(14336, 4096), (4096, 14336), (1024, 8192), (300, 2560),
                                 (17, 768), (1, 256)])
def test_vs_oracle(ftc, oracle, m, n, k):
    w = S.weight(F.Q4_K, n, k, seed=n + k + m, name="imma")
    x = S.activations_f32(m, k, seed=m, name="imma.x")
    y = gemv(ftc, w, n, k, x)
    ref = oracle.matmul(x, w, F.Q4_K, k, threads=THREADS)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("m", [2, 6, 8])
def test_one_hot_columns_exact(ftc, oracle, m):
    """x = one-hot per token: y[t] is a column of the dequantized weight,
    bit for bit (each x fits the digit planes exactly)."""
    n, k = 333, 4096
    w = S.weight(F.Q4_K, n, k, seed=5, name="imma.oh")
    deq = oracle.dequant_rows(w, F.Q4_K, k)
    cols = [3, 255, 256, 1000, 2047, 4000, 4095, 17][:m]
    x = np.zeros((m, k), dtype=np.float32)
    for t, c in enumerate(cols):
        x[t, c] = 1.0
    y = gemv(ftc, w, n, k, x)
    for t, c in enumerate(cols):
        assert np.array_equal(y[t].view(np.uint32), np.ascontiguousarray(deq[:, c]).view(np.uint32))


@pytest.mark.parametrize("m", [2, 4, 8])
def test_deterministic_and_scale_exact(ftc, m):
    """Two launches give the same bits; doubling x doubles y exactly
    (power-of-two block scales), including rows finished through the
    split-row-tile slots (1024 x 8192: 64 row-tiles over all SMs)."""
    for n, k in ((1024, 8192), (4096, 14336)):
        w = S.weight(F.Q4_K, n, k, seed=9, name="imma.det")
        x = S.activations_f32(m, k, seed=9, name="imma.det.x")
        a, b = gemv(ftc, w, n, k, x), gemv(ftc, w, n, k, x)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        c = gemv(ftc, w, n, k, 2.0 * x)
        assert np.array_equal(c.view(np.uint32), (2.0 * a).astype(np.float32).view(np.uint32))


def test_grouped_matrices_equal_single(ftc, oracle):
    """q/k/v in one launch (ftc_mul_mat_vec_multi) equal three launches."""
    k, m = 4096, 4
    ns = (4096, 1024, 1024)
    ws = [S.weight(F.Q4_K, n, k, seed=i, name="imma.g") for i, n in enumerate(ns)]
    x = S.activations_f32(m, k, seed=2, name="imma.g.x")
    ys = ftc.mul_mat_vec_multi([dev(w) for w in ws], F.Q4_K, list(ns), k, dev(x))
    torch.cuda.synchronize()
    for w, n, yg in zip(ws, ns, ys):
        ref = oracle.matmul(x, w, F.Q4_K, k, threads=THREADS)
        assert rel_err(yg.cpu().numpy(), ref) <= TOL
