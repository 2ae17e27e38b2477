"""GPU parity of the dequant and GEMV kernels against the CPU oracle (and,
through the golden fixtures, against the reference's own outputs).

Tolerance for float-accumulated outputs: max_i |y_i - ref_i| / (|ref_i| +
FLOOR * rms(ref)) <= 2e-3 -- relative error with a small absolute floor, as
the reference's own expert test does (ft/src/tests/test_core.cpp:342-344).
FLOOR = 1e-2: the reference's sequential fp32 sum over K = 4096..14336 terms
is itself off by ~3e-6 * rms(y) from the exact sum, so near-zero outputs need
a floor above that.  Dequantized weights are compared bit for bit."""
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


def run_gemv(ftc, w, t, n, k, x, row_stride=None):
    y = ftc.mul_mat_vec(dev(w), t, n, k, dev(x), row_stride=row_stride)
    torch.cuda.synchronize()
    return y.cpu().numpy()


# ------------------------------------------------------------ dequant

def test_dequant_matches_reference_golden(ftc, golden):
    g = golden("ref_q8_0_gemv.npz")
    for tag, k in (("k4096", 4096), ("k96", 96), ("k2080", 2080)):
        out = ftc.dequant(dev(g[f"{tag}_w"]), F.Q8_0, g[f"{tag}_w"].shape[0], k)
        torch.cuda.synchronize()
        assert np.array_equal(bits(out.cpu().numpy()), bits(g[f"{tag}_dequant"])), tag
    f = golden("ref_dequant_formats.npz")
    for name, t in (("f16", F.F16), ("bf16", F.BF16), ("q4_0", F.Q4_0), ("q4_1", F.Q4_1)):
        out = ftc.dequant(dev(f[name + "_w"]), t, 2, 64)
        torch.cuda.synchronize()
        assert np.array_equal(bits(out.cpu().numpy()), bits(f[name + "_dequant"])), name
    q = golden("ref_test_quant.npz")
    out = ftc.dequant(dev(q["q8row"][None]), F.Q8_0, 1, 64).cpu().numpy()[0]
    assert np.array_equal(bits(out), bits(q["dequant_q8"]))


def test_dequant_kquant_matches_gguf_golden(ftc, golden):
    g = golden("gguf_kquant.npz")
    for name, t in (("q4_k", F.Q4_K), ("q6_k", F.Q6_K)):
        blocks = g[name + "_blocks"]
        out = ftc.dequant(dev(blocks), t, blocks.shape[0], 256).cpu().numpy()
        assert np.array_equal(bits(out), bits(g[name + "_dequant"])), name


@pytest.mark.parametrize("t", [F.Q8_0, F.Q4_K, F.Q6_K])
def test_dequant_random_bit_exact(ftc, oracle, t):
    w = S.weight(t, 64, 4096, seed=11)
    out = ftc.dequant(dev(w), t, 64, 4096).cpu().numpy()
    assert np.array_equal(bits(out), bits(oracle.dequant_rows(w, t, 4096)))


# ------------------------------------------- fast decoders, bit for bit

@pytest.mark.parametrize("t,k", [(F.Q4_K, 4096), (F.Q4_K, 14336), (F.Q8_0, 4096),
                                 (F.Q6_K, 4096)])
def test_fast_path_one_hot_columns_exact(ftc, oracle, t, k):
    """x = one-hot rows: y[m][n] is exactly W[n][k_m], so the fast kernels'
    in-register decoders must reproduce the dequantized column."""
    n = 96
    w = S.weight(t, n, k, seed=5)
    deq = oracle.dequant_rows(w, t, k)
    rng = np.random.default_rng(0)
    picks = np.concatenate([np.arange(0, 256, 17), rng.integers(0, k, 40)])
    for s in range(0, len(picks), 8):
        ks = picks[s:s + 8]
        x = np.zeros((len(ks), k), dtype=np.float32)
        x[np.arange(len(ks)), ks] = 1.0
        y = run_gemv(ftc, w, t, n, k, x)
        assert np.array_equal(y, deq[:, ks].T), f"k positions {ks}"


@pytest.mark.parametrize("k", [4096, 14336, 2560])
def test_q4_k_batch1_one_hot_exact(ftc, oracle, k):
    """Batch 1 takes the dp4a kernel (activations as exact 24-bit integers with
    power-of-two block scales): one-hot inputs must still give the dequantized
    column exactly."""
    n = 40
    w = S.weight(F.Q4_K, n, k, seed=6)
    deq = oracle.dequant_rows(w, F.Q4_K, k)
    rng = np.random.default_rng(1)
    for kk in np.concatenate([np.arange(0, 256, 9), rng.integers(0, k, 12)]):
        x = np.zeros((1, k), dtype=np.float32)
        x[0, kk] = 1.0
        y = run_gemv(ftc, w, F.Q4_K, n, k, x)[0]
        assert np.array_equal(y, deq[:, kk]), f"k={kk}"


@pytest.mark.parametrize("t,k", [(F.Q6_K, 4096), (F.Q6_K, 2048), (F.Q6_K, 6144),
                                 (F.Q8_0, 4096), (F.Q8_0, 2048), (F.Q8_0, 6144)])
def test_kq_batch1_one_hot_exact(ftc, oracle, t, k):
    """Batch-1 Q6_K and Q8_0 take the same dp4a kernel (signed codes as bytes;
    Q6_K's int8 scales per 16 weights, Q8_0's fp16 scale per 32): one-hot
    inputs give the dequantized column exactly, every position of a 256-weight
    stretch included."""
    n = 40
    w = S.weight(t, n, k, seed=16)
    deq = oracle.dequant_rows(w, t, k)
    rng = np.random.default_rng(2)
    for kk in np.concatenate([np.arange(0, 256, 5), rng.integers(0, k, 12)]):
        x = np.zeros((1, k), dtype=np.float32)
        x[0, kk] = 1.0
        y = run_gemv(ftc, w, t, n, k, x)[0]
        assert np.array_equal(y, deq[:, kk]), f"k={kk}"


@pytest.mark.parametrize("t", [F.Q6_K, F.Q8_0])
@pytest.mark.parametrize("n", [1, 7, 13, 300, 4099])
def test_kq_batch1_row_counts(ftc, oracle, t, n):
    """Row counts that leave partial chunks and idle CTAs, Q6_K and Q8_0 at
    batch 1."""
    k = 4096
    w = S.weight(t, n, k, seed=18)
    x = S.activations_f32(1, k, seed=18) * np.float32(3.0)
    assert rel_err(run_gemv(ftc, w, t, n, k, x), oracle.matmul(x, w, t, k)) <= TOL
    assert ftc.device_status() == 0


@pytest.mark.parametrize("n", [1, 7, 13, 300, 4099])
def test_q4_k_batch1_row_counts(ftc, oracle, n):
    """Row counts that leave partial chunks and idle CTAs."""
    k = 4096
    w = S.weight(F.Q4_K, n, k, seed=8)
    x = S.activations_f32(1, k, seed=8) * np.float32(3.0)
    assert rel_err(run_gemv(ftc, w, F.Q4_K, n, k, x), oracle.matmul(x, w, F.Q4_K, k)) <= TOL
    assert ftc.device_status() == 0


@pytest.mark.parametrize("ns,k", [((4096, 1024, 1024), 4096), ((14336, 14336), 4096),
                                  ((7, 300, 1), 2560), ((4096, 4096), 14336)])
def test_grouped_gemv_equals_single(ftc, oracle, ns, k):
    """q/k/v- and gate/up-style groups in one launch give each matrix exactly
    its single-launch result."""
    ws = [S.weight(F.Q4_K, n, k, seed=i, name=f"grp.{i}") for i, n in enumerate(ns)]
    x = S.activations_f32(1, k, seed=5, name="grp")
    xd = dev(x)
    wd = [dev(w) for w in ws]
    ys = ftc.mul_mat_vec_multi(wd, F.Q4_K, list(ns), k, xd)
    singles = [ftc.mul_mat_vec(w, F.Q4_K, n, k, xd) for w, n in zip(wd, ns)]
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
    for w, y, y1 in zip(ws, ys, singles):
        assert torch.equal(y, y1)
        assert rel_err(y.cpu().numpy(), oracle.matmul(x, w, F.Q4_K, k, threads=THREADS)) <= TOL


# ------------------------------------------------ config shapes, full size

CONFIG2 = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)]


@pytest.mark.parametrize("n,k", CONFIG2)
@pytest.mark.parametrize("m", [1, 4, 8])
def test_q4_k_gemv_config2(ftc, oracle, n, k, m):
    w = S.weight(F.Q4_K, n, k, seed=0, name=f"c2.{n}x{k}")
    x = S.activations_f32(m, k, seed=0, name=f"c2.{m}")
    y = run_gemv(ftc, w, F.Q4_K, n, k, x)
    ref = oracle.matmul(x, w, F.Q4_K, k, threads=THREADS)
    assert rel_err(y, ref) <= TOL


def test_q8_0_gemv_config1_vs_reference(ftc, oracle):
    """Config 1 against the reference's own CpuBackend::matmul (M=1)."""
    n = k = 4096
    w = S.weight(F.Q8_0, n, k, seed=0, name="c1")
    x = S.activations_f32(1, k, seed=0, name="c1")
    y = run_gemv(ftc, w, F.Q8_0, n, k, x)[0]
    ref = oracle.ref_matmul(x, w, F.Q8_0, k, threads=THREADS) if oracle.have_ref() else \
        oracle.matmul(x, w, F.Q8_0, k, threads=THREADS)[0]
    assert rel_err(y, ref) <= TOL
    for m in (4, 8):
        xm = S.activations_f32(m, k, seed=1, name="c1")
        assert rel_err(run_gemv(ftc, w, F.Q8_0, n, k, xm),
                       oracle.matmul(xm, w, F.Q8_0, k, threads=THREADS)) <= TOL


def test_q8_0_golden_reference_outputs(ftc, golden):
    g = golden("ref_q8_0_gemv.npz")
    for tag, k in (("k4096", 4096), ("k96", 96), ("k2080", 2080)):
        w, x = g[f"{tag}_w"], g[f"{tag}_x"]
        y = run_gemv(ftc, w, F.Q8_0, w.shape[0], k, x[:1])[0]
        assert rel_err(y, g[f"{tag}_matmul_m1"]) <= TOL, tag


def test_q6_k_head_full_size(ftc, oracle):
    n, k = 128256, 4096
    w = S.weight(F.Q6_K, n, k, seed=0, name="head")
    x = S.activations_f32(1, k, seed=0, name="head")
    y = run_gemv(ftc, w, F.Q6_K, n, k, x)
    ref = oracle.matmul(x, w, F.Q6_K, k, threads=THREADS)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("m", [2, 4, 8])
def test_q6_k_batched(ftc, oracle, m):
    n, k = 2048, 4096
    w = S.weight(F.Q6_K, n, k, seed=2, name="q6b")
    x = S.activations_f32(m, k, seed=2)
    assert rel_err(run_gemv(ftc, w, F.Q6_K, n, k, x),
                   oracle.matmul(x, w, F.Q6_K, k, threads=THREADS)) <= TOL


# ---------------------------------------------------- ragged and generic

@pytest.mark.parametrize("t,k", [(F.Q4_K, 256), (F.Q4_K, 768), (F.Q4_K, 2560), (F.Q8_0, 96),
                                 (F.Q8_0, 2080), (F.Q6_K, 768), (F.Q6_K, 256)])
@pytest.mark.parametrize("m", [1, 3, 5, 6, 7])
def test_ragged_shapes(ftc, oracle, t, k, m):
    n = 77
    w = S.weight(t, n, k, seed=9)
    x = S.activations_f32(m, k, seed=9)
    assert rel_err(run_gemv(ftc, w, t, n, k, x), oracle.matmul(x, w, t, k)) <= TOL


@pytest.mark.parametrize("t", [F.Q4_K, F.Q8_0, F.Q6_K])
def test_unaligned_weights_take_generic_path(ftc, oracle, t):
    """A weight pointer 2 bytes off a 16-byte boundary and a padded row
    stride must still give the right answer (element-wise kernel)."""
    n, k = 50, 2048
    w = S.weight(t, n, k, seed=4)
    rb = w.shape[1]
    stride = rb + 6
    buf = np.zeros(2 + n * stride, dtype=np.uint8)
    for r in range(n):
        buf[2 + r * stride: 2 + r * stride + rb] = w[r]
    x = S.activations_f32(2, k, seed=4)
    d = dev(buf)
    y = ftc.mul_mat_vec(d[2:], t, n, k, dev(x), row_stride=stride)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), oracle.matmul(x, w, t, k)) <= TOL


@pytest.mark.parametrize("t", [F.F32, F.F16, F.BF16, F.Q4_0, F.Q4_1])
def test_other_formats(ftc, oracle, t):
    n, k = 33, 512
    g = np.random.default_rng(t)
    eb, bb = F.BLOCK[t]
    w = g.integers(0, 256, size=(n, k // eb * bb), dtype=np.uint8)
    if t in (F.F32,):
        w = g.standard_normal((n, k), dtype=np.float32).view(np.uint8)
    elif t == F.F16:
        w = g.standard_normal((n, k)).astype(np.float16).view(np.uint8)
    elif t == F.BF16:
        w = S.f32_to_bf16_bits(g.standard_normal((n, k)).astype(np.float32)).view(np.uint8)
    else:  # sane fp16 scale fields
        w = w.reshape(n, k // eb, bb)
        w[:, :, 0:2] = np.array([0x2E66], dtype=np.uint16).view(np.uint8)
        if t == F.Q4_1:
            w[:, :, 2:4] = np.array([0x2A66], dtype=np.uint16).view(np.uint8)
        w = w.reshape(n, -1)
    x = S.activations_f32(3, k, seed=1)
    assert rel_err(run_gemv(ftc, w, t, n, k, x), oracle.matmul(x, w, t, k)) <= TOL
    out = ftc.dequant(dev(w), t, n, k).cpu().numpy()
    assert np.array_equal(bits(out), bits(oracle.dequant_rows(w, t, k)))


def test_kquant_edge_blocks_through_fast_path(ftc, oracle, golden):
    g = golden("gguf_kquant.npz")
    for name, t in (("q4_k", F.Q4_K), ("q6_k", F.Q6_K)):
        blocks = g[name + "_blocks"]
        nb = blocks.shape[0]
        # rows of 16 blocks (16-byte aligned for both formats), edge blocks
        # cycled into every position
        rows = np.stack([np.concatenate([blocks[(r + j) % nb] for j in range(16)])
                         for r in range(nb)])
        k = 16 * 256
        x = S.activations_f32(1, k, seed=7)
        y = run_gemv(ftc, rows, t, nb, k, x)
        ref = oracle.matmul(x, rows, t, k)
        assert rel_err(y, ref) <= TOL, name
