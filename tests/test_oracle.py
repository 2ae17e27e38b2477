"""The CPU oracle pinned against the reference's own outputs (golden fixtures
made by the reference's compiled CPU code) and, for Q4_K/Q6_K, against the
GGUF format's Python package.  No GPU."""
import numpy as np
import pytest

from xwfes_b200 import formats as F, synth as S


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("tag,k", [("k4096", 4096), ("k96", 96), ("k2080", 2080)])
def test_q8_0_matches_reference_bit_exact(golden, oracle, tag, k):
    g = golden("ref_q8_0_gemv.npz")
    w, x = g[f"{tag}_w"], g[f"{tag}_x"]
    assert np.array_equal(bits(oracle.dequant_rows(w, F.Q8_0, k)), bits(g[f"{tag}_dequant"]))
    dots = np.array([oracle.dot_row(x[0], w[r], F.Q8_0, k) for r in range(w.shape[0])],
                    dtype=np.float32)
    assert np.array_equal(bits(dots), bits(g[f"{tag}_dot"]))
    # CpuBackend::matmul at M=1 == per-row oracle, bit for bit
    y1 = oracle.matmul(x[:1], w, F.Q8_0, k, threads=2)
    assert np.array_equal(bits(y1.ravel()), bits(g[f"{tag}_matmul_m1"]))


def test_reference_matmul_row_sum_divergence(golden, oracle):
    """The reference folds M>1 rows into y[n]; the oracle keeps per-row
    outputs whose per-n sum (in the reference's order) reproduces it."""
    g = golden("ref_q8_0_gemv.npz")
    w, x = g["k4096_w"], g["k4096_x"]
    y = oracle.matmul(x, w, F.Q8_0, 4096)
    acc = y[0].copy()
    for m in range(1, 3):
        acc = (acc + y[m]).astype(np.float32)
    assert np.array_equal(bits(acc), bits(g["k4096_matmul_m3_rowsum"]))


def test_reference_test_quant_known_answer(golden, oracle):
    """ft/src/tests/test_core.cpp:239-293 rebuilt; the reference's dots are
    reproduced bit for bit and sit within the reference test's own bounds."""
    g = golden("ref_test_quant.npz")
    x = g["x"]
    for t, row, key, tol, floor in ((F.F16, "f16row", "dot_f16", 0.02, 1e-6),
                                     (F.Q8_0, "q8row", "dot_q8", 0.02, 1e-6),
                                     (F.Q4_0, "q4row", "dot_q4", 0.35, 1e-4)):
        d = np.float32(oracle.dot_row(x, g[row], t, 64))
        assert bits(d) == bits(g[key])
        assert abs(d - g["refdot"]) / (abs(g["refdot"]) + floor) < tol
    assert np.array_equal(bits(oracle.dequant_rows(g["q8row"][None], F.Q8_0, 64)[0]),
                          bits(g["dequant_q8"]))
    assert np.array_equal(bits(oracle.dequant_rows(g["q4row"][None], F.Q4_0, 64)[0]),
                          bits(g["dequant_q4"]))


def test_float_to_half_matches_reference_generator(golden, oracle):
    g = golden("ref_test_quant.npz")
    lib = oracle.lib()
    got = np.array([lib.ftor_float_to_half(float(v)) for v in g["ref"]], dtype=np.uint16)
    assert np.array_equal(got, g["f16row"].view(np.uint16))


def test_half_to_float_exhaustive(oracle):
    lib = oracle.lib()
    h = np.arange(65536, dtype=np.uint16)
    got = np.array([lib.ftor_half_to_float(int(v)) for v in h], dtype=np.float32)
    want = h.view(np.float16).astype(np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(bits(got[finite]), bits(want[finite]))
    assert np.all(np.isnan(got[~finite]) == np.isnan(want[~finite]))


def test_chunker_matches_reference(golden, oracle):
    g = golden("ref_chunker_f32.npz")
    x, K, C = g["x"], 16, int(g["window"])
    out = np.zeros_like(g["out"])
    for i0 in range(0, 48, C):
        oracle.expert_chunk(x, out, g["gate"][i0:i0 + C].view(np.uint8),
                            g["up"][i0:i0 + C].view(np.uint8),
                            g["down"][i0:i0 + C].view(np.uint8), F.F32, K, C)
    assert np.array_equal(bits(out), bits(g["out"]))
    # and the reference test's naive loop, within its 1e-4 bound (test_core.cpp:326-345)
    ref = np.zeros_like(out)
    for m in range(3):
        for i in range(48):
            gg = np.float32(np.dot(x[m].astype(np.float64), g["gate"][i]))
            uu = np.float32(np.dot(x[m].astype(np.float64), g["up"][i]))
            h = gg / (1 + np.exp(-gg)) * uu
            ref[m] += h * g["down"][i]
    assert np.max(np.abs(ref - out) / (np.abs(ref) + 1e-3)) < 1e-4


def test_expert_chunk_q8_0_matches_reference(golden, oracle):
    g = golden("ref_expert_q8_0.npz")
    out = g["out_in"].copy()
    oracle.expert_chunk(g["x"], out, g["gate"], g["up"], g["down"], F.Q8_0, 256, 64, threads=3)
    assert np.array_equal(bits(out), bits(g["out"]))


@pytest.mark.parametrize("name,t", [("q8_0", F.Q8_0), ("f16", F.F16), ("q4_0", F.Q4_0)])
def test_down_axpy_matches_reference(golden, oracle, name, t):
    """ft::matmul_down_axpy (transposed down rows, zero activations skipped,
    y accumulated) bit for bit, split over threads."""
    g = golden("ref_down_axpy.npz")
    y = g[name + "_y0"].copy()
    oracle.matmul_down_axpy(g[name + "_x"], g[name + "_w"], t, y.shape[1], y, threads=3)
    assert np.array_equal(bits(y), bits(g[name + "_y"]))


@pytest.mark.parametrize("t", [F.Q4_K, F.Q6_K])
def test_down_axpy_kquant_is_the_row_walk(oracle, t):
    """For the K-quants (no reference decoder) the oracle's down projection is
    the reference's loop over dequantized rows, restated in numpy."""
    n_in, n = 24, 512
    w = S.weight(t, n_in, n, seed=5, name="axpy.kq")
    x = S.activations_f32(2, n_in, seed=5, name="axpy.kq.x")
    x[0, 3] = 0.0
    y0 = S.activations_f32(2, n, seed=6, name="axpy.kq.y")
    deq = oracle.dequant_rows(w, t, n)
    ref = y0.copy()
    for i in range(n_in):
        for m in range(2):
            if x[m, i] != 0:
                ref[m] = ref[m] + x[m, i] * deq[i]
    got = oracle.matmul_down_axpy(x, w, t, n, y0.copy(), threads=2)
    assert np.array_equal(bits(got), bits(ref))


@pytest.mark.parametrize("name,t", [("f16", F.F16), ("bf16", F.BF16), ("q4_0", F.Q4_0),
                                    ("q4_1", F.Q4_1)])
def test_other_formats_match_reference(golden, oracle, name, t):
    g = golden("ref_dequant_formats.npz")
    assert np.array_equal(bits(oracle.dequant_rows(g[name + "_w"], t, 64)),
                          bits(g[name + "_dequant"]))


@pytest.mark.parametrize("name,t", [("q4_k", F.Q4_K), ("q6_k", F.Q6_K)])
def test_kquant_matches_gguf_py(golden, oracle, name, t):
    g = golden("gguf_kquant.npz")
    got = oracle.dequant_rows(g[name + "_blocks"], t, 256)
    assert np.array_equal(bits(got), bits(g[name + "_dequant"]))


@pytest.mark.parametrize("t", [F.Q4_K, F.Q6_K])
def test_kquant_dot_chunks_consistent(oracle, t):
    """dot_row_f32's 2048-chunk walk over K-quant rows equals a flat loop."""
    k = 4096
    w = S.weight(t, 2, k, seed=3)
    x = S.activations_f32(1, k, seed=3)[0]
    deq = oracle.dequant_rows(w, t, k)
    for r in range(2):
        acc = np.float32(0)
        for i in range(k):
            acc = np.float32(acc + np.float32(x[i] * deq[r, i]))
        assert bits(np.float32(oracle.dot_row(x, w[r], t, k))) == bits(acc)


def test_route_topk_semantics(oracle):
    logits = S.router_logits(64, 8, seed=0)
    idx, w = oracle.route_topk(logits, 2)
    p = np.exp(logits - logits.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    want = np.argsort(-p, axis=1, kind="stable")[:, :2]
    assert np.array_equal(idx, want)
    assert np.allclose(w.sum(1), 1.0, atol=1e-6)
    assert np.all(w[:, 0] >= w[:, 1])


def test_moe_ffn_equals_per_token_expert_sum(oracle):
    T, K, FF, E, U = 5, 256, 64, 4, 2
    t = F.Q8_0
    gate = S.expert_weights(t, E, FF, K, seed=0, name="g")
    up = S.expert_weights(t, E, FF, K, seed=0, name="u")
    down = S.expert_weights(t, E, K, FF, seed=0, name="d")
    x = S.activations_f32(T, K, seed=0)
    logits = S.router_logits(T, E, seed=0)
    out = oracle.moe_ffn(x, logits, gate, up, down, t, K, FF, U)
    idx, w = oracle.route_topk(logits, U)
    want = np.zeros_like(out)
    for m in range(T):
        for u in range(U):
            e = idx[m, u]
            acc = np.zeros((1, K), dtype=np.float32)
            oracle.expert_ffn(x[m:m + 1], acc, gate[e], up[e], down[e], t, K, FF)
            want[m] += w[m, u] * acc[0]
    assert np.allclose(out, want, rtol=1e-5, atol=1e-5)
