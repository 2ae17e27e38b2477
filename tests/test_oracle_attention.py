"""The oracle's restatement of the engine's attention and RoPE, pinned bit
for bit to the reference's own code (ft/src/engine.cpp:137-177 attn, 43-60
rope_vec), which oracle/Makefile compiles into _ref/libftref_engine.so."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.skipif(O.ref_engine() is None,
                                reason="_ref/libftref_engine.so not built (no reference tree)")


def case(M, nh, nkv, hd, base, seed):
    rng = np.random.default_rng(seed)
    dk = nkv * hd
    q = rng.standard_normal((M, nh * hd), dtype=np.float32)
    kc = rng.standard_normal((max(base, 1), dk), dtype=np.float32)
    vc = rng.standard_normal((max(base, 1), dk), dtype=np.float32)
    kb = rng.standard_normal((M, dk), dtype=np.float32)
    vb = rng.standard_normal((M, dk), dtype=np.float32)
    return q, kc, vc, kb, vb


def ref_attn(q, nh, nkv, hd, kc, vc, base, kb, vb, threads):
    R = O.ref_engine()
    out = np.empty_like(q)
    p = lambda a: a.ctypes.data_as(O._p)  # noqa: E731
    assert R.ftref_attn(p(q), q.shape[0], nh, nkv, hd, p(kc), p(vc), base, p(kb), p(vb), p(out),
                        threads) == 0
    return out


@pytest.mark.parametrize("M,nh,nkv,hd,base", [
    (1, 4, 4, 64, 0), (1, 8, 2, 128, 37), (1, 32, 8, 128, 300), (5, 8, 2, 64, 11),
    (16, 4, 1, 128, 0), (3, 6, 2, 32, 1000),
])
def test_attention_matches_reference(M, nh, nkv, hd, base):
    q, kc, vc, kb, vb = case(M, nh, nkv, hd, base, seed=M * 1000 + base)
    for threads in (1, 4):
        got = O.attention(q, nh, nkv, hd, kc, vc, base, kb, vb, threads=threads)
        want = ref_attn(q, nh, nkv, hd, kc, vc, base, kb, vb, threads)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_attention_peaked_scores_skip_zero_weights():
    """Scores far apart: most softmax weights underflow to zero and the
    reference skips those positions; the restatement does the same."""
    M, nh, nkv, hd, base = 2, 2, 1, 64, 50
    q, kc, vc, kb, vb = case(M, nh, nkv, hd, base, seed=7)
    q *= 40.0
    got = O.attention(q, nh, nkv, hd, kc, vc, base, kb, vb)
    want = ref_attn(q, nh, nkv, hd, kc, vc, base, kb, vb, 1)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("neox", [False, True])
@pytest.mark.parametrize("theta", [10000.0, 500000.0])
def test_rope_matches_reference(neox, theta):
    rng = np.random.default_rng(3)
    M, heads, hd, base = 4, 3, 128, 131067
    x = rng.standard_normal((M, heads * hd), dtype=np.float32)
    got = O.rope(x, heads, hd, base, theta, neox)
    want = x.copy()
    R = O.ref_engine()
    for m in range(M):
        for h in range(heads):
            row = want[m, h * hd:(h + 1) * hd]
            buf = np.ascontiguousarray(row)
            R.ftref_rope_vec(buf.ctypes.data_as(O._p), hd, base + m, theta, 1 if neox else 0)
            want[m, h * hd:(h + 1) * hd] = buf
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
