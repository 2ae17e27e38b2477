"""The device attention's algorithm (xwfes_b200/csrc/attention.cu) restated
in float32 numpy and checked on the CPU against the oracle's restatement of
Engine::Impl::attn (ft/src/engine.cpp:137-177): positions cut into splits of
whole 32-position chunks, per chunk the scores, an online softmax (running
maximum and sum, the accumulator rescaled by exp(old max - new max)) and the
weighted V sum, then the splits combined in split order with weights
exp(max_s - max).  Any split length must give the reference's result to fp32
summation noise, including splits whose every weight underflows."""
import numpy as np
import pytest

CHUNK = 32


def split_attention(q, kc, vc, base, kb, vb, nh, nkv, hd, L):
    """One row block through the split / chunk / combine scheme (float32)."""
    M = q.shape[0]
    gqa = nh // nkv
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    out = np.zeros((M, nh * hd), np.float32)
    K = np.concatenate([kc[:base], kb]) if base else kb
    V = np.concatenate([vc[:base], vb]) if base else vb
    for m in range(M):
        n_len = base + m + 1
        S = -(-n_len // L)
        for h in range(nh):
            kvh = h // gqa
            qv = q[m, h * hd:(h + 1) * hd]
            stats, parts = [], []
            for s in range(S):
                p0, p1 = s * L, min((s + 1) * L, n_len)
                mrun, lrun = np.float32(-np.inf), np.float32(0)
                acc = np.zeros(hd, np.float32)
                for c0 in range(p0, p1, CHUNK):
                    c1 = min(c0 + CHUNK, p1)
                    k = K[c0:c1, kvh * hd:(kvh + 1) * hd]
                    v = V[c0:c1, kvh * hd:(kvh + 1) * hd]
                    sc = (k @ qv).astype(np.float32) * scale
                    mn = np.float32(max(mrun, sc.max()))
                    e = np.exp(sc - mn).astype(np.float32)
                    al = np.float32(np.exp(mrun - mn)) if np.isfinite(mrun) else np.float32(0)
                    lrun = lrun * al + e.sum(dtype=np.float32)
                    acc = acc * al + (e[:, None] * v).sum(axis=0, dtype=np.float32)
                    mrun = mn
                stats.append((mrun, lrun))
                parts.append(acc)
            if S == 1:
                out[m, h * hd:(h + 1) * hd] = parts[0] / stats[0][1]
                continue
            mx = max(st[0] for st in stats)
            w = [np.float32(np.exp(st[0] - mx)) for st in stats]
            tot = np.float32(0)
            for st, ws in zip(stats, w):
                tot += st[1] * ws
            o = np.zeros(hd, np.float32)
            for pa, ws in zip(parts, w):
                o += pa * ws
            out[m, h * hd:(h + 1) * hd] = o / tot
    return out


def close(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return np.linalg.norm(y - ref) / np.linalg.norm(ref) <= 5e-5


@pytest.mark.parametrize("L", [32, 64, 96, 448])
@pytest.mark.parametrize("M,nh,nkv,hd,base", [(1, 8, 2, 64, 700), (5, 4, 4, 32, 61),
                                              (3, 6, 2, 64, 0)])
def test_split_scheme_matches_oracle(oracle, L, M, nh, nkv, hd, base):
    rng = np.random.default_rng(L + base)
    dk = nkv * hd
    q = rng.standard_normal((M, nh * hd), dtype=np.float32)
    kc = rng.standard_normal((max(base, 1), dk), dtype=np.float32)
    vc = rng.standard_normal((max(base, 1), dk), dtype=np.float32)
    kb = rng.standard_normal((M, dk), dtype=np.float32)
    vb = rng.standard_normal((M, dk), dtype=np.float32)
    got = split_attention(q, kc, vc, base, kb, vb, nh, nkv, hd, L)
    want = oracle.attention(q, nh, nkv, hd, kc[:base], vc[:base], base, kb, vb)
    assert close(got, want)


def test_splits_that_underflow_entirely(oracle):
    """One position dominates: every other split's weights underflow to zero
    (its maximum is far below the global one), so its combine weight is 0."""
    nh, nkv, hd, base, M = 2, 1, 64, 300, 1
    rng = np.random.default_rng(5)
    q = rng.standard_normal((M, nh * hd), dtype=np.float32)
    kc = rng.standard_normal((base, hd), dtype=np.float32) * np.float32(0.01)
    vc = rng.standard_normal((base, hd), dtype=np.float32)
    kc[137] = q[0, :hd] * np.float32(40.0)  # head 0 attends position 137 alone
    kb = rng.standard_normal((M, hd), dtype=np.float32) * np.float32(0.01)
    vb = rng.standard_normal((M, hd), dtype=np.float32)
    for L in (32, 64):
        got = split_attention(q, kc, vc, base, kb, vb, nh, nkv, hd, L)
        want = oracle.attention(q, nh, nkv, hd, kc, vc, base, kb, vb)
        assert close(got, want)
        assert np.allclose(got[0, :hd], vc[137], rtol=0, atol=1e-6)
