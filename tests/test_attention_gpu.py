"""Attention and RoPE on the GPU against the oracle's restatement of the
engine's code (ft/src/engine.cpp:137-177 attn, 43-60 rope_vec; the oracle is
pinned bit for bit to the reference in tests/test_oracle_attention.py).

Attention sums in a different order than the reference (splits, fused
multiply-adds), so outputs are compared with north_star's float bound (2e-3,
element-wise relative with a floor of 1e-2 of the output's rms) and, tighter,
normwise within 5e-5 (fp32 summation noise; outputs that average thousands
of V rows come out near zero, where the element-wise figure inflates); RoPE
uses the reference's double-precision
angles and separately rounded float products, so it is compared to within
one float rounding (almost every value is identical)."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

THR = os.cpu_count() or 8


@pytest.fixture(scope="module")
def ftc():
    assert torch.cuda.is_available(), "GPU test needs CUDA"
    from xwfes_b200 import ftc as mod
    mod.lib()
    return mod


def rel_err(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(y - ref) / (np.abs(ref) + 1e-2 * rms)))


def close(y, ref):
    """north_star's element bound and a normwise fp32-noise bound."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    norm = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    return rel_err(y, ref) <= 2e-3 and norm <= 5e-5


def inputs(M, nh, nkv, hd, base, seed, stride=None):
    rng = np.random.default_rng(seed)
    dk = nkv * hd
    ks = stride or dk
    q = rng.standard_normal((M, nh * hd), dtype=np.float32)
    kc = rng.standard_normal((base + M, ks), dtype=np.float32)
    vc = rng.standard_normal((base + M, ks), dtype=np.float32)
    return q, kc, vc


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("M,nh,nkv,hd,base", [
    (1, 32, 8, 128, 0), (1, 32, 8, 128, 31), (1, 32, 8, 128, 64), (1, 32, 8, 128, 4095),
    (1, 64, 8, 128, 1000), (1, 8, 8, 64, 200), (1, 12, 4, 64, 77), (1, 16, 2, 256, 300),
    (17, 32, 8, 128, 40), (64, 8, 2, 64, 0), (3, 12, 4, 128, 2049),
])
def test_attention_matches_oracle(ftc, oracle, M, nh, nkv, hd, base):
    """Block rows in the cache itself (the engine's write_kv path): K/V rows
    [0, base + M) of one buffer, the block at row base."""
    q, kc, vc = inputs(M, nh, nkv, hd, base, seed=M * 7919 + base)
    dkc, dvc = dev(kc), dev(vc)
    got = ftc.attention(dev(q), nh, nkv, hd, dkc[base:], dvc[base:], base=base, k_cache=dkc,
                        v_cache=dvc)
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
    want = oracle.attention(q, nh, nkv, hd, kc[:base], vc[:base], base, kc[base:], vc[base:],
                            threads=THR)
    assert close(got.cpu().numpy(), want)


def test_attention_separate_block_and_padded_rows(ftc, oracle):
    """Block rows in their own buffer (the engine's no-write path) and K/V
    rows with a pitch above n_head_kv * head_dim."""
    M, nh, nkv, hd, base, stride = 5, 32, 8, 128, 300, 1024 + 64
    q, kc, vc = inputs(M, nh, nkv, hd, base, seed=11, stride=stride)
    rng = np.random.default_rng(12)
    kb = rng.standard_normal((M, stride), dtype=np.float32)
    vb = rng.standard_normal((M, stride), dtype=np.float32)
    got = ftc.attention(dev(q), nh, nkv, hd, dev(kb), dev(vb), base=base, k_cache=dev(kc[:base]),
                        v_cache=dev(vc[:base]), kv_stride=stride)
    torch.cuda.synchronize()
    dk = nkv * hd
    want = oracle.attention(q, nh, nkv, hd, kc[:base, :dk], vc[:base, :dk], base, kb[:, :dk],
                            vb[:, :dk], threads=THR)
    assert close(got.cpu().numpy(), want)


def test_attention_peaked_scores(ftc, oracle):
    """Large scores: most softmax weights underflow to zero."""
    M, nh, nkv, hd, base = 2, 8, 2, 64, 700
    q, kc, vc = inputs(M, nh, nkv, hd, base, seed=3)
    q *= 30.0
    dkc, dvc = dev(kc), dev(vc)
    got = ftc.attention(dev(q), nh, nkv, hd, dkc[base:], dvc[base:], base=base, k_cache=dkc,
                        v_cache=dvc)
    torch.cuda.synchronize()
    want = oracle.attention(q, nh, nkv, hd, kc[:base], vc[:base], base, kc[base:], vc[base:])
    assert close(got.cpu().numpy(), want)


def test_attention_graph_replay_is_deterministic(ftc):
    M, nh, nkv, hd, base = 1, 32, 8, 128, 3000
    q, kc, vc = inputs(M, nh, nkv, hd, base, seed=5)
    dq, dkc, dvc = dev(q), dev(kc), dev(vc)
    outs = []
    for _ in range(3):
        outs.append(ftc.attention(dq, nh, nkv, hd, dkc[base:], dvc[base:], base=base,
                                  k_cache=dkc, v_cache=dvc).cpu().numpy())
    assert all(np.array_equal(o.view(np.uint32), outs[0].view(np.uint32)) for o in outs)


def test_attention_rejects_bad_shapes(ftc):
    x = torch.zeros(4096, dtype=torch.float32, device="cuda")
    p = x.data_ptr()
    L = ftc.lib()
    assert L.ftc_attention(p, 1, 32, 8, 96, p, p, 768, 4, p, p, p, None, 0, None) != 0
    assert "head_dim" in ftc.last_error()
    assert L.ftc_attention(p, 1, 30, 8, 128, p, p, 1024, 4, p, p, p, None, 0, None) != 0
    assert L.ftc_attention(p, 1, 32, 8, 128, p, p, 1000, 4, p, p, p, None, 0, None) != 0
    assert "kv_stride" in ftc.last_error()
    assert L.ftc_attention(p + 4, 1, 32, 8, 128, p, p, 1024, 4, p, p, p, None, 0, None) != 0
    assert "aligned" in ftc.last_error()
    need = L.ftc_attention_workspace_bytes(1, 32, 8, 128, 4000)
    assert need > 0
    assert L.ftc_attention(p, 1, 32, 8, 128, p, p, 1024, 4000, p, p, p, None, 0, None) != 0
    assert "workspace" in ftc.last_error()
    assert ftc.device_status() == 0  # nothing was launched


@pytest.mark.parametrize("neox", [False, True])
def test_rope_matches_oracle(ftc, oracle, neox):
    rng = np.random.default_rng(9)
    M, heads, hd, base, theta = 33, 8, 128, 65519, 500000.0
    x = rng.standard_normal((M, heads * hd), dtype=np.float32)
    got = ftc.rope(dev(x), heads, hd, base, theta, neox).cpu().numpy()
    want = oracle.rope(x, heads, hd, base, theta, neox)
    diff = np.abs(got.astype(np.float64) - want)
    assert np.mean(got == want) >= 0.999
    assert diff.max() <= 4e-7 * np.abs(want).max()


def test_backend_kv_cache_decode_sequence(ftc, oracle):
    """ftc_backend_kv_alloc + ftc_backend_attention as the engine uses them:
    a prefill block written into the device cache, then decode steps, each
    attending everything written so far; a call without write_kv uses its
    block once and leaves the cache as it was."""
    nh, nkv, hd, L = 32, 8, 128, 2
    dk = nkv * hd
    be = ftc.CudaBackend(0)
    try:
        be.kv_alloc(L, 256, dk)
        rng = np.random.default_rng(21)
        cache_k = {l: np.zeros((0, dk), np.float32) for l in range(L)}
        cache_v = {l: np.zeros((0, dk), np.float32) for l in range(L)}
        base = 0
        for M in (7, 1, 1, 3, 1):
            for layer in range(L):
                q = rng.standard_normal((M, nh * hd), dtype=np.float32)
                kn = rng.standard_normal((M, dk), dtype=np.float32)
                vn = rng.standard_normal((M, dk), dtype=np.float32)
                # a look-ahead without writing: the cache must not change
                qa = rng.standard_normal((1, nh * hd), dtype=np.float32)
                ka = rng.standard_normal((1, dk), dtype=np.float32)
                va = rng.standard_normal((1, dk), dtype=np.float32)
                got_a = be.attention(layer, base, qa, ka, va, nh, nkv, hd, write_kv=False)
                want_a = oracle.attention(qa, nh, nkv, hd, cache_k[layer], cache_v[layer], base,
                                          ka, va, threads=THR)
                assert close(got_a, want_a)
                got = be.attention(layer, base, q, kn, vn, nh, nkv, hd, write_kv=True)
                want = oracle.attention(q, nh, nkv, hd, cache_k[layer], cache_v[layer], base, kn,
                                        vn, threads=THR)
                assert close(got, want), (layer, base, M)
                cache_k[layer] = np.concatenate([cache_k[layer], kn])
                cache_v[layer] = np.concatenate([cache_v[layer], vn])
            base += M
        with pytest.raises(ftc.FtcError):  # beyond the capacity
            be.attention(0, 256, np.zeros((1, nh * hd), np.float32), np.zeros((1, dk), np.float32),
                         np.zeros((1, dk), np.float32), nh, nkv, hd)
        with pytest.raises(ftc.FtcError):  # another head layout than the cache's
            be.attention(0, base, np.zeros((1, 16 * hd), np.float32),
                         np.zeros((1, 4 * hd), np.float32), np.zeros((1, 4 * hd), np.float32),
                         16, 4, hd)
    finally:
        be.close()


def test_backend_kv_snapshot_and_restore(ftc, oracle):
    """ftc_backend_kv_read / kv_write as the engine's prefix cache uses them
    (ft/src/engine.cpp:605-645): rows written by attention calls read back
    bit for bit, a snapshot restored into a fresh cache serves the next
    attention call as if the prefix had been computed there."""
    nh, nkv, hd, L = 8, 2, 128, 2
    dk = nkv * hd
    rng = np.random.default_rng(31)
    a = ftc.CudaBackend(0)
    b = ftc.CudaBackend(0)
    try:
        a.kv_alloc(L, 64, dk)
        b.kv_alloc(L, 64, dk)
        M = 20
        ks = {l: rng.standard_normal((M, dk), dtype=np.float32) for l in range(L)}
        vs = {l: rng.standard_normal((M, dk), dtype=np.float32) for l in range(L)}
        for l in range(L):
            q = rng.standard_normal((M, nh * hd), dtype=np.float32)
            a.attention(l, 0, q, ks[l], vs[l], nh, nkv, hd, write_kv=True)
        snap = {l: a.kv_read(l, 0, M, dk) for l in range(L)}
        for l in range(L):
            assert np.array_equal(snap[l][0], ks[l]) and np.array_equal(snap[l][1], vs[l])
            b.kv_write(l, 0, *snap[l])
        for l in range(L):
            q = rng.standard_normal((1, nh * hd), dtype=np.float32)
            kn = rng.standard_normal((1, dk), dtype=np.float32)
            vn = rng.standard_normal((1, dk), dtype=np.float32)
            got = b.attention(l, M, q, kn, vn, nh, nkv, hd, write_kv=True)
            want = oracle.attention(q, nh, nkv, hd, ks[l], vs[l], M, kn, vn, threads=THR)
            assert close(got, want)
        with pytest.raises(ftc.FtcError):  # rows beyond the capacity
            b.kv_read(0, 60, 8, dk)
    finally:
        a.close()
        b.close()
