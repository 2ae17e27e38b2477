"""The reference-facing boundary on the GPU: the ft::IBackend mirror over the
ftc_backend_* C ABI, with host buffers in and out, read like the
reference's own tests (ft/src/tests/test_core.cpp:239-346)."""
import os

import numpy as np
import pytest

from xwfes_b200 import formats as F, synth as S

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 8


def rel_err(y, ref, floor_frac=1e-2):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(y - ref) / (np.abs(ref) + floor_frac * rms)))


@pytest.fixture(scope="module")
def be():
    from xwfes_b200 import ftc
    b = ftc.CudaBackend(0)
    yield b
    b.close()


def test_backend_metadata(be):
    info = be.info()
    assert be.ready()
    assert info["name"].startswith("CUDA:") and "B200" in info["name"]
    assert info["mem_bytes"] > 100 * 2**30 and not info["integrated"]


def test_matmul_q4_k_host_buffers(be, oracle):
    from xwfes_b200 import ftc
    n = k = 4096
    W = ftc.HostTensor(S.weight(F.Q4_K, n, k, seed=0, name="be"), F.Q4_K, (k, n))
    for m in (1, 3, 8, 11, 64, 257):
        x = S.activations_f32(m, k, seed=m)
        y = np.full((m, n), np.nan, dtype=np.float32)
        be.matmul(x, m, k, W, y)
        ref = oracle.matmul(x, W.data, F.Q4_K, k, threads=THREADS)
        if m <= 8:  # fp32 GEMV
            assert rel_err(y, ref) <= 2e-3
        else:  # tensor-core GEMM: fp16 operands, error relative to the largest output
            assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) <= 2e-3


def test_matmul_q8_0_vs_reference_cpu_backend(be, golden):
    """M=1 through the C ABI against the reference's CpuBackend::matmul output."""
    from xwfes_b200 import ftc
    g = golden("ref_q8_0_gemv.npz")
    for tag, k in (("k4096", 4096), ("k96", 96), ("k2080", 2080)):
        w = g[f"{tag}_w"]
        W = ftc.HostTensor(w, F.Q8_0, (k, w.shape[0]))
        y = np.zeros((1, w.shape[0]), dtype=np.float32)
        be.matmul(g[f"{tag}_x"][:1].copy(), 1, k, W, y)
        assert rel_err(y[0], g[f"{tag}_matmul_m1"]) <= 2e-3, tag


def test_weight_cache_upload_once(be):
    from xwfes_b200 import ftc
    n, k = 512, 4096
    W = ftc.HostTensor(S.weight(F.Q4_K, n, k, seed=3), F.Q4_K, (k, n))
    be.upload(W)
    before = be.cached_bytes()
    assert be.device_ptr(W) is not None
    x = S.activations_f32(1, k, seed=3)
    y = np.zeros((1, n), dtype=np.float32)
    be.matmul(x, 1, k, W, y)
    be.upload(W)  # same range again: no-op
    assert be.cached_bytes() == before
    be.evict(W)
    assert be.cached_bytes() == before - W.nbytes
    assert be.device_ptr(W) is None


def test_reused_host_buffer_is_not_served_stale(be, oracle):
    """A weight that was never uploaded is copied per call: rewriting the
    same host buffer (same address, new blocks, even a different format)
    between calls must change the result.  An implicit address-keyed cache
    returned the first weight's device copy here."""
    from xwfes_b200 import ftc
    n, k, m = 512, 4096, 3
    buf = np.zeros(ftc.row_bytes(F.Q4_K, k) * 2 * n, dtype=np.uint8)
    x = S.activations_f32(m, k, seed=7)
    cases = ((F.Q4_K, 2 * n, 1), (F.Q4_K, 2 * n, 2), (F.Q8_0, n, 3), (F.Q6_K, n, 4))
    for t, rows, seed in cases:
        w = S.weight(t, rows, k, seed=seed, name="reuse")
        buf[:w.size] = w.reshape(-1)
        W = ftc.HostTensor(buf[:w.size].reshape(w.shape), t, (k, rows))
        assert W.ptr() == buf.ctypes.data
        y = np.full((m, rows), np.nan, dtype=np.float32)
        be.matmul(x, m, k, W, y)
        ref = oracle.matmul(x, w, t, k, threads=THREADS)
        assert rel_err(y, ref) <= 2e-3, F.NAMES[t]
    assert be.device_ptr(ftc.HostTensor(buf, F.Q8_0, (k, n))) is None  # nothing cached


def test_expert_chunk_reference_chunker_case(be, golden):
    """ft/src/tests/test_core.cpp:307-346 shapes (F32, K=16, FF=48, M=3,
    windows of 8) against the reference's run_expert_chunk outputs, with
    that test's own bound: |d| / (|ref| + 1e-3) < 1e-4."""
    g = golden("ref_chunker_f32.npz")
    K, C = 16, int(g["window"])
    gate, up, down = (np.ascontiguousarray(g[n]) for n in ("gate", "up", "down"))
    out = np.zeros((3, K), dtype=np.float32)
    stride = K * 4
    for i0 in range(0, 48, C):
        be.run_expert_chunk(g["x"], out, gate.ctypes.data + stride * i0,
                            up.ctypes.data + stride * i0, down.ctypes.data + stride * i0,
                            F.F32, 3, K, C, stride, stride)
    ref = g["out"]
    assert np.max(np.abs(out - ref) / (np.abs(ref) + 1e-3)) < 1e-4


def test_expert_chunk_q8_0_vs_reference(be, golden):
    g = golden("ref_expert_q8_0.npz")
    out = g["out_in"].copy()
    gate, up, down = (np.ascontiguousarray(g[n]) for n in ("gate", "up", "down"))
    be.run_expert_chunk(g["x"], out, gate.ctypes.data, up.ctypes.data, down.ctypes.data,
                        F.Q8_0, 3, 256, 64, gate.shape[1], down.shape[1])
    assert rel_err(out, g["out"]) <= 2e-3


def test_expert_chunk_cached_windows(be, oracle):
    """Windows inside an uploaded expert tensor are used in place."""
    from xwfes_b200 import ftc
    K, FF, M, C = 4096, 512, 4, 128
    t = F.Q4_K
    gate = ftc.HostTensor(S.weight(t, FF, K, seed=1, name="g"), t, (K, FF))
    up = ftc.HostTensor(S.weight(t, FF, K, seed=1, name="u"), t, (K, FF))
    down = ftc.HostTensor(S.weight(t, FF, K, seed=1, name="d"), t, (K, FF))
    for T in (gate, up, down):
        be.upload(T)
    x = S.activations_f32(M, K, seed=1)
    out = np.zeros((M, K), dtype=np.float32)
    ref = np.zeros((M, K), dtype=np.float32)
    rs = gate.row_stride_bytes()
    for i0 in range(0, FF, C):
        be.run_expert_chunk(x, out, gate.ptr(rs * i0), up.ptr(rs * i0), down.ptr(rs * i0),
                            t, M, K, C, rs, rs)
        oracle.expert_chunk(x, ref, gate.data[i0:i0 + C], up.data[i0:i0 + C],
                            down.data[i0:i0 + C], t, K, C, threads=THREADS)
    assert rel_err(out, ref) <= 2e-3


def test_errors_raise_like_the_reference(be, monkeypatch):
    from xwfes_b200 import ftc
    W = ftc.HostTensor(S.weight(F.Q4_K, 8, 256, seed=0), F.Q4_K, (256, 8))
    x = np.zeros((1, 300), dtype=np.float32)
    y = np.zeros((1, 8), dtype=np.float32)
    with pytest.raises(ftc.FtcError) as e:
        be.matmul(x, 1, 300, ftc.HostTensor(np.zeros(8 * 2 * 144, np.uint8), F.Q4_K, (300, 8)), y)
    assert e.value.rc == -1
    monkeypatch.setenv("FTC_INJECT_FAIL", "ftc_backend_matmul")
    with pytest.raises(ftc.FtcError) as e:
        be.matmul(np.zeros((1, 256), np.float32), 1, 256, W, y)
    assert e.value.rc == -5
    monkeypatch.delenv("FTC_INJECT_FAIL")
    be.matmul(np.zeros((1, 256), np.float32), 1, 256, W, y)  # usable afterwards
    assert np.all(y == 0)
