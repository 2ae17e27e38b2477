"""ftc_backend_matmul's graph replay (the default; FTC_BACKEND_GRAPHS=0 at
creation turns it off): each (weight, shape) call is captured once and
replayed as a CUDA graph.  The replayed work is the
same kernels on the same buffers, so every output must equal the direct
path's bit for bit: repeated calls (replays), a new shape, a larger call that
moves the staging buffers (all graphs dropped and captured again), and a
call after the weight was evicted (copied for that call, not replayed).
Graphs are kept for uploaded weights only.  Runs late in the suite."""
import numpy as np
import pytest

from xwfes_b200 import formats as F, synth as S

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ftc():
    assert torch.cuda.is_available(), "GPU test needs CUDA"
    from xwfes_b200 import ftc as mod
    mod.lib()
    return mod


def backend(ftc, monkeypatch, graphs):
    if graphs:
        monkeypatch.delenv("FTC_BACKEND_GRAPHS", raising=False)
    else:
        monkeypatch.setenv("FTC_BACKEND_GRAPHS", "0")
    return ftc.CudaBackend(0)


def test_graph_replays_equal_direct_calls(ftc, monkeypatch):
    k = 4096
    Ws = [ftc.HostTensor(S.weight(F.Q4_K, n, k, seed=i, name=f"bg.{i}"), F.Q4_K, (k, n))
          for i, n in enumerate((4096, 1024, 14336))]
    W8 = ftc.HostTensor(S.weight(F.Q8_0, 512, k, seed=9, name="bg.q8"), F.Q8_0, (k, 512))
    calls = [(0, 1), (1, 1), (0, 1), (2, 1), (0, 4), (0, 1), (2, 8), (2, 3)]
    outs = {}
    for graphs in (False, True):
        be = backend(ftc, monkeypatch, graphs)
        try:
            for W in Ws + [W8]:
                be.upload(W)
            got = []
            for rep in range(2):
                for wi, m in calls:
                    W = Ws[wi]
                    x = S.activations_f32(m, k, seed=10 * wi + m + rep, name="bg.x")
                    y = np.full((m, W.rows()), np.nan, dtype=np.float32)
                    be.matmul(x, m, k, W, y)
                    got.append(y)
                x = S.activations_f32(8, k, seed=rep, name="bg.x8")
                y = np.empty((8, 512), dtype=np.float32)
                be.matmul(x, 8, k, W8, y)
                got.append(y)
            # a larger call (16 rows: the tensor-core path) moves the staging
            # buffers; then an earlier shape again, captured anew
            x = S.activations_f32(16, k, seed=5, name="bg.big")
            y = np.empty((16, 14336), dtype=np.float32)
            be.matmul(x, 16, k, Ws[2], y)
            got.append(y)
            x = S.activations_f32(1, k, seed=7, name="bg.again")
            y = np.empty((1, 4096), dtype=np.float32)
            be.matmul(x, 1, k, Ws[0], y)
            got.append(y)
            be.evict(Ws[0])
            x = S.activations_f32(1, k, seed=6, name="bg.ev")
            y = np.empty((1, 4096), dtype=np.float32)
            be.matmul(x, 1, k, Ws[0], y)
            got.append(y)
            outs[graphs] = got
        finally:
            be.close()
    for a, b in zip(outs[False], outs[True]):
        assert np.array_equal(a, b)
