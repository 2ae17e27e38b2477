"""MatmulSequence: a decode step's list of ftc_backend_matmul calls replayed
from native code (xwfes_b200/host/call_loop.c).  It runs the same C ABI
calls as CudaBackend.matmul, so every output must equal a per-call Python
loop's bit for bit, on every repetition, and match the CPU oracle's
restatement of CpuBackend::matmul (ft/src/cpu_backend.cpp:90-104, per row)
within the GEMV tolerance.  Runs late in the suite."""
import os

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


def rel_err(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(y - ref) / (np.abs(ref) + 1e-2 * rms)))


def test_sequence_equals_per_call_loop(ftc, oracle):
    shapes = [(F.Q4_K, 4096, 4096, 1), (F.Q4_K, 1024, 4096, 1), (F.Q4_K, 4096, 14336, 1),
              (F.Q8_0, 512, 4096, 1), (F.Q4_K, 1024, 4096, 3), (F.Q6_K, 256, 4096, 2)]
    be = ftc.CudaBackend(0)
    try:
        Ws, xs = [], []
        for i, (t, n, k, m) in enumerate(shapes):
            W = ftc.HostTensor(S.weight(t, n, k, seed=i, name=f"cl.{i}"), t, (k, n))
            if i != 3:  # one weight left un-uploaded: copied for each call
                be.upload(W)
            Ws.append(W)
            xs.append(S.activations_f32(m, k, seed=i, name="cl.x"))
        ys = [np.full((m, n), np.nan, dtype=np.float32) for (_, n, _, m) in shapes]
        seq = be.matmul_sequence([(xs[i], shapes[i][3], shapes[i][2], Ws[i], ys[i])
                                  for i in range(len(shapes))])
        want = []
        for i, (t, n, k, m) in enumerate(shapes):
            y = np.empty((m, n), dtype=np.float32)
            be.matmul(xs[i], m, k, Ws[i], y)
            want.append(y)
        for rep in range(3):
            for y in ys:
                y.fill(np.nan)
            seq.run(1 + rep)  # 1, 2 and 3 passes over the list
            for i in range(len(shapes)):
                assert np.array_equal(ys[i].view(np.uint32), want[i].view(np.uint32)), (rep, i)
        thr = os.cpu_count() or 8
        for i, (t, n, k, m) in enumerate(shapes):
            ref = oracle.matmul(xs[i], Ws[i].data, t, k, threads=thr)
            assert rel_err(ys[i], ref) <= 2e-3, (F.NAMES[t], n, k, m)
    finally:
        be.close()
