"""ftc_expert_chunk_static: the expert chunk for callers that cannot allocate
device memory (fixed-budget engines, code inside another component's stream
capture).  It must give the same result as the allocating entry point,
ftc_backend_run_expert_chunk, call after call, although both calls reuse the
library's one static scratch array; and both must match the CPU oracle's
restatement of the reference's CpuBackend::run_expert_chunk
(ft/src/cpu_backend.cpp:106-149), so a fault in the kernels they share
cannot pass unseen.

Kept in its own file, collected last, so that a failure here cannot stop a
`-x` run before the other tests have run; it also passes on its own in a
fresh process."""
import ctypes as C
import os

import numpy as np
import pytest

from xwfes_b200 import formats as F, synth as S

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MAX_HC = 65536  # FTC_EXPERT_STATIC_MAX_HC in include/ftc.h


def rel_err(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(y - ref) / (np.abs(ref) + 1e-2 * rms)))


@pytest.fixture(scope="module")
def ftc():
    assert torch.cuda.is_available()
    from xwfes_b200 import ftc as mod
    mod.lib()
    return mod


def run_static(ftc, t, x, out, gate, up, down, M, K, IC):
    """One call through the C ABI with device buffers; returns out (host)."""
    dev = torch.device("cuda", 0)
    dx = torch.from_numpy(x).to(dev)
    dout = torch.from_numpy(out.copy()).to(dev)
    dg, du, dd = (torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in (gate, up, down))
    rc = ftc.lib().ftc_expert_chunk_static(
        t, dx.data_ptr(), dout.data_ptr(), dg.data_ptr(), du.data_ptr(), dd.data_ptr(), M, K, IC,
        gate.shape[1], down.shape[1], C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, ftc.last_error()
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
    return dout.cpu().numpy()


def run_allocating(be, t, x, out, gate, up, down, M, K, IC):
    res = out.copy()
    be.run_expert_chunk(x, res, gate.ctypes.data, up.ctypes.data, down.ctypes.data, t, M, K, IC,
                        gate.shape[1], down.shape[1])
    return res


def case(t, M, K, IC, seed):
    gate = S.weight(t, IC, K, seed=seed, name="na.gate")
    up = S.weight(t, IC, K, seed=seed, name="na.up")
    down = S.weight(t, IC, K, seed=seed, name="na.down")  # neuron-major window
    x = S.activations_f32(M, K, seed=seed, name="na.x")
    out = S.activations_f32(M, K, seed=seed + 1, name="na.acc")  # accumulated into
    return x, out, gate, up, down


def test_static_scratch_matches_allocating_entry_point_twice(ftc, oracle):
    be = ftc.CudaBackend(0)
    try:
        # two calls in a row, different formats and sizes: the second must
        # not see anything the first left in the shared scratch array
        for t, M, K, IC, seed in ((F.Q4_K, 6, 4096, 512, 1), (F.Q8_0, 3, 2048, 96, 2)):
            x, out, gate, up, down = case(t, M, K, IC, seed)
            got = run_static(ftc, t, x, out, gate, up, down, M, K, IC)
            want = run_allocating(be, t, x, out, gate, up, down, M, K, IC)
            ref = out.copy()
            oracle.expert_chunk(x, ref, gate, up, down, t, K, IC, threads=os.cpu_count() or 8)
            assert rel_err(got, want) <= 2e-3, F.NAMES[t]
            assert rel_err(got, ref) <= 2e-3, F.NAMES[t]
            assert rel_err(want, ref) <= 2e-3, F.NAMES[t]
    finally:
        be.close()


def test_static_scratch_rejects_oversized_windows(ftc, oracle):
    dummy = torch.zeros(16, dtype=torch.uint8, device="cuda")
    p = dummy.data_ptr()
    rc = ftc.lib().ftc_expert_chunk_static(F.Q4_K, p, p, p, p, p, 2, 256, MAX_HC, 144, 144, None)
    assert rc == -1 and "FTC_EXPERT_STATIC_MAX_HC" in ftc.last_error()
    assert ftc.device_status() == 0  # nothing was launched
    # a window that fits is accepted afterwards, and still matches the oracle
    t, M, K, IC = F.Q4_K, 2, 1024, MAX_HC // 2
    x, out, gate, up, down = case(t, M, K, IC, 5)
    got = run_static(ftc, t, x, out, gate, up, down, M, K, IC)
    ref = out.copy()
    oracle.expert_chunk(x, ref, gate, up, down, t, K, IC, threads=os.cpu_count() or 8)
    assert rel_err(got, ref) <= 2e-3
