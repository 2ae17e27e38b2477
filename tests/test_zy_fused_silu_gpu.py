"""The SiLU product folded into the decode GEMV's activation load
(ftc_mul_mat_vec_silu): y = (silu(gate) * up) . W^T for one token must equal
ftc_silu_mul_rows followed by ftc_mul_mat_vec bit for bit (one expression,
silu_gate, in both), and the CPU oracle within the GEMV tolerance; on two
GPUs the fused allreduce variant must equal the separate SiLU, GEMV and
ftc_peer_ar_sum_f32 on every rank.  Runs late in the suite, after the
kernels it shares (the decode GEMV, the silu rows, the peer allreduce)."""
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


@pytest.mark.parametrize("n,k,pad", [(8192, 3584, 0), (4096, 14336, 0), (1000, 1024, 64),
                                     (28672, 8192, 0)])
def test_fused_silu_equals_separate(ftc, oracle, n, k, pad):
    """pad > 0: gate and up are not adjacent (up at k + pad)."""
    w = S.weight(F.Q4_K, n, k, seed=1, name="fsilu")
    g = np.random.default_rng(k + n)
    gu = np.zeros((1, 2 * k + pad), dtype=np.float32)
    gu[0, :k] = 4 * g.standard_normal(k)
    gu[0, k + pad:] = g.standard_normal(k)
    wd = torch.from_numpy(w).cuda()
    gud = torch.from_numpy(gu).cuda()
    yf = ftc.mul_mat_vec_silu(wd, F.Q4_K, n, k, gud, up_offset=k + pad)
    adjacent = gud if pad == 0 else torch.cat([gud[:, :k], gud[:, k + pad:]], dim=1).contiguous()
    h = ftc.silu_mul_rows(adjacent, k)
    ys = ftc.mul_mat_vec(wd, F.Q4_K, n, k, h)
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
    assert torch.equal(yf, ys)
    gate, up = gu[0, :k], gu[0, k + pad:]
    hx = (gate / (1 + np.exp(-gate.astype(np.float64))) * up).astype(np.float32)
    ref = oracle.matmul(hx.reshape(1, k), w, F.Q4_K, k, threads=8)
    assert rel_err(yf.cpu().numpy(), ref) <= 2e-3


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_fused_silu_allreduce_matches_separate(tmp_path):
    import test_peer_ar_gpu as T
    r0, r1 = T._run(tmp_path, "fused_silu")
    for i in range(2):
        for r in (r0, r1):
            assert np.array_equal(r[f"sf{i}"], r[f"sr{i}"]), i
        assert np.array_equal(r0[f"sf{i}"], r1[f"sf{i}"]), i
