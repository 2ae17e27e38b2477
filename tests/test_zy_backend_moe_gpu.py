"""The routed experts of the engine's moe_ffn (ft/src/engine.cpp:179-241)
through the backend with host buffers (ftc_backend_moe_ffn, the C++
adapter's CudaBackend::moe_ffn): router bias added to the logits, routing,
expert FFNs and combine on the device, the result added into the engine's
tmpo.  Checked against the oracle's MoE (the reference's routing and expert
arithmetic): decode-sized calls (T * top_k <= 4) run fp32 GEMVs and meet the
GEMV tolerance; larger ones run the tensor-core GEMMs on fp16 operands and
meet max |diff| / max |ref| <= 2e-3.  Runs late in the suite."""
import numpy as np
import pytest

from xwfes_b200 import formats as F, synth as S

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

E, U, K, FF = 8, 2, 1024, 2048


@pytest.fixture(scope="module")
def ftc():
    assert torch.cuda.is_available(), "GPU test needs CUDA"
    from xwfes_b200 import ftc as mod
    mod.lib()
    return mod


@pytest.fixture(scope="module")
def experts():
    return (S.expert_weights(F.Q4_K, E, FF, K, seed=4, name="bmoe.gate"),
            S.expert_weights(F.Q4_K, E, FF, K, seed=4, name="bmoe.up"),
            S.expert_weights(F.Q4_K, E, K, FF, seed=4, name="bmoe.down"))


def rel_err(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(y - ref) / (np.abs(ref) + 1e-2 * rms)))


def norm_err(y, ref):
    return float(np.max(np.abs(np.float64(y) - ref)) / np.max(np.abs(ref)))


@pytest.mark.parametrize("T,with_bias", [(1, False), (2, True), (5, False), (64, True)])
def test_backend_moe_matches_oracle(ftc, oracle, experts, T, with_bias):
    g, u, d = experts
    x = S.activations_f32(T, K, seed=T, name="bmoe.x")
    logits = S.router_logits(T, E, seed=T)
    bias = np.random.default_rng(T).standard_normal(E).astype(np.float32) if with_bias else None
    out0 = S.activations_f32(T, K, seed=T + 1, name="bmoe.out")
    out = out0.copy()
    be = ftc.CudaBackend(0)
    try:
        G = ftc.HostTensor(g, F.Q4_K, (K, FF, E))
        Uu = ftc.HostTensor(u, F.Q4_K, (K, FF, E))
        D = ftc.HostTensor(d, F.Q4_K, (FF, K, E))
        be.moe_ffn(x, logits, G, Uu, D, U, out, bias=bias)
    finally:
        be.close()
    biased = logits + bias[None, :] if with_bias else logits
    ref = oracle.moe_ffn(x, biased, g, u, d, F.Q4_K, K, FF, U, threads=8)
    got = out - out0 if T * U > 4 else out
    if T * U <= 4:  # fp32 decode GEMVs: compare the sums as the engine sees them
        assert rel_err(out, ref + out0) <= 2e-3
    else:
        assert norm_err(got, ref) <= 2e-3


def test_backend_moe_no_tokens(ftc, experts):
    g, u, d = experts
    out = np.ones((0, K), dtype=np.float32)
    be = ftc.CudaBackend(0)
    try:
        be.moe_ffn(np.zeros((0, K), np.float32), np.zeros((0, E), np.float32),
                   ftc.HostTensor(g, F.Q4_K, (K, FF, E)), ftc.HostTensor(u, F.Q4_K, (K, FF, E)),
                   ftc.HostTensor(d, F.Q4_K, (FF, K, E)), U, out)
    finally:
        be.close()
