"""GPU parity of the routed-expert MoE FFN (ftc_moe_ffn).

The oracle is the reference's Engine::Impl::moe_ffn (ft/src/engine.cpp:
179-241) restated in oracle/ftoracle.c (ftor_route_topk, ftor_moe_ffn): fp32
softmax routing, top-k, renormalised weights, per-expert SiLU FFN with fp32
dequantized weights and fp32 sums, weighted sum in expert first-use order.

Routing is compared exactly (expert ids, token counts) and to 1e-6 relative
(weights: CUDA's expf and the host's may differ in the last bit).

The expert matmuls run on the tensor cores with fp16 operands (x rows and h
rows scaled by powers of two into fp16's range, weights dequantized to fp16)
and fp32 accumulation, so the output is held to the north-star float bound
normwise: max|out - ref| / max|ref| <= 2e-3 (measured ~3e-4)."""
import os

import numpy as np
import pytest

from xwfes_b200 import formats as F, synth as S

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 8
TOL = 2e-3


@pytest.fixture(scope="module")
def ftc():
    assert torch.cuda.is_available()
    from xwfes_b200 import ftc as mod
    mod.lib()
    return mod


def norm_err(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(y - ref)) / np.max(np.abs(ref)))


def make_layer(ftc, E, K, FF, U, seed):
    g = S.expert_weights(F.Q4_K, E, FF, K, seed=seed, name="moe.gate")
    u = S.expert_weights(F.Q4_K, E, FF, K, seed=seed, name="moe.up")
    d = S.expert_weights(F.Q4_K, E, K, FF, seed=seed, name="moe.down")
    dev = [torch.from_numpy(a).cuda() for a in (g, u, d)]
    layer = ftc.MoeLayer(*dev, n_experts=E, top_k=U, n_embd=K, n_ff=FF)
    return layer, (g, u, d)


def x_input(T, K, xt, seed, scale=1.0):
    x32 = S.activations_f32(T, K, seed=seed, name="moe.x") * np.float32(scale)
    if xt == F.BF16:
        bits = S.f32_to_bf16_bits(x32)
        return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16), S.bf16_bits_to_f32(bits)
    if xt == F.F16:
        x16 = x32.astype(np.float16)
        return torch.from_numpy(x16), x16.astype(np.float32)
    return torch.from_numpy(x32), x32


# ---------------------------------------------------------------- routing

@pytest.mark.parametrize("T,E,U", [(1, 8, 2), (64, 8, 2), (1024, 8, 2), (2500, 8, 2),
                                   (333, 16, 4), (50, 256, 8), (7, 4, 4)])
def test_route_matches_oracle(ftc, oracle, T, E, U):
    layer, _ = make_layer(ftc, E, 256, 256, U, seed=11)
    logits = S.router_logits(T, E, seed=T + E)
    x, _ = x_input(T, 256, F.BF16, seed=1)
    layer(torch.from_numpy(logits).cuda(), x.cuda())
    torch.cuda.synchronize()
    idx, w, cnt = (a.cpu().numpy() for a in layer.routing(T))
    oi, ow = oracle.route_topk(logits, U)
    assert np.array_equal(idx, oi)
    np.testing.assert_allclose(w, ow, rtol=1e-6, atol=0)
    assert np.array_equal(cnt, np.bincount(oi.ravel(), minlength=E))


# ------------------------------------------------- reduced shapes vs oracle

@pytest.mark.parametrize("xt", [F.BF16, F.F32])
@pytest.mark.parametrize("T", [1, 2, 5, 64, 300])
def test_moe_vs_oracle(ftc, oracle, T, xt):
    """T * top_k <= 4 runs the decode path (a GEMV per (token, slot) pair on
    the experts chosen on the device), larger T the grouped GEMMs."""
    E, U, K, FF = 8, 2, 1024, 2048
    layer, (g, u, d) = make_layer(ftc, E, K, FF, U, seed=5)
    logits = S.router_logits(T, E, seed=T)
    x, x32 = x_input(T, K, xt, seed=T)
    out = layer(torch.from_numpy(logits).cuda(), x.cuda())
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
    ref = oracle.moe_ffn(x32, logits, g, u, d, F.Q4_K, K, FF, U, threads=THREADS)
    assert norm_err(out.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("T,E,U", [(3, 4, 1), (8, 4, 1), (1, 16, 4)])
def test_moe_top_k(ftc, oracle, T, E, U):
    K, FF = 512, 1024
    layer, (g, u, d) = make_layer(ftc, E, K, FF, U, seed=13)
    logits = S.router_logits(T, E, seed=5)
    x, x32 = x_input(T, K, F.F16 if U == 1 else F.BF16, seed=6)
    out = layer(torch.from_numpy(logits).cuda(), x.cuda())
    torch.cuda.synchronize()
    ref = oracle.moe_ffn(x32, logits, g, u, d, F.Q4_K, K, FF, U, threads=THREADS)
    assert norm_err(out.cpu().numpy(), ref) <= TOL


def test_moe_skewed_routing(ftc, oracle):
    """Every token picks expert 3 first (600 rows: token tiles of 256, 256 and
    88), half of them expert 5 second; experts 0-2 get nothing."""
    E, U, K, FF, T = 8, 2, 512, 768, 600
    layer, (g, u, d) = make_layer(ftc, E, K, FF, U, seed=6)
    logits = S.router_logits(T, E, seed=9)
    logits[:, 3] += 20.0
    logits[: T // 2, 5] += 10.0
    logits[:, :3] -= 30.0
    x, x32 = x_input(T, K, F.BF16, seed=3)
    out = layer(torch.from_numpy(logits).cuda(), x.cuda())
    torch.cuda.synchronize()
    cnt = layer.routing(T)[2].cpu().numpy()
    assert cnt[3] == T and cnt[5] >= T // 2 and cnt[:3].sum() == 0
    ref = oracle.moe_ffn(x32, logits, g, u, d, F.Q4_K, K, FF, U, threads=THREADS)
    assert norm_err(out.cpu().numpy(), ref) <= TOL


@pytest.mark.parametrize("scale", [1e-5, 3e4])
def test_moe_input_range(ftc, oracle, scale):
    """fp16 operands with per-row power-of-two scales: inputs far outside
    fp16's range (h reaches ~1e16 at scale 3e4) keep the same accuracy."""
    E, U, K, FF, T = 8, 2, 512, 512, 24
    layer, (g, u, d) = make_layer(ftc, E, K, FF, U, seed=7)
    logits = S.router_logits(T, E, seed=4)
    x, x32 = x_input(T, K, F.F32, seed=8, scale=scale)
    out = layer(torch.from_numpy(logits).cuda(), x.cuda()).cpu().numpy()
    ref = oracle.moe_ffn(x32, logits, g, u, d, F.Q4_K, K, FF, U, threads=THREADS)
    assert np.all(np.isfinite(out))
    assert norm_err(out, ref) <= TOL


@pytest.mark.parametrize("T", [1, 77])
def test_moe_deterministic_and_graph_capturable(ftc, T):
    """No atomics on the data path: repeated calls agree bit for bit, and the
    whole layer replays from a CUDA graph (no host round trip inside), for
    the decode path (T=1) and the grouped-GEMM path."""
    E, U, K, FF = 8, 2, 1024, 1024
    layer, _ = make_layer(ftc, E, K, FF, U, seed=12)
    logits = torch.from_numpy(S.router_logits(T, E, seed=2)).cuda()
    x = x_input(T, K, F.BF16, seed=5)[0].cuda()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        a = layer(logits, x, stream=s).clone()
        b = layer(logits, x, stream=s).clone()
        out = torch.empty_like(a)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            layer(logits, x, out=out, stream=s)
        out.zero_()
        graph.replay()
    s.synchronize()
    assert torch.equal(a, b) and torch.equal(out, a)


# ------------------------------------------------------ config 5, full size

@pytest.fixture(scope="module")
def config5(ftc):
    E, U, K, FF = 8, 2, 4096, 14336
    layer, host = make_layer(ftc, E, K, FF, U, seed=0)
    return layer, host, (E, U, K, FF)


def _torch_moe_ref(ftc, host, logits, x32, E, U, K, FF, oracle):
    """fp32 reference on the GPU: weights dequantized bit-exactly
    (ftc_dequant, pinned against the reference's dequant in test_gemv_gpu),
    routing from the oracle, fp32 matmuls, weighted sum in first-use order."""
    g, u, d = host
    idx, w = oracle.route_topk(logits, U)
    xd = torch.from_numpy(x32).cuda()
    out = torch.zeros((x32.shape[0], K), dtype=torch.float64, device="cuda")
    order = []
    for e in idx.ravel():
        if e not in order:
            order.append(int(e))
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for e in order:
            tok, slot = np.nonzero(idx == e)
            G = ftc.dequant(torch.from_numpy(g[e]).cuda(), F.Q4_K, FF, K)
            Uw = ftc.dequant(torch.from_numpy(u[e]).cuda(), F.Q4_K, FF, K)
            D = ftc.dequant(torch.from_numpy(d[e]).cuda(), F.Q4_K, K, FF)
            xe = xd[torch.from_numpy(tok).cuda()]
            gv = xe @ G.T
            h = gv / (1 + torch.exp(-gv)) * (xe @ Uw.T)
            ye = h @ D.T
            wt = torch.from_numpy(w[tok, slot]).cuda()[:, None]
            out[torch.from_numpy(tok).cuda()] += (wt * ye).double()
            del G, Uw, D
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return out.cpu().numpy(), idx


@pytest.mark.parametrize("T", [1, 64, 1024])
def test_moe_config5(ftc, oracle, config5, T):
    layer, host, (E, U, K, FF) = config5
    logits = S.router_logits(T, E, seed=0)
    x, x32 = x_input(T, K, F.BF16, seed=0)
    out = layer(torch.from_numpy(logits).cuda(), x.cuda())
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
    ref, idx = _torch_moe_ref(ftc, host, logits, x32, E, U, K, FF, oracle)
    cnt = layer.routing(T)[2].cpu().numpy()
    assert np.array_equal(cnt, np.bincount(idx.ravel(), minlength=E))
    assert norm_err(out.cpu().numpy(), ref) <= TOL
    if T == 1:  # the C oracle itself on the decode case
        ora = oracle.moe_ffn(x32, logits, *host, F.Q4_K, K, FF, U, threads=THREADS)
        assert norm_err(out.cpu().numpy(), ora) <= TOL
