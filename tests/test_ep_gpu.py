"""GPU parity of the expert-parallel MoE layer (config 5 structure, reduced
sizes).  With one rank the layer is routing + grouped expert GEMMs + combine
and must reproduce ftc_moe_ffn's grouped path; across two GPUs (NCCL) the rows
exchanged between ranks must give the same result again.

Each output row depends only on its own token and experts, but the two
layers tile their GEMMs differently: the token tile follows the caller's
bound on rows per expert (all tokens on one GPU, the rank's capacity under
EP), and a launch with few output tiles cuts K into ranges whose fp32
partials are summed in a fixed order that follows the launch's tile count.
So gate/up agree to fp32 summation order only (~1e-6 relative), and where
h = silu(gate) * up lies next to an fp16 rounding boundary its 16-bit copy
for the down GEMM can differ by one fp16 ulp (2^-11 relative).  A few such
elements per row move the output by ~1e-5 of its scale (measured up to
~2e-5 of an element on two B200s), so the bound is 1e-4 relative to the
largest output; the one-token case below compares different paths
altogether and keeps the GEMM tolerance."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from xwfes_b200 import ep, formats as F, synth as S

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
E, U, K, FF = 8, 2, 1024, 2048


def weights():
    return (S.expert_weights(F.Q4_K, E, FF, K, seed=4, name="epg.gate"),
            S.expert_weights(F.Q4_K, E, FF, K, seed=4, name="epg.up"),
            S.expert_weights(F.Q4_K, E, K, FF, seed=4, name="epg.down"))


def inputs(T):
    x = S.activations_bf16(T, K, seed=T, name="epg.x")
    return S.router_logits(T, E, seed=T), x


def to_dev(logits, xbits):
    return (torch.from_numpy(logits).cuda(),
            torch.from_numpy(xbits.view(np.int16)).cuda().view(torch.bfloat16))


def close(got, want):  # bound: see the module docstring
    return got.shape == want.shape and \
        float(np.max(np.abs(got - want))) <= 1e-4 * float(np.max(np.abs(want)))


def single_gpu(T):
    from xwfes_b200 import ftc
    g, u, d = (torch.from_numpy(a).cuda() for a in weights())
    layer = ftc.MoeLayer(g, u, d, n_experts=E, top_k=U, n_embd=K, n_ff=FF)
    lg, x = to_dev(*inputs(T))
    return layer(lg, x).cpu().numpy()


@pytest.mark.parametrize("T", [64, 300])
def test_one_rank_equals_moe_layer(T):
    g, u, d = (torch.from_numpy(a).cuda() for a in weights())
    ops = ep.CudaEPOps(torch.device("cuda", 0), g, u, d, E, U, K, FF)
    layer = ep.EPMoE(E, U, K, 1, 0, ops, max_tokens=T)
    lg, x = to_dev(*inputs(T))
    out = layer.forward(lg, x)
    torch.cuda.synchronize()
    assert close(out.cpu().numpy(), single_gpu(T))


_CHILD = r"""
import os, sys, datetime, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, {root!r})
sys.path.insert(0, os.path.join({root!r}, "tests"))
from xwfes_b200 import ep
import test_ep_gpu as T
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                        device_id=torch.device("cuda", rank))
g, u, d = T.weights()
e0, e1 = ep.expert_range(T.E, world, rank)
dev = torch.device("cuda", rank)
ops = ep.CudaEPOps(dev, *(torch.from_numpy(a[e0:e1]).to(dev) for a in (g, u, d)),
                   e1 - e0, T.U, T.K, T.FF)
layer = ep.EPMoE(T.E, T.U, T.K, world, rank, ops, max_tokens=150)
for n in (64, 300, 1):  # 1 token: rank 1 has none and still takes part
    logits, x = T.inputs(n)
    t0, t1 = ep.token_range(n, world, rank)
    lg = torch.from_numpy(logits[t0:t1]).to(dev)
    xb = torch.from_numpy(x[t0:t1].view(np.int16)).to(dev).view(torch.bfloat16)
    out = layer.forward(lg, xb)
    torch.cuda.synchronize()
    np.save(os.path.join({out!r}, f"out{{n}}_{{rank}}.npy"), out.cpu().numpy())
dist.barrier()
dist.destroy_process_group()
"""


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_gpus_nccl(tmp_path):
    code = _CHILD.format(root=ROOT, out=str(tmp_path))
    port = _free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, "-c", code], env=env, cwd=ROOT))
    for p in procs:
        assert p.wait(timeout=300) == 0
    for n in (64, 300):
        got = np.concatenate([np.load(tmp_path / f"out{n}_{r}.npy") for r in range(2)])
        assert close(got, single_gpu(n))
    # one token: the single-GPU layer takes its decode path (fp32 GEMVs), the
    # expert-parallel one the grouped GEMMs (16-bit operands), so they agree
    # to the GEMM tolerance only
    got = np.concatenate([np.load(tmp_path / f"out1_{r}.npy") for r in range(2)])
    assert got.shape == (1, K)
    want = single_gpu(1)
    assert float(np.max(np.abs(got - want))) <= 2e-3 * float(np.max(np.abs(want)))


@pytest.mark.parametrize("T,world", [(1, 1), (37, 2), (64, 4), (300, 8)])
def test_pack_and_regroup_match_host_reference(T, world):
    """ftc_ep_pack / ftc_ep_regroup against the host restatement in ep.py,
    element for element, on the device routing of random logits."""
    from xwfes_b200 import ftc
    cap = T * U + 3
    lg, xb = to_dev(*inputs(T))
    route = ftc.moe_route(lg, U)
    send, pp = ftc.ep_pack(xb, route, world, cap)
    torch.cuda.synchronize()
    h = {k: v.cpu().numpy() for k, v in route.items()}
    src, pp_ref = ep.pack_slots(h["counts"], h["row_token"], h["idx"], h["pos"], world, cap)
    assert np.array_equal(pp.cpu().numpy(), pp_ref)
    sv, xv = send.cpu().view(torch.int16).numpy(), xb.cpu().view(torch.int16).numpy()
    for d in range(world):
        valid = src[d] >= 0
        assert np.array_equal(sv[d][valid], xv[src[d][valid]])
    # receive side: counts of `world` sources for the n_local experts of one rank
    El = E // world
    rng = np.random.default_rng(T)
    rc = rng.integers(0, 4, size=(world, El)).astype(np.int32)
    rc = np.minimum(rc, cap // max(1, El))
    got = ftc.ep_regroup(torch.from_numpy(rc.ravel()).cuda(), world, El, cap)
    ref = ep.regroup(rc, cap)
    for g, r in zip(got, ref):
        assert np.array_equal(g.cpu().numpy(), r)
