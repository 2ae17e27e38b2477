"""GPU parity of the tensor-parallel block (config 4 shapes, reduced sizes).

The oracle is the reference's arithmetic for each matmul (per-row
dot_row_f32 on fp32 dequantized weights, oracle.matmul) chained through the
block on the CPU.  M <= 8 runs the fp32 decode GEMVs (agreement ~1e-6); larger
M the tcgen05 GEMM on fp16 rows with power-of-two row scales, held to the
north-star bound normwise: max|y - ref| / max|ref| <= 2e-3.

Sharding is checked on one GPU by running every rank's shards and summing
the row-parallel partials by hand, and across two GPUs with NCCL when the
machine has them."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from xwfes_b200 import formats as F, tp

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MID = {"n_embd": 1024, "n_ff": 2048, "n_q": 1024, "n_kv": 256}
TOL = 2e-3


def norm_err(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / np.max(np.abs(ref)))


def oracle_block(oracle, w, d, x):
    mm = lambda a, nm, k: oracle.matmul(a, w[nm], F.Q4_K, k, threads=os.cpu_count() or 8)
    q = mm(x, "q", d["n_embd"])
    h = mm(q, "o", d["n_q"])
    g, u = mm(h, "gate", d["n_embd"]), mm(h, "up", d["n_embd"])
    with np.errstate(over="ignore"):
        a = (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float32)
    return mm(a, "down", d["n_ff"])


def x_rows(M, d, seed=0):
    return np.random.default_rng(seed).standard_normal((M, d["n_embd"])).astype(np.float32)


@pytest.fixture(scope="module")
def weights():
    return tp.full_weights(MID, seed=2)


@pytest.mark.parametrize("M", [1, 4, 16, 100])
def test_block_single_gpu_vs_oracle(oracle, weights, M):
    ops = tp.CudaOps(torch.device("cuda", 0))
    blk = tp.TPBlock.build(MID, 1, 0, ops, tp.shard(weights, MID, 1, 0))
    x = x_rows(M, MID, seed=M)
    out, _ = blk.forward(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    ref = oracle_block(oracle, weights, MID, x)
    assert norm_err(out.cpu().numpy(), ref) <= (1e-5 if M <= 8 else TOL)


@pytest.mark.parametrize("G", [2, 4])
@pytest.mark.parametrize("M", [1, 16])
def test_sharded_ranks_on_one_gpu(oracle, weights, G, M):
    """Every rank's shards through the kernels (K slices of whole
    super-blocks for o and down; stacked q/k/v and gate/up rows), partials
    summed by hand."""
    ops = tp.CudaOps(torch.device("cuda", 0))
    ranks = [tp.TPBlock.build(MID, G, r, ops, tp.shard(weights, MID, G, r)) for r in range(G)]
    x = torch.from_numpy(x_rows(M, MID, seed=7)).cuda()
    nq, nf = MID["n_q"] // G, MID["n_ff"] // G
    qs = [ops.matmuls(x, [b.shards["qkv"]])[0][:, :nq] for b in ranks]
    h = sum(ops.matmuls(q, [b.shards["o"]])[0] for q, b in zip(qs, ranks))
    out = 0
    for b in ranks:
        gu = ops.matmuls(h, [b.shards["gate_up"]])[0]
        out = out + ops.silu_matmul(gu, nf, b.shards["down"])
    torch.cuda.synchronize()
    ref = oracle_block(oracle, weights, MID, x.cpu().numpy())
    assert norm_err(out.cpu().numpy(), ref) <= (1e-5 if M <= 8 else TOL)


_CHILD = r"""
import os, sys, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, {root!r})
from xwfes_b200 import tp
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
import datetime
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                        device_id=torch.device("cuda", rank))
from xwfes_b200 import ftc
d = {dims!r}
w = tp.full_weights(d, seed=2)
peer = ftc.PeerAllreduce(16 * d["n_embd"]) if {peer!r} else None
blk = tp.TPBlock.build(d, world, rank, tp.CudaOps(torch.device("cuda", rank)),
                       tp.shard(w, d, world, rank), peer=peer)
for M in (1, 16, 40):
    x = np.random.default_rng(M).standard_normal((M, d["n_embd"])).astype(np.float32)
    out, _ = blk.forward(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    np.save(os.path.join({out!r}, f"out{{M}}_{{rank}}.npy"), out.cpu().numpy())
dist.barrier()
if peer is not None:
    peer.close()
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
@pytest.mark.parametrize("peer", [False, True], ids=["nccl", "peer_allreduce"])
def test_two_gpus(oracle, weights, tmp_path, peer):
    """Two ranks on two GPUs; the row-parallel partials summed by NCCL, or
    (peer) by ftc_peer_ar for M <= 16 and NCCL for M = 40."""
    code = _CHILD.format(root=ROOT, dims=MID, out=str(tmp_path), peer=peer)
    port = _free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, "-c", code], env=env, cwd=ROOT))
    for p in procs:
        assert p.wait(timeout=300) == 0
    for M in (1, 16, 40):
        o0, o1 = (np.load(tmp_path / f"out{M}_{r}.npy") for r in range(2))
        assert np.array_equal(o0, o1)
        ref = oracle_block(oracle, weights, MID, np.random.default_rng(M).standard_normal(
            (M, MID["n_embd"])).astype(np.float32))
        assert norm_err(o0, ref) <= (1e-5 if M <= 8 else TOL)


@pytest.mark.parametrize("M", [1, 5, 33])
def test_silu_mul_rows(M):
    """ftc_silu_mul_rows equals ftc_silu_mul on the split halves (fp32 rows)
    and ftc_rows_to_f16 of that result (fp16 rows), bit for bit."""
    from xwfes_b200 import ftc
    n = 3584
    gu = torch.randn(M, 2 * n + 8, device="cuda") * 3
    g, u = gu[:, :n].contiguous(), gu[:, n:2 * n].contiguous()
    ref = ftc.silu_mul(g, u)
    assert torch.equal(ftc.silu_mul_rows(gu, n), ref)
    h16, e = ftc.silu_mul_rows(gu, n, to_f16=True)
    r16, re = ftc.rows_to_f16(ref)
    assert torch.equal(h16, r16) and torch.equal(e, re)
