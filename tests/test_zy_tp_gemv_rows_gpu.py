"""The tensor-parallel block with more than 8 rows through the fp32 decode
GEMV (tp.CudaOps(gemv_max_m=...): 8 rows per pass over each weight) instead
of the tensor-core GEMM: every output row is the GEMV's, so the block meets
the GEMV agreement (1e-5 normwise) against the oracle, on one GPU and with
every rank's shards summed by hand.  Runs late in the suite (the default
path still sends more than 8 rows to the GEMM)."""
import numpy as np
import pytest

from xwfes_b200 import tp

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from test_tp_gpu import MID, norm_err, oracle_block, x_rows  # noqa: E402


@pytest.fixture(scope="module")
def weights():
    return tp.full_weights(MID, seed=2)


@pytest.mark.parametrize("M", [9, 16, 30])
def test_block_gemv_rows_vs_oracle(oracle, weights, M):
    ops = tp.CudaOps(torch.device("cuda", 0), gemv_max_m=32)
    blk = tp.TPBlock.build(MID, 1, 0, ops, tp.shard(weights, MID, 1, 0))
    x = x_rows(M, MID, seed=M)
    out, _ = blk.forward(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    assert norm_err(out.cpu().numpy(), oracle_block(oracle, weights, MID, x)) <= 1e-5


def test_sharded_gemv_rows(oracle, weights):
    G, M = 4, 16
    ops = tp.CudaOps(torch.device("cuda", 0), gemv_max_m=32)
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
    assert norm_err(np.asarray(out.cpu().numpy()), ref) <= 1e-5
