"""Tensor-parallel block (config 4) host logic on the CPU: shard arithmetic
and the column/row-parallel decomposition with a real allreduce between
gloo ranks.  The per-rank matmuls here are the oracle's (the reference's
per-row dot_row_f32 arithmetic), so the TP result must equal the unsharded
block up to the order of the fp32 partial sums."""
import os
import socket

import numpy as np
import pytest

from xwfes_b200 import formats as F, tp

torch = pytest.importorskip("torch")

SMALL = {"n_embd": 512, "n_ff": 1024, "n_q": 512, "n_kv": 256}
MID = {"n_embd": 1024, "n_ff": 2048, "n_q": 1024, "n_kv": 256}


def test_shard_ranges_cover_and_align():
    for n, G in [(8192, 8), (1024, 8), (28672, 4), (1024, 1)]:
        spans = [tp.col_rows(n, G, r) for r in range(G)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    # row-parallel K slices are whole super-blocks: 70B o (8192) and down (28672)
    assert tp.k_slice(8192, 8, 1) == (1024, 2048)
    assert tp.k_slice(28672, 8, 7) == (25088, 28672)
    assert tp.k_slice(28672, 16, 1) == (1792, 3584)  # 7 super-blocks per rank
    with pytest.raises(ValueError):
        tp.k_slice(28672, 32, 0)  # 896 is not a multiple of 256
    with pytest.raises(ValueError):
        tp.col_rows(1000, 3, 0)


def test_shards_reassemble_the_weight():
    w = tp.full_weights(MID, seed=3)
    for G in (1, 2, 4):
        parts = [tp.shard(w, MID, G, r) for r in range(G)]
        for nm, n, k, kind in tp.layout(MID):
            if kind == "col":
                got = np.concatenate([p[nm][0] for p in parts], axis=0)
            else:
                got = np.concatenate([p[nm][0] for p in parts], axis=1)
                assert all(p[nm][0].shape[1] == F.row_bytes(F.Q4_K, k // G) for p in parts)
            assert np.array_equal(got, w[nm]), (nm, G)


def test_config4_shapes():
    d = tp.DIMS_70B
    assert tp.weight_bytes(d) == 481_296_384  # the block's Q4_K bytes
    for G in (1, 2, 4, 8):
        for nm, n, k, kind in tp.layout(d):
            (tp.col_rows(n, G, 0) if kind == "col" else tp.k_slice(k, G, 0))


class OracleOps:
    """The block's matmuls on the CPU with the oracle (fp32 dequant, fp32 sums)."""

    def __init__(self):
        from oracle import oracle as O
        self.O = O

    def upload(self, arr):
        return arr

    def matmuls(self, x, ws):
        xn = np.ascontiguousarray(x.numpy())
        return [torch.from_numpy(self.O.matmul(xn, w, F.Q4_K, k, threads=2)) for w, n, k in ws]

    def silu_matmul(self, gu, n, w):
        gn, un = gu.numpy()[:, :n], gu.numpy()[:, n:2 * n]
        with np.errstate(over="ignore"):  # exp(-g) = inf gives silu = -0, as in C
            h = (gn / (np.float32(1) + np.exp(-gn)) * un).astype(np.float32)
        return self.matmuls(torch.from_numpy(np.ascontiguousarray(h)), [w])[0]


def _rank_main(rank, world, port, out_dir, dims=None):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        d = dims or SMALL
        w = tp.full_weights(d, seed=1)
        blk = tp.TPBlock.build(d, world, rank, OracleOps(), tp.shard(w, d, world, rank))
        x = torch.from_numpy(np.random.default_rng(0).standard_normal((3, d["n_embd"]))
                             .astype(np.float32))
        out, (q, _, _) = blk.forward(x)
        np.save(os.path.join(out_dir, f"out{rank}.npy"), out.numpy())
        np.save(os.path.join(out_dir, f"q{rank}.npy"), q.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_tp_two_ranks_match_unsharded(tmp_path, oracle):
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    w = tp.full_weights(SMALL, seed=1)
    ref_blk = tp.TPBlock.build(SMALL, 1, 0, OracleOps(), tp.shard(w, SMALL, 1, 0))
    x = torch.from_numpy(np.random.default_rng(0).standard_normal((3, SMALL["n_embd"]))
                         .astype(np.float32))
    ref, (qref, _, _) = ref_blk.forward(x)
    ref = ref.numpy()
    o0, o1 = (np.load(tmp_path / f"out{r}.npy") for r in range(2))
    assert np.array_equal(o0, o1)  # every rank holds the same allreduced output
    assert np.max(np.abs(o0 - ref)) <= 1e-5 * np.max(np.abs(ref))
    # column-parallel q slices are the unsharded q's halves, bit for bit
    q = np.concatenate([np.load(tmp_path / f"q{r}.npy") for r in range(2)], axis=1)
    assert np.array_equal(q, qref.numpy())


def test_tp_four_ranks_match_unsharded(tmp_path, oracle):
    """Four gloo ranks on the MID block: row-parallel K slices of one (o) and
    two (down) super-blocks, column slices of 256 / 64 / 512 rows."""
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main, args=(4, _free_port(), str(tmp_path), MID), nprocs=4,
                       start_method="spawn", join=True)
    w = tp.full_weights(MID, seed=1)
    ref_blk = tp.TPBlock.build(MID, 1, 0, OracleOps(), tp.shard(w, MID, 1, 0))
    x = torch.from_numpy(np.random.default_rng(0).standard_normal((3, MID["n_embd"]))
                         .astype(np.float32))
    ref, (qref, _, _) = ref_blk.forward(x)
    outs = [np.load(tmp_path / f"out{r}.npy") for r in range(4)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
    assert np.max(np.abs(outs[0] - ref.numpy())) <= 1e-5 * np.max(np.abs(ref.numpy()))
    q = np.concatenate([np.load(tmp_path / f"q{r}.npy") for r in range(4)], axis=1)
    assert np.array_equal(q, qref.numpy())
