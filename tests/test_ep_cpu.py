"""Expert-parallel MoE (config 5) host logic on the CPU: expert and token
shards, the regrouping of received rows, and the whole exchange (count
all-to-all, row all-to-all, reverse all-to-all, combine) between gloo ranks.
The per-rank compute here is the oracle's (the reference's routing and
expert FFN arithmetic), so the expert-parallel result must equal the oracle's
single-process moe_ffn."""
import os
import socket

import numpy as np
import pytest

from xwfes_b200 import ep, formats as F, synth as S

torch = pytest.importorskip("torch")

E, U, K, FF, T = 4, 2, 256, 512, 10


def test_ranges():
    assert [ep.expert_range(8, 4, r) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        ep.expert_range(8, 3, 0)
    spans = [ep.token_range(10, 4, r) for r in range(4)]
    assert spans == [(0, 3), (3, 6), (6, 8), (8, 10)]
    assert ep.token_range(1, 8, 0) == (0, 1) and ep.token_range(1, 8, 5) == (1, 1)


def test_regroup_orders_rows_by_expert():
    rc = np.array([[2, 0, 1], [1, 3, 0]])  # [source][local expert], cap 4
    perm, inv, counts, offsets = ep.regroup(rc, 4)
    # slots: s0 -> 0 1 (e0) 2 (e2) 3 (pad); s1 -> 4 (e0) 5 6 7 (e1)
    assert perm.tolist() == [0, 1, 4, 5, 6, 7, 2, 3]
    assert (perm[inv] == np.arange(8)).all() and (inv[perm] == np.arange(8)).all()
    assert counts.tolist() == [3, 3, 1] and offsets.tolist() == [0, 3, 6]
    perm, _, counts, _ = ep.regroup(np.zeros((2, 2), np.int64), 3)
    assert perm.tolist() == list(range(6)) and counts.tolist() == [0, 0]


def test_pack_slots():
    # 4 experts on 2 ranks; 3 tokens, top-2
    idx = np.array([[0, 3], [2, 0], [1, 2]])
    counts = np.bincount(idx.ravel(), minlength=4)          # [2, 1, 2, 1]
    order = sorted(range(6), key=lambda r: (idx.ravel()[r], r))
    row_token = np.array([r // 2 for r in order])
    pos = np.empty(6, np.int64)
    pos[order] = np.arange(6)
    src, pp = ep.pack_slots(counts, row_token, idx, pos.reshape(3, 2), 2, 6)
    assert src[0].tolist() == [0, 1, 2, -1, -1, -1]          # experts 0, 1
    assert src[1].tolist() == [1, 2, 0, -1, -1, -1]          # experts 2, 3
    assert pp.tolist() == [[0, 8], [6, 1], [2, 7]]


def np_route(oracle, logits, u):
    """The device routing (ftc_moe_route) restated on the oracle's top-k."""
    idx, w = oracle.route_topk(logits, u)
    t, e = logits.shape
    counts = np.bincount(idx.ravel(), minlength=e).astype(np.int32)
    pos = np.zeros_like(idx)
    row_token = np.zeros(t * u, np.int32)
    row = 0
    for ex in range(e):
        for tk in range(t):
            for s in range(u):
                if idx[tk, s] == ex:
                    pos[tk, s] = row
                    row_token[row] = tk
                    row += 1
    first = {}
    for k, ex in enumerate(idx.ravel()):
        first.setdefault(int(ex), k)
    order = sorted(first, key=first.get)
    rank = np.full(e, -1, np.int32)
    for r, ex in enumerate(order):
        rank[ex] = r
    return {"idx": idx, "w": w, "counts": torch.from_numpy(counts), "pos": pos,
            "row_token": row_token, "rank": rank}


class OracleEPOps:
    def __init__(self, oracle, gate, up, down):
        self.O, self.gate, self.up, self.down = oracle, gate, up, down

    def route(self, logits, u):
        if logits.shape[0] == 0:  # a rank without tokens (T < world)
            z = np.zeros((0, u), np.int64)
            return {"idx": z, "w": z.astype(np.float32), "pos": z, "row_token": np.zeros(0, np.int64),
                    "counts": torch.zeros(logits.shape[1], dtype=torch.int32),
                    "rank": np.full(logits.shape[1], -1, np.int32)}
        return np_route(self.O, logits.numpy(), u)

    def pack(self, x, route, world, cap):
        src, pp = ep.pack_slots(route["counts"].numpy(), route["row_token"], route["idx"],
                                route["pos"], world, cap)
        send = torch.zeros((world, cap, x.shape[1]), dtype=x.dtype)
        valid = torch.from_numpy(src >= 0)
        send[valid] = x[torch.from_numpy(src[src >= 0])]
        return send, pp

    def regroup(self, recv_counts, world, n_local, cap):
        perm, inv, counts, offsets = ep.regroup(recv_counts.numpy().reshape(world, n_local), cap)
        return torch.from_numpy(perm), torch.from_numpy(inv), counts, offsets

    def experts(self, x, counts, offsets, max_rows):
        xn = x.numpy().astype(np.float32)
        y = np.zeros_like(xn)
        for e, (c, o) in enumerate(zip(counts, offsets)):
            if c:
                out = np.zeros((c, K), np.float32)
                self.O.expert_ffn(xn[o:o + c], out, self.gate[e], self.up[e], self.down[e],
                                  F.Q4_K, K, FF, threads=2)
                y[o:o + c] = out
        return torch.from_numpy(y)

    def combine(self, y, route, pos):
        yn = y.numpy().reshape(-1, K)
        idx, w, rank = route["idx"], route["w"], route["rank"]
        out = np.zeros((idx.shape[0], K), np.float32)
        for t in range(idx.shape[0]):
            for s in sorted(range(idx.shape[1]), key=lambda s: rank[idx[t, s]]):
                out[t] = out[t] + np.float32(w[t, s]) * yn[pos[t, s]]
        return torch.from_numpy(out)


def _weights():
    return (S.expert_weights(F.Q4_K, E, FF, K, seed=3, name="ep.gate"),
            S.expert_weights(F.Q4_K, E, FF, K, seed=3, name="ep.up"),
            S.expert_weights(F.Q4_K, E, K, FF, seed=3, name="ep.down"))


def _inputs(T=T):
    return (S.router_logits(T, E, seed=7),
            S.activations_f32(T, K, seed=7, name="ep.x"))


def _rank_main(rank, world, port, out_dir, T=T):
    import torch.distributed as dist
    from oracle import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g, u, d = _weights()
        e0, e1 = ep.expert_range(E, world, rank)
        layer = ep.EPMoE(E, U, K, world, rank, OracleEPOps(O, g[e0:e1], u[e0:e1], d[e0:e1]),
                         max_tokens=-(-T // world))
        logits, x = _inputs(T)
        t0, t1 = ep.token_range(T, world, rank)
        out = layer.forward(torch.from_numpy(logits[t0:t1]), torch.from_numpy(x[t0:t1]))
        np.save(os.path.join(out_dir, f"out{rank}.npy"), out.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_two_ranks_match_single_process_moe(tmp_path, oracle):
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    got = np.concatenate([np.load(tmp_path / f"out{r}.npy") for r in range(2)])
    g, u, d = _weights()
    logits, x = _inputs()
    ref = oracle.moe_ffn(x, logits, g, u, d, F.Q4_K, K, FF, U, threads=2)
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6 * np.abs(ref).max())


@pytest.mark.parametrize("T_,world", [(1, 2), (5, 4)])
def test_ranks_without_tokens_or_with_fewer_experts_than_top_k(tmp_path, oracle, T_, world):
    """T < world leaves ranks without tokens (they still take part in every
    exchange); 4 ranks of a 4-expert top-2 layer hold one expert each."""
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), T_), nprocs=world,
                       start_method="spawn", join=True)
    got = np.concatenate([np.load(tmp_path / f"out{r}.npy") for r in range(world)])
    g, u, d = _weights()
    logits, x = _inputs(T_)
    ref = oracle.moe_ffn(x, logits, g, u, d, F.Q4_K, K, FF, U, threads=2)
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6 * np.abs(ref).max())
