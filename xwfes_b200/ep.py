"""Expert-parallel MoE layer (config 5): the experts split over G GPUs, one
process per GPU, the token exchange over NCCL.

The reference runs every expert in one process (Engine::Impl::moe_ffn,
ft/src/engine.cpp:179-241: route, group tokens per expert, expert FFN,
weighted sum).  Here rank r holds experts [r*E/G, (r+1)*E/G) (whole GGUF
expert planes, uploaded only there) and a shard of the tokens:

  1. route its tokens on the device (ftc_moe_route): top-k experts, weights,
     rows grouped by expert -- which is grouped by destination rank, since
     each rank's experts are contiguous;
  2. pack the rows for each destination into a send buffer of fixed capacity
     (ftc_ep_pack: cap rows per destination, cap = the layer's token
     capacity per rank x top_k) and note where each row's output comes back;
  3. all-to-all of the per-expert row counts and of the row buffers, both
     with equal splits -- no split size goes to the host, so the whole
     forward runs without a host synchronisation and can be captured in a
     CUDA graph;
  4. regroup the received rows by local expert (ftc_ep_regroup: a
     permutation computed on the device) and run the local expert FFNs
     (ftc_moe_experts: grouped tcgen05 dequant-GEMMs on device counts);
  5. the reverse all-to-all of the fp32 expert outputs (equal splits);
  6. the weighted sum in expert first-use order (ftc_moe_combine).

Every token's result is the arithmetic of the single-GPU layer
(ftc_moe_ffn's grouped path) on the same rows, up to the GEMMs' tiling:
the token tile follows the bound on rows per expert and the cut of the last
wave of tiles follows the launch's tile count, so fp32 partial sums may be
ordered differently (and an fp16 rounding of h may then differ by one ulp).

The compute is injected (``ops``): :class:`CudaEPOps` runs the library's
kernels, the CPU tests run the same orchestration with the oracle under gloo.
"""
import numpy as np

# config 5: Mixtral-8x7B-shaped MoE layer
DIMS_MIXTRAL = {"n_experts": 8, "top_k": 2, "n_embd": 4096, "n_ff": 14336}


def expert_range(E, G, r):
    """Experts [e0, e1) held by rank r."""
    if E % G:
        raise ValueError(f"{E} experts do not split evenly over {G} ranks")
    return r * E // G, (r + 1) * E // G


def token_range(T, G, r):
    """Tokens [t0, t1) of rank r (as even as possible)."""
    base, extra = divmod(T, G)
    t0 = r * base + min(r, extra)
    return t0, t0 + base + (1 if r < extra else 0)


def rank_spans(counts, G):
    """(off_d, cnt_d) of every rank d: its experts' rows in the expert order."""
    c = np.asarray(counts, dtype=np.int64).reshape(G, -1).sum(axis=1)
    return np.concatenate([[0], np.cumsum(c)[:-1]]), c


def pack_slots(counts, row_token, idx, pos, G, cap):
    """What ftc_ep_pack computes, on the host: src[d][i] = the token whose
    row goes to slot i of rank d (-1: padding) and pos_padded [T, U]."""
    off, cnt = rank_spans(counts, G)
    src = np.full((G, cap), -1, np.int64)
    for d in range(G):
        src[d, :cnt[d]] = row_token[off[d]:off[d] + cnt[d]]
    El = len(counts) // G
    d_of = np.asarray(idx) // El
    return src, (d_of * cap + (np.asarray(pos) - off[d_of])).astype(np.int32)


def regroup(recv_counts, cap):
    """What ftc_ep_regroup computes, on the host.  recv_counts[s][e]: rows of
    local expert e received from rank s, stored at slots s*cap + (rows of
    s's earlier experts) + i.  Returns (perm, inv, counts, offsets): perm[j]
    is the slot at position j of the expert-major order (valid rows first,
    source-major within an expert, then the padding), inv its inverse."""
    rc = np.asarray(recv_counts, dtype=np.int64)
    G, El = rc.shape
    counts = rc.sum(axis=0)
    offsets = np.concatenate([[0], np.cumsum(counts)[:-1]])
    base = np.concatenate([np.zeros((G, 1), np.int64), np.cumsum(rc, axis=1)[:, :-1]], axis=1)
    order = [s * cap + base[s, e] + i for e in range(El) for s in range(G) for i in range(rc[s, e])]
    order += [s * cap + i for s in range(G) for i in range(rc[s].sum(), cap)]
    perm = np.asarray(order, dtype=np.int64)
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.size)
    return perm, inv, counts.astype(np.int32), offsets.astype(np.int32)


class CudaEPOps:
    """This rank's experts on this GPU through the library's kernels."""

    def __init__(self, device, gate_local, up_local, down_local, n_local, top_k, n_embd, n_ff):
        import torch
        from . import ftc
        self.torch, self.ftc = torch, ftc
        self.layer = ftc.MoeLayer(gate_local, up_local, down_local, n_experts=n_local,
                                  top_k=top_k, n_embd=n_embd, n_ff=n_ff)
        self.device = device

    def route(self, logits, top_k):
        return self.ftc.moe_route(logits, top_k)

    def pack(self, x, route, world, cap):
        return self.ftc.ep_pack(x, route, world, cap)

    def regroup(self, recv_counts, world, n_local, cap):
        return self.ftc.ep_regroup(recv_counts, world, n_local, cap)

    def experts(self, x, counts, offsets, max_rows):
        return self.layer.experts(x, counts, offsets, max_rows)

    def combine(self, y, route, pos):
        return self.ftc.moe_combine(y, route, pos=pos)


class EPMoE:
    """Rank r of G of an expert-parallel MoE layer for up to ``max_tokens``
    tokens per rank (the exchange capacity)."""

    def __init__(self, n_experts, top_k, n_embd, G, rank, ops, max_tokens, group=None):
        self.E, self.U, self.K, self.G, self.rank = n_experts, top_k, n_embd, G, rank
        self.El = n_experts // G
        expert_range(n_experts, G, rank)
        self.ops, self.group = ops, group
        self.max_tokens = int(max_tokens)
        self.cap = self.max_tokens * top_k

    def _a2a(self, out, inp):
        import torch.distributed as dist
        dist.all_to_all_single(out, inp, group=self.group)
        return out

    def forward(self, logits, x):
        """logits: fp32 [T_r, E] and x: [T_r, n_embd] of this rank's tokens
        (T_r <= max_tokens); returns their MoE outputs (fp32 [T_r, n_embd])."""
        ops, G, El, U, K, cap = self.ops, self.G, self.El, self.U, self.K, self.cap
        T = logits.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the layer's capacity of {self.max_tokens} per rank")
        route = ops.route(logits, U)
        send, pos = ops.pack(x, route, G, cap)
        counts = route["counts"]
        if G > 1:
            recv_counts = self._a2a(counts.new_empty(counts.shape), counts)
            recv = self._a2a(send.new_empty(send.shape), send)
        else:
            recv_counts, recv = counts, send
        perm, inv, lcounts, loffsets = ops.regroup(recv_counts, G, El, cap)
        xl = recv.reshape(G * cap, K).index_select(0, perm)
        yl = ops.experts(xl, lcounts, loffsets, G * cap)
        yr = yl.index_select(0, inv)
        yb = self._a2a(yr.new_empty(yr.shape), yr) if G > 1 else yr
        return ops.combine(yb, route, pos)
