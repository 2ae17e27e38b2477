"""Expert-parallel MoE layer (config 5): the experts split over G GPUs, one
process per GPU, the token exchange over NCCL.

The reference runs every expert in one process (Engine::Impl::moe_ffn,
ft/src/engine.cpp:179-241: route, group tokens per expert, expert FFN,
weighted sum).  Here rank r holds experts [r*E/G, (r+1)*E/G) (whole GGUF
expert planes, uploaded only there) and a shard of the tokens:

  1. route its tokens on the device (ftc_moe_route): top-k experts, weights,
     rows grouped by expert -- which is grouped by destination rank, since
     each rank's experts are contiguous;
  2. all-to-all of the per-expert row counts (int32 [E]); the split sizes go
     to the host once (NCCL's all-to-all takes them there);
  3. all-to-all of the token rows (their own dtype, bf16 for config 5);
  4. the received rows, regrouped by local expert, through the local expert
     FFNs (ftc_moe_experts: grouped tcgen05 dequant-GEMMs);
  5. the reverse all-to-all of the fp32 expert outputs;
  6. the weighted sum in expert first-use order (ftc_moe_combine).

Every token's result is the same arithmetic as the single-GPU layer
(ftc_moe_ffn's grouped path): each output row depends only on its own token
and expert, not on which other rows share a tile or a GPU.

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


def regroup(recv_counts):
    """recv_counts[s][e]: rows of local expert e received from rank s, stored
    source-major ([s][e][rows]).  Returns (perm, counts, offsets): perm[i] is
    the received row that goes to position i of the expert-major order."""
    rc = np.asarray(recv_counts, dtype=np.int64)
    G, El = rc.shape
    start = np.zeros_like(rc)
    start.reshape(-1)[1:] = np.cumsum(rc.reshape(-1))[:-1]
    perm = np.concatenate([np.arange(start[s, e], start[s, e] + rc[s, e])
                           for e in range(El) for s in range(G)] or [np.zeros(0, np.int64)])
    counts = rc.sum(axis=0)
    offsets = np.concatenate([[0], np.cumsum(counts)[:-1]])
    return perm.astype(np.int64), counts.astype(np.int32), offsets.astype(np.int32)


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

    def gather(self, x, route, rows):
        return x.index_select(0, route["row_token"][:rows].long())

    def experts(self, x, counts, offsets):
        t = self.torch
        if x.shape[0] == 0:
            return t.empty((0, x.shape[1]), dtype=t.float32, device=x.device)
        return self.layer.experts(x, self.index(counts), self.index(offsets), int(counts.max()))

    def combine(self, y, route):
        return self.ftc.moe_combine(y, route)

    def to_host(self, *ts):
        """One device-to-host read of several int32 vectors (one sync)."""
        t = self.torch
        flat = t.cat([v.reshape(-1) for v in ts]).cpu().numpy()
        out, o = [], 0
        for v in ts:
            out.append(flat[o:o + v.numel()])
            o += v.numel()
        return out

    def index(self, n):
        """Host index array to the device through pinned memory, without
        waiting for the GPU (stream-ordered)."""
        t = self.torch
        h = t.from_numpy(np.ascontiguousarray(n)).pin_memory()
        return h.to(self.device, non_blocking=True)


class EPMoE:
    """Rank r of G of an expert-parallel MoE layer."""

    def __init__(self, n_experts, top_k, n_embd, G, rank, ops, group=None):
        self.E, self.U, self.K, self.G, self.rank = n_experts, top_k, n_embd, G, rank
        self.El = n_experts // G
        expert_range(n_experts, G, rank)
        self.ops, self.group = ops, group

    def _a2a(self, out, inp, out_splits=None, in_splits=None):
        import torch.distributed as dist
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        return out

    def forward(self, logits, x):
        """logits: fp32 [T_r, E] and x: [T_r, n_embd] of this rank's tokens;
        returns their MoE outputs (fp32 [T_r, n_embd])."""
        import torch
        ops, G, El, U = self.ops, self.G, self.El, self.U
        T = logits.shape[0]
        R = T * U
        route = ops.route(logits, U)
        counts = route["counts"]
        if G > 1:
            recv_counts = self._a2a(torch.empty_like(counts), counts)
        else:
            recv_counts = counts
        # the split sizes on the host: the layer's one synchronisation
        c, rc = ops.to_host(counts, recv_counts)
        c, rc = c.reshape(G, El), rc.reshape(G, El)
        send_splits = [int(v) for v in c.sum(axis=1)]
        recv_splits = [int(v) for v in rc.sum(axis=1)]
        xg = ops.gather(x, route, R)  # rows in expert order = destination order
        if G > 1:
            xr = self._a2a(x.new_empty((sum(recv_splits), x.shape[1])), xg, recv_splits,
                           send_splits)
        else:
            xr = xg
        perm, lcounts, loffsets = regroup(rc)
        pi = ops.index(perm)
        yl = ops.experts(xr.index_select(0, pi), lcounts, loffsets)
        yr = torch.empty_like(yl)
        yr[pi] = yl
        if G > 1:
            yb = self._a2a(yl.new_empty((R, yl.shape[1])), yr, send_splits, recv_splits)
        else:
            yb = yr
        return ops.combine(yb, route)
