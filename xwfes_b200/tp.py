"""Tensor-parallel Llama-3-70B-shaped linear block (config 4), one process per
GPU, NCCL over NVLink for the exchange.

The reference engine runs every layer in one process (ft/src/engine.cpp:
485-600: q/k/v, o, gate/up, down matmuls through IBackend::matmul); this is
the same chain of Q4_K matmuls split across G GPUs:

  column-parallel  q, k, v, gate, up: rank r holds rows [r*N/G, (r+1)*N/G)
                   of W, computes that slice of the outputs, no exchange;
  row-parallel     o, down: rank r holds the 256-aligned column slice
                   [r*K/G, (r+1)*K/G) of every row (whole GGUF super-blocks,
                   K/G a multiple of 256), multiplies the matching slice of
                   its input, and the partial [M, n_embd] outputs are summed
                   by an allreduce.

  h   = allreduce_r( q_r . o_r )              (q_r stands in for the rank's
                                               attention heads: attention is
                                               not part of this path)
  a_r = silu(h . gate_r) * (h . up_r)
  out = allreduce_r( a_r . down_r )

Every rank uploads only its own shard (contiguous GGUF blocks; a K slice of a
row is a run of whole super-blocks).  A rank's q, k and v rows are stacked
into one weight, and so are its gate and up rows, so each group is one
matmul launch (rows are independent: the stacked product is the row-wise
concatenation of the separate ones, bit for bit); silu(gate) * up is taken
on the [gate | up] output rows by one kernel that also produces the fp16
operand of the down GEMM (at one token, by the down GEMV itself as it loads
its activation: ftc_mul_mat_vec_silu).  Matmuls: M <= 8 tokens use the decode
GEMV (fp32 activations), larger M the tcgen05 GEMM on fp16 rows with
power-of-two row scales (ftc_rows_to_f16 / ftc_gemm_rowscaled), fp32 outputs.
The allreduce sums fp32 partials: small ones (decode-sized M) through
ftc_peer_ar (one-shot over NVLink peer memory, a few microseconds) when the
block is given a :class:`~xwfes_b200.ftc.PeerAllreduce`, the rest through
torch.distributed (NCCL on GPUs, any group on the CPU).

The compute is injected (``ops``): :class:`CudaOps` runs the library's
kernels; tests run the same orchestration with the CPU oracle under gloo.
"""
from dataclasses import dataclass

import numpy as np

from . import formats as F, synth as S

# config 4: Llama-3-70B layer shapes
DIMS_70B = {"n_embd": 8192, "n_ff": 28672, "n_q": 8192, "n_kv": 1024}
QK = 256  # Q4_K super-block
# longest n_ff slice whose down GEMV takes silu(gate) * up itself (measured:
# at 28672 the fused GEMV is 11 us slower than SiLU + GEMV, each CTA then
# reading 229 KB of [gate | up]; at 3584 it saves the SiLU launch)
FUSED_SILU_MAX_K = 8192


def col_rows(n, G, r):
    """Rows [r0, r1) of an n-row column-parallel weight held by rank r."""
    if n % G:
        raise ValueError(f"{n} rows do not split evenly over {G} ranks")
    return r * n // G, (r + 1) * n // G


def k_slice(k, G, r):
    """Columns [k0, k1) of a row-parallel weight held by rank r; whole
    super-blocks only."""
    if k % (G * QK):
        raise ValueError(f"K={k} does not split into whole super-blocks over {G} ranks")
    return r * k // G, (r + 1) * k // G


def shard_rows(w, n, G, r):
    r0, r1 = col_rows(n, G, r)
    return np.ascontiguousarray(w[r0:r1])


def shard_k(w, k, G, r, dtype=F.Q4_K):
    """The rank's K slice of every row as contiguous rows of whole blocks."""
    eb, bb = F.BLOCK[F.dtype_id(dtype)]
    k0, k1 = k_slice(k, G, r)
    return np.ascontiguousarray(w[:, (k0 // eb) * bb:(k1 // eb) * bb])


# (name, rows N, cols K, kind) of the block's weights
def layout(d):
    return [("q", d["n_q"], d["n_embd"], "col"), ("k", d["n_kv"], d["n_embd"], "col"),
            ("v", d["n_kv"], d["n_embd"], "col"), ("o", d["n_embd"], d["n_q"], "row"),
            ("gate", d["n_ff"], d["n_embd"], "col"), ("up", d["n_ff"], d["n_embd"], "col"),
            ("down", d["n_embd"], d["n_ff"], "row")]


def full_weights(d, seed=0):
    """Unsharded synthetic Q4_K weights of one block (host uint8 arrays)."""
    return {nm: S.weight(F.Q4_K, n, k, seed=seed, name=f"tp.{nm}") for nm, n, k, _ in layout(d)}


def shard(weights, d, G, r):
    """Rank r's shards of full weights: {name: (array, rows, cols)}."""
    out = {}
    for nm, n, k, kind in layout(d):
        if kind == "col":
            r0, r1 = col_rows(n, G, r)
            out[nm] = (shard_rows(weights[nm], n, G, r), r1 - r0, k)
        else:
            k0, k1 = k_slice(k, G, r)
            out[nm] = (shard_k(weights[nm], k, G, r), n, k1 - k0)
    return out


def rank_shards(d, G, r, seed=0):
    """Rank r's shards drawn directly (synthetic weights of the right shapes
    and distributions without building the full block: for benchmarks)."""
    out = {}
    for nm, n, k, kind in layout(d):
        if kind == "col":
            r0, r1 = col_rows(n, G, r)
            out[nm] = (S.weight(F.Q4_K, r1 - r0, k, seed=seed, name=f"tp.{nm}.{G}.{r}"), r1 - r0, k)
        else:
            k0, k1 = k_slice(k, G, r)
            out[nm] = (S.weight(F.Q4_K, n, k1 - k0, seed=seed, name=f"tp.{nm}.{G}.{r}"), n, k1 - k0)
    return out


def weight_bytes(d):
    return sum(F.row_bytes(F.Q4_K, k) * n for _, n, k, _ in layout(d))


def flops(d, M):
    return 2.0 * M * sum(n * k for _, n, k, _ in layout(d))


class CudaOps:
    """The block's matmuls on this GPU through the library's kernels: up to
    ``gemv_max_m`` rows through the fp32 decode GEMV (8 rows per pass over
    the weight), more through the tcgen05 GEMM on row-scaled fp16 operands."""

    def __init__(self, device, gemv_max_m=8):
        import torch
        from . import ftc
        self.torch, self.ftc, self.device = torch, ftc, device
        self.gemv_max_m = max(8, int(gemv_max_m))

    def _gemv_rows(self, x, w, n, k):
        """x . W^T for M <= gemv_max_m rows, 8 rows per GEMV launch."""
        M = x.shape[0]
        if M <= 8:
            return self.ftc.mul_mat_vec(w, F.Q4_K, n, k, x)
        y = self.torch.empty((M, n), dtype=self.torch.float32, device=x.device)
        for m0 in range(0, M, 8):
            self.ftc.mul_mat_vec(w, F.Q4_K, n, k, x[m0:m0 + 8], y=y[m0:m0 + 8])
        return y

    def upload(self, arr):
        return self.torch.from_numpy(arr).to(self.device)

    def silu_matmul(self, gu, n, w, peer=None):
        """(silu(gate) * up) . W^T for rows gu = [gate (n) | up (n)]; with
        ``peer`` (one token) the product is also summed over the ranks."""
        ftc, M = self.ftc, gu.shape[0]
        wt, wn, wk = w
        if M == 1 and wk == n and n <= FUSED_SILU_MAX_K and gu.is_contiguous() and n % 4 == 0:
            # one token, a rank's short n_ff slice: the SiLU product is taken
            # as the GEMV loads its activation (no separate launch), with the
            # allreduce fused too.  Every CTA of that GEMV reads the whole
            # [gate | up] row, so for long rows the separate SiLU is faster.
            if peer is not None:
                return peer.silu_mul_mat_vec_sum(wt, F.Q4_K, wn, wk, gu, up_offset=n)
            return ftc.mul_mat_vec_silu(wt, F.Q4_K, wn, wk, gu, up_offset=n)
        if M <= self.gemv_max_m:
            h = ftc.silu_mul_rows(gu, n)
            if peer is not None:
                return peer.mul_mat_vec_sum(wt, F.Q4_K, wn, wk, h)
            return self._gemv_rows(h, wt, wn, wk)
        x16, e = ftc.silu_mul_rows(gu, n, to_f16=True)
        return ftc.gemm_rowscaled(wt, F.Q4_K, wn, wk, x16, e)

    def matmul_sum(self, x, w, peer):
        """x . W^T summed over the ranks, GEMV and allreduce fused (one token)."""
        wt, wn, wk = w
        return peer.mul_mat_vec_sum(wt, F.Q4_K, wn, wk, x.contiguous())

    def matmuls(self, x, ws):
        """[x . W^T for (W, n, k) in ws], x fp32 [M, k] shared by all."""
        ftc, M = self.ftc, x.shape[0]
        k = ws[0][2]
        if M <= 8:
            x = x.contiguous()
            if len(ws) == 1:
                w, n, _ = ws[0]
                return [ftc.mul_mat_vec(w, F.Q4_K, n, k, x)]
            return ftc.mul_mat_vec_multi([w for w, _, _ in ws], F.Q4_K, [n for _, n, _ in ws], k, x)
        if M <= self.gemv_max_m:
            x = x.contiguous()
            return [self._gemv_rows(x, w, n, k) for w, n, _ in ws]
        x16, e = ftc.rows_to_f16(x)
        return [ftc.gemm_rowscaled(w, F.Q4_K, n, k, x16, e) for w, n, _ in ws]

    def silu_mul(self, g, u):
        return self.ftc.silu_mul(g, u)


@dataclass
class TPBlock:
    """Rank r of G: its uploaded shards and the forward pass."""
    dims: dict
    G: int
    rank: int
    ops: object
    shards: dict
    group: object = None
    peer: object = None  # optional PeerAllreduce for partials that fit its buffer

    @classmethod
    def build(cls, dims, G, rank, ops, host_shards, group=None, peer=None):
        h = dict(host_shards)
        for grp, names in (("qkv", ("q", "k", "v")), ("gate_up", ("gate", "up"))):
            parts = [h.pop(nm) for nm in names]
            h[grp] = (np.concatenate([a for a, _, _ in parts], axis=0),
                      sum(n for _, n, _ in parts), parts[0][2])
        dev = {nm: (ops.upload(a), n, k) for nm, (a, n, k) in h.items()}
        return cls(dims, G, rank, ops, dev, group, peer)

    def _allreduce(self, t):
        if self.G > 1:
            if self.peer is not None and self.peer.fits(t):
                return self.peer.sum_(t)
            import torch.distributed as dist
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        return t

    def forward(self, x):
        """x: fp32 [M, n_embd] on this rank's device (replicated); returns the
        block output (fp32 [M, n_embd], identical on every rank) and this
        rank's q/k/v slices."""
        W, d, G = self.shards, self.dims, self.G
        nq, nkv, nf = d["n_q"] // G, d["n_kv"] // G, d["n_ff"] // G
        qkv = self.ops.matmuls(x, [W["qkv"]])[0]
        q, k, v = qkv[:, :nq], qkv[:, nq:nq + nkv], qkv[:, nq + nkv:]
        if self._fused(x):  # one token: the row-parallel GEMVs carry their allreduce
            h = self.ops.matmul_sum(q, W["o"], self.peer)
            gu = self.ops.matmuls(h, [W["gate_up"]])[0]
            return self.ops.silu_matmul(gu, nf, W["down"], peer=self.peer), (q, k, v)
        h = self._allreduce(self.ops.matmuls(q, [W["o"]])[0])
        gu = self.ops.matmuls(h, [W["gate_up"]])[0]
        out = self._allreduce(self.ops.silu_matmul(gu, nf, W["down"]))
        return out, (q, k, v)

    def _fused(self, x):
        return (self.G > 1 and self.peer is not None and x.shape[0] == 1 and
                hasattr(self.ops, "matmul_sum"))
