"""The batch-1 dp4a GEMV's per-lane arithmetic for Q6_K and Q8_0 rows
(q6k_row_partial / q80_row_partial in xwfes_b200/csrc/gemv_q4k.cu),
restated step for step in integer numpy and checked on the CPU against the
oracle's dequantization (ft/include/ft/quant.h:10-84 for Q8_0; the GGUF
K-quant layout, pinned to gguf-py, for Q6_K).

The kernel's lane t of a quartet holds weights [64t, 64t + 64) of each
256-weight stretch as exact activation integers split into three byte
planes (hi signed, mid and lo unsigned).  Its integer sums per plane are
exact, so for integer activations the restatement must give exactly
sum_k dequant(W)[k] * x[k]: a wrong byte index, shift, sign extension or
scale byte shows up as a mismatch here, without a GPU."""
import numpy as np
import pytest

from xwfes_b200 import formats as F, synth as S


def words(b, off, n):
    """n little-endian 32-bit words of the bytes at off (any alignment, as
    the kernel's funnel-shifted reads give)."""
    return [int.from_bytes(bytes(b[off + 4 * i: off + 4 * i + 4]), "little") for i in range(n)]


def sbyte(v):
    return v - 256 if v >= 128 else v


def dp4a(a, b, a_signed, b_signed):
    s = 0
    for i in range(4):
        x, y = (a >> (8 * i)) & 0xFF, (b >> (8 * i)) & 0xFF
        s += (sbyte(x) if a_signed else x) * (sbyte(y) if b_signed else y)
    return s


def lane_planes(xi, t):
    """The lane's 16 plane words per digit plane for x integers [64t, 64t+64)."""
    xs = [int(v) for v in xi[64 * t: 64 * t + 64]]

    def plane(shift):
        return [sum(((xs[4 * u + b] >> shift) & 0xFF) << (8 * b) for b in range(4))
                for u in range(16)]
    return plane(16), plane(8), plane(0)


def q6k_lane(blk, t, H, M, L):
    """q6k_row_partial without the final float steps: (ph, pm, pl), d."""
    h, qq = t >> 1, t & 1
    ql, qh = words(blk, 64 * h, 16), words(blk, 128 + 32 * h, 8)
    scw = words(blk, 192 + 8 * h + 4 * qq, 1)[0]
    d = float(np.frombuffer(bytes(blk[208:210]), dtype=np.float16)[0])
    ph = pm = pl = 0
    for j in range(2):
        for g in range(2):
            sh = sm = sl = 0
            for uu in range(4):
                u = 4 * g + uu
                lo = (ql[8 * j + u] >> (4 * qq)) & 0x0F0F0F0F
                hx = ((qh[u] >> (4 * qq + 2 * j)) & 0x03030303) ^ 0x02020202
                s6 = (lo + hx * 16) & 0xFFFFFFFF
                q = (s6 + (s6 & 0x20202020) * 6) & 0xFFFFFFFF
                sh += dp4a(q, H[8 * j + u], True, True)
                sm += dp4a(q, M[8 * j + u], True, False)
                sl += dp4a(q, L[8 * j + u], True, False)
            sc = sbyte((scw >> (8 * (2 * j + g))) & 0xFF)
            ph, pm, pl = ph + sc * sh, pm + sc * sm, pl + sc * sl
    for v in (ph, pm, pl):
        assert -(1 << 31) <= v < (1 << 31)  # the kernel's int32 sums cannot overflow
    return d * (65536.0 * ph + 256.0 * pm + pl)


def q80_lane(unit, t, H, M, L):
    """q80_row_partial without the block scale's float rounding."""
    tot = 0.0
    for j in range(2):
        off = 34 * (2 * t + j)
        d = float(np.frombuffer(bytes(unit[off:off + 2]), dtype=np.float16)[0])
        q = words(unit, off + 2, 8)
        sh = sum(dp4a(q[u], H[8 * j + u], True, True) for u in range(8))
        sm = sum(dp4a(q[u], M[8 * j + u], True, False) for u in range(8))
        sl = sum(dp4a(q[u], L[8 * j + u], True, False) for u in range(8))
        tot += d * (65536.0 * sh + 256.0 * sm + sl)
    return tot


def check_rows(w, dtype, k, lane_fn, unit_bytes, oracle, seed):
    deq = oracle.dequant_rows(w, dtype, k).astype(np.float64)
    rng = np.random.default_rng(seed)
    xi = rng.integers(-(1 << 21), 1 << 21, k)  # 22-bit activation integers, both signs
    for r in range(w.shape[0]):
        got = 0.0
        for sb in range(k // 256):
            unit = w[r, sb * unit_bytes:(sb + 1) * unit_bytes + 4]  # + the kernel's over-read
            for t in range(4):
                H, M, L = lane_planes(xi[256 * sb: 256 * sb + 256], t)
                got += lane_fn(unit, t, H, M, L)
        want = float(np.dot(deq[r], xi.astype(np.float64)))
        assert got == want, (r, got, want)


def test_q6k_lane_math_random_rows(oracle):
    w = S.weight(F.Q6_K, 6, 512, seed=41)
    w = np.concatenate([w, np.zeros((w.shape[0], 4), np.uint8)], axis=1)
    check_rows(w, F.Q6_K, 512, q6k_lane, 210, oracle, seed=1)


def test_q6k_lane_math_gguf_edge_blocks(oracle, golden):
    """gguf-py's edge-case Q6_K blocks (extreme codes and scales)."""
    g = golden("gguf_kquant.npz")
    blocks = g["q6_k_blocks"]
    w = np.concatenate([blocks, np.zeros((blocks.shape[0], 4), np.uint8)], axis=1)
    deq = g["q6_k_dequant"].astype(np.float64)
    assert np.array_equal(oracle.dequant_rows(blocks, F.Q6_K, 256), g["q6_k_dequant"])
    rng = np.random.default_rng(2)
    xi = rng.integers(-(1 << 21), 1 << 21, 256)
    for r in range(blocks.shape[0]):
        got = sum(q6k_lane(w[r], t, *lane_planes(xi, t)) for t in range(4))
        assert got == float(np.dot(deq[r], xi.astype(np.float64))), r


def test_q80_lane_math_random_rows(oracle):
    w = S.weight(F.Q8_0, 6, 512, seed=43)
    w = np.concatenate([w, np.zeros((w.shape[0], 4), np.uint8)], axis=1)
    check_rows(w, F.Q8_0, 512, q80_lane, 272, oracle, seed=3)


@pytest.mark.parametrize("u", range(64))
def test_q6_sign_extension_every_code(u):
    """(q6 ^ 32) + 0xC0 where bit 5 is set is q6 - 32 as a signed byte, for
    every 6-bit code, in every byte position, without carries."""
    for pos in range(4):
        hi2, lo4 = u >> 4, u & 0xF
        lo = lo4 << (8 * pos)
        hx = (hi2 ^ 2) << (8 * pos)
        s6 = lo + hx * 16
        q = (s6 + (s6 & 0x20202020) * 6) & 0xFFFFFFFF
        assert sbyte((q >> (8 * pos)) & 0xFF) == u - 32
        assert q & ~(0xFF << (8 * pos)) == 0
