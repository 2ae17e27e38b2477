"""GPU parity of the tcgen05 prefill dequant-GEMM (ftc_gemm).

Exactness first: with one-hot activation rows, y[m][n] is a single product
1.0 * w16[n][k_m] accumulated in fp32, so it must equal the 16-bit operand the
on-chip dequant produces (q4k_operand16 restates its arithmetic) -- this pins
the dequant, the 128-byte swizzled operand layout and the token/row mapping
bit for bit.

Float tolerance: the GEMM multiplies 16-bit operands (activations as given,
weights rounded to the same 16-bit type) with fp32 accumulation.
  * Against an fp32 reference on the SAME 16-bit operands (isolates the
    kernel's own arithmetic): relative error <= 2e-3 with a floor of
    0.1 * rms(y).  The tensor cores sum each 16-product MMA step internally
    before the fp32 accumulate, which over K = 14336 differs from sequential
    fp32 FMAs by ~2e-5 * rms(y), hence the larger floor than the GEMV's.
  * Against the exact-weight oracle (the reference's arithmetic on fp32
    dequantized weights): max|y - ref| / max|ref| <= 2e-3; the rounding of
    the weights to 16 bits is the extra error the tensor-core path adds."""
import os

import numpy as np
import pytest

from xwfes_b200 import formats as F, synth as S

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 8


@pytest.fixture(scope="module")
def ftc():
    assert torch.cuda.is_available()
    from xwfes_b200 import ftc as mod
    mod.lib()
    return mod


def rel_err(y, ref, floor=1e-2):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(y - ref) / (np.abs(ref) + floor * rms)))


def norm_err(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(y - ref)) / np.max(np.abs(ref)))


TDT = {F.BF16: torch.bfloat16, F.F16: torch.float16}


def to16(a32, t):
    return torch.from_numpy(np.ascontiguousarray(a32, dtype=np.float32)).to(TDT[t])


def q4k_operand16(w, n, k, xt):
    """The 16-bit weights the tensor-core path multiplies, emulated exactly.
    fp16 operands: w16 = fp16(q * fp16(d*sc) - fp16(dmin*m)), one rounding of
    the fused multiply-add (q*DL - ML is exact in float64).  bf16 operands:
    bf16 of the fp32 dequantized weight (d*sc*q exact, the subtraction
    rounded once), i.e. the reference's dequant_row value rounded once."""
    blk = np.ascontiguousarray(w).reshape(n, k // 256, 144)
    d = blk[:, :, 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    dmin = blk[:, :, 2:4].copy().view(np.float16)[..., 0].astype(np.float32)
    sp = blk[:, :, 4:16].astype(np.int32)
    sc = np.empty((n, k // 256, 8), np.int32)
    mn = np.empty_like(sc)
    sc[..., :4] = sp[..., 0:4] & 63
    mn[..., :4] = sp[..., 4:8] & 63
    sc[..., 4:] = (sp[..., 8:12] & 15) | ((sp[..., 0:4] >> 6) << 4)
    mn[..., 4:] = (sp[..., 8:12] >> 4) | ((sp[..., 4:8] >> 6) << 4)
    DL = (d[..., None] * sc.astype(np.float32)).astype(np.float16).astype(np.float64)
    ML = (dmin[..., None] * mn.astype(np.float32)).astype(np.float16).astype(np.float64)
    qs = blk[:, :, 16:].astype(np.int64)
    q = np.empty((n, k // 256, 256), np.int64)
    for g in range(4):
        q[:, :, 64 * g:64 * g + 32] = qs[:, :, 32 * g:32 * g + 32] & 15
        q[:, :, 64 * g + 32:64 * g + 64] = qs[:, :, 32 * g:32 * g + 32] >> 4
    sub = np.arange(256) // 32
    if xt == F.BF16:
        dl = (d[..., None] * sc.astype(np.float32)).astype(np.float32)
        ml = (dmin[..., None] * mn.astype(np.float32)).astype(np.float32)
        w32 = (q.astype(np.float32) * dl[:, :, sub] - ml[:, :, sub]).astype(np.float32)
        return S.bf16_bits_to_f32(S.f32_to_bf16_bits(w32)).reshape(n, k)
    w16 = (q * DL[:, :, sub] - ML[:, :, sub]).astype(np.float16).astype(np.float32)
    return w16.reshape(n, k)


@pytest.mark.parametrize("xt", [F.F16, F.BF16])
@pytest.mark.parametrize("m,n,k", [(128, 256, 1024), (256, 384, 512), (200, 130, 256)])
def test_gemm_one_hot_exact(ftc, oracle, xt, m, n, k):
    w = S.weight(F.Q4_K, n, k, seed=2, name="gemm.onehot")
    w16 = q4k_operand16(w, n, k, xt)
    # the operand is the exact dequantized weight to within one 16-bit ulp of
    # the largest weight (d*sc and dmin*m are rounded to fp16 before the
    # multiply-add, so cancelling weights carry that scale's rounding)
    deq = oracle.dequant_rows(w, F.Q4_K, k)
    ulp = 2.0 ** (-10 if xt == F.F16 else -7)
    assert np.max(np.abs(w16 - deq)) <= ulp * np.abs(deq).max()
    ks = (np.arange(m) * 37 + 11) % k
    x = np.zeros((m, k), dtype=np.float32)
    x[np.arange(m), ks] = 1.0
    y = ftc.gemm(torch.from_numpy(w).cuda(), F.Q4_K, n, k, to16(x, xt).cuda(), y_dtype=F.F32)
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
    got = y.cpu().numpy()
    assert np.array_equal(got, w16[:, ks].T)


def _torch_ref(ftc, w, n, k, x16):
    """fp32 reference on the same 16-bit operands the kernel multiplies."""
    xt = F.F16 if x16.dtype == torch.float16 else F.BF16
    w16 = torch.from_numpy(q4k_operand16(w, n, k, xt)).to(x16.device)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    ref = x16.float() @ w16.T
    torch.backends.cuda.matmul.allow_tf32 = prev
    return ref


@pytest.mark.parametrize("xt", [F.F16, F.BF16])
@pytest.mark.parametrize("m,n,k", [(256, 512, 2048), (130, 1000, 4096), (512, 256, 14336)])
def test_gemm_random_vs_oracle(ftc, oracle, xt, m, n, k):
    w = S.weight(F.Q4_K, n, k, seed=3, name="gemm.rand")
    xb = S.activations_f32(m, k, seed=3)
    x16 = to16(xb, xt)
    wd = torch.from_numpy(w).cuda()
    y = ftc.gemm(wd, F.Q4_K, n, k, x16.cuda(), y_dtype=F.F32)
    ref16 = _torch_ref(ftc, w, n, k, x16.cuda())
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
    got = y.cpu().numpy()
    assert rel_err(got, ref16.cpu().numpy(), floor=0.1) <= 2e-3
    # the reference's own arithmetic (fp32 weights, fp32 accumulate) on the
    # same activations, for a row subset
    rows = slice(0, min(m, 64))
    ora = oracle.matmul(x16.float().numpy()[rows], w, F.Q4_K, k, threads=THREADS)
    assert norm_err(got[rows], ora) <= 2e-3


@pytest.mark.parametrize("n,k", [(14336, 4096), (4096, 14336)])
@pytest.mark.parametrize("m", [128, 512, 2048, 8192])
def test_gemm_config3(ftc, oracle, n, k, m):
    """Config 3 at full size, bf16 activations and bf16 output."""
    w = S.weight(F.Q4_K, n, k, seed=0, name=f"c3.{n}x{k}")
    wd = torch.from_numpy(w).cuda()
    x16 = torch.from_numpy(S.activations_bf16(m, k, seed=0, name=f"c3.{m}")).cuda().view(
        torch.bfloat16)
    y = ftc.gemm(wd, F.Q4_K, n, k, x16, y_dtype=F.BF16)
    y32 = ftc.gemm(wd, F.Q4_K, n, k, x16, y_dtype=F.F32)
    ref = _torch_ref(ftc, w, n, k, x16)
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
    # fp32 output against the same-operand fp32 reference
    assert rel_err(y32.cpu().numpy(), ref.cpu().numpy(), floor=0.1) <= 2e-3
    # bf16 output is the fp32 result rounded once
    assert torch.equal(y, y32.to(torch.bfloat16))
    rows = slice(0, 16)
    ora = oracle.matmul(x16[rows].float().cpu().numpy(), w, F.Q4_K, k, threads=THREADS)
    assert norm_err(y32[rows].cpu().numpy(), ora) <= 2e-3


@pytest.mark.parametrize("m,n,k", [(16, 128, 8192), (77, 384, 14336), (300, 256, 4096)])
def test_gemm_split_k(ftc, oracle, m, n, k):
    """Shapes with fewer output tiles than SMs: the K range is split over
    several CTAs (on 148 SMs each of these tiles is cut into aligned pieces,
    none crossing a tile) and the partials are summed in a fixed order, so
    the result matches the reference and repeats bit for bit, also when
    replayed from a CUDA graph."""
    _check_cut_tiles(ftc, oracle, m, n, k)


# The tail plans of the tile schedule on a 148-SM B200 (whole waves, then
# the last partial wave run whole, cut into aligned pieces, or cut stream-K
# with ranges that cross tile boundaries); every plan must give the same
# arithmetic per tile up to the fp32 order of its pieces.
@pytest.mark.parametrize("m,n,k", [
    (16, 10240, 4096),    # 80 tiles: stream-K over all SMs, ranges crossing tiles
    (16, 21504, 4096),    # 168 tiles: a whole wave, then 20 tiles in aligned pieces
    (16, 29440, 4096),    # 230 tiles: a whole wave, then a stream-K tail
    (100, 10240, 4096),   # 128-token tile (A in tensor memory), stream-K
    (300, 10240, 4096),   # 256-token tile, a whole wave, then aligned pieces
    (2048, 4096, 14336),  # 256-token tile, a whole wave, then a stream-K tail
])
def test_gemm_tail_plans(ftc, oracle, m, n, k):
    _check_cut_tiles(ftc, oracle, m, n, k)


def _check_cut_tiles(ftc, oracle, m, n, k):
    w = S.weight(F.Q4_K, n, k, seed=5, name="gemm.split")
    x16 = to16(S.activations_f32(m, k, seed=5), F.BF16).cuda()
    wd = torch.from_numpy(w).cuda()
    y1 = ftc.gemm(wd, F.Q4_K, n, k, x16, y_dtype=F.F32)
    y2 = ftc.gemm(wd, F.Q4_K, n, k, x16, y_dtype=F.F32)
    yb = ftc.gemm(wd, F.Q4_K, n, k, x16, y_dtype=F.BF16)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg = ftc.gemm(wd, F.Q4_K, n, k, x16, y_dtype=F.F32)
    g.replay()
    g.replay()
    ref = _torch_ref(ftc, w, n, k, x16)
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
    assert torch.equal(y1, y2) and torch.equal(yg, y1)
    assert torch.equal(yb, y1.to(torch.bfloat16))
    assert rel_err(y1.cpu().numpy(), ref.cpu().numpy(), floor=0.1) <= 2e-3
    rows = slice(0, 16)
    ora = oracle.matmul(x16[rows].float().cpu().numpy(), w, F.Q4_K, k, threads=THREADS)
    assert norm_err(y1[rows].cpu().numpy(), ora) <= 2e-3
