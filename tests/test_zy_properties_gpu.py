"""Size-independent properties at the BASELINE configs' full sizes, where the
CPU oracle would be slow:

* token permutation: every output row depends on its own token only (per-row
  fp16 scales, row-independent MMAs, top-2 combine of two terms), so
  permuting the tokens of a batch-8 config-2 GEMV permutes the outputs and
  changes no bit.  The tensor-core GEMM (config 3, and the config-5 MoE
  layer's expert GEMMs) schedules stream-K: a tile cut by a CTA's range
  boundary sums fp32 partials of its k pieces, and which tiles are cut
  depends on their place in the schedule, so a token moved to another tile
  may see its k sum split differently -- there the permuted output must
  match within 1e-5 of the output scale (the order of fp32 additions);
* scaling by two: the decode GEMV's activation blocks carry power-of-two
  scales, so y(2x) == 2 y(x) exactly (batch 1, dp4a kernel; batch 4, fp32).

Runs late in the suite."""
import numpy as np
import pytest

from xwfes_b200 import formats as F, synth as S

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ftc():
    assert torch.cuda.is_available(), "GPU test needs CUDA"
    from xwfes_b200 import ftc as mod
    mod.lib()
    return mod


def bf16_rows(T, K, seed):
    bits = S.f32_to_bf16_bits(S.activations_f32(T, K, seed=seed, name="prop.x"))
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("T", [64, 1024])
def test_moe_config5_token_permutation(ftc, T):
    E, U, K, FF = 8, 2, 4096, 14336
    ws = [torch.from_numpy(S.expert_weights(F.Q4_K, E, n, k, seed=1, name=f"prop.{nm}")).cuda()
          for nm, n, k in (("gate", FF, K), ("up", FF, K), ("down", K, FF))]
    layer = ftc.MoeLayer(*ws, n_experts=E, top_k=U, n_embd=K, n_ff=FF)
    logits = torch.from_numpy(S.router_logits(T, E, seed=3)).cuda()
    x = bf16_rows(T, K, seed=3).cuda()
    perm = torch.from_numpy(np.random.default_rng(T).permutation(T)).cuda()
    y = layer(logits, x).clone()
    yp = layer(logits[perm].contiguous(), x[perm].contiguous())
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
    assert close_rows(yp, y[perm])


def close_rows(a, b, tol=1e-5):
    """max |a - b| within tol of max |b| (fp32 summation order only)."""
    a, b = a.float(), b.float()
    return float((a - b).abs().max()) <= tol * float(b.abs().max())


def test_gemm_config3_row_permutation(ftc):
    n, k, m = 14336, 4096, 2048
    w = torch.from_numpy(S.weight(F.Q4_K, n, k, seed=2, name="prop.gemm")).cuda()
    x = bf16_rows(m, k, seed=4).cuda()
    perm = torch.from_numpy(np.random.default_rng(5).permutation(m)).cuda()
    y = ftc.gemm(w, F.Q4_K, n, k, x, y_dtype=F.F32)
    yp = ftc.gemm(w, F.Q4_K, n, k, x[perm].contiguous(), y_dtype=F.F32)
    torch.cuda.synchronize()
    assert ftc.device_status() == 0
    assert close_rows(yp, y[perm])


def test_gemv_batch8_token_permutation(ftc):
    n, k = 14336, 4096
    w = torch.from_numpy(S.weight(F.Q4_K, n, k, seed=6, name="prop.gemv")).cuda()
    x = torch.from_numpy(S.activations_f32(8, k, seed=6, name="prop.x8")).cuda()
    perm = torch.tensor([3, 7, 0, 5, 1, 6, 2, 4], device="cuda")
    y = ftc.mul_mat_vec(w, F.Q4_K, n, k, x)
    yp = ftc.mul_mat_vec(w, F.Q4_K, n, k, x[perm].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(yp, y[perm])


@pytest.mark.parametrize("m", [1, 4])
@pytest.mark.parametrize("n,k", [(14336, 4096), (4096, 14336)])
def test_gemv_scaling_by_two_is_exact(ftc, n, k, m):
    w = torch.from_numpy(S.weight(F.Q4_K, n, k, seed=7, name=f"prop.{n}x{k}")).cuda()
    x = torch.from_numpy(S.activations_f32(m, k, seed=7, name="prop.s")).cuda()
    y1 = ftc.mul_mat_vec(w, F.Q4_K, n, k, x)
    y2 = ftc.mul_mat_vec(w, F.Q4_K, n, k, (2 * x).contiguous())
    torch.cuda.synchronize()
    assert torch.equal(y2, 2 * y1)
