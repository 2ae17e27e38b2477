"""Generate the golden fixtures under tests/golden/.

Run where the reference tree exists (it needs oracle/_ref/libftref.so, the
reference's own CPU code built by oracle/Makefile) and where gguf-py is
importable:

    make -C oracle && python tests/golden/gen_golden.py

Fixtures (all small, numpy .npz):

* ref_q8_0_gemv.npz  -- Q8_0 rows from the config-1 generator plus ragged
  K (96: three blocks; 2080: crosses dot_row_f32's 2048-element chunk),
  with the reference's dequant_row, dot_row_f32 and CpuBackend::matmul
  outputs (M=1 and its row-summing M=3 behaviour).
* ref_test_quant.npz -- the reference test's own construction
  (ft/src/tests/test_core.cpp:239-293): LCG values, F16/Q8_0/Q4_0 rows
  built with the reference's float_to_half, and the reference's dots.
* ref_chunker_f32.npz -- the reference chunker test's shapes
  (ft/src/tests/test_core.cpp:307-346): F32 K=16, FF=48, M=3, windows of 8,
  run window by window through CpuBackend::run_expert_chunk.
* ref_expert_q8_0.npz -- one Q8_0 expert chunk through run_expert_chunk.
* ref_dequant_formats.npz -- F16/BF16/Q4_0/Q4_1 rows through dequant_row.
* ref_down_axpy.npz -- the engine's down projection ft::matmul_down_axpy
  (ft/src/cpu_backend.cpp:60-75) on Q8_0, F16 and Q4_0 rows in the
  reference's transposed layout, activations with zeros (the skipped rows)
  and a non-zero starting y.
* gguf_kquant.npz -- Q4_K/Q6_K blocks (random and edge cases) with the
  dequantized values from the GGUF format's Python package (gguf-py); the
  reference has no K-quant decoder, so this is the only external pin.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from xwfes_b200 import formats as F, synth as S  # noqa: E402


def save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **arrays)
    print(f"wrote {name}: {os.path.getsize(path)} bytes")


def lcg_stream(n, state=123456789):
    """The reference test's rnd() (ft/src/tests/test_core.cpp:79-83), started
    from its initial state."""
    out = np.empty(n, dtype=np.float32)
    for i in range(n):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32(((state >> 9) & 0x7FFF) / 32768.0) * np.float32(2.0) - np.float32(1.0)
    return out, state


def gen_q8_0_gemv():
    cases = {}
    for tag, n, k in (("k4096", 4, 4096), ("k96", 3, 96), ("k2080", 2, 2080)):
        w = S.weight(F.Q8_0, n, k, seed=0, name=f"golden.{tag}")
        x = S.activations_f32(3, k, seed=0, name=f"golden.{tag}")
        cases[f"{tag}_w"] = w
        cases[f"{tag}_x"] = x
        cases[f"{tag}_dequant"] = O.ref_dequant_rows(w, F.Q8_0, k)
        cases[f"{tag}_dot"] = np.array([O.ref_dot_row(x[0], w[r], F.Q8_0, k) for r in range(n)],
                                       dtype=np.float32)
        cases[f"{tag}_matmul_m1"] = O.ref_matmul(x[:1], w, F.Q8_0, k, threads=2)
        # the reference's CpuBackend::matmul with M=3 writes y[n] = sum_m dot(x_m, W_n)
        cases[f"{tag}_matmul_m3_rowsum"] = O.ref_matmul(x, w, F.Q8_0, k, threads=2)[:n]
    save("ref_q8_0_gemv.npz", **cases)


def gen_test_quant():
    r = O.ref()
    vals, _ = lcg_stream(128)
    refv, x = vals[:64], vals[64:]
    f16 = np.array([r.ftref_float_to_half(float(v)) for v in refv], dtype=np.uint16)
    f16row = f16.view(np.uint8)
    q8 = np.zeros(2 * 34, dtype=np.uint8)
    q4 = np.zeros(2 * 18, dtype=np.uint8)
    for b in range(2):
        blk = refv[b * 32:(b + 1) * 32]
        mx = np.float32(np.abs(blk).max())
        d = mx / np.float32(127) if mx > 0 else np.float32(1e-8)
        dh = r.ftref_float_to_half(float(d))
        q8[b * 34:b * 34 + 2] = np.array([dh], dtype=np.uint16).view(np.uint8)
        for j in range(32):
            qi = int(np.clip(round_half_away(blk[j] / d), -127, 127))
            q8[b * 34 + 2 + j] = np.uint8(qi & 0xFF)
        d4 = mx / np.float32(7) if mx > 0 else np.float32(1e-8)
        dh4 = r.ftref_float_to_half(float(d4))
        q4[b * 18:b * 18 + 2] = np.array([dh4], dtype=np.uint16).view(np.uint8)
        for j in range(32):
            nib = int(np.clip(round_half_away(blk[j] / d4) + 8, 0, 15))
            if j & 1:
                q4[b * 18 + 2 + (j >> 1)] |= np.uint8(nib << 4)
            else:
                q4[b * 18 + 2 + (j >> 1)] = np.uint8(nib)
    refdot = np.float32(0)
    for i in range(64):
        refdot = np.float32(refdot + np.float32(refv[i] * x[i]))
    save("ref_test_quant.npz", ref=refv, x=x, refdot=np.float32(refdot),
         f16row=f16row, q8row=q8, q4row=q4,
         dot_f16=np.float32(O.ref_dot_row(x, f16row, F.F16, 64)),
         dot_q8=np.float32(O.ref_dot_row(x, q8, F.Q8_0, 64)),
         dot_q4=np.float32(O.ref_dot_row(x, q4, F.Q4_0, 64)),
         dequant_q8=O.ref_dequant_rows(q8[None], F.Q8_0, 64)[0],
         dequant_q4=O.ref_dequant_rows(q4[None], F.Q4_0, 64)[0])


def round_half_away(v):
    """std::lround: nearest integer, halves away from zero."""
    v = float(v)
    return int(np.floor(abs(v) + 0.5)) * (1 if v >= 0 else -1)


def gen_chunker():
    K, FF, M, C = 16, 48, 3, 8
    g = S.rng(0, "golden.chunker")
    gate = (g.uniform(-1, 1, size=(FF, K)) * 0.5).astype(np.float32)
    up = (g.uniform(-1, 1, size=(FF, K)) * 0.5).astype(np.float32)
    down = (g.uniform(-1, 1, size=(FF, K)) * 0.5).astype(np.float32)
    x = g.uniform(-1, 1, size=(M, K)).astype(np.float32)
    out = np.zeros((M, K), dtype=np.float32)
    # ExpertStreamer::run without staging (ft/include/ft/chunker.h:49-78)
    for i0 in range(0, FF, C):
        ic = min(C, FF - i0)
        O.ref_expert_chunk(x, out, gate[i0:i0 + ic].view(np.uint8),
                           up[i0:i0 + ic].view(np.uint8), down[i0:i0 + ic].view(np.uint8),
                           F.F32, K, ic, threads=1)
    save("ref_chunker_f32.npz", x=x, gate=gate, up=up, down=down, out=out, window=np.int64(C))


def gen_expert_q8_0():
    M, K, IC = 3, 256, 64
    gate = S.weight(F.Q8_0, IC, K, seed=0, name="golden.ex.gate")
    up = S.weight(F.Q8_0, IC, K, seed=0, name="golden.ex.up")
    down = S.weight(F.Q8_0, IC, K, seed=0, name="golden.ex.down")  # neuron-major
    x = S.activations_f32(M, K, seed=0, name="golden.ex")
    out = S.activations_f32(M, K, seed=1, name="golden.ex.acc")  # accumulates onto this
    out0 = out.copy()
    O.ref_expert_chunk(x, out, gate, up, down, F.Q8_0, K, IC, threads=2)
    save("ref_expert_q8_0.npz", x=x, gate=gate, up=up, down=down, out_in=out0, out=out)


def gen_formats():
    g = S.rng(0, "golden.formats")
    arrays = {}
    vals = g.standard_normal(size=(2, 64)).astype(np.float32)
    arrays["f16_w"] = vals.astype(np.float16).view(np.uint8)
    arrays["bf16_w"] = S.f32_to_bf16_bits(vals).view(np.uint8)
    arrays["q4_0_w"] = g.integers(0, 256, size=(2, 2 * 18), dtype=np.uint8)
    arrays["q4_1_w"] = g.integers(0, 256, size=(2, 2 * 20), dtype=np.uint8)
    for t, name in ((F.Q4_0, "q4_0_w"), (F.Q4_1, "q4_1_w")):  # sane fp16 scales
        bb = F.BLOCK[t][1]
        w = arrays[name]
        for b in range(2):
            w[:, b * bb:b * bb + 2] = np.array([0x2E66], dtype=np.uint16).view(np.uint8)
            if t == F.Q4_1:
                w[:, b * bb + 2:b * bb + 4] = np.array([0x2A66], dtype=np.uint16).view(np.uint8)
    for t, name in ((F.F16, "f16"), (F.BF16, "bf16"), (F.Q4_0, "q4_0"), (F.Q4_1, "q4_1")):
        arrays[name + "_dequant"] = O.ref_dequant_rows(arrays[name + "_w"], t, 64)
    save("ref_dequant_formats.npz", **arrays)


def gen_down_axpy():
    arrays = {}
    for t, name, n_in, n in ((F.Q8_0, "q8_0", 96, 256), (F.F16, "f16", 40, 64),
                             (F.Q4_0, "q4_0", 72, 96)):
        if t == F.F16:
            vals = S.rng(0, "golden.axpy.f16").standard_normal(size=(n_in, n)).astype(np.float32)
            w = vals.astype(np.float16).view(np.uint8)
        elif t == F.Q4_0:
            g = S.rng(0, "golden.axpy.q4_0")
            w = g.integers(0, 256, size=(n_in, (n // 32) * 18), dtype=np.uint8)
            for b in range(n // 32):  # sane fp16 scales
                w[:, b * 18:b * 18 + 2] = np.array([0x2E66], dtype=np.uint16).view(np.uint8)
        else:
            w = S.weight(t, n_in, n, seed=0, name="golden.axpy." + name)
        x = S.activations_f32(3, n_in, seed=0, name="golden.axpy.x." + name)
        x[:, ::7] = 0.0       # rows the reference skips
        x[1, 5] = -0.0
        y0 = S.activations_f32(3, n, seed=1, name="golden.axpy.y." + name)
        y = y0.copy()
        O.ref_matmul_down_axpy(x, w, t, n, y)
        arrays.update({name + "_w": w, name + "_x": x, name + "_y0": y0, name + "_y": y})
    save("ref_down_axpy.npz", **arrays)


def kquant_edge_blocks(t):
    """Hand-made edge blocks: zero / subnormal / negative / largest scales."""
    bb = F.BLOCK[t][1]
    out = []
    def blank():
        return np.zeros(bb, dtype=np.uint8)
    def put16(b, off, v):
        b[off:off + 2] = np.array([v], dtype=np.uint16).view(np.uint8)
    if t == F.Q4_K:
        for d, dmin, sc, mn, code in ((0x0000, 0x0000, 63, 63, 0xFF), (0x0001, 0x03FF, 1, 63, 0x5A),
                                      (0xBC00, 0x3C00, 63, 0, 0xF0), (0x7BFF, 0x7BFF, 63, 63, 0xFF),
                                      (0x3C00, 0x8001, 17, 42, 0x0F)):
            b = blank()
            put16(b, 0, d)
            put16(b, 2, dmin)
            b[4:16] = S.pack_q4k_scales(np.full(8, sc), np.full(8, mn))
            b[16:] = code
            out.append(b)
        b = blank()  # every scale/min different, to pin the 12-byte packing
        put16(b, 0, 0x3C00)
        put16(b, 2, 0x3800)
        b[4:16] = S.pack_q4k_scales(np.array([1, 7, 15, 31, 32, 48, 61, 63]),
                                    np.array([63, 50, 33, 16, 8, 4, 2, 0]))
        b[16:] = np.arange(128, dtype=np.uint8) * 37
        out.append(b)
    else:
        for d, sc, ql, qh in ((0x0000, 127, 0xFF, 0xFF), (0x0001, -128, 0x00, 0x00),
                              (0xBC00, -1, 0xA5, 0x3C), (0x7BFF, 127, 0xFF, 0xFF),
                              (0x3C00, 0, 0x12, 0xE4)):
            b = blank()
            b[0:128] = ql
            b[128:192] = qh
            b[192:208] = np.full(16, sc, dtype=np.int8).view(np.uint8)
            put16(b, 208, d)
            out.append(b)
        b = blank()
        b[0:128] = np.arange(128, dtype=np.uint8) * 29
        b[128:192] = np.arange(64, dtype=np.uint8) * 53
        b[192:208] = np.arange(-8, 8, dtype=np.int8).view(np.uint8) * 9
        put16(b, 208, 0x3555)
        out.append(b)
    return np.stack(out)


def gen_kquant():
    from gguf import GGMLQuantizationType as GT
    from gguf.quants import dequantize
    arrays = {}
    for t, gt, name in ((F.Q4_K, GT.Q4_K, "q4_k"), (F.Q6_K, GT.Q6_K, "q6_k")):
        rnd = S.weight(t, 12, 256, seed=0, name=f"golden.{name}")
        edge = kquant_edge_blocks(t)
        blocks = np.concatenate([rnd, edge])
        deq = dequantize(blocks, gt).astype(np.float32).reshape(blocks.shape[0], 256)
        arrays[name + "_blocks"] = blocks
        arrays[name + "_dequant"] = deq
    import gguf
    meta = getattr(gguf, "__version__", None)
    if meta is None:
        from importlib.metadata import version
        meta = version("gguf")
    arrays["gguf_py_version"] = np.array(meta)
    save("gguf_kquant.npz", **arrays)


if __name__ == "__main__":
    if not O.have_ref():
        sys.exit("oracle/_ref/libftref.so missing: run make -C oracle where the reference exists")
    gens = {"q8_0_gemv": gen_q8_0_gemv, "test_quant": gen_test_quant, "chunker": gen_chunker,
            "expert_q8_0": gen_expert_q8_0, "formats": gen_formats, "kquant": gen_kquant,
            "down_axpy": gen_down_axpy}
    # `gen_golden.py name ...` regenerates only the named fixtures
    for key in sys.argv[1:] or list(gens):
        gens[key]()
