"""The engine-side GGUF reader (ft::Gguf, xwfes_b200/host/gguf.cpp), which
loads the K-quant tensors (Q4_K, Q6_K) the reference's reader rejects
(ft/src/gguf.cpp:129-137).  Files are written by tests/gguf_write.py; a
small C++ probe (tests/cpp/test_gguf.cpp) prints what the reader sees.  CPU
only."""
import os
import subprocess

import numpy as np
import pytest

import gguf_write as G
from xwfes_b200 import formats as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "xwfes_b200", "host")


@pytest.fixture(scope="module")
def probe(tmp_path_factory):
    from oracle import oracle as O
    O.lib()  # builds oracle/liboracle.so if needed
    exe = str(tmp_path_factory.mktemp("gguf") / "test_gguf")
    odir = os.path.join(ROOT, "oracle")
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-I", os.path.join(HOST, "compat"), "-I", odir,
           os.path.join(ROOT, "tests", "cpp", "test_gguf.cpp"), os.path.join(HOST, "gguf.cpp"),
           "-L", odir, "-loracle", "-Wl,-rpath," + odir, "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr

    def run(path, *args):
        p = subprocess.run([exe, str(path), *args], capture_output=True, text=True, timeout=60)
        return p.returncode, p.stdout.strip()
    return run


def fnv1a(b):
    h = 1469598103934665603
    for x in b:
        h = ((h ^ x) * 1099511628211) & (2 ** 64 - 1)
    return h


GGML = {"F32": 0, "F16": 1, "Q4_0": 2, "Q4_1": 3, "Q8_0": 8, "Q4_K": 12, "Q6_K": 14, "BF16": 30}
BLOCK = {"F32": (1, 4), "F16": (1, 2), "BF16": (1, 2), "Q4_0": (32, 18), "Q4_1": (32, 20),
         "Q8_0": (32, 34), "Q4_K": (256, 144), "Q6_K": (256, 210)}


def tensor(name, dtype, dims, seed):
    eb, bb = BLOCK[dtype]
    n = dims[0] // eb * bb * int(np.prod(dims[1:]))
    raw = np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8).tobytes()
    return (name, dims, GGML[dtype], raw)


TENSORS = [tensor("a.f32", "F32", (7, 3), 1), tensor("b.f16", "F16", (64, 2), 2),
           tensor("c.bf16", "BF16", (16,), 3), tensor("d.q8_0", "Q8_0", (64, 5), 4),
           tensor("e.q4_0", "Q4_0", (96, 2), 5), tensor("f.q4_1", "Q4_1", (32, 3), 6),
           tensor("g.q4_k", "Q4_K", (512, 3), 7), tensor("h.q6_k_exps", "Q6_K", (256, 2, 4), 8)]
KV = [("general.name", G.STR, "tiny"), ("x.u8", G.U8, 250), ("x.i8", G.I8, -7),
      ("x.u16", G.U16, 65000), ("x.i16", G.I16, -300), ("x.u32", G.U32, 4000000000),
      ("x.i32", G.I32, -123456), ("x.f32", G.F32, 0.25), ("x.bool", G.BOOL, 1),
      ("x.u64", G.U64, 2 ** 40 + 3), ("x.i64", G.I64, -(2 ** 40)), ("x.f64", G.F64, 1.0 / 3),
      ("tok.list", G.ARR, (G.STR, ["<s>", "hello", ""])),
      ("arr.f32", G.ARR, (G.F32, [0.5, -2.0, 3.25])), ("arr.i32", G.ARR, (G.I32, [1, -2, 3]))]


@pytest.mark.parametrize("alignment", [32, 64])
def test_tensors_round_trip(tmp_path, probe, alignment):
    kv = KV + ([("general.alignment", G.U32, alignment)] if alignment != 32 else [])
    path = G.write_gguf(tmp_path / "m.gguf", kv, TENSORS, alignment=alignment)
    rc, out = probe(path, "tensors")
    assert rc == 0, out
    lines = {ln.split()[0]: ln.split()[1:] for ln in out.splitlines()}
    assert set(lines) == {t[0] for t in TENSORS}
    for name, dims, gt, raw in TENSORS:
        nd, n0, n1, n2, n3, dt, nbytes, off, h = lines[name]
        full = list(dims) + [1] * (4 - len(dims))
        assert int(nd) == len(dims) and [int(n0), int(n1), int(n2), int(n3)] == full, name
        assert int(dt) == gt and int(nbytes) == len(raw) and int(h) == fnv1a(raw), name
        assert int(off) % alignment == 0
    # the K-quant row and plane geometry the backend relies on
    assert int(lines["g.q4_k"][6]) == F.row_bytes(F.Q4_K, 512) * 3
    assert int(lines["h.q6_k_exps"][6]) == F.row_bytes(F.Q6_K, 256) * 2 * 4


def test_metadata(tmp_path, probe):
    path = G.write_gguf(tmp_path / "m.gguf", KV, TENSORS[:1])
    q = lambda *a: probe(path, *a)
    assert q("str", "general.name") == (0, "tiny")
    assert q("str", "missing") == (0, "<default>")
    for key, want in [("x.u8", 250), ("x.i8", -7), ("x.u16", 65000), ("x.i16", -300),
                      ("x.u32", 4000000000), ("x.i32", -123456), ("x.u64", 2 ** 40 + 3),
                      ("x.i64", -(2 ** 40)), ("missing", -12345)]:
        assert q("i64", key) == (0, str(want)), key
    assert float(q("f64", "x.f32")[1]) == 0.25
    assert float(q("f64", "x.f64")[1]) == 1.0 / 3
    assert q("bool", "x.bool") == (0, "1") and q("bool", "missing") == (0, "0")
    assert q("has", "x.u8") == (0, "1") and q("has", "nope") == (0, "0")
    assert q("str_arr", "tok.list")[1].split("\n")[:2] == ["<s>", "hello"]
    assert [float(v) for v in q("f32_arr", "arr.f32")[1].split()] == [0.5, -2.0, 3.25]
    assert q("i32_arr", "arr.i32")[1].split() == ["1", "-2", "3"]
    rc, out = q("i64", "general.name")  # a string is not a number
    assert rc == 2 and "is not a number" in out


def test_version_2_accepted(tmp_path, probe):
    path = G.write_gguf(tmp_path / "v2.gguf", KV[:2], TENSORS[:2], version=2)
    assert probe(path, "tensors")[0] == 0


@pytest.mark.parametrize("case,needle", [
    ("magic", "not a GGUF file"), ("version", "unsupported version"),
    ("truncated", "truncated"), ("dtype", "unsupported tensor type 10"),
    ("outside", "lies outside the file"), ("blocks", "not whole blocks"),
    ("alignment", "power of two")])
def test_damaged_files_are_rejected(tmp_path, probe, case, needle):
    kv, tensors, kw = list(KV[:3]), [TENSORS[6]], {}
    if case == "magic":
        kw["magic"] = 0x12345678
    elif case == "version":
        kw["version"] = 1
    elif case == "dtype":
        name, dims, _, raw = tensors[0]
        tensors = [(name, dims, 10, raw)]  # Q2_K
    elif case == "outside":
        kw["offsets"] = [1 << 20]
    elif case == "blocks":
        name, _, gt, raw = tensors[0]
        tensors = [(name, (300, 3), gt, raw)]
    elif case == "alignment":
        kv.append(("general.alignment", G.U32, 48))
    data = G.gguf_bytes(kv, tensors, **kw)
    if case == "truncated":
        data = data[:60]
    path = tmp_path / f"{case}.gguf"
    path.write_bytes(data)
    rc, out = probe(path, "tensors")
    assert rc == 2 and needle in out, out


def test_kquant_rows_through_the_reader_view(tmp_path, probe, oracle):
    """A Q4_K matrix and a 3-D Q6_K expert tensor with real block contents
    (finite scales): rows read through the reader's slice / row-stride view
    dequantize (oracle) exactly as the same rows taken from the written
    bytes."""
    from xwfes_b200 import synth as S
    q4 = S.weight(F.Q4_K, 3, 512, seed=11, name="gg.q4")               # [3][2 x 144]
    q6 = np.stack([S.weight(F.Q6_K, 2, 256, seed=12 + e, name=f"gg.q6.{e}") for e in range(4)])
    tensors = [("q4", (512, 3), GGML["Q4_K"], q4.tobytes()),
               ("q6_exps", (256, 2, 4), GGML["Q6_K"], q6.tobytes())]
    path = G.write_gguf(tmp_path / "k.gguf", KV[:1], tensors)
    for name, arr, t, k, planes, rows in (("q4", q4[None], F.Q4_K, 512, 1, 3),
                                          ("q6_exps", q6, F.Q6_K, 256, 4, 2)):
        for p in range(planes):
            for r in range(rows):
                rc, out = probe(path, "dequant", name, str(p), str(r))
                assert rc == 0, out
                want = oracle.dequant_rows(np.ascontiguousarray(arr[p][r:r + 1]), t, k)
                assert int(out) == fnv1a(np.asarray(want, np.float32).tobytes()), (name, p, r)
