"""Seeded synthetic weights and activations with the benchmark configs' shapes
and value distributions.

No real checkpoint or dataset is used; every tensor is drawn from a seeded
numpy ``PCG64`` stream, one independent stream per (seed, tensor name).

* Q8_0 (config 1): per block draw 32 values ~ N(0, 0.02), set
  ``d = fp16(max|w| / 127)``, then codes iid uniform in [-127, 127].
* Q4_K (configs 2-5): ``d``, ``dmin`` = fp16(|N(0, 0.01)|); 6-bit scales and
  mins uniform in [0, 63], packed into the 12-byte field; codes uniform in
  [0, 15] (uniform code bytes).
* Q6_K (head of config 2): ``d`` = fp16(|N(0, 0.01)|); int8 scales uniform in
  [-128, 127]; 6-bit codes uniform in [0, 63] (uniform ql / qh bytes).
* Activations: fp32 N(0, 1); bf16 ones are the fp32 draws rounded to nearest
  even.
"""
import zlib

import numpy as np

from . import formats as F


def rng(seed, name):
    """Independent generator for tensor ``name`` under ``seed``."""
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence(
        [int(seed) & 0xFFFFFFFF, zlib.crc32(name.encode())])))


def _fp16_bits(a):
    return np.asarray(a, dtype=np.float32).astype(np.float16).view(np.uint16)


def pack_q4k_scales(sc, mn):
    """Pack 6-bit scales ``sc[..., 8]`` and mins ``mn[..., 8]`` into the
    12-byte Q4_K field (the inverse of the decoder's unpacking)."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.zeros(sc.shape[:-1] + (12,), dtype=np.uint8)
    out[..., 0:4] = sc[..., 0:4] | ((sc[..., 4:8] >> 4) << 6)
    out[..., 4:8] = mn[..., 0:4] | ((mn[..., 4:8] >> 4) << 6)
    out[..., 8:12] = (sc[..., 4:8] & 0x0F) | ((mn[..., 4:8] & 0x0F) << 4)
    return out


def q8_0_blocks(nblocks, seed=0, name="w"):
    g = rng(seed, name + ".q8_0")
    w = g.normal(0.0, 0.02, size=(nblocks, 32)).astype(np.float32)
    d = (np.abs(w).max(axis=1) / np.float32(127)).astype(np.float32)
    blk = np.empty((nblocks, 34), dtype=np.uint8)
    blk[:, 0:2] = _fp16_bits(d).reshape(-1, 1).view(np.uint8).reshape(nblocks, 2)
    blk[:, 2:] = g.integers(-127, 128, size=(nblocks, 32), dtype=np.int8).view(np.uint8)
    return blk


def q4_k_blocks(nblocks, seed=0, name="w"):
    g = rng(seed, name + ".q4_k")
    d = np.abs(g.normal(0.0, 0.01, size=nblocks)).astype(np.float32)
    dmin = np.abs(g.normal(0.0, 0.01, size=nblocks)).astype(np.float32)
    sc = g.integers(0, 64, size=(nblocks, 8), dtype=np.uint8)
    mn = g.integers(0, 64, size=(nblocks, 8), dtype=np.uint8)
    blk = np.empty((nblocks, 144), dtype=np.uint8)
    blk[:, 0:2] = _fp16_bits(d).view(np.uint8).reshape(nblocks, 2)
    blk[:, 2:4] = _fp16_bits(dmin).view(np.uint8).reshape(nblocks, 2)
    blk[:, 4:16] = pack_q4k_scales(sc, mn)
    blk[:, 16:] = g.integers(0, 256, size=(nblocks, 128), dtype=np.uint8)
    return blk


def q6_k_blocks(nblocks, seed=0, name="w"):
    g = rng(seed, name + ".q6_k")
    d = np.abs(g.normal(0.0, 0.01, size=nblocks)).astype(np.float32)
    blk = np.empty((nblocks, 210), dtype=np.uint8)
    blk[:, 0:192] = g.integers(0, 256, size=(nblocks, 192), dtype=np.uint8)
    blk[:, 192:208] = g.integers(-128, 128, size=(nblocks, 16), dtype=np.int8).view(np.uint8)
    blk[:, 208:210] = _fp16_bits(d).view(np.uint8).reshape(nblocks, 2)
    return blk


_BLOCK_GEN = {F.Q8_0: q8_0_blocks, F.Q4_K: q4_k_blocks, F.Q6_K: q6_k_blocks}


def weight(dtype, n, k, seed=0, name="w"):
    """GGUF-layout weight ``W[n][k]`` as a uint8 array ``[n, row_bytes]``."""
    t = F.dtype_id(dtype)
    eb, bb = F.BLOCK[t]
    if k % eb:
        raise ValueError(f"K={k} is not a multiple of the {F.NAMES[t]} block ({eb})")
    blocks = _BLOCK_GEN[t](n * (k // eb), seed=seed, name=name)
    return blocks.reshape(n, (k // eb) * bb)


def expert_weights(dtype, n_exp, n, k, seed=0, name="w"):
    """``n_exp`` stacked planes ``[n_exp, n, row_bytes]`` (GGUF ``*_exps``)."""
    return np.stack([weight(dtype, n, k, seed, f"{name}.{e}") for e in range(n_exp)])


def activations_f32(m, k, seed=0, name="x"):
    return rng(seed, name + ".f32").standard_normal(size=(m, k), dtype=np.float32)


def f32_to_bf16_bits(a):
    """Round fp32 to bf16 (nearest even); returns the uint16 bit patterns."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_bits_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def activations_bf16(m, k, seed=0, name="x"):
    """bf16 N(0,1) activations as uint16 bit patterns ``[m, k]``."""
    return f32_to_bf16_bits(activations_f32(m, k, seed, name))


def router_logits(t, e, seed=0, name="router"):
    return rng(seed, name + ".logits").standard_normal(size=(t, e), dtype=np.float32)
