"""FP8 (e4m3) KV-pool restatement (test infrastructure only).

The FP8 pool is an opt-in storage mode of this library with no counterpart in
the reference (whose pool holds the activation dtype, kv_cache.py:20-22), so
its stored bytes are pinned against this numpy restatement of the format
(include/pagedkv.h, "FP8 (e4m3) KV pool"), which tests/test_oracle_golden.py
cross-checks against torch's float8_e4m3fn conversion:

  scale = amax / 448, e = RNE(x * (448 / amax)) saturated to +-448, with
  amax = max |x| over the 128 values of one token and KV head (x = k after
  the reference's bf16 RoPE, or v), each quotient one fp32 division; an
  all-zero row stores zeros and scale 1.  A row reads back as e * scale.

Chunk layout per (16-token block, KV head), 4224 bytes: K rows of 128 bytes
(16-byte group c of token t at group c ^ (t & 7), byte 4i+u of a group holds
element 2i+u for u < 2, 2i+8+u-2 for u >= 2), V transposed (128 dim rows of
16 token bytes, same in-group order), fp32 K scales, fp32 V scales.
"""
from __future__ import annotations

import numpy as np

CHUNK = 4224
V_OFF, KS_OFF, VS_OFF = 2048, 4096, 4160
F32 = np.float32


def fp8_pos(e):
    """Byte position inside a 16-byte group of element e (0..15)."""
    e = np.asarray(e)
    return np.where(e < 8, 4 * (e >> 1) + (e & 1), 4 * ((e - 8) >> 1) + 2 + (e & 1))


def e4m3_encode(x) -> np.ndarray:
    """fp32 -> e4m3 bit patterns, round to nearest even, saturating to +-448
    (finite values only)."""
    x = np.asarray(x, F32)
    sign = np.signbit(x).astype(np.uint8) << 7
    a = np.abs(x).astype(np.float64)
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.maximum(e, -6.0)                     # below 2^-6: subnormal quantum 2^-9
    q = np.exp2(e - 3.0)
    r = np.minimum(np.rint(a / q) * q, 448.0)   # exact: q is a power of two
    with np.errstate(divide="ignore"):
        er = np.floor(np.log2(np.where(r > 0, r, 1.0)))
    normal = r >= 2.0 ** -6
    mant_n = np.rint(r / np.exp2(er) * 8.0 - 8.0)
    code_n = ((er + 7.0).astype(np.int64) << 3) | mant_n.astype(np.int64)
    code_s = np.rint(r / 2.0 ** -9).astype(np.int64)
    code = np.where(normal, code_n, code_s).astype(np.uint8)
    return code | sign


def e4m3_decode(b) -> np.ndarray:
    b = np.asarray(b, np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 7
    v = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    return (s * v).astype(F32)


def quantize_rows(x):
    """x [..., 128] fp32 (bf16 values) -> (e4m3 bytes [..., 128], scale [...])."""
    x = np.asarray(x, F32)
    amax = np.abs(x).max(axis=-1).astype(F32)
    pos = amax > 0
    inv = np.where(pos, F32(448.0) / np.where(pos, amax, F32(1)), F32(0)).astype(F32)
    scale = np.where(pos, amax / F32(448.0), F32(1)).astype(F32)
    y = (x * inv[..., None]).astype(F32)
    return e4m3_encode(y), scale


def write_token(chunk: np.ndarray, tok: int, k_row, v_row) -> None:
    """Store one token's quantised K and V rows into a 4224-byte chunk."""
    kb, ks = quantize_rows(k_row)
    vb, vs = quantize_rows(v_row)
    d = np.arange(128)
    koff = tok * 128 + (((d >> 4) ^ (tok & 7)) << 4) + fp8_pos(d & 15)
    chunk[koff] = kb
    chunk[V_OFF + d * 16 + int(fp8_pos(tok & 15))] = vb
    chunk[KS_OFF + 4 * tok:KS_OFF + 4 * tok + 4] = np.frombuffer(np.float32(ks).tobytes(), np.uint8)
    chunk[VS_OFF + 4 * tok:VS_OFF + 4 * tok + 4] = np.frombuffer(np.float32(vs).tobytes(), np.uint8)


def read_token(chunk: np.ndarray, tok: int):
    """(K row, V row) of one token as fp32 e4m3 * scale."""
    d = np.arange(128)
    koff = tok * 128 + (((d >> 4) ^ (tok & 7)) << 4) + fp8_pos(d & 15)
    kb = chunk[koff]
    vb = chunk[V_OFF + d * 16 + int(fp8_pos(tok & 15))]
    ks = np.frombuffer(chunk[KS_OFF + 4 * tok:KS_OFF + 4 * tok + 4].tobytes(), F32)[0]
    vs = np.frombuffer(chunk[VS_OFF + 4 * tok:VS_OFF + 4 * tok + 4].tobytes(), F32)[0]
    return e4m3_decode(kb) * ks, e4m3_decode(vb) * vs


def gather_rows(pool8_layer: np.ndarray, table, n: int, h: int):
    """K, V [n, 128] (fp32, dequantised) of one row's first n positions for KV
    head h, read through its block table (slot of position p: table[p // 16],
    token p % 16)."""
    p = np.arange(n)
    tok = p % 16
    chunks = np.ascontiguousarray(pool8_layer[np.asarray(table)[p // 16], h])  # [n, CHUNK]
    d = np.arange(128)
    koff = tok[:, None] * 128 + (((d >> 4)[None, :] ^ (tok[:, None] & 7)) << 4) + fp8_pos(d & 15)[None, :]
    voff = V_OFF + d[None, :] * 16 + fp8_pos(tok)[:, None]
    kb = np.take_along_axis(chunks, koff, axis=1)
    vb = np.take_along_axis(chunks, voff, axis=1)
    ks = np.ascontiguousarray(chunks[:, KS_OFF:KS_OFF + 64]).view(F32)[p, tok]
    vs = np.ascontiguousarray(chunks[:, VS_OFF:VS_OFF + 64]).view(F32)[p, tok]
    return e4m3_decode(kb) * ks[:, None], e4m3_decode(vb) * vs[:, None]
