"""Temperature sampling as the device sampler draws it, restated in numpy
(test oracle).

TEST INFRASTRUCTURE ONLY.  The reference samples with
`torch.multinomial(F.softmax(logits.float() / T, dim=-1), 1)` (chat.py:103-107),
which draws from the categorical softmax(logits / T) with torch's generator.
The product's pkv_sample draws from the same categorical by the Gumbel-max
trick, with its own counter-based noise, so the reference's draws cannot be
reproduced id for id; two things are checked instead:
  * this restatement of the product's draw (same noise, same arithmetic up
    to the rounding of a fast log) against the kernel, id for id;
  * the kernel's empirical frequencies against softmax(logits / T), the
    reference's distribution (tests/test_sample_gpu.py).

Philox-4x32-10 follows J. Salmon, M. Moraes, R. Dror, D. Shaw, "Parallel
random numbers: as easy as 1, 2, 3" (SC'11): per round, with multipliers
M0, M1 and key (k0, k1), (c0, c1, c2, c3) -> (hi(M1*c2) ^ c1 ^ k0,
lo(M1*c2), hi(M0*c0) ^ c3 ^ k1, lo(M0*c0)); the key is bumped by the Weyl
constants W0, W1 between rounds.  Pinned by the known-answer vectors the
paper's Random123 distribution publishes (tests/test_oracle_golden.py).
"""
from __future__ import annotations

import numpy as np

M0, M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
W0, W1 = 0x9E3779B9, 0xBB67AE85
MASK32 = np.uint64(0xFFFFFFFF)


def philox4x32_10(ctr: np.ndarray, key: tuple[int, int]) -> np.ndarray:
    """ctr: uint32 [..., 4] -> uint32 [..., 4] (vectorised over leading dims)."""
    c = [ctr[..., i].astype(np.uint64) for i in range(4)]
    k0, k1 = key[0] & 0xFFFFFFFF, key[1] & 0xFFFFFFFF
    for _ in range(10):
        p0 = M0 * c[0]
        p1 = M1 * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & MASK32
        hi1, lo1 = p1 >> np.uint64(32), p1 & MASK32
        c = [hi1 ^ c[1] ^ np.uint64(k0), lo1, hi0 ^ c[3] ^ np.uint64(k1), lo0]
        k0 = (k0 + W0) & 0xFFFFFFFF
        k1 = (k1 + W1) & 0xFFFFFFFF
    return np.stack([x.astype(np.uint32) for x in c], axis=-1)


def gumbel(bits: np.ndarray) -> np.ndarray:
    """Gumbel(0, 1) from uint32 bits, float64: G = -ln E, E = -ln(1 - V),
    V = (bits >> 9) / 2^23 + 2^-24; E from the series V + V^2/2 + V^3/3 + V^4/4
    where V < 1/16 (as the kernel does), from the log elsewhere."""
    v = (bits >> np.uint32(9)).astype(np.float64) / 8388608.0 + 1.0 / 16777216.0
    v = v.astype(np.float32).astype(np.float64)  # exact in fp32 (as on the device)
    series = v * (1.0 + v * (0.5 + v * (0.3333333432674408 + v * 0.25)))
    e = np.where(v < 0.0625, series, -np.log1p(-v))
    return -np.log(e)


def scores(logits: np.ndarray, temperature: float, seed: int, call: int) -> np.ndarray:
    """float64 [rows, vocab]: logits / T + Gumbel noise of (seed, call, row, element)."""
    rows, vocab = logits.shape
    quads = (vocab + 3) // 4
    q = np.arange(quads, dtype=np.uint32)
    r = np.arange(rows, dtype=np.uint32)
    ctr = np.zeros((rows, quads, 4), dtype=np.uint32)
    ctr[..., 0] = q[None, :]
    ctr[..., 1] = r[:, None]
    ctr[..., 2] = np.uint32(call & 0xFFFFFFFF)
    ctr[..., 3] = np.uint32((call >> 32) & 0xFFFFFFFF)
    bits = philox4x32_10(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    g = gumbel(bits.reshape(rows, quads * 4))[:, :vocab]
    inv_t = float(np.float32(1.0) / np.float32(temperature))
    return logits.astype(np.float64) * inv_t + g


def sample(logits: np.ndarray, temperature: float, seed: int, call: int) -> np.ndarray:
    """int64 [rows]: argmax of scores(), lower index on ties; -1 for a row
    without a finite score."""
    s = scores(logits, temperature, seed, call)
    s = np.where(np.isnan(s), -np.inf, s)
    ids = np.argmax(s, axis=1)
    best = s[np.arange(s.shape[0]), ids]
    return np.where(np.isfinite(best), ids, -1)
