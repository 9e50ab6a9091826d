"""CPU checks of the FP8 pool restatement (oracle/fp8_ref.py): its e4m3
rounding agrees with torch's float8_e4m3fn conversion bit for bit (round to
nearest even, ties included), and a chunk written then read returns each row
within half an e4m3 step."""
import numpy as np
import torch

from oracle import fp8_ref


def test_e4m3_encode_matches_torch_float8():
    rng = np.random.default_rng(0)
    x = rng.standard_normal(100000).astype(np.float32)
    x *= np.exp2(rng.integers(-14, 9, x.size)).astype(np.float32)
    x = np.clip(x, -448, 448)
    # exact ties between neighbouring e4m3 values, both signs, and the edges
    ties = np.array([1.0625, 1.1875, 2 ** -9 * 2.5, 2 ** -9 * 1.5, 3 * 2 ** -10, 440.0,
                     -1.0625, 0.0, -0.0, 448.0, 2 ** -6, 2 ** -6 * 0.9375], np.float32)
    x = np.concatenate([x, ties])
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(fp8_ref.e4m3_encode(x), want)
    back = torch.from_numpy(want).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(fp8_ref.e4m3_decode(want), back)


def test_chunk_round_trip_and_layout():
    rng = np.random.default_rng(1)
    chunk = np.zeros(fp8_ref.CHUNK, np.uint8)
    K = rng.standard_normal((16, 128)).astype(np.float32)
    V = rng.standard_normal((16, 128)).astype(np.float32)
    K[3] = 0.0  # an all-zero row: zeros with scale 1
    for t in range(16):
        fp8_ref.write_token(chunk, t, K[t], V[t])
    for t in range(16):
        k, v = fp8_ref.read_token(chunk, t)
        for x, y in ((k, K[t]), (v, V[t])):
            step = np.abs(y).max() / 448 * 32  # e4m3 spacing at the top binade
            assert np.abs(x - y).max() <= step / 2 + 1e-12
    assert np.frombuffer(chunk[fp8_ref.KS_OFF + 12:fp8_ref.KS_OFF + 16].tobytes(), np.float32)[0] == 1
    # the in-group byte order is a permutation of 0..15
    assert sorted(fp8_ref.fp8_pos(np.arange(16)).tolist()) == list(range(16))
