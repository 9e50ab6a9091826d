"""pkv_sample, the device sampler behind chat.py's _sample (reference
chat.py:103-107: softmax(logits.float() / T) then torch.multinomial).

It draws from the same categorical distribution with its own counter-based
noise, so the checks are: the kernel's ids equal the CPU restatement of its
draw (oracle/sample_ref.py) id for id; its frequencies match softmax(logits /
T); the same (seed, call) repeats; degenerate rows come back as -1 and
chat._sample raises on them as torch.multinomial does."""
import numpy as np
import pytest
import torch

from oracle.sample_ref import sample as ref_sample
from oracle.sample_ref import scores as ref_scores

pytestmark = pytest.mark.gpu


def _lib():
    import pagedkv

    return pagedkv


@pytest.mark.parametrize("rows,vocab,ld,dtype,temp", [
    (4, 151936, 151936, torch.bfloat16, 1.0),   # the model's vocabulary, a decode step
    (64, 151936, 151936, torch.bfloat16, 0.7),
    (1, 151936, 151936, torch.bfloat16, 1.0),   # a prompt's first token
    (3, 1001, 1008, torch.float32, 1.0),        # ragged vocab, padded rows
    (5, 37, 37, torch.bfloat16, 2.0),           # rows not 4-element aligned: scalar loads
    (300, 4096, 4096, torch.float32, 1.0),
])
def test_sample_matches_oracle(cuda, rows, vocab, ld, dtype, temp):
    pk = _lib()
    g = torch.Generator().manual_seed(rows * 7 + vocab)
    full = (3.0 * torch.randn(rows, ld, generator=g)).to(dtype)
    logits = full.to(cuda)[:, :vocab]
    seed, call = 0x1234_5678_9ABC, 17
    got = pk.sample(logits, temp, seed=seed, call=call).cpu().numpy()
    x = full[:, :vocab].float().numpy()
    want = ref_sample(x, temp, seed, call)
    diff = np.nonzero(got != want)[0]
    if diff.size:  # only near-ties may differ (a fast log on the device)
        s = ref_scores(x, temp, seed, call)
        for r in diff:
            assert got[r] >= 0 and abs(s[r, got[r]] - s[r, want[r]]) < 1e-4, (r, got[r], want[r])
    assert diff.size <= max(1, rows // 100)


@pytest.mark.parametrize("temp", [1.0, 0.5])
def test_sample_frequencies_follow_softmax(cuda, temp):
    pk = _lib()
    base = torch.tensor([1.5, 0.0, -1.0, 2.0, 0.5, -3.0, 1.0, 0.25])
    logits = base.repeat(4096, 1).to(cuda)
    ids = torch.cat([pk.sample(logits, temp, seed=99, call=c) for c in range(8)]).cpu().numpy()
    p = torch.softmax(base / temp, 0).numpy()
    freq = np.bincount(ids, minlength=8) / ids.size
    sigma = np.sqrt(p * (1 - p) / ids.size)
    assert np.all(np.abs(freq - p) < 5 * sigma + 1e-3), (freq, p)


def test_sample_degenerate_rows(cuda):
    pk = _lib()
    V = 1000
    x = torch.randn(6, V)
    x[0] = -float("inf")
    x[0, 321] = 0.0                 # one finite logit: always that one
    x[1] = -1e9
    x[1, 5] = 0.0                   # the scheduler tests' one-hot logits
    x[2] = -float("inf")            # nothing finite
    x[3] = float("nan")             # nothing finite
    x[4, 17] = float("nan")         # one NaN among finite logits: never drawn
    x[5, 2] = float("inf")          # +inf: softmax is NaN in the reference
    for dtype in (torch.float32, torch.bfloat16):
        for call in range(20):
            ids = pk.sample(x.to(dtype).to(cuda), 1.0, seed=5, call=call).tolist()
            assert ids[0] == 321 and ids[1] == 5
            assert ids[2] == -1 and ids[3] == -1 and ids[5] == -1
            assert 0 <= ids[4] < V and ids[4] != 17


def test_sample_is_reproducible_per_seed_and_call(cuda):
    pk = _lib()
    logits = torch.randn(64, 151936, device=cuda).to(torch.bfloat16)
    a = pk.sample(logits, 1.0, seed=7, call=3)
    b = pk.sample(logits, 1.0, seed=7, call=3)
    c = pk.sample(logits, 1.0, seed=7, call=4)
    d = pk.sample(logits, 1.0, seed=8, call=3)
    assert torch.equal(a, b)
    assert not torch.equal(a, c) and not torch.equal(a, d)
    # default keys come from torch's generator: torch.manual_seed repeats them
    torch.manual_seed(11)
    e = [pk.sample(logits).tolist() for _ in range(3)]
    torch.manual_seed(11)
    f = [pk.sample(logits).tolist() for _ in range(3)]
    assert e == f and e[0] != e[1]


def test_chat_sample_uses_device_sampler_and_raises_like_multinomial(cuda):
    import chat

    logits = torch.zeros(3, 500, device=cuda, dtype=torch.bfloat16)
    logits[1, 42] = 50.0
    ids = chat._sample(logits)
    assert len(ids) == 3 and ids[1] == 42 and all(0 <= i < 500 for i in ids)
    bad = logits.clone()
    bad[2] = float("nan")
    with pytest.raises(RuntimeError, match="probability tensor"):
        chat._sample(bad)
