"""The product scheduler (chat.py on the device-table cache) makes exactly the
reference scheduler's decisions: replayed tick by tick against the reference's
recorded trace (tests/golden/scheduler_trace.json) it admits, defers, rejects,
evicts, prefills, decodes, trims and releases identically -- same model calls
(rows, T, token ids), same LRU order, same free-block counts and block tables."""
import json

import torch

from oracle.scheduler_trace import run_trace


def test_scheduler_matches_reference_trace(golden):
    import chat
    from kv_cache import BlockTables

    fx = json.loads((golden / "scheduler_trace.json").read_text())
    saved = chat.DEVICE
    chat.DEVICE = torch.device("cpu")  # the fake model runs on the host
    try:
        got = run_trace(chat, lambda n: chat.init(kv_cache=BlockTables(n, 16), start_worker=False))
    finally:
        chat.DEVICE = saved
        chat._kv_cache = None
    assert len(got["trace"]) == len(fx["trace"])
    for mine, ref in zip(got["trace"], fx["trace"]):
        assert mine == ref, f"tick {ref['tick']} differs"
    assert got["replies"] == fx["replies"]


def test_mixed_prefill_mode_keeps_replies_and_block_accounting(golden):
    """Opt-in mixed ticks (chat.MIXED_PREFILL_MIN_TOKENS): a long enough prompt
    admitted while other jobs decode shares their forward (model.forward_mixed).
    The fake model's next token depends only on (sequence id, length), so
    every reply must still equal the reference scheduler's; blocks are
    conserved at every tick, and only prompts at the threshold go mixed."""
    import chat
    from kv_cache import BlockTables

    fx = json.loads((golden / "scheduler_trace.json").read_text())
    saved = chat.DEVICE, chat.MIXED_PREFILL_MIN_TOKENS
    chat.DEVICE = torch.device("cpu")
    try:
        for threshold, want_mixed in ((1, 5), (80, 2)):
            chat.MIXED_PREFILL_MIN_TOKENS = threshold
            chat._mixed.clear()
            got = run_trace(chat, lambda n: chat.init(kv_cache=BlockTables(n, 16),
                                                      start_worker=False))
            mixed = [c for t in got["trace"] for c in t["calls"] if c.get("mixed")]
            assert len(mixed) == want_mixed
            for c in mixed:
                assert c["T"] >= threshold and c["seqs"] and c["prefill_seq"] not in c["seqs"]
            for t in got["trace"]:
                held = sum(len(b) for b in t["tables"].values())
                assert held + t["free"] == 14, f"tick {t['tick']}"
                # never more than one mixed forward per tick
                assert sum(1 for c in t["calls"] if c.get("mixed")) <= 1
            assert got["replies"] == fx["replies"]
            assert not chat._mixed
    finally:
        chat.DEVICE, chat.MIXED_PREFILL_MIN_TOKENS = saved
        chat._mixed.clear()
        chat._kv_cache = None


def test_installing_a_new_cache_forgets_resident_sequences():
    """chat.init with a new pool: resident chats drop their sequence ids (the
    K/V lived in the old pool) so a later eviction never frees an id in the
    new pool; refused while a message is in flight."""
    import pytest

    import chat
    from kv_cache import BlockTables
    from oracle.scheduler_trace import FakeTokenizer

    try:
        old = chat.init(kv_cache=BlockTables(8, 16), start_worker=False)
        c = chat.Chat(FakeTokenizer())
        c.seq = old.alloc()
        chat._resident.append(c)
        chat.init(kv_cache=BlockTables(8, 16), start_worker=False)
        assert c.seq is None and not chat._resident
        chat.active.append(object())
        with pytest.raises(RuntimeError, match="in flight"):
            chat.init(kv_cache=BlockTables(8, 16), start_worker=False)
    finally:
        chat.active.clear()
        chat._resident.clear()
        chat._kv_cache = None
