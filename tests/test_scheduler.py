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


def test_chunked_mixed_prefill_keeps_replies_and_block_accounting(golden):
    """Opt-in chunked prefill (chat.MIXED_PREFILL_CHUNK with mixed ticks): a
    mixed prompt longer than the chunk runs as near-equal chunks on
    consecutive ticks, each in that tick's decode forward, its rows
    appended after the ones before.  Replies still equal the reference
    scheduler's (the fake model's token depends on sequence id and length
    only, and a prompt's first token comes from its last chunk, so a lost or
    repeated chunk would change every later token of that chat); blocks are
    conserved at every tick; a prompt's chunks are near-equal and within the
    limit."""
    import chat
    from kv_cache import BlockTables

    fx = json.loads((golden / "scheduler_trace.json").read_text())
    saved = chat.DEVICE, chat.MIXED_PREFILL_MIN_TOKENS, chat.MIXED_PREFILL_CHUNK
    chat.DEVICE = torch.device("cpu")
    try:
        for threshold, chunk in ((1, 8), (40, 16), (80, 1000)):
            chat.MIXED_PREFILL_MIN_TOKENS, chat.MIXED_PREFILL_CHUNK = threshold, chunk
            chat._mixed.clear()
            got = run_trace(chat, lambda n: chat.init(kv_cache=BlockTables(n, 16),
                                                      start_worker=False))
            # one prompt is in flight at a time: consecutive mixed calls of a
            # sequence are the chunks of one prompt
            prompts = []
            for c in (c for t in got["trace"] for c in t["calls"] if c.get("mixed")):
                assert c["prefill_seq"] not in c["seqs"] and 1 <= c["T"] <= chunk
                if prompts and prompts[-1][0] == c["prefill_seq"]:
                    prompts[-1][1].append(c["T"])
                else:
                    prompts.append((c["prefill_seq"], [c["T"]]))
            assert prompts
            for _, parts in prompts:
                assert max(parts) - min(parts) <= 1  # near-equal chunks
            if chunk < threshold + 40:
                assert any(len(p) > 1 for _, p in prompts), "no prompt was chunked"
            for t in got["trace"]:
                held = sum(len(b) for b in t["tables"].values())
                assert held + t["free"] == 14, f"tick {t['tick']}"
                assert sum(1 for c in t["calls"] if c.get("mixed")) <= 1
            assert got["replies"] == fx["replies"]
            assert not chat._mixed
    finally:
        chat.DEVICE, chat.MIXED_PREFILL_MIN_TOKENS, chat.MIXED_PREFILL_CHUNK = saved
        chat._mixed.clear()
        chat._kv_cache = None


def test_chunk_lengths_are_near_equal():
    import chat

    saved = chat.MIXED_PREFILL_CHUNK
    try:
        chat.MIXED_PREFILL_CHUNK = 512
        for n in (1, 511, 512, 513, 1000, 1025, 4096, 4097):
            parts, r = [], n
            while r:
                parts.append(chat._chunk_len(r))
                r -= parts[-1]
            assert sum(parts) == n and max(parts) <= 512
            assert len(parts) == -(-n // 512) and max(parts) - min(parts) <= 1
        chat.MIXED_PREFILL_CHUNK = None
        assert chat._chunk_len(5000) == 5000
    finally:
        chat.MIXED_PREFILL_CHUNK = saved


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
