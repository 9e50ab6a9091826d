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
