"""Deterministic driver for a chat.py-style scheduler (test infrastructure only).

Runs the body of the reference worker loop (chat.py:232-254) on the calling
thread against a scheduler module -- the reference's chat.py or the product's
-- with a fake tokenizer and a fake model, and records what the scheduler
decided at every tick: which messages were admitted, rejected or deferred,
the active / resident (LRU) lists, every model call (rows, T, input ids), the
free-block count and every live block table.  The fake model does only the
host half of a forward pass (reserve blocks, advance lengths, like
KVCache.prepare + advance) and returns one-hot logits, so sampling is
deterministic.
"""
from __future__ import annotations

import queue

import torch

VOCAB = 64
EOS = 7


class FakeTokenizer:
    encoder = {"<|endoftext|>": EOS}

    def encode(self, text):
        return [10 + (ord(c) * 31 + i * 7) % 50 for i, c in enumerate(text)]

    def decode(self, ids):
        return "a" * len(ids)


class FakeModel:
    """Host half of a forward: reserve + advance; one-hot logits (never EOS
    for the first tokens of a reply, EOS sometimes later)."""

    def __init__(self, log):
        self.log = log

    def __call__(self, input_ids, cache, seqs):
        B, T = input_ids.shape
        self.log.append({"seqs": list(seqs), "T": T, "ids": input_ids.cpu().tolist()})
        for s in seqs:
            cache.ensure_capacity(s, cache.length(s) + T)
        cache.advance(seqs, T)
        return self._logits(cache, seqs)[:, None]

    def forward_mixed(self, prefill_ids, prefill_seq, decode_ids, decode_seqs, cache):
        """The product's optional mixed step: a prompt and decode rows in one
        call; logits [1 + B, vocab] (the prompt's last token first)."""
        T = prefill_ids.shape[1]
        self.log.append({"mixed": True, "prefill_seq": prefill_seq, "T": T,
                         "ids": prefill_ids.cpu().tolist(), "seqs": list(decode_seqs),
                         "decode_ids": decode_ids.cpu().tolist()})
        cache.ensure_capacity(prefill_seq, cache.length(prefill_seq) + T)
        for s in decode_seqs:
            cache.ensure_capacity(s, cache.length(s) + 1)
        cache.advance([prefill_seq], T)
        cache.advance(decode_seqs, 1)
        return self._logits(cache, [prefill_seq] + list(decode_seqs))

    @staticmethod
    def _logits(cache, seqs):
        """One-hot [len(seqs), VOCAB]: the next token is a function of the
        sequence id and its length only."""
        logits = torch.full((len(seqs), VOCAB), -1e9)
        for b, s in enumerate(seqs):
            n = cache.length(s)
            tok = 10 + (s * 13 + n * 5) % 50
            if n % 23 == 0:
                tok = EOS
            logits[b, tok] = 0.0
        return logits


# (tick, chat index, message text) submissions and (tick, chat index) releases
SUBMIT = [
    (0, 0, "hello there, how are you"),
    (0, 1, "tell me a story about a cat and a dog"),
    (0, 2, "x" * 70),
    (2, 3, "short"),
    (4, 4, "this message is long enough to need several blocks" * 2),
    (12, 0, "and a follow up question"),
    (14, 5, "y" * 120),
    (20, 1, "second turn for chat one"),
    (26, 2, "second turn for chat two"),
    (30, 6, "z" * 400),  # can never fit: rejected
    (31, 3, "again"),
]
RELEASE = [(18, 4), (40, 5)]


def run_trace(chat_mod, install_cache, num_blocks=14, max_reply=12, ticks=90):
    """Drive `chat_mod` for `ticks` worker ticks; returns the recorded trace."""
    calls = []
    model = FakeModel(calls)
    chat_mod._job_queue = queue.Queue()  # a private queue: no worker thread can take jobs
    chat_mod.active.clear()
    chat_mod._deferred.clear()
    cache = install_cache(num_blocks)
    chat_mod._resident.clear()
    chat_mod.MAX_REPLY_TOKENS = max_reply
    chat_mod.STOP_SEQUENCES = ["\nUser:", "\nUser"]
    tok = FakeTokenizer()
    chats = [chat_mod.Chat(tok) for _ in range(7)]
    outs = {}
    trace = []
    released = set()
    for tick in range(ticks):
        for t, ci, text in SUBMIT:
            if t == tick:
                chats[ci].pending.append(text)
                q = queue.Queue()
                outs.setdefault(ci, []).append(q)
                chat_mod._job_queue.put(chat_mod._Job(chats[ci], model, text, q))
        for t, ci in RELEASE:
            # release only idle chats (a reply in flight would lose its blocks,
            # which the reference does not guard against); else retry next tick
            if t <= tick and ci not in released and chats[ci].in_progress is None \
                    and not chats[ci].pending:
                chats[ci].release()
                released.add(ci)
        n_calls = len(calls)
        # chat.py:_worker loop body, without blocking or sleeping
        for job in list(chat_mod._deferred):
            if chat_mod._make_room(job):
                chat_mod._deferred.remove(job)
                chat_mod._admit(job)
        if not chat_mod.active and not chat_mod._deferred:
            if not chat_mod._job_queue.empty():
                chat_mod._try_admit_or_defer(chat_mod._job_queue.get())
        elif not chat_mod.active and chat_mod._deferred:
            pass
        elif not chat_mod._job_queue.empty():
            chat_mod._try_admit_or_defer(chat_mod._job_queue.get())
        chat_mod._process(chat_mod.active)
        idx = {id(c): i for i, c in enumerate(chats)}
        trace.append({
            "tick": tick,
            "calls": calls[n_calls:],
            "active": [idx[id(j.chat)] for j in chat_mod.active],
            "deferred": [idx[id(j.chat)] for j in chat_mod._deferred],
            "resident": [idx[id(c)] for c in chat_mod._resident],
            "seqs": [c.seq for c in chats],
            "free": cache.free_block_count(),
            "tables": {str(c.seq): list(cache._block_tables[c.seq]) for c in chats
                       if c.seq is not None},
            "ids": [list(c.ids) for c in chats],
        })
    replies = {ci: [_drain(q) for q in qs] for ci, qs in outs.items()}
    return {"trace": trace, "replies": {str(k): v for k, v in replies.items()}}


def _drain(q):
    out = []
    while not q.empty():
        out.append(q.get())
    return out
