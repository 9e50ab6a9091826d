"""Continuous-batching scheduler on the device-table KV cache (drop-in for the
reference's chat.py:1-377).

Every scheduling decision is the reference's, in the same order and with the
same module-level names (the reference's benchmark monkey-patches `_admit`,
`_finish`, `STOP_SEQUENCES`, `MAX_REPLY_TOKENS` on this module):
  * a message reserves history + prompt + MAX_REPLY_TOKENS + trailing "\\n"
    blocks up front (chat.py:117-125) and is rejected if that can never fit
    (chat.py:214-229);
  * idle chats are evicted least-recently-used first under `_cache_lock`
    until the new message fits, else it is deferred (chat.py:128-146);
  * at most one prefill per worker tick (chat.py:232-254), then one batched
    decode step for every active job with a single device sync for sampling
    (chat.py:257-308, :103-107);
  * `_finish` trims unused reserved blocks (chat.py:194-211); `Chat.release`
    frees a chat's blocks from a request thread (chat.py:325-330).
What changes is underneath: the cache's block tables live on the device, the
decode step can replay a captured CUDA graph (model.DecodeGraphs), sampling
is one device kernel (pagedkv.sample: the same softmax(logits / T)
distribution, drawn by Gumbel-max), a prompt's first token is read back only
when the decode tick reaches its job (so the host work for the jobs ahead of
it overlaps the prefill), and nothing is allocated or started at import --
`KV_CACHE` is created on first use and the worker thread on the first
message (`init()` sets both up explicitly).

Not provided, being outside the attention path: weight loading from a
checkpoint directory and the single-sequence `generate` loop of the
reference (chat.py:39-46, :72-88).  A caller builds the model itself
(model.Qwen2ForCausalLM + load_state_dict) and drives chats through `Chat`.

One opt-in departure (off by default, so the decisions above stay the
reference's): with MIXED_PREFILL_MIN_TOKENS set, a tick that admits a prompt
of at least that many tokens while other jobs are decoding runs the prompt
and their decode rows as ONE forward (model.forward_mixed: one pass over the
weights, one sampling sync).  The admitted job then takes its first decode
step in the next tick instead of this one; every other decision (admission,
eviction, deferral, trimming, FIFO order) is unchanged.  With
MIXED_PREFILL_CHUNK also set, such a prompt longer than the chunk runs as
ceil(len / chunk) near-equal chunks on consecutive ticks, each sharing that
tick's decode forward (chunked prefill: every chunk attends to the ones
before it through the cache); the job joins the decode batch after its
last chunk, whose last-token logits give its first token.
"""
from __future__ import annotations

import array
import queue
import sys
import threading
import time

import torch
import torch.nn.functional as F

import pagedkv
from kv_cache import KVCache

MAX_REPLY_TOKENS = 512  # safety net against a reply that never hits EOS
TEMPERATURE = 1

BLOCK_SIZE = 16
KV_CACHE_TOKENS = 8 * 2048  # the reference's 448 MB budget (1024 blocks)
MAX_SEQ_LEN = 2048

# opt-in mixed prefill + decode ticks (see the module docstring); None = off
MIXED_PREFILL_MIN_TOKENS = None
# with mixed ticks on: a mixed prompt longer than this many tokens is split
# into near-equal chunks, one per tick (chunked prefill); None = whole prompt
MIXED_PREFILL_CHUNK = None

DEVICE = torch.device("cuda")
DTYPE = torch.bfloat16

_kv_cache = None


def _kv():
    global _kv_cache
    if _kv_cache is None:
        _kv_cache = KVCache(KV_CACHE_TOKENS // BLOCK_SIZE, BLOCK_SIZE, DEVICE, dtype=DTYPE)
    return _kv_cache


def __getattr__(name):  # module attribute KV_CACHE, created on first access
    if name == "KV_CACHE":
        return _kv()
    raise AttributeError(name)


def init(kv_cache=None, start_worker=True):
    """Install a cache (default: the reference's 1024-block budget) and start
    the worker thread now instead of on the first message.  Installing a new
    cache forgets every resident chat's sequence (its K/V lived in the old
    pool; its next message prefills the whole history again) and is refused
    while a message is in flight."""
    global _kv_cache
    if kv_cache is not None and kv_cache is not _kv_cache:
        if active or _deferred or _mixed:
            raise RuntimeError("cannot replace the KV cache while messages are in flight")
        for c in _resident:
            c.seq = None
        _resident.clear()
        _kv_cache = kv_cache
    _kv()
    if start_worker:
        _ensure_worker()
    return _kv_cache


STOP_SEQUENCES = ["\nUser:", "\nUser"]


def _hold_back(text, patterns):
    """Split a reply's undelivered text for streaming: returns (ready, held,
    stopped).  If any stop pattern occurs, everything before its earliest
    occurrence is ready and the reply stops.  Otherwise the longest tail of
    `text` that is a proper prefix of some pattern (it may still grow into a
    stop) is held back and the rest is ready.  Same pieces as the reference's
    streaming (chat.py:51-69, :281-294)."""
    hits = [i for i in (text.find(p) for p in patterns if p) if i >= 0]
    if hits:
        return text[:min(hits)], "", True
    longest = max((len(p) for p in patterns), default=1) - 1
    for k in range(min(longest, len(text)), 0, -1):
        tail = text[len(text) - k:]
        if any(len(p) > k and p.startswith(tail) for p in patterns):
            return text[:len(text) - k], tail, False
    return text, "", False


class _Job:
    def __init__(self, chat, model, text, out_queue):
        self.chat = chat
        self.model = model
        self.text = text
        self.out_queue = out_queue
        self.buffer = ""
        self.steps = 0
        self.next_token = None
        self.new_ids = chat.tokenizer.encode(f"User: {text}\nAssistant:")


def _sample_async(logits):
    """Enqueue sampling of one token id per row of [B, vocab] logits from
    softmax(logits / TEMPERATURE); the ids stay on the logits' device.

    CUDA logits: one pkv_sample kernel (Gumbel-max over the logits, keyed
    from torch's default generator) instead of the float copy, softmax and
    torch.multinomial of the reference (chat.py:103-107), whose argument
    checks also cost ~0.5 ms of host time per call.  Host logits only come
    from a stand-in model (the scheduler's CPU tests) and take the
    reference's own three ops."""
    if logits.is_cuda:
        return pagedkv.sample(logits, TEMPERATURE)
    x = logits.float()
    if TEMPERATURE != 1:  # x / 1 is x: skip the extra pass over [B, vocab]
        x = x / TEMPERATURE
    probs = F.softmax(x, dim=-1)
    return torch.multinomial(probs, num_samples=1).squeeze(1)


def _read_ids(ids):
    """Sampled ids as Python ints (one device sync); a row the kernel could
    not sample (no finite logit) raises as torch.multinomial does."""
    out = ids.tolist()
    if out and min(out) < 0:
        raise RuntimeError("probability tensor contains either `inf`, `nan` or element < 0")
    return out


def _sample(logits):
    """One token id per row of [B, vocab] logits, one device sync for the batch."""
    return _read_ids(_sample_async(logits))


class _PendingToken:
    """A prompt's first sampled token, not yet read back: `_prefill` enqueues
    the sampling and `_process` reads the id when it reaches the job, which
    is last in FIFO order, so the host work for the jobs ahead of it runs
    while the prefill is still on the GPU.  Same ids, same order of sampling
    draws and of every scheduling decision as reading it at once."""

    __slots__ = ("ids",)

    def __init__(self, ids):
        self.ids = ids

    def get(self):
        return _read_ids(self.ids)[0]


_job_queue = queue.Queue()
active = []
_deferred = []
_resident = []
_cache_lock = threading.Lock()
_worker_thread = None
_worker_lock = threading.Lock()
_mixed = []  # at most one (job, prompt ids) whose prefill joins this tick's decode step


def _reserve_len(job):
    trailing = len(job.chat.tokenizer.encode("\n"))
    return len(job.chat.ids) + len(job.new_ids) + MAX_REPLY_TOKENS + trailing


def _blocks_needed(job):
    return _kv().blocks_needed(job.chat.seq, _reserve_len(job))


def _evict(chat):
    _kv().free(chat.seq)
    chat.seq = None
    _resident.remove(chat)


def _make_room(job):
    busy = {j.chat for j in active} | {j.chat for j, _ in _mixed} | {job.chat}
    with _cache_lock:
        while _blocks_needed(job) > _kv().free_block_count():
            idle = [c for c in _resident if c not in busy]
            if not idle:
                return False
            _evict(idle[0])
    return True


def _touch(chat):
    with _cache_lock:
        if chat in _resident:
            _resident.remove(chat)
        _resident.append(chat)


def _admit(job):
    """Prefill one job (chat.py:157-185)."""
    chat, model, text = job.chat, job.model, job.text
    cache = _kv()
    reserve_len = _reserve_len(job)
    chat.pending.remove(text)
    chat.messages.append(("user", text))
    chat.ids.extend(job.new_ids)
    chat.listeners = [job.out_queue]
    chat.in_progress = ""
    if chat.seq is None:
        chat.seq = cache.alloc()
    prefill_ids = chat.ids[cache.length(chat.seq):]
    cache.ensure_capacity(chat.seq, reserve_len)
    _touch(chat)
    if (MIXED_PREFILL_MIN_TOKENS is not None and active and not _mixed
            and len(prefill_ids) >= MIXED_PREFILL_MIN_TOKENS and hasattr(model, "forward_mixed")):
        _mixed.append((job, prefill_ids))  # runs inside this tick's decode step
        return
    _prefill(job, prefill_ids)


def _host_ids(ids):
    """[1, T] int32 host tensor over a token-id list: one C-level copy
    (array) instead of torch's per-element list conversion, ~8x faster for a
    2k-token prompt.  The model moves it to the device (or copies it into a
    captured graph's pinned input) itself."""
    return torch.frombuffer(array.array("i", ids), dtype=torch.int32).view(1, -1)


def _prefill(job, prefill_ids):
    input_ids = _host_ids(prefill_ids)
    with torch.no_grad():
        logits = job.model(input_ids, _kv(), [job.chat.seq])
    job.next_token = _PendingToken(_sample_async(logits[:, -1]))
    active.append(job)


def _emit(job, piece):
    job.chat.in_progress += piece
    for q in job.chat.listeners:
        q.put(piece)


def _finish(job):
    chat = job.chat
    chat.ids.extend(chat.tokenizer.encode("\n"))
    with _cache_lock:
        _kv().trim(chat.seq)
    _touch(chat)
    chat.messages.append(("assistant", chat.in_progress))
    chat.in_progress = None
    for q in chat.listeners:
        q.put(None)
    chat.listeners = []
    active.remove(job)


def _reject(job, reason):
    job.chat.pending.remove(job.text)
    job.out_queue.put(f"[error: {reason}]")
    job.out_queue.put(None)


def _try_admit_or_defer(job):
    cache = _kv()
    if cache.blocks_needed(None, _reserve_len(job)) > cache.num_blocks:
        _reject(job, "conversation is too long for the KV cache")
    elif _make_room(job):
        _admit(job)
    else:
        _deferred.append(job)


def _tick(block=True):
    """One pass of the worker loop (chat.py:232-254).  Returns False when there
    was nothing to do and `block` is False."""
    for job in list(_deferred):
        if _make_room(job):
            _deferred.remove(job)
            _admit(job)
    if not active and not _deferred:
        if not block and _job_queue.empty():
            return False
        _try_admit_or_defer(_job_queue.get())
    elif not active and _deferred:
        time.sleep(0.05)
    elif not _job_queue.empty():
        _try_admit_or_defer(_job_queue.get())
    _process(active)
    return True


def _worker():
    while True:
        _tick(block=True)


def run_until_idle():
    """Drive the worker loop on the calling thread until every queued,
    deferred and active job is done (deterministic, for benchmarks/tests)."""
    while _tick(block=False) or active or _deferred:
        pass


def _ensure_worker():
    global _worker_thread
    with _worker_lock:
        if _worker_thread is None:
            _worker_thread = threading.Thread(target=_worker, daemon=True)
            _worker_thread.start()


def _chunk_len(n):
    """Tokens of an n-token mixed prompt remainder to run this tick: all of
    it, or with MIXED_PREFILL_CHUNK = c the first of ceil(n / c) near-equal
    chunks (no short tail chunk)."""
    c = MIXED_PREFILL_CHUNK
    if not c or n <= c:
        return n
    return -(-n // -(-n // c))


def _process(active):
    """One decode step for every job currently active, in FIFO order."""
    continuing = []
    for job in list(active):
        chat = job.chat
        token_id = job.next_token
        if type(token_id) is _PendingToken:
            token_id = job.next_token = token_id.get()
        chat.ids.append(token_id)

        if token_id == chat.eos_id:
            _finish(job)
            continue

        ready, job.buffer, stopped = _hold_back(job.buffer + chat.tokenizer.decode([token_id]),
                                                STOP_SEQUENCES)
        if ready:
            _emit(job, ready)
        if stopped:
            _finish(job)
            continue

        job.steps += 1
        if job.steps >= MAX_REPLY_TOKENS:
            if job.buffer:
                _emit(job, job.buffer)
            _finish(job)
            continue

        continuing.append(job)

    mixed = _mixed.pop() if _mixed else None
    if mixed is not None and not continuing:  # nothing left to share the forward with
        _prefill(*mixed)
        return
    if not continuing:
        return

    model = continuing[0].model
    seqs = [job.chat.seq for job in continuing]
    if mixed is not None:
        new_job, prefill_ids = mixed
        chunk = _chunk_len(len(prefill_ids))
        # host tensors: a mixed-step graph copies them with its other inputs
        with torch.no_grad():
            logits = model.forward_mixed(
                _host_ids(prefill_ids[:chunk]), new_job.chat.seq,
                torch.tensor([job.next_token for job in continuing]).view(-1, 1), seqs, _kv())
        tokens = _sample(logits)
        for job, token_id in zip(continuing, tokens[1:]):
            job.next_token = token_id
        if chunk < len(prefill_ids):  # more of the prompt next tick
            _mixed.append((new_job, prefill_ids[chunk:]))
            return
        new_job.next_token = tokens[0]
        active.append(new_job)
        return

    # host tensor: the decode graph copies ids with the step's other inputs
    input_ids = torch.tensor([job.next_token for job in continuing]).view(-1, 1)
    if not getattr(model, "_graphs", None):
        input_ids = input_ids.to(DEVICE)
    with torch.no_grad():
        logits = model(input_ids, _kv(), seqs)

    for job, token_id in zip(continuing, _sample(logits[:, -1])):
        job.next_token = token_id


class Chat:
    """One conversation: its token ids, its sequence in the shared cache (None
    while evicted) and its messages.  Same attributes and methods as the
    reference's Chat (chat.py:314-377), which the scheduler and the
    reference's benchmark use."""

    def __init__(self, tokenizer):
        self.tokenizer = tokenizer
        self.ids = []          # every token of the conversation so far
        self.seq = None        # KV-cache sequence id, None when not resident
        self.messages = []     # finished (role, text) pairs
        self.pending = []      # submitted user texts not yet admitted
        self.in_progress = None  # the reply being streamed, if any
        self.listeners = []    # queues receiving the streamed reply pieces
        self.eos_id = tokenizer.encoder["<|endoftext|>"]

    def release(self):
        """Give this chat's blocks back to the pool (a later message prefills
        the whole history again)."""
        with _cache_lock:
            if self.seq is None:
                return
            _evict(self)

    def submit(self, model, text):
        """Queue a message without starting the worker thread; returns the
        queue its reply pieces (then None) arrive on."""
        self.pending.append(text)
        out_queue = queue.Queue()
        _job_queue.put(_Job(self, model, text, out_queue))
        return out_queue

    def send_stream(self, model, text):
        """Yield the reply's pieces as the worker produces them."""
        pieces = self.submit(model, text)
        _ensure_worker()
        for piece in iter(pieces.get, None):
            yield piece

    def all_messages(self):
        """Finished messages, then the reply in progress, then queued texts."""
        live = [] if self.in_progress is None else [("assistant", self.in_progress)]
        return [*self.messages, *live, *[("user", t) for t in self.pending]]

    def watch(self):
        """(text so far, queue of further pieces) of the reply in progress,
        or (None, None) when none is."""
        if self.in_progress is None:
            return None, None
        listener = queue.Queue()
        self.listeners.append(listener)
        return self.in_progress, listener

    def send(self, model, text):
        """Blocking helper: stream the reply to stdout, return its text."""
        for piece in self.send_stream(model, text):
            sys.stdout.write(piece)
            sys.stdout.flush()
        sys.stdout.write("\n")
        return self.messages[-1][1]

    def transcript(self):
        """The whole conversation decoded from its token ids."""
        return self.tokenizer.decode(self.ids)
