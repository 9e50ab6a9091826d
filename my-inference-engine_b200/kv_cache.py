"""Paged KV cache with device-resident int32 block tables (drop-in for the
reference's kv_cache.py:8-121).

Host semantics are the reference's, decision for decision: a Python free list
popped from its tail (kv_cache.py:26, :64), blocks returned by `free`/`trim`
appended at the tail and therefore reused first (:47-50, :66-72), monotonic
sequence ids (:31-45), `RuntimeError("KV cache exhausted ...")` when the pool
runs dry (:58-61), lengths kept as plain ints so reading them never syncs.

What moves to the device:
  * `block_tables` -- int32 [max_seqs, table_pitch]; each live sequence owns a
    row.  New block ids are queued on the host and uploaded in one copy at the
    next `prepare`, so there is no per-token host loop and no [B, S] index
    tensor (the reference builds both every step, kv_cache.py:88-100).
  * `prepare(seqs, T)` uploads one int32 [3, B] array (table row, start,
    kv_len per batch row) and returns a `PagedStep` in the two positions the
    reference returns slot_mapping and gather_idx.
  * `write()` scatters through the table on the GPU; `read()` returns
    zero-copy `PagedKV` handles instead of a dense gathered copy;
    `append()` fuses RoPE on q and k with the write.

`buf` keeps the reference layout [NUM_LAYERS, 2, num_blocks*16, NUM_KV_HEADS,
HEAD_DIM] (kv_cache.py:20-22), so code that inspects it (bytes per token in
metrics/benchmark_concurrency.py:25-26) and the CPU oracle read it unchanged.
"""
from __future__ import annotations

import itertools
import math
from dataclasses import dataclass

import numpy as np
import torch

import pagedkv
from model import HEAD_DIM, NUM_KV_HEADS, NUM_LAYERS

BLOCK_SIZE = 16  # the kernels' block geometry (chat.py:22 uses 16 too)


@dataclass
class PagedStep:
    """Device description of one forward step over B rows (built by prepare)."""
    cache: "KVCache"
    T: int
    starts_host: list
    rows: torch.Tensor      # int32 [B] table row of each batch row
    starts: torch.Tensor    # int32 [B] length before this step
    kv_lens: torch.Tensor   # int32 [B] starts + T
    max_kv_len: int         # host-side max(kv_lens), sizes decode grids
    q_lens: torch.Tensor | None = None  # int32 [B] real tokens of right-padded rows

    @property
    def batch(self) -> int:
        return len(self.starts_host)


class PagedKV:
    """Zero-copy stand-in for one of the dense K/V tensors `read()` returned in
    the reference: a layer's K (which=0) or V (which=1) plane plus the step's
    block tables.  `shape` mirrors the dense [B, Hkv, S, D] it replaces."""

    def __init__(self, cache: "KVCache", layer_idx: int, which: int, step: PagedStep):
        self.cache, self.layer_idx, self.which, self.step = cache, layer_idx, which, step

    @property
    def plane(self) -> torch.Tensor:
        return self.cache.buf[self.layer_idx, self.which]

    @property
    def fp8(self) -> bool:
        return self.cache.fp8

    @property
    def shape(self) -> torch.Size:
        return torch.Size((self.step.batch, NUM_KV_HEADS, self.step.max_kv_len, HEAD_DIM))

    @property
    def dtype(self) -> torch.dtype:
        return torch.bfloat16  # what the attention sees (an FP8 pool reads back as bf16)

    @property
    def device(self) -> torch.device:
        return self.cache.device

    @property
    def is_cuda(self) -> bool:
        return self.cache.device.type == "cuda"

    def materialize(self) -> torch.Tensor:
        """Dense [B, Hkv, S, D] copy (test/debug only; the kernels never use it).
        Positions past a row's kv_len read block 0's slots, as the reference's
        padded gather does (kv_cache.py:95); an FP8 pool reads back as
        bf16(e4m3 * scale), zeros past kv_len."""
        c, st = self.cache, self.step
        S = st.max_kv_len
        if c.fp8:
            kd, vd = c.dequant_step(self.layer_idx, st, S)
            return (kd if self.which == 0 else vd).view(st.batch, -1, NUM_KV_HEADS, HEAD_DIM)[
                :, :S].transpose(1, 2)
        nb = math.ceil(S / c.block_size)
        tbl = c.block_tables[st.rows.long(), :nb].long()
        lens_blocks = (st.kv_lens.long() + c.block_size - 1) // c.block_size
        valid = torch.arange(nb, device=tbl.device)[None, :] < lens_blocks[:, None]
        tbl = torch.where(valid, tbl, torch.zeros_like(tbl))
        pos = torch.arange(S, device=tbl.device)
        idx = tbl[:, pos // c.block_size] * c.block_size + pos % c.block_size
        return self.plane[idx].transpose(1, 2)


class BlockTables:
    """Host half of the cache: free list, per-sequence block lists, lengths and
    table rows (no device memory; unit-testable on the CPU).  Every decision
    matches the reference KVCache (kv_cache.py:24-72)."""

    def __init__(self, num_blocks, block_size, max_seqs=None, max_blocks_per_seq=None):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self._free_blocks = list(range(num_blocks))
        self._block_tables = {}  # seq id -> list of block ids, in logical order
        self._lengths = {}  # seq id -> tokens written so far
        self._next_seq = 0
        self.max_seqs = int(max_seqs or min(num_blocks, 4096))
        self.table_pitch = int(max_blocks_per_seq or min(num_blocks, 8192))
        self._row_of = {}  # seq id -> table row
        self._free_rows = list(range(self.max_seqs - 1, -1, -1))
        self._pending = {}  # (row, col) -> block id not yet on the device (last write wins)

    def free_block_count(self):
        return len(self._free_blocks)

    def blocks_needed(self, seq, total_len):
        """Extra blocks `seq` (None for a brand-new sequence) needs to hold total_len tokens."""
        held = len(self._block_tables[seq]) if seq is not None else 0
        return max(0, math.ceil(total_len / self.block_size) - held)

    def alloc(self):
        """Start a new, empty sequence (and give it a device table row)."""
        if not self._free_rows:
            raise RuntimeError(f"KV cache exhausted: all {self.max_seqs} sequence rows in use")
        seq = self._next_seq
        self._next_seq += 1
        self._block_tables[seq] = []
        self._lengths[seq] = 0
        self._row_of[seq] = self._free_rows.pop()
        return seq

    def free(self, seq):
        """Return every block (and the table row) this sequence holds."""
        self._free_blocks.extend(self._block_tables.pop(seq))
        del self._lengths[seq]
        self._free_rows.append(self._row_of.pop(seq))

    def length(self, seq):
        return self._lengths[seq]

    def ensure_capacity(self, seq, total_len):
        """Grow seq's block table until it covers total_len tokens. Raises if the pool runs dry."""
        need = self.blocks_needed(seq, total_len)
        if need > len(self._free_blocks):
            raise RuntimeError(
                f"KV cache exhausted: seq {seq} needs {need} more blocks, only {len(self._free_blocks)} free"
            )
        table = self._block_tables[seq]
        if len(table) + need > self.table_pitch:
            raise RuntimeError(
                f"KV cache exhausted: seq {seq} would hold {len(table) + need} blocks, "
                f"the device table holds {self.table_pitch} per sequence")
        if need == 0:
            return
        row = self._row_of[seq]
        # the blocks `need` pops from the tail of the free list would return,
        # in pop order, taken as one slice
        blks = self._free_blocks[-need:][::-1]
        del self._free_blocks[-need:]
        col0 = len(table)
        self._pending.update(zip(zip(itertools.repeat(row, need), range(col0, col0 + need)), blks))
        table.extend(blks)

    def trim(self, seq):
        """Give back any blocks past the one holding seq's last written token."""
        table = self._block_tables[seq]
        keep = math.ceil(self._lengths[seq] / self.block_size)
        self._free_blocks.extend(table[keep:])
        del table[keep:]

    def advance(self, seqs, T):
        """Record that every seq in `seqs` now holds T more tokens (after all layers wrote)."""
        for s in seqs:
            self._lengths[s] += T

    def table_row(self, seq):
        return self._row_of[seq]

    def host_table(self, seq):
        return list(self._block_tables[seq])

    def take_pending(self):
        """(row, col, block) entries queued since the last call."""
        pend = [(r, c, b) for (r, c), b in self._pending.items()]
        self._pending = {}
        return pend

    def take_pending_flat(self):
        """The queued entries as one int64 numpy array [2, n]: flat table
        index (row * table_pitch + col) and block id, in queue order (one
        entry per cell, the last write).  None when nothing is queued."""
        pend, self._pending = self._pending, {}
        n = len(pend)
        if not n:
            return None
        rc = np.fromiter(itertools.chain.from_iterable(pend.keys()), dtype=np.int64, count=2 * n)
        out = np.empty((2, n), dtype=np.int64)
        np.multiply(rc[0::2], self.table_pitch, out=out[0])
        out[0] += rc[1::2]
        out[1] = np.fromiter(pend.values(), dtype=np.int64, count=n)
        return out

    def step_rows(self, seqs, T):
        """Host part of prepare(): reserve blocks, return (starts, rows)."""
        starts = [self._lengths[s] for s in seqs]
        bs, tables = self.block_size, self._block_tables
        for s, start in zip(seqs, starts):
            if start + T > len(tables[s]) * bs:  # otherwise ensure_capacity adds nothing
                self.ensure_capacity(s, start + T)
        return starts, [self._row_of[s] for s in seqs]


class _PinnedUpload:
    """One persistent pinned staging buffer for small host-to-device uploads
    (block-table deltas, per-step row vectors): no pinned allocation per
    step.  A CUDA event recorded after each copy guards the buffer, so the
    host never refills it while the previous copy is still queued (the host
    can run ahead of the stream when no sync separates two steps)."""

    def __init__(self, dtype):
        self.dtype = dtype
        self.buf = None
        self.done = None

    def send(self, flat: np.ndarray, device) -> torch.Tensor:
        n = flat.shape[0]
        if self.done is not None:
            self.done.synchronize()  # usually long complete: returns at once
        if self.buf is None or self.buf.numel() < n:
            cap = max(n, 2 * (self.buf.numel() if self.buf is not None else 0), 1024)
            self.buf = torch.empty(cap, dtype=self.dtype, pin_memory=True)
        self.buf.numpy()[:n] = flat
        out = self.buf[:n].to(device, non_blocking=True)
        if self.done is None:
            self.done = torch.cuda.Event()
        self.done.record()
        return out


class KVCache(BlockTables):
    """Paged KV cache shared by every concurrently active sequence.

    Same constructor and methods as the reference (kv_cache.py:19-121), plus
    two optional sizing knobs for the device tables:
      max_seqs            table rows, i.e. sequences alive at once
      max_blocks_per_seq  table pitch, i.e. longest sequence in blocks
    """

    def __init__(self, num_blocks, block_size, device, dtype, max_seqs=None,
                 max_blocks_per_seq=None, num_layers=NUM_LAYERS, kv_format="bf16"):
        device = torch.device(device)
        assert device.type == "cuda", "KVCache needs a CUDA device (no CPU fallback)"
        assert block_size == BLOCK_SIZE, f"block_size must be {BLOCK_SIZE}"
        assert dtype == torch.bfloat16, "the paged kernels store bf16 K/V"
        assert kv_format in ("bf16", "fp8_e4m3"), "kv_format is 'bf16' or 'fp8_e4m3'"
        super().__init__(num_blocks, block_size, max_seqs, max_blocks_per_seq)
        # num_layers < 28 only for single-layer attention workloads (kernel
        # tests and benchmarks); the model needs the full pool
        self.kv_format = kv_format
        if kv_format == "fp8_e4m3":
            # opt-in FP8 pool: [layer][block][kv head][chunk] bytes, half the
            # bytes per token (layout in include/pagedkv.h); no bf16 planes
            self.buf = None
            self.pool8 = torch.zeros(num_layers, num_blocks, NUM_KV_HEADS,
                                     pagedkv.fp8_block_bytes(), device=device, dtype=torch.uint8)
        else:
            self.pool8 = None
            self.buf = torch.zeros(num_layers, 2, num_blocks * block_size, NUM_KV_HEADS,
                                   HEAD_DIM, device=device, dtype=dtype)
        self.device = device
        self.block_tables = torch.zeros(self.max_seqs, self.table_pitch, dtype=torch.int32,
                                        device=device)
        self.err_flag = torch.zeros(1, dtype=torch.int32, device=device)
        self._tables_up = _PinnedUpload(torch.int64)  # (flat index, block id) pairs
        self._step_up = _PinnedUpload(torch.int32)  # (row, start, kv_len) per batch row

    # ---- device side ----
    def flush_tables(self):
        """Upload queued (row, col, block) entries in one copy + one scatter."""
        host = self.take_pending_flat()
        if host is None:
            return
        n = host.shape[1]
        d = self._tables_up.send(host.reshape(-1), self.device).view(2, n)
        self.block_tables.view(-1).index_copy_(0, d[0], d[1].to(torch.int32))

    def prepare(self, seqs, T):
        """Set up one forward step that appends T tokens to every seq in `seqs`.

        Returns (starts, step, step): each row's length before this step as
        plain ints (as the reference), and a PagedStep where the reference
        returned slot_mapping and gather_idx (kv_cache.py:74-101).
        """
        starts, rows = self.step_rows(seqs, T)
        self.flush_tables()
        B = len(seqs)
        host = np.empty((3, B), dtype=np.int32)
        host[0] = rows
        host[1] = starts
        np.add(host[1], T, out=host[2])
        dev = self._step_up.send(host.reshape(-1), self.device).view(3, B)
        step = PagedStep(self, T, starts, dev[0], dev[1], dev[2], max(starts) + T)
        return starts, step, step

    @property
    def fp8(self) -> bool:
        return self.pool8 is not None

    def write(self, layer_idx, slot_mapping, k, v):
        """Scatter this step's new k/v for one layer into their physical slots
        (reference kv_cache.py:108-115).  k, v: [B, NUM_KV_HEADS, T, HEAD_DIM];
        slot_mapping is the PagedStep from prepare().  FP8 mode quantises them."""
        step = slot_mapping
        if self.fp8:
            pagedkv.append_rope_fp8(None, k, v, None, None, None, self.pool8[layer_idx],
                                    self.block_tables, step.rows, step.starts, self.err_flag,
                                    step.q_lens)
            return
        pagedkv.append_rope(None, k, v, None, None, None, self.buf[layer_idx, 0],
                            self.buf[layer_idx, 1], self.block_tables, step.rows, step.starts,
                            self.err_flag, step.q_lens)

    def append(self, layer_idx, step, q, k, v, rope_cos, rope_sin, q_out):
        """Fused apply_rope(q, k) + write (model.py:92-96): roped q goes to
        q_out, roped k and v into the pool.  rope_cos/sin: bf16 [positions, 128]."""
        if self.fp8:
            pagedkv.append_rope_fp8(q, k, v, rope_cos, rope_sin, q_out, self.pool8[layer_idx],
                                    self.block_tables, step.rows, step.starts, self.err_flag,
                                    step.q_lens)
            return
        pagedkv.append_rope(q, k, v, rope_cos, rope_sin, q_out, self.buf[layer_idx, 0],
                            self.buf[layer_idx, 1], self.block_tables, step.rows, step.starts,
                            self.err_flag, step.q_lens)

    def dequant_step(self, layer_idx, step, S):
        """FP8 mode: the step's rows (positions < kv_len) as bf16 K and V
        planes in the bf16 pool layout, [B * S16, NUM_KV_HEADS, HEAD_DIM] each
        with S16 = S rounded up to 16: row b's position p at plane slot
        b * S16 + p, i.e. row b owns blocks b * S16 / 16 ... (see
        identity_tables).  Positions past kv_len are zero."""
        B = step.batch
        S16 = -(-max(S, 1) // BLOCK_SIZE) * BLOCK_SIZE
        kd = torch.zeros(B * S16, NUM_KV_HEADS, HEAD_DIM, device=self.device, dtype=torch.bfloat16)
        vd = torch.zeros_like(kd)
        # [B, Hkv, S16, D] views of the [B*S16, Hkv, D] planes
        k4 = kd.view(B, S16, NUM_KV_HEADS, HEAD_DIM).transpose(1, 2)
        v4 = vd.view(B, S16, NUM_KV_HEADS, HEAD_DIM).transpose(1, 2)
        pagedkv.fp8_dequant(self.pool8[layer_idx], self.block_tables, step.rows, step.kv_lens,
                            S16, k4, v4, self.err_flag)
        return kd, vd

    @staticmethod
    def identity_tables(B, S16, device):
        """Block tables of dequant_step's planes: row b -> blocks b*n .. b*n+n-1."""
        n = S16 // BLOCK_SIZE
        return torch.arange(B * n, device=device, dtype=torch.int32).view(B, n)

    def read(self, layer_idx, gather_idx):
        """This layer's K and V as zero-copy PagedKV handles (the reference
        returned dense gathered copies, kv_cache.py:117-121)."""
        step = gather_idx
        return PagedKV(self, layer_idx, 0, step), PagedKV(self, layer_idx, 1, step)

    def check_errors(self):
        """Read (and clear) the device error flag; raises RuntimeError if a kernel
        met an out-of-range block id or position.  Synchronises."""
        v = int(self.err_flag.item())
        if v:
            self.err_flag.zero_()
            raise RuntimeError(f"paged KV kernel reported device error bits {v:#x}")
