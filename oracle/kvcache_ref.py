"""Restatement of the reference KVCache (kv_cache.py:8-121) on the CPU.

TEST INFRASTRUCTURE ONLY.  Same decisions as the reference: the pool is
[L, 2, num_blocks*block_size, Hkv, D] (kv_cache.py:20-22); the free list is a
Python list whose tail is popped (:64) and to whose tail freed/trimmed blocks
are appended (:49, :71); prepare() computes slot = table[p//bs]*bs + p%bs per
new token (:88-91) and a [B, S] gather index with tables padded by block 0
(:93-100); write() scatters with index_copy_ (:108-115); read() gathers a
dense copy (:117-121).
"""
from __future__ import annotations

import math

import torch

NUM_LAYERS, NUM_KV_HEADS, HEAD_DIM = 28, 2, 128


class RefKVCache:
    def __init__(self, num_blocks, block_size=16, dtype=torch.float32, num_layers=NUM_LAYERS,
                 with_pool=True, fp8=False):
        # fp8: every written k / v row goes through the FP8 pool's e4m3
        # round trip (oracle/fp8_ref.py) before it is stored -- the oracle of
        # the product's opt-in FP8 mode, which the reference does not have
        self.fp8 = fp8
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.buf = (torch.zeros(num_layers, 2, num_blocks * block_size, NUM_KV_HEADS, HEAD_DIM,
                                dtype=dtype) if with_pool else None)
        self.free_blocks = list(range(num_blocks))
        self.tables = {}
        self.lengths = {}
        self.next_seq = 0

    # kv_cache.py:31-53
    def free_block_count(self):
        return len(self.free_blocks)

    def blocks_needed(self, seq, total_len):
        held = len(self.tables[seq]) if seq is not None else 0
        return max(0, math.ceil(total_len / self.block_size) - held)

    def alloc(self):
        seq = self.next_seq
        self.next_seq += 1
        self.tables[seq] = []
        self.lengths[seq] = 0
        return seq

    def free(self, seq):
        self.free_blocks.extend(self.tables.pop(seq))
        del self.lengths[seq]

    def length(self, seq):
        return self.lengths[seq]

    # kv_cache.py:55-64
    def ensure_capacity(self, seq, total_len):
        need = self.blocks_needed(seq, total_len)
        if need > len(self.free_blocks):
            raise RuntimeError(f"KV cache exhausted: seq {seq} needs {need} more blocks, "
                               f"only {len(self.free_blocks)} free")
        for _ in range(need):
            self.tables[seq].append(self.free_blocks.pop())

    # kv_cache.py:66-72
    def trim(self, seq):
        keep = math.ceil(self.lengths[seq] / self.block_size)
        self.free_blocks.extend(self.tables[seq][keep:])
        del self.tables[seq][keep:]

    # kv_cache.py:74-101 (host lists instead of device tensors)
    def prepare(self, seqs, T):
        bs = self.block_size
        starts = [self.lengths[s] for s in seqs]
        for s, st in zip(seqs, starts):
            self.ensure_capacity(s, st + T)
        slot_mapping = []
        for s, st in zip(seqs, starts):
            tb = self.tables[s]
            slot_mapping += [tb[p // bs] * bs + p % bs for p in range(st, st + T)]
        # [B, S] gather index with tables padded by block 0, built with tensor
        # ops as the reference does (kv_cache.py:93-100)
        S = max(starts) + T
        nb = math.ceil(S / bs)
        tables = torch.tensor([(self.tables[s] + [0] * nb)[:nb] for s in seqs], dtype=torch.long)
        pos = torch.arange(S)
        gather = tables[:, pos // bs] * bs + pos % bs
        return starts, slot_mapping, gather

    def advance(self, seqs, T):
        for s in seqs:
            self.lengths[s] += T

    # kv_cache.py:108-115
    def write(self, layer, slot_mapping, k, v):
        B, H, T, D = k.shape
        idx = torch.as_tensor(slot_mapping, dtype=torch.long)
        if self.fp8:
            k, v = fp8_round_trip(k), fp8_round_trip(v)
        self.buf[layer, 0].index_copy_(0, idx, k.transpose(1, 2).reshape(B * T, H, D).to(self.buf.dtype))
        self.buf[layer, 1].index_copy_(0, idx, v.transpose(1, 2).reshape(B * T, H, D).to(self.buf.dtype))

    # kv_cache.py:117-121
    def read(self, layer, gather):
        idx = torch.as_tensor(gather, dtype=torch.long)
        return self.buf[layer, 0][idx].transpose(1, 2), self.buf[layer, 1][idx].transpose(1, 2)


def fp8_round_trip(x: torch.Tensor) -> torch.Tensor:
    """Rows of 128 (last dim) through the FP8 pool's quantisation: the fp32
    value e4m3 * scale each row reads back as."""
    import numpy as np

    from oracle import fp8_ref

    rows = x.detach().float().cpu().numpy().reshape(-1, x.shape[-1])
    b, scale = fp8_ref.quantize_rows(rows)
    back = fp8_ref.e4m3_decode(b) * scale[:, None]
    return torch.from_numpy(np.ascontiguousarray(back.reshape(x.shape))).to(x.device)
