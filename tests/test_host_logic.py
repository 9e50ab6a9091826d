"""Host half of the product KVCache (BlockTables) makes the reference's
decisions: replayed against the reference's recorded op script it yields the
same free list, block tables, lengths, slots and errors, and it queues exactly
the device-table entries the kernels will need."""
import json
import math
import random

import pytest

from kv_cache import BlockTables


def _slots(bt, seqs, starts, T):
    out = []
    for s, st in zip(seqs, starts):
        tb = bt.host_table(s)
        out += [tb[p // 16] * 16 + p % 16 for p in range(st, st + T)]
    return out


def test_block_tables_replay_reference_script(golden):
    fx = json.loads((golden / "kvcache_ops.json").read_text())
    bt = BlockTables(fx["num_blocks"], fx["block_size"])
    bt._free_blocks = list(fx["initial_perm"])
    device_table = {}  # row -> {col: block} as the GPU would hold it
    for op, st in zip(fx["script"], fx["states"]):
        err = extra = None
        try:
            if op[0] == "alloc":
                extra = bt.alloc()
            elif op[0] == "prepare_advance":
                starts, rows = bt.step_rows(op[1], op[2])
                extra = {"starts": starts, "slot_mapping": _slots(bt, op[1], starts, op[2])}
                bt.advance(op[1], op[2])
            elif op[0] == "ensure_capacity":
                bt.ensure_capacity(op[1], op[2])
            elif op[0] == "trim":
                bt.trim(op[1])
            elif op[0] == "free":
                bt.free(op[1])
        except RuntimeError as e:
            err = str(e)
        for r, c, b in bt.take_pending():
            device_table.setdefault(r, {})[c] = b
        if err is not None:
            assert st["extra"] == {"error": err}
        elif op[0] == "alloc":
            assert st["extra"] == extra
        elif op[0] == "prepare_advance":
            assert st["extra"]["starts"] == extra["starts"]
            assert st["extra"]["slot_mapping"] == extra["slot_mapping"]
        assert st["free"] == bt._free_blocks
        assert st["tables"] == {str(k): v for k, v in bt._block_tables.items()}
        assert st["lengths"] == {str(k): v for k, v in bt._lengths.items()}
        # the device copy of every live row covers its host table
        for s, tb in bt._block_tables.items():
            row = bt.table_row(s)
            assert [device_table.get(row, {}).get(i) for i in range(len(tb))] == tb


def test_pending_updates_last_write_wins():
    bt = BlockTables(8, 16, max_seqs=2)
    a = bt.alloc()
    bt.ensure_capacity(a, 40)  # 3 blocks
    bt.free(a)
    b = bt.alloc()  # reuses a's row before any flush
    bt.ensure_capacity(b, 20)
    pend = bt.take_pending()
    cells = {}
    for r, c, blk in pend:
        assert (r, c) not in cells, "duplicate (row, col) would race in index_copy_"
        cells[(r, c)] = blk
    row = bt.table_row(b)
    assert [cells[(row, i)] for i in range(2)] == bt.host_table(b)


def test_exhaustion_errors_match_reference_wording():
    bt = BlockTables(4, 16, max_seqs=2, max_blocks_per_seq=3)
    s = bt.alloc()
    with pytest.raises(RuntimeError, match="KV cache exhausted: seq 0 needs 5 more blocks, only 4 free"):
        bt.ensure_capacity(s, 80)
    with pytest.raises(RuntimeError, match="device table holds 3"):
        bt.ensure_capacity(s, 64)  # 4 blocks > pitch 3
    bt.alloc()
    with pytest.raises(RuntimeError, match="sequence rows"):
        bt.alloc()


def test_random_ops_against_oracle_cache():
    from oracle.kvcache_ref import RefKVCache

    rng = random.Random(11)
    for trial in range(20):
        N = rng.randint(8, 80)
        perm = list(range(N))
        rng.shuffle(perm)
        ref = RefKVCache(N, 16, with_pool=False)
        ref.free_blocks = list(perm)
        bt = BlockTables(N, 16, max_seqs=1000, max_blocks_per_seq=N)
        bt._free_blocks = list(perm)
        live = []
        for _ in range(200):
            r = rng.random()
            try:
                if r < 0.2 or not live:
                    a, b = ref.alloc(), bt.alloc()
                    assert a == b
                    live.append(a)
                elif r < 0.6:
                    seqs = rng.sample(live, rng.randint(1, len(live)))
                    T = rng.choice([1, 1, 3, 16, 31])
                    e1 = e2 = None
                    try:
                        s1, slot, _ = ref.prepare(seqs, T)
                        ref.advance(seqs, T)
                    except RuntimeError as e:
                        e1 = str(e)
                    try:
                        s2, _ = bt.step_rows(seqs, T)
                        slot2 = _slots(bt, seqs, s2, T)
                        bt.advance(seqs, T)
                    except RuntimeError as e:
                        e2 = str(e)
                    assert e1 == e2
                    if e1 is None:
                        assert s1 == s2 and slot == slot2
                elif r < 0.75:
                    s = rng.choice(live)
                    ref.trim(s)
                    bt.trim(s)
                else:
                    s = rng.choice(live)
                    ref.free(s)
                    bt.free(s)
                    live.remove(s)
            finally:
                assert ref.free_blocks == bt._free_blocks
                assert ref.tables == bt._block_tables


def test_oracle_model_reproduces_reference_greedy_ids(golden):
    """The restated model (oracle) gives the reference's greedy ids on the CPU in
    fp32 with identical seeded weights (pins the whole-model oracle)."""
    import torch

    from oracle.kvcache_ref import RefKVCache
    from oracle.model_ref import RefQwen2
    from oracle.weights import random_state_dict

    fx = json.loads((golden / "model_greedy.json").read_text())
    torch.set_num_threads(max(1, min(8, torch.get_num_threads())))
    m = RefQwen2()
    m.load_state_dict(random_state_dict(fx["seed"], torch.float32))
    cache = RefKVCache(64, 16, torch.float32)
    seqs = [cache.alloc(), cache.alloc()]
    ids = [[], []]
    nxt = []
    for r in range(2):
        lg = m(torch.tensor([fx["prompts"][r]]), cache, [seqs[r]])[:, -1]
        nxt.append(int(lg[0].argmax()))
        ids[r].append(nxt[-1])
    for _ in range(fx["steps"]):
        lg = m(torch.tensor([[nxt[0]], [nxt[1]]]), cache, seqs)[:, -1]
        nxt = [int(lg[r].argmax()) for r in range(2)]
        for r in range(2):
            ids[r].append(nxt[r])
    assert ids == fx["ids"]


def test_pending_flat_arrays_match_pending_entries():
    """The flat [2, n] upload array (what KVCache.flush_tables copies to the
    device) holds exactly take_pending()'s cells: row * pitch + col and the
    block id, last write winning."""
    import numpy as np

    def ops(bt):
        a = bt.alloc()
        bt.ensure_capacity(a, 70)  # 5 blocks
        b = bt.alloc()
        bt.ensure_capacity(b, 33)  # 3 blocks
        bt.free(a)
        c = bt.alloc()  # reuses a's row before any flush: its cells are rewritten
        bt.ensure_capacity(c, 20)
        bt.ensure_capacity(b, 64)

    ref, flat = BlockTables(32, 16, max_seqs=4, max_blocks_per_seq=8), \
        BlockTables(32, 16, max_seqs=4, max_blocks_per_seq=8)
    ops(ref)
    ops(flat)
    want = {r * ref.table_pitch + c: blk for r, c, blk in ref.take_pending()}
    got = flat.take_pending_flat()
    assert got.dtype == np.int64 and got.shape == (2, len(want))
    assert dict(zip(got[0].tolist(), got[1].tolist())) == want
    assert flat.take_pending_flat() is None  # the queue is empty after a take
    assert flat._block_tables == ref._block_tables and flat._free_blocks == ref._free_blocks
