"""Generate the golden fixtures in this directory by running the REFERENCE
implementation (shubhav1/my-inference-engine, pure Python/PyTorch) on the CPU.

    python tests/golden/make_golden.py --reference /path/to/reference
    (or PKV_REFERENCE_DIR=/path/to/reference python tests/golden/make_golden.py)

Run only where the reference checkout exists (it is never read by tests, the
bench or smoke(); the fixtures it writes are what travels).  Every fixture
records the exact reference call sequence it came from:

  kvcache_ops.json     KVCache (kv_cache.py:8-121) driven by a seeded op
                       script: block tables, free list and lengths after every
                       op, prepare()'s slot_mapping / gather_idx.
  rope_append.npz      model.rope_cos_sin + apply_rope + KVCache.write in bf16
                       (model.py:58-65, :151-155; kv_cache.py:108-115):
                       bit patterns of roped q and of the written pool slots.
  attention_cases.npz  kernels/test_fa2.py CASES (:17-23) with its seed (0),
                       PAD_VALUE (100) and fp32 SDPA reference (:28-35).
  decode_config0.npz   BASELINE config 0: paged decode, B=4, ctx
                       {37,128,511,1000}, 1024-block pool from a seeded
                       permutation, through KVCache.prepare/write/read + the
                       model's SDPA branch in fp32 (model.py:104-107).
  prefill_config1.npz  BASELINE config 1 (reduced to 3 rows for size): ragged
                       causal prefill + append into a shuffled pool.
  scheduler_trace.json chat.py's scheduler (chat.py:110-311) driven tick by tick
                       with a fake model/tokenizer (oracle.scheduler_trace).
  model_greedy.json    Qwen2ForCausalLM (fp32, CPU, SDPA branch) with
                       oracle.weights.random_state_dict(seed) weights: greedy
                       ids of a 2-row batched prefill + decode through
                       KVCache.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---------------------------------------------------------------- KVCache ops
def gen_kvcache_ops(kv_cache_mod):
    rng = np.random.default_rng(1234)
    N = 64
    cache = kv_cache_mod.KVCache(N, 16, "cpu", torch.float32)
    perm = [int(x) for x in rng.permutation(N)]
    cache._free_blocks = list(perm)
    script, states = [], []
    live = []

    def snap(op, extra=None):
        states.append({
            "op": op,
            "free": list(cache._free_blocks),
            "tables": {str(k): list(v) for k, v in cache._block_tables.items()},
            "lengths": {str(k): v for k, v in cache._lengths.items()},
            "extra": extra,
        })

    for step in range(60):
        r = rng.random()
        if r < 0.15 or not live:
            s = cache.alloc()
            live.append(s)
            script.append(["alloc"])
            snap("alloc", s)
        elif r < 0.55:
            k = int(rng.integers(1, min(4, len(live)) + 1))
            seqs = [int(x) for x in rng.choice(live, size=k, replace=False)]
            T = int(rng.choice([1, 1, 1, 5, 16, 23]))
            try:
                starts, slot, gidx = cache.prepare(seqs, T)
                cache.advance(seqs, T)
                script.append(["prepare_advance", seqs, T])
                snap("prepare_advance", {"starts": starts, "slot_mapping": slot.tolist(),
                                         "gather_idx": gidx.tolist()})
            except RuntimeError as e:
                script.append(["prepare_advance", seqs, T])
                snap("prepare_advance", {"error": str(e)})
        elif r < 0.70:
            s = int(rng.choice(live))
            total = cache.length(s) + int(rng.integers(0, 60))
            try:
                cache.ensure_capacity(s, total)
                snap("ensure_capacity", None)
            except RuntimeError as e:
                snap("ensure_capacity", {"error": str(e)})
            script.append(["ensure_capacity", s, total])
        elif r < 0.85:
            s = int(rng.choice(live))
            cache.trim(s)
            script.append(["trim", s])
            snap("trim", None)
        else:
            s = int(rng.choice(live))
            cache.free(s)
            live.remove(s)
            script.append(["free", s])
            snap("free", None)
        # blocks_needed / free_block_count probes
        states[-1]["free_count"] = cache.free_block_count()
        states[-1]["blocks_needed"] = {str(s): cache.blocks_needed(s, cache.length(s) + 17) for s in live}
        states[-1]["blocks_needed_new_40"] = cache.blocks_needed(None, 40)
    return {"num_blocks": N, "block_size": 16, "initial_perm": perm, "script": script,
            "states": states}


# ---------------------------------------------------------------- rope + append
def gen_rope_append(model_mod, kv_cache_mod):
    g = torch.Generator().manual_seed(7)
    N = 24
    B, T = 3, 20
    prior = [5, 0, 37]  # tokens already in each row
    cache = kv_cache_mod.KVCache(N, 16, "cpu", torch.bfloat16)
    perm = torch.randperm(N, generator=g).tolist()
    cache._free_blocks = list(perm)
    seqs = [cache.alloc() for _ in range(B)]
    for s, n in zip(seqs, prior):  # pretend earlier steps wrote n tokens
        cache.ensure_capacity(s, n)
        cache._lengths[s] = n
    # pool starts with a recognisable non-zero pattern so untouched slots are checked too
    cache.buf.copy_(torch.randn(cache.buf.shape, generator=g).to(torch.bfloat16))
    pool_before = cache.buf.clone()
    Hq, Hkv, D = model_mod.NUM_HEADS, model_mod.NUM_KV_HEADS, model_mod.HEAD_DIM
    q = (torch.randn(B, Hq, T, D, generator=g) * 2.0).to(torch.bfloat16)
    k = (torch.randn(B, Hkv, T, D, generator=g) * 2.0).to(torch.bfloat16)
    v = (torch.randn(B, Hkv, T, D, generator=g) * 2.0).to(torch.bfloat16)
    m = model_mod.Qwen2ForCausalLM.__new__(model_mod.Qwen2ForCausalLM)
    torch.nn.Module.__init__(m)
    inv_freq = 1.0 / (model_mod.ROPE_THETA ** (torch.arange(0, D, 2).float() / D))
    m.register_buffer("inv_freq", inv_freq, persistent=False)
    starts, slot_mapping, gather_idx = cache.prepare(seqs, T)
    position_ids = torch.tensor(starts)[:, None] + torch.arange(T)[None, :]
    cos, sin = m.rope_cos_sin(position_ids, torch.bfloat16)
    qr, kr = model_mod.apply_rope(q, k, cos, sin)
    layer = 3
    cache.write(layer, slot_mapping, kr, v)
    tables = [list(cache._block_tables[s]) for s in seqs]
    width = max(len(t) for t in tables)
    tables_np = np.full((B, width), -1, np.int32)
    for i, t in enumerate(tables):
        tables_np[i, :len(t)] = t
    return dict(
        num_blocks=np.int64(N), layer=np.int64(layer), starts=np.array(starts, np.int32),
        T=np.int64(T), perm=np.array(perm, np.int32), tables=tables_np,
        q=bits(q), k=bits(k), v=bits(v), pool_before=bits(pool_before[layer]),
        cos=bits(cos[:, 0]), sin=bits(sin[:, 0]), q_roped=bits(qr), k_roped=bits(kr),
        pool_after=bits(cache.buf[layer]), slot_mapping=slot_mapping.numpy(),
        pool_other_layers_unchanged=np.bool_(torch.equal(
            torch.cat([cache.buf[:layer], cache.buf[layer + 1:]]),
            torch.cat([pool_before[:layer], pool_before[layer + 1:]]))),
    )


# ---------------------------------------------------------------- test_fa2 cases
PREFILL_ROW_STRIDE = 7  # the 300-token case keeps every 7th query row (fixture size)


def fa2_reference(model_mod, q, k, v, is_causal):
    # kernels/test_fa2.py:28-35
    q, k, v = q.float(), model_mod.repeat_kv(k.float()), model_mod.repeat_kv(v.float())
    T, S = q.shape[2], k.shape[2]
    mask = None
    if is_causal:
        mask = torch.arange(S)[None, :] <= torch.arange(T)[:, None] + (S - T)
    return F.scaled_dot_product_attention(q, k, v, attn_mask=mask)


def gen_attention_cases(model_mod):
    from oracle.cases import fa2_cases, sha as isha
    out = {}
    for ci, (name, q, k, v, lens, causal) in enumerate(fa2_cases()):
        B, T = q.shape[0], q.shape[2]
        ref = torch.zeros(B, 12, T, 128)
        for b, n in enumerate(lens):  # per row on its real keys (test_fa2.py:54-57)
            ref[b:b + 1] = fa2_reference(model_mod, q[b:b + 1], k[b:b + 1, :, :n], v[b:b + 1, :, :n], causal)
        rows = np.arange(0, T, PREFILL_ROW_STRIDE) if T == 300 else np.arange(T)
        out[f"c{ci}_rows"] = rows.astype(np.int32)
        out[f"c{ci}_out"] = ref[:, :, rows].numpy().astype(np.float32)
        out[f"c{ci}_lens"] = np.array(lens, np.int32)
        out[f"c{ci}_meta"] = np.array([T, int(causal)], np.int32)
        out[f"c{ci}_input_sha"] = np.array(isha(q, k, v))
    return out


def _drive_history(kv_cache_mod, cache, seqs, hist_k, hist_v):
    for s, kk, vv in zip(seqs, hist_k, hist_v):
        n = kk.shape[2]
        if n:
            st, sm, gi = cache.prepare([s], n)
            cache.write(0, sm, kk.float(), vv.float())
            cache.advance([s], n)


def _tables(cache, seqs):
    w = max(len(cache._block_tables[s]) for s in seqs)
    t = np.full((len(seqs), w), -1, np.int32)
    for i, s in enumerate(seqs):
        x = cache._block_tables[s]
        t[i, :len(x)] = x
    return t


def _model_mask(starts, T):
    # model.py:186-195: ragged starts -> explicit bottom-right mask [B,1,T,S]
    S = max(starts) + T
    key_pos = torch.arange(S)
    query_pos = torch.tensor(starts)[:, None] + torch.arange(T)[None, :]
    return (key_pos[None, None, :] <= query_pos[:, :, None]).unsqueeze(1)


# ---------------------------------------------------------------- config 0 decode
def gen_decode_config0(model_mod, kv_cache_mod):
    """BASELINE config 0 through the reference's own cache + SDPA branch (fp32)."""
    from oracle.cases import decode_config0_inputs, sha as isha
    inp = decode_config0_inputs()
    cache = kv_cache_mod.KVCache(inp["num_blocks"], 16, "cpu", torch.float32)
    cache._free_blocks = list(inp["perm"])
    seqs = [cache.alloc() for _ in inp["lens"]]
    _drive_history(kv_cache_mod, cache, seqs, inp["hist_k"], inp["hist_v"])
    starts, slot, gidx = cache.prepare(seqs, 1)
    cache.write(0, slot, inp["k_new"].float(), inp["v_new"].float())
    k, v = cache.read(0, gidx)
    mask = _model_mask(starts, 1)
    out = F.scaled_dot_product_attention(inp["q"].float(), model_mod.repeat_kv(k),
                                         model_mod.repeat_kv(v), attn_mask=mask)
    return dict(
        tables=_tables(cache, seqs), starts=np.array(starts, np.int32),
        slot_mapping=slot.numpy(), out=out.numpy().astype(np.float32),
        input_sha=np.array(isha(inp["q"], inp["k_new"], inp["v_new"], *inp["hist_k"], *inp["hist_v"])),
        pool_sha=np.array(isha(cache.buf[0].to(torch.bfloat16))),
    )


# ---------------------------------------------------------------- config 1 prefill
def gen_prefill_config1(model_mod, kv_cache_mod):
    """Ragged causal prefill + append (BASELINE config 1 shapes, 3 rows)."""
    from oracle.cases import prefill_config1_inputs, sha as isha
    inp = prefill_config1_inputs()
    T = inp["T"]
    cache = kv_cache_mod.KVCache(inp["num_blocks"], 16, "cpu", torch.float32)
    cache._free_blocks = list(inp["perm"])
    seqs = [cache.alloc() for _ in inp["prior"]]
    _drive_history(kv_cache_mod, cache, seqs, inp["hist_k"], inp["hist_v"])
    starts, slot, gidx = cache.prepare(seqs, T)
    cache.write(0, slot, inp["k_new"].float(), inp["v_new"].float())
    k, v = cache.read(0, gidx)
    mask = _model_mask(starts, T)
    out = F.scaled_dot_product_attention(inp["q"].float(), model_mod.repeat_kv(k),
                                         model_mod.repeat_kv(v), attn_mask=mask)
    return dict(
        tables=_tables(cache, seqs), starts=np.array(starts, np.int32),
        slot_mapping=slot.numpy(), out=out.numpy().astype(np.float32),
        input_sha=np.array(isha(inp["q"], inp["k_new"], inp["v_new"], *inp["hist_k"], *inp["hist_v"])),
        pool_sha=np.array(isha(cache.buf[0].to(torch.bfloat16))),
    )


# ---------------------------------------------------------------- whole model
def gen_model_greedy(model_mod, kv_cache_mod, seed=2024):
    sys.path.insert(0, str(REPO))
    from oracle.weights import random_state_dict

    torch.manual_seed(0)
    m = model_mod.Qwen2ForCausalLM()
    m.load_state_dict(random_state_dict(seed, torch.float32))
    m.eval()
    cache = kv_cache_mod.KVCache(64, 16, "cpu", torch.float32)
    seqs = [cache.alloc(), cache.alloc()]
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, model_mod.VOCAB_SIZE, (n,), generator=g).tolist() for n in (13, 29)]
    steps = 6
    ids = [[], []]
    margins = [[], []]
    with torch.no_grad():
        # prefill one row at a time (chat.py:_admit), then batched decode (chat.py:_process)
        nxt = []
        for r in range(2):
            logits = m(torch.tensor([prompts[r]]), cache, [seqs[r]])[:, -1].float()
            top = torch.topk(logits[0], 2)
            nxt.append(int(top.indices[0]))
            ids[r].append(nxt[-1])
            margins[r].append(float(top.values[0] - top.values[1]))
        for _ in range(steps):
            logits = m(torch.tensor([[nxt[0]], [nxt[1]]]), cache, seqs)[:, -1].float()
            nxt = []
            for r in range(2):
                top = torch.topk(logits[r], 2)
                nxt.append(int(top.indices[0]))
                ids[r].append(nxt[-1])
                margins[r].append(float(top.values[0] - top.values[1]))
    return {"seed": seed, "prompts": prompts, "steps": steps, "ids": ids, "margins": margins}


# ---------------------------------------------------------------- scheduler
def gen_scheduler_trace(reference):
    """The reference chat.py's own scheduling functions (admission, deferral,
    LRU eviction, one prefill per tick, batched decode, trim, release) driven
    deterministically by oracle.scheduler_trace."""
    import chat as chat_mod  # the reference's chat.py (CPU: fp32 cache, worker idle)
    import kv_cache as kv_cache_mod
    from oracle.scheduler_trace import run_trace

    assert Path(chat_mod.__file__).resolve().parent == Path(reference).resolve()

    def install(num_blocks):
        chat_mod.KV_CACHE = kv_cache_mod.KVCache(num_blocks, 16, "cpu", torch.float32)
        return chat_mod.KV_CACHE

    return run_trace(chat_mod, install)


def main():
    sys.path.insert(0, str(REPO))
    ap = argparse.ArgumentParser()
    env = os.environ.get("PKV_REFERENCE_DIR")
    ap.add_argument("--reference", default=env, required=env is None,
                    help="reference checkout (or set PKV_REFERENCE_DIR)")
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    import kv_cache as kv_cache_mod  # the reference's modules
    import model as model_mod

    assert Path(model_mod.__file__).resolve().parent == Path(a.reference).resolve(), \
        "imported the wrong model module"
    torch.set_num_threads(8)
    want = (a.only or "kvcache,rope,attn,dec0,pre1,model,sched").split(",")
    if "kvcache" in want:
        (HERE / "kvcache_ops.json").write_text(json.dumps(gen_kvcache_ops(kv_cache_mod)))
    if "rope" in want:
        np.savez_compressed(HERE / "rope_append.npz", **gen_rope_append(model_mod, kv_cache_mod))
    if "attn" in want:
        np.savez_compressed(HERE / "attention_cases.npz", **gen_attention_cases(model_mod))
    if "dec0" in want:
        np.savez_compressed(HERE / "decode_config0.npz", **gen_decode_config0(model_mod, kv_cache_mod))
    if "pre1" in want:
        np.savez_compressed(HERE / "prefill_config1.npz", **gen_prefill_config1(model_mod, kv_cache_mod))
    if "model" in want:
        (HERE / "model_greedy.json").write_text(json.dumps(gen_model_greedy(model_mod, kv_cache_mod)))
    if "sched" in want:
        (HERE / "scheduler_trace.json").write_text(json.dumps(gen_scheduler_trace(a.reference)))
    print("wrote", ", ".join(want))


if __name__ == "__main__":
    main()
