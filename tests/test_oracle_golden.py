"""The CPU oracle reproduces the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py from the reference checkout).  This pins the oracle
before any GPU result is compared with it."""
import json

import numpy as np
import pytest
import torch

from oracle import attention_ref, cases, rope_ref
from oracle.kvcache_ref import RefKVCache


def test_oracle_kvcache_matches_reference_op_by_op(golden):
    fx = json.loads((golden / "kvcache_ops.json").read_text())
    c = RefKVCache(fx["num_blocks"], fx["block_size"], with_pool=False)
    c.free_blocks = list(fx["initial_perm"])
    for op, st in zip(fx["script"], fx["states"]):
        extra = None
        err = None
        try:
            if op[0] == "alloc":
                extra = c.alloc()
            elif op[0] == "prepare_advance":
                starts, slot, gather = c.prepare(op[1], op[2])
                c.advance(op[1], op[2])
                extra = {"starts": starts, "slot_mapping": slot, "gather_idx": gather.tolist()}
            elif op[0] == "ensure_capacity":
                c.ensure_capacity(op[1], op[2])
            elif op[0] == "trim":
                c.trim(op[1])
            elif op[0] == "free":
                c.free(op[1])
        except RuntimeError as e:
            err = str(e)
        if err is not None:
            assert st["extra"] == {"error": err}
        elif op[0] in ("alloc", "prepare_advance"):
            assert st["extra"] == extra
        assert st["free"] == c.free_blocks
        assert st["tables"] == {str(k): v for k, v in c.tables.items()}
        assert st["lengths"] == {str(k): v for k, v in c.lengths.items()}
        assert st["free_count"] == c.free_block_count()
        assert st["blocks_needed_new_40"] == c.blocks_needed(None, 40)


def test_oracle_rope_is_bit_exact_with_reference(golden):
    fx = np.load(golden / "rope_append.npz")
    T = int(fx["T"])
    pos = fx["starts"][:, None] + np.arange(T)[None, :]
    cos, sin = rope_ref.rope_table_bits(pos.reshape(-1))
    assert np.array_equal(cos.reshape(fx["cos"].shape), fx["cos"])
    assert np.array_equal(sin.reshape(fx["sin"].shape), fx["sin"])
    c = fx["cos"][:, None]  # [B,1,T,D]
    s = fx["sin"][:, None]
    assert np.array_equal(rope_ref.rope_bits(fx["q"], c, s), fx["q_roped"])
    assert np.array_equal(rope_ref.rope_bits(fx["k"], c, s), fx["k_roped"])


def test_oracle_append_matches_reference_pool(golden):
    fx = np.load(golden / "rope_append.npz")
    layer = int(fx["layer"])
    N = int(fx["num_blocks"])
    c = RefKVCache(N, 16, dtype=torch.bfloat16, num_layers=layer + 1)
    c.buf[layer] = cases.from_bits(fx["pool_before"]).view(c.buf[layer].shape)
    c.free_blocks = [int(x) for x in fx["perm"]]
    starts = [int(x) for x in fx["starts"]]
    seqs = [c.alloc() for _ in starts]
    for s, n in zip(seqs, starts):
        c.ensure_capacity(s, n)
        c.lengths[s] = n
    st, slot, _ = c.prepare(seqs, int(fx["T"]))
    assert np.array_equal(np.array(slot), fx["slot_mapping"])
    c.write(layer, slot, cases.from_bits(fx["k_roped"]), cases.from_bits(fx["v"]))
    assert np.array_equal(cases.bits(c.buf[layer]), fx["pool_after"])


@pytest.mark.parametrize("ci", range(len(cases.FA2_CASES)))
def test_oracle_attention_matches_reference_fa2_cases(golden, ci):
    fx = np.load(golden / "attention_cases.npz")
    name, q, k, v, lens, causal = cases.fa2_cases()[ci]
    assert cases.sha(q, k, v) == str(fx[f"c{ci}_input_sha"]), "torch CPU RNG drifted"
    rows = fx[f"c{ci}_rows"]
    want = fx[f"c{ci}_out"]
    got = attention_ref.attention_np(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                     lens, causal)[:, :, rows]
    assert np.abs(got - want).max() < 1e-4, name


def _paged_oracle(inp, T_new):
    """Drive RefKVCache like the reference model does for one layer and return
    (starts, slot_mapping, tables, fp32 output)."""
    c = RefKVCache(inp["num_blocks"], 16, dtype=torch.float32, num_layers=1)
    c.free_blocks = list(inp["perm"])
    seqs = [c.alloc() for _ in inp["hist_k"]]
    for s, kk, vv in zip(seqs, inp["hist_k"], inp["hist_v"]):
        n = kk.shape[2]
        if n:
            st, sm, _ = c.prepare([s], n)
            c.write(0, sm, kk.float(), vv.float())
            c.advance([s], n)
    starts, slot, gather = c.prepare(seqs, T_new)
    c.write(0, slot, inp["k_new"].float(), inp["v_new"].float())
    k, v = c.read(0, gather)
    out = attention_ref.sdpa_reference(inp["q"].float(), k, v,
                                       attention_ref.bottom_right_mask(starts, T_new))
    tables = [c.tables[s] for s in seqs]
    return starts, slot, tables, out, c


def test_oracle_decode_config0_matches_reference(golden):
    fx = np.load(golden / "decode_config0.npz")
    inp = cases.decode_config0_inputs()
    assert cases.sha(inp["q"], inp["k_new"], inp["v_new"], *inp["hist_k"], *inp["hist_v"]) == \
        str(fx["input_sha"])
    starts, slot, tables, out, c = _paged_oracle(inp, 1)
    assert starts == list(fx["starts"])
    assert np.array_equal(np.array(slot), fx["slot_mapping"])
    for i, t in enumerate(tables):
        assert t == [x for x in fx["tables"][i] if x >= 0]
    assert np.abs(out.numpy() - fx["out"]).max() < 1e-5
    assert cases.sha(c.buf[0].to(torch.bfloat16)) == str(fx["pool_sha"])


def test_oracle_prefill_config1_matches_reference(golden):
    fx = np.load(golden / "prefill_config1.npz")
    inp = cases.prefill_config1_inputs()
    assert cases.sha(inp["q"], inp["k_new"], inp["v_new"], *inp["hist_k"], *inp["hist_v"]) == \
        str(fx["input_sha"])
    starts, slot, tables, out, c = _paged_oracle(inp, inp["T"])
    assert np.array_equal(np.array(slot), fx["slot_mapping"])
    assert np.abs(out.numpy() - fx["out"]).max() < 1e-5
    assert cases.sha(c.buf[0].to(torch.bfloat16)) == str(fx["pool_sha"])
    # float64 restatement on the dense history agrees with the reference SDPA
    B, T = inp["q"].shape[0], inp["T"]
    kd = [torch.cat([h, n], dim=2) for h, n in zip(
        [x.float() for x in inp["hist_k"]], inp["k_new"].float().split(1))]
    vd = [torch.cat([h, n], dim=2) for h, n in zip(
        [x.float() for x in inp["hist_v"]], inp["v_new"].float().split(1))]
    for b in range(B):
        got = attention_ref.attention_np(inp["q"][b:b + 1].float().numpy(), kd[b].numpy(),
                                         vd[b].numpy(), [kd[b].shape[2]], True)
        assert np.abs(got - fx["out"][b:b + 1]).max() < 1e-4


def test_oracle_philox_matches_published_known_answers():
    """The sampler oracle's Philox-4x32-10 against the known-answer vectors of
    the generator's authors (Random123 kat_vectors: zero, all-ones, and the
    pi-digits counter/key)."""
    import numpy as np

    from oracle.sample_ref import philox4x32_10

    kats = [
        ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
        ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
        ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
         (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
    ]
    for ctr, key, want in kats:
        got = philox4x32_10(np.array([ctr], dtype=np.uint32), key)[0]
        assert [int(x) for x in got] == list(want)


def test_oracle_gumbel_sampling_follows_softmax():
    """The oracle's Gumbel-max draw has the reference sampler's distribution
    (softmax(logits / T), chat.py:103-107) on a small vocabulary."""
    import numpy as np

    from oracle.sample_ref import sample

    logits = np.array([[1.5, 0.0, -1.0, 2.0, 0.5, -3.0, 1.0, 0.25]], dtype=np.float32)
    for temp in (1.0, 0.6):
        ids = np.concatenate([sample(np.repeat(logits, 4000, 0), temp, 1234, c) for c in range(5)])
        p = np.exp(logits[0] / temp - (logits[0] / temp).max())
        p /= p.sum()
        freq = np.bincount(ids, minlength=8) / ids.size
        sigma = np.sqrt(p * (1 - p) / ids.size)
        assert np.all(np.abs(freq - p) < 5 * sigma + 1e-3), (temp, freq, p)
