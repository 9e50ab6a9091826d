"""Host-side pieces of the mixed-step graphs, the persistent decode-layers
entry point and the paged decode kernel's partitioning (no GPU): bucket
choice, argument checks before any device call, and the work splits the
kernels' plans rely on."""
import ctypes

import pytest
import torch


def test_prefill_buckets_cover_every_length_with_bounded_padding():
    import model as M

    b = M._prefill_buckets(4096)
    assert b[0] == 64 and b[-1] == 4096 and b == sorted(set(b))
    for T in range(2, 4097, 7):
        Tp = next(x for x in b if x >= T)
        # 64 at least; up to 256 tokens the buckets double; above, steps of 128
        if T > 64:
            assert (Tp - T < Tp // 2) if T <= 256 else (Tp - T < 128)
    assert M._prefill_buckets(100) == [64, 100]


def test_decode_layers_rejects_bad_arguments_before_touching_the_device():
    import pagedkv

    L = pagedkv.lib()
    tab = pagedkv.LayerTable([{"qkv_w": torch.zeros(4)}])
    arr = ctypes.cast(tab.arr, ctypes.c_void_p)
    # no layers / too many layers / too many rows: refused up front
    assert L.pkv_decode_layers(arr, 0, None, None, None, 4, None, 0, None, 0, None, None, None,
                               None, 0, 1e-6, None, 0, None, None) == pagedkv.PKV_OK + 2
    assert L.pkv_decode_layers(arr, 33, None, None, None, 4, None, 0, None, 0, None, None, None,
                               None, 0, 1e-6, None, 0, None, None) == 2
    assert L.pkv_decode_layers(arr, 1, None, None, None, 33, None, 0, None, 0, None, None, None,
                               None, 0, 1e-6, None, 0, None, None) == 2
    # null activations
    assert L.pkv_decode_layers(arr, 1, None, None, None, 4, None, 0, None, 0, None, None, None,
                               None, 0, 1e-6, None, 0, None, None) == 1
    assert L.pkv_decode_layers_workspace_size(0) == 0
    assert L.pkv_decode_layers_workspace_size(33) == 0


def test_layer_table_requires_contiguous_weights():
    import pagedkv

    w = torch.zeros(8, 8)
    with pytest.raises(ValueError):
        pagedkv.LayerTable([{"qkv_w": w.t()}])
    with pytest.raises(ValueError):
        pagedkv.LayerTable([])
    t = pagedkv.LayerTable([{"qkv_w": w, "o_w": w}])
    assert len(t) == 1 and t.arr[0].qkv_w == w.data_ptr() and t.arr[0].down_w is None


@pytest.mark.parametrize("sms", [132, 148, 160])
def test_decode_layers_work_split(sms):
    """The split the kernel uses (a restatement of layers.cu's unit ranges):
    every unit of every phase has exactly one owner, a CTA's range spans at
    most two 128-row tiles, the gate/up phase gives whole tiles to CTAs, and
    each split tile's partials are read back in CTA order."""
    phases = {"qkv": (16, 24), "o": (12, 24), "gu": (140, 24), "down": (12, 140)}

    def begin(ph, c):
        T, C = phases[ph]
        if ph == "gu" and T <= sms:
            return min(c, T) * C
        return (c * T * C + sms - 1) // sms

    for ph, (T, C) in phases.items():
        owners = {}
        for c in range(sms):
            u0, u1 = begin(ph, c), begin(ph, c + 1)
            assert u1 >= u0
            if u1 > u0:
                assert (u1 - 1) // C - u0 // C <= 1
            for u in range(u0, u1):
                assert u not in owners
                owners[u] = c
        assert sorted(owners) == list(range(T * C))
        for t in range(T):
            cs = sorted({owners[u] for u in range(t * C, (t + 1) * C)})
            assert cs == list(range(cs[0], cs[-1] + 1))  # consecutive CTAs
            if ph == "gu" and T <= sms:
                assert cs == [t]


def _decode_rule(units, nblk):
    """min_blocks_per_part_for (csrc/decode.cu): 32 when rows of nblk blocks
    would keep 600 CTAs of 32 blocks busy, 16 likewise, else 4."""
    if units * (nblk // 32) >= 600:
        return 32
    if units * (nblk // 16) >= 600:
        return 16
    return 4


def _decode_host_plan(batch, hkv, max_kv_len, fp8):
    """plan_decode + the per-launch thresholds of launch_decode (decode.cu)."""
    units = batch * hkv
    nblk = max(1, -(-max_kv_len // 16))
    target = (2 if fp8 else 1) * 148 * 2 * 6
    parts = min(-(-target // units), 16)
    mb = _decode_rule(units, nblk)
    bpp = max(-(-nblk // parts), mb)
    bpp = -(-bpp // 4) * 4
    max_parts = -(-nblk // bpp)
    need = -(-600 // units)
    wave = (2 if fp8 else 1) * (148 if units >= 128 else 296)
    return {"units": units, "min_bpp": mb, "max_parts": max_parts, "busy32": need * 32,
            "busy16": need * 16, "wave_parts": max(1, wave // units)}


def _decode_row_parts(plan, kv_len):
    """The kernel's partitioning of one row (paged_decode_kernel): returns the
    (first block, block count) of every non-empty partition."""
    nblk = -(-kv_len // 16)
    row_min = 32 if nblk >= plan["busy32"] else 16 if nblk >= plan["busy16"] else 4
    min_bpp = min(plan["min_bpp"], row_min)
    np_ = min(plan["max_parts"], max(1, nblk // min_bpp))
    if row_min < 32:
        np_ = min(np_, plan["wave_parts"])
    per = -(-nblk // np_)
    bpp = max(4, -(-per // 4) * 4)
    nparts = -(-nblk // bpp)
    out = []
    for part in range(plan["max_parts"]):
        if part * 4 >= nblk or part >= nparts:  # the kernel's early exits
            continue
        b0 = part * bpp
        out.append((b0, min(nblk, b0 + bpp) - b0))
    return out


@pytest.mark.parametrize("fp8", [False, True])
def test_decode_partitions_cover_every_block_once(fp8):
    """Per-row partition minimum and the one-wave cap (decode.cu): for plans
    made for the rows' maximum or for a 16k-token graph capacity, every row's
    partitions cover its blocks exactly once, never exceed the grid's
    partitions, and a row below the busy threshold gets at most the
    one-wave share of partitions (so a launch of such rows stays within
    about one wave of resident CTAs)."""
    import random

    rng = random.Random(5)
    for _ in range(400):
        batch = rng.choice([1, 2, 8, 16, 32, 64, 128, 256])
        lens = [rng.randint(1, 9000) for _ in range(batch)]
        for plan_len in (max(lens), 16384):
            plan = _decode_host_plan(batch, 2, plan_len, fp8)
            for n in lens:
                parts = _decode_row_parts(plan, n)
                nblk = -(-n // 16)
                covered = [b for b0, cnt in parts for b in range(b0, b0 + cnt)]
                assert covered == list(range(nblk)), (batch, n, plan_len)
                assert 1 <= len(parts) <= plan["max_parts"]
                if nblk < plan["busy32"]:
                    assert len(parts) <= plan["wave_parts"], (batch, n, plan_len)


def test_decode_thresholds_restate_the_rule():
    """The host's block thresholds give the rule's answer for every length."""
    for units in (2, 16, 32, 64, 128, 256, 512, 1024):
        plan = _decode_host_plan(units // 2, 2, 8192, False)
        for nblk in range(0, 700):
            row = 32 if nblk >= plan["busy32"] else 16 if nblk >= plan["busy16"] else 4
            assert row == _decode_rule(units, nblk)
