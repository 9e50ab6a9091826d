"""Host-side pieces of the mixed-step graphs and the persistent decode-layers
entry point (no GPU): bucket choice, argument checks before any device
call, and the work split the kernel's plan relies on."""
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
