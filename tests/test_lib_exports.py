"""libpagedkv.so loads without a GPU and exports every symbol of the header."""
import ctypes
import re

from conftest import REPO


def _header_symbols():
    text = (REPO / "include" / "pagedkv.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(pkv_\w+)\s*\(", text, re.M)))


def test_header_declares_expected_entry_points():
    syms = _header_symbols()
    for s in ["pkv_append_rope", "pkv_paged_decode", "pkv_paged_prefill", "pkv_dense_attention",
              "pkv_decode_workspace_size", "pkv_decode_plan", "pkv_version", "pkv_status_string", "pkv_last_error"]:
        assert s in syms


def test_library_builds_loads_and_exports_all_symbols():
    import pagedkv_build

    path = pagedkv_build.build()
    lib = ctypes.CDLL(str(path))
    for s in _header_symbols():
        assert hasattr(lib, s), f"{s} declared in pagedkv.h but not exported"
    import pagedkv

    L = pagedkv.lib()
    assert set(pagedkv.exported_symbols()) == set(_header_symbols()), \
        "the ctypes binding and the header disagree"
    assert L.pkv_version() >= 100
    assert L.pkv_status_string(0) == b"ok"
    assert L.pkv_status_string(6) == b"workspace too small"


def test_decode_workspace_plan_is_host_only_and_sane():
    import pagedkv

    L = pagedkv.lib()
    # short contexts need no split-K scratch
    assert L.pkv_decode_workspace_size(4, 12, 2, 37) == 0
    # long contexts split into partitions: scratch is needed, and bounded by
    # the planner's CTA target (~1776 partitions) plus the 256 KiB counter head
    for B in (1, 4, 8, 64, 256):
        n = L.pkv_decode_workspace_size(B, 12, 2, 8192)
        assert 0 < n < (256 << 10) + 4000 * 8 * 129 * 4, (B, n)
    # a batch that alone fills the machine needs no split (for either pool
    # format: the FP8 kernel plans for twice the resident CTAs)
    assert L.pkv_decode_workspace_size(2048, 12, 2, 8192) == 0
    # invalid head counts report 0 instead of failing
    assert L.pkv_decode_workspace_size(4, 12, 5, 8192) == 0


def test_decode_plan_branches():
    """pkv_decode_plan reports the partition sizing of a launch: the timed
    config-3 launch (256 rows up to 8192 tokens) and the engine's 128-row
    ~2100-token decode take 32-block partitions, a 4-row launch 4-block ones."""
    import pagedkv

    p = pagedkv.decode_plan(256, 12, 2, 8192)
    assert (p["blocks_per_part"], p["min_blocks_per_part"], p["max_parts"]) == (128, 32, 4), p
    p = pagedkv.decode_plan(128, 12, 2, 2100)
    assert (p["min_blocks_per_part"], p["max_parts"]) == (32, 5), p
    p = pagedkv.decode_plan(4, 12, 2, 8192)
    assert p["min_blocks_per_part"] == 4 and p["sub_groups"] == 1, p
    assert pagedkv.lib().pkv_decode_plan(4, 12, 5, 8192, None) == 1


def test_entry_points_reject_bad_arguments_without_a_gpu():
    """Validation runs before any CUDA call, so it is testable on the CPU."""
    import pagedkv

    L = pagedkv.lib()
    # head_dim 64 -> PKV_ERR_UNSUPPORTED
    st = L.pkv_paged_decode(16, 0, 0, 16, 16, 16, 16, 1, None, 16, 1, 1, 12, 2, 64, 1.0,
                            16, 0, 0, None, 0, None, None)
    assert st == 2 and b"head_dim" in L.pkv_last_error()
    # Hq not a multiple of Hkv -> PKV_ERR_INVALID
    st = L.pkv_paged_prefill(16, 0, 0, 0, 16, 16, 16, 16, 1, None, 16, None, 1, 1, 1, 12, 5, 128,
                             1, 1.0, 16, 0, 0, 0, None, None)
    assert st == 1
    # misaligned pool plane -> PKV_ERR_ALIGN
    st = L.pkv_paged_decode(16, 0, 0, 18, 16, 16, 16, 1, None, 16, 1, 1, 12, 2, 128, 1.0,
                            16, 0, 0, None, 0, None, None)
    assert st == 3
    # num_slots not a multiple of 16 -> PKV_ERR_INVALID
    st = L.pkv_append_rope(None, 0, 0, 0, 16, 0, 0, 0, 16, 0, 0, 0, None, None, 0, None, 0, 0, 0,
                           16, 16, 17, 16, 1, None, 16, None, 1, 12, 2, 1, 128, None, None)
    assert st == 1


def test_linear_workspace_plan_and_validation_without_a_gpu():
    import pagedkv

    L = pagedkv.lib()
    # the fused entries keep the bf16 GEMM output: rows * n * 2 bytes
    for rows, n, k in ((1, 2048, 1536), (16, 1536, 8960), (256, 17920, 1536)):
        assert L.pkv_linear_workspace_size(rows, n, k) == rows * n * 2
    for bad in ((0, 2048, 1536), (257, 2048, 1536), (16, 2000, 1536), (16, 2048, 1000)):
        assert L.pkv_linear_workspace_size(*bad) == 0
    # argument checks come before any CUDA call
    st = L.pkv_linear(16, 1536, 16, 1536, 0, None, 300, 2048, 1536, 16, 2048, None, 0, None, None)
    assert st == 2  # PKV_ERR_UNSUPPORTED: more than 256 rows
    st = L.pkv_linear(16, 1536, 16, 1536, 0, None, 16, 2048, 1000, 16, 2048, None, 0, None, None)
    assert st == 2  # k not a multiple of 64
    st = L.pkv_linear(8, 1536, 16, 1536, 0, None, 16, 2048, 1536, 16, 2048, None, 0, None, None)
    assert st == 3  # PKV_ERR_ALIGN: x not 16-byte aligned
    st = L.pkv_linear_silu_mul(16, 1536, 16, 1536, 0, 16, 100, 1536, 16, 100, None, 0, None, None)
    assert st == 2  # inter not a multiple of 64
    st = L.pkv_linear_silu_mul(16, 1536, 16, 1536, 0, 16, 8960, 1536, 16, 8960, None, 0, None,
                               None)
    assert st == 6  # PKV_ERR_WORKSPACE: the fused entries need their intermediate
    st = L.pkv_linear(16, 1536, 16, 1536, 7, None, 16, 2048, 1536, 16, 2048, None, 0, None, None)
    assert st == 1  # unknown weight layout
    st = L.pkv_linear_pack_weight(16, 1536, 2000, 1536, 16, None)
    assert st == 2  # n not a multiple of 128
    st = L.pkv_linear_pair_gate_up(16, 1536, 100, 1536, 16, None)
    assert st == 2  # inter not a multiple of 64
    st = L.pkv_linear(16, 1536, 16, 1536, 2, None, 16, 17920, 1536, 16, 17920, None, 0, None, None)
    assert st == 1  # the paired gate/up layout is only for pkv_linear_silu_mul


def test_sample_validation_without_a_gpu():
    """pkv_sample checks its arguments before any CUDA call."""
    import pagedkv

    L = pagedkv.lib()
    out = 16
    # dtype must be 0 (bf16) or 1 (f32)
    assert L.pkv_sample(16, 1000, 4, 1000, 2, 1.0, 1, 0, out, None) == 2
    # temperature must be positive and finite
    assert L.pkv_sample(16, 1000, 4, 1000, 0, 0.0, 1, 0, out, None) == 1
    assert L.pkv_sample(16, 1000, 4, 1000, 0, -1.0, 1, 0, out, None) == 1
    assert L.pkv_sample(16, 1000, 4, 1000, 0, float("inf"), 1, 0, out, None) == 1
    assert L.pkv_sample(16, 1000, 4, 1000, 0, float("nan"), 1, 0, out, None) == 1
    # ld shorter than the vocabulary, too many rows, null pointers
    assert L.pkv_sample(16, 999, 4, 1000, 0, 1.0, 1, 0, out, None) == 1
    assert L.pkv_sample(16, 1000, 70000, 1000, 0, 1.0, 1, 0, out, None) == 1
    assert L.pkv_sample(None, 1000, 4, 1000, 0, 1.0, 1, 0, out, None) == 1
    assert L.pkv_sample(16, 1000, 4, 1000, 0, 1.0, 1, 0, None, None) == 1
    # f32 logits not 4-byte aligned
    assert L.pkv_sample(18, 1000, 4, 1000, 1, 1.0, 1, 0, out, None) == 3
    # zero rows: nothing to launch
    assert L.pkv_sample(16, 1000, 0, 1000, 0, 1.0, 1, 0, out, None) == 0


def test_chat_reads_sampled_ids_and_raises_on_unsampled_rows():
    """Host half of chat's sampling: ids come back as Python ints; a row the
    device sampler marked -1 (no finite logit) raises as torch.multinomial
    does on such a row (reference chat.py:103-107)."""
    import pytest
    import torch

    import chat

    assert chat._read_ids(torch.tensor([3, 0, 7], dtype=torch.int32)) == [3, 0, 7]
    assert chat._read_ids(torch.tensor([], dtype=torch.int32)) == []
    with pytest.raises(RuntimeError, match="probability tensor"):
        chat._read_ids(torch.tensor([3, -1], dtype=torch.int32))
    tok = chat._PendingToken(torch.tensor([42], dtype=torch.int32))
    assert tok.get() == 42
