"""pkv_paged_decode_static_scratch: paged decode for callers that cannot call
cudaMalloc (their host owns the device allocator, or forbids allocation while
serving).  It takes the same inputs and outputs as pkv_paged_decode but keeps
its split-K scratch in a static device array inside the library, so the caller
passes no workspace.  These tests call both entry points through the C ABI on
the same inputs and require the same answer, on two calls in a row with
different shapes (the array keeps the previous call's contents), and check
that a shape needing more scratch than the array holds is refused.

The file name sorts last so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
import ctypes
import math

import pytest
import torch

from gpu_helpers import build_cache, max_err, write_history
from oracle import cases

pytestmark = pytest.mark.gpu


def _case(device, lens, seed):
    """Pool, tables and one decode step's q for rows of `lens` tokens (PAD-poisoned pool)."""
    g = torch.Generator().manual_seed(seed)
    N = sum(math.ceil(n / 16) for n in lens) + 8
    cache = build_cache(N, torch.randperm(N, generator=g).tolist(), device)
    cache.buf.fill_(cases.PAD_VALUE)
    seqs = [cache.alloc() for _ in lens]
    hk = [torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16) for n in lens]
    hv = [torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16) for n in lens]
    write_history(cache, seqs, hk, hv)
    # decode over the rows' existing lengths: kv_lens = lens
    rows = torch.tensor([cache.table_row(s) for s in seqs], dtype=torch.int32, device=device)
    kv_lens = torch.tensor(lens, dtype=torch.int32, device=device)
    q = torch.randn(len(lens), 12, 128, generator=g).to(torch.bfloat16).to(device)
    torch.cuda.synchronize()
    return cache, rows, kv_lens, q


def _call_static(lib, cache, rows, kv_lens, q, out, max_kv_len):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.pkv_paged_decode_static_scratch(
        q.data_ptr(), q.stride(0), q.stride(1),
        cache.buf[0, 0].data_ptr(), cache.buf[0, 1].data_ptr(), cache.buf.shape[2],
        cache.block_tables.data_ptr(), cache.block_tables.stride(0),
        rows.data_ptr(), kv_lens.data_ptr(), max_kv_len, q.shape[0], 12, 2, 128,
        1.0 / math.sqrt(128), out.data_ptr(), out.stride(0), out.stride(1),
        cache.err_flag.data_ptr(), stream)


def _call_workspace(lib, cache, rows, kv_lens, q, out, max_kv_len):
    """The existing entry point, with a workspace this test allocates."""
    need = lib.pkv_decode_workspace_size(q.shape[0], 12, 2, max_kv_len)
    ws = torch.zeros(max(need, 16), dtype=torch.uint8, device=q.device)
    stream = torch.cuda.current_stream().cuda_stream
    st = lib.pkv_paged_decode(
        q.data_ptr(), q.stride(0), q.stride(1),
        cache.buf[0, 0].data_ptr(), cache.buf[0, 1].data_ptr(), cache.buf.shape[2],
        cache.block_tables.data_ptr(), cache.block_tables.stride(0),
        rows.data_ptr(), kv_lens.data_ptr(), max_kv_len, q.shape[0], 12, 2, 128,
        1.0 / math.sqrt(128), out.data_ptr(), out.stride(0), out.stride(1),
        ws.data_ptr(), ws.numel(), cache.err_flag.data_ptr(), stream)
    torch.cuda.synchronize()
    return st


def test_static_scratch_decode_matches_workspace_decode_twice(cuda):
    import pagedkv

    lib = pagedkv.lib()
    # two calls in a row with different shapes; both need split-K scratch
    for lens, seed in (([8192, 5000, 300, 37, 16, 1], 1), ([4096, 2049, 7000], 2)):
        cache, rows, kv_lens, q = _case(cuda, lens, seed)
        max_kv_len = max(lens)
        assert lib.pkv_decode_workspace_size(len(lens), 12, 2, max_kv_len) > 0
        want = torch.empty_like(q)
        assert _call_workspace(lib, cache, rows, kv_lens, q, want, max_kv_len) == 0
        got = torch.full_like(q, float("nan"))
        st = _call_static(lib, cache, rows, kv_lens, q, got, max_kv_len)
        assert st == 0, lib.pkv_last_error().decode()
        torch.cuda.synchronize()
        cache.check_errors()
        # same kernel, same plan, same merge order: identical bits, so leftover
        # contents of the shared array from the previous call cannot leak in
        assert torch.equal(got, want), (lens, max_err(got, want))
        assert torch.isfinite(got.float()).all()


def test_static_scratch_refuses_shapes_beyond_its_size(cuda):
    import pagedkv

    lib = pagedkv.lib()
    B, max_kv_len = 400, 8192  # needs ~10 MB of split-K scratch
    need = lib.pkv_decode_workspace_size(B, 12, 2, max_kv_len)
    limit = 8 << 20
    assert need > limit
    # small, valid buffers: the call must refuse on the host and launch nothing
    cache = build_cache(4, [0, 1, 2, 3], cuda, max_seqs=B, max_blocks_per_seq=512)
    rows = torch.arange(B, dtype=torch.int32, device=cuda)
    kv_lens = torch.full((B,), 16, dtype=torch.int32, device=cuda)
    q = torch.zeros(B, 12, 128, dtype=torch.bfloat16, device=cuda)
    out = torch.zeros_like(q)
    st = _call_static(lib, cache, rows, kv_lens, q, out, max_kv_len)
    assert st == 6  # PKV_ERR_WORKSPACE
    msg = lib.pkv_last_error().decode()
    assert "static" in msg and str(limit) in msg
    torch.cuda.synchronize()
    assert int(out.count_nonzero()) == 0
