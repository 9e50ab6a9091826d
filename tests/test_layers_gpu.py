"""pkv_decode_layers (every decoder layer of a small decode step in one
persistent launch) against the per-op kernels it replaces.

Both arms run the same random-init Qwen2.5-1.5B on identical caches; the
persistent kernel computes the same ops with the same bf16 rounding points,
and differs only in fp32 summation order (its k-split sums and the RMSNorm
sums of squares), so logits, the residual stream and the appended K/V agree
to a few bf16 ulps.  The greedy ids against the oracle (with the persistent
step on) are in tests/test_model_gpu.py (`persistent` path)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(cuda):
    import model as M

    torch.manual_seed(0)
    m = M.Qwen2ForCausalLM().to(cuda, torch.bfloat16).eval()
    g = torch.Generator(device=cuda).manual_seed(7)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if name.endswith("layernorm.weight") or name == "norm.weight":
                p.normal_(1.0, 0.1, generator=g)
            else:
                p.normal_(0.0, 0.02, generator=g)
    return m.fuse_weights_()


def _run(m, cuda, prompts, steps, persistent, graphs=False, cublas=False):
    from kv_cache import KVCache

    c = KVCache(1024, 16, cuda, torch.bfloat16)
    seqs = [c.alloc() for _ in prompts]
    saved = m.persistent_decode, m.skinny_linears
    out = []
    try:
        with torch.no_grad():
            m.persistent_decode = False  # identical prefills in every arm
            for s, p in zip(seqs, prompts):
                m(torch.tensor([p], device=cuda), c, [s])
            m.persistent_decode = persistent
            m.skinny_linears = not cublas
            if graphs:
                dg = m.enable_decode_graphs(c, max_batch=len(prompts) + 3)
                dg.buckets = [len(prompts) + 3]  # padded, inactive rows in the step
            for i in range(steps):
                ids = torch.tensor([[100 + 7 * i + r] for r in range(len(prompts))])
                out.append(m(ids if graphs else ids.to(cuda), c, seqs)[:, -1].float().clone())
        torch.cuda.synchronize()
        c.check_errors()
    finally:
        m.persistent_decode, m.skinny_linears = saved
        m._graphs.clear()
    return out, c


@pytest.mark.parametrize("rows", [1, 5, 16, 17, 32])
def test_decode_layers_matches_per_op_kernels(cuda, model, rows):
    g = torch.Generator().manual_seed(rows)
    lens = [int(x) for x in torch.randint(1, 300, (rows,), generator=g)]
    lens[0] = 1  # one row attends to its first token only
    if rows > 2:
        lens[1] = 290  # and one to many blocks
    prompts = [torch.randint(0, 151936, (n,), generator=g).tolist() for n in lens]
    ref, c_ref = _run(model, cuda, prompts, 3, persistent=False)
    got, c_got = _run(model, cuda, prompts, 3, persistent=True)
    # the yardstick: the same per-op step with every projection on cuBLAS,
    # which differs from the skinny GEMMs only in fp32 summation order too
    alt, c_alt = _run(model, cuda, prompts, 3, persistent=False, cublas=True)
    for a, b, y in zip(ref, got, alt):
        d, dy = (a - b).abs(), (a - y).abs()
        msg = (f"persistent vs per-op: max {float(d.max()):.4f} mean {float(d.mean()):.5f}; "
               f"cuBLAS vs per-op: max {float(dy.max()):.4f} mean {float(dy.mean()):.5f}")
        print(msg)
        assert float(d.max()) <= max(0.05, 3 * float(dy.max())), msg
        assert float(d.mean()) <= max(0.005, 3 * float(dy.mean())), msg
        # the top token agrees wherever the reference's top-2 margin is clear
        top = torch.topk(a, 2, dim=-1)
        clear = (top.values[:, 0] - top.values[:, 1]) > 4 * float(dy.max()) + 0.02
        assert torch.equal(a.argmax(-1)[clear], b.argmax(-1)[clear])
    # the pool: same blocks, the appended K/V rows within the same noise
    assert c_ref._block_tables == c_got._block_tables
    d = (c_ref.buf.float() - c_got.buf.float()).abs()
    dy = (c_ref.buf.float() - c_alt.buf.float()).abs()
    live = (c_ref.buf != 0) | (c_got.buf != 0)
    assert float(d.max()) <= max(0.05, 3 * float(dy.max()))
    assert float(d[live].mean()) <= max(1e-3, 3 * float(dy[live].mean()))
    used = {x for t in c_got._block_tables.values() for x in t}
    unused = [x for x in range(c_got.num_blocks) if x not in used]
    view = c_got.buf.view(c_got.buf.shape[0], 2, c_got.num_blocks, 16, -1)
    assert int(view[:, :, unused].count_nonzero()) == 0


def test_decode_layers_in_a_graph_with_inactive_rows(cuda, model):
    """The persistent launch captured in a CUDA graph (DecodeGraphs), the
    step padded with inactive rows (start -1: nothing appended, outputs
    unread), against the same launch run eagerly on the live rows only: the
    padding must change nothing.  A row's GEMM sums never depend on the other
    rows, and these rows are short enough (<= 9 blocks) that the attention
    splits them into the same two partitions at 5 and at 8 rows."""
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 151936, (n,), generator=g).tolist() for n in (40, 7, 133, 64, 2)]
    ref, c_ref = _run(model, cuda, prompts, 4, persistent=True)
    got, c_got = _run(model, cuda, prompts, 4, persistent=True, graphs=True)
    # same kernel, same rows: the padded graph replay is bit-identical
    for a, b in zip(ref, got):
        assert torch.equal(a, b)
    assert torch.equal(c_ref.buf, c_got.buf)
    used = {x for t in c_got._block_tables.values() for x in t}
    unused = [x for x in range(c_got.num_blocks) if x not in used]
    view = c_got.buf.view(c_got.buf.shape[0], 2, c_got.num_blocks, 16, -1)
    assert int(view[:, :, unused].count_nonzero()) == 0


def test_decode_layers_rejects_bad_arguments(cuda, model):
    import ctypes

    import pagedkv

    L = pagedkv.lib()
    z = torch.zeros(4, 1536, dtype=torch.bfloat16, device=cuda)
    tab = model._layer_table()
    ws = pagedkv.decode_layers_workspace(cuda)
    arr = ctypes.cast(tab.arr, ctypes.c_void_p)
    zp = z.data_ptr()
    st = L.pkv_decode_layers(arr, 0, zp, zp, zp, 4, None, 0, None, 0, None, None, None, None, 0,
                             1e-6, ws.data_ptr(), ws.numel(), None, None)
    assert st != 0  # no layers
    st = L.pkv_decode_layers(arr, len(tab), zp, zp, zp, 33, None, 0, None, 0, None, None, None,
                             None, 0, 1e-6, ws.data_ptr(), ws.numel(), None, None)
    assert st != 0  # more rows than the kernel takes
    assert L.pkv_decode_layers_workspace_size(0) == 0
    assert L.pkv_decode_layers_workspace_size(33) == 0
