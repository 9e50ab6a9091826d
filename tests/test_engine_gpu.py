"""The engine on the GPU: CUDA-graph decode steps give the eager forward's
logits, and chat.py's scheduler drives the real model through prefill,
batched graph decode, deferral and eviction to completion."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small_model(cuda):
    import model as M

    torch.manual_seed(0)
    m = M.Qwen2ForCausalLM().to(cuda, torch.bfloat16).eval()
    g = torch.Generator(device=cuda).manual_seed(3)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if name.endswith("layernorm.weight") or name == "norm.weight":
                p.fill_(1.0)
            else:
                p.normal_(0.0, 0.02, generator=g)
    return m


def test_decode_graph_matches_eager(cuda, small_model):
    from kv_cache import KVCache

    m = small_model.fuse_weights_()  # both arms on the engine's fused path
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 151936, (n,), generator=g).tolist() for n in (5, 40, 17)]
    caches, logits = [], []
    for use_graph in (False, True):
        c = KVCache(64, 16, cuda, torch.bfloat16)
        if use_graph:
            m.enable_decode_graphs(c, max_batch=4)
        seqs = [c.alloc() for _ in prompts]
        with torch.no_grad():
            for s, p in zip(seqs, prompts):
                m(torch.tensor([p], device=cuda), c, [s])
            out = []
            ids = [[11], [12], [13]]
            for step in range(5):
                lg = m(torch.tensor(ids), c, seqs)[:, -1].float()
                out.append(lg)
                ids = [[int(x)] for x in lg.argmax(-1).tolist()]
        torch.cuda.synchronize()
        c.check_errors()
        caches.append(c)
        logits.append(out)
    m._graphs.clear()
    for a, b in zip(*logits):
        assert float((a - b).abs().max()) < 0.05
        assert torch.equal(a.argmax(-1), b.argmax(-1))
    # the pools hold the same K/V up to split-K rounding, and the graph's
    # padding rows wrote nothing: blocks no sequence owns are still zero
    assert float((caches[0].buf.float() - caches[1].buf.float()).abs().max()) < 0.05
    c = caches[1]
    used = {b for t in c._block_tables.values() for b in t}
    unused = [b for b in range(c.num_blocks) if b not in used]
    view = c.buf.view(c.buf.shape[0], 2, c.num_blocks, 16, -1)
    assert int(view[:, :, unused].count_nonzero()) == 0


def test_graph_inputs_survive_back_to_back_calls(cuda, small_model):
    """A graph bucket's pinned input buffer is refilled on the next call; a
    CUDA event makes the host wait until the previous copy out of it has run.
    Three prompts of one prefill bucket, then two decode steps of one batch
    bucket, each issued right after the other with host-side token ids and no
    synchronisation between them, must give the eager forward's logits."""
    from kv_cache import KVCache

    m = small_model.fuse_weights_()
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 151936, (n,), generator=g).tolist() for n in (40, 50, 33)]
    results = []
    for use_graph in (False, True):
        c = KVCache(64, 16, cuda, torch.bfloat16)
        if use_graph:
            dg = m.enable_decode_graphs(c, max_batch=4)
            pg = m.enable_prefill_graphs(c, max_len=256)
        seqs = [c.alloc() for _ in prompts]
        outs = []
        with torch.no_grad():
            for s, p in zip(seqs, prompts):  # same 64-token bucket, back to back
                outs.append(m(torch.tensor([p]), c, [s])[:, -1].float().clone())
            for ids in ([[11], [12], [13]], [[21], [22], [23]]):  # same 4-row bucket
                outs.append(m(torch.tensor(ids), c, seqs)[:, -1].float().clone())
        torch.cuda.synchronize()
        c.check_errors()
        if use_graph:
            assert set(pg.graphs) == {64} and set(dg.graphs) == {4}
        results.append(outs)
    m._graphs.clear()
    m._prefill_graphs.clear()
    for a, b in zip(*results):
        assert float((a - b).abs().max()) < 0.05
        # the graph's top token is a top token of the eager logits (up to
        # GEMM rounding: a padded graph can run another cuBLAS algorithm)
        pick = a.gather(-1, b.argmax(-1, keepdim=True)).squeeze(-1)
        assert bool((pick >= a.max(-1).values - 0.05).all())


@pytest.mark.parametrize("mixed,mixed_graphs", [(None, False), (1, False), (1, True)])
def test_engine_serves_chats_with_eviction(cuda, small_model, mixed, mixed_graphs):
    """mixed=1: every prompt admitted while others decode joins their step
    (chat.MIXED_PREFILL_MIN_TOKENS, model.forward_mixed); mixed_graphs: those
    steps replay captured graphs (model.MixedGraphs)."""
    import chat
    from kv_cache import KVCache

    class Tok:
        encoder = {"<|endoftext|>": -1}

        def encode(self, text):
            if text == "\n":
                return [198]
            body = text.split("User: ", 1)[1].split("\n", 1)[0]
            return [100 + (ord(ch) * 7 + i) % 5000 for i, ch in enumerate(body)]

        def decode(self, ids):
            return "."

    m = small_model
    cache = KVCache(40, 16, cuda, torch.bfloat16)
    chat.init(kv_cache=cache, start_worker=False)
    m.enable_decode_graphs(cache, max_batch=8)
    if mixed_graphs:
        mg = m.enable_mixed_graphs(cache, max_len=256, max_batch=8)
    saved = (chat.MAX_REPLY_TOKENS, chat.STOP_SEQUENCES, chat.MIXED_PREFILL_MIN_TOKENS)
    chat.MAX_REPLY_TOKENS = 24
    chat.STOP_SEQUENCES = []
    chat.MIXED_PREFILL_MIN_TOKENS = mixed
    try:
        tok = Tok()
        chats = [chat.Chat(tok) for _ in range(6)]
        texts = ["a" * 30, "b" * 120, "c" * 60, "d" * 5, "e" * 200, "f" * 90]
        qs = [c.submit(m, t) for c, t in zip(chats, texts)]
        chat.run_until_idle()
        # second turns: the pool (640 tokens) cannot hold everyone -> LRU eviction
        qs2 = [c.submit(m, "second turn " + t[:20]) for c, t in zip(chats, texts)]
        chat.run_until_idle()
        torch.cuda.synchronize()
        cache.check_errors()
        for q in qs + qs2:
            pieces = []
            while not q.empty():
                pieces.append(q.get())
            assert pieces[-1] is None and len(pieces) == 24 + 1  # 24 tokens, then done
        for c in chats:
            assert len(c.messages) == 4
        if mixed_graphs:
            assert mg.graphs, "no mixed step replayed a graph"
    finally:
        chat.MAX_REPLY_TOKENS, chat.STOP_SEQUENCES, chat.MIXED_PREFILL_MIN_TOKENS = saved
        chat._mixed.clear()
        chat._kv_cache = None
        m._graphs.clear()
        m._mixed_graphs.clear()


@pytest.mark.parametrize("gemm", ["cublas", "skinny"])
def test_prefill_graph_matches_eager(cuda, small_model, gemm):
    """One-row prefills replayed from padded-length graphs give the eager
    prefill's logits and K/V (up to GEMM rounding), and only real tokens land
    in the pool.  A padded graph has more rows than the eager call, so the
    row-count policy could pick another GEMM for it: each run pins one GEMM
    family for both arms (cuBLAS, or the skinny GEMMs at every row count)."""
    m = small_model.fuse_weights_()
    saved = m.skinny_linears, m.skinny_rows
    m.skinny_linears = gemm == "skinny"
    m.skinny_rows = {op: 256 for op in saved[1]}
    try:
        _prefill_graph_vs_eager(cuda, m)
    finally:
        m.skinny_linears, m.skinny_rows = saved


def _prefill_graph_vs_eager(cuda, m):
    from kv_cache import KVCache

    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 151936, (n,), generator=g).tolist() for n in (70, 5, 200, 64)]
    res = []
    for use_graph in (False, True):
        c = KVCache(96, 16, cuda, torch.bfloat16)
        if use_graph:
            m.enable_prefill_graphs(c, max_len=256)
        seqs = [c.alloc() for _ in prompts]
        with torch.no_grad():
            lg = [m(torch.tensor([p], device=cuda), c, [s])[:, -1].float()
                  for s, p in zip(seqs, prompts)]
            # a decode step on top (eager) sees the same history
            lg.append(m(torch.tensor([[1], [2], [3], [4]], device=cuda), c, seqs)[:, -1].float())
        torch.cuda.synchronize()
        c.check_errors()
        res.append((lg, c))
    m._prefill_graphs.clear()
    (la, ca), (lb, cb) = res
    for a, b in zip(la, lb):
        assert float((a - b).abs().max()) < 0.05
        assert torch.equal(a.argmax(-1), b.argmax(-1))
    assert float((ca.buf.float() - cb.buf.float()).abs().max()) < 0.05
    used = {x for t in cb._block_tables.values() for x in t}
    unused = [x for x in range(cb.num_blocks) if x not in used]
    view = cb.buf.view(cb.buf.shape[0], 2, cb.num_blocks, 16, -1)
    assert int(view[:, :, unused].count_nonzero()) == 0


@pytest.mark.parametrize("gemm", ["cublas", "skinny"])
def test_mixed_forward_matches_separate_calls(cuda, small_model, gemm):
    """forward_mixed (a prompt + decode rows through shared GEMMs) gives the
    logits and K/V of a prefill call followed by a decode call, up to GEMM
    rounding (the shared GEMMs have more rows, so cuBLAS may tile them
    differently), and advances every sequence the same way."""
    from kv_cache import KVCache

    m = small_model.fuse_weights_()
    saved = m.skinny_linears, m.skinny_rows
    m.skinny_linears = gemm == "skinny"
    m.skinny_rows = {op: 256 for op in saved[1]}
    g = torch.Generator().manual_seed(4)
    hist = [torch.randint(0, 151936, (n,), generator=g).tolist() for n in (33, 7, 130)]
    prompt = torch.randint(0, 151936, (1, 90), generator=g)
    dec = torch.tensor([[5], [6], [7]])
    res = []
    try:
        for mixed in (False, True):
            c = KVCache(64, 16, cuda, torch.bfloat16)
            seqs = [c.alloc() for _ in hist]
            new = c.alloc()
            with torch.no_grad():
                for s, p in zip(seqs, hist):
                    m(torch.tensor([p], device=cuda), c, [s])
                if mixed:
                    lg = m.forward_mixed(prompt.to(cuda), new, dec.to(cuda), seqs, c).float()
                else:
                    lp = m(prompt.to(cuda), c, [new])[:, -1]
                    ld = m(dec.to(cuda), c, seqs)[:, -1]
                    lg = torch.cat([lp, ld]).float()
            torch.cuda.synchronize()
            c.check_errors()
            res.append((lg, c, [c.length(s) for s in seqs + [new]]))
    finally:
        m.skinny_linears, m.skinny_rows = saved
    (la, ca, na), (lb, cb, nb) = res
    assert na == nb == [34, 8, 131, 90]
    assert lb.shape == (4, 151936)
    # the decode rows' GEMMs run with 3 rows in one arm and 93 in the other,
    # so their split-k summation order differs; the bf16 rounding differences
    # compound over 28 layers (a few ulps of logits near 1)
    d = (la - lb).abs()
    assert float(d.max()) < 0.1 and float(d.mean()) < 0.01
    assert torch.equal(la.argmax(-1), lb.argmax(-1))
    live = (ca.buf != 0) | (cb.buf != 0)
    d = (ca.buf.float() - cb.buf.float()).abs()
    assert float(d.max()) < 0.1 and float(d[live].mean()) < 0.005
    # same block ownership, and blocks no sequence owns stay zero
    assert ca._block_tables == cb._block_tables
    used = {x for t in cb._block_tables.values() for x in t}
    unused = [x for x in range(cb.num_blocks) if x not in used]
    view = cb.buf.view(cb.buf.shape[0], 2, cb.num_blocks, 16, -1)
    assert int(view[:, :, unused].count_nonzero()) == 0


def test_mixed_graph_matches_eager(cuda, small_model):
    """Mixed steps replayed from (padded prompt, padded decode batch) graphs
    give the eager forward_mixed's logits and K/V and advance every sequence
    the same way.  Two steps of one bucket run back to back with host-side
    ids and no synchronisation between them (the bucket's pinned input is
    refilled while the first copy may still be pending); the prompt tails and
    the padded decode rows must leave the pool untouched.  Both arms run the
    skinny GEMMs (the padded graph has more rows, which could otherwise pick
    another GEMM)."""
    from kv_cache import KVCache

    m = small_model.fuse_weights_()
    saved = m.skinny_linears, m.skinny_rows
    m.skinny_linears = True
    m.skinny_rows = {op: 256 for op in saved[1]}
    g = torch.Generator().manual_seed(6)
    hist = [torch.randint(0, 151936, (n,), generator=g).tolist() for n in (33, 7, 130)]
    prompts = [torch.randint(0, 151936, (1, n), generator=g) for n in (90, 101)]
    decs = [torch.tensor([[5], [6], [7]]), torch.tensor([[8], [9], [10]])]
    res = []
    try:
        for use_graph in (False, True):
            c = KVCache(64, 16, cuda, torch.bfloat16)
            if use_graph:
                mg = m.enable_mixed_graphs(c, max_len=256, max_batch=16)
            seqs = [c.alloc() for _ in hist]
            with torch.no_grad():
                for s, p in zip(seqs, hist):
                    m(torch.tensor([p], device=cuda), c, [s])
                new = [c.alloc() for _ in prompts]
                lg = [m.forward_mixed(p, n, d, seqs, c).float().clone()
                      for p, n, d in zip(prompts, new, decs)]
            torch.cuda.synchronize()
            c.check_errors()
            if use_graph:
                assert set(mg.graphs) == {(128, 16)}
            res.append((lg, c, [c.length(s) for s in seqs + new]))
    finally:
        m.skinny_linears, m.skinny_rows = saved
        m._mixed_graphs.clear()
    (la, ca, na), (lb, cb, nb) = res
    assert na == nb == [35, 9, 132, 90, 101]
    for a, b in zip(la, lb):
        assert b.shape == (4, 151936)
        d = (a - b).abs()
        assert float(d.max()) < 0.1 and float(d.mean()) < 0.01
        assert torch.equal(a.argmax(-1), b.argmax(-1))
    live = (ca.buf != 0) | (cb.buf != 0)
    d = (ca.buf.float() - cb.buf.float()).abs()
    assert float(d.max()) < 0.1 and float(d[live].mean()) < 0.005
    assert ca._block_tables == cb._block_tables
    used = {x for t in cb._block_tables.values() for x in t}
    unused = [x for x in range(cb.num_blocks) if x not in used]
    view = cb.buf.view(cb.buf.shape[0], 2, cb.num_blocks, 16, -1)
    assert int(view[:, :, unused].count_nonzero()) == 0
