"""Qwen2.5-1.5B with its attention call sites moved onto the paged-KV kernels
(drop-in for the reference's model.py:1-207).

Unchanged from the reference (consumed as-is, cuBLAS/torch): embeddings,
RMSNorm in fp32 (model.py:43-55), q/k/v/o projections with bias
(model.py:81-84), SwiGLU MLP (model.py:112-120), residual blocks
(model.py:123-138), last-position logits through the tied embedding
(model.py:204-206).

Changed (the hot path):
  * RoPE cos/sin come from a table built once, on the CPU, with exactly the
    reference's fp32 formula (model.py:148-155) and rounded to the
    activation dtype; the fused append kernel indexes it by position.
  * apply_rope + cache.write + cache.read + FA2 (model.py:92-103) become
    cache.append (RoPE on q and k, K/V into their blocks) and one paged
    attention launch that reads the blocks in place (kernels/fa2.py).
  * No mask or SDPA branch: there is no CPU fallback (model.py:102-107).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

# Qwen2.5-1.5B architecture constants (model.py:18-27)
HIDDEN_SIZE = 1536
NUM_LAYERS = 28
NUM_HEADS = 12
NUM_KV_HEADS = 2
N_REP = NUM_HEADS // NUM_KV_HEADS
HEAD_DIM = HIDDEN_SIZE // NUM_HEADS
INTERMEDIATE_SIZE = 8960
VOCAB_SIZE = 151936
RMS_NORM_EPS = 1e-6
ROPE_THETA = 1_000_000.0


class RMSNorm(torch.nn.Module):
    def __init__(self, dim, eps):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        input_dtype = x.dtype
        x = x.to(torch.float32)
        variance = x.pow(2).mean(-1, keepdim=True)
        x = x * torch.rsqrt(variance + self.eps)
        return self.weight * x.to(input_dtype)


def rotate_half(x):
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def apply_rope(q, k, cos, sin):
    """Unfused RoPE with the reference's op sequence (model.py:62-65); the
    engine uses the fused append kernel instead."""
    q = (q * cos) + (rotate_half(q) * sin)
    k = (k * cos) + (rotate_half(k) * sin)
    return q, k


def repeat_kv(x):
    if N_REP == 1:
        return x
    b, h, s, d = x.shape
    return x[:, :, None, :, :].expand(b, h, N_REP, s, d).reshape(b, h * N_REP, s, d)


def rope_table(num_positions, dtype, device):
    """cos/sin [num_positions, HEAD_DIM] for positions 0..num_positions-1,
    computed on the CPU exactly as rope_cos_sin (model.py:148-155) does:
    fp32 inv_freq, fp32 position * inv_freq, cat(freqs, freqs), cos/sin in
    fp32, then a cast to the activation dtype."""
    inv_freq = 1.0 / (ROPE_THETA ** (torch.arange(0, HEAD_DIM, 2).float() / HEAD_DIM))
    pos = torch.arange(num_positions, dtype=torch.int64).to(torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype).to(device), emb.sin().to(dtype).to(device)


class QwenAttention(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.q_proj = torch.nn.Linear(HIDDEN_SIZE, NUM_HEADS * HEAD_DIM, bias=True)
        self.k_proj = torch.nn.Linear(HIDDEN_SIZE, NUM_KV_HEADS * HEAD_DIM, bias=True)
        self.v_proj = torch.nn.Linear(HIDDEN_SIZE, NUM_KV_HEADS * HEAD_DIM, bias=True)
        self.o_proj = torch.nn.Linear(NUM_HEADS * HEAD_DIM, HIDDEN_SIZE, bias=False)

    def forward(self, x, cos, sin, mask, is_causal, kv_lens, cache, layer_idx, slot_mapping, gather_idx):
        from kernels.fa2 import flash_attention

        B, T, _ = x.shape
        if hasattr(self, "qkv_weight"):  # one GEMM over the merged q/k/v weights
            qkv = F.linear(x, self.qkv_weight, self.qkv_bias).view(B, T, NUM_HEADS + 2 * NUM_KV_HEADS, HEAD_DIM)
            q = qkv[:, :, :NUM_HEADS].transpose(1, 2)
            k = qkv[:, :, NUM_HEADS:NUM_HEADS + NUM_KV_HEADS].transpose(1, 2)
            v = qkv[:, :, NUM_HEADS + NUM_KV_HEADS:].transpose(1, 2)
        else:
            q = self.q_proj(x).view(B, T, NUM_HEADS, HEAD_DIM).transpose(1, 2)
            k = self.k_proj(x).view(B, T, NUM_KV_HEADS, HEAD_DIM).transpose(1, 2)
            v = self.v_proj(x).view(B, T, NUM_KV_HEADS, HEAD_DIM).transpose(1, 2)

        # RoPE on q and k + K/V into their pool blocks, one launch
        q_rot = torch.empty(B, T, NUM_HEADS, HEAD_DIM, device=x.device, dtype=x.dtype)
        cache.append(layer_idx, slot_mapping, q, k, v, cos, sin, q_rot.transpose(1, 2))
        k_blocks, v_blocks = cache.read(layer_idx, gather_idx)

        # paged attention straight from the blocks; O lands in [B, T, H, D]
        out = torch.empty(B, T, NUM_HEADS, HEAD_DIM, device=x.device, dtype=x.dtype)
        flash_attention(q_rot.transpose(1, 2), k_blocks, v_blocks, is_causal, kv_lens,
                        out=out.transpose(1, 2))
        return self.o_proj(out.view(B, T, NUM_HEADS * HEAD_DIM))


class QwenMLP(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.gate_proj = torch.nn.Linear(HIDDEN_SIZE, INTERMEDIATE_SIZE, bias=False)
        self.up_proj = torch.nn.Linear(HIDDEN_SIZE, INTERMEDIATE_SIZE, bias=False)
        self.down_proj = torch.nn.Linear(INTERMEDIATE_SIZE, HIDDEN_SIZE, bias=False)

    def forward(self, x):
        if hasattr(self, "gate_up_weight"):  # one GEMM + the fused SwiGLU kernel
            import pagedkv

            shp = x.shape
            gu = F.linear(x.reshape(-1, shp[-1]), self.gate_up_weight)
            return self.down_proj(pagedkv.silu_mul(gu)).view(*shp[:-1], HIDDEN_SIZE)
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class QwenBlock(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.input_layernorm = RMSNorm(HIDDEN_SIZE, RMS_NORM_EPS)
        self.self_attn = QwenAttention()
        self.post_attention_layernorm = RMSNorm(HIDDEN_SIZE, RMS_NORM_EPS)
        self.mlp = QwenMLP()

    def forward(self, x, cos, sin, mask, is_causal, kv_lens, cache, layer_idx, slot_mapping, gather_idx):
        attention_output = self.self_attn(
            self.input_layernorm(x), cos, sin, mask, is_causal, kv_lens,
            cache, layer_idx, slot_mapping, gather_idx,
        )
        x = x + attention_output
        x = x + self.mlp(self.post_attention_layernorm(x))
        return x


class Qwen2ForCausalLM(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.embed_tokens = torch.nn.Embedding(VOCAB_SIZE, HIDDEN_SIZE)
        self.layers = torch.nn.ModuleList(QwenBlock() for _ in range(NUM_LAYERS))
        self.norm = RMSNorm(HIDDEN_SIZE, RMS_NORM_EPS)

        inv_freq = 1.0 / (ROPE_THETA ** (torch.arange(0, HEAD_DIM, 2).float() / HEAD_DIM))
        self.register_buffer("inv_freq", inv_freq, persistent=False)
        self._rope = {}  # (device, dtype) -> (cos, sin) tables
        self._rope_retired = []  # outgrown tables stay alive: captured graphs may point at them
        self._graphs = {}  # id(cache) -> DecodeGraphs
        self._prefill_graphs = {}  # id(cache) -> PrefillGraphs
        self._mixed_graphs = {}  # id(cache) -> MixedGraphs

    def rope_tables(self, num_positions, dtype, device):
        key = (str(device), dtype)
        tab = self._rope.get(key)
        if tab is None or tab[0].shape[0] < num_positions:
            if tab is not None:
                self._rope_retired.append(tab)
            n = max(num_positions, 2 * (tab[0].shape[0] if tab is not None else 0), 4096)
            tab = rope_table(n, dtype, device)
            self._rope[key] = tab
        return tab

    def forward(self, input_ids, cache, seqs):
        """input_ids: [B, T]. cache: a KVCache. seqs: that cache's sequence id for
        each batch item.  Returns logits for each row's last position: [B, 1, vocab].

        A T == 1 step for which decode graphs were enabled (enable_decode_graphs)
        replays a captured CUDA graph; everything else runs eagerly."""
        _, T = input_ids.shape
        if T == 1:
            runner = self._graphs.get(id(cache))
            if runner is not None and runner.covers(len(seqs)):
                return runner.run(input_ids, seqs)[:, None]
        else:
            runner = self._prefill_graphs.get(id(cache))
            if runner is not None and runner.covers(len(seqs), T):
                return runner.run(input_ids, seqs)[:, None]
        if input_ids.device != cache.device:
            input_ids = input_ids.to(cache.device, non_blocking=True)
        starts_list, slot_mapping, gather_idx = cache.prepare(seqs, T)
        logits = self.forward_step(input_ids, cache, gather_idx)
        cache.advance(seqs, T)
        return logits

    def forward_step(self, input_ids, cache, step):
        """Device-only part of forward(): embeddings, 28 layers over the step's
        device tables, last-position logits.  No host synchronisation, so it can
        be captured in a CUDA graph for a fixed batch."""
        B, T = input_ids.shape
        x = self.embed_tokens(input_ids)
        cos, sin = self.rope_tables(cache.table_pitch * cache.block_size, x.dtype, x.device)
        kv_lens = step.kv_lens
        is_causal = T > 1  # a single query row sees every key up to kv_lens anyway
        if not self.fused:
            for layer_idx, layer in enumerate(self.layers):
                x = layer(x, cos, sin, None, is_causal, kv_lens, cache, layer_idx, step, step)
            if step.q_lens is not None:  # right-padded rows: their last real token
                x = x[torch.arange(B, device=x.device), step.q_lens.long() - 1][:, None]
            else:
                x = x[:, -1:]
            x = self.norm(x)
            return x @ self.embed_tokens.weight.T
        # fused: residual add + RMSNorm in one kernel, the residual stream x
        # updated in place; same op order as QwenBlock.forward (model.py:131-138)
        import pagedkv

        N = B * T
        xs = x.view(N, HIDDEN_SIZE)
        h = pagedkv.add_rmsnorm(xs, None, self.layers[0].input_layernorm.weight, RMS_NORM_EPS)
        m = self._fused_layers(h, xs, B, T, cos, sin, is_causal, kv_lens, cache, step)
        # last position only (model.py:204-206): x + mlp, then the final norm
        if step.q_lens is not None:  # right-padded rows: their last real token
            rows = torch.arange(B, device=x.device)
            last = step.q_lens.long() - 1
            m_last = m.view(B, T, HIDDEN_SIZE)[rows, last]
            x_last = x.view(B, T, HIDDEN_SIZE)[rows, last]
        else:
            m_last = m.view(B, T, HIDDEN_SIZE)[:, T - 1]
            x_last = x.view(B, T, HIDDEN_SIZE)[:, T - 1]
        h = pagedkv.add_rmsnorm(m_last, x_last, self.norm.weight, RMS_NORM_EPS)
        return (h @ self.embed_tokens.weight.T)[:, None]

    def _fused_layers(self, h, xs, B, T, cos, sin, is_causal, kv_lens, cache, step, segs=None):
        """The 28 layers on the merged weights, same op order and bf16 rounding
        points as QwenBlock.forward (model.py:131-138): q/k/v GEMM + bias ->
        RoPE + K/V append -> paged attention -> o_proj -> residual add + RMSNorm
        -> gate/up GEMM -> SwiGLU -> down_proj -> residual add + the next
        layer's RMSNorm.  h: the first layer's normed input [N, 1536]; xs: the
        residual stream, updated in place.  Each projection runs as a skinny
        tensor-core GEMM fused with the op after it when the step has at most
        skinny_rows[op] rows (where it beats cuBLAS), else as cuBLAS + the
        separate fused kernel.  Returns the last layer's MLP output (before its
        residual add).

        segs: row segments [(first row, B, T, PagedStep, causal)] that share
        the GEMMs but append and attend separately (a mixed prefill + decode
        step); default one segment (0, B, T, step, is_causal)."""
        import pagedkv
        from kernels.fa2 import flash_attention

        N = xs.shape[0]
        if segs is None:
            segs = [(0, B, T, step, is_causal)]
        if (self.persistent_decode and len(segs) == 1 and segs[0][2] == 1
                and 0 < N <= pagedkv.LAYERS_MAX_ROWS and not cache.fp8
                and segs[0][3].q_lens is None and len(self.layers) <= pagedkv.LAYERS_MAX_LAYERS):
            # a small decode step: every layer in one persistent launch
            st = segs[0][3]
            m = torch.empty_like(xs)
            return pagedkv.decode_layers(self._layer_table(), h, xs, m, cache.buf,
                                         cache.block_tables, st.rows, st.starts, cos, sin,
                                         RMS_NORM_EPS, err=cache.err_flag)
        use = {op: self.skinny_linears and N <= lim for op, lim in self.skinny_rows.items()}
        # the q/k/v GEMM's fused RoPE + append epilogue writes the bf16 pool;
        # an FP8 pool takes the separate quantising append
        fused_qkv = use["qkv"] and len(segs) == 1 and not cache.fp8
        err = cache.err_flag
        m = None
        last = len(self.layers) - 1
        for li, layer in enumerate(self.layers):
            at, mlp = layer.self_attn, layer.mlp
            q_rot = torch.empty(N, NUM_HEADS, HEAD_DIM, device=xs.device, dtype=xs.dtype)
            if fused_qkv:
                pagedkv.linear_rope_append(
                    h, at.qkv_weight, at.qkv_bias, cos, sin,
                    q_rot.view(B, T, NUM_HEADS, HEAD_DIM).transpose(1, 2), cache.buf[li, 0],
                    cache.buf[li, 1], cache.block_tables, step.rows, step.starts, NUM_KV_HEADS,
                    err=err, q_lens=step.q_lens)
            else:
                qkv = (pagedkv.linear(h, at.qkv_weight, at.qkv_bias, err=err) if use["qkv"]
                       else F.linear(h, at.qkv_weight, at.qkv_bias))
                qkv = qkv.view(N, NUM_HEADS + 2 * NUM_KV_HEADS, HEAD_DIM)
                for r0, Bs, Ts, st, _ in segs:
                    part = qkv[r0:r0 + Bs * Ts].view(Bs, Ts, NUM_HEADS + 2 * NUM_KV_HEADS, HEAD_DIM)
                    cache.append(li, st, part[:, :, :NUM_HEADS].transpose(1, 2),
                                 part[:, :, NUM_HEADS:NUM_HEADS + NUM_KV_HEADS].transpose(1, 2),
                                 part[:, :, NUM_HEADS + NUM_KV_HEADS:].transpose(1, 2), cos, sin,
                                 q_rot[r0:r0 + Bs * Ts].view(Bs, Ts, NUM_HEADS, HEAD_DIM)
                                 .transpose(1, 2))
            out = torch.empty(N, NUM_HEADS, HEAD_DIM, device=xs.device, dtype=xs.dtype)
            for r0, Bs, Ts, st, causal in segs:
                k_blocks, v_blocks = cache.read(li, st)
                qs = q_rot[r0:r0 + Bs * Ts].view(Bs, Ts, NUM_HEADS, HEAD_DIM).transpose(1, 2)
                os_ = out[r0:r0 + Bs * Ts].view(Bs, Ts, NUM_HEADS, HEAD_DIM).transpose(1, 2)
                flash_attention(qs, k_blocks, v_blocks, causal, st.kv_lens, out=os_)
            o_in = out.view(N, NUM_HEADS * HEAD_DIM)
            post_w = layer.post_attention_layernorm.weight
            if use["o"]:
                h = pagedkv.linear_add_rmsnorm(o_in, at.o_proj.weight, xs, post_w, RMS_NORM_EPS,
                                               resid_out=xs, err=err)
            else:
                h = pagedkv.add_rmsnorm(F.linear(o_in, at.o_proj.weight), xs, post_w, RMS_NORM_EPS,
                                        resid_out=xs)
            if use["gate_up"]:  # SwiGLU in the GEMM's epilogue (paired gate/up rows)
                act = pagedkv.linear_silu_mul(h, self._paired_gate_up(mlp), err=err)
            else:
                act = pagedkv.silu_mul(F.linear(h, mlp.gate_up_weight))
            if li < last:
                nxt = self.layers[li + 1]
                norm_w = nxt.input_layernorm.weight
                if use["down"]:
                    h = pagedkv.linear_add_rmsnorm(act, mlp.down_proj.weight, xs, norm_w,
                                                   RMS_NORM_EPS, resid_out=xs, err=err)
                else:
                    h = pagedkv.add_rmsnorm(F.linear(act, mlp.down_proj.weight), xs, norm_w,
                                            RMS_NORM_EPS, resid_out=xs)
            elif use["down"]:
                m = pagedkv.linear(act, mlp.down_proj.weight, err=err)
            else:
                m = F.linear(act, mlp.down_proj.weight)
        return m

    def forward_mixed_step(self, ids, step_p, step_d, Tp, Bp, cache):
        """Device-only mixed step (no host synchronisation, capturable): ids
        [Tp + Bp] int32 = the prompt's Tp (right-padded, step_p.q_lens real)
        tokens then the Bp decode rows' tokens (rows with start -1 inactive).
        Returns logits [1 + Bp, vocab]: the prompt's last real token, then
        each decode row."""
        import pagedkv

        x = self.embed_tokens(ids.long())
        cos, sin = self.rope_tables(cache.table_pitch * cache.block_size, x.dtype, x.device)
        xs = x.view(Tp + Bp, HIDDEN_SIZE)
        h = pagedkv.add_rmsnorm(xs, None, self.layers[0].input_layernorm.weight, RMS_NORM_EPS)
        segs = [(0, 1, Tp, step_p, True), (Tp, Bp, 1, step_d, False)]
        m = self._fused_layers(h, xs, 0, 0, cos, sin, None, None, cache, None, segs=segs)
        last = torch.cat([step_p.q_lens.long() - 1,
                          torch.arange(Tp, Tp + Bp, device=x.device)])
        hl = pagedkv.add_rmsnorm(m[last], xs[last], self.norm.weight, RMS_NORM_EPS)
        return hl @ self.embed_tokens.weight.T

    def forward_mixed(self, prefill_ids, prefill_seq, decode_ids, decode_seqs, cache):
        """One forward over a prompt and a batch of decode rows (a mixed
        prefill + decode step): prefill_ids [1, T] for sequence prefill_seq,
        decode_ids [B, 1] for decode_seqs.  The projections, norms and SwiGLU
        run once over all T + B rows (one pass over the weights); RoPE + K/V
        append and attention run per part (the causal prefill kernel for the
        prompt, the decode kernel for the rest).  Returns logits
        [1 + B, vocab]: the prompt's last token, then each decode row.
        Replays a captured graph when enable_mixed_graphs covers (T, B), else
        runs eagerly.  Needs the fused weights (fuse_weights_)."""
        import pagedkv

        runner = self._mixed_graphs.get(id(cache))
        if runner is not None and runner.covers(prefill_ids.shape[1], len(decode_seqs)):
            return runner.run(prefill_ids, prefill_seq, decode_ids, decode_seqs)
        self.fuse_weights_()
        dev = cache.device
        T, B = prefill_ids.shape[1], len(decode_seqs)
        _, step_p, _ = cache.prepare([prefill_seq], T)
        _, step_d, _ = cache.prepare(decode_seqs, 1)
        ids = torch.cat([prefill_ids.reshape(-1), decode_ids.reshape(-1)]).to(dev, non_blocking=True)
        x = self.embed_tokens(ids)
        cos, sin = self.rope_tables(cache.table_pitch * cache.block_size, x.dtype, dev)
        xs = x.view(T + B, HIDDEN_SIZE)
        h = pagedkv.add_rmsnorm(xs, None, self.layers[0].input_layernorm.weight, RMS_NORM_EPS)
        segs = [(0, 1, T, step_p, True), (T, B, 1, step_d, False)]
        m = self._fused_layers(h, xs, 0, 0, cos, sin, None, None, cache, None, segs=segs)
        last = torch.cat([torch.tensor([T - 1]), torch.arange(T, T + B)]).to(dev, non_blocking=True)
        hl = pagedkv.add_rmsnorm(m[last], xs[last], self.norm.weight, RMS_NORM_EPS)
        cache.advance([prefill_seq], T)
        cache.advance(decode_seqs, 1)
        return hl @ self.embed_tokens.weight.T

    @staticmethod
    def _paired_gate_up(mlp):
        """The merged gate/up weight in the PKV_W_GATE_UP_PAIRED layout, made
        on first use on the weight's device and kept (55 MB per layer; not part
        of the state dict).  refresh_packed_weights() drops it after the
        weights change."""
        pw = getattr(mlp, "_gate_up_paired", None)
        if pw is None:
            import pagedkv

            pw = pagedkv.PairedGateUp(mlp.gate_up_weight)
            mlp._gate_up_paired = pw
        return pw

    def refresh_packed_weights(self):
        for layer in self.layers:
            layer.mlp.__dict__.pop("_gate_up_paired", None)
        self.__dict__.pop("_layers_table", None)

    def _layer_table(self):
        """The per-layer weight table of pagedkv.decode_layers (merged q/k/v,
        the paired gate/up copy), made on first use and kept."""
        tab = self.__dict__.get("_layers_table")
        if tab is None:
            import pagedkv

            ents = []
            for layer in self.layers:
                at, mlp = layer.self_attn, layer.mlp
                ents.append({"qkv_w": at.qkv_weight, "qkv_b": at.qkv_bias,
                             "o_w": at.o_proj.weight,
                             "post_norm_w": layer.post_attention_layernorm.weight,
                             "gate_up_w": self._paired_gate_up(mlp).data,
                             "down_w": mlp.down_proj.weight,
                             "in_norm_w": layer.input_layernorm.weight})
            tab = self.__dict__["_layers_table"] = pagedkv.LayerTable(ents)
        return tab

    @property
    def fused(self):
        return getattr(self, "_fused", False)

    # Fused path: a projection of a step with at most skinny_rows[op] rows
    # runs as the skinny tensor-core GEMM (pkv_linear*), larger ones on
    # cuBLAS; the limits are where the skinny GEMM stops beating cuBLAS on a
    # B200 (measured per projection, CUDA-graph replay).
    skinny_linears = True
    skinny_rows = {"qkv": 32, "o": 32, "gate_up": 32, "down": 128}
    # A decode step (one token per row) of at most pagedkv.LAYERS_MAX_ROWS
    # rows on a bf16 pool runs all layers as one persistent launch
    # (pkv_decode_layers) instead of the per-op kernels.
    persistent_decode = False

    def fuse_weights_(self):
        """Merge q/k/v (weights + biases) and gate/up weights into single
        tensors so each needs one GEMM; the original parameters become views
        of the merged tensors (no extra memory, state_dict unchanged).  Also
        switches forward to the fused residual-add + RMSNorm kernels."""
        if self.fused:
            return self
        with torch.no_grad():
            for layer in self.layers:
                at, mlp = layer.self_attn, layer.mlp
                w = torch.cat([at.q_proj.weight, at.k_proj.weight, at.v_proj.weight]).contiguous()
                b = torch.cat([at.q_proj.bias, at.k_proj.bias, at.v_proj.bias]).contiguous()
                nq, nk = at.q_proj.weight.shape[0], at.k_proj.weight.shape[0]
                at.q_proj.weight = nn.Parameter(w[:nq], requires_grad=False)
                at.k_proj.weight = nn.Parameter(w[nq:nq + nk], requires_grad=False)
                at.v_proj.weight = nn.Parameter(w[nq + nk:], requires_grad=False)
                at.q_proj.bias = nn.Parameter(b[:nq], requires_grad=False)
                at.k_proj.bias = nn.Parameter(b[nq:nq + nk], requires_grad=False)
                at.v_proj.bias = nn.Parameter(b[nq + nk:], requires_grad=False)
                at.register_buffer("qkv_weight", w, persistent=False)
                at.register_buffer("qkv_bias", b, persistent=False)
                gu = torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight]).contiguous()
                ni = mlp.gate_proj.weight.shape[0]
                mlp.gate_proj.weight = nn.Parameter(gu[:ni], requires_grad=False)
                mlp.up_proj.weight = nn.Parameter(gu[ni:], requires_grad=False)
                mlp.register_buffer("gate_up_weight", gu, persistent=False)
        self._fused = True
        return self

    # ---- CUDA-graph decode ----
    def enable_decode_graphs(self, cache, max_batch=256):
        """Capture the T == 1 forward per batch bucket (lazily, on first use).
        Merges the projection weights first (fuse_weights_)."""
        self.fuse_weights_()
        self._graphs[id(cache)] = DecodeGraphs(self, cache, max_batch)
        return self._graphs[id(cache)]

    def enable_mixed_graphs(self, cache, max_len=4096, max_batch=256):
        """Capture mixed prefill + decode steps (forward_mixed) per (padded
        prompt length, padded decode batch) bucket, lazily on first use or
        ahead of time with MixedGraphs.capture."""
        self.fuse_weights_()
        self._mixed_graphs[id(cache)] = MixedGraphs(self, cache, max_len, max_batch)
        return self._mixed_graphs[id(cache)]

    def enable_prefill_graphs(self, cache, max_len=4096):
        """Capture one-row prefills (chat.py admits one message per tick) per
        padded length bucket, lazily on first use."""
        self.fuse_weights_()
        self._prefill_graphs[id(cache)] = PrefillGraphs(self, cache, max_len)
        return self._prefill_graphs[id(cache)]


def _prefill_buckets(top):
    """Padded prompt lengths: 64, 128, 256, then every 128 tokens up to top
    (above 256 tokens a prompt pads by < 128 tokens, under a third of its
    bucket)."""
    out, b = [], 64
    while b < top:
        out.append(b)
        b = b * 2 if b < 256 else b + 128
    out.append(top)
    return out


def _pinned_free(events, key):
    """Wait until the last copy out of bucket `key`'s pinned input buffer has
    run, so the host can refill it.  Without a sampling sync between two
    steps (two prompts admitted in one scheduler tick, or back-to-back
    calls) the host runs ahead of the stream; usually the copy is long done
    and this returns at once."""
    ev = events.get(key)
    if ev is not None:
        ev.synchronize()


def _pinned_used(events, key):
    """Mark the copies just enqueued out of bucket `key`'s pinned buffer."""
    ev = events.get(key)
    if ev is None:
        ev = events[key] = torch.cuda.Event()
    ev.record()


def _buckets(max_batch):
    b, out = 1, []
    while b < max_batch:
        out.append(b)
        b = b * 2 if b < 16 else b + 16
    out.append(max_batch)
    return out


class DecodeGraphs:
    """CUDA graphs of the batched one-token forward, one per batch bucket.

    Graph inputs are four int32 device vectors per bucket (token id, table
    row, start, kv_len); a step fills them with ONE host-to-device copy from
    pinned memory and replays the graph, so a decode step costs one copy, one
    replay and the sampling that follows (chat.py:_process) instead of ~600
    eager launches.  Rows beyond the live batch are inactive padding (start
    -1, kv_len 0): the append kernel skips them and attention writes NaN for
    them, which the caller never reads.  The decode kernels are captured with
    max_kv_len = the cache's per-sequence capacity; partitions past a row's
    length exit at once.
    """

    def __init__(self, model, cache, max_batch):
        self.model, self.cache = model, cache
        self.max_batch = min(max_batch, cache.max_seqs)
        self.buckets = _buckets(self.max_batch)
        self.graphs = {}
        self.pool = torch.cuda.graph_pool_handle()
        self.capacity = cache.table_pitch * cache.block_size
        self._copied = {}  # bucket -> event after the last copy out of its pinned inputs

    def covers(self, B):
        return 0 < B <= self.max_batch

    def _bucket(self, B):
        return next(b for b in self.buckets if b >= B)

    def _capture(self, Bp):
        from kv_cache import PagedStep

        dev = self.cache.device
        ins = torch.zeros(4, Bp, dtype=torch.int32, device=dev)
        ins[2].fill_(-1)
        step = PagedStep(self.cache, 1, [0] * Bp, ins[1], ins[2], ins[3], self.capacity)
        host = torch.empty(4, Bp, dtype=torch.int32, pin_memory=True)
        # warm up on a side stream (lazy library / workspace set-up happens here)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.model.forward_step(ins[0].view(Bp, 1).long(), self.cache, step)
        torch.cuda.current_stream(dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.pool):
            logits = self.model.forward_step(ins[0].view(Bp, 1).long(), self.cache, step)
        self.graphs[Bp] = (g, ins, host, logits)
        return self.graphs[Bp]

    def run(self, input_ids, seqs):
        B = len(seqs)
        Bp = self._bucket(B)
        g, ins, host, logits = self.graphs.get(Bp) or self._capture(Bp)
        starts, rows = self.cache.step_rows(seqs, 1)
        self.cache.flush_tables()
        _pinned_free(self._copied, Bp)
        h = host.numpy()  # the pinned buffer, filled in place (no per-row torch ops)
        if not input_ids.is_cuda:
            h[0, :B] = input_ids.view(-1).numpy()
        h[1, :B] = rows
        h[2, :B] = starts
        np.add(h[2, :B], 1, out=h[3, :B])
        if Bp > B:
            h[0, B:] = 0
            h[1, B:] = 0
            h[2, B:] = -1
            h[3, B:] = 0
        ins.copy_(host, non_blocking=True)
        _pinned_used(self._copied, Bp)
        if input_ids.is_cuda:  # device ids: a device-side copy, no host sync
            ins[0, :B].copy_(input_ids.view(-1))
        g.replay()
        self.cache.advance(seqs, 1)
        return logits[:B, 0]


class PrefillGraphs:
    """CUDA graphs of a one-row prefill, one per padded length bucket
    (64, 128, 256, then every 128 tokens).

    A prompt of T tokens replays the graph of the smallest bucket Tp >= T:
    the token ids are right-padded, and the step's q_lens (= T) makes the
    append kernel store only the real tokens and the prefill kernel attend
    (and write) only the real queries; the logits come from token T-1.  The
    padded tail costs some GEMM work but removes the per-layer Python launch
    overhead and the per-length GEMM heuristics of an eager prefill.
    """

    def __init__(self, model, cache, max_len):
        self.model, self.cache = model, cache
        self.capacity = cache.table_pitch * cache.block_size
        self.buckets = _prefill_buckets(min(max_len, self.capacity))
        self.graphs = {}
        self.pool = torch.cuda.graph_pool_handle()
        self._copied = {}  # bucket -> event after the last copy out of its pinned inputs

    def covers(self, B, T):
        return B == 1 and 1 < T <= self.buckets[-1]

    def _capture(self, Tp):
        from kv_cache import PagedStep

        dev = self.cache.device
        ids = torch.zeros(1, Tp, dtype=torch.int32, device=dev)
        meta = torch.zeros(4, 1, dtype=torch.int32, device=dev)  # row, start, kv_len, q_len
        meta[1].fill_(-1)  # inactive until a real prompt is copied in
        step = PagedStep(self.cache, Tp, [0], meta[0], meta[1], meta[2], self.capacity,
                         q_lens=meta[3])
        host = torch.zeros(4 + Tp, dtype=torch.int32, pin_memory=True)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.model.forward_step(ids.long(), self.cache, step)
        torch.cuda.current_stream(dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.pool):
            logits = self.model.forward_step(ids.long(), self.cache, step)
        self.graphs[Tp] = (g, ids, meta, host, logits)
        return self.graphs[Tp]

    def run(self, input_ids, seqs):
        T = input_ids.shape[1]
        Tp = next(b for b in self.buckets if b >= T)
        g, ids, meta, host, logits = self.graphs.get(Tp) or self._capture(Tp)
        starts, rows = self.cache.step_rows(seqs, T)
        self.cache.flush_tables()
        _pinned_free(self._copied, Tp)
        h = host.numpy()
        h[:4] = (rows[0], starts[0], starts[0] + T, T)
        if not input_ids.is_cuda:
            h[4:4 + T] = input_ids.view(-1).numpy()
        meta.view(-1).copy_(host[:4], non_blocking=True)
        if input_ids.is_cuda:
            ids[0, :T].copy_(input_ids.view(-1))
        else:
            ids.view(-1).copy_(host[4:4 + Tp], non_blocking=True)
        _pinned_used(self._copied, Tp)
        g.replay()
        self.cache.advance(seqs, T)
        return logits[:, 0]


class MixedGraphs:
    """CUDA graphs of the mixed prefill + decode step (forward_mixed), one per
    (padded prompt length Tp, padded decode batch Bp) bucket: Tp as
    PrefillGraphs (the prompt right-padded, its q_len making the append and
    the prefill kernel skip the padding), Bp in 16, 32, 64, 128, 256 (padded
    decode rows inactive, start -1).  One pinned host buffer per bucket holds
    the step's ids and both segments' (row, start, kv_len) and goes over in
    one copy; the graph then runs the whole step -- ~600 eager launches --
    as one replay.  Both segments' attention grids are planned for the
    cache's per-sequence capacity, as the other graph runners do."""

    def __init__(self, model, cache, max_len, max_batch):
        self.model, self.cache = model, cache
        self.capacity = cache.table_pitch * cache.block_size
        self.t_buckets = _prefill_buckets(min(max_len, self.capacity))
        mb = min(max_batch, cache.max_seqs)
        self.b_buckets = [b for b in (16, 32, 64, 128, 256) if b < mb] + [mb]
        self.graphs = {}
        self.pool = torch.cuda.graph_pool_handle()
        self._copied = {}

    def covers(self, T, B):
        return 1 < T <= self.t_buckets[-1] and 0 < B <= self.b_buckets[-1]

    def buckets(self, T, B):
        return (next(t for t in self.t_buckets if t >= T), next(b for b in self.b_buckets if b >= B))

    def capture(self, Tp, Bp):
        from kv_cache import PagedStep

        if (Tp, Bp) in self.graphs:
            return self.graphs[(Tp, Bp)]
        dev = self.cache.device
        # one device buffer: [ids (Tp + Bp) | prompt row, start, kv_len, q_len |
        # decode rows (Bp) | decode starts | decode kv_lens]
        n = Tp + Bp + 4 + 3 * Bp
        dev_in = torch.zeros(n, dtype=torch.int32, device=dev)
        ids = dev_in[:Tp + Bp]
        mp = dev_in[Tp + Bp:Tp + Bp + 4]
        md = dev_in[Tp + Bp + 4:].view(3, Bp)
        mp[1].fill_(-1)  # inactive until a real step is copied in
        md[1].fill_(-1)
        step_p = PagedStep(self.cache, Tp, [0], mp[0:1], mp[1:2], mp[2:3], self.capacity,
                           q_lens=mp[3:4])
        step_d = PagedStep(self.cache, 1, [0] * Bp, md[0], md[1], md[2], self.capacity)
        host = torch.zeros(n, dtype=torch.int32, pin_memory=True)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.model.forward_mixed_step(ids, step_p, step_d, Tp, Bp, self.cache)
        torch.cuda.current_stream(dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.pool):
            logits = self.model.forward_mixed_step(ids, step_p, step_d, Tp, Bp, self.cache)
        self.graphs[(Tp, Bp)] = (g, dev_in, host, logits)
        return self.graphs[(Tp, Bp)]

    def run(self, prefill_ids, prefill_seq, decode_ids, decode_seqs):
        T, B = prefill_ids.shape[1], len(decode_seqs)
        Tp, Bp = self.buckets(T, B)
        g, dev_in, host, logits = self.capture(Tp, Bp)
        sp, rp = self.cache.step_rows([prefill_seq], T)
        sd, rd = self.cache.step_rows(decode_seqs, 1)
        self.cache.flush_tables()
        _pinned_free(self._copied, (Tp, Bp))
        h = host.numpy()
        h[:Tp + Bp] = 0
        if not prefill_ids.is_cuda:
            h[:T] = prefill_ids.reshape(-1).numpy()
        if not decode_ids.is_cuda:
            h[Tp:Tp + B] = decode_ids.reshape(-1).numpy()
        o = Tp + Bp
        h[o:o + 4] = (rp[0], sp[0], sp[0] + T, T)
        md = h[o + 4:].reshape(3, Bp)
        md[0, :B] = rd
        md[1, :B] = sd
        np.add(md[1, :B], 1, out=md[2, :B])
        md[0, B:] = 0
        md[1, B:] = -1
        md[2, B:] = 0
        dev_in.copy_(host, non_blocking=True)
        _pinned_used(self._copied, (Tp, Bp))
        if prefill_ids.is_cuda:  # device ids: device-side copies, no host sync
            dev_in[:T].copy_(prefill_ids.reshape(-1))
        if decode_ids.is_cuda:
            dev_in[Tp:Tp + B].copy_(decode_ids.reshape(-1))
        g.replay()
        self.cache.advance([prefill_seq], T)
        self.cache.advance(decode_seqs, 1)
        return logits[:1 + B]
