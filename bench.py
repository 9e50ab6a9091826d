#!/usr/bin/env python
"""Benchmark of the paged-KV decode attention path on B200.

Workload (one "step" = one decode token for every row through all 28 layers
of the attention path): 256 rows with contexts U[2048, 8192] (seeded), a
bf16 KV pool of ~150 GB whose blocks are handed out from a seeded random
permutation, and per layer the fused RoPE + K/V append followed by paged
decode attention over the blocks in place.  Q/K/V are synthetic N(0,1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

value  : algorithmic HBM bytes of the path per step (K+V of every visible
         token, q/k/v in, q/out, block tables) / device time, GB/s, summed
         over ranks (replicas: each GPU owns its own pool and rows).
e2e    : the same bytes over the time of the public API driven from pinned
         host buffers (q/k/v H2D and O D2H every layer inside the timed region).
--impl reference : the reference's CPU path (fp32 KVCache gather + SDPA,
         restated in oracle/) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "my-inference-engine_b200"
for _p in (str(REPO), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

L, HQ, HKV, D = 28, 12, 2, 128
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seqs", type=int, default=256)
    ap.add_argument("--ctx-min", type=int, default=2048)
    ap.add_argument("--ctx-max", type=int, default=8192)
    ap.add_argument("--pool-gb", type=float, default=150.0)
    ap.add_argument("--layers", type=int, default=L)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seqs", type=int, default=4, help="rows in the CPU baseline sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-engine", action="store_true")
    ap.add_argument("--engine-chats", type=int, default=16)
    ap.add_argument("--engine-reply", type=int, default=64)
    ap.add_argument("--engine-prompt", type=int, nargs=2, default=[32, 1000])
    ap.add_argument("--engine-blocks", type=int, default=1024)
    ap.add_argument("--no-engine-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-engine4", action="store_true")
    ap.add_argument("--engine4-chats", type=int, default=1024)
    ap.add_argument("--engine4-prompt", type=int, nargs=2, default=[32, 4096])
    ap.add_argument("--engine4-reply", type=int, default=128)
    ap.add_argument("--engine4-pool-gb", type=float, default=120.0)
    ap.add_argument("--engine-mixed", type=int, default=32, metavar="MIN_TOKENS",
                    help="also serve config 2 with chat.MIXED_PREFILL_MIN_TOKENS=MIN_TOKENS "
                         "(graph-replayed mixed prefill + decode steps); 0 = skip")
    ap.add_argument("--engine4-mixed", type=int, default=1024, metavar="MIN_TOKENS",
                    help="also serve config 4 with chat.MIXED_PREFILL_MIN_TOKENS=MIN_TOKENS "
                         "(prompts of at least MIN_TOKENS share the tick's decode forward, "
                         "replayed from CUDA graphs); 0 = skip")
    ap.add_argument("--engine4-chunk", type=int, default=0, metavar="TOKENS",
                    help="also serve config 4 with mixed steps (--engine4-mixed threshold) and "
                         "chat.MIXED_PREFILL_CHUNK=TOKENS (chunked prefill); 0 = skip")
    ap.add_argument("--no-fp8", action="store_true", help="skip the FP8-pool decode line")
    ap.add_argument("--no-engine3", action="store_true")
    ap.add_argument("--engine3-chats", type=int, default=256)
    ap.add_argument("--engine3-reply", type=int, default=512)
    ap.add_argument("--engine3-arrival-reply", type=int, default=16)
    ap.add_argument("--engine3-pool-gb", type=float, default=150.0)
    ap.add_argument("--engine3-overflow", type=float, default=0.03,
                    help="wave-2 reservations exceed the free blocks by this fraction of the pool")
    ap.add_argument("--engine3-followups", type=int, default=16)
    ap.add_argument("--prefill-steps", type=int, default=20)
    # diagnostics (print their own JSON lines and exit; not the bench line)
    ap.add_argument("--linear-sweep", type=str, default=None, metavar="ROWS",
                    help="comma-separated row counts: per-projection GEMM + fused-op times, "
                         "skinny tensor-core GEMMs vs cuBLAS, CUDA-graph replay")
    ap.add_argument("--decode-step", type=str, default=None, metavar="B:CTX[:PITCH]",
                    help="whole-model decode step time (CUDA graph) at B rows of CTX tokens, "
                         "skinny-GEMM policy vs cuBLAS")
    ap.add_argument("--prefill-step", type=int, default=None, metavar="T",
                    help="whole-model one-row prefill of T tokens (CUDA graph of the padded "
                         "bucket, as chat.py admits a message)")
    ap.add_argument("--prefill-sweep", type=str, default=None, metavar="BxT,...",
                    help="causal prefill attention on dense K/V (12 q / 2 kv heads, d 128) "
                         "per shape and per kernel (PKV_PREFILL_KERNEL one, pair), 20 "
                         "launches per CUDA graph")
    ap.add_argument("--linear-one", type=str, default=None, metavar="OP:ROWS",
                    help="one fused projection (qkv, o, gate_up or down) at ROWS rows, "
                         "5 eager calls (a small case for an ncu capture of linear_tc_kernel)")
    ap.add_argument("--sample-one", type=str, default=None, metavar="ROWS,...",
                    help="pkv_sample on [ROWS, 151936] bf16 logits: device time per call "
                         "(CUDA graph of 20 calls) and GB/s of logits read")
    ap.add_argument("--persistent", action="store_true",
                    help="with --decode-step --profile-range: profile the persistent "
                         "all-layers launch")
    ap.add_argument("--profile-range", action="store_true",
                    help="with --decode-step / --prefill-step: one eager step inside "
                         "cudaProfilerStart/Stop "
                         "(for ncu --profile-from-start off)")
    return ap.parse_args()


def context_lengths(args):
    g = torch.Generator().manual_seed(args.seed)
    return torch.randint(args.ctx_min, args.ctx_max + 1, (args.seqs,), generator=g).tolist()


def decode_bytes(lens):
    """Algorithmic bytes of one paged decode launch (one layer)."""
    B = len(lens)
    kv = sum(lens) * HKV * D * 2 * 2
    qo = 2 * B * HQ * D * 2
    tables = sum(math.ceil(n / 16) for n in lens) * 4 + 2 * B * 4
    return kv + qo + tables


def append_bytes(B):
    """Algorithmic bytes of one fused RoPE + append launch (one layer, T=1)."""
    reads = B * (HQ + 2 * HKV) * D * 2 + 2 * B * D * 2 + 3 * B * 4 + B * 4
    writes = B * HQ * D * 2 + B * 2 * HKV * D * 2
    return reads + writes


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return {"hbm_gbs": FALLBACK_HBM_GBS}, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.lines = []
        self.proc = None
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", uuid, "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- our arm
class DecodeWorkload:
    def __init__(self, args, device):
        import model
        from kv_cache import KVCache

        self.device = device
        self.lens = context_lengths(args)
        self.layers = args.layers
        B = len(self.lens)
        bytes_per_block = L * 2 * 16 * HKV * D * 2
        num_blocks = int(args.pool_gb * 1e9 // bytes_per_block)
        need = sum(math.ceil(n / 16) for n in self.lens)
        assert num_blocks >= need, f"pool of {num_blocks} blocks cannot hold {need}"
        pitch = math.ceil((args.ctx_max + 1) / 16)
        self.cache = KVCache(num_blocks, 16, device, torch.bfloat16, max_seqs=B,
                             max_blocks_per_seq=pitch)
        g = torch.Generator().manual_seed(args.seed + 1)
        self.cache._free_blocks = torch.randperm(num_blocks, generator=g).tolist()
        self.seqs = [self.cache.alloc() for _ in self.lens]
        for s, n in zip(self.seqs, self.lens):
            self.cache.ensure_capacity(s, n)
            self.cache._lengths[s] = n - 1  # history in the pool; this step appends token n-1
        gd = torch.Generator(device=device).manual_seed(args.seed + 2)
        for l in range(L):  # synthetic history, layer by layer to bound temporaries
            self.cache.buf[l].normal_(generator=gd)
        _, self.step, _ = self.cache.prepare(self.seqs, 1)
        self.cos, self.sin = model.rope_table(pitch * 16, torch.bfloat16, device)
        self.q = torch.randn(self.layers, B, HQ, 1, D, device=device, generator=gd).to(torch.bfloat16)
        self.k = torch.randn(self.layers, B, HKV, 1, D, device=device, generator=gd).to(torch.bfloat16)
        self.v = torch.randn(self.layers, B, HKV, 1, D, device=device, generator=gd).to(torch.bfloat16)
        self.q_rot = torch.empty_like(self.q)
        self.out = torch.empty(self.layers, B, HQ, 1, D, device=device, dtype=torch.bfloat16)
        self.handles = [self.cache.read(l, self.step) for l in range(self.layers)]
        self.bytes_decode = decode_bytes(self.lens)
        self.bytes_append = append_bytes(B)
        torch.cuda.synchronize()

    def run_layer(self, l, ev=None):
        from kernels.fa2 import flash_attention

        self.cache.append(l, self.step, self.q[l], self.k[l], self.v[l], self.cos, self.sin,
                          self.q_rot[l])
        kh, vh = self.handles[l]
        if ev is not None:
            ev[0].record()
        flash_attention(self.q_rot[l], kh, vh, False, self.step.kv_lens, out=self.out[l])
        if ev is not None:
            ev[1].record()

    def run_step(self, evs=None):
        for l in range(self.layers):
            self.run_layer(l, evs[l] if evs is not None else None)

    def step_bytes(self):
        return self.layers * (self.bytes_decode + self.bytes_append)


def fp8_decode_bytes(lens):
    """Algorithmic bytes of one FP8-pool decode launch (one layer): per
    visible token and KV head 128 B of K, 128 B of V and two fp32 scales."""
    B = len(lens)
    kv = sum(lens) * HKV * (2 * D + 8)
    qo = 2 * B * HQ * D * 2
    tables = sum(math.ceil(n / 16) for n in lens) * 4 + 2 * B * 4
    return kv + qo + tables


def fp8_decode_run(args, device, bf16_ms_per_step):
    """BASELINE config 3's decode step on the opt-in FP8 pool
    (KVCache(kv_format="fp8_e4m3")): the same 256 rows, contexts, block
    permutation and layer count as the bf16 step, the pool holding random
    e4m3 history (valid codes, scales U[0.001, 0.011]); per layer the
    quantising RoPE + append and the FP8 paged decode kernel."""
    import model
    from kernels.fa2 import flash_attention
    from kv_cache import KVCache

    lens = context_lengths(args)
    B = len(lens)
    bytes_per_block = L * 2 * 16 * HKV * D * 2
    num_blocks = int(args.pool_gb * 1e9 // bytes_per_block)  # same blocks as the bf16 pool
    pitch = math.ceil((args.ctx_max + 1) / 16)
    cache = KVCache(num_blocks, 16, device, torch.bfloat16, max_seqs=B,
                    max_blocks_per_seq=pitch, num_layers=args.layers, kv_format="fp8_e4m3")
    g = torch.Generator().manual_seed(args.seed + 1)
    cache._free_blocks = torch.randperm(num_blocks, generator=g).tolist()
    seqs = [cache.alloc() for _ in lens]
    for s_, n in zip(seqs, lens):
        cache.ensure_capacity(s_, n)
        cache._lengths[s_] = n - 1
    gd = torch.Generator(device=device).manual_seed(args.seed + 2)
    for l in range(args.layers):
        body = cache.pool8[l, :, :, :4096]
        body.random_(0, 256, generator=gd)
        body[(body & 0x7F) == 0x7F] ^= 1  # no NaN codes
        sc = torch.rand(num_blocks, HKV, 32, device=device, generator=gd) * 0.01 + 0.001
        cache.pool8[l, :, :, 4096:] = sc.view(torch.uint8).view(num_blocks, HKV, 128)
        del sc
    _, step, _ = cache.prepare(seqs, 1)
    cos, sin = model.rope_table(pitch * 16, torch.bfloat16, device)
    q = torch.randn(args.layers, B, HQ, 1, D, device=device, generator=gd).to(torch.bfloat16)
    k = torch.randn(args.layers, B, HKV, 1, D, device=device, generator=gd).to(torch.bfloat16)
    v = torch.randn(args.layers, B, HKV, 1, D, device=device, generator=gd).to(torch.bfloat16)
    q_rot = torch.empty_like(q)
    out = torch.empty_like(q)
    handles = [cache.read(l, step) for l in range(args.layers)]
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.layers)]

    def one(events=False):
        for l in range(args.layers):
            cache.append(l, step, q[l], k[l], v[l], cos, sin, q_rot[l])
            kh, vh = handles[l]
            if events:
                ev[l][0].record()
            flash_attention(q_rot[l], kh, vh, False, step.kv_lens, out=out[l])
            if events:
                ev[l][1].record()

    for _ in range(max(3, args.warmup)):
        one()
    torch.cuda.synchronize()
    steps = max(5, args.steps // 4)
    kern = []  # mean decode-launch time of each step (CUDA events on the stream)
    for _ in range(steps):
        one(events=True)
        torch.cuda.synchronize()
        kern.append(statistics.mean(a.elapsed_time(b) for a, b in ev))
    cache.check_errors()
    kern_ms = statistics.mean(kern)
    # whole-step time without the per-step host sync of the kernel timing
    t2, t3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t2.record()
    for _ in range(steps):
        one()
    t3.record()
    t3.synchronize()
    ms = t2.elapsed_time(t3) / steps
    bytes_decode = fp8_decode_bytes(lens)
    step_bytes = args.layers * (bytes_decode + append_bytes(B))
    peaks, src = measured_peaks()
    peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    achieved = bytes_decode / (kern_ms * 1e-3) / 1e9
    # every view of the pool (the step's handles, the fill loop's slice) goes
    # before the cache is returned to the driver: the next runs need the memory
    del cache, q, k, v, q_rot, out, handles, step, body, cos, sin
    gc.collect()
    torch.cuda.empty_cache()
    return {"metric": "paged decode-attn HBM GB/s on the FP8 (e4m3) pool", "kv_format": "fp8_e4m3",
            "value": round(step_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "step_bytes": step_bytes,
            "ms_per_step": round(ms, 4), "steps": steps,
            "tokens_per_s": round(B / (ms * 1e-3), 1),
            "speedup_vs_bf16_step": round(bf16_ms_per_step / ms, 3),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_source": src,
                         "kernel": "paged_decode_kernel<fp8>", "bytes_per_launch": bytes_decode,
                         "avg_launch_ms": round(kern_ms, 4)},
            "config": f"config3 decode on an FP8 pool: {B} rows, ctx U[{args.ctx_min},"
                      f"{args.ctx_max}], {num_blocks}-block pool (528 B per token and layer), "
                      f"{args.layers} layers of quantising RoPE+append + FP8 paged decode"}


def e2e_run(w: DecodeWorkload, steps, warmup):
    """Public API from pinned host buffers: per layer H2D q/k/v, append +
    attention, D2H O, all inside the timed region.  The copies run on a
    second stream, pipelined against the kernels as a serving engine would:
    layer l's inputs are copied while earlier layers compute (each layer has
    its own device buffers; a layer's next-step copy waits for its last
    use), and O_l is copied back while later layers compute.  The timed
    region ends when the last D2H has landed."""
    from kernels.fa2 import flash_attention

    B = len(w.lens)
    hq = torch.empty(B, HQ, 1, D, dtype=torch.bfloat16).pin_memory()
    hk = torch.empty(B, HKV, 1, D, dtype=torch.bfloat16).pin_memory()
    hv = torch.empty(B, HKV, 1, D, dtype=torch.bfloat16).pin_memory()
    hq.copy_(w.q[0].cpu())
    hk.copy_(w.k[0].cpu())
    hv.copy_(w.v[0].cpu())
    hout = [torch.empty(B, HQ, 1, D, dtype=torch.bfloat16).pin_memory() for _ in range(w.layers)]
    dev_bufs = [[torch.empty(t.shape, dtype=t.dtype, device=w.device) for t in (hq, hk, hv, hq, hq)]
                for _ in range(w.layers)]  # q, k, v, roped q, O per layer
    main = torch.cuda.current_stream()
    copy = torch.cuda.Stream()
    inputs_in = [torch.cuda.Event() for _ in range(w.layers)]
    layer_done = [torch.cuda.Event() for _ in range(w.layers)]
    used = [False] * w.layers

    def one():
        with torch.cuda.stream(copy):
            for l in range(w.layers):
                dq, dk, dv, _, _ = dev_bufs[l]
                if used[l]:
                    copy.wait_event(layer_done[l])  # last step's kernels are done with them
                dq.copy_(hq, non_blocking=True)
                dk.copy_(hk, non_blocking=True)
                dv.copy_(hv, non_blocking=True)
                inputs_in[l].record(copy)
        for l in range(w.layers):
            dq, dk, dv, qr, do = dev_bufs[l]
            main.wait_event(inputs_in[l])
            w.cache.append(l, w.step, dq, dk, dv, w.cos, w.sin, qr)
            kh, vh = w.handles[l]
            flash_attention(qr, kh, vh, False, w.step.kv_lens, out=do)
            layer_done[l].record(main)
            used[l] = True
            with torch.cuda.stream(copy):
                copy.wait_event(layer_done[l])
                hout[l].copy_(do, non_blocking=True)
        main.wait_stream(copy)

    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        one()
    e.record()
    e.synchronize()
    ms = s.elapsed_time(e) / steps
    h2d = w.layers * (hq.numel() + hk.numel() + hv.numel()) * 2
    d2h = w.layers * hout[0].numel() * 2
    return ms, h2d, d2h


# ---------------------------------------------------------------- CPU path
CPU_WARMUP, CPU_MIN_STEPS, CPU_MIN_SECONDS = 3, 10, 10.0


class CpuPath:
    """Reference CPU path (oracle restatement) on a bounded sample: the first
    --cpu-seqs rows of the same length distribution, all layers, fp32."""

    def __init__(self, args):
        from oracle.reference_path import CpuDecodePath

        self.lens = context_lengths(args)[: args.cpu_seqs]
        self.layers = args.layers
        self.path = CpuDecodePath(self.lens, args.layers, seed=args.seed)
        self.bytes = args.layers * (decode_bytes(self.lens) + append_bytes(len(self.lens)))

    def sample(self):
        return (f"{len(self.lens)} rows (ctx {self.lens}) x {self.layers} layers per step, "
                f"fp32 torch CPU")

    def measure(self, warmup=CPU_WARMUP, min_steps=CPU_MIN_STEPS, min_seconds=CPU_MIN_SECONDS):
        """The one timing rule both arms use for the CPU path: `warmup`
        untimed steps, then steps timed one by one until at least `min_steps`
        steps AND `min_seconds` have passed.  Returns the median seconds per
        step and the spread (min, max, n)."""
        for _ in range(warmup):
            self.path.step()
        times, t0 = [], time.perf_counter()
        while len(times) < min_steps or time.perf_counter() - t0 < min_seconds:
            t = time.perf_counter()
            self.path.step()
            times.append(time.perf_counter() - t)
        return statistics.median(times), {"min_ms": round(min(times) * 1e3, 2),
                                          "max_ms": round(max(times) * 1e3, 2),
                                          "median_ms": round(statistics.median(times) * 1e3, 2),
                                          "steps": len(times), "warmup": warmup}


def cpu_info():
    name = ""
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                name = ln.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return name


# ---------------------------------------------------------------- prefill
def prefill_run(args, device, seed=0):
    """BASELINE config 1 on the tcgen05 prefill kernel: 8 rows with prompt
    lengths U[16,1024] (seeded) appended to empty caches in a shuffled pool,
    then per layer ONE causal attention launch over the paged K/V with the
    queries left-padded to the longest prompt (bottom-right alignment puts each
    row's real queries on its own keys; padded query rows see no key).
    Useful FLOPs = sum_b 4*12*128*L_b(L_b+1)/2 per layer."""
    from kernels.fa2 import flash_attention
    from kv_cache import KVCache, PagedStep

    g = torch.Generator().manual_seed(seed + 42)
    lens = torch.randint(16, 1025, (8,), generator=g).tolist()
    T = max(lens)
    N = sum(math.ceil(n / 16) for n in lens) + 16
    cache = KVCache(N, 16, device, torch.bfloat16)
    cache._free_blocks = torch.randperm(N, generator=g).tolist()
    seqs = [cache.alloc() for _ in lens]
    gd = torch.Generator(device=device).manual_seed(seed + 43)
    for s_, n in zip(seqs, lens):  # prompt K/V appended through the product path
        k = torch.randn(1, HKV, n, D, device=device, generator=gd).to(torch.bfloat16)
        v = torch.randn(1, HKV, n, D, device=device, generator=gd).to(torch.bfloat16)
        _, st, _ = cache.prepare([s_], n)
        for l in range(L):
            cache.write(l, st, k, v)
        cache.advance([s_], n)
    rows = torch.tensor([cache.table_row(x) for x in seqs], dtype=torch.int32, device=device)
    kvl = torch.tensor(lens, dtype=torch.int32, device=device)
    step = PagedStep(cache, T, [0] * len(lens), rows, kvl - T, kvl, T)
    q = torch.randn(L, len(lens), HQ, T, D, device=device, generator=gd).to(torch.bfloat16)
    out = torch.empty_like(q)
    handles = [cache.read(l, step) for l in range(L)]

    def one():
        for l in range(L):
            kh, vh = handles[l]
            flash_attention(q[l], kh, vh, True, kvl, out=out[l])

    for _ in range(3):
        one()
    torch.cuda.synchronize()
    # the 28 launches replayed from a CUDA graph (as the engine runs its
    # prefills), so the device time is the kernels', not the host's
    # per-launch argument packing
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        one()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.prefill_steps):
        graph.replay()
    e1.record()
    e1.synchronize()
    cache.check_errors()
    ms = e0.elapsed_time(e1) / args.prefill_steps / L
    del graph
    flops = sum(4 * HQ * D * n * (n + 1) / 2 for n in lens)
    peaks, src = measured_peaks()
    peak = float(peaks.get("bf16_tflops", 1590.0))
    tf = flops / (ms * 1e-3) / 1e12
    del cache, q, out, handles
    torch.cuda.empty_cache()
    return {"metric": "paged causal prefill attention, useful TFLOP/s", "value": round(tf, 1),
            "unit": "TFLOP/s", "kernel": "prefill_tc_kernel (tcgen05 + TMEM)",
            "ms_per_launch": round(ms, 4), "flops_per_launch": flops,
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(tf / peak, 4), "peak_source": src},
            "config": f"config1: 8 rows, prompt lengths {lens} from empty caches, shuffled "
                      f"{N}-block pool, causal, queries left-padded to {T}, one launch per layer, "
                      f"28 layers replayed from a CUDA graph"}


# ---------------------------------------------------------------- engine
WEIGHT_BYTES = None  # filled from the model's parameter count


def random_init_(model, seed, std=0.02):
    """Random-init weights: N(0, std) for weights and
    biases, RMSNorm weights 1, generated on the model's device."""
    g = torch.Generator(device=next(model.parameters()).device).manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("layernorm.weight") or name == "norm.weight":
                p.fill_(1.0)
            else:
                p.normal_(0.0, std, generator=g)


class SyntheticTokenizer:
    """Token ids stand in for text: message "p<i>" encodes to prompt i."""

    encoder = {"<|endoftext|>": -1}  # never sampled: replies run their full length

    def __init__(self, prompts):
        self.prompts = prompts

    def encode(self, text):
        if text == "\n":
            return [198]
        i = int(text.split("User: p", 1)[1].split("\n", 1)[0])
        return list(self.prompts[i])

    def decode(self, ids):
        return ""


class _CountingModel:
    """Forwards to the model and records (B, T, sum of kv lens) per call."""

    def __init__(self, model, cache):
        self.model, self.cache, self.calls = model, cache, []
        self.last_mixed = None

    @property
    def _graphs(self):
        return self.model._graphs

    def __call__(self, input_ids, cache, seqs):
        B, T = input_ids.shape
        starts = [cache.length(s) for s in seqs]
        kv = sum(starts) + B * T
        # causal (query, key) pairs of the attention: query i of a row that
        # starts at s sees s + i + 1 keys
        pairs = sum(T * s + T * (T + 1) // 2 for s in starts)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = self.model(input_ids, cache, seqs)
        e1.record()
        self.calls.append(("decode" if T == 1 else "prefill", B * T, kv, e0, e1, pairs))
        return out

    def forward_mixed(self, prefill_ids, prefill_seq, decode_ids, decode_seqs, cache):
        T, B = prefill_ids.shape[1], len(decode_seqs)
        kv = sum(cache.length(s) for s in decode_seqs) + B + cache.length(prefill_seq) + T
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        s0 = cache.length(prefill_seq)
        pairs = T * s0 + T * (T + 1) // 2 + sum(cache.length(s) + 1 for s in decode_seqs)
        out = self.model.forward_mixed(prefill_ids, prefill_seq, decode_ids, decode_seqs, cache)
        e1.record()
        self.calls.append(("mixed", T + B, kv, e0, e1, pairs))
        self.last_mixed = {"T": T, "B": B, "prompt_start": s0,
                           "max_decode_len": max(cache.length(s) for s in decode_seqs)}
        return out


ROOFLINE_BASIS = ("per call: decode = (weights + KV read) / measured HBM; prefill = max((2*params"
                  "*tokens + 4*12*128*causal pairs*28) / measured bf16 peak, bytes / HBM)")


def call_roofline(calls, nparams):
    """Per-call roofline time of an engine run and the device time split.

    decode call : weights + every visible key's K/V read once at the measured
                  HBM bandwidth;
    prefill / mixed call : max(GEMM FLOPs 2 * params * rows + attention FLOPs
                  4 * 12 heads * 128 * causal pairs * 28 layers at the measured
                  bf16 peak, the same bytes at HBM)."""
    peaks, _ = measured_peaks()
    bw = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS)) * 1e9
    flops_peak = float(peaks.get("bf16_tflops", 1590.0)) * 1e12
    wbytes = nparams * 2
    kv_tok = L * 2 * HKV * D * 2
    out = {"t_roof": 0.0, "decode_steps": 0, "prefills": 0, "mixed": 0, "decode_ms": 0.0,
           "prefill_ms": 0.0, "mixed_ms": 0.0}
    for kind, rows, kv, e0, e1, pairs in calls:
        ms = e0.elapsed_time(e1)
        if kind == "decode":
            out["decode_steps"] += 1
            out["decode_ms"] += ms
            out["t_roof"] += (wbytes + kv * kv_tok) / bw
        else:
            key = "mixed" if kind == "mixed" else "prefills"
            out[key] += 1
            out["mixed_ms" if kind == "mixed" else "prefill_ms"] += ms
            flops = 2 * nparams * rows + 4 * HQ * D * pairs * L
            out["t_roof"] += max(flops / flops_peak, (wbytes + kv * kv_tok) / bw)
    return out


def engine_run(device, *, label, chats_total, prompt_range, reply, blocks, max_batch,
               rank=0, world=1, seed=0, mixed_min=None, mixed_graphs=True, mixed_chunk=None):
    """Serve `chats_total` chats through chat.py (uniform random token-id prompts
    in `prompt_range`, `reply`-token replies with EOS and stop sequences off as
    metrics/benchmark_concurrency.py:122,143 does, temperature-1 sampling, one
    prefill per tick).  Rank r serves chats i with i % world == r from one
    seeded prompt set, on its own model replica and `blocks`-block pool.
    mixed_min: chat.MIXED_PREFILL_MIN_TOKENS for this run (None: the
    reference's scheduling); its mixed steps replay captured graphs
    (model.MixedGraphs) unless mixed_graphs is False; mixed_chunk:
    chat.MIXED_PREFILL_CHUNK (chunked prefill).  Returns this rank's tokens, wall time and a
    roofline."""
    import chat
    import model as M
    from kv_cache import KVCache

    gc.collect()  # the previous run's pool back to the driver before this one's
    torch.cuda.empty_cache()
    torch.manual_seed(seed + rank)
    m = M.Qwen2ForCausalLM().to(device, torch.bfloat16).eval()
    random_init_(m, seed + 11)
    cache = KVCache(blocks, 16, device, torch.bfloat16)
    chat.init(kv_cache=cache, start_worker=False)
    chat.STOP_SEQUENCES = []
    chat.MIXED_PREFILL_MIN_TOKENS = mixed_min
    chat.MIXED_PREFILL_CHUNK = mixed_chunk
    lo, hi = prompt_range
    runner = m.enable_decode_graphs(cache, max_batch=max_batch)
    for b in runner.buckets:  # capture outside the timed region
        runner._capture(b)
    prunner = m.enable_prefill_graphs(cache, max_len=hi)
    for b in prunner.buckets:
        prunner._capture(b)
    mrunner = None
    if mixed_min is not None and mixed_graphs and mixed_min <= hi:
        mrunner = m.enable_mixed_graphs(cache, max_len=hi, max_batch=max_batch)
        # chunks of a prompt above mixed_chunk tokens are longer than half of it
        shortest = min(mixed_min, mixed_chunk // 2 + 1) if mixed_chunk else mixed_min
        t0 = mrunner.buckets(max(shortest, 2), 1)[0]
        for tp in mrunner.t_buckets:
            for bp in mrunner.b_buckets:
                if tp >= t0:
                    mrunner.capture(tp, bp)
    g = torch.Generator().manual_seed(seed + 5)
    prompts = [torch.randint(0, M.VOCAB_SIZE, (int(torch.randint(lo, hi + 1, (1,), generator=g)),),
                             generator=g).tolist() for _ in range(chats_total + 1)]
    tok = SyntheticTokenizer(prompts)
    cm = _CountingModel(m, cache)

    def one_round(idx, nreply):
        chat.MAX_REPLY_TOKENS = nreply
        chats = []
        for i in idx:
            c = chat.Chat(tok)
            c.eos_id = -1
            c.submit(cm, f"p{i}")
            chats.append(c)
        t0 = time.perf_counter()
        chat.run_until_idle()
        torch.cuda.synchronize()
        el = time.perf_counter() - t0
        toks = sum(len(c.ids) - len(tok.prompts[i]) - 1 for c, i in zip(chats, idx))
        for c in chats:
            c.release()
        return el, toks

    one_round([chats_total], 4)  # warm-up: sampling, one graph of each kind
    cm.calls.clear()
    mine = [i for i in range(chats_total) if i % world == rank]
    try:
        el, toks = one_round(mine, reply)
    except RuntimeError as e:
        # name the failing step: the device error word and the last mixed step
        bits = int(cache.err_flag.item())
        raise RuntimeError(f"{label} run failed: {e}; device error bits {bits:#x}; "
                           f"{len(cm.calls)} model calls; last mixed step {cm.last_mixed}") from e
    torch.cuda.synchronize()
    nparams = sum(p.numel() for p in m.parameters())
    cr = call_roofline(cm.calls, nparams)
    t_roof, decode_steps, prefills, mixed = cr["t_roof"], cr["decode_steps"], cr["prefills"], cr["mixed"]
    gpu_decode, gpu_prefill, gpu_mixed = cr["decode_ms"], cr["prefill_ms"], cr["mixed_ms"]
    chat._kv_cache = None
    chat.MIXED_PREFILL_MIN_TOKENS = None
    chat.MIXED_PREFILL_CHUNK = None
    m._graphs.clear()  # the graph runners and the model refer to each other
    m._prefill_graphs.clear()
    m._mixed_graphs.clear()
    mixed_kind = "CUDA-graph" if mrunner is not None else "eager"
    del runner, prunner, mrunner, m, cache, cm
    gc.collect()
    torch.cuda.empty_cache()
    return {"tok_s": round(toks / el, 1), "tokens": toks, "wall_s": round(el, 4),
            "decode_steps": decode_steps, "prefills": prefills,
            **({"mixed_steps": mixed, "mixed_min_tokens": mixed_min} if mixed_min is not None else {}),
            "model_ms": {"decode_total": round(gpu_decode, 2), "prefill_total": round(gpu_prefill, 2),
                         **({"mixed_total": round(gpu_mixed, 2)} if mixed_min is not None else {}),
                         "decode_per_step": round(gpu_decode / max(decode_steps, 1), 3),
                         "note": "CUDA events around each model call on the stream"},
            "roofline_tok_s": round(toks / t_roof, 1), "frac": round(t_roof / el, 4),
            "roofline_basis": ROOFLINE_BASIS,
            "config": f"{label}: {chats_total} chats ({len(mine)} on this GPU), prompts "
                      f"U[{lo},{hi}] random ids, {reply}-token replies, {blocks}-block pool, "
                      f"random-init bf16 Qwen2.5-1.5B (std 0.02), temperature-1 sampling, "
                      f"one prefill per tick (chat.py), CUDA-graph decode and prefill"
                      + (f"; prompts >= {mixed_min} tokens admitted while others decode share "
                         f"their forward ({mixed_kind} "
                         f"mixed step)" if mixed_min is not None else "")
                      + (f", in chunks of at most {mixed_chunk} tokens, one per tick"
                         if mixed_min is not None and mixed_chunk else "")}


def engine3_run(args, device, seed=0):
    """BASELINE config 3 as an engine run through chat.py: a ~150 GB pool,
    256 chats with prompts U[2048, 8192] decoding together, then arrivals
    whose reservations exceed the free blocks, so chat.py's LRU eviction of
    idle chats fires (chat.py:117-125 reserve, :128-146 _make_room), then
    follow-up messages to evicted chats, whose whole history is prefilled
    again (chat.py:157-185 _admit).  Three waves, each driven to idle:

      wave 1  256 chats, prompts U[ctx_min, ctx_max], `engine3_reply`-token
              replies (512 = the reference's MAX_REPLY_TOKENS): one prefill
              per tick while the admitted chats decode, up to 256 rows per
              decode step;
      wave 2  chats with prompts U[ctx_min, ctx_max] and short replies, drawn
              until their reservations exceed the free blocks left by wave 1
              by `engine3_overflow` of the pool: the idle wave-1 chats are
              evicted, least recently used first;
      wave 3  a 64-token follow-up to each of the first `engine3_followups`
              wave-1 chats (evicted first): re-prefill of history + message.

    Token ids are random (seeded), weights random-init (std 0.02); EOS and
    stop sequences are off so replies run their full length (as
    metrics/benchmark_concurrency.py does).  Decode steps and one-row
    prefills replay CUDA graphs captured before the timed region."""
    import chat
    import model as M
    from kv_cache import KVCache

    torch.manual_seed(seed)
    gc.collect()
    torch.cuda.empty_cache()
    m = M.Qwen2ForCausalLM().to(device, torch.bfloat16).eval()
    random_init_(m, seed + 11)
    block_bytes = L * 2 * 16 * HKV * D * 2
    blocks = int(args.engine3_pool_gb * 1e9 // block_bytes)
    lo, hi = args.ctx_min, args.ctx_max
    r1, r2, r3 = args.engine3_reply, args.engine3_arrival_reply, 64
    follow = 64
    longest = hi + r1 + 1 + follow + r3 + 1  # a re-prefilled follow-up's whole reservation
    pitch = -(-longest // 16) + 1
    cache = KVCache(blocks, 16, device, torch.bfloat16, max_seqs=2048, max_blocks_per_seq=pitch)
    chat.init(kv_cache=cache, start_worker=False)
    saved = chat.STOP_SEQUENCES, chat.MAX_REPLY_TOKENS, chat.MIXED_PREFILL_MIN_TOKENS
    chat.STOP_SEQUENCES = []
    chat.MIXED_PREFILL_MIN_TOKENS = None
    runner = m.enable_decode_graphs(cache, max_batch=256)
    prunner = m.enable_prefill_graphs(cache, max_len=hi + r1 + 1 + follow)
    t0 = time.perf_counter()
    for b in runner.buckets:  # capture outside the timed region
        runner._capture(b)
    for b in prunner.buckets:
        prunner._capture(b)
    capture_s = time.perf_counter() - t0
    g = torch.Generator().manual_seed(seed + 7)

    def draw(n_tokens):
        return torch.randint(0, M.VOCAB_SIZE, (n_tokens,), generator=g).tolist()

    def draw_len():
        return int(torch.randint(lo, hi + 1, (1,), generator=g))

    prompts = [draw(draw_len()) for _ in range(args.engine3_chats)]
    tok = SyntheticTokenizer(prompts)
    cm = _CountingModel(m, cache)
    evictions = [0]
    real_evict = chat._evict

    def counting_evict(c):
        evictions[0] += 1
        real_evict(c)

    chat._evict = counting_evict

    def run_wave(pairs, nreply):
        """pairs: (Chat, message index); returns (wall s, generated tokens)."""
        chat.MAX_REPLY_TOKENS = nreply
        before = [len(c.ids) for c, _ in pairs]
        for c, i in pairs:
            c.submit(cm, f"p{i}")
        t = time.perf_counter()
        chat.run_until_idle()
        torch.cuda.synchronize()
        el = time.perf_counter() - t
        toks = sum(len(c.ids) - b - len(tok.prompts[i]) - 1 for (c, i), b in zip(pairs, before))
        return el, toks

    def new_chat():
        c = chat.Chat(tok)
        c.eos_id = -1
        return c

    try:
        # warm-up: sampling and one graph of each kind, outside the timed region
        tok.prompts.append(draw(lo))
        wc = new_chat()
        run_wave([(wc, len(tok.prompts) - 1)], 4)
        wc.release()
        cm.calls.clear()
        evictions[0] = 0
        waves = {}
        chats1 = [new_chat() for _ in range(args.engine3_chats)]
        el, toks = run_wave([(c, i) for i, c in enumerate(chats1)], r1)
        peak_batch = max((rows for kind, rows, *_ in cm.calls if kind == "decode"), default=0)
        waves["wave1"] = {"chats": len(chats1), "wall_s": round(el, 3), "tokens": toks,
                          "tok_s": round(toks / el, 1), "peak_decode_rows": peak_batch,
                          "free_blocks_after": cache.free_block_count()}
        # wave 2: arrivals whose reservations exceed the free blocks
        free = cache.free_block_count()
        want = free + int(args.engine3_overflow * blocks)
        first, need = len(tok.prompts), 0
        while need <= want:
            n = draw_len()
            tok.prompts.append(draw(n))
            need += -(-(n + r2 + 1) // 16)
        chats2 = [new_chat() for _ in range(first, len(tok.prompts))]
        el2, toks2 = run_wave([(c, first + j) for j, c in enumerate(chats2)], r2)
        ev2 = evictions[0]
        n_calls2 = len(cm.calls)
        waves["wave2"] = {"chats": len(chats2), "wall_s": round(el2, 3), "tokens": toks2,
                          "tok_s": round(toks2 / el2, 1), "reserved_blocks": need,
                          "free_blocks_before": free, "evictions": ev2}
        # wave 3: follow-ups to the least recently used wave-1 chats
        fol = chats1[:args.engine3_followups]
        evicted = sum(1 for c in fol if c.seq is None)
        first = len(tok.prompts)
        for _ in fol:
            tok.prompts.append(draw(follow))
        el3, toks3 = run_wave([(c, first + j) for j, c in enumerate(fol)], r3)
        # a follow-up to a resident chat prefills its 64 new tokens and the
        # previous reply's trailing newline; an evicted one its whole history
        re = [rows for kind, rows, *_ in cm.calls[n_calls2:] if kind == "prefill"
              and rows > follow + 1]
        re_prefills, re_prefill_tokens = len(re), sum(re)
        waves["wave3"] = {"chats": len(fol), "wall_s": round(el3, 3), "tokens": toks3,
                          "tok_s": round(toks3 / el3, 1), "evicted_before_followup": evicted,
                          "evictions": evictions[0] - ev2}
        torch.cuda.synchronize()
        cache.check_errors()
        nparams = sum(p.numel() for p in m.parameters())
        cr = call_roofline(cm.calls, nparams)
        wall = el + el2 + el3
        tokens = toks + toks2 + toks3
    finally:
        chat._evict = real_evict
        chat.STOP_SEQUENCES, chat.MAX_REPLY_TOKENS, chat.MIXED_PREFILL_MIN_TOKENS = saved
        chat._kv_cache = None
        m._graphs.clear()
        m._prefill_graphs.clear()
    del runner, prunner, m, cache, cm
    gc.collect()
    torch.cuda.empty_cache()
    return {"tok_s": round(tokens / wall, 1), "tokens": tokens, "wall_s": round(wall, 3),
            "evictions": evictions[0], "re_prefills": re_prefills,
            "re_prefill_tokens": re_prefill_tokens, "pool_blocks": blocks,
            "decode_steps": cr["decode_steps"], "prefills": cr["prefills"], "waves": waves,
            "model_ms": {"decode_total": round(cr["decode_ms"], 2),
                         "prefill_total": round(cr["prefill_ms"], 2),
                         "decode_per_step": round(cr["decode_ms"] / max(cr["decode_steps"], 1), 3),
                         "note": "CUDA events around each model call on the stream"},
            "roofline_tok_s": round(tokens / cr["t_roof"], 1),
            "frac": round(cr["t_roof"] / wall, 4), "roofline_basis": ROOFLINE_BASIS,
            "graph_capture_s": round(capture_s, 2),
            "config": f"config3 engine: {blocks}-block pool (~{args.engine3_pool_gb:g} GB bf16), "
                      f"{len(chats1)} chats with prompts U[{lo},{hi}] random ids and "
                      f"{r1}-token replies, then {len(chats2)} arrivals (prompts U[{lo},{hi}], "
                      f"{r2}-token replies) reserving more than the free blocks, then "
                      f"{len(fol)} {follow}-token follow-ups to the least recently used "
                      f"wave-1 chats; random-init bf16 Qwen2.5-1.5B, temperature-1 sampling, "
                      f"one prefill per tick (chat.py), CUDA-graph decode and prefill"}


def engine_cpu_sample(seconds_budget=60.0):
    """The reference engine's own CPU path (restated model + gather/SDPA cache,
    fp32, chat.py's CPU dtype) on a bounded sample: 2 chats, 32-token prompts,
    4-token replies, batched decode."""
    from oracle.kvcache_ref import RefKVCache
    from oracle.model_ref import RefQwen2

    torch.manual_seed(0)
    m = RefQwen2().eval()
    random_init_(m, 11)
    cache = RefKVCache(16, 16, torch.float32)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 151936, (32,), generator=g).tolist() for _ in range(2)]
    seqs = [cache.alloc(), cache.alloc()]
    t0 = time.perf_counter()
    nxt = []
    for r in range(2):
        lg = m(torch.tensor([prompts[r]]), cache, [seqs[r]])[:, -1]
        nxt.append(int(torch.multinomial(torch.softmax(lg.float(), -1), 1)[0]))
    toks = 2
    for _ in range(3):
        lg = m(torch.tensor([[x] for x in nxt]), cache, seqs)[:, -1]
        nxt = torch.multinomial(torch.softmax(lg.float(), -1), 1)[:, 0].tolist()
        toks += 2
    el = time.perf_counter() - t0
    return {"tok_s": round(toks / el, 3), "cores": torch.get_num_threads(), "kind": "port",
            "sample": "2 chats, 32-token prompts, 4-token replies, fp32 torch CPU (prefill included)"}


# ---------------------------------------------------------------- ranks
def reset_chat_scheduler():
    """Drop chat.py's scheduler state after a run that raised mid-tick (its
    jobs, deferred and resident chats, queued messages, cache), so the next
    engine run starts clean."""
    import chat

    chat.active.clear()
    chat._deferred.clear()
    chat._mixed.clear()
    for c in chat._resident:
        c.seq = None
    chat._resident.clear()
    while not chat._job_queue.empty():
        chat._job_queue.get_nowait()
    chat._kv_cache = None
    chat.MIXED_PREFILL_MIN_TOKENS = None


def opt_in_run(fn, device, world):
    """Run one opt-in engine leg (a mixed-step mode): returns (result, None),
    or (None, error text) on every rank if it raised on any rank, so that a
    failure there is reported in the JSON line instead of losing the line,
    and every rank still takes the same collectives."""
    err = None
    try:
        r = fn()
    except RuntimeError as e:
        r, err = None, f"{type(e).__name__}: {e}"[:600]
        reset_chat_scheduler()
        gc.collect()
        torch.cuda.empty_cache()
    if cross_rank(1.0 if err else 0.0, torch.distributed.ReduceOp.MAX if world > 1 else None,
                  device, world) > 0:
        return None, err or "failed on another rank"
    return r, None


def cross_rank(value, op, device, world):
    """all_reduce of one float over the ranks (MAX or SUM); identity at N=1."""
    if world == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=op)
    return float(t.item())


def gather_ranks(obj, world):
    """Every rank's `obj` (a small dict), in rank order; every rank calls it
    at the same point (a collective)."""
    if world == 1:
        return [obj]
    out = [None] * world
    torch.distributed.all_gather_object(out, obj)
    return out


def rank_summary(rank, r):
    """One rank's share of an engine run: its own tokens, wall time and the
    device-time split of its model calls."""
    return {"rank": rank, "tok_s": r["tok_s"], "tokens": r["tokens"], "wall_s": r["wall_s"],
            "decode_steps": r["decode_steps"], "prefills": r["prefills"],
            "decode_ms": r["model_ms"]["decode_total"], "prefill_ms": r["model_ms"]["prefill_total"],
            "decode_ms_per_step": r["model_ms"]["decode_per_step"], "frac": r["frac"]}


def replica_rate(units_per_rank, ms_local, device, world):
    """Whole-job rate of N independent replicas: every rank processed
    units_per_rank in its own time; the job took the slowest rank's time.
    Returns (max ms over ranks, units of all ranks per second)."""
    ms_max = cross_rank(ms_local, torch.distributed.ReduceOp.MAX if world > 1 else None, device,
                        world)
    return ms_max, units_per_rank * world / (ms_max * 1e-3)


# ---------------------------------------------------------------- main


# ---------------------------------------------------------------- diagnostics
def _graph_us(fn, calls):
    """Mean device time per call of `fn` (which makes `calls` calls), replayed
    from one CUDA graph; median of 10 replays."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(10):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b) * 1e3 / calls)
    return statistics.median(ts)


def linear_sweep(rows_list, device):
    """Each Qwen2.5-1.5B projection with the op it feeds, as one decode layer
    runs it: 28 distinct weight copies (weights stream from HBM as in a real
    step), one CUDA graph of 28 calls.  cuBLAS (F.linear) + the separate fused
    kernel vs the fused skinny-GEMM entry."""
    import pagedkv

    peaks, src = measured_peaks()
    peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    nw = torch.ones(1536, device=device, dtype=torch.bfloat16)
    paired = None
    for n, k, op in ((2048, 1536, "qkv"), (1536, 1536, "o+add_rmsnorm"),
                     (17920, 1536, "gate_up+silu_mul"), (1536, 8960, "down+add_rmsnorm")):
        ws = [(0.02 * torch.randn(n, k, device=device)).to(torch.bfloat16) for _ in range(L)]
        for rows in rows_list:
            x = torch.randn(rows, k, device=device).to(torch.bfloat16)
            resid = torch.randn(rows, 1536, device=device).to(torch.bfloat16)
            outs = [torch.empty(rows, n, device=device, dtype=torch.bfloat16) for _ in range(L)]
            if op == "qkv":
                def cub():
                    for w, o in zip(ws, outs):
                        torch.matmul(x, w.T, out=o)

                def ours():
                    for w, o in zip(ws, outs):
                        pagedkv.linear(x, w, out=o)
            elif op.startswith("gate_up"):
                acts = [torch.empty(rows, n // 2, device=device, dtype=torch.bfloat16)
                        for _ in range(L)]
                if rows == rows_list[0]:  # the model's layout: SwiGLU in the GEMM epilogue
                    paired = [pagedkv.PairedGateUp(w) for w in ws]

                def cub():
                    for w, o, a in zip(ws, outs, acts):
                        torch.matmul(x, w.T, out=o)
                        pagedkv.silu_mul(o, out=a)

                def ours():
                    for w, a in zip(paired, acts):
                        pagedkv.linear_silu_mul(x, w, out=a)
            else:
                hs = [torch.empty(rows, 1536, device=device, dtype=torch.bfloat16)
                      for _ in range(L)]

                def cub():
                    for w, o, h in zip(ws, outs, hs):
                        torch.matmul(x, w.T, out=o)
                        pagedkv.add_rmsnorm(o, resid, nw, 1e-6, resid_out=resid, out=h)

                def ours():
                    for w, h in zip(ws, hs):
                        pagedkv.linear_add_rmsnorm(x, w, resid, nw, 1e-6, resid_out=resid, out=h)
            t_c, t_o = _graph_us(cub, L), _graph_us(ours, L)
            wb = n * k * 2
            print(json.dumps({"diag": "linear_sweep", "op": op, "rows": rows, "n": n, "k": k,
                              "cublas_us": round(t_c, 2), "skinny_us": round(t_o, 2),
                              "skinny_weight_gbs": round(wb / t_o / 1e3, 1),
                              "skinny_frac_of_hbm": round(wb / t_o / 1e3 / peak, 3),
                              "peak_source": src}), flush=True)
        del ws
        paired = None


def linear_one(spec, device):
    """5 eager calls of one fused projection entry at ROWS rows (layer shapes
    of Qwen2.5-1.5B), then the mean time of 20 more; prints one JSON line."""
    import pagedkv

    op, rows = spec.split(":")
    rows = int(rows)
    n, k = {"qkv": (2048, 1536), "o": (1536, 1536), "gate_up": (17920, 1536),
            "down": (1536, 8960)}[op]
    g = torch.Generator(device=device).manual_seed(rows)
    w = (0.02 * torch.randn(n, k, device=device, generator=g)).to(torch.bfloat16)
    x = torch.randn(rows, k, device=device, generator=g).to(torch.bfloat16)
    resid = torch.randn(rows, 1536, device=device, generator=g).to(torch.bfloat16)
    nw = torch.ones(1536, device=device, dtype=torch.bfloat16)
    h = torch.empty(rows, 1536, device=device, dtype=torch.bfloat16)
    if op == "gate_up":
        w = pagedkv.PairedGateUp(w)
        act = torch.empty(rows, n // 2, device=device, dtype=torch.bfloat16)
        call = lambda: pagedkv.linear_silu_mul(x, w, out=act)  # noqa: E731
    elif op == "qkv":
        y = torch.empty(rows, n, device=device, dtype=torch.bfloat16)
        call = lambda: pagedkv.linear(x, w, out=y)  # noqa: E731
    else:
        call = lambda: pagedkv.linear_add_rmsnorm(x, w, resid, nw, 1e-6, out=h)  # noqa: E731
    for _ in range(5):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        call()
    e1.record()
    e1.synchronize()
    print(json.dumps({"diag": "linear_one", "op": op, "rows": rows, "n": n, "k": k,
                      "eager_us_per_call": round(e0.elapsed_time(e1) / 20 * 1e3, 2)}), flush=True)


def sample_one(spec, device):
    """Device time of pkv_sample (the engine's sampler) on the model's
    vocabulary: 20 calls per CUDA graph, median of 5 replays; bytes = the
    bf16 logits read once."""
    import pagedkv

    peaks, src = measured_peaks()
    peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    vocab = 151936
    for rows in (int(r) for r in spec.split(",")):
        g = torch.Generator(device=device).manual_seed(rows)
        logits = torch.randn(rows, vocab, device=device, generator=g).to(torch.bfloat16)
        out = torch.empty(rows, dtype=torch.int32, device=device)
        for c in range(3):
            pagedkv.sample(logits, 1.0, seed=1, call=c, out=out)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for c in range(20):
                pagedkv.sample(logits, 1.0, seed=1, call=c, out=out)
        graph.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3 / 20)
        us = statistics.median(ts)
        gbs = rows * vocab * 2 / (us * 1e-6) / 1e9
        print(json.dumps({"diag": "sample_one", "rows": rows, "vocab": vocab,
                          "us_per_call": round(us, 2), "logits_gbs": round(gbs, 1),
                          "frac_of_hbm": round(gbs / peak, 3), "peak_source": src}), flush=True)
        del graph


def decode_step_diag(spec, device, profile_range=False, persistent_profile=False):
    """Whole-model decode step (random-init Qwen2.5-1.5B, B rows of CTX
    tokens of history) replayed from a CUDA graph, under the skinny-GEMM
    policy, with every projection on cuBLAS and (B <= 32) as the persistent
    all-layers launch (pkv_decode_layers).  persistent_profile: the profiled
    eager step uses the persistent launch."""
    import model as M
    from kv_cache import KVCache

    parts = [int(v) for v in spec.split(":")]
    B, ctx = parts[0], parts[1]
    pitch = parts[2] if len(parts) > 2 else None  # table pitch in blocks (None: the default)
    m = M.Qwen2ForCausalLM().to(device, torch.bfloat16).eval()
    random_init_(m, 11)
    m.fuse_weights_()
    cache = KVCache(B * (ctx // 16 + 8) + 16, 16, device, torch.bfloat16, max_seqs=max(B, 16),
                    max_blocks_per_seq=pitch)
    seqs = [cache.alloc() for _ in range(B)]
    for s_ in seqs:  # a history of ctx tokens per row (pool contents irrelevant to timing)
        cache.ensure_capacity(s_, ctx)
    cache.advance(seqs, ctx)
    ids = torch.randint(0, 1000, (B, 1), device=device)
    res = {}
    import pagedkv

    policies = ("skinny", "cublas") + (("persistent",) if B <= pagedkv.LAYERS_MAX_ROWS else ())
    with torch.no_grad():
        for policy in policies:
            m.skinny_linears = policy != "cublas"
            m.persistent_decode = policy == "persistent"
            m.enable_decode_graphs(cache, max_batch=max(B, 16))
            for _ in range(3):
                m(ids, cache, seqs)
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(10):
                m(ids, cache, seqs)
            b.record()
            b.synchronize()
            res[policy] = round(a.elapsed_time(b) / 10, 4)
            m._graphs.clear()
        cache.check_errors()
        m.skinny_linears = True
        m.persistent_decode = persistent_profile and "persistent" in res
        if profile_range:
            m(ids, cache, seqs)
            torch.cuda.synchronize()
            torch.cuda.profiler.start()
            m(ids, cache, seqs)
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
    print(json.dumps({"diag": "decode_step", "rows": B, "ctx": ctx, "table_pitch": cache.table_pitch,
                      "graph_ms_skinny_policy": res["skinny"], "graph_ms_cublas": res["cublas"],
                      **({"graph_ms_persistent": res["persistent"]} if "persistent" in res else {}),
                      "skinny_rows": M.Qwen2ForCausalLM.skinny_rows}), flush=True)


def prefill_sweep(shapes, device):
    """Causal prefill attention per (B, T) on dense K/V, each kernel pinned by
    PKV_PREFILL_KERNEL: 20 launches captured in a CUDA graph, CUDA events
    around two replays.  Useful FLOPs = B * 4 * Hq * D * T(T+1)/2."""
    from kernels.fa2 import flash_attention

    peaks, src = measured_peaks()
    peak = float(peaks.get("bf16_tflops", 1590.0))
    saved = os.environ.get("PKV_PREFILL_KERNEL")
    try:
        for kern in ("one", "pair"):
            os.environ["PKV_PREFILL_KERNEL"] = kern
            for B, T in shapes:
                g = torch.Generator(device=device).manual_seed(B * 100000 + T)
                q = torch.randn(B, HQ, T, D, device=device, generator=g).to(torch.bfloat16)
                k = torch.randn(B, HKV, T, D, device=device, generator=g).to(torch.bfloat16)
                v = torch.randn(B, HKV, T, D, device=device, generator=g).to(torch.bfloat16)
                out = torch.empty_like(q)
                for _ in range(3):
                    flash_attention(q, k, v, True, None, out=out)
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for _ in range(20):
                        flash_attention(q, k, v, True, None, out=out)
                graph.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                graph.replay()
                graph.replay()
                e1.record()
                e1.synchronize()
                us = e0.elapsed_time(e1) / 40 * 1e3
                tf = B * 4 * HQ * D * T * (T + 1) / 2 / (us * 1e-6) / 1e12
                print(json.dumps({"diag": "prefill_sweep", "kernel": kern, "B": B, "T": T,
                                  "us_per_launch": round(us, 1), "tflops": round(tf, 1),
                                  "frac_of_bf16_peak": round(tf / peak, 3), "peak_source": src}),
                      flush=True)
                del graph, q, k, v, out
    finally:
        if saved is None:
            os.environ.pop("PKV_PREFILL_KERNEL", None)
        else:
            os.environ["PKV_PREFILL_KERNEL"] = saved


def prefill_step_diag(T, device, profile_range=False):
    """One-row prefill of T tokens from an empty cache (random-init model):
    CUDA-graph replay of the padded bucket (the engine's path) and eager;
    model FLOPs/s against the measured bf16 peak."""
    import model as M
    from kv_cache import KVCache

    m = M.Qwen2ForCausalLM().to(device, torch.bfloat16).eval()
    random_init_(m, 11)
    m.fuse_weights_()
    cache = KVCache(T // 16 + 64, 16, device, torch.bfloat16, max_seqs=16)
    ids = torch.randint(0, 1000, (1, T), device=device)
    nparams = sum(p.numel() for n_, p in m.named_parameters() if "embed" not in n_)
    flops = 2 * nparams * T + 4 * HQ * D * T * (T + 1) / 2 * L
    res = {}
    with torch.no_grad():
        for mode in ("graph", "eager"):
            if mode == "graph":
                m.enable_prefill_graphs(cache, max_len=max(T, 64))
            else:
                m._prefill_graphs.clear()
            ts = []
            for it in range(4):
                s_ = cache.alloc()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                m(ids, cache, [s_])
                b.record()
                b.synchronize()
                if it:
                    ts.append(a.elapsed_time(b))
                cache.free(s_)
            res[mode] = round(statistics.median(ts), 3)
        if profile_range:
            s_ = cache.alloc()
            torch.cuda.synchronize()
            torch.cuda.profiler.start()
            m(ids, cache, [s_])
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
            cache.free(s_)
    peaks, src = measured_peaks()
    pk = float(peaks.get("bf16_tflops", 1590.0))
    tf = flops / res["graph"] / 1e9
    print(json.dumps({"diag": "prefill_step", "T": T, "graph_ms": res["graph"],
                      "eager_ms": res["eager"], "model_tflops_graph": round(tf, 1),
                      "frac_of_bf16_peak": round(tf / pk, 3), "peak_source": src}), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    metric = "paged decode-attn HBM GB/s"
    default_c3 = (args.seqs, args.ctx_min, args.ctx_max, args.pool_gb, args.layers) == \
        (256, 2048, 8192, 150.0, L)
    config = {"workload": f"{'config3' if default_c3 else 'config3-shaped'}: {args.seqs} rows, "
                          f"ctx U[{args.ctx_min},{args.ctx_max}], ~{args.pool_gb:g} GB bf16 pool, "
                          f"{args.layers} layers of RoPE+append + paged decode per step",
              "seqs": args.seqs, "ctx_range": [args.ctx_min, args.ctx_max],
              "pool_gb": args.pool_gb, "layers": args.layers, "block_size": 16,
              "heads": [HQ, HKV, D], "l2": "inputs larger than L2 (KV read per step >> 126 MB)",
              "parallelism": f"replicas x{args.gpus} (request-sharded, no collective)"}

    if (args.linear_sweep or args.decode_step or args.prefill_step or args.prefill_sweep
            or args.linear_one or args.sample_one):
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        if args.sample_one:
            sample_one(args.sample_one, dev)
        if args.linear_one:
            linear_one(args.linear_one, dev)
        if args.prefill_sweep:
            prefill_sweep([tuple(int(v) for v in x.split("x")) for x in args.prefill_sweep.split(",")],
                          dev)
        if args.linear_sweep:
            linear_sweep([int(r) for r in args.linear_sweep.split(",")], dev)
        if args.decode_step:
            decode_step_diag(args.decode_step, dev, args.profile_range, args.persistent)
        if args.prefill_step:
            prefill_step_diag(args.prefill_step, dev, args.profile_range)
        return

    if args.impl == "reference":
        if rank != 0:
            return
        torch.set_num_threads(os.cpu_count() or 1)
        threads = torch.get_num_threads()
        # each timed step is a bounded sample: one pass of the CPU path over
        # --cpu-seqs rows and every layer
        cp = CpuPath(args)
        # the same rule as the cpu_baseline leg of our arm (CpuPath.measure),
        # at least the driver's warm-up and step counts
        per_step, spread = cp.measure(warmup=max(args.warmup, CPU_WARMUP),
                                      min_steps=max(args.steps, CPU_MIN_STEPS))
        val = cp.bytes / per_step / 1e9
        sample = cp.sample() + ", median of the timed steps"
        line = {"metric": metric, "value": round(val, 3), "unit": "GB/s", "impl": "reference",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(per_step * 1e3, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": config,
                "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": threads,
                                 "kind": "port", "sample": sample, "cpu": cpu_info(),
                                 "spread": spread},
                "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    if world > 1:
        torch.cuda.set_device(local)
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", torch.cuda.current_device())

    w = DecodeWorkload(args, dev)
    for _ in range(args.warmup):
        w.run_step()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(w.layers)] for _ in range(args.steps)]
    clocks = ClockSampler(dev)
    barrier()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record()
    for i in range(args.steps):
        w.run_step(evs[i])
    t_end.record()
    barrier()
    clk = clocks.stop()
    ms = t_start.elapsed_time(t_end) / args.steps
    kern_ms = statistics.mean(a.elapsed_time(b) for st in evs for a, b in st)
    step_bytes, bytes_decode, layers = w.step_bytes(), w.bytes_decode, w.layers
    ms_max, rate = replica_rate(step_bytes, ms, dev, world)
    total_bytes = step_bytes * world
    value = rate / 1e9

    e2e = None
    if not args.no_e2e:
        e_ms, h2d, d2h = e2e_run(w, max(2, args.steps // 2), max(3, args.warmup))
        e_max, e_rate = replica_rate(step_bytes, e_ms, dev, world)
        e2e = {"value": round(e_rate / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": round(e_max, 3),
               "note": "copies on a second stream, pipelined against the kernels; no "
                       "per-launch events here, while value's timed region records an "
                       "event pair around every decode launch for the roofline, which "
                       "stops consecutive launches from overlapping"}

    del w
    torch.cuda.empty_cache()
    fp8 = None
    if not args.no_fp8:
        fp8 = fp8_decode_run(args, dev, ms)
        # replicas: every rank ran the same step on its own pool
        f_ms, f_rate = replica_rate(fp8.pop("step_bytes"), fp8["ms_per_step"], dev, world)
        fp8.update({"value": round(f_rate / 1e9, 2), "ms_per_step": round(f_ms, 4),
                    "tokens_per_s": round(args.seqs * world / (f_ms * 1e-3), 1), "n_gpus": world})
    prefill = None if args.no_prefill else prefill_run(args, dev, seed=args.seed)
    engine = engine4 = engine4_mixed = engine4_chunked = None
    engine_mixed = None
    if not args.no_engine:
        # config 2 on every GPU (weak scaling: 16 chats per GPU), with the
        # reference's schedule and (--engine-mixed) with mixed ticks
        c2 = {}
        for mixed_min in [None] + ([args.engine_mixed] if args.engine_mixed > 0 else []):
            def leg(mixed_min=mixed_min):
                return engine_run(dev, label="config2", chats_total=args.engine_chats,
                                  prompt_range=args.engine_prompt, reply=args.engine_reply,
                                  blocks=args.engine_blocks, max_batch=max(args.engine_chats, 1),
                                  seed=args.seed + rank, mixed_min=mixed_min)
            if mixed_min is None:
                r = leg()
            else:
                r, err = opt_in_run(leg, dev, world)
                if err is not None:
                    c2[mixed_min] = {"error": err, "mixed_min_tokens": mixed_min}
                    continue
            wall_max, tok_rate = replica_rate(r["tokens"], r["wall_s"] * 1e3, dev, world)
            r["tok_s_all_gpus"] = round(tok_rate, 1)
            r["wall_s_max_over_gpus"] = round(wall_max / 1e3, 4)
            r["n_gpus"] = world
            r["scaling"] = "weak (each GPU serves its own chats)"
            r["per_rank"] = gather_ranks(rank_summary(rank, r), world)
            c2[mixed_min] = r
        engine = c2[None]
        engine_mixed = c2.get(args.engine_mixed) if args.engine_mixed > 0 else None
    if not args.no_engine4:
        # config 4: 1024 chats split round-robin over the GPUs (strong scaling)
        block_bytes = L * 2 * 16 * HKV * D * 2
        per_gpu = -(-args.engine4_chats // world)
        need = per_gpu * -(-(args.engine4_prompt[1] + args.engine4_reply + 1) // 16) + 64
        blocks = int(min(need, args.engine4_pool_gb * 1e9 // block_bytes))
        runs = {}
        mixed_on = args.engine4_mixed is not None and args.engine4_mixed > 0
        legs = [(None, None)] + ([(args.engine4_mixed, None)] if mixed_on else [])
        if mixed_on and args.engine4_chunk > 0:
            legs.append((args.engine4_mixed, args.engine4_chunk))
        for mixed_min, chunk in legs:
            def leg(mixed_min=mixed_min, chunk=chunk):
                return engine_run(dev, label="config4", chats_total=args.engine4_chats,
                                  prompt_range=args.engine4_prompt, reply=args.engine4_reply,
                                  blocks=blocks, max_batch=256, rank=rank, world=world,
                                  seed=args.seed, mixed_min=mixed_min, mixed_chunk=chunk)
            if mixed_min is None:
                r = leg()
            else:
                r, err = opt_in_run(leg, dev, world)
                if err is not None:
                    runs[(mixed_min, chunk)] = {"error": err, "mixed_min_tokens": mixed_min,
                                                **({"chunk_tokens": chunk} if chunk else {})}
                    continue
            if chunk:
                r["chunk_tokens"] = chunk
            toks_all = cross_rank(r["tokens"], torch.distributed.ReduceOp.SUM if world > 1 else None,
                                  dev, world)
            wall_max = cross_rank(r["wall_s"], torch.distributed.ReduceOp.MAX if world > 1 else None,
                                  dev, world)
            r.update({"tok_s_all_gpus": round(toks_all / wall_max, 1),
                      "tokens_all_gpus": int(toks_all), "wall_s_max_over_gpus": round(wall_max, 4),
                      "n_gpus": world,
                      "scaling": f"strong ({args.engine4_chats} chats split over the GPUs)",
                      "per_rank": gather_ranks(rank_summary(rank, r), world)})
            runs[(mixed_min, chunk)] = r
        engine4 = runs[(None, None)]
        engine4_mixed = runs.get((args.engine4_mixed, None)) if mixed_on else None
        engine4_chunked = (runs.get((args.engine4_mixed, args.engine4_chunk))
                           if mixed_on and args.engine4_chunk > 0 else None)
        if engine is not None and rank == 0 and world == 1 and not args.no_engine_cpu:
            torch.set_num_threads(os.cpu_count() or 1)
            engine["cpu_baseline"] = engine_cpu_sample()

    engine3 = None
    if not args.no_engine3 and world == 1:
        # config 3 is a one-GPU configuration: the 1-GPU run serves it
        engine3 = engine3_run(args, dev, seed=args.seed)

    peaks, src = measured_peaks()
    peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    achieved = bytes_decode / (kern_ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": src,
                "frac_of_nominal_8tbs": round(achieved / NOMINAL_HBM_GBS, 4),
                "kernel": "paged_decode_kernel", "bytes_per_launch": bytes_decode,
                "avg_launch_ms": round(kern_ms, 4),
                "traffic": None}
    prof = REPO / "profiles" / "decode_traffic.json"
    if prof.exists():
        # not measured in this run: ncu's dram bytes of one decode launch on a
        # smaller case, scaled to this launch by algorithmic bytes
        try:
            t = json.loads(prof.read_text())
            ratio = float(t["traffic_over_algorithmic"])
            roofline["traffic"] = int(round(ratio * bytes_decode))
            roofline["traffic_source"] = (
                f"ncu dram__bytes_read.sum + dram__bytes_write.sum on {t.get('case', 'a smaller case')}"
                f" ({t.get('source')}), not this run; traffic/algorithmic = {ratio} scaled to "
                f"this launch's algorithmic bytes")
        except Exception:
            pass

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        cp = CpuPath(args)
        per_step, spread = cp.measure()
        cpu = {"value": round(cp.bytes / per_step / 1e9, 3), "unit": "GB/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": cp.sample() + ", median of the timed steps", "cpu": cpu_info(),
               "spread": spread}

    if rank == 0:
        line = {"metric": metric, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic", "config": config, "roofline": roofline,
                "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
                "gpu_launches": args.steps * layers * 2,
                "kv_bytes_per_step": step_bytes, "prefill": prefill, "engine": engine, "engine_config4": engine4,
                **({"engine_config3": engine3} if engine3 is not None else {}),
                **({"fp8_decode": fp8} if fp8 is not None else {}),
                **({"engine_config4_mixed": engine4_mixed} if engine4_mixed is not None else {}),
                **({"engine_config4_chunked": engine4_chunked}
                   if engine4_chunked is not None else {}),
                **({"engine_mixed": engine_mixed} if engine_mixed is not None else {})}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
