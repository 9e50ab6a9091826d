"""ctypes binding of libpagedkv.so (the C ABI in include/pagedkv.h).

PyTorch only provides device memory and the current stream here: every call
passes raw pointers, element strides and `torch.cuda.current_stream()` to the
library, which validates, encodes TMA descriptors and launches its own
sm_100a kernels.  There is deliberately no fallback: if the library is
missing or cannot be loaded, `lib()` raises.
"""
from __future__ import annotations

import ctypes
import math
import threading
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libpagedkv.so"

PKV_OK = 0
PKV_DEVERR_BLOCK_ID = 1
PKV_DEVERR_POSITION = 2
PKV_DEVERR_TIMEOUT = 4

HEAD_DIM = 128
BLOCK_TOKENS = 16
LINEAR_MAX_ROWS = 256  # PKV_LINEAR_MAX_ROWS
LAYERS_MAX_ROWS = 32  # PKV_LAYERS_MAX_ROWS
LAYERS_MAX_LAYERS = 32  # PKV_LAYERS_MAX_LAYERS
W_ROWMAJOR, W_TILED, W_GATE_UP_PAIRED = 0, 1, 2  # PKV_W_* layouts

_c_i32p = ctypes.POINTER(ctypes.c_int32)
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32

# argument signatures, in header order
_SIGNATURES = {
    "pkv_version": ([], ctypes.c_int),
    "pkv_status_string": ([ctypes.c_int], ctypes.c_char_p),
    "pkv_last_error": ([], ctypes.c_char_p),
    "pkv_append_rope": (
        [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64,
         _vp, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _vp, _vp,
         _i32, _i32, _i32, _i32, _i32, _vp, _vp], ctypes.c_int),
    "pkv_decode_workspace_size": ([_i32, _i32, _i32, _i32], ctypes.c_size_t),
    "pkv_decode_plan": ([_i32, _i32, _i32, _i32, _vp], ctypes.c_int),
    "pkv_paged_decode": (
        [_vp, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
         ctypes.c_float, _vp, _i64, _i64, _vp, ctypes.c_size_t, _vp, _vp], ctypes.c_int),
    "pkv_paged_prefill": (
        [_vp, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _i32, _i32, _i32, _i32,
         _i32, _i32, _i32, ctypes.c_float, _vp, _i64, _i64, _i64, _vp, _vp], ctypes.c_int),
    "pkv_fp8_block_bytes": ([], ctypes.c_size_t),
    "pkv_append_rope_fp8": (
        [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64,
         _vp, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _vp,
         _i32, _i32, _i32, _i32, _i32, _vp, _vp], ctypes.c_int),
    "pkv_paged_decode_fp8": (
        [_vp, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
         ctypes.c_float, _vp, _i64, _i64, _vp, ctypes.c_size_t, _vp, _vp], ctypes.c_int),
    "pkv_fp8_dequant": (
        [_vp, _i64, _vp, _i64, _vp, _vp, _i32, _i32, _i32, _vp, _i64, _i64, _i64, _vp, _i64,
         _i64, _i64, _vp, _vp], ctypes.c_int),
    "pkv_add_rmsnorm": (
        [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _i32, _i32, ctypes.c_float, _vp],
        ctypes.c_int),
    "pkv_silu_mul": ([_vp, _i64, _vp, _i64, _i32, _i32, _vp], ctypes.c_int),
    "pkv_sample": (
        [_vp, _i64, _i32, _i32, _i32, ctypes.c_float, ctypes.c_uint64, ctypes.c_uint64, _vp, _vp],
        ctypes.c_int),
    "pkv_paged_decode_static_scratch": (
        [_vp, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
         ctypes.c_float, _vp, _i64, _i64, _vp, _vp], ctypes.c_int),
    "pkv_linear_workspace_size": ([_i32, _i32, _i32], ctypes.c_size_t),
    "pkv_linear_pair_gate_up": ([_vp, _i64, _i32, _i32, _vp, _vp], ctypes.c_int),
    "pkv_linear_pack_weight": ([_vp, _i64, _i32, _i32, _vp, _vp], ctypes.c_int),
    "pkv_linear": (
        [_vp, _i64, _vp, _i64, _i32, _vp, _i32, _i32, _i32, _vp, _i64, _vp, ctypes.c_size_t, _vp,
         _vp], ctypes.c_int),
    "pkv_linear_add_rmsnorm": (
        [_vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _i64, _vp, ctypes.c_float,
         _vp, _i64, _vp, ctypes.c_size_t, _vp, _vp], ctypes.c_int),
    "pkv_linear_silu_mul": (
        [_vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, _vp, _i64, _vp, ctypes.c_size_t, _vp, _vp],
        ctypes.c_int),
    "pkv_linear_rope_append": (
        [_vp, _i64, _vp, _i64, _i32, _vp, _i32, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _vp,
         _i64, _vp, _i64, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp, ctypes.c_size_t, _vp,
         _vp], ctypes.c_int),
    "pkv_decode_layers_workspace_size": ([_i32], ctypes.c_size_t),
    "pkv_decode_layers": (
        [_vp, _i32, _vp, _vp, _vp, _i32, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _i64,
         ctypes.c_float, _vp, ctypes.c_size_t, _vp, _vp], ctypes.c_int),
    "pkv_dense_attention": (
        [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i32, _i32,
         _i32, _i32, _i32, _i32, _i32, ctypes.c_float, _vp, _i64, _i64, _i64, _vp,
         ctypes.c_size_t, _vp, _vp], ctypes.c_int),
}

_lib = None
_lib_lock = threading.Lock()


class PagedKVError(RuntimeError):
    """A libpagedkv call returned a nonzero pkv_status."""


def lib() -> ctypes.CDLL:
    """Load libpagedkv.so (built in-tree by pagedkv_build.py); raise if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python {HERE / 'pagedkv_build.py'}` "
                    "(there is no non-CUDA fallback)")
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (args, res) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = args
                fn.restype = res
            _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def _check(status: int, what: str) -> None:
    if status != PKV_OK:
        L = lib()
        raise PagedKVError(f"{what}: {L.pkv_status_string(status).decode()} "
                           f"({L.pkv_last_error().decode()})")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ---------------------------------------------------------------- workspace
_workspaces: dict[int, torch.Tensor] = {}
_retired_workspaces: list[torch.Tensor] = []  # outgrown buffers stay alive (captured graphs)


def decode_plan(batch: int, num_q_heads: int, num_kv_heads: int, max_kv_len: int) -> dict:
    """The split-K plan pkv_paged_decode uses for these sizes (host arithmetic)."""
    out = (ctypes.c_int32 * 4)()
    _check(lib().pkv_decode_plan(batch, num_q_heads, num_kv_heads, max_kv_len, out), "decode_plan")
    return {"blocks_per_part": out[0], "min_blocks_per_part": out[1], "max_parts": out[2],
            "sub_groups": out[3]}


def decode_workspace(batch: int, num_q_heads: int, num_kv_heads: int, max_kv_len: int,
                     device: torch.device) -> torch.Tensor | None:
    """Grow-only, zero-initialised split-K scratch for `device` (None if unneeded).

    The kernel re-arms its counters to zero, so the buffer only has to be
    zeroed when it is (re)allocated.  Calls on one device share it, so they
    must be ordered on one stream.
    """
    need = lib().pkv_decode_workspace_size(batch, num_q_heads, num_kv_heads, max_kv_len)
    if need == 0:
        return None
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < need:
        if ws is not None:
            _retired_workspaces.append(ws)
        size = max(need, 2 * (ws.numel() if ws is not None else 0))
        ws = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
        _workspaces[idx] = ws
    return ws


_lin_workspaces: dict[int, torch.Tensor] = {}


def linear_workspace(rows: int, n: int, k: int, device: torch.device) -> torch.Tensor:
    """Grow-only scratch of the fused skinny linear entries for `device` (their
    bf16 GEMM output; the same retire-but-keep-alive rule as decode_workspace)."""
    need = max(int(lib().pkv_linear_workspace_size(rows, n, k)), 16)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _lin_workspaces.get(idx)
    if ws is None or ws.numel() < need:
        if ws is not None:
            _retired_workspaces.append(ws)
        size = max(need, 2 * (ws.numel() if ws is not None else 0), 1 << 20)
        ws = torch.empty(size, dtype=torch.uint8, device=torch.device("cuda", idx))
        _lin_workspaces[idx] = ws
    return ws


# ---------------------------------------------------------------- entry points
def append_rope(q: torch.Tensor | None, k: torch.Tensor, v: torch.Tensor,
                rope_cos: torch.Tensor | None, rope_sin: torch.Tensor | None,
                q_out: torch.Tensor | None, k_plane: torch.Tensor, v_plane: torch.Tensor,
                tables: torch.Tensor, rows: torch.Tensor | None, starts: torch.Tensor,
                err: torch.Tensor | None = None, q_lens: torch.Tensor | None = None) -> None:
    """pkv_append_rope.  q/k/v/q_out are [B, H, T, 128] bf16 views; the pool
    planes are [num_slots, Hkv, 128] bf16; tables [rows, pitch] int32."""
    B, Hkv, T, D = k.shape
    Hq = q.shape[1] if q is not None else Hkv
    qs = q.stride() if q is not None else (0, 0, 0, 1)
    qos = q_out.stride() if q_out is not None else (0, 0, 0, 1)
    st = lib().pkv_append_rope(
        _ptr(q), qs[0], qs[1], qs[2], _ptr(k), k.stride(0), k.stride(1), k.stride(2),
        _ptr(v), v.stride(0), v.stride(1), v.stride(2),
        _ptr(rope_cos), _ptr(rope_sin), rope_cos.shape[0] if rope_cos is not None else 0,
        _ptr(q_out), qos[0], qos[1], qos[2], _ptr(k_plane), _ptr(v_plane), k_plane.shape[0],
        _ptr(tables), tables.stride(0), _ptr(rows), _ptr(starts), _ptr(q_lens),
        B, Hq, Hkv, T, D, _ptr(err), _stream(k.device))
    _check(st, "pkv_append_rope")


def paged_decode(q: torch.Tensor, k_plane: torch.Tensor, v_plane: torch.Tensor,
                 tables: torch.Tensor, rows: torch.Tensor | None, kv_lens: torch.Tensor,
                 max_kv_len: int, out: torch.Tensor, sm_scale: float,
                 num_kv_heads: int, err: torch.Tensor | None = None) -> None:
    """pkv_paged_decode.  q, out: [B, Hq, 128] (any strides, dim contiguous)."""
    B, Hq, D = q.shape
    ws = decode_workspace(B, Hq, num_kv_heads, max_kv_len, q.device)
    st = lib().pkv_paged_decode(
        _ptr(q), q.stride(0), q.stride(1), _ptr(k_plane), _ptr(v_plane), k_plane.shape[0],
        _ptr(tables), tables.stride(0), _ptr(rows), _ptr(kv_lens), max_kv_len, B, Hq,
        num_kv_heads, D, sm_scale, _ptr(out), out.stride(0), out.stride(1),
        _ptr(ws), ws.numel() if ws is not None else 0, _ptr(err), _stream(q.device))
    _check(st, "pkv_paged_decode")


# ---------------------------------------------------------------- FP8 pool
def fp8_block_bytes() -> int:
    """Bytes of one (16-token block, KV head) chunk of the FP8 pool."""
    return int(lib().pkv_fp8_block_bytes())


def append_rope_fp8(q: torch.Tensor | None, k: torch.Tensor, v: torch.Tensor,
                    rope_cos: torch.Tensor | None, rope_sin: torch.Tensor | None,
                    q_out: torch.Tensor | None, pool8: torch.Tensor, tables: torch.Tensor,
                    rows: torch.Tensor | None, starts: torch.Tensor,
                    err: torch.Tensor | None = None, q_lens: torch.Tensor | None = None) -> None:
    """pkv_append_rope_fp8.  q/k/v [B, H, T, 128]; pool8 uint8 [blocks, Hkv, chunk]."""
    B, Hkv, T, D = k.shape
    Hq = q.shape[1] if q is not None else Hkv
    qs = q.stride() if q is not None else (0, 0, 0, 1)
    qos = q_out.stride() if q_out is not None else (0, 0, 0, 1)
    st = lib().pkv_append_rope_fp8(
        _ptr(q), qs[0], qs[1], qs[2], _ptr(k), k.stride(0), k.stride(1), k.stride(2),
        _ptr(v), v.stride(0), v.stride(1), v.stride(2),
        _ptr(rope_cos), _ptr(rope_sin), rope_cos.shape[0] if rope_cos is not None else 0,
        _ptr(q_out), qos[0], qos[1], qos[2], _ptr(pool8), pool8.shape[0],
        _ptr(tables), tables.stride(0), _ptr(rows), _ptr(starts), _ptr(q_lens),
        B, Hq, Hkv, T, D, _ptr(err), _stream(k.device))
    _check(st, "pkv_append_rope_fp8")


def paged_decode_fp8(q: torch.Tensor, pool8: torch.Tensor, tables: torch.Tensor,
                     rows: torch.Tensor | None, kv_lens: torch.Tensor, max_kv_len: int,
                     out: torch.Tensor, sm_scale: float, err: torch.Tensor | None = None) -> None:
    """pkv_paged_decode_fp8.  q, out: [B, Hq, 128]; pool8 uint8 [blocks, Hkv, chunk]."""
    B, Hq, D = q.shape
    Hkv = pool8.shape[1]
    ws = decode_workspace(B, Hq, Hkv, max_kv_len, q.device)
    st = lib().pkv_paged_decode_fp8(
        _ptr(q), q.stride(0), q.stride(1), _ptr(pool8), pool8.shape[0],
        _ptr(tables), tables.stride(0), _ptr(rows), _ptr(kv_lens), max_kv_len, B, Hq,
        Hkv, D, sm_scale, _ptr(out), out.stride(0), out.stride(1),
        _ptr(ws), ws.numel() if ws is not None else 0, _ptr(err), _stream(q.device))
    _check(st, "pkv_paged_decode_fp8")


def fp8_dequant(pool8: torch.Tensor, tables: torch.Tensor, rows: torch.Tensor | None,
                kv_lens: torch.Tensor, seq_len: int, k_out: torch.Tensor, v_out: torch.Tensor,
                err: torch.Tensor | None = None) -> None:
    """pkv_fp8_dequant into dense bf16 k_out / v_out [B, Hkv, seq_len, 128]."""
    B = k_out.shape[0]
    st = lib().pkv_fp8_dequant(
        _ptr(pool8), pool8.shape[0], _ptr(tables), tables.stride(0), _ptr(rows), _ptr(kv_lens),
        B, pool8.shape[1], seq_len, _ptr(k_out), k_out.stride(0), k_out.stride(1),
        k_out.stride(2), _ptr(v_out), v_out.stride(0), v_out.stride(1), v_out.stride(2),
        _ptr(err), _stream(k_out.device))
    _check(st, "pkv_fp8_dequant")


def paged_prefill(q: torch.Tensor, k_plane: torch.Tensor, v_plane: torch.Tensor,
                  tables: torch.Tensor, rows: torch.Tensor | None, kv_lens: torch.Tensor,
                  max_kv_len: int, out: torch.Tensor, causal: bool, sm_scale: float,
                  num_kv_heads: int, err: torch.Tensor | None = None,
                  q_lens: torch.Tensor | None = None) -> None:
    """pkv_paged_prefill.  q, out: [B, Hq, T, 128]; q_lens: right-padded rows."""
    B, Hq, T, D = q.shape
    st = lib().pkv_paged_prefill(
        _ptr(q), q.stride(0), q.stride(1), q.stride(2), _ptr(k_plane), _ptr(v_plane),
        k_plane.shape[0], _ptr(tables), tables.stride(0), _ptr(rows), _ptr(kv_lens),
        _ptr(q_lens), max_kv_len,
        B, T, Hq, num_kv_heads, D, int(causal), sm_scale, _ptr(out), out.stride(0),
        out.stride(1), out.stride(2), _ptr(err), _stream(q.device))
    _check(st, "pkv_paged_prefill")


def dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_lens: torch.Tensor,
                    out: torch.Tensor, causal: bool, sm_scale: float,
                    err: torch.Tensor | None = None) -> None:
    """pkv_dense_attention.  q, out: [B, Hq, T, 128]; k, v: [B, Hkv, S, 128]."""
    B, Hq, T, D = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    ws = decode_workspace(B, Hq, Hkv, S, q.device) if T == 1 else None
    st = lib().pkv_dense_attention(
        _ptr(q), q.stride(0), q.stride(1), q.stride(2), _ptr(k), k.stride(0), k.stride(1),
        k.stride(2), _ptr(v), v.stride(0), v.stride(1), v.stride(2), _ptr(kv_lens), B, T, S,
        Hq, Hkv, D, int(causal), sm_scale, _ptr(out), out.stride(0), out.stride(1),
        out.stride(2), _ptr(ws), ws.numel() if ws is not None else 0, _ptr(err),
        _stream(q.device))
    _check(st, "pkv_dense_attention")


def add_rmsnorm(a: torch.Tensor, resid: torch.Tensor | None, weight: torch.Tensor,
                eps: float, resid_out: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """pkv_add_rmsnorm over the last dim of 2-D row views (any row stride)."""
    rows, dim = a.shape
    if out is None:
        out = torch.empty(rows, dim, dtype=a.dtype, device=a.device)
    st = lib().pkv_add_rmsnorm(
        _ptr(a), a.stride(0), _ptr(resid), resid.stride(0) if resid is not None else 0,
        _ptr(resid_out), resid_out.stride(0) if resid_out is not None else 0, _ptr(weight),
        _ptr(out), out.stride(0), rows, dim, eps, _stream(a.device))
    _check(st, "pkv_add_rmsnorm")
    return out


def silu_mul(gu: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """pkv_silu_mul: gu [rows, 2*inter] -> [rows, inter]."""
    rows, two_inter = gu.shape
    inter = two_inter // 2
    if out is None:
        out = torch.empty(rows, inter, dtype=gu.dtype, device=gu.device)
    st = lib().pkv_silu_mul(_ptr(gu), gu.stride(0), _ptr(out), out.stride(0), rows, inter,
                            _stream(gu.device))
    _check(st, "pkv_silu_mul")
    return out


def sample(logits: torch.Tensor, temperature: float = 1.0, *, seed: int | None = None,
           call: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """pkv_sample: one token id per row of logits [rows, vocab] (bf16 or f32,
    CUDA) drawn from softmax(logits / temperature) -> int32 [rows] on the same
    device; -1 marks a row without a finite logit.

    Without a seed, each call draws its 63-bit key from torch's default
    (CPU) generator, so after torch.manual_seed(s) a run repeats its draws
    call for call, as torch.multinomial's would."""
    assert logits.is_cuda and logits.dim() == 2, "logits must be a 2-D CUDA tensor"
    if logits.dtype == torch.bfloat16:
        dtype = 0
    elif logits.dtype == torch.float32:
        dtype = 1
    else:
        raise AssertionError(f"logits must be bf16 or float32, got {logits.dtype}")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    if seed is None:
        seed = int(torch.randint(1 << 62, (1,)).item())
    rows, vocab = logits.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    st = lib().pkv_sample(_ptr(logits), logits.stride(0), rows, vocab, dtype, float(temperature),
                          seed & 0xFFFFFFFFFFFFFFFF, call & 0xFFFFFFFFFFFFFFFF, _ptr(out),
                          _stream(logits.device))
    _check(st, "pkv_sample")
    return out


class TiledWeight:
    """A weight w[n, k] packed into the PKV_W_TILED layout ([n/128][k/64][128][64]),
    so the skinny GEMM streams it as contiguous 16 KiB runs.  `shape` is the
    logical [n, k]."""

    def __init__(self, w: torch.Tensor):
        n, k = w.shape
        self.shape = torch.Size((n, k))
        self.data = torch.empty(n * k, dtype=w.dtype, device=w.device)
        st = lib().pkv_linear_pack_weight(_ptr(w), w.stride(0), n, k, _ptr(self.data),
                                          _stream(w.device))
        _check(st, "pkv_linear_pack_weight")


class PairedGateUp:
    """A merged gate/up weight [2*inter, k] reordered into the
    PKV_W_GATE_UP_PAIRED layout (each 128-row tile: 64 gate rows, then their
    64 up rows), for linear_silu_mul with SwiGLU in the GEMM's epilogue."""

    def __init__(self, w_gate_up: torch.Tensor):
        n, k = w_gate_up.shape
        self.shape = torch.Size((n, k))
        self.data = torch.empty(n, k, dtype=w_gate_up.dtype, device=w_gate_up.device)
        st = lib().pkv_linear_pair_gate_up(_ptr(w_gate_up), w_gate_up.stride(0), n // 2, k,
                                           _ptr(self.data), _stream(w_gate_up.device))
        _check(st, "pkv_linear_pair_gate_up")


def _w_args(w) -> tuple[int, int, int]:
    """(pointer, ldw, layout) of a plain row-major weight, a TiledWeight or a
    PairedGateUp."""
    if isinstance(w, TiledWeight):
        return w.data.data_ptr(), w.shape[1], W_TILED
    if isinstance(w, PairedGateUp):
        return w.data.data_ptr(), w.shape[1], W_GATE_UP_PAIRED
    return w.data_ptr(), w.stride(0), W_ROWMAJOR


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
           out: torch.Tensor | None = None, err: torch.Tensor | None = None) -> torch.Tensor:
    """pkv_linear: x [rows, k] . w[n, k]^T (+ bias) -> [rows, n] bf16, rows <= 256."""
    rows, k = x.shape
    n = w.shape[0]
    if out is None:
        out = torch.empty(rows, n, dtype=x.dtype, device=x.device)
    wp, ldw, lay = _w_args(w)
    st = lib().pkv_linear(_ptr(x), x.stride(0), wp, ldw, lay, _ptr(bias), rows, n, k,
                          _ptr(out), out.stride(0), None, 0, _ptr(err), _stream(x.device))
    _check(st, "pkv_linear")
    return out


def linear_add_rmsnorm(x: torch.Tensor, w: torch.Tensor, resid: torch.Tensor | None,
                       weight: torch.Tensor, eps: float, resid_out: torch.Tensor | None = None,
                       out: torch.Tensor | None = None,
                       err: torch.Tensor | None = None) -> torch.Tensor:
    """pkv_linear_add_rmsnorm: add_rmsnorm(x . w^T, resid, weight) in two launches."""
    rows, k = x.shape
    n = w.shape[0]
    if out is None:
        out = torch.empty(rows, n, dtype=x.dtype, device=x.device)
    ws = linear_workspace(rows, n, k, x.device)
    wp, ldw, lay = _w_args(w)
    st = lib().pkv_linear_add_rmsnorm(
        _ptr(x), x.stride(0), wp, ldw, lay, rows, n, k,
        _ptr(resid), resid.stride(0) if resid is not None else 0,
        _ptr(resid_out), resid_out.stride(0) if resid_out is not None else 0,
        _ptr(weight), eps, _ptr(out), out.stride(0), _ptr(ws), ws.numel(), _ptr(err),
        _stream(x.device))
    _check(st, "pkv_linear_add_rmsnorm")
    return out


def linear_silu_mul(x: torch.Tensor, w_gate_up: torch.Tensor, out: torch.Tensor | None = None,
                    err: torch.Tensor | None = None) -> torch.Tensor:
    """pkv_linear_silu_mul: silu_mul(x . w_gate_up^T) -> [rows, inter]."""
    rows, k = x.shape
    inter = w_gate_up.shape[0] // 2
    if out is None:
        out = torch.empty(rows, inter, dtype=x.dtype, device=x.device)
    wp, ldw, lay = _w_args(w_gate_up)
    # the paired layout finishes SwiGLU in the GEMM: no intermediate
    ws = linear_workspace(rows, 2 * inter, k, x.device) if lay != W_GATE_UP_PAIRED else None
    st = lib().pkv_linear_silu_mul(_ptr(x), x.stride(0), wp, ldw, lay, rows, inter, k,
                                   _ptr(out), out.stride(0), _ptr(ws),
                                   ws.numel() if ws is not None else 0, _ptr(err),
                                   _stream(x.device))
    _check(st, "pkv_linear_silu_mul")
    return out


def linear_rope_append(x: torch.Tensor, w_qkv: torch.Tensor, bias: torch.Tensor | None,
                       rope_cos: torch.Tensor, rope_sin: torch.Tensor, q_out: torch.Tensor,
                       k_plane: torch.Tensor, v_plane: torch.Tensor, tables: torch.Tensor,
                       rows: torch.Tensor | None, starts: torch.Tensor, num_kv_heads: int,
                       err: torch.Tensor | None = None,
                       q_lens: torch.Tensor | None = None) -> None:
    """pkv_linear_rope_append: the merged q/k/v GEMM (+ bias) then append_rope.
    x: [B*T, k] rows in (b, t) order; q_out: [B, Hq, T, 128] view."""
    B, Hq, T, D = q_out.shape
    n_rows, k = x.shape
    n = w_qkv.shape[0]
    ws = linear_workspace(n_rows, n, k, x.device)
    qs = q_out.stride()
    wp, ldw, lay = _w_args(w_qkv)
    st = lib().pkv_linear_rope_append(
        _ptr(x), x.stride(0), wp, ldw, lay, _ptr(bias), k, _ptr(rope_cos),
        _ptr(rope_sin), rope_cos.shape[0], _ptr(q_out), qs[0], qs[1], qs[2], _ptr(k_plane),
        _ptr(v_plane), k_plane.shape[0], _ptr(tables), tables.stride(0), _ptr(rows),
        _ptr(starts), _ptr(q_lens), B, Hq, num_kv_heads, T, D, _ptr(ws), ws.numel(), _ptr(err),
        _stream(x.device))
    _check(st, "pkv_linear_rope_append")


def default_scale(d: int = HEAD_DIM) -> float:
    """1/sqrt(d), as kernels/fa2.py:173 computes it."""
    return 1.0 / math.sqrt(d)


# ---------------------------------------------------------------- decode layers
_LAYER_FIELDS = ("qkv_w", "qkv_b", "o_w", "post_norm_w", "gate_up_w", "down_w", "in_norm_w")


class _LayerWeightsC(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in _LAYER_FIELDS]


class LayerTable:
    """The host array of pkv_layer_weights that pkv_decode_layers reads: one
    entry per decoder layer (tensors keyed by the struct's field names:
    qkv_w, qkv_b, o_w, post_norm_w, gate_up_w in the PKV_W_GATE_UP_PAIRED
    layout, down_w, in_norm_w).  Keeps the tensors alive."""

    def __init__(self, layers: list[dict]):
        if not 0 < len(layers) <= LAYERS_MAX_LAYERS:
            raise ValueError(f"1..{LAYERS_MAX_LAYERS} layers supported, got {len(layers)}")
        self.tensors = layers
        self.arr = (_LayerWeightsC * len(layers))()
        for i, d in enumerate(layers):
            for name in _LAYER_FIELDS:
                t = d.get(name)
                if t is not None and not t.is_contiguous():
                    raise ValueError(f"layer {i}: {name} must be contiguous")
                setattr(self.arr[i], name, None if t is None else t.data_ptr())

    def __len__(self) -> int:
        return len(self.tensors)


_layers_ws: dict[int, torch.Tensor] = {}


def decode_layers_workspace(device: torch.device) -> torch.Tensor:
    """Per-device scratch of pkv_decode_layers, sized for PKV_LAYERS_MAX_ROWS
    rows so one buffer serves every step (and the graphs that captured it)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _layers_ws.get(idx)
    if ws is None:
        need = int(lib().pkv_decode_layers_workspace_size(LAYERS_MAX_ROWS))
        if need <= 0:
            raise PagedKVError("pkv_decode_layers_workspace_size: no plan for this device")
        ws = torch.empty(need, dtype=torch.uint8, device=device)
        _layers_ws[idx] = ws
    return ws


def decode_layers(table: LayerTable, h0: torch.Tensor, xs: torch.Tensor, m_out: torch.Tensor,
                  kv_pool: torch.Tensor, tables: torch.Tensor, rows: torch.Tensor | None,
                  starts: torch.Tensor, rope_cos: torch.Tensor, rope_sin: torch.Tensor,
                  eps: float, err: torch.Tensor | None = None) -> torch.Tensor:
    """pkv_decode_layers: every decoder layer of a one-token-per-row step in
    one launch.  h0, xs, m_out: [rows, 1536] bf16 (xs updated in place, the
    last layer's MLP output into m_out); kv_pool: the cache's whole
    [layers, 2, slots, 2, 128] buffer."""
    n = h0.shape[0]
    ws = decode_layers_workspace(h0.device)
    st = lib().pkv_decode_layers(
        ctypes.cast(table.arr, _vp), len(table), _ptr(h0), _ptr(xs), _ptr(m_out), n,
        _ptr(kv_pool), kv_pool.shape[2], _ptr(tables), tables.stride(0), _ptr(rows),
        _ptr(starts), _ptr(rope_cos), _ptr(rope_sin), rope_cos.shape[0], eps, _ptr(ws),
        ws.numel(), _ptr(err), _stream(h0.device))
    _check(st, "pkv_decode_layers")
    return m_out
