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
    "pkv_paged_decode": (
        [_vp, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
         ctypes.c_float, _vp, _i64, _i64, _vp, ctypes.c_size_t, _vp, _vp], ctypes.c_int),
    "pkv_paged_prefill": (
        [_vp, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _i32, _i32, _i32, _i32,
         _i32, _i32, _i32, ctypes.c_float, _vp, _i64, _i64, _i64, _vp, _vp], ctypes.c_int),
    "pkv_add_rmsnorm": (
        [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _i32, _i32, ctypes.c_float, _vp],
        ctypes.c_int),
    "pkv_silu_mul": ([_vp, _i64, _vp, _i64, _i32, _i32, _vp], ctypes.c_int),
    "pkv_paged_decode_static_scratch": (
        [_vp, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
         ctypes.c_float, _vp, _i64, _i64, _vp, _vp], ctypes.c_int),
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


def default_scale(d: int = HEAD_DIM) -> float:
    """1/sqrt(d), as kernels/fa2.py:173 computes it."""
    return 1.0 / math.sqrt(d)
