// Fused RoPE + K/V append into the paged pool (sm_100a).
//
// Reference behaviour (bit-exact):
//   model.py:151-155  cos/sin = cat(freqs, freqs).cos()/.sin() -> activation dtype
//   model.py:58-65    rotate_half(x) = cat(-x2, x1);
//                     x' = (x * cos) + (rotate_half(x) * sin)  -- each torch op on
//                     bf16 tensors rounds its fp32 result to bf16 (RNE)
//   kv_cache.py:108-115  index_copy_ of k, v into buf[layer, 0|1][slot]
//   kv_cache.py:88-91    slot = table[p // 16] * 16 + p % 16
// The cos/sin rows come from a table indexed by position, so the caller can
// build it with exactly the reference's fp32 formula.
//
// One warp per (row, step token, head-of-{q, k, v}); lane l owns dims
// {2l, 2l+1} and their rotation partners {64+2l, 64+2l+1}.
#include <cuda_fp8.h>

#include "pkv_device.cuh"
#include "pkv_kernels.h"

namespace pkv {
namespace {

__device__ __forceinline__ float bf(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 rn(float x) { return __float2bfloat16_rn(x); }

// bf16(bf16(x*c) + bf16(r*s)) with the multiplies and the add each rounded
// separately (no FMA contraction), as three separate torch ops compute it.
__device__ __forceinline__ __nv_bfloat16 rope1(__nv_bfloat16 x, __nv_bfloat16 c, __nv_bfloat16 r,
                                               __nv_bfloat16 s) {
  const __nv_bfloat16 xc = rn(__fmul_rn(bf(x), bf(c)));
  const __nv_bfloat16 rs = rn(__fmul_rn(bf(r), bf(s)));
  return rn(__fadd_rn(bf(xc), bf(rs)));
}

__global__ void __launch_bounds__(256) append_rope_kernel(const AppendLaunch a, int32_t num_blocks) {
  pdl_trigger();
  pdl_wait();
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const int64_t item = gid >> 5;
  const int per_tok = (a.q_out ? a.num_q_heads : 0) + 2 * a.num_kv_heads;
  const int64_t total = static_cast<int64_t>(a.batch) * a.seq_len_q * per_tok;
  if (item >= total) return;
  const int which = static_cast<int>(item % per_tok);
  const int64_t bt = item / per_tok;
  const int tt = static_cast<int>(bt % a.seq_len_q);
  const int b = static_cast<int>(bt / a.seq_len_q);
  const DevErr err{a.err};

  const int start = a.starts[b];
  if (start < 0) return;  // inactive (padding) row: nothing to rotate or store
  if (a.q_lens && tt >= a.q_lens[b]) return;  // right padding of a shorter row
  const int pos = start + tt;
  const bool rope = a.rope_cos != nullptr;
  const int nq = a.q_out ? a.num_q_heads : 0;

  // source row and destination row for this item
  const __nv_bfloat16* src;
  __nv_bfloat16* dst;
  bool do_rope = rope;
  if (which < nq) {
    src = static_cast<const __nv_bfloat16*>(a.q) + b * a.q_sb + which * a.q_sh + tt * a.q_st;
    dst = static_cast<__nv_bfloat16*>(a.q_out) + b * a.qo_sb + which * a.qo_sh + tt * a.qo_st;
  } else {
    const bool is_k = which < nq + a.num_kv_heads;
    const int h = is_k ? which - nq : which - nq - a.num_kv_heads;
    // destination slot through the block table
    const int row = a.rows ? a.rows[b] : b;
    const int64_t bi = pos >> 4;
    if (pos < 0 || bi >= a.pitch) {
      if (lane == 0) err.raise(PKV_DEVERR_POSITION);
      return;
    }
    const int blk = a.tables[static_cast<int64_t>(row) * a.pitch + bi];
    if (blk < 0 || blk >= num_blocks) {
      if (lane == 0) err.raise(PKV_DEVERR_BLOCK_ID);
      return;
    }
    const int64_t slot = static_cast<int64_t>(blk) * kBlockTokens + (pos & 15);
    if (is_k) {
      src = static_cast<const __nv_bfloat16*>(a.k) + b * a.k_sb + h * a.k_sh + tt * a.k_st;
      dst = static_cast<__nv_bfloat16*>(a.k_pool) + (slot * a.num_kv_heads + h) * kHeadDim;
    } else {
      src = static_cast<const __nv_bfloat16*>(a.v) + b * a.v_sb + h * a.v_sh + tt * a.v_st;
      dst = static_cast<__nv_bfloat16*>(a.v_pool) + (slot * a.num_kv_heads + h) * kHeadDim;
      do_rope = false;
    }
  }

  const int d = 2 * lane;
  const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(src + d);
  const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(src + 64 + d);
  if (!do_rope) {
    *reinterpret_cast<__nv_bfloat162*>(dst + d) = lo;
    *reinterpret_cast<__nv_bfloat162*>(dst + 64 + d) = hi;
    return;
  }
  if (pos < 0 || pos >= a.rope_rows) {
    if (lane == 0) err.raise(PKV_DEVERR_POSITION);
    return;
  }
  const __nv_bfloat16* cr = static_cast<const __nv_bfloat16*>(a.rope_cos) + static_cast<int64_t>(pos) * kHeadDim;
  const __nv_bfloat16* sr = static_cast<const __nv_bfloat16*>(a.rope_sin) + static_cast<int64_t>(pos) * kHeadDim;
  const __nv_bfloat162 clo = *reinterpret_cast<const __nv_bfloat162*>(cr + d);
  const __nv_bfloat162 chi = *reinterpret_cast<const __nv_bfloat162*>(cr + 64 + d);
  const __nv_bfloat162 slo = *reinterpret_cast<const __nv_bfloat162*>(sr + d);
  const __nv_bfloat162 shi = *reinterpret_cast<const __nv_bfloat162*>(sr + 64 + d);
  // first half: x*cos + (-x2)*sin ; second half: x*cos + x1*sin
  __nv_bfloat162 olo, ohi;
  olo.x = rope1(lo.x, clo.x, __hneg(hi.x), slo.x);
  olo.y = rope1(lo.y, clo.y, __hneg(hi.y), slo.y);
  ohi.x = rope1(hi.x, chi.x, lo.x, shi.x);
  ohi.y = rope1(hi.y, chi.y, lo.y, shi.y);
  *reinterpret_cast<__nv_bfloat162*>(dst + d) = olo;
  *reinterpret_cast<__nv_bfloat162*>(dst + 64 + d) = ohi;
}

// One warp per (row, step token, chunk of heads): 16 lanes per head, two
// heads per pass; lane l owns dims 4l..4l+3 and their rotation partners
// 64+4l..64+4l+3 (8-byte accesses).  The token's cos/sin and pool slot are
// looked up once per warp.  A decode step has few tokens, so its heads are
// split over up to `chunks` warps (one pass each at most) instead of one
// warp walking all of them; and a warp issues the loads of up to kVecPass
// passes before any of their stores, so the passes' memory latencies
// overlap.  Same arithmetic per element as append_rope_kernel.
constexpr int kVecPass = 4;

__global__ void __launch_bounds__(256) append_rope_vec_kernel(const AppendLaunch a,
                                                              int32_t num_blocks, int32_t chunks) {
  pdl_trigger();
  pdl_wait();
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t tok = w / chunks;
  const int chunk = static_cast<int>(w % chunks);
  if (tok >= static_cast<int64_t>(a.batch) * a.seq_len_q) return;
  const int tt = static_cast<int>(tok % a.seq_len_q);
  const int b = static_cast<int>(tok / a.seq_len_q);
  const DevErr err{a.err};
  const int start = a.starts[b];
  if (start < 0) return;                      // inactive (padding) row
  if (a.q_lens && tt >= a.q_lens[b]) return;  // right padding of a shorter row
  const int pos = start + tt;
  const bool rope = a.rope_cos != nullptr;
  const int nq = a.q_out ? a.num_q_heads : 0;
  const int per_tok = nq + 2 * a.num_kv_heads;
  const int passes = (per_tok + 1) >> 1;
  const int per_chunk = (passes + chunks - 1) / chunks;
  const int p_begin = chunk * per_chunk, p_end = min(passes, p_begin + per_chunk);
  if (p_begin >= p_end) return;
  const int d = 4 * (lane & 15);
  // errors are reported by the warp of chunk 0 only (one report per token)
  const bool reporter = lane == 0 && chunk == 0;

  // pool slot of this token (k and v heads), checked once
  int64_t slot = -1;
  {
    const int row = a.rows ? a.rows[b] : b;
    const int64_t bi = pos >> 4;
    if (pos < 0 || bi >= a.pitch) {
      if (reporter) err.raise(PKV_DEVERR_POSITION);
    } else {
      const int blk = a.tables[static_cast<int64_t>(row) * a.pitch + bi];
      if (blk < 0 || blk >= num_blocks) {
        if (reporter) err.raise(PKV_DEVERR_BLOCK_ID);
      } else {
        slot = static_cast<int64_t>(blk) * kBlockTokens + (pos & 15);
      }
    }
  }
  // cos/sin of this position (dims d..d+3 and 64+d..64+d+3)
  bool rope_ok = rope;
  __nv_bfloat16 c[8], sn[8];
  if (rope) {
    if (pos < 0 || pos >= a.rope_rows) {
      if (reporter) err.raise(PKV_DEVERR_POSITION);
      rope_ok = false;
    } else {
      const __nv_bfloat16* cr = static_cast<const __nv_bfloat16*>(a.rope_cos) + static_cast<int64_t>(pos) * kHeadDim;
      const __nv_bfloat16* sr = static_cast<const __nv_bfloat16*>(a.rope_sin) + static_cast<int64_t>(pos) * kHeadDim;
      *reinterpret_cast<uint2*>(c) = *reinterpret_cast<const uint2*>(cr + d);
      *reinterpret_cast<uint2*>(c + 4) = *reinterpret_cast<const uint2*>(cr + 64 + d);
      *reinterpret_cast<uint2*>(sn) = *reinterpret_cast<const uint2*>(sr + d);
      *reinterpret_cast<uint2*>(sn + 4) = *reinterpret_cast<const uint2*>(sr + 64 + d);
    }
  }

  for (int p0 = p_begin; p0 < p_end; p0 += kVecPass) {
    __nv_bfloat16 x[kVecPass][8];
    __nv_bfloat16* dst[kVecPass];
    bool do_rope[kVecPass];
    // loads of every pass of this round first
#pragma unroll
    for (int i = 0; i < kVecPass; ++i) {
      dst[i] = nullptr;
      do_rope[i] = rope;
      const int which = 2 * (p0 + i) + (lane >> 4);
      if (p0 + i >= p_end || which >= per_tok) continue;
      const __nv_bfloat16* src;
      if (which < nq) {
        if (!rope_ok) continue;  // q needs its rotation
        src = static_cast<const __nv_bfloat16*>(a.q) + b * a.q_sb + which * a.q_sh + tt * a.q_st;
        dst[i] = static_cast<__nv_bfloat16*>(a.q_out) + b * a.qo_sb + which * a.qo_sh + tt * a.qo_st;
      } else {
        const bool is_k = which < nq + a.num_kv_heads;
        const int h = is_k ? which - nq : which - nq - a.num_kv_heads;
        if (slot < 0) continue;
        if (is_k) {
          if (rope && !rope_ok) continue;
          src = static_cast<const __nv_bfloat16*>(a.k) + b * a.k_sb + h * a.k_sh + tt * a.k_st;
          dst[i] = static_cast<__nv_bfloat16*>(a.k_pool) + (slot * a.num_kv_heads + h) * kHeadDim;
        } else {
          src = static_cast<const __nv_bfloat16*>(a.v) + b * a.v_sb + h * a.v_sh + tt * a.v_st;
          dst[i] = static_cast<__nv_bfloat16*>(a.v_pool) + (slot * a.num_kv_heads + h) * kHeadDim;
          do_rope[i] = false;
        }
      }
      *reinterpret_cast<uint2*>(x[i]) = *reinterpret_cast<const uint2*>(src + d);
      *reinterpret_cast<uint2*>(x[i] + 4) = *reinterpret_cast<const uint2*>(src + 64 + d);
    }
    // then the rotations and stores
#pragma unroll
    for (int i = 0; i < kVecPass; ++i) {
      if (!dst[i]) continue;
      if (do_rope[i]) {
        __nv_bfloat16 o[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // first half: x*cos + (-x2)*sin ; second half: x*cos + x1*sin
          o[e] = rope1(x[i][e], c[e], __hneg(x[i][4 + e]), sn[e]);
          o[4 + e] = rope1(x[i][4 + e], c[4 + e], x[i][e], sn[4 + e]);
        }
        *reinterpret_cast<uint2*>(dst[i] + d) = *reinterpret_cast<const uint2*>(o);
        *reinterpret_cast<uint2*>(dst[i] + 64 + d) = *reinterpret_cast<const uint2*>(o + 4);
      } else {
        *reinterpret_cast<uint2*>(dst[i] + d) = *reinterpret_cast<const uint2*>(x[i]);
        *reinterpret_cast<uint2*>(dst[i] + 64 + d) = *reinterpret_cast<const uint2*>(x[i] + 4);
      }
    }
  }
}

bool vec8_ok(const AppendLaunch& a) {
  auto al8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; };
  auto m4 = [](int64_t v) { return (v & 3) == 0; };
  if (!al8(a.k) || !al8(a.v) || !m4(a.k_sb) || !m4(a.k_sh) || !m4(a.k_st) || !m4(a.v_sb) ||
      !m4(a.v_sh) || !m4(a.v_st))
    return false;
  if (a.q_out && (!al8(a.q) || !al8(a.q_out) || !m4(a.q_sb) || !m4(a.q_sh) || !m4(a.q_st) ||
                  !m4(a.qo_sb) || !m4(a.qo_sh) || !m4(a.qo_st)))
    return false;
  if (a.rope_cos && (!al8(a.rope_cos) || !al8(a.rope_sin))) return false;
  return true;
}

}  // namespace

// ---------------------------------------------------------------- FP8 pool
// Byte position inside a 16-byte group of the FP8 pool that holds element e
// (0..15) of that group: the order of an m16n8k16 A fragment (byte 4i+u holds
// element 2i+u for u < 2 and 2i+8+u-2 for u >= 2), so one ldmatrix of the
// bytes as 16-bit pairs hands each lane the two pairs its fragment needs.
__device__ __forceinline__ int fp8_pos(int e) {
  return e < 8 ? 4 * (e >> 1) + (e & 1) : 4 * ((e - 8) >> 1) + 2 + (e & 1);
}

// One warp per (row, step token, q / k / v head) as append_rope_kernel; lane
// l owns dims {2l, 2l+1, 64+2l, 64+2l+1}.  q heads: roped q to q_out (same
// bits as the bf16 path).  k (roped, same bits) and v rows are quantised to
// e4m3 with one scale per row: scale = amax / 448, e = RNE(x * (448 / amax))
// saturated to +-448 (448 / amax and amax / 448 each one IEEE division;
// amax = 0 stores zeros with scale 1), into the token's slot of its block's
// FP8 chunk (layout in pkv_kernels.h).
__global__ void __launch_bounds__(256) append_rope_fp8_kernel(const AppendLaunch a,
                                                              int32_t num_blocks) {
  pdl_trigger();
  pdl_wait();
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const int64_t item = gid >> 5;
  const int nq = a.q_out ? a.num_q_heads : 0;
  const int per_tok = nq + 2 * a.num_kv_heads;
  const int64_t total = static_cast<int64_t>(a.batch) * a.seq_len_q * per_tok;
  if (item >= total) return;
  const int which = static_cast<int>(item % per_tok);
  const int64_t bt = item / per_tok;
  const int tt = static_cast<int>(bt % a.seq_len_q);
  const int b = static_cast<int>(bt / a.seq_len_q);
  const DevErr err{a.err};
  const int start = a.starts[b];
  if (start < 0) return;                      // inactive (padding) row
  if (a.q_lens && tt >= a.q_lens[b]) return;  // right padding of a shorter row
  const int pos = start + tt;
  const bool rope = a.rope_cos != nullptr;

  const __nv_bfloat16* src;
  uint8_t* chunk = nullptr;
  __nv_bfloat16* qdst = nullptr;
  bool is_k = false;
  if (which < nq) {
    src = static_cast<const __nv_bfloat16*>(a.q) + b * a.q_sb + which * a.q_sh + tt * a.q_st;
    qdst = static_cast<__nv_bfloat16*>(a.q_out) + b * a.qo_sb + which * a.qo_sh + tt * a.qo_st;
  } else {
    is_k = which < nq + a.num_kv_heads;
    const int h = is_k ? which - nq : which - nq - a.num_kv_heads;
    const int row = a.rows ? a.rows[b] : b;
    const int64_t bi = pos >> 4;
    if (pos < 0 || bi >= a.pitch) {
      if (lane == 0) err.raise(PKV_DEVERR_POSITION);
      return;
    }
    const int blk = a.tables[static_cast<int64_t>(row) * a.pitch + bi];
    if (blk < 0 || blk >= num_blocks) {
      if (lane == 0) err.raise(PKV_DEVERR_BLOCK_ID);
      return;
    }
    chunk = a.kv8 + (static_cast<int64_t>(blk) * a.num_kv_heads + h) * kFp8HeadBlockBytes;
    src = is_k ? static_cast<const __nv_bfloat16*>(a.k) + b * a.k_sb + h * a.k_sh + tt * a.k_st
               : static_cast<const __nv_bfloat16*>(a.v) + b * a.v_sb + h * a.v_sh + tt * a.v_st;
  }
  const int d = 2 * lane;
  __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(src + d);
  __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(src + 64 + d);
  if (rope && (qdst || is_k)) {
    if (pos < 0 || pos >= a.rope_rows) {
      if (lane == 0) err.raise(PKV_DEVERR_POSITION);
      return;
    }
    const __nv_bfloat16* cr =
        static_cast<const __nv_bfloat16*>(a.rope_cos) + static_cast<int64_t>(pos) * kHeadDim;
    const __nv_bfloat16* sr =
        static_cast<const __nv_bfloat16*>(a.rope_sin) + static_cast<int64_t>(pos) * kHeadDim;
    const __nv_bfloat162 clo = *reinterpret_cast<const __nv_bfloat162*>(cr + d);
    const __nv_bfloat162 chi = *reinterpret_cast<const __nv_bfloat162*>(cr + 64 + d);
    const __nv_bfloat162 slo = *reinterpret_cast<const __nv_bfloat162*>(sr + d);
    const __nv_bfloat162 shi = *reinterpret_cast<const __nv_bfloat162*>(sr + 64 + d);
    __nv_bfloat162 olo, ohi;
    olo.x = rope1(lo.x, clo.x, __hneg(hi.x), slo.x);
    olo.y = rope1(lo.y, clo.y, __hneg(hi.y), slo.y);
    ohi.x = rope1(hi.x, chi.x, lo.x, shi.x);
    ohi.y = rope1(hi.y, chi.y, lo.y, shi.y);
    lo = olo;
    hi = ohi;
  }
  if (qdst) {
    *reinterpret_cast<__nv_bfloat162*>(qdst + d) = lo;
    *reinterpret_cast<__nv_bfloat162*>(qdst + 64 + d) = hi;
    return;
  }
  const float x[4] = {bf(lo.x), bf(lo.y), bf(hi.x), bf(hi.y)};
  float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float inv = amax > 0.f ? __fdiv_rn(448.f, amax) : 0.f;
  const float scale = amax > 0.f ? __fdiv_rn(amax, 448.f) : 1.f;
  const int tok = pos & 15;
  const int dims[4] = {d, d + 1, 64 + d, 64 + d + 1};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint8_t q8 = static_cast<uint8_t>(
        __nv_cvt_float_to_fp8(__fmul_rn(x[e], inv), __NV_SATFINITE, __NV_E4M3));
    const int dim = dims[e];
    int off;
    if (is_k) {
      const int c = dim >> 4;
      off = tok * 128 + ((c ^ (tok & 7)) << 4) + fp8_pos(dim & 15);
    } else {
      off = kFp8VOff + dim * 16 + fp8_pos(tok);
    }
    chunk[off] = q8;
  }
  if (lane == 0)
    *reinterpret_cast<float*>(chunk + (is_k ? kFp8KScaleOff : kFp8VScaleOff) + tok * 4) = scale;
}

// One warp per (row, position < kv_len, KV head, K|V); lane l writes dims
// 4l..4l+3 of bf16(e4m3 * scale).
__global__ void __launch_bounds__(256) fp8_dequant_kernel(const Fp8DequantLaunch a) {
  pdl_trigger();
  pdl_wait();
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t per_row = static_cast<int64_t>(a.seq_len) * a.num_kv_heads * 2;
  if (w >= per_row * a.batch) return;
  const int b = static_cast<int>(w / per_row);
  const int64_t r = w - b * per_row;
  const int pos = static_cast<int>(r / (a.num_kv_heads * 2));
  const int hv = static_cast<int>(r - static_cast<int64_t>(pos) * a.num_kv_heads * 2);
  const int h = hv >> 1;
  const bool is_k = (hv & 1) == 0;
  if (pos >= a.kv_lens[b]) return;
  const DevErr err{a.err};
  const int row = a.rows ? a.rows[b] : b;
  const int64_t bi = pos >> 4;
  if (bi >= a.pitch) {
    if (lane == 0) err.raise(PKV_DEVERR_POSITION);
    return;
  }
  const int blk = a.tables[static_cast<int64_t>(row) * a.pitch + bi];
  if (blk < 0 || blk >= a.num_blocks) {
    if (lane == 0) err.raise(PKV_DEVERR_BLOCK_ID);
    return;
  }
  const uint8_t* chunk = a.kv8 + (static_cast<int64_t>(blk) * a.num_kv_heads + h) * kFp8HeadBlockBytes;
  const int tok = pos & 15;
  const float scale =
      *reinterpret_cast<const float*>(chunk + (is_k ? kFp8KScaleOff : kFp8VScaleOff) + tok * 4);
  __nv_bfloat16 out4[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int dim = 4 * lane + e;
    const int off = is_k ? tok * 128 + ((((dim >> 4) ^ (tok & 7))) << 4) + fp8_pos(dim & 15)
                         : kFp8VOff + dim * 16 + fp8_pos(tok);
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(chunk[off], __NV_E4M3);
    out4[e] = rn(__fmul_rn(__half2float(__half(hr)), scale));
  }
  __nv_bfloat16* dst = is_k ? static_cast<__nv_bfloat16*>(a.k_out) + b * a.k_sb + h * a.k_sh +
                                  static_cast<int64_t>(pos) * a.k_ss
                            : static_cast<__nv_bfloat16*>(a.v_out) + b * a.v_sb + h * a.v_sh +
                                  static_cast<int64_t>(pos) * a.v_ss;
  *reinterpret_cast<uint2*>(dst + 4 * lane) = *reinterpret_cast<const uint2*>(out4);
}

cudaError_t launch_fp8_dequant(const Fp8DequantLaunch& a, cudaStream_t stream) {
  const int64_t warps = static_cast<int64_t>(a.batch) * a.seq_len * a.num_kv_heads * 2;
  if (warps == 0) return cudaSuccess;
  return launch_k(fp8_dequant_kernel, dim3(static_cast<unsigned>((warps * 32 + 255) / 256)),
                  dim3(256), 0, stream, a);
}

cudaError_t launch_append(const AppendLaunch& a, cudaStream_t stream) {
  if (a.kv8) {
    const int per_tok = (a.q_out ? a.num_q_heads : 0) + 2 * a.num_kv_heads;
    const int64_t warps = static_cast<int64_t>(a.batch) * a.seq_len_q * per_tok;
    if (warps == 0) return cudaSuccess;
    return launch_k(append_rope_fp8_kernel, dim3(static_cast<unsigned>((warps * 32 + 255) / 256)),
                    dim3(256), 0, stream, a, static_cast<int32_t>(a.num_slots / kBlockTokens));
  }
  const int32_t num_blocks_vec = static_cast<int32_t>(a.num_slots / kBlockTokens);
  if (vec8_ok(a)) {
    const int64_t tokens = static_cast<int64_t>(a.batch) * a.seq_len_q;
    if (tokens == 0) return cudaSuccess;
    // ~4096 warps in flight: a prefill keeps one or two warps per token, a
    // decode step spreads each token's heads over up to one warp per pass
    const int passes = ((a.q_out ? a.num_q_heads : 0) + 2 * a.num_kv_heads + 1) / 2;
    const int64_t want = (4096 + tokens - 1) / tokens;
    const int32_t chunks = static_cast<int32_t>(want < passes ? want : passes);
    const int64_t warps = tokens * (chunks > 0 ? chunks : 1);
    return launch_k(append_rope_vec_kernel, dim3(static_cast<unsigned>((warps * 32 + 255) / 256)),
                    dim3(256), 0, stream, a, num_blocks_vec, chunks > 0 ? chunks : 1);
  }
  const int per_tok = (a.q_out ? a.num_q_heads : 0) + 2 * a.num_kv_heads;
  const int64_t warps = static_cast<int64_t>(a.batch) * a.seq_len_q * per_tok;
  if (warps == 0) return cudaSuccess;
  const int64_t blocks = (warps * 32 + 255) / 256;
  const int32_t num_blocks = static_cast<int32_t>(a.num_slots / kBlockTokens);
  return launch_k(append_rope_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, a,
                  num_blocks);
}

}  // namespace pkv
