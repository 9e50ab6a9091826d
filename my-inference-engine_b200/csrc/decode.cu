// Paged decode attention (one query token per row) for sm_100a.
//
// Reference behaviour: kernels/fa2.py:23-162 launched with SEQLEN_Q = 1 and
// is_causal = False (model.py:103, model.py:185), over K/V that
// kv_cache.py:117-121 gathered densely.  Here K/V blocks are read in place:
//
//   grid  = (partitions, kv_heads * sub_groups, batch)
//   block = 4 warps; warp w takes blocks w, w+4, w+8 ... of its partition and
//           streams them through its own NST-deep ring of TMA stages
//           (K and V of one KV head for one 16-token block = 8 KiB / stage).
//
// Math per 16-token block, one warp, all query heads of the KV group at once
// (mma.sync m16n8k16, tokens in M, query heads in N):
//   S^T[16 tok x 8 heads] = K[16 x 128] . Q^T[128 x 8]          (8 MMAs)
//   online softmax per head over tokens (shuffles across the 8 row lanes)
//   O^T[128 x 8]        += V^T[128 x 16] . P^T[16 x 8]          (8 MMAs)
// P^T reaches the B-operand layout with movmatrix.trans, V^T the A layout with
// ldmatrix.trans, so nothing round-trips through shared memory.  The four
// warps merge (m, l, O) in shared memory; with several partitions each CTA
// stores a normalised partial plus its log2-sum-exp and the last CTA of a
// (row, kv head) to finish merges them (flash-decoding), ordered by partition
// index so the result does not depend on which CTA finished last.
#include <math.h>

#include <algorithm>
#include <mutex>

#include "pkv_device.cuh"
#include "pkv_kernels.h"

namespace pkv {
namespace {

constexpr int kDecodeWarps = 4;
constexpr int kDecodeStages = 3;  // per warp
constexpr int kStageBytes = 2 * kHeadBlockBytes;  // K + V, one head, one block
constexpr int kMaxHeadsPerCta = 8;
// Lazy softmax rescaling threshold (log2 units of the scaled scores): a
// probability is at most 2^kLazyLog2 before its row sum divides it out.
constexpr float kLazyLog2 = 8.f;
// Partition plan.  Every (row, KV head) unit gets up to kMaxParts
// partitions, enough for kTargetCtas CTAs in total (several waves of 2
// resident CTAs per SM).  A partition holds at least kMinBlocksPerPart blocks
// (8 per warp) when the launch has work for kBusyCtas CTAs of that size, so
// per-CTA set-up and the split-K merge stay amortised; smaller launches (few
// rows, short contexts: latency-bound) go down to 16 or 4 blocks.
#ifndef PKV_DECODE_TARGET_CTAS
#define PKV_DECODE_TARGET_CTAS (148 * 2 * 6)
#endif
#ifndef PKV_DECODE_MIN_BLOCKS_PER_PART
#define PKV_DECODE_MIN_BLOCKS_PER_PART 32
#endif
constexpr int kTargetCtas = PKV_DECODE_TARGET_CTAS;
constexpr int kMinBlocksPerPart = PKV_DECODE_MIN_BLOCKS_PER_PART;
constexpr int kMaxParts = 16;
constexpr int64_t kBusyCtas = 600;
constexpr int kMinBlocksPerPartSmall = kDecodeWarps;
constexpr int64_t kWaveCtas = 148 * 2;  // resident bf16 CTAs (the FP8 kernel fits twice as many)
constexpr int64_t kFillUnits = 128;     // units that, one CTA each, occupy most of the 148 SMs

// The per-partition minimum for `units` (row, KV head) units of `nblk`
// blocks each.  The host plans the grid with it for the launch's longest row
// (or a CUDA graph's capacity); the kernel applies it again to each row's
// own length (through block thresholds the host derives for the launch), so
// rows far shorter than planned -- a graph captured for the cache's capacity
// replaying short histories -- are split as an eager launch of their real
// length would split them.
inline int min_blocks_per_part_for(int64_t units, int nblk) {
  if (units * (nblk / kMinBlocksPerPart) >= kBusyCtas) return kMinBlocksPerPart;
  if (units * (nblk / 16) >= kBusyCtas) return 16;
  return kMinBlocksPerPartSmall;
}

// split-K completion counters: one int32 per (row, kv head, head sub-group)
constexpr int64_t kDecodeMaxUnits = 1 << 16;
constexpr size_t kDecodeCounterBytes = kDecodeMaxUnits * sizeof(int32_t);

struct DecodeParams {
  const __nv_bfloat16* q;
  int64_t q_sb, q_sh;
  __nv_bfloat16* out;
  int64_t o_sb, o_sh;
  const int32_t* kv_lens;
  const int32_t* tables;
  int64_t pitch;
  const int32_t* rows;
  int32_t num_blocks;
  int32_t group;       // query heads per KV head
  int32_t sub_groups;  // CTAs per KV head (group > 8)
  int32_t max_parts;   // grid.x: partitions available to every row
  int32_t min_blocks_per_part;
  // min_blocks_per_part_for(units, nblk) of this launch's units as block
  // thresholds (nblk >= busy32: 32, >= busy16: 16, else the small minimum),
  // and the partitions per row of about one wave of resident CTAs
  int32_t busy32, busy16, wave_parts;
  float scale_log2;
  float* part_o;
  float* part_lse;
  int32_t* counters;
  int32_t* err;
  const uint8_t* kv8;  // FP8 pool of the layer (FP8 kernel only)
};

// FP8 pool: one stage is one (block, KV head) chunk, half the bytes of a bf16
// stage, so each warp keeps more of them in flight.
constexpr int kDecodeStagesFp8 = 3;  // 4 CTAs per SM: 16 warps hide the per-block latency

template <int NST, bool kFp8>
constexpr int decode_stage_bytes() {
  return kFp8 ? kFp8HeadBlockBytes : kStageBytes;
}
template <int NST, bool kFp8 = false>
constexpr int decode_smem_bytes() {
  return kDecodeWarps * NST * decode_stage_bytes<NST, kFp8>() + kDecodeWarps * NST * 8 + 1024;
}

// kFp8: K/V come from the FP8 pool (layout in pkv_kernels.h) by one bulk copy
// per (block, KV head); K and V fragments are e4m3 pairs loaded with
// ldmatrix and widened to f16 in registers (exact), the products run as f16
// MMAs with Q scaled by 1/16 (exact: keeps any bf16 q inside f16 range), and
// each token's K scale (with the 16) multiplies its scores, its V scale its
// probabilities after the row sum.  Everything else is the bf16 kernel.
template <bool kPaged, int NST, bool kFp8 = false>
__global__ void __launch_bounds__(kDecodeWarps * 32, kFp8 ? 4 : 2)
    paged_decode_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap) {
  constexpr int kSB = decode_stage_bytes<NST, kFp8>();
  static_assert(NST <= 32, "the prologue's block ids come from the first 32-id chunk");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDecodeWarps * NST * kSB);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int b = blockIdx.z;
  const int y = blockIdx.y;
  const int kvh = y / p.sub_groups;
  const int sub = y - kvh * p.sub_groups;
  const int head0 = kvh * p.group + sub * kMaxHeadsPerCta;
  const int nheads = min(kMaxHeadsPerCta, p.group - sub * kMaxHeadsPerCta);
  const int part = blockIdx.x;
  const DevErr err{p.err};
  pdl_trigger();
  pdl_wait();

  int kv_len = max(p.kv_lens[b], 0);
  int nblk = (kv_len + kBlockTokens - 1) / kBlockTokens;
  const int32_t* trow = nullptr;
  if constexpr (kPaged) {
    const int row = p.rows ? p.rows[b] : b;
    trow = p.tables + static_cast<int64_t>(row) * p.pitch;
    if (nblk > p.pitch) {
      if (part == 0 && tid == 0) err.raise(PKV_DEVERR_POSITION);
      nblk = static_cast<int>(p.pitch);
      kv_len = nblk * kBlockTokens;
    }
  }
  if (kv_len == 0) {
    // fa2.py:151 divides by a zero row sum: the reference yields NaN.
    if (part == 0) {
      for (int i = tid; i < nheads * kHeadDim; i += blockDim.x) {
        const int h = i / kHeadDim, d = i % kHeadDim;
        p.out[b * p.o_sb + (head0 + h) * p.o_sh + d] = __float2bfloat16(__int_as_float(0x7fc00000));
      }
    }
    return;
  }
  // Every row splits into up to gridDim.x equal partitions of at least
  // min_bpp blocks (rounded to the warp count), sized from its own length:
  // the grid is planned for the longest row (or a captured capacity), shorter
  // rows use fewer partitions instead of tiny ones, and the minimum itself is
  // the one a launch of rows of this length would take (never above the
  // plan's).
  // No partition holds fewer than kMinBlocksPerPartSmall blocks: a CTA past
  // that many partitions of its row has no work and leaves at once (a grid
  // planned for a graph's capacity has many such CTAs).
  if (part * kMinBlocksPerPartSmall >= nblk) return;
  const int row_min =
      nblk >= p.busy32 ? kMinBlocksPerPart : (nblk >= p.busy16 ? 16 : kMinBlocksPerPartSmall);
  const int min_bpp = min(p.min_blocks_per_part, row_min);
  int np = min(p.max_parts, max(1, nblk / min_bpp));
  // a latency-bound launch (rows like this one would not keep kBusyCtas CTAs
  // busy) takes at most about one wave of CTAs: more partitions only add
  // waves of set-up and merge
  if (row_min < kMinBlocksPerPart) np = min(np, p.wave_parts);
  const int per = (nblk + np - 1) / np;
  const int bpp = max(kDecodeWarps, (per + kDecodeWarps - 1) / kDecodeWarps * kDecodeWarps);
  const int nparts = (nblk + bpp - 1) / bpp;
  if (part >= nparts) return;
  const int blk_begin = part * bpp;
  const int blk_end = min(nblk, blk_begin + bpp);
  const int span = blk_end - blk_begin;
  const int my_n = span > warp ? (span - warp + kDecodeWarps - 1) / kDecodeWarps : 0;

  uint8_t* wstage = smem + warp * NST * kSB;
  uint64_t* wbar = bars + warp * NST;
  if (lane == 0) {
    for (int s = 0; s < NST; ++s) mbar_init(&wbar[s], 1);
    fence_mbar_init();
    if (warp == 0 && !kFp8) {
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
    }
  }
  __syncwarp();

  const uint64_t policy = policy_evict_first();
  // Block ids of this warp's iterations, 32 at a time: lane k holds the id of
  // iteration 32c + k (ids_cur) and of 32(c + 1) + k (ids_next, loaded one
  // chunk ahead).  The id a refill needs is a shuffle away, so the copy
  // issue never waits on a table load from global memory.
  auto load_ids = [&](int c) -> int {
    const int it = c * 32 + lane;
    return (kPaged && it < my_n) ? __ldg(trow + blk_begin + warp + kDecodeWarps * it) : 0;
  };
  int ids_cur = load_ids(0);
  int ids_next = my_n > 32 ? load_ids(1) : 0;
  auto issue = [&](int i, int blk) {
    const int j = blk_begin + warp + kDecodeWarps * i;
    const int st = i % NST;
    uint8_t* kst = wstage + st * kSB;
    uint8_t* vst = kst + kHeadBlockBytes;
    mbar_arrive_expect_tx(&wbar[st], kSB);
    if constexpr (kFp8) {
      if (blk < 0 || blk >= p.num_blocks) {
        err.raise(PKV_DEVERR_BLOCK_ID);
        blk = 0;
      }
      bulk_load(kst, p.kv8 + (static_cast<int64_t>(blk) * (gridDim.y / p.sub_groups) + kvh) * kSB,
                kSB, &wbar[st], policy);
    } else if constexpr (kPaged) {
      if (blk < 0 || blk >= p.num_blocks) {
        err.raise(PKV_DEVERR_BLOCK_ID);
        blk = 0;
      }
      const int slot = blk * kBlockTokens;
      tma_load_3d(kst, &kmap, &wbar[st], 0, kvh, slot, policy);
      tma_load_3d(kst + kBoxBytes, &kmap, &wbar[st], 64, kvh, slot, policy);
      tma_load_3d(vst, &vmap, &wbar[st], 0, kvh, slot, policy);
      tma_load_3d(vst + kBoxBytes, &vmap, &wbar[st], 64, kvh, slot, policy);
    } else {
      const int tok = j * kBlockTokens;
      tma_load_4d(kst, &kmap, &wbar[st], 0, tok, kvh, b, policy);
      tma_load_4d(kst + kBoxBytes, &kmap, &wbar[st], 64, tok, kvh, b, policy);
      tma_load_4d(vst, &vmap, &wbar[st], 0, tok, kvh, b, policy);
      tma_load_4d(vst + kBoxBytes, &vmap, &wbar[st], 64, tok, kvh, b, policy);
    }
  };
  for (int i = 0; i < min(NST, my_n); ++i) {  // NST <= 32: all in chunk 0
    const int blk = __shfl_sync(0xffffffffu, ids_cur, i);
    if (lane == 0) issue(i, blk);
  }

  // Q^T as the B operand: lane (g, t) holds query head g, dims 2t..2t+1 and
  // 2t+8..2t+9 of every 16-dim k-step.  Heads >= nheads are zero columns.
  uint32_t qb[8][2];
  {
    const bool live = g < nheads;
    const __nv_bfloat16* qp = p.q + b * p.q_sb + (head0 + (live ? g : 0)) * p.q_sh;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      qb[kk][0] = live ? *reinterpret_cast<const uint32_t*>(qp + kk * 16 + 2 * t) : 0u;
      qb[kk][1] = live ? *reinterpret_cast<const uint32_t*>(qp + kk * 16 + 8 + 2 * t) : 0u;
      if constexpr (kFp8) {  // bf16 pairs -> f16 pairs of q / 16
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&qb[kk][h]);
          const float2 f = __bfloat1622float2(v);
          qb[kk][h] = pack_f16(f.x * 0.0625f, f.y * 0.0625f);
        }
      }
    }
  }

  float m0 = -INFINITY, m1 = -INFINITY;  // running max, heads 2t and 2t+1
  float l0 = 0.f, l1 = 0.f;              // per-lane partial row sums
  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

  // ldmatrix lane roles (constant across blocks)
  const int a_row = (lane & 7) + ((lane >> 3) & 1) * 8;  // K rows for S^T
  const int a_chk = lane >> 4;
  const int v_tok = (lane & 7) + ((lane >> 4) & 1) * 8;  // V rows for O^T
  const int v_chk = (lane >> 3) & 1;

  int i = 0;
  bool ok = true;
  for (; i < my_n; ++i) {
    const int st = i % NST;
    ok = mbar_wait(&wbar[st], (i / NST) & 1, err);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) break;
    const uint32_t kst = smem_u32(wstage + st * kSB);
    const uint32_t vst = kst + (kFp8 ? kFp8VOff : kHeadBlockBytes);
    const int j = blk_begin + warp + kDecodeWarps * i;

    float s[4] = {0.f, 0.f, 0.f, 0.f};
    float s2[4] = {0.f, 0.f, 0.f, 0.f};
    float ks0 = p.scale_log2, ks1 = p.scale_log2;  // score scale of tokens g and g+8
    float vs0 = 1.f, vs1 = 1.f;                    // probability scale of tokens g, g+8
    if constexpr (kFp8) {
      // ldmatrix of e4m3 pairs: matrix m covers tokens (m & 1) * 8 + 0..7 of
      // 16-dim group 2c + (m >> 1); each register widens to the A fragment
      // halves of one k-step (a0 | a2 from the low | high pair)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int chunk = 2 * c + a_chk;
        uint32_t r0, r1, r2, r3, a0, a1, a2, a3, b0, b1, b2, b3;
        ldsm_x4(kst + a_row * 128 + ((chunk ^ (a_row & 7)) << 4), r0, r1, r2, r3);
        e4m3x4_to_f16x2x2(r0, a0, a2);
        e4m3x4_to_f16x2x2(r1, a1, a3);
        e4m3x4_to_f16x2x2(r2, b0, b2);
        e4m3x4_to_f16x2x2(r3, b1, b3);
        mma_f16(s, a0, a1, a2, a3, qb[2 * c][0], qb[2 * c][1]);
        mma_f16(s2, b0, b1, b2, b3, qb[2 * c + 1][0], qb[2 * c + 1][1]);
      }
      const float* sc = reinterpret_cast<const float*>(wstage + st * kSB + kFp8KScaleOff);
      ks0 = sc[g] * (16.f * p.scale_log2);
      ks1 = sc[g + 8] * (16.f * p.scale_log2);
      vs0 = sc[16 + g];
      vs1 = sc[16 + g + 8];
    } else {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kst + (kk >> 2) * kBoxBytes + swz128(a_row, (kk & 3) * 2 + a_chk), a0, a1, a2,
                a3);
        if (kk & 1)
          mma_bf16(s2, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
        else
          mma_bf16(s, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
      }
    }
    const int tok0 = j * kBlockTokens + g;
    float x0 = (s[0] + s2[0]) * ks0;
    float x1 = (s[1] + s2[1]) * ks0;
    float x2 = (s[2] + s2[2]) * ks1;
    float x3 = (s[3] + s2[3]) * ks1;
    if (tok0 >= kv_len) x0 = x1 = -INFINITY;
    if (tok0 + 8 >= kv_len) x2 = x3 = -INFINITY;

    // Lazy rescaling: the running base moves (and O and l are rescaled)
    // only when some score of the block exceeds its head's base by more than
    // 2^kLazyLog2; otherwise probabilities are taken against the old base
    // and stay <= 2^kLazyLog2.  Each lane tests its own scores and one vote
    // makes the decision warp-uniform, so the block maximum (three shuffle
    // rounds across the token lanes) is only reduced when the base moves.
    float mb0 = fmaxf(x0, x2), mb1 = fmaxf(x1, x3);
    if (__any_sync(0xffffffffu, mb0 > m0 + kLazyLog2 || mb1 > m1 + kLazyLog2)) {
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mb0 = fmaxf(mb0, __shfl_xor_sync(0xffffffffu, mb0, off));
        mb1 = fmaxf(mb1, __shfl_xor_sync(0xffffffffu, mb1, off));
      }
      const float mn0 = fmaxf(m0, mb0), mn1 = fmaxf(m1, mb1);
      const float al0 = ex2(m0 - (mn0 == -INFINITY ? 0.f : mn0));
      const float al1 = ex2(m1 - (mn1 == -INFINITY ? 0.f : mn1));
      l0 *= al0;
      l1 *= al1;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= al0;
        o[mt][1] *= al1;
        o[mt][2] *= al0;
        o[mt][3] *= al1;
      }
    }
    const float base0 = m0 == -INFINITY ? 0.f : m0;
    const float base1 = m1 == -INFINITY ? 0.f : m1;
    const float p0 = ex2(x0 - base0), p2 = ex2(x2 - base0);
    const float p1 = ex2(x1 - base1), p3 = ex2(x3 - base1);
    l0 += p0 + p2;
    l1 += p1 + p3;
    if constexpr (kFp8) {
      const uint32_t pb0 = movm_t(pack_f16(p0 * vs0, p1 * vs0));
      const uint32_t pb1 = movm_t(pack_f16(p2 * vs1, p3 * vs1));
      // V^T rows (dims) of 16 e4m3 tokens: matrix m covers dims
      // 16 * (2c + (m >> 1)) + (m & 1) * 8 + 0..7
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r0, r1, r2, r3, a0, a1, a2, a3, b0, b1, b2, b3;
        ldsm_x4(vst + (32 * c + (lane & 7) + ((lane >> 3) & 1) * 8 + (lane >> 4) * 16) * 16, r0,
                r1, r2, r3);
        e4m3x4_to_f16x2x2(r0, a0, a2);
        e4m3x4_to_f16x2x2(r1, a1, a3);
        e4m3x4_to_f16x2x2(r2, b0, b2);
        e4m3x4_to_f16x2x2(r3, b1, b3);
        mma_f16(o[2 * c], a0, a1, a2, a3, pb0, pb1);
        mma_f16(o[2 * c + 1], b0, b1, b2, b3, pb0, pb1);
      }
    } else {
      const uint32_t pb0 = movm_t(pack_bf16(p0, p1));
      const uint32_t pb1 = movm_t(pack_bf16(p2, p3));
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(vst + (mt >> 2) * kBoxBytes + swz128(v_tok, (mt & 3) * 2 + v_chk), a0, a1, a2,
                  a3);
        mma_bf16(o[mt], a0, a1, a2, a3, pb0, pb1);
      }
    }
    __syncwarp();
    const int nx = i + NST;
    if (nx < my_n) {  // warp-uniform
      if ((nx & 31) == 0) {
        ids_cur = ids_next;
        ids_next = load_ids((nx >> 5) + 1);
      }
      const int blk = __shfl_sync(0xffffffffu, ids_cur, nx & 31);
      if (lane == 0) issue(nx, blk);
    }
  }
  if (!ok) {
    // Give loads still in flight a bounded chance to land before the shared
    // memory is reused, and contribute nothing from this warp.
    for (int k = i; k < min(my_n, i + NST); ++k) mbar_wait(&wbar[k % NST], (k / NST) & 1, err);
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }

  // ---- merge the four warps (reuses the stage ring) ----
  __syncthreads();
  float* cm = reinterpret_cast<float*>(smem);                   // [4][8]
  float* cl = cm + kDecodeWarps * 8;                             // [4][8]
  float* co = reinterpret_cast<float*>(smem + 1024);             // [4][8][128]
  if (g == 0) {
    cm[warp * 8 + 2 * t] = m0;
    cm[warp * 8 + 2 * t + 1] = m1;
    cl[warp * 8 + 2 * t] = l0;
    cl[warp * 8 + 2 * t + 1] = l1;
  }
  {
    float* cw = co + warp * 8 * kHeadDim;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      const int d = mt * 16 + g;
      cw[(2 * t) * kHeadDim + d] = o[mt][0];
      cw[(2 * t + 1) * kHeadDim + d] = o[mt][1];
      cw[(2 * t) * kHeadDim + d + 8] = o[mt][2];
      cw[(2 * t + 1) * kHeadDim + d + 8] = o[mt][3];
    }
  }
  __syncthreads();

  const int h = tid >> 4;         // 0..7
  const int d0 = (tid & 15) * 8;  // 8 dims per thread
  float acc[8];
  float L = 0.f, M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kDecodeWarps; ++w) M = fmaxf(M, cm[w * 8 + h]);
  const float mbase = M == -INFINITY ? 0.f : M;
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
  for (int w = 0; w < kDecodeWarps; ++w) {
    const float f = ex2(cm[w * 8 + h] - mbase);
    L += f * cl[w * 8 + h];
    const float* src = co + (w * 8 + h) * kHeadDim + d0;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += f * src[e];
  }

  if (nparts == 1) {
    if (h < nheads) {
      const float inv = 1.f / L;
      uint4 pk;
      pk.x = pack_bf16(acc[0] * inv, acc[1] * inv);
      pk.y = pack_bf16(acc[2] * inv, acc[3] * inv);
      pk.z = pack_bf16(acc[4] * inv, acc[5] * inv);
      pk.w = pack_bf16(acc[6] * inv, acc[7] * inv);
      *reinterpret_cast<uint4*>(p.out + b * p.o_sb + (head0 + h) * p.o_sh + d0) = pk;
    }
    return;
  }

  // ---- split-K: store this partition, last CTA merges ----
  const int64_t unit = static_cast<int64_t>(b) * gridDim.y + y;
  {
    const int64_t slot = unit * p.max_parts + part;
    const float inv = 1.f / L;
    float4* dst = reinterpret_cast<float4*>(p.part_o + (slot * 8 + h) * kHeadDim + d0);
    dst[0] = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
    dst[1] = make_float4(acc[4] * inv, acc[5] * inv, acc[6] * inv, acc[7] * inv);
    if ((tid & 15) == 0) p.part_lse[slot * 8 + h] = mbase + log2f(L);
  }
  __threadfence();
  __syncthreads();
  __shared__ int s_last;
  if (tid == 0) {
    const int prev = atomicAdd(&p.counters[unit], 1);
    s_last = (prev == nparts - 1);
    if (s_last) p.counters[unit] = 0;  // every partition has arrived: rearm
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (h >= nheads) return;
  const float* lse = p.part_lse + unit * p.max_parts * 8 + h;
  float LM = -INFINITY;
  for (int q = 0; q < nparts; ++q) LM = fmaxf(LM, __ldcg(lse + q * 8));
  float W = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  for (int q = 0; q < nparts; ++q) {
    const float w = ex2(__ldcg(lse + q * 8) - LM);
    W += w;
    const float4* src =
        reinterpret_cast<const float4*>(p.part_o + ((unit * p.max_parts + q) * 8 + h) * kHeadDim + d0);
    const float4 u = __ldcg(src), v = __ldcg(src + 1);
    acc[0] += w * u.x;
    acc[1] += w * u.y;
    acc[2] += w * u.z;
    acc[3] += w * u.w;
    acc[4] += w * v.x;
    acc[5] += w * v.y;
    acc[6] += w * v.z;
    acc[7] += w * v.w;
  }
  const float inv = 1.f / W;
  uint4 pk;
  pk.x = pack_bf16(acc[0] * inv, acc[1] * inv);
  pk.y = pack_bf16(acc[2] * inv, acc[3] * inv);
  pk.z = pack_bf16(acc[4] * inv, acc[5] * inv);
  pk.w = pack_bf16(acc[6] * inv, acc[7] * inv);
  *reinterpret_cast<uint4*>(p.out + b * p.o_sb + (head0 + h) * p.o_sh + d0) = pk;
}

}  // namespace

size_t decode_counter_bytes() { return kDecodeCounterBytes; }
int64_t decode_max_units() { return kDecodeMaxUnits; }

namespace {


template <bool kPaged, bool kFp8 = false>
cudaError_t launch_decode_t(const DecodeParams& prm, const KVSource& src, dim3 grid,
                            cudaStream_t stream) {
  constexpr int NST = kFp8 ? kDecodeStagesFp8 : kDecodeStages;
  auto kern = paged_decode_kernel<kPaged, NST, kFp8>;
  constexpr int smem = decode_smem_bytes<NST, kFp8>();
  static_assert(smem <= (kFp8 ? 56 : 113) * 1024, "decode CTAs per SM (2 bf16, 4 FP8)");
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
  return launch_k(kern, grid, dim3(kDecodeWarps * 32), static_cast<size_t>(smem), stream, prm,
                  src.kmap, src.vmap);
}

}  // namespace

DecodePlan plan_decode(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                       int32_t max_kv_len, bool fp8) {
  DecodePlan pl{};
  const int group = num_q_heads / num_kv_heads;
  pl.sub_groups = (group + kMaxHeadsPerCta - 1) / kMaxHeadsPerCta;
  const int64_t units = static_cast<int64_t>(batch) * num_kv_heads * pl.sub_groups;
  const int nblk = max(1, (max_kv_len + kBlockTokens - 1) / kBlockTokens);
  const int64_t units1 = units > 0 ? units : 1;
  // the FP8 kernel keeps twice the CTAs resident per SM (4 vs 2): the same
  // number of waves takes twice the CTAs
  const int64_t target = fp8 ? 2 * static_cast<int64_t>(kTargetCtas) : kTargetCtas;
  const int64_t want = (target + units1 - 1) / units1;
  const int64_t parts = want < kMaxParts ? want : kMaxParts;
  const int min_bpp = min_blocks_per_part_for(units, nblk);
  int bpp = static_cast<int>((nblk + parts - 1) / parts);
  bpp = max(bpp, min_bpp);
  bpp = (bpp + kDecodeWarps - 1) / kDecodeWarps * kDecodeWarps;
  pl.blocks_per_part = bpp;
  pl.min_blocks_per_part = min_bpp;
  pl.max_parts = (nblk + bpp - 1) / bpp;
  if (pl.max_parts > 1) {
    const int64_t slots = units * pl.max_parts;
    pl.workspace_bytes = kDecodeCounterBytes + static_cast<size_t>(slots) * 8 * sizeof(float) +
                         static_cast<size_t>(slots) * 8 * kHeadDim * sizeof(float);
  } else {
    pl.workspace_bytes = 0;
  }
  return pl;
}

cudaError_t launch_decode(const DecodeLaunch& a, const KVSource& src, const DecodePlan& plan,
                          cudaStream_t stream) {
  DecodeParams prm{};
  prm.q = static_cast<const __nv_bfloat16*>(a.q);
  prm.q_sb = a.q_sb;
  prm.q_sh = a.q_sh;
  prm.out = static_cast<__nv_bfloat16*>(a.out);
  prm.o_sb = a.o_sb;
  prm.o_sh = a.o_sh;
  prm.kv_lens = a.kv_lens;
  prm.tables = src.tables;
  prm.pitch = src.pitch;
  prm.rows = src.rows;
  prm.num_blocks = src.num_blocks;
  prm.group = a.num_q_heads / a.num_kv_heads;
  prm.sub_groups = plan.sub_groups;
  prm.max_parts = plan.max_parts;
  prm.min_blocks_per_part = plan.min_blocks_per_part;
  {
    const int64_t units = static_cast<int64_t>(a.batch) * a.num_kv_heads * plan.sub_groups;
    const int64_t need = (kBusyCtas + units - 1) / units;  // units * (nblk / m) >= kBusyCtas
    prm.busy32 = static_cast<int32_t>(std::min<int64_t>(need * kMinBlocksPerPart, 1 << 30));
    prm.busy16 = static_cast<int32_t>(std::min<int64_t>(need * 16, 1 << 30));
    // when one partition per row already puts a CTA on most SMs, splitting
    // further only doubles the CTAs per SM and adds a merge (64 rows x 512
    // tokens: 12.8 us unsplit vs 15.0 us in two)
    const int64_t wave = (a.kv8 ? 2 : 1) * (units >= kFillUnits ? kWaveCtas / 2 : kWaveCtas);
    prm.wave_parts = static_cast<int32_t>(std::max<int64_t>(1, wave / units));
  }
  prm.scale_log2 = a.sm_scale * 1.4426950408889634f;
  prm.err = a.err;
  prm.kv8 = a.kv8;
  if (plan.max_parts > 1) {
    const int64_t units = static_cast<int64_t>(a.batch) * a.num_kv_heads * plan.sub_groups;
    const int64_t slots = units * plan.max_parts;
    // Counters always live in the first kDecodeCounterBytes, whatever the
    // plan, so a workspace reused with another shape never reads partials
    // as counters; every launch leaves the counters it used at zero.
    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    prm.counters = reinterpret_cast<int32_t*>(ws);
    prm.part_lse = reinterpret_cast<float*>(ws + kDecodeCounterBytes);
    prm.part_o = prm.part_lse + slots * 8;
  }
  dim3 grid(plan.max_parts, a.num_kv_heads * plan.sub_groups, a.batch);
  if (a.kv8) return launch_decode_t<true, true>(prm, src, grid, stream);
  return src.paged ? launch_decode_t<true>(prm, src, grid, stream)
                   : launch_decode_t<false>(prm, src, grid, stream);
}

// ---------------------------------------------------------------------------
// Decode with library-owned scratch, for callers that cannot allocate device
// memory (see pkv_paged_decode_static_scratch in pagedkv.h).
//
// The split-K scratch lives in this file-scope device array instead of a
// caller-provided workspace.  Host code must not pass `g_decode_scratch`
// itself to a kernel: on the host that name only stands in for the device
// symbol.  The device address is looked up once per device, with that device
// current, through cudaGetSymbolAddress, and that pointer is what the kernel
// receives.  Every GPU that loads the library keeps these bytes until exit.
// ---------------------------------------------------------------------------
static __device__ __align__(256) uint8_t g_decode_scratch[PKV_DECODE_STATIC_SCRATCH_BYTES];

namespace {
constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxScratchDevices] = {};
}  // namespace

cudaError_t decode_static_scratch(void** ptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxScratchDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *ptr = g_scratch_ptr[dev];
  return cudaSuccess;
}

cudaError_t launch_decode_static(const DecodeLaunch& a, const KVSource& src,
                                 const DecodePlan& plan, cudaStream_t stream) {
  void* scratch = nullptr;
  cudaError_t e = decode_static_scratch(&scratch);
  if (e != cudaSuccess) return e;
  if (plan.max_parts > 1) {
    // The array keeps whatever the previous call left in it.  Only the
    // split-K completion counters must start at zero; clear the ones this
    // launch uses (partials are always written before they are read).
    const int64_t units = static_cast<int64_t>(a.batch) * a.num_kv_heads * plan.sub_groups;
    e = cudaMemsetAsync(scratch, 0, static_cast<size_t>(units) * sizeof(int32_t), stream);
    if (e != cudaSuccess) return e;
  }
  DecodeLaunch b = a;
  b.workspace = scratch;
  b.workspace_bytes = PKV_DECODE_STATIC_SCRATCH_BYTES;
  return launch_decode(b, src, plan, stream);
}

}  // namespace pkv
