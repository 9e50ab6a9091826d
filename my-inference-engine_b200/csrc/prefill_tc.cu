// Ragged causal prefill attention on the 5th-generation tensor cores
// (tcgen05 + TMEM, sm_100a).
//
// Contract: kernels/fa2.py:23-162 with is_causal = T > 1 (model.py:185):
// query i of row b sits at key i + kv_len - T (bottom-right, fa2.py:110-111),
// keys >= kv_len are masked (fa2.py:132-136), online softmax in fp32, P
// rounded to bf16 before the PV product (fa2.py:145), O / l at the end
// (fa2.py:151).
//
//   grid  = (Hq, B, ceil(T/128)): one CTA per 128 query rows of one head,
//           heaviest (last) q-tiles first
//   block = 7 warps
//     warp 0    TMA producer (one thread): Q tile once, then 128-key K tiles
//               (eight 16-token blocks each, through the block table) into a
//               2-deep ring, one tile ahead: a K stage is refilled as soon as
//               its Q.K^T retired, so the next K tile loads during the current
//               softmax; block ids read one tile ahead
//     warp 6    TMA producer of the V tiles (their own 2-deep ring)
//     warp 1    owns TMEM (512 columns: S0, S1, O) and issues tcgen05.mma:
//               S[b] = Q.K^T (M=128, N=128, K=128 in 8 steps), then
//               O += P.V (K = 16 keys per step, only the loaded blocks)
//     warps 2-5 softmax: warp w owns TMEM lanes 32*(w%4).., i.e. one query
//               row per thread, so row max / sum need no shuffles; writes P
//               (bf16 pairs) over the first 64 columns of its S buffer, which
//               P.V reads as its A operand from tensor memory; rescales O in
//               TMEM when a row's max moved; epilogue
// Shared-memory operands use the canonical 128B-swizzled layouts: Q, K
// K-major (rows of 64 elements, 8-row groups 1024 B apart, k-steps advance
// the start address by 32 B), V MN-major (64-dim groups 16 KB apart, 8-key
// groups 1024 B apart).  Every wait is bounded.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "pkv_device.cuh"
#include "pkv_kernels.h"
#include "tc_device.cuh"

namespace pkv {
namespace {

constexpr int kRows = 128;                         // query rows per CTA (MMA M)
constexpr int kKeys = 128;                         // keys per tile (N of Q.K^T, K of P.V)
constexpr int kTileBlocks = kKeys / kBlockTokens;  // 8
constexpr int kRegion = kRows * 128;               // 16 KiB: 128 rows x 64 bf16
constexpr int kOperand = 2 * kRegion;              // 32 KiB: dims (or keys) 0-63 | 64-127
constexpr int kStages = 2;
// warp 6 issues the V tiles while warp 0 issues Q and the K tiles: a tile's
// 32 TMA boxes otherwise take one thread most of a tile period to issue
constexpr bool kSplitProducer = true;
constexpr int kThreads = kSplitProducer ? 224 : 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// smem map (offsets from the 1024-aligned base)
constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + kOperand;  // stage s: K at +s*64K, V at +32K
constexpr int kOffBar = kOffKV + kStages * 2 * kOperand;
constexpr int kNumBars = 1 + 4 * kStages + 2 + 2 + 1 + 1;
constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;

// instruction descriptors (kind::f16): fp32 accumulate, bf16 A/B, M=128, N=128
constexpr uint32_t kIdescBase = (1u << 4) | (1u << 7) | (1u << 10) | ((kKeys >> 3) << 17) |
                                ((kRows >> 4) << 24);
constexpr uint32_t kIdescQK = kIdescBase;               // A K-major, B K-major
constexpr uint32_t kIdescPV = kIdescBase | (1u << 16);  // B (V) MN-major

struct TcParams {
  __nv_bfloat16* out;
  int64_t o_sb, o_sh, o_st;
  const int32_t* kv_lens;
  const int32_t* q_lens;  // nullable
  const int32_t* tables;
  int64_t pitch;
  const int32_t* rows;
  int32_t num_blocks;
  int32_t T;
  int32_t group;
  int32_t causal;
  float scale_log2;
  int32_t* err;
};

// K-major operand (Q, K or P): 128 rows, k-step kk covers elements
// [16kk, 16kk+16) -> region kk/4, +32 B per step inside the 128 B row.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  return sdesc(base + (kk >> 2) * kRegion + (kk & 3) * 32, 16, 1024);
}

// Epilogue store of one softmax warp's 32 output rows.  Lane i holds row i
// of O (fp32, from TMEM); a direct store would have every lane write its own
// 256-byte row, 32 lines per instruction.  Instead the rows go through an
// 8 KiB shared-memory stage (16-byte chunk c of row i at slot c ^ (i & 15):
// conflict-free both ways) and come back out two whole rows per instruction.
// `obase` is the warp's first row; rows at or past `rows_valid` are not
// written.
__device__ __forceinline__ void store_o_rows(uint8_t* stage, const float (&v)[4][32], float inv,
                                             int lane, __nv_bfloat16* obase, int64_t o_st,
                                             int rows_valid) {
  uint8_t* mine = stage + lane * 256;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
#pragma unroll
    for (int e = 0; e < 32; e += 8) {
      uint4 pk;
      pk.x = pack_bf16(v[c][e + 0] * inv, v[c][e + 1] * inv);
      pk.y = pack_bf16(v[c][e + 2] * inv, v[c][e + 3] * inv);
      pk.z = pack_bf16(v[c][e + 4] * inv, v[c][e + 5] * inv);
      pk.w = pack_bf16(v[c][e + 6] * inv, v[c][e + 7] * inv);
      const int chunk = c * 4 + e / 8;
      *reinterpret_cast<uint4*>(mine + ((chunk ^ (lane & 15)) << 4)) = pk;
    }
  }
  __syncwarp();
  const int ch = lane & 15;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int row = 2 * i + (lane >> 4);
    const uint4 val =
        *reinterpret_cast<const uint4*>(stage + row * 256 + ((ch ^ (row & 15)) << 4));
    if (row < rows_valid)
      *reinterpret_cast<uint4*>(obase + static_cast<int64_t>(row) * o_st + ch * 8) = val;
  }
}

template <bool kPaged>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap qmap,
                      const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;
  // K and V have separate rings: a K stage is free once Q.K^T retired, a V
  // stage once P.V retired, so K(j+2) streams in during tile j's softmax
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + kStages;
  uint64_t* v_full = k_empty + kStages;
  uint64_t* v_empty = v_full + kStages;
  // S[b] is rewritten by Q.K^T(j+2) only after P.V(j) (issue order), which
  // waited for P(j): that also means the softmax has read S(j)
  uint64_t* s_full = v_empty + kStages;
  // P(j) ready (one arrival per softmax warp), per parity of j like S: a
  // warp that skipped its P.V wait can be a whole tile ahead of the slowest
  // warp, and with one barrier its arrival for tile j+1 would complete tile
  // j's phase before the slow warp's P(j) was written.  Two barriers also
  // keep the MMA issuer from missing a phase: tile j+2's arrivals need
  // S(j+2), which is issued only after P.V(j+1), i.e. after the issuer saw
  // tile j's phase.
  uint64_t* p_full = s_full + 2;  // [tile & 1]
  uint64_t* pv_done = p_full + 2;
  uint64_t* mma_done = pv_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  // grid (Hq, B, q-tiles) with the q-tile index slowest and reversed: the
  // heaviest causal tiles (most keys) are scheduled first, the light ones
  // fill in behind them
  const int hq = blockIdx.x;
  const int b = blockIdx.y;
  const int kvh = hq / p.group;
  const int q0 = (gridDim.z - 1 - blockIdx.z) * kRows;
  // the tensor maps are launch parameters: fetch them while the predecessor
  // grid drains
  if (tid == 0) {
    prefetch_tmap(&qmap);
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
  }
  // this row's real query count (right padding beyond it is not written)
  pdl_wait();
  const int T = p.q_lens ? min(max(p.q_lens[b], 0), p.T) : p.T;
  const DevErr err{p.err};

  int kv_len = max(p.kv_lens[b], 0);
  const int32_t* trow = nullptr;
  if constexpr (kPaged) {
    const int row = p.rows ? p.rows[b] : b;
    trow = p.tables + static_cast<int64_t>(row) * p.pitch;
    if (kv_len > p.pitch * kBlockTokens) {
      if (tid == 0 && q0 == 0 && hq == 0) err.raise(PKV_DEVERR_POSITION);
      kv_len = static_cast<int>(p.pitch) * kBlockTokens;
    }
  }
  const int offset = kv_len - T;
  int kv_end = kv_len;
  if (p.causal) kv_end = min(kv_len, min(q0 + kRows, T) + offset);
  kv_end = max(kv_end, 0);
  const int nblk = (kv_end + kBlockTokens - 1) / kBlockTokens;
  const int ntiles = (nblk + kTileBlocks - 1) / kTileBlocks;

  if (ntiles == 0) {
    // no visible key for any row of this tile (e.g. left padding): 0/0 rows,
    // as the reference, without touching TMEM
    const uint32_t nan2 = 0x7fc07fc0u;  // two bf16 quiet NaNs
    const uint4 nv = make_uint4(nan2, nan2, nan2, nan2);
    for (int i = tid; i < kRows * 16; i += kThreads) {
      const int qi = q0 + i / 16;
      if (qi < T)
        *reinterpret_cast<uint4*>(p.out + b * p.o_sb + hq * p.o_sh +
                                  static_cast<int64_t>(qi) * p.o_st + (i % 16) * 8) = nv;
    }
    return;
  }

  // ---- producer helpers (used by thread 0 only: warp 0 lane 0 issues every
  // TMA load).  A tile's eight block ids are loaded together one tile ahead,
  // so table reads never serialise the issue.
  const uint64_t keep = policy_evict_last();
  auto fetch = [&](int j, int (&ids)[kTileBlocks]) {
    if constexpr (kPaged) {
#pragma unroll
      for (int jb = 0; jb < kTileBlocks; ++jb) {
        const int lb = j * kTileBlocks + jb;
        // blocks past the row's end load the row's first block: finite
        // data, masked out of S and never multiplied into O
        ids[jb] = trow[lb < nblk ? lb : 0];
      }
#pragma unroll
      for (int jb = 0; jb < kTileBlocks; ++jb) {
        if (ids[jb] < 0 || ids[jb] >= p.num_blocks) {
          err.raise(PKV_DEVERR_BLOCK_ID);
          ids[jb] = 0;
        }
      }
    }
  };
  // K runs one tile ahead of V: issue K(j+1), then V(j)
  auto issue = [&](int j, const int (&ids)[kTileBlocks], bool is_v) -> bool {
    const int st = j % kStages;
    uint64_t* full = is_v ? &v_full[st] : &k_full[st];
    uint64_t* empty = is_v ? &v_empty[st] : &k_empty[st];
    if (j >= kStages && !mbar_wait(empty, ((j / kStages) - 1) & 1, err)) return false;
    uint8_t* dst = smem + kOffKV + st * 2 * kOperand + (is_v ? kOperand : 0);
    const CUtensorMap* map = is_v ? &vmap : &kmap;
    mbar_arrive_expect_tx(full, kOperand);
#pragma unroll
    for (int jb = 0; jb < kTileBlocks; ++jb) {
      if constexpr (kPaged) {
        const int slot = ids[jb] * kBlockTokens;
        tma_load_3d(dst + jb * 2048, map, full, 0, kvh, slot, keep);
        tma_load_3d(dst + kRegion + jb * 2048, map, full, 64, kvh, slot, keep);
      } else {
        const int tok = (j * kTileBlocks + jb) * kBlockTokens;
        tma_load_4d(dst + jb * 2048, map, full, 0, tok, kvh, b, keep);
        tma_load_4d(dst + kRegion + jb * 2048, map, full, 64, tok, kvh, b, keep);
      }
    }
    return true;
  };
  int idk[kTileBlocks] = {}, idv[kTileBlocks] = {};
  bool first_ok = false;

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 1);   // producer's arrive.expect_tx
      mbar_init(&k_empty[s], 1);  // tcgen05.commit after the tile's Q.K^T
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);  // tcgen05.commit after the tile's P.V
    }
    for (int s = 0; s < 2; ++s) mbar_init(&s_full[s], 1);  // tcgen05.commit after Q.K^T
    for (int s = 0; s < 2; ++s) mbar_init(&p_full[s], 4);
    mbar_init(pv_done, 1);
    mbar_init(mma_done, 1);
    fence_mbar_init();
    // Q and the first K tile are requested before the TMEM allocation and
    // the CTA barrier, so their latency overlaps the set-up; Q goes first,
    // so its load overlaps the block-table read that K(0) depends on
    mbar_arrive_expect_tx(q_full, kOperand);
    tma_load_4d(smem + kOffQ, &qmap, q_full, 0, q0, hq, b, keep);
    tma_load_4d(smem + kOffQ + kRegion, &qmap, q_full, 64, q0, hq, b, keep);
    fetch(0, idk);
    first_ok = issue(0, idk, false);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();  // dependents launch once this CTA holds its TMEM
  const uint32_t tmem = *tmem_slot;
  const uint32_t sQ = smem_u32(smem + kOffQ);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      if (first_ok) {
        for (int j = 0; j < ntiles; ++j) {
#pragma unroll
          for (int jb = 0; jb < kTileBlocks; ++jb) idv[jb] = idk[jb];
          if (j + 1 < ntiles) {
            fetch(j + 1, idk);
            if (!issue(j + 1, idk, false)) break;
          }
          if (!kSplitProducer && !issue(j, idv, true)) break;
        }
      }
    }
  } else if (kSplitProducer && warp == 6) {
    // ------------------------------------------------------------ V producer
    if (lane == 0) {
      for (int j = 0; j < ntiles; ++j) {
        fetch(j, idv);
        if (!issue(j, idv, true)) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool dead = !mbar_wait(q_full, 0, err);
      auto issue_pv = [&](int i) -> bool {
        if (!mbar_wait(&p_full[i & 1], (i >> 1) & 1, err)) return false;
        const int st = i % kStages;
        if (!mbar_wait(&v_full[st], (i / kStages) & 1, err)) return false;
        tc_fence_after();
        const uint32_t sV = smem_u32(smem + kOffKV + st * 2 * kOperand + kOperand);
        const uint32_t pS = tmem + ((i & 1) ? kColS1 : kColS0);  // P(i): 8 columns per 16 keys
        const int nb = min(kTileBlocks, nblk - i * kTileBlocks);
        for (int kb = 0; kb < nb; ++kb) {
          umma_ts(tmem + kColO, pS + kb * 8, sdesc(sV + kb * 2048, kRegion, 1024), kIdescPV,
                  (i > 0 || kb > 0) ? 1u : 0u);
        }
        umma_commit(pv_done);
        umma_commit(&v_empty[st]);
        return true;
      };
      for (int j = 0; j < ntiles && !dead; ++j) {
        const int st = j % kStages;
        const int sb = j & 1;
        if (!mbar_wait(&k_full[st], (j / kStages) & 1, err)) {
          dead = true;
          break;
        }
        tc_fence_after();
        const uint32_t sK = smem_u32(smem + kOffKV + st * 2 * kOperand);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma(tmem + (sb ? kColS1 : kColS0), kmajor_desc(sQ, kk), kmajor_desc(sK, kk), kIdescQK,
               kk > 0 ? 1u : 0u);
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[st]);
        if (j >= 1 && !issue_pv(j - 1)) {
          dead = true;
          break;
        }
      }
      if (!dead) issue_pv(ntiles - 1);
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, err);  // every MMA retired before TMEM is freed
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile == TMEM lane
    const int qi = q0 + r;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const int lim = p.causal ? min(kv_len, qi + offset + 1) : kv_len;  // keys < lim visible
    float m = -INFINITY, l = 0.f;
    bool dead = false;
    for (int j = 0; j < ntiles && !dead; ++j) {
      const int sb = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[sb], (j >> 1) & 1, err))) {
        dead = true;
        break;
      }
      tc_fence_after();
      float s[128];
      tmem_ld32x4_sync(lane_addr + (sb ? kColS1 : kColS0), s);

      const int key0 = j * kKeys;
      // Row max of the raw scores (scale_log2 > 0 commutes with max), as 8
      // independent partial maxima instead of one 128-long dependency chain.
      float pm[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) pm[u] = -INFINITY;
      if (key0 + kKeys <= lim) {
#pragma unroll
        for (int i = 0; i < 128; ++i) pm[i & 7] = fmaxf(pm[i & 7], s[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 128; ++i) {
          if (key0 + i >= lim) s[i] = -INFINITY;
          pm[i & 7] = fmaxf(pm[i & 7], s[i]);
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                             fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7]))) *
                       p.scale_log2;
      // Lazy rescaling: keep the running max unless this tile raises it by
      // more than 2^8 (P <= 256 then, exact in fp32 and bf16-representable);
      // O is rescaled in TMEM only when some row of the warp moved its max.
      float mn = m;
      if (mx > m + kRescaleThreshold || m == -INFINITY) mn = mx;
      const float base = mn == -INFINITY ? 0.f : mn;
      const float alpha = (mn == m) ? 1.f : ex2(m - base);
      // p = 2^(s*scale - base): scale and shift in one FMA; the row sum as 8
      // partial sums
      float ps[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) ps[u] = 0.f;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        s[i] = ex2(fmaf(s[i], p.scale_log2, -base));
        ps[i & 7] += s[i];
      }
      const float rs = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
      l = l * alpha + rs;
      m = mn;
      const bool rescale = __any_sync(0xffffffffu, alpha != 1.f);
      // O is stable once the previous tile's P.V retired
      if (j >= 1 && rescale) {
        if (!__all_sync(0xffffffffu, mbar_wait(pv_done, (j - 1) & 1, err))) {
          dead = true;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32_sync(lane_addr + kColO + c * 32, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tmem_st32(lane_addr + kColO + c * 32, v);
        }
      }
      // P(j) as bf16 pairs over columns [0, 64) of S[sb] (already read)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack_bf16(s[c * 32 + 2 * i], s[c * 32 + 2 * i + 1]);
        tmem_st16u(lane_addr + (sb ? kColS1 : kColS0) + c * 16, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
    }
    // ------------------------------------------------------------ epilogue
    // tcgen05.ld is warp-collective: every lane loads, only rows < T store
    // every product retired: the softmax skips P.V waits on tiles without a
    // rescale, so pv_done may be two phases behind here; mma_done is
    // committed once, after the last P.V
    bool have = !dead;
    if (have) have = __all_sync(0xffffffffu, mbar_wait(mma_done, 0, err));
    __nv_bfloat16* orow =
        p.out + b * p.o_sb + hq * p.o_sh + static_cast<int64_t>(min(qi, T - 1)) * p.o_st;
    if (have) {
      tc_fence_after();
      const float inv = 1.f / l;  // 0/0 -> NaN for a row with no visible key
      float v[4][32];  // all of O's row, one wait
      tmem_ld32x4_sync(lane_addr + kColO, *reinterpret_cast<float(*)[128]>(&v[0][0]));
      // direct row stores: staging through shared memory (store_o_rows, as
      // the head-pair kernel does) cost this kernel two registers and ~5%
      // of its main-loop speed on every measured shape
      if (qi < T) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 pk;
            pk.x = pack_bf16(v[c][e + 0] * inv, v[c][e + 1] * inv);
            pk.y = pack_bf16(v[c][e + 2] * inv, v[c][e + 3] * inv);
            pk.z = pack_bf16(v[c][e + 4] * inv, v[c][e + 5] * inv);
            pk.w = pack_bf16(v[c][e + 6] * inv, v[c][e + 7] * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + e) = pk;
          }
        }
      }
    } else if (qi < T) {
      // a timed-out wait: NaN rows rather than stale data
      const uint32_t nan2 = 0x7fc07fc0u;
      const uint4 nv = make_uint4(nan2, nan2, nan2, nan2);
#pragma unroll
      for (int e = 0; e < 128; e += 8) *reinterpret_cast<uint4*>(orow + e) = nv;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------- head pairs
// Two query heads of one KV group per CTA (GQA groups of even size): the K/V
// tiles are loaded once for both, halving the L2 -> SM traffic per head-tile
// that sets the tile period of the one-head kernel.  Warp 0 TMA, warp 1 MMA,
// warps 4-7 softmax of head A, warps 8-11 softmax of head B (each warpgroup
// covers the four TMEM lane quarters).  TMEM: S_A, S_B, O_A, O_B.
// One shared P buffer is filled in a fixed order (P_A(j), then P_B(j) once
// P.V_A(j) retired, then P_A(j+1) once P.V_B(j) retired), so shared memory
// holds both Q tiles, two K and two V stages and P (224 KiB); Q.K^T of the
// next tile is issued before the current tile's two P.V products, so the
// exponentials of tile j+1 overlap the P.V chain of tile j.
// 12 warps in three warpgroups, registers split with setmaxnreg: warpgroup
// 0 (warp 0 TMA, warp 1 MMA, warps 2-3 idle) drops to kPairRegsLow, the
// softmax warpgroups (warps 4-7 head A, 8-11 head B) rise to kPairRegsHigh.
// Launched at kPairRegsLaunch per thread: 384 x 168 = 64512 >= 128 x 80 +
// 256 x 208 = 63488 (the producer and MMA code spills below 80); the host
// launches the kernel only when
// the compiled kernel has exactly kPairRegsLaunch registers, so the split
// always fits what the block was given.  (10 warps without the split put
// three warps on one SM sub-partition, capping every thread at ~170
// registers, where the softmax spilled.)
constexpr int kPairThreads = 384;
constexpr int kPairRegsLaunch = 168;
constexpr int kPairRegsLow = 80;
constexpr int kPairRegsHigh = 208;
static_assert(128 * kPairRegsLow + 256 * kPairRegsHigh <= kPairThreads * kPairRegsLaunch,
              "register split exceeds the launch allocation");
constexpr uint32_t kPColSA = 0, kPColSB = 128, kPColOA = 256, kPColOB = 384;
constexpr int kPOffQ = 0;                          // Q_A, Q_B: 2 x 32 KiB
constexpr int kPOffK = kPOffQ + 2 * kOperand;      // K stage s at +s*32 KiB
constexpr int kPOffV = kPOffK + kStages * kOperand;
constexpr int kPOffP = kPOffV + kStages * kOperand;
constexpr int kPOffBar = kPOffP + kOperand;
constexpr int kPNumBars = 1 + 4 * kStages + 2 * 5 + 1;
constexpr int kPSmemBytes = kPOffBar + kPNumBars * 8 + 16 + 1024;
static_assert(kPSmemBytes <= 227 * 1024, "paired prefill shared memory exceeds the per-CTA limit");

template <bool kPaged>
__global__ void __launch_bounds__(kPairThreads, 1)
    prefill_tc_pair_kernel(const TcParams p, const __grid_constant__ CUtensorMap qmap,
                           const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPOffBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + kStages;
  uint64_t* v_full = k_empty + kStages;
  uint64_t* v_empty = v_full + kStages;
  uint64_t* s_full = v_empty + kStages;  // [head]
  uint64_t* s_free = s_full + 2;         // [head], one arrival per softmax warp
  uint64_t* p_full = s_free + 2;         // [head], one arrival per softmax warp
  uint64_t* pv_done = p_full + 2;        // [head]
  uint64_t* mma_done = pv_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kPNumBars);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int hq0 = 2 * blockIdx.x;  // heads hq0 (A) and hq0 + 1 (B), same KV head
  const int b = blockIdx.y;
  const int kvh = hq0 / p.group;
  const int q0 = (gridDim.z - 1 - blockIdx.z) * kRows;  // heaviest q-tiles first
  if (tid == 0) {  // launch parameters: fetched while the predecessor drains
    prefetch_tmap(&qmap);
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
  }
  pdl_wait();
  const int T = p.q_lens ? min(max(p.q_lens[b], 0), p.T) : p.T;
  const DevErr err{p.err};

  int kv_len = max(p.kv_lens[b], 0);
  const int32_t* trow = nullptr;
  if constexpr (kPaged) {
    const int row = p.rows ? p.rows[b] : b;
    trow = p.tables + static_cast<int64_t>(row) * p.pitch;
    if (kv_len > p.pitch * kBlockTokens) {
      if (tid == 0 && q0 == 0 && hq0 == 0) err.raise(PKV_DEVERR_POSITION);
      kv_len = static_cast<int>(p.pitch) * kBlockTokens;
    }
  }
  const int offset = kv_len - T;
  int kv_end = kv_len;
  if (p.causal) kv_end = min(kv_len, min(q0 + kRows, T) + offset);
  kv_end = max(kv_end, 0);
  const int nblk = (kv_end + kBlockTokens - 1) / kBlockTokens;
  const int ntiles = (nblk + kTileBlocks - 1) / kTileBlocks;

  if (ntiles == 0) {
    // no visible key for any row of this tile: 0/0 rows, as the reference
    const uint32_t nan2 = 0x7fc07fc0u;
    const uint4 nv = make_uint4(nan2, nan2, nan2, nan2);
    for (int i = tid; i < 2 * kRows * 16; i += kPairThreads) {
      const int hh = i / (kRows * 16), r = (i / 16) % kRows, c = i % 16;
      const int qi = q0 + r;
      if (qi < T)
        *reinterpret_cast<uint4*>(p.out + b * p.o_sb + (hq0 + hh) * p.o_sh +
                                  static_cast<int64_t>(qi) * p.o_st + c * 8) = nv;
    }
    return;
  }

  // ---- producer helpers (thread 0, warp 0 lane 0, issues every TMA load)
  const uint64_t keep = policy_evict_last();
  auto fetch = [&](int j, int (&ids)[kTileBlocks]) {
    if constexpr (kPaged) {
#pragma unroll
      for (int jb = 0; jb < kTileBlocks; ++jb) {
        const int lb = j * kTileBlocks + jb;
        ids[jb] = trow[lb < nblk ? lb : 0];  // past the end: finite, masked
      }
#pragma unroll
      for (int jb = 0; jb < kTileBlocks; ++jb) {
        if (ids[jb] < 0 || ids[jb] >= p.num_blocks) {
          err.raise(PKV_DEVERR_BLOCK_ID);
          ids[jb] = 0;
        }
      }
    }
  };
  auto issue = [&](int j, const int (&ids)[kTileBlocks], bool is_v) -> bool {
    const int st = j % kStages;
    uint64_t* full = is_v ? &v_full[st] : &k_full[st];
    uint64_t* empty = is_v ? &v_empty[st] : &k_empty[st];
    if (j >= kStages && !mbar_wait(empty, ((j / kStages) - 1) & 1, err)) return false;
    uint8_t* dst = smem + (is_v ? kPOffV : kPOffK) + st * kOperand;
    const CUtensorMap* map = is_v ? &vmap : &kmap;
    mbar_arrive_expect_tx(full, kOperand);
#pragma unroll
    for (int jb = 0; jb < kTileBlocks; ++jb) {
      if constexpr (kPaged) {
        const int slot = ids[jb] * kBlockTokens;
        tma_load_3d(dst + jb * 2048, map, full, 0, kvh, slot, keep);
        tma_load_3d(dst + kRegion + jb * 2048, map, full, 64, kvh, slot, keep);
      } else {
        const int tok = (j * kTileBlocks + jb) * kBlockTokens;
        tma_load_4d(dst + jb * 2048, map, full, 0, tok, kvh, b, keep);
        tma_load_4d(dst + kRegion + jb * 2048, map, full, 64, tok, kvh, b, keep);
      }
    }
    return true;
  };
  int idk[kTileBlocks] = {}, idv[kTileBlocks] = {};
  bool first_ok = false;

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&s_full[h], 1);
      mbar_init(&s_free[h], 4);
      mbar_init(&p_full[h], 4);
      mbar_init(&pv_done[h], 1);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
    // both Q tiles and the first K tile are requested before the TMEM
    // allocation and the CTA barrier, so their latency overlaps the set-up;
    // Q goes first, overlapping the block-table read that K(0) depends on
    mbar_arrive_expect_tx(q_full, 2 * kOperand);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint8_t* qd = smem + kPOffQ + h * kOperand;
      tma_load_4d(qd, &qmap, q_full, 0, q0, hq0 + h, b, keep);
      tma_load_4d(qd + kRegion, &qmap, q_full, 64, q0, hq0 + h, b, keep);
    }
    fetch(0, idk);
    first_ok = issue(0, idk, false);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();  // dependents launch once this CTA holds its TMEM
  const uint32_t tmem = *tmem_slot;
  const uint32_t sP = smem_u32(smem + kPOffP);

  // Each role's code sits inside the branch that set its register limit, so
  // the compiler allocates that role's registers under that limit.
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kPairRegsLow));
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      if (first_ok) {
        for (int j = 0; j < ntiles; ++j) {
#pragma unroll
          for (int jb = 0; jb < kTileBlocks; ++jb) idv[jb] = idk[jb];
          if (j + 1 < ntiles) {
            fetch(j + 1, idk);
            if (!issue(j + 1, idk, false)) break;
          }
          if (!issue(j, idv, true)) break;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool dead = !mbar_wait(q_full, 0, err);
      const uint32_t sQA = smem_u32(smem + kPOffQ), sQB = sQA + kOperand;
      auto issue_qk = [&](int j) -> bool {
        const int st = j % kStages;
        if (!mbar_wait(&k_full[st], (j / kStages) & 1, err)) return false;
        const uint32_t sK = smem_u32(smem + kPOffK + st * kOperand);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          // S_h is free once softmax h read tile j-1's scores
          if (j >= 1 && !mbar_wait(&s_free[h], (j - 1) & 1, err)) return false;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma(tmem + (h ? kPColSB : kPColSA), kmajor_desc(h ? sQB : sQA, kk),
                 kmajor_desc(sK, kk), kIdescQK, kk > 0 ? 1u : 0u);
          umma_commit(&s_full[h]);
        }
        umma_commit(&k_empty[st]);
        return true;
      };
      auto issue_pv = [&](int j, int h) -> bool {
        if (!mbar_wait(&p_full[h], j & 1, err)) return false;
        const int st = j % kStages;
        if (h == 0 && !mbar_wait(&v_full[st], (j / kStages) & 1, err)) return false;
        tc_fence_after();
        const uint32_t sV = smem_u32(smem + kPOffV + st * kOperand);
        const int nb = min(kTileBlocks, nblk - j * kTileBlocks);
        for (int kb = 0; kb < nb; ++kb)
          umma(tmem + (h ? kPColOB : kPColOA), kmajor_desc(sP, kb),
               sdesc(sV + kb * 2048, kRegion, 1024), kIdescPV, (j > 0 || kb > 0) ? 1u : 0u);
        umma_commit(&pv_done[h]);
        if (h == 1) umma_commit(&v_empty[st]);
        return true;
      };
      if (!dead) dead = !issue_qk(0);
      for (int j = 0; j < ntiles && !dead; ++j) {
        if (j + 1 < ntiles && !issue_qk(j + 1)) {
          dead = true;
          break;
        }
        if (!issue_pv(j, 0) || !issue_pv(j, 1)) {
          dead = true;
          break;
        }
      }
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, err);  // every MMA retired before TMEM is freed
    }
  }  // warps 2-3: register donors only
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kPairRegsHigh));
    // ------------------------------------------------------------ softmax
    const int h = warp >= 8 ? 1 : 0;  // warps 4-7: head A, 8-11: head B
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile == TMEM lane
    const int qi = q0 + r;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t colS = h ? kPColSB : kPColSA, colO = h ? kPColOB : kPColOA;
    const int lim = p.causal ? min(kv_len, qi + offset + 1) : kv_len;  // keys < lim visible
    float m = -INFINITY, l = 0.f;
    bool dead = false;
    for (int j = 0; j < ntiles && !dead; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[h], j & 1, err))) {
        dead = true;
        break;
      }
      tc_fence_after();
      float s[128];
      tmem_ld32x4_sync(lane_addr + colS, s);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[h]);

      const int key0 = j * kKeys;
      float pm[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) pm[u] = -INFINITY;
      if (key0 + kKeys <= lim) {
#pragma unroll
        for (int i = 0; i < 128; ++i) pm[i & 7] = fmaxf(pm[i & 7], s[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 128; ++i) {
          if (key0 + i >= lim) s[i] = -INFINITY;
          pm[i & 7] = fmaxf(pm[i & 7], s[i]);
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                             fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7]))) *
                       p.scale_log2;
      float mn = m;
      if (mx > m + kRescaleThreshold || m == -INFINITY) mn = mx;
      const float base = mn == -INFINITY ? 0.f : mn;
      const float alpha = (mn == m) ? 1.f : ex2(m - base);
      float ps[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) ps[u] = 0.f;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        s[i] = ex2(fmaf(s[i], p.scale_log2, -base));
        ps[i & 7] += s[i];
      }
      const float rs = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
      l = l * alpha + rs;
      m = mn;
      const bool rescale = __any_sync(0xffffffffu, alpha != 1.f);
      // The shared P buffer is free (and O_h stable) once the product
      // before this one in the order P_A(j), P_B(j), P_A(j+1) retired:
      // head A waits P.V_B(j-1), head B waits P.V_A(j)
      bool ok = true;
      if (h == 0) {
        if (j >= 1) ok = mbar_wait(&pv_done[1], (j - 1) & 1, err);
      } else {
        ok = mbar_wait(&pv_done[0], j & 1, err);
      }
      if (!__all_sync(0xffffffffu, ok)) {
        dead = true;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int reg = 0; reg < 2; ++reg) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int k = reg * 64 + c * 8;
          uint4 pk;
          pk.x = pack_bf16(s[k + 0], s[k + 1]);
          pk.y = pack_bf16(s[k + 2], s[k + 3]);
          pk.z = pack_bf16(s[k + 4], s[k + 5]);
          pk.w = pack_bf16(s[k + 6], s[k + 7]);
          *reinterpret_cast<uint4*>(smem + kPOffP + reg * kRegion + swz128(r, c)) = pk;
        }
      }
      fence_async_smem();
      if (j >= 1 && rescale) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32_sync(lane_addr + colO + c * 32, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tmem_st32(lane_addr + colO + c * 32, v);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[h]);
    }
    // ------------------------------------------------------------ epilogue
    bool have = !dead;
    if (have) have = __all_sync(0xffffffffu, mbar_wait(&pv_done[h], (ntiles - 1) & 1, err));
    __nv_bfloat16* orow = p.out + b * p.o_sb + (hq0 + h) * p.o_sh +
                          static_cast<int64_t>(min(qi, T - 1)) * p.o_st;
    if (have) {
      tc_fence_after();
      const float inv = 1.f / l;  // 0/0 -> NaN for a row with no visible key
      float v[4][32];  // all of O's row, one wait
      tmem_ld32x4_sync(lane_addr + colO, *reinterpret_cast<float(*)[128]>(&v[0][0]));
      // Q_h is free: pv_done[h] of the last tile retired every earlier MMA,
      // this head's Q.K^T products included
      const int w0 = q0 + quarter * 32;
      store_o_rows(smem + kPOffQ + h * kOperand + quarter * 8192, v, inv, lane,
                   p.out + b * p.o_sb + (hq0 + h) * p.o_sh + static_cast<int64_t>(w0) * p.o_st,
                   p.o_st, T - w0);
    } else if (qi < T) {
      const uint32_t nan2 = 0x7fc07fc0u;  // a timed-out wait: NaN rows, not stale data
      const uint4 nv = make_uint4(nan2, nan2, nan2, nan2);
#pragma unroll
      for (int e = 0; e < 128; e += 8) *reinterpret_cast<uint4*>(orow + e) = nv;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

enum class TcKernel { kOneHead, kHeadPair };

template <bool kPaged, TcKernel kKind>
cudaError_t launch_tc_t(const TcParams& prm, const CUtensorMap& qmap, const KVSource& src,
                        dim3 grid, cudaStream_t stream) {
  constexpr bool kPair = kKind == TcKernel::kHeadPair;
  auto kern = kPair ? prefill_tc_pair_kernel<kPaged> : prefill_tc_kernel<kPaged>;
  const int smem = kPair ? kPSmemBytes : kSmemBytes;
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
  return launch_k(kern, grid, dim3(kPair ? kPairThreads : kThreads), static_cast<size_t>(smem),
                  stream, prm, qmap, src.kmap, src.vmap);
}

// The head-pair kernel's register split assumes the block was launched with
// exactly kPairRegsLaunch registers per thread (setmaxnreg.inc draws on that
// allocation); a build where the compiler chose another count must not run it.
bool pair_kernel_usable() {
  static int ok = -1;
  if (ok < 0) {
    cudaFuncAttributes a0{}, a1{};
    ok = cudaFuncGetAttributes(&a0, prefill_tc_pair_kernel<false>) == cudaSuccess &&
         cudaFuncGetAttributes(&a1, prefill_tc_pair_kernel<true>) == cudaSuccess &&
         a0.numRegs == kPairRegsLaunch && a1.numRegs == kPairRegsLaunch;
    if (!ok) cudaGetLastError();
  }
  return ok == 1;
}

template <TcKernel kKind>
cudaError_t launch_tc_kind(const TcParams& prm, const CUtensorMap& qmap, const KVSource& src,
                           dim3 grid, cudaStream_t stream) {
  return src.paged ? launch_tc_t<true, kKind>(prm, qmap, src, grid, stream)
                   : launch_tc_t<false, kKind>(prm, qmap, src, grid, stream);
}

}  // namespace

cudaError_t launch_prefill_tc(const PrefillLaunch& a, const CUtensorMap& qmap, const KVSource& src,
                              cudaStream_t stream) {
  TcParams prm{};
  prm.out = static_cast<__nv_bfloat16*>(a.out);
  prm.o_sb = a.o_sb;
  prm.o_sh = a.o_sh;
  prm.o_st = a.o_st;
  prm.kv_lens = a.kv_lens;
  prm.q_lens = a.q_lens;
  prm.tables = src.tables;
  prm.pitch = src.pitch;
  prm.rows = src.rows;
  prm.num_blocks = src.num_blocks;
  prm.T = a.seq_len_q;
  prm.group = a.num_q_heads / a.num_kv_heads;
  prm.causal = a.causal;
  prm.scale_log2 = a.sm_scale * 1.4426950408889634f;
  prm.err = a.err;
  const unsigned qtiles = (a.seq_len_q + kRows - 1) / kRows;
  // Head pairs share their K/V tiles and overlap one head's exponentials
  // with the other's products, but stage P through shared memory and keep
  // one S buffer per head; the one-head kernel double-buffers S and keeps P
  // in tensor memory.  Measured: pairs are 1-4% faster while every row is
  // at most 1024 tokens (8 q-tiles) and the paired grid covers the SMs
  // (config 1, 8 x 768, 8 x 1024); one head per CTA is 7-20% faster on
  // longer rows (8 x 2048, 2 x 4096, 1 x 16384).  PKV_PREFILL_KERNEL=one|pair
  // pins a kernel (pair needs an even GQA group).
  int sms = 148;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int64_t pair_ctas = static_cast<int64_t>(a.num_q_heads / 2) * a.batch * qtiles;
  TcKernel kind = (prm.group % 2 == 0 && qtiles <= 8 && pair_ctas >= sms) ? TcKernel::kHeadPair
                                                                          : TcKernel::kOneHead;
  if (const char* force = getenv("PKV_PREFILL_KERNEL")) {
    if (!strcmp(force, "one")) kind = TcKernel::kOneHead;
    if (!strcmp(force, "pair") && prm.group % 2 == 0) kind = TcKernel::kHeadPair;
  }
  if (kind == TcKernel::kHeadPair && !pair_kernel_usable()) kind = TcKernel::kOneHead;
  if (kind == TcKernel::kHeadPair)
    return launch_tc_kind<TcKernel::kHeadPair>(prm, qmap, src,
                                               dim3(a.num_q_heads / 2, a.batch, qtiles), stream);
  return launch_tc_kind<TcKernel::kOneHead>(prm, qmap, src,
                                            dim3(a.num_q_heads, a.batch, qtiles), stream);
}

}  // namespace pkv
