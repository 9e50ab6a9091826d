// The decoder layers of one decode step (T = 1, up to 32 rows) as ONE
// persistent launch on sm_100a: one CTA per SM runs all 28 layers.
//
// Reference behaviour: the per-layer op sequence of model.py:131-138 with the
// attention of model.py:88-108 (q/k/v projections + bias, RoPE, K/V write
// into the paged cache kv_cache.py:86-101, attention over the row's blocks,
// o_proj, residual add + RMSNorm, SwiGLU MLP, residual add + RMSNorm), for a
// step whose rows each add one token.  The same arithmetic and bf16 rounding
// points as the per-op kernels (linear_tc.cu, append.cu, decode.cu,
// fused.cu); what changes is that a small decode step is one launch instead
// of ~170 dependent ones, so the weight stream never stops at a kernel
// boundary.
//
// Per layer, five phases separated by grid-wide barriers:
//   QKV   h . Wqkv^T + b, RoPE, K/V rows into the pool, q_rot to global
//   ATT   paged decode attention (mma.sync, split over partitions)
//   O     att . Wo^T, xs += o, per-tile sums of squares of xs
//   GU    rmsnorm(xs) . Wgu^T (paired gate/up tiles), SwiGLU -> act
//   DOWN  act . Wd^T, xs += d (last layer: the MLP output itself)
// Every GEMM phase splits its (128-row W tile, 64-wide K chunk) units evenly
// over the CTAs (CTA c owns units [ceil(cU/G), ceil((c+1)U/G))); a CTA's
// range covers at most two tiles.  Each tile segment accumulates in TMEM
// (tcgen05.mma, W as the M=128 side, the step's rows as N), is written as an
// fp32 partial, and the last CTA to finish a tile (an atomic counter) sums
// the tile's partials in CTA order (deterministic) and applies the tile's
// epilogue.  The next phase's activations are built in shared memory by the
// CTA itself (the RMSNorm folded into that load from the per-tile sums of
// squares), so no phase needs a separate normalisation pass.
//
//   block = 6 warps
//     warp 0     TMA producer: streams this CTA's W boxes for every phase of
//                every layer through an NW-deep ring.  The weights do not
//                depend on the activations, so the ring keeps filling across
//                the barriers and the attention phase.
//     warp 1     TMEM owner and MMA issuer (two accumulators, Mpad columns
//                each, so a segment's epilogue overlaps the next segment)
//     warps 2-5  workers: activation loads, TMEM epilogues, tile reductions,
//                the attention phase, the grid barriers
// Every wait is bounded; a timeout raises PKV_DEVERR_TIMEOUT and sets an
// abort word that every other wait polls, so the whole grid leaves quickly,
// after draining its own copies in flight and freeing its TMEM.
#include <mutex>

#include "pkv_device.cuh"
#include "pkv_kernels.h"
#include "tc_device.cuh"

namespace pkv {
namespace {

constexpr int kHid = 1536;
constexpr int kInter = 8960;
constexpr int kQkvN = 2048;
constexpr int kHq = 12;
constexpr int kHkv = 2;
constexpr int kGroup = kHq / kHkv;
constexpr int kLThreads = 192;
constexpr int kWBox = 128 * 128;  // 128 W rows x 64 K bf16 = 16 KiB, 128B-swizzled
constexpr int kAttWarps = 4;
constexpr int kAttStages = 2;
constexpr int kAttStageBytes = 2 * kHeadBlockBytes;  // K + V of one head, one block
constexpr int kAttRingBytes = kAttWarps * kAttStages * kAttStageBytes;
constexpr int kMaxTiles = 2 * kInter / 128;  // 140 (gate/up)
constexpr uint32_t kGridSpin = 1u << 22;

enum { kSQkv = 0, kSO = 1, kSGu = 2, kSDown = 3 };

__host__ __device__ constexpr int stage_tiles(int s) {
  return s == kSQkv ? kQkvN / 128 : s == kSGu ? 2 * kInter / 128 : kHid / 128;
}
__host__ __device__ constexpr int stage_chunks(int s) { return s == kSDown ? kInter / 64 : kHid / 64; }

// 32-bit: c * U and u * G stay below 2^31 for these shapes (U <= 3360,
// G <= a few hundred SMs)
__host__ __device__ inline int unit_begin(int c, int U, int G) { return (c * U + G - 1) / G; }
__host__ __device__ inline int unit_owner(int u, int U, int G) { return (u * G) / U; }

__device__ __forceinline__ float bf(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 rn(float x) { return __float2bfloat16_rn(x); }
__device__ __forceinline__ float rope1(float x, float c, float r, float sn) {
  return bf(rn(__fadd_rn(bf(rn(__fmul_rn(x, c))), bf(rn(__fmul_rn(r, sn))))));
}
__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// generic-proxy global writes <-> async-proxy (TMA) global reads
__device__ __forceinline__ void fence_proxy_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void workers_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

struct LayersShared {
  uint32_t tmem;
  int flag;         // broadcast: last arriver / abort decisions
  float rnorm[32];  // per-row 1 / rms of the phase's normalised input
  int seg_off[64];  // float4 offset of each partial a tile gather reads
};

// Bounded mbarrier wait that also gives up once another CTA has aborted.
__device__ bool wait_bar(uint64_t* bar, uint32_t parity, const uint32_t* abort_word,
                         const DevErr& err) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_test(bar, parity)) return true;
    if ((i & 1023u) == 1023u && ld_volatile(abort_word)) return false;
  }
  err.raise(PKV_DEVERR_TIMEOUT);
  atomicExch(const_cast<uint32_t*>(abort_word), 1u);
  return false;
}

template <int MPAD>
struct Geo {
  static constexpr int kXSlot = MPAD * 128;  // one 64-wide K chunk of the rows, 128B-swizzled
  static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) |
                                     ((static_cast<uint32_t>(MPAD) >> 3) << 17) |
                                     ((128u >> 4) << 24);
};

// CTA c's first unit of phase s (it owns [stage_begin(c), stage_begin(c+1)))
// and the owner of unit u.  The gate/up phase gives each CTA one whole tile
// (140 tiles <= the grid), so its tiles need no cross-CTA reduction; the
// other phases spread their units evenly, CTA c owning
// [ceil(cU/G), ceil((c+1)U/G)).
__host__ __device__ inline int stage_begin(int s, int c, int G) {
  const int C = stage_chunks(s), T = stage_tiles(s);
  if (s == kSGu && T <= G) return min(c, T) * C;
  return unit_begin(c, T * C, G);
}
__host__ __device__ inline int stage_owner(int s, int u, int G) {
  const int C = stage_chunks(s), T = stage_tiles(s);
  if (s == kSGu && T <= G) return u / C;
  return unit_owner(u, T * C, G);
}

// One CTA's share of GEMM phase s: units [u0, u1), tiles t0..t1.
struct Range {
  int u0, u1, t0, t1;
};
__device__ __forceinline__ Range range_of(int s, int c, int G) {
  const int C = stage_chunks(s);
  Range r;
  r.u0 = stage_begin(s, c, G);
  r.u1 = stage_begin(s, c + 1, G);
  r.t0 = r.u0 / C;
  r.t1 = r.u1 > r.u0 ? (r.u1 - 1) / C : r.t0 - 1;
  return r;
}
// the reduced tile [32 rows][128] fp32 in shared memory
constexpr int kRedBytes = 32 * 128 * 4;

// Shared-memory carve-up, identical in every role (the dynamic block,
// 1024-aligned): W ring | x slots or the attention ring | reduced tile |
// mbarriers | LayersShared.
struct SmemMap {
  uint8_t* wring;
  uint8_t* xbuf;
  float* red;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* acc_full;   // [2]
  uint64_t* acc_empty;  // [2]
  uint64_t* x_full;
  uint64_t* mma_done;
  uint64_t* att_bar;    // [kAttWarps][kAttStages]
  LayersShared* sh;
};
template <int MPAD>
__device__ __forceinline__ SmemMap smem_map(const LayersParams& __restrict__ p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  SmemMap m;
  m.wring = smem;
  m.xbuf = smem + p.nw * kWBox;
  const int xbytes = max(p.xslots * Geo<MPAD>::kXSlot, kAttRingBytes);
  m.red = reinterpret_cast<float*>(m.xbuf + xbytes);
  m.full = reinterpret_cast<uint64_t*>(m.xbuf + xbytes + kRedBytes);
  m.empty = m.full + p.nw;
  m.acc_full = m.empty + p.nw;
  m.acc_empty = m.acc_full + 2;
  m.x_full = m.acc_empty + 2;
  m.mma_done = m.x_full + 1;
  m.att_bar = m.mma_done + 1;
  m.sh = reinterpret_cast<LayersShared*>(m.att_bar + kAttWarps * kAttStages);
  return m;
}

// The worker roles (warps 2-5) are separate functions, so each gets the
// whole register file: the attention loop, the tile gathers and the
// activation loads never compete for registers.  Each rebuilds its view of
// the block from the thread index and the shared-memory map.
#define LAYERS_WORKER_VIEW                                           \
  using Gm = Geo<MPAD>;                                              \
  const SmemMap sm = smem_map<MPAD>(p);                              \
  const int tid = threadIdx.x;                                       \
  const int warp = tid >> 5, lane = tid & 31;                        \
  const int wt = tid - 64, ww = warp - 2, q4 = warp & 3;             \
  const int c = blockIdx.x, G = p.G;                                 \
  const DevErr err{p.err};                                           \
  const uint32_t* abort_word = p.sync + 2;                           \
  uint8_t* xbuf = sm.xbuf;                                           \
  float* red = sm.red;                                               \
  LayersShared* sh = sm.sh;                                          \
  (void)sizeof(Gm);                                                  \
  (void)lane;                                                        \
  (void)wt;                                                          \
  (void)warp;                                                        \
  (void)ww;                                                          \
  (void)q4;                                                          \
  (void)c;                                                           \
  (void)G;                                                           \
  (void)err;                                                         \
  (void)abort_word;                                                  \
  (void)xbuf;                                                        \
  (void)red;                                                         \
  (void)sh

// Grid-wide barrier of the workers: all workers of this CTA, then one
// arrival per CTA on the arrival word; `target` = arrivals expected so far.
// Returns false once any CTA has aborted.
template <int MPAD>
__device__ __noinline__ bool w_grid_barrier(const LayersParams& __restrict__ p, uint32_t target) {
  LAYERS_WORKER_VIEW;

  __threadfence();
  workers_sync();
  if (wt == 0) {
    int ok = 0;
    if (!ld_volatile(abort_word)) {
      __threadfence();  // cumulative: the CTA's writes, ordered by the barrier above
      atomicAdd(p.sync, 1u);
      // poll with relaxed loads; the fence below orders what follows
      for (uint32_t i = 0; i < kGridSpin; ++i) {
        if (ld_volatile(p.sync) >= target) {
          ok = 1;
          break;
        }
        if ((i & 255u) == 255u && ld_volatile(abort_word)) break;
      }
      if (!ok && !ld_volatile(abort_word)) {
        err.raise(PKV_DEVERR_TIMEOUT);
        atomicExch(const_cast<uint32_t*>(abort_word), 1u);
      }
    }
    __threadfence();
    sh->flag = ok;
  }
  workers_sync();
  const bool alive = sh->flag != 0;
  workers_sync();
  return alive;
}

// x operand of GEMM phase s in layer l: this CTA's K chunks, one slot per
// unit, 128B-swizzled (16-byte group j of row m at j ^ (m & 7)).  Only
// rows < M are written: the MMA's column m reads x row m alone, so the
// stale rows behind them only feed accumulator columns nobody reads.
// Loads go out kXBatch at a time per thread before any is used.
template <int MPAD>
__device__ __noinline__ void w_load_x(const LayersParams& __restrict__ p, int s, int l, Range r) {
  LAYERS_WORKER_VIEW;

  constexpr int kXBatch = 2;
  const int C = stage_chunks(s);
  const __nv_bfloat16* src;
  const __nv_bfloat16* normw = nullptr;
  int ld = kHid;
  if (s == kSQkv) {
    src = l == 0 ? p.h0 : p.xs;
    if (l > 0) normw = p.in_w[l];
  } else if (s == kSO) {
    src = p.att_out;
  } else if (s == kSGu) {
    src = p.xs;
    normw = p.post_w[l];
  } else {
    src = p.act;
    ld = kInter;
  }
  if (normw) {
    if (wt < p.M) {
      float tot = 0.f;
      for (int t = 0; t < kHid / 128; ++t) tot += __ldcg(p.ss + t * 32 + wt);
      sh->rnorm[wt] = rsqrtf(__fadd_rn(tot * (1.0f / static_cast<float>(kHid)), p.eps));
    }
    workers_sync();
  }
  const int per_slot = p.M * 8;
  const int groups = (r.u1 - r.u0) * per_slot;
  for (int base = wt; base < groups; base += 128 * kXBatch) {
    uint4 v[kXBatch], wv[kXBatch];
#pragma unroll
    for (int k = 0; k < kXBatch; ++k) {
      const int i = base + 128 * k;
      if (i < groups) {
        const int slot = i / per_slot, rem = i - slot * per_slot;
        const int m = rem >> 3, col = ((r.u0 + slot) % C) * 64 + (rem & 7) * 8;
        v[k] = __ldcg(reinterpret_cast<const uint4*>(src + static_cast<int64_t>(m) * ld + col));
        if (normw) wv[k] = __ldg(reinterpret_cast<const uint4*>(normw + col));
      }
    }
#pragma unroll
    for (int k = 0; k < kXBatch; ++k) {
      const int i = base + 128 * k;
      if (i < groups) {
        const int slot = i / per_slot, rem = i - slot * per_slot;
        const int m = rem >> 3, g8 = rem & 7;
        uint4 o = v[k];
        if (normw) {
          const float rr = sh->rnorm[m];
          const __nv_bfloat16* hp = reinterpret_cast<const __nv_bfloat16*>(&v[k]);
          const __nv_bfloat16* wp = reinterpret_cast<const __nv_bfloat16*>(&wv[k]);
          __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            op[e] = rn(__fmul_rn(bf(wp[e]), bf(rn(__fmul_rn(bf(hp[e]), rr)))));
        }
        *reinterpret_cast<uint4*>(xbuf + slot * Gm::kXSlot + m * 128 + ((g8 ^ (m & 7)) << 4)) = o;
      }
    }
  }
  fence_async_smem();
  __syncwarp();
  if (lane == 0) mbar_arrive(sm.x_full);
}

// The last CTA of a split tile t: its partials summed in CTA order into
// `red` (rows < M).  Every load of a batch is issued before any is used;
// each tile entry is owned by one thread (or, below 4 rows, by a fixed
// group of threads combined in group order), so the sums are deterministic.
template <int MPAD>
__device__ __noinline__ void w_gather(const LayersParams& __restrict__ p, int s, int t) {
  LAYERS_WORKER_VIEW;

  constexpr int kGatherBatch = 8;
  const int C = stage_chunks(s);
  const int cf = stage_owner(s, t * C, G), cl = stage_owner(s, (t + 1) * C - 1, G);
  const int nseg = cl - cf + 1;
  const int items = p.M * 32;  // float4 entries of the tile's live rows
  float4* red4 = reinterpret_cast<float4*>(red);
  const float4* part4 = reinterpret_cast<const float4*>(p.part);
  if (wt < nseg) {  // this tile's segment of CTA cf + wt is that CTA's j-th
    const int cc = cf + wt;
    sh->seg_off[wt] = (cc * 2 + (t - stage_begin(s, cc, G) / C)) * 32 * 32;
  }
  workers_sync();
  auto src = [&](int sg, int item) { return __ldcg(part4 + sh->seg_off[sg] + item); };
  auto add4 = [](float4& a, const float4& b) {
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
  };
  if (items >= 128) {
    const int nit = (items - wt + 127) / 128;  // this thread's entries wt, wt + 128, ...
    const int n = nit * nseg;
    for (int base = 0; base < n; base += kGatherBatch) {
      float4 v[kGatherBatch];
#pragma unroll
      for (int k = 0; k < kGatherBatch; ++k) {
        const int idx = base + k;
        if (idx < n) {
          const int ii = idx / nseg;
          v[k] = src(idx - ii * nseg, wt + 128 * ii);
        }
      }
#pragma unroll
      for (int k = 0; k < kGatherBatch; ++k) {
        const int idx = base + k;
        if (idx < n) {
          const int ii = idx / nseg, sg = idx - ii * nseg;
          float4* d = red4 + wt + 128 * ii;
          if (sg == 0)
            *d = v[k];
          else
            add4(*d, v[k]);
        }
      }
    }
  } else {
    // 1 or 2 rows: `groups` threads per entry, thread (grp, item) adding
    // segments grp, grp + groups, ...; combined below in group order
    // through rows 8.. of `red` (unused with so few rows)
    const int groups = 128 / items >= 4 ? 4 : (128 / items >= 2 ? 2 : 1);
    float4* scr = red4 + 8 * 32;
    if (wt < groups * items) {
      const int grp = wt / items, item = wt - grp * items;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int base = grp; base < nseg; base += kGatherBatch * groups) {
        float4 v[kGatherBatch];
#pragma unroll
        for (int k = 0; k < kGatherBatch; ++k)
          if (base + k * groups < nseg) v[k] = src(base + k * groups, item);
#pragma unroll
        for (int k = 0; k < kGatherBatch; ++k)
          if (base + k * groups < nseg) add4(acc, v[k]);
      }
      scr[grp * items + item] = acc;
    }
    workers_sync();
    if (wt < items) {
      float4 acc = scr[wt];
      for (int g2 = 1; g2 < groups; ++g2) add4(acc, scr[g2 * items + wt]);
      red4[wt] = acc;
    }
  }
}

// Finish tile t of phase s from the fp32 sums in `red`.
template <int MPAD>
__device__ __noinline__ void w_finish(const LayersParams& __restrict__ p, int s, int l, int t) {
  LAYERS_WORKER_VIEW;

  const bool paired = s == kSQkv || s == kSGu;
  const int qn = paired ? 16 : 32;  // float4 groups per row handled
  auto sum4 = [&](int m, int n) { return *reinterpret_cast<const float4*>(red + m * 128 + n); };
  for (int m = ww; m < p.M; m += kAttWarps) {
    float sq = 0.f;
    if (lane < qn) {
      const int d = lane * 4;
      if (s == kSQkv) {
        const float4 lo4 = sum4(m, d), hi4 = sum4(m, 64 + d);
        const int start = p.starts[m];
        if (start >= 0) {
          float xl[4] = {lo4.x, lo4.y, lo4.z, lo4.w}, xh[4] = {hi4.x, hi4.y, hi4.z, hi4.w};
          const __nv_bfloat16* bias = p.qkv_b[l] + t * 128;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            xl[e] = bf(rn(xl[e] + bf(bias[d + e])));
            xh[e] = bf(rn(xh[e] + bf(bias[64 + d + e])));
          }
          const bool is_q = t < kHq, is_v = t >= kHq + kHkv;
          __nv_bfloat16* dst = nullptr;
          bool good = true;
          if (is_q) {
            dst = p.q_rot + (static_cast<int64_t>(m) * kHq + t) * kHeadDim;
          } else {
            const int h = is_v ? t - kHq - kHkv : t - kHq;
            const int row = p.rows ? p.rows[m] : m;
            const int64_t bi = start >> 4;
            if (bi >= p.pitch) {
              err.raise(PKV_DEVERR_POSITION);
              good = false;
            } else {
              const int blk = p.tables[static_cast<int64_t>(row) * p.pitch + bi];
              if (blk < 0 || blk >= p.num_blocks) {
                err.raise(PKV_DEVERR_BLOCK_ID);
                good = false;
              } else {
                const int64_t slot = static_cast<int64_t>(blk) * kBlockTokens + (start & 15);
                dst = p.pool + ((static_cast<int64_t>(2 * l + (is_v ? 1 : 0)) * p.num_slots + slot) *
                                    kHkv + h) * kHeadDim;
              }
            }
          }
          float ol[4], oh[4];
          if (good && !is_v) {
            if (start >= p.rope_rows) {
              err.raise(PKV_DEVERR_POSITION);
              good = false;
            } else {
              const __nv_bfloat16* cr = p.cos + static_cast<int64_t>(start) * kHeadDim;
              const __nv_bfloat16* sr = p.sin + static_cast<int64_t>(start) * kHeadDim;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                ol[e] = rope1(xl[e], bf(cr[d + e]), -xh[e], bf(sr[d + e]));
                oh[e] = rope1(xh[e], bf(cr[64 + d + e]), xl[e], bf(sr[64 + d + e]));
              }
            }
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) ol[e] = xl[e], oh[e] = xh[e];
          }
          if (good) {
            uint2 o;
            o.x = pack_bf16(ol[0], ol[1]);
            o.y = pack_bf16(ol[2], ol[3]);
            *reinterpret_cast<uint2*>(dst + d) = o;
            o.x = pack_bf16(oh[0], oh[1]);
            o.y = pack_bf16(oh[2], oh[3]);
            *reinterpret_cast<uint2*>(dst + 64 + d) = o;
          }
        }
      } else if (s == kSGu) {
        const float4 g = sum4(m, d), u = sum4(m, 64 + d);
        const float gv[4] = {g.x, g.y, g.z, g.w}, uv[4] = {u.x, u.y, u.z, u.w};
        float rr[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float gb = bf(rn(gv[e]));
          const float sb = bf(rn(gb / (1.0f + expf(-gb))));
          rr[e] = __fmul_rn(sb, bf(rn(uv[e])));
        }
        uint2 o;
        o.x = pack_bf16(rr[0], rr[1]);
        o.y = pack_bf16(rr[2], rr[3]);
        *reinterpret_cast<uint2*>(p.act + static_cast<int64_t>(m) * kInter + t * 64 + d) = o;
      } else {
        const float4 y4 = sum4(m, d);
        const float yv[4] = {y4.x, y4.y, y4.z, y4.w};
        const int n = t * 128 + d;
        if (s == kSDown && l == p.L - 1) {
          uint2 o;
          o.x = pack_bf16(yv[0], yv[1]);
          o.y = pack_bf16(yv[2], yv[3]);
          *reinterpret_cast<uint2*>(p.m_out + static_cast<int64_t>(m) * kHid + n) = o;
        } else {
          // residual add in bf16 (both operands bf16, one rounding), then
          // this tile's part of the row's sum of squares
          const uint2 xr = __ldcg(reinterpret_cast<const uint2*>(p.xs + static_cast<int64_t>(m) * kHid + n));
          const __nv_bfloat16* xp = reinterpret_cast<const __nv_bfloat16*>(&xr);
          float hv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            hv[e] = bf(rn(__fadd_rn(bf(xp[e]), bf(rn(yv[e])))));
            sq = __fadd_rn(sq, __fmul_rn(hv[e], hv[e]));
          }
          uint2 o;
          o.x = pack_bf16(hv[0], hv[1]);
          o.y = pack_bf16(hv[2], hv[3]);
          *reinterpret_cast<uint2*>(p.xs + static_cast<int64_t>(m) * kHid + n) = o;
        }
      }
    }
    if (!paired && !(s == kSDown && l == p.L - 1)) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
      if (lane == 0) p.ss[t * 32 + m] = sq;
    }
  }
}

// TMEM -> the tile's sums for segment number sc (tile t, this CTA's j-th
// segment of the phase).  A tile this CTA computes alone goes straight to
// `red`; a split tile's segment goes out as an fp32 partial, and the last
// CTA to finish the tile (completion counter) gathers them.
template <int MPAD>
__device__ __noinline__ void w_epilogue(const LayersParams& __restrict__ p, int s, int l, int t, int j, int sc) {
  LAYERS_WORKER_VIEW;
  const uint32_t tmem = sh->tmem;
  uint64_t* acc_full = sm.acc_full;
  uint64_t* acc_empty = sm.acc_empty;

  const int C = stage_chunks(s);
  const int nseg = stage_owner(s, (t + 1) * C - 1, G) - stage_owner(s, t * C, G) + 1;
  const int buf = sc & 1;
  const bool ok = __all_sync(0xffffffffu, wait_bar(&acc_full[buf], (sc >> 1) & 1, abort_word, err));
  float v[MPAD];
  if (ok) {
    tc_fence_after();
    const uint32_t ta = tmem + (static_cast<uint32_t>(q4 * 32) << 16) + static_cast<uint32_t>(buf * MPAD);
    if constexpr (MPAD == 32)
      tmem_ld16x2_sync(ta, *reinterpret_cast<float(*)[32]>(&v[0]));
    else
      tmem_ld16_sync(ta, *reinterpret_cast<float(*)[16]>(&v[0]));
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(&acc_empty[buf]);
  const int n = q4 * 32 + lane;
  if (nseg == 1) {
    if (ok) {
#pragma unroll
      for (int m = 0; m < MPAD; ++m)
        if (m < p.M) red[m * 128 + n] = v[m];
    }
    workers_sync();
    w_finish<MPAD>(p, s, l, t);
    workers_sync();  // `red` is rewritten by the next tile
    return;
  }
  if (ok) {
    float* dst = p.part + (static_cast<int64_t>(c) * 2 + j) * 32 * 128 + n;
#pragma unroll
    for (int m = 0; m < MPAD; ++m)
      if (m < p.M) dst[m * 128] = v[m];
  }
  __threadfence();
  workers_sync();
  if (wt == 0) {
    __threadfence();
    const int prev = atomicAdd(&p.tile_cnt[t], 1);
    const int last = prev == nseg - 1;
    if (last) p.tile_cnt[t] = 0;
    sh->flag = last;
  }
  workers_sync();
  const bool last = sh->flag != 0;
  if (last) {
    __threadfence();
    w_gather<MPAD>(p, s, t);
    workers_sync();
    w_finish<MPAD>(p, s, l, t);
  }
  workers_sync();  // sh->flag and `red` are rewritten by the next segment
}

// Paged decode attention of layer l over this CTA's (row, KV head,
// partition) units; att_it: this warp's attention-ring sequence, returned
// advanced.
template <int MPAD>
__device__ __noinline__ uint32_t w_attention(const LayersParams& __restrict__ p, const LayersMaps& __restrict__ maps, int l,
                                             uint32_t att_it) {
  LAYERS_WORKER_VIEW;
  uint64_t* att_bar = sm.att_bar;
  const int g = lane >> 2, tq = lane & 3;

  uint8_t* wstage = xbuf + ww * kAttStages * kAttStageBytes;
  uint64_t* wbar = att_bar + ww * kAttStages;
  if (lane == 0) fence_proxy_global();  // K/V rows appended by generic stores
  const uint64_t policy = policy_evict_first();
  const int units = p.M * kHkv * p.P;
  const int a_row = (lane & 7) + ((lane >> 3) & 1) * 8;
  const int a_chk = lane >> 4;
  const int v_tok = (lane & 7) + ((lane >> 4) & 1) * 8;
  const int v_chk = (lane >> 3) & 1;
  for (int u = c; u < units; u += G) {
    const int bk = u / p.P, part = u - bk * p.P;
    const int b = bk / kHkv, kvh = bk - b * kHkv;
    const int start = p.starts[b];
    int kv_len = start < 0 ? 0 : start + 1;
    int nblk = (kv_len + kBlockTokens - 1) / kBlockTokens;
    const int row = p.rows ? p.rows[b] : b;
    const int32_t* trow = p.tables + static_cast<int64_t>(row) * p.pitch;
    if (nblk > p.pitch) {
      if (part == 0 && wt == 0) err.raise(PKV_DEVERR_POSITION);
      nblk = static_cast<int>(p.pitch);
      kv_len = nblk * kBlockTokens;
    }
    __nv_bfloat16* outp = p.att_out + static_cast<int64_t>(b) * kHid + kvh * kGroup * kHeadDim;
    if (kv_len == 0) {  // no visible key: 0/0 as the reference (an inactive row)
      if (part == 0)
        for (int i = wt; i < kGroup * kHeadDim; i += 128) outp[i] = rn(__int_as_float(0x7fc00000));
      continue;
    }
    const int np = min(p.P, max(1, nblk / p.min_blocks));
    const int per = (nblk + np - 1) / np;
    const int bpp = max(kAttWarps, (per + kAttWarps - 1) / kAttWarps * kAttWarps);
    const int nparts = (nblk + bpp - 1) / bpp;
    if (part >= nparts) continue;
    const int blk_begin = part * bpp;
    const int span = min(nblk, blk_begin + bpp) - blk_begin;
    const int my_n = span > ww ? (span - ww + kAttWarps - 1) / kAttWarps : 0;

    auto load_ids = [&](int ch) -> int {
      const int itn = ch * 32 + lane;
      return itn < my_n ? __ldg(trow + blk_begin + ww + kAttWarps * itn) : 0;
    };
    int ids_cur = load_ids(0);
    int ids_next = my_n > 32 ? load_ids(1) : 0;
    auto issue = [&](int i, int blk) {
      const uint32_t gi = att_it + static_cast<uint32_t>(i);
      const int st = static_cast<int>(gi % kAttStages);
      uint8_t* kst = wstage + st * kAttStageBytes;
      uint8_t* vst = kst + kHeadBlockBytes;
      if (blk < 0 || blk >= p.num_blocks) {
        err.raise(PKV_DEVERR_BLOCK_ID);
        blk = 0;
      }
      const int slot = blk * kBlockTokens;
      mbar_arrive_expect_tx(&wbar[st], kAttStageBytes);
      tma_load_4d(kst, &maps.pool, &wbar[st], 0, kvh, slot, 2 * l, policy);
      tma_load_4d(kst + kBoxBytes, &maps.pool, &wbar[st], 64, kvh, slot, 2 * l, policy);
      tma_load_4d(vst, &maps.pool, &wbar[st], 0, kvh, slot, 2 * l + 1, policy);
      tma_load_4d(vst + kBoxBytes, &maps.pool, &wbar[st], 64, kvh, slot, 2 * l + 1, policy);
    };
    for (int i = 0; i < min(kAttStages, my_n); ++i) {
      const int blk = __shfl_sync(0xffffffffu, ids_cur, i);
      if (lane == 0) issue(i, blk);
    }
    uint32_t qb[8][2];
    {
      const bool live = g < kGroup;
      const __nv_bfloat16* qp =
          p.q_rot + (static_cast<int64_t>(b) * kHq + kvh * kGroup + (live ? g : 0)) * kHeadDim;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        qb[kk][0] = live ? __ldcg(reinterpret_cast<const unsigned int*>(qp + kk * 16 + 2 * tq)) : 0u;
        qb[kk][1] = live ? __ldcg(reinterpret_cast<const unsigned int*>(qp + kk * 16 + 8 + 2 * tq)) : 0u;
      }
    }
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[8][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    int i = 0;
    bool ok = true;
    for (; i < my_n; ++i) {
      const uint32_t gi = att_it + static_cast<uint32_t>(i);
      const int st = static_cast<int>(gi % kAttStages);
      ok = __all_sync(0xffffffffu, wait_bar(&wbar[st], (gi / kAttStages) & 1, abort_word, err));
      if (!ok) break;
      const uint32_t kst = smem_u32(wstage + st * kAttStageBytes);
      const uint32_t vst = kst + kHeadBlockBytes;
      const int j = blk_begin + ww + kAttWarps * i;
      float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kst + (kk >> 2) * kBoxBytes + swz128(a_row, (kk & 3) * 2 + a_chk), a0, a1, a2, a3);
        if (kk & 1)
          mma_bf16(sb, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
        else
          mma_bf16(sa, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
      }
      const int tok0 = j * kBlockTokens + g;
      float x0 = (sa[0] + sb[0]) * p.scale_log2, x1 = (sa[1] + sb[1]) * p.scale_log2;
      float x2 = (sa[2] + sb[2]) * p.scale_log2, x3 = (sa[3] + sb[3]) * p.scale_log2;
      if (tok0 >= kv_len) x0 = x1 = -INFINITY;
      if (tok0 + 8 >= kv_len) x2 = x3 = -INFINITY;
      float mb0 = fmaxf(x0, x2), mb1 = fmaxf(x1, x3);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mb0 = fmaxf(mb0, __shfl_xor_sync(0xffffffffu, mb0, off));
        mb1 = fmaxf(mb1, __shfl_xor_sync(0xffffffffu, mb1, off));
      }
      const float mn0 = fmaxf(m0, mb0), mn1 = fmaxf(m1, mb1);
      const float base0 = mn0 == -INFINITY ? 0.f : mn0;
      const float base1 = mn1 == -INFINITY ? 0.f : mn1;
      const float al0 = ex2(m0 - base0), al1 = ex2(m1 - base1);
      const float p0 = ex2(x0 - base0), p2 = ex2(x2 - base0);
      const float p1 = ex2(x1 - base1), p3 = ex2(x3 - base1);
      l0 = l0 * al0 + p0 + p2;
      l1 = l1 * al1 + p1 + p3;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= al0;
        o[mt][1] *= al1;
        o[mt][2] *= al0;
        o[mt][3] *= al1;
      }
      const uint32_t pb0 = movm_t(pack_bf16(p0, p1));
      const uint32_t pb1 = movm_t(pack_bf16(p2, p3));
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(vst + (mt >> 2) * kBoxBytes + swz128(v_tok, (mt & 3) * 2 + v_chk), a0, a1, a2, a3);
        mma_bf16(o[mt], a0, a1, a2, a3, pb0, pb1);
      }
      __syncwarp();
      const int nx = i + kAttStages;
      if (nx < my_n) {
        if ((nx & 31) == 0) {
          ids_cur = ids_next;
          ids_next = load_ids((nx >> 5) + 1);
        }
        const int blk = __shfl_sync(0xffffffffu, ids_cur, nx & 31);
        if (lane == 0) issue(nx, blk);
      }
    }
    if (!ok) {
      for (int k = i; k < min(my_n, i + kAttStages); ++k) {
        const uint32_t gk = att_it + static_cast<uint32_t>(k);
        mbar_wait(&wbar[gk % kAttStages], (gk / kAttStages) & 1, err);
      }
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    }
    att_it += static_cast<uint32_t>(my_n);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    // merge the four warps (over the attention ring)
    workers_sync();
    float* cm = reinterpret_cast<float*>(xbuf);
    float* cl = cm + kAttWarps * 8;
    float* co = reinterpret_cast<float*>(xbuf + 1024);
    if (g == 0) {
      cm[ww * 8 + 2 * tq] = m0;
      cm[ww * 8 + 2 * tq + 1] = m1;
      cl[ww * 8 + 2 * tq] = l0;
      cl[ww * 8 + 2 * tq + 1] = l1;
    }
    {
      float* cw = co + ww * 8 * kHeadDim;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int dd = mt * 16 + g;
        cw[(2 * tq) * kHeadDim + dd] = o[mt][0];
        cw[(2 * tq + 1) * kHeadDim + dd] = o[mt][1];
        cw[(2 * tq) * kHeadDim + dd + 8] = o[mt][2];
        cw[(2 * tq + 1) * kHeadDim + dd + 8] = o[mt][3];
      }
    }
    workers_sync();
    const int h = wt >> 4;
    const int d0 = (wt & 15) * 8;
    float acc[8];
    float Ls = 0.f, Ms = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttWarps; ++w) Ms = fmaxf(Ms, cm[w * 8 + h]);
    const float mbase = Ms == -INFINITY ? 0.f : Ms;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
    for (int w = 0; w < kAttWarps; ++w) {
      const float f = ex2(cm[w * 8 + h] - mbase);
      Ls += f * cl[w * 8 + h];
      const float* src = co + (w * 8 + h) * kHeadDim + d0;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += f * src[e];
    }
    workers_sync();  // the ring is refilled by the next unit
    if (nparts == 1) {
      if (h < kGroup) {
        const float inv = 1.f / Ls;
        uint4 pk;
        pk.x = pack_bf16(acc[0] * inv, acc[1] * inv);
        pk.y = pack_bf16(acc[2] * inv, acc[3] * inv);
        pk.z = pack_bf16(acc[4] * inv, acc[5] * inv);
        pk.w = pack_bf16(acc[6] * inv, acc[7] * inv);
        *reinterpret_cast<uint4*>(outp + h * kHeadDim + d0) = pk;
      }
      continue;
    }
    {
      const int64_t slot = static_cast<int64_t>(u);
      const float inv = 1.f / Ls;
      float4* dst = reinterpret_cast<float4*>(p.att_o + (slot * 8 + h) * kHeadDim + d0);
      dst[0] = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
      dst[1] = make_float4(acc[4] * inv, acc[5] * inv, acc[6] * inv, acc[7] * inv);
      if ((wt & 15) == 0) p.att_lse[slot * 8 + h] = mbase + log2f(Ls);
    }
    __threadfence();
    workers_sync();
    if (wt == 0) {
      __threadfence();
      const int prev = atomicAdd(&p.att_cnt[bk], 1);
      const int last = prev == nparts - 1;
      if (last) p.att_cnt[bk] = 0;
      sh->flag = last;
    }
    workers_sync();
    const bool last = sh->flag != 0;
    workers_sync();
    if (!last || h >= kGroup) continue;
    __threadfence();
    const int64_t base = static_cast<int64_t>(bk) * p.P;
    float LM = -INFINITY;
    for (int q = 0; q < nparts; ++q) LM = fmaxf(LM, __ldcg(p.att_lse + (base + q) * 8 + h));
    float W = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    for (int q = 0; q < nparts; ++q) {
      const float w = ex2(__ldcg(p.att_lse + (base + q) * 8 + h) - LM);
      W += w;
      const float4* src = reinterpret_cast<const float4*>(p.att_o + ((base + q) * 8 + h) * kHeadDim + d0);
      const float4 a = __ldcg(src), bq = __ldcg(src + 1);
      acc[0] += w * a.x;
      acc[1] += w * a.y;
      acc[2] += w * a.z;
      acc[3] += w * a.w;
      acc[4] += w * bq.x;
      acc[5] += w * bq.y;
      acc[6] += w * bq.z;
      acc[7] += w * bq.w;
    }
    const float inv = 1.f / W;
    uint4 pk;
    pk.x = pack_bf16(acc[0] * inv, acc[1] * inv);
    pk.y = pack_bf16(acc[2] * inv, acc[3] * inv);
    pk.z = pack_bf16(acc[4] * inv, acc[5] * inv);
    pk.w = pack_bf16(acc[6] * inv, acc[7] * inv);
    *reinterpret_cast<uint4*>(outp + h * kHeadDim + d0) = pk;
  }
  return att_it;
}

template <int MPAD>
__global__ void __launch_bounds__(kLThreads, 1)
    decode_layers_kernel(const __grid_constant__ LayersParams p,
                         const __grid_constant__ LayersMaps maps) {
  using Gm = Geo<MPAD>;
  const SmemMap sm = smem_map<MPAD>(p);
  uint8_t* wring = sm.wring;
  uint8_t* xbuf = sm.xbuf;
  uint64_t* full = sm.full;
  uint64_t* empty = sm.empty;
  uint64_t* acc_full = sm.acc_full;
  uint64_t* acc_empty = sm.acc_empty;
  uint64_t* x_full = sm.x_full;
  uint64_t* mma_done = sm.mma_done;
  uint64_t* att_bar = sm.att_bar;
  LayersShared* sh = sm.sh;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, G = p.G;
  const DevErr err{p.err};
  const uint32_t* abort_word = p.sync + 2;
  if (tid == 0) {
    for (int s = 0; s < p.nw; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kAttWarps);
    }
    mbar_init(x_full, kAttWarps);
    mbar_init(mma_done, 1);
    for (int s = 0; s < kAttWarps * kAttStages; ++s) mbar_init(&att_bar[s], 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&sh->tmem, MPAD <= 16 ? 32u : 64u);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int l = 0; l < p.L; ++l)
        for (int s = 0; s < 4; ++s) prefetch_tmap(&maps.w[l][s]);
      const uint64_t once = policy_evict_first();
      int it = 0;
      bool ok = true;
      for (int l = 0; l < p.L && ok; ++l) {
        for (int s = 0; s < 4 && ok; ++s) {
          const Range r = range_of(s, c, G);
          const int C = stage_chunks(s);
          for (int u = r.u0; u < r.u1; ++u, ++it) {
            const int st = it % p.nw;
            if (it >= p.nw && !wait_bar(&empty[st], ((it / p.nw) - 1) & 1, abort_word, err)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[st], kWBox);
            tma_load_2d(wring + st * kWBox, &maps.w[l][s], &full[st], (u % C) * 64, (u / C) * 128,
                        once);
          }
        }
      }
      // the ring's last loads must land before the CTA can exit
      for (int i = max(0, it - p.nw); i < it; ++i) mbar_wait(&full[i % p.nw], (i / p.nw) & 1, err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, sc = 0, gs = 0;
      bool ok = true;
      for (int l = 0; l < p.L && ok; ++l) {
        for (int s = 0; s < 4 && ok; ++s, ++gs) {
          if (!wait_bar(x_full, gs & 1, abort_word, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const Range r = range_of(s, c, G);
          const int C = stage_chunks(s);
          for (int t = r.t0; t <= r.t1 && ok; ++t, ++sc) {
            const int buf = sc & 1;
            if (sc >= 2 && !wait_bar(&acc_empty[buf], ((sc >> 1) - 1) & 1, abort_word, err)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const int ua = max(r.u0, t * C), ub = min(r.u1, (t + 1) * C);
            const uint32_t d = tmem + static_cast<uint32_t>(buf * MPAD);
            for (int u = ua; u < ub; ++u, ++it) {
              const int st = it % p.nw;
              if (!wait_bar(&full[st], (it / p.nw) & 1, abort_word, err)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t sw = smem_u32(wring + st * kWBox);
              const uint32_t sx = smem_u32(xbuf + (u - r.u0) * Gm::kXSlot);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                umma(d, sdesc(sw + kk * 32, 16, 1024), sdesc(sx + kk * 32, 16, 1024), Gm::kIdesc,
                     (u > ua || kk > 0) ? 1u : 0u);
              umma_commit(&empty[st]);
            }
            if (ok) umma_commit(&acc_full[buf]);
          }
        }
      }
      // every MMA issued has retired before TMEM is freed
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, err);
    }
  } else {
    // ------------------------------------------------------------ workers
    int sc = 0;               // segment sequence (matches the MMA issuer)
    uint32_t target = 0;      // grid barrier arrivals expected so far
    uint32_t att_it = 0;      // this warp's attention ring sequence
    auto gemm_phase = [&](int s, int l) {
      const Range r = range_of(s, c, G);
      w_load_x<MPAD>(p, s, l, r);
      for (int t = r.t0; t <= r.t1; ++t, ++sc) w_epilogue<MPAD>(p, s, l, t, t - r.t0, sc);
    };
    auto barrier = [&]() {
      target += static_cast<uint32_t>(G);
      return w_grid_barrier<MPAD>(p, target);
    };
    for (int l = 0; l < p.L; ++l) {
      gemm_phase(kSQkv, l);
      fence_proxy_global();  // this CTA's K/V stores before the TMA reads of other CTAs
      if (!barrier()) break;
      att_it = w_attention<MPAD>(p, maps, l, att_it);
      if (!barrier()) break;
      gemm_phase(kSO, l);
      if (!barrier()) break;
      gemm_phase(kSGu, l);
      if (!barrier()) break;
      gemm_phase(kSDown, l);
      if (l + 1 < p.L && !barrier()) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, MPAD <= 16 ? 32u : 64u);
  }
}

}  // namespace

LayersPlan plan_decode_layers(int32_t rows, int32_t sms) {
  LayersPlan pl{};
  pl.mpad = rows <= 16 ? 16 : 32;
  pl.grid = sms;
  pl.partitions = max(1, sms / max(1, rows * kHkv));
  pl.min_blocks = 4;
  int xs = 0;
  bool two = true;
  for (int s = 0; s < 4; ++s) {
    const int C = stage_chunks(s);
    for (int c = 0; c < sms; ++c) {
      const int u0 = stage_begin(s, c, sms), u1 = stage_begin(s, c + 1, sms);
      xs = max(xs, u1 - u0);
      if (u1 > u0 && (u1 - 1) / C - u0 / C > 1) two = false;
    }
    for (int t = 0; t < stage_tiles(s); ++t)  // a tile's gather reads at most 64 partials
      if (stage_owner(s, (t + 1) * C - 1, sms) - stage_owner(s, t * C, sms) + 1 > 64) two = false;
  }
  pl.xslots = xs;
  pl.valid = two && sms > 0;
  const int xbytes = max(xs * pl.mpad * 128, kAttRingBytes);
  const int bars = 8 * (2 * 16 + 2 + 2 + 1 + 1 + kAttWarps * kAttStages) + static_cast<int>(sizeof(LayersShared));
  // deepest W ring that fits next to the x slots
  int nw = (227 * 1024 - 1024 - xbytes - kRedBytes - bars) / kWBox;
  if (nw > 16) nw = 16;
  pl.nw = nw;
  pl.smem_bytes = 1024 + nw * kWBox + xbytes + kRedBytes +
                  8 * (2 * nw + 2 + 2 + 1 + 1 + kAttWarps * kAttStages) +
                  static_cast<int>(sizeof(LayersShared));
  if (nw < 4) pl.valid = false;
  return pl;
}

size_t decode_layers_workspace_bytes(int32_t rows, int32_t sms) {
  const LayersPlan pl = plan_decode_layers(rows, sms);
  size_t b = 0;
  b += 4096;                                                     // sync words + counters
  b += static_cast<size_t>(sms) * 2 * 32 * 128 * 4;               // GEMM partials
  b += static_cast<size_t>(rows) * kHkv * pl.partitions * 8 * 128 * 4;  // attention partials
  b += static_cast<size_t>(rows) * kHkv * pl.partitions * 8 * 4 + 256;
  b += 12 * 32 * 4;                                               // sums of squares
  b += static_cast<size_t>(rows) * kHq * kHeadDim * 2 + 256;      // q_rot
  b += static_cast<size_t>(rows) * kHid * 2 + 256;                // attention output
  b += static_cast<size_t>(rows) * kInter * 2 + 256;              // SwiGLU output
  return b + 4096;
}

size_t decode_layers_sync_bytes() { return 4096; }

// Carve the workspace (16-byte aligned pieces) into the kernel's buffers.
void carve_decode_layers(LayersParams& p, void* ws, int32_t rows, int32_t sms, int32_t partitions) {
  uint8_t* b = static_cast<uint8_t*>(ws);
  auto take = [&](size_t n) {
    uint8_t* r = b;
    b += (n + 255) / 256 * 256;
    return r;
  };
  uint8_t* sync = take(4096);
  p.sync = reinterpret_cast<uint32_t*>(sync);
  p.tile_cnt = reinterpret_cast<int32_t*>(sync + 64);
  p.att_cnt = reinterpret_cast<int32_t*>(sync + 64 + kMaxTiles * 4);
  p.part = reinterpret_cast<float*>(take(static_cast<size_t>(sms) * 2 * 32 * 128 * 4));
  p.att_o = reinterpret_cast<float*>(take(static_cast<size_t>(rows) * kHkv * partitions * 8 * 128 * 4));
  p.att_lse = reinterpret_cast<float*>(take(static_cast<size_t>(rows) * kHkv * partitions * 8 * 4));
  p.ss = reinterpret_cast<float*>(take(12 * 32 * 4));
  p.q_rot = reinterpret_cast<__nv_bfloat16*>(take(static_cast<size_t>(rows) * kHq * kHeadDim * 2));
  p.att_out = reinterpret_cast<__nv_bfloat16*>(take(static_cast<size_t>(rows) * kHid * 2));
  p.act = reinterpret_cast<__nv_bfloat16*>(take(static_cast<size_t>(rows) * kInter * 2));
}

cudaError_t launch_decode_layers(const LayersParams& p, const LayersMaps& maps, const LayersPlan& pl,
                                 cudaStream_t stream) {
  static std::mutex mu;
  static int configured[2] = {-1, -1};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const int which = pl.mpad == 16 ? 0 : 1;
  void (*kern)(LayersParams, LayersMaps) =
      which == 0 ? decode_layers_kernel<16> : decode_layers_kernel<32>;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (configured[which] != dev) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      if (e != cudaSuccess) return e;
      configured[which] = dev;
    }
  }
  // the barrier words and completion counters start at zero every launch
  e = cudaMemsetAsync(p.sync, 0, decode_layers_sync_bytes(), stream);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kLThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(pl.smem_bytes);
  cfg.stream = stream;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeCooperative;  // every CTA resident at once (grid barriers)
  attr.val.cooperative = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p, maps);
}

}  // namespace pkv
