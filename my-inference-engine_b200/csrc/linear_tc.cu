// Skinny linear layers on the 5th-generation tensor cores (tcgen05 + TMEM,
// sm_100a): y[M, N] = x[M, K] . W[N, K]^T for the row counts of a decode
// step (M <= 256), where reading W once from HBM is the whole cost.
//
// The Qwen2 block's projections (model.py:83-86 q/k/v/o, :114-116 gate/up/down)
// are nn.Linear layers; torch runs them as cuBLAS GEMMs whose tiles are shaped
// for large M.  Here the roles are swapped: the weight tile is the MMA's
// M side (128 rows of W) and the batch rows are its N side (M padded to a
// multiple of 16 by TMA zero fill), so one tcgen05.mma per 16-wide K step
// covers the whole batch and every CTA streams its own slice of W exactly once.
//
//   grid  = (N / 128, splits): CTA (t, s) owns W rows [128t, 128t+128) and an
//           equal share of the K/64 chunks; splits is chosen so that the grid
//           fills the SMs once
//   block = 6 warps
//     warp 0    TMA producer (one thread): per chunk one 128x64 W box
//               (evict-first: streamed once) and one Mpad x 64 x box
//               (evict-last: every CTA reads it) into a stages-deep ring.
//               W is row-major [N][K] (a box = 128 pieces of 128 B, one per
//               row) or packed as [N/128][K/64][128][64] (PKV_W_TILED), where
//               a box is one contiguous 16 KiB run and a CTA's chunks are
//               adjacent: each CTA then streams one contiguous range of HBM
//     warp 1    owns TMEM (Mpad columns, fp32) and issues the MMAs:
//               D[128, Mpad] += W[128, 16] . x[Mpad, 16]^T, 4 per chunk
//     warps 2-5 epilogue: warp w reads TMEM lanes 32*(w%4).., i.e. one W row
//               (one output feature n) per thread, all batch rows as columns
// RoPE + append mode (pkv_linear_rope_append): each 128-row W tile is one
// head of the merged q/k/v projection, so the epilogue adds the bias, rounds
// to bf16, rotates q and k (partner dims d and d+64 are both in the tile) and
// stores q_rot and the new K/V rows into their pool slots: no intermediate,
// no second kernel.
// SwiGLU mode (pkv_linear_silu_mul with PKV_W_GATE_UP_PAIRED): every W tile
// pairs 64 gate rows with the matching 64 up rows, so the epilogue finishes
// the activation and y is the [M][N/2] SwiGLU output.
// Epilogue: each CTA moves its fp32 accumulators from TMEM to its own shared
// memory (over the drained ring).  Split-k: the `splits` CTAs of one W tile
// form a thread-block cluster (1 x splits); each pushes its partial rows into
// the receive buffer of the CTA that owns them (distributed shared memory
// stores + a remote mbarrier arrive), and owner r adds batch rows
// [r*M/splits, ...) in split order (deterministic).  Bias, one bf16 rounding
// and 8-byte row-contiguous stores of y; nothing else goes to global memory.
// Every wait is bounded.
#include <map>
#include <mutex>
#include <tuple>

#include "pkv_device.cuh"
#include "pkv_kernels.h"
#include "tc_device.cuh"

namespace pkv {
namespace {

constexpr int kTileN = 128;            // W rows per CTA (MMA M)
constexpr int kChunkK = 64;            // K elements per stage: one 128 B swizzle row
constexpr int kWBytes = kTileN * 128;  // 16 KiB W box per stage
constexpr int kLinThreads = 192;
constexpr int kMaxStages = 8;
constexpr int kSmemCap = 227 * 1024;
constexpr int kMaxSplits = 16;  // non-portable cluster size limit

__device__ __forceinline__ float bf(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 rn(float x) { return __float2bfloat16_rn(x); }

// bf16(bf16(x*c) + bf16(r*s)), each op rounded separately as the reference's
// three torch ops (model.py:58-65) compute it
__device__ __forceinline__ float rope1(float x, float c, float r, float sn) {
  return bf(rn(__fadd_rn(bf(rn(__fmul_rn(x, c))), bf(rn(__fmul_rn(r, sn))))));
}

struct LinParams {
  __nv_bfloat16* y;  // [M][ldy]
  int64_t ldy;
  const __nv_bfloat16* bias;  // nullable
  int32_t M, N, chunks, splits, stages, mpad;
  uint32_t tmem_cols, idesc;
  int32_t recv_off;  // split-k receive buffer: [splits][rows per owner][128] fp32
  int32_t w_tiled;   // W packed as [N/128][K/64][128][64]: one contiguous 16 KiB box per chunk
  int32_t swiglu;    // W tiles pair 64 gate rows with their 64 up rows: y = SwiGLU, N/2 wide
  int32_t* err;
  // RoPE + K/V append epilogue (rope.q_out != nullptr): tile = one head of
  // the merged q/k/v output, row m = batch row m / T, step token m % T
  RopeAppend rope;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cta address -> the same offset in cluster CTA `rank`
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_cluster4(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
// arrive on an mbarrier of another CTA of the cluster, releasing this
// thread's earlier (and, through a preceding bar.sync, the CTA's) writes
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile(
      "fence.acq_rel.cluster;\n\t"
      "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
      : "memory");
}
__device__ __forceinline__ bool mbar_wait_acq_cluster(uint64_t* bar, uint32_t parity,
                                                      const DevErr& err) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  err.raise(PKV_DEVERR_TIMEOUT);
  return false;
}

__global__ void __launch_bounds__(kLinThreads, 1)
    linear_tc_kernel(const LinParams p, const __grid_constant__ CUtensorMap wmap,
                     const __grid_constant__ CUtensorMap xmap) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int stage_bytes = kWBytes + p.mpad * 128;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.stages * stage_bytes);
  uint64_t* empty = full + p.stages;
  uint64_t* done = empty + p.stages;
  uint64_t* recv_bar = done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  float* recv = reinterpret_cast<float*>(smem + p.recv_off);
  const bool clustered = p.splits > 1;
  const int per = (p.M + p.splits - 1) / p.splits;  // batch rows each cluster CTA owns

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int c0 = static_cast<int>(static_cast<int64_t>(split) * p.chunks / p.splits);
  const int nc = static_cast<int>(static_cast<int64_t>(split + 1) * p.chunks / p.splits) - c0;
  const DevErr err{p.err};

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);   // producer's arrive.expect_tx
      mbar_init(&empty[s], 1);  // tcgen05.commit after the chunk's MMAs
    }
    mbar_init(done, 1);
    if (clustered) mbar_init(recv_bar, p.splits);  // one arrival per cluster CTA
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Dependents launch only once every CTA of this grid holds its TMEM, so a
  // dependent that allocates before its griddepcontrol.wait cannot take
  // columns this grid still needs.
  pdl_trigger();
  const uint32_t tmem = *tmem_slot;
  // every CTA's recv_bar is initialised before any CTA arrives on it: the
  // matching wait sits before the epilogue's remote stores
  if (clustered) cluster_arrive();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&wmap);
      prefetch_tmap(&xmap);
      const uint64_t once = policy_evict_first();
      const uint64_t keep = policy_evict_last();
      const uint32_t bytes = static_cast<uint32_t>(stage_bytes);
      auto load_w = [&](int i, int st) {
        uint8_t* sw = smem + st * stage_bytes;
        mbar_arrive_expect_tx(&full[st], bytes);  // W + x land on the same barrier
        if (p.w_tiled)
          tma_load_3d(sw, &wmap, &full[st], 0, 0, tile * p.chunks + c0 + i, once);
        else
          tma_load_2d(sw, &wmap, &full[st], (c0 + i) * kChunkK, tile * kTileN, once);
      };
      auto load_x = [&](int i, int st) {
        tma_load_2d(smem + st * stage_bytes + kWBytes, &xmap, &full[st], (c0 + i) * kChunkK, 0, keep);
      };
      // The weights do not depend on earlier kernels: fill the ring with W
      // before waiting for the predecessor grid, then load x.
      const int pre = nc < p.stages ? nc : p.stages;
      for (int i = 0; i < pre; ++i) load_w(i, i);
      pdl_wait();
      for (int i = 0; i < pre; ++i) load_x(i, i);
      for (int i = pre; i < nc; ++i) {
        const int st = i % p.stages;
        if (!mbar_wait(&empty[st], ((i / p.stages) - 1) & 1, err)) break;
        load_w(i, st);
        load_x(i, st);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      for (int i = 0; i < nc; ++i) {
        const int st = i % p.stages;
        if (!mbar_wait(&full[st], (i / p.stages) & 1, err)) break;
        tc_fence_after();
        const uint32_t sw = smem_u32(smem + st * stage_bytes);
        const uint32_t sx = sw + kWBytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma(tmem, sdesc(sw + kk * 32, 16, 1024), sdesc(sx + kk * 32, 16, 1024), p.idesc,
               (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[st]);
      }
      umma_commit(done);
      mbar_wait(done, 0, err);  // every MMA retired before TMEM is freed
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int nl = quarter * 32 + lane;  // W row within the tile == TMEM lane
    const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    if (__all_sync(0xffffffffu, mbar_wait(done, 0, err))) {
      tc_fence_after();
      // this CTA's accumulators as [mpad][128] fp32 over the drained ring
      float* red = reinterpret_cast<float*>(smem);
      for (int c = 0; c < p.mpad; c += 16) {
        float v[16];
        tmem_ld16_sync(taddr + c, v);
#pragma unroll
        for (int e = 0; e < 16; ++e) red[(c + e) * kTileN + nl] = v[e];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
  // Store: bias, one bf16 rounding (the value F.linear stores), 8-byte
  // row-contiguous stores of y.  SwiGLU tiles: features i and 64 + i of a
  // tile are gate and up of output 64*tile + i, combined exactly as
  // pkv_silu_mul does: bf16(bf16(silu(bf16 g)) * bf16 u).
  const float* red = reinterpret_cast<const float*>(smem);
  auto store4 = [&](int m, int nl, float4 acc) {
    const int n = tile * kTileN + nl;
    if (p.bias) {
      acc.x += bf(p.bias[n + 0]);
      acc.y += bf(p.bias[n + 1]);
      acc.z += bf(p.bias[n + 2]);
      acc.w += bf(p.bias[n + 3]);
    }
    uint2 o;
    o.x = pack_bf16(acc.x, acc.y);
    o.y = pack_bf16(acc.z, acc.w);
    *reinterpret_cast<uint2*>(p.y + m * p.ldy + n) = o;
  };
  auto store_swiglu4 = [&](int m, int i, float4 g, float4 u) {
    const float gv[4] = {g.x, g.y, g.z, g.w}, uv[4] = {u.x, u.y, u.z, u.w};
    float r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float gb = bf(__float2bfloat16_rn(gv[e]));
      const float sb = bf(__float2bfloat16_rn(gb / (1.0f + expf(-gb))));
      r[e] = __fmul_rn(sb, bf(__float2bfloat16_rn(uv[e])));
    }
    uint2 o;
    o.x = pack_bf16(r[0], r[1]);
    o.y = pack_bf16(r[2], r[3]);
    *reinterpret_cast<uint2*>(p.y + m * p.ldy + tile * (kTileN / 2) + i) = o;
  };
  // RoPE + append (pkv_linear_rope_append): this tile is head `tile` of
  // [q heads | k heads | v heads]; the thread owns dims d..d+3 and their
  // rotation partners 64+d..64+d+3 of one token, exactly as append_rope_kernel
  // treats the bf16 output of the q/k/v GEMM (bias added, one rounding)
  const RopeAppend& ra = p.rope;
  auto store_rope8 = [&](int m, int d, float4 lo, float4 hi) {
    const int b = m / ra.T, tt = m - b * ra.T;
    const int start = ra.starts[b];
    if (start < 0) return;                        // inactive (padding) row
    if (ra.q_lens && tt >= ra.q_lens[b]) return;  // right padding of a shorter row
    const int pos = start + tt;
    float xl[4] = {lo.x, lo.y, lo.z, lo.w}, xh[4] = {hi.x, hi.y, hi.z, hi.w};
    const int n0 = tile * kTileN;
#pragma unroll
    for (int e = 0; e < 4; ++e) {  // the GEMM output in bf16, as F.linear stores it
      const float bl = p.bias ? bf(p.bias[n0 + d + e]) : 0.f;
      const float bh = p.bias ? bf(p.bias[n0 + 64 + d + e]) : 0.f;
      xl[e] = bf(rn(xl[e] + bl));
      xh[e] = bf(rn(xh[e] + bh));
    }
    const bool is_q = tile < ra.hq;
    const bool is_v = tile >= ra.hq + ra.hkv;
    __nv_bfloat16* dst;
    if (is_q) {
      dst = ra.q_out + b * ra.qo_sb + tile * ra.qo_sh + tt * ra.qo_st;
    } else {
      const int h = is_v ? tile - ra.hq - ra.hkv : tile - ra.hq;
      const int row = ra.rows ? ra.rows[b] : b;
      const int64_t bi = pos >> 4;
      if (pos < 0 || bi >= ra.pitch) {
        err.raise(PKV_DEVERR_POSITION);
        return;
      }
      const int blk = ra.tables[static_cast<int64_t>(row) * ra.pitch + bi];
      if (blk < 0 || blk >= ra.num_blocks) {
        err.raise(PKV_DEVERR_BLOCK_ID);
        return;
      }
      const int64_t slot = static_cast<int64_t>(blk) * kBlockTokens + (pos & 15);
      dst = (is_v ? ra.v_pool : ra.k_pool) + (slot * ra.hkv + h) * kHeadDim;
    }
    float ol[4], oh[4];
    if (is_v) {
#pragma unroll
      for (int e = 0; e < 4; ++e) ol[e] = xl[e], oh[e] = xh[e];
    } else {
      if (pos < 0 || pos >= ra.rope_rows) {
        err.raise(PKV_DEVERR_POSITION);
        return;
      }
      const __nv_bfloat16* cr = ra.cos + static_cast<int64_t>(pos) * kHeadDim;
      const __nv_bfloat16* sr = ra.sin + static_cast<int64_t>(pos) * kHeadDim;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        // first half: x*cos + (-x2)*sin ; second half: x*cos + x1*sin
        ol[e] = rope1(xl[e], bf(cr[d + e]), -xh[e], bf(sr[d + e]));
        oh[e] = rope1(xh[e], bf(cr[64 + d + e]), xl[e], bf(sr[64 + d + e]));
      }
    }
    uint2 o;
    o.x = pack_bf16(ol[0], ol[1]);
    o.y = pack_bf16(ol[2], ol[3]);
    *reinterpret_cast<uint2*>(dst + d) = o;
    o.x = pack_bf16(oh[0], oh[1]);
    o.y = pack_bf16(oh[2], oh[3]);
    *reinterpret_cast<uint2*>(dst + 64 + d) = o;
  };
  // quads per row: 32 features x 4, or 16 gate/up (or rotation) pairs x 4
  const bool paired = p.swiglu || ra.q_out;
  const int quads = paired ? kTileN / 8 : kTileN / 4;
  if (!clustered) {
    for (int idx = tid; idx < p.M * quads; idx += kLinThreads) {
      const int m = idx / quads, nl = (idx % quads) * 4;
      const float4 a = *reinterpret_cast<const float4*>(red + m * kTileN + nl);
      if (!paired)
        store4(m, nl, a);
      else if (p.swiglu)
        store_swiglu4(m, nl, a, *reinterpret_cast<const float4*>(red + m * kTileN + 64 + nl));
      else
        store_rope8(m, nl, a, *reinterpret_cast<const float4*>(red + m * kTileN + 64 + nl));
    }
    return;
  }
  // Split-k over the cluster: CTA r owns batch rows [r*per, r*per + per).
  // Push this split's partial rows into their owners' receive buffers (slot
  // = this CTA's rank), then arrive on each owner's recv_bar; an owner waits
  // for all `splits` arrivals and adds the slots in split order.  Nothing is
  // read from another CTA, so no CTA has to wait for the others to exit.
  cluster_wait();
  const uint32_t rank = cluster_rank();
  const uint32_t recv_base = smem_u32(recv);
  for (int idx = tid; idx < p.M * (kTileN / 4); idx += kLinThreads) {
    const int m = idx / (kTileN / 4), nl = (idx % (kTileN / 4)) * 4;
    const int owner = m / per;
    const uint32_t dst = recv_base + static_cast<uint32_t>(((rank * per + (m - owner * per)) * kTileN + nl) * 4);
    st_cluster4(map_rank(dst, static_cast<uint32_t>(owner)),
                *reinterpret_cast<const float4*>(red + m * kTileN + nl));
  }
  __syncthreads();
  if (tid < p.splits && tid * per < p.M)
    mbar_arrive_remote(map_rank(smem_u32(recv_bar), static_cast<uint32_t>(tid)));
  const int m0 = static_cast<int>(rank) * per;
  const int m1 = min(p.M, m0 + per);
  auto sum4 = [&](int j, int nl) {
    float4 acc = *reinterpret_cast<const float4*>(recv + j * kTileN + nl);
    for (int sp = 1; sp < p.splits; ++sp) {
      const float4 v = *reinterpret_cast<const float4*>(recv + (sp * per + j) * kTileN + nl);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    return acc;
  };
  if (m0 < m1 && mbar_wait_acq_cluster(recv_bar, 0, err)) {
    for (int idx = tid; idx < (m1 - m0) * quads; idx += kLinThreads) {
      const int j = idx / quads, nl = (idx % quads) * 4;
      if (!paired)
        store4(m0 + j, nl, sum4(j, nl));
      else if (p.swiglu)
        store_swiglu4(m0 + j, nl, sum4(j, nl), sum4(j, 64 + nl));
      else
        store_rope8(m0 + j, nl, sum4(j, nl), sum4(j, 64 + nl));
    }
  }
}

// w[n][k] (row stride ldw) -> [n/128][k/64][128][64]; one thread per 16 bytes
__global__ void __launch_bounds__(256)
    pack_weight_kernel(const __nv_bfloat16* __restrict__ w, int64_t ldw, int chunks,
                       int64_t total16, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total16) return;
  const int j8 = static_cast<int>(i & 7);
  const int r = static_cast<int>((i >> 3) & 127);
  const int64_t tc = i >> 10;  // tile * chunks + chunk
  const int c = static_cast<int>(tc % chunks);
  const int64_t t = tc / chunks;
  const uint4 v = *reinterpret_cast<const uint4*>(w + (t * kTileN + r) * ldw + c * kChunkK + j8 * 8);
  *reinterpret_cast<uint4*>(out + i * 8) = v;
}

// w_gate_up [2*inter][k] (gate rows, then up rows; row stride ldw) ->
// [2*inter][k] with tile t = rows [128t, 128t+128) holding gate rows
// [64t, 64t+64) then up rows [64t, 64t+64); one thread per 16 bytes
__global__ void __launch_bounds__(256)
    pair_gate_up_kernel(const __nv_bfloat16* __restrict__ w, int64_t ldw, int inter, int k,
                        int64_t total16, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total16) return;
  const int per_row = k / 8;
  const int64_t r = i / per_row;
  const int c = static_cast<int>(i % per_row) * 8;
  const int64_t t = r / kTileN;
  const int within = static_cast<int>(r % kTileN);
  const int64_t src = within < 64 ? t * 64 + within : inter + t * 64 + (within - 64);
  *reinterpret_cast<uint4*>(out + r * k + c) = *reinterpret_cast<const uint4*>(w + src * ldw + c);
}

int sm_count() {
  static int count = 0;
  if (count == 0) {
    int dev = 0, c = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && c > 0)
      count = c;
    else
      return 148;
  }
  return count;
}

// Per-device one-time function attributes: the full shared-memory opt-in and
// clusters of up to 16 CTAs.
cudaError_t configure_kernel() {
  static int configured_device = -1;
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  if (configured_device == dev) return cudaSuccess;
  e = cudaFuncSetAttribute(linear_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(linear_tc_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  configured_device = dev;
  return cudaSuccess;
}

// Clusters of `splits` CTAs (each with smem_bytes of shared memory) that can
// be resident at once, from the occupancy API; cached per (device, shape).
int max_clusters(int splits, int smem_bytes, int tiles) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const auto key = std::make_tuple(dev, splits, smem_bytes);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  if (configure_kernel() != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(tiles, splits);
  cfg.blockDim = dim3(kLinThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem_bytes);
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 1;
  attr.val.clusterDim.y = static_cast<unsigned>(splits);
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, linear_tc_kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();  // a failed query leaves no error behind for the next call
    n = 0;
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = n;
  return n;
}

}  // namespace

// Shared-memory layout: TMA ring | mbarriers + TMEM slot | split-k receive
// buffer; the ring doubles as the CTA's [mpad][128] fp32 accumulator copy.
static void size_smem(LinearPlan& pl, int M, int splits, int stages) {
  const int stage_bytes = kWBytes + pl.mpad * 128;
  pl.stages = stages;
  const int bars = (2 * stages + 2) * 8 + 4;
  pl.recv_off = (stages * stage_bytes + bars + 15) / 16 * 16;
  const int per = (M + splits - 1) / splits;
  const int recv = splits > 1 ? splits * per * kTileN * 4 : 0;
  pl.smem_bytes = pl.recv_off + recv + 1024;
}

LinearPlan plan_linear(int32_t M, int32_t N, int32_t K) {
  LinearPlan pl{};
  pl.mpad = (M + 15) / 16 * 16;
  if (pl.mpad < 16) pl.mpad = 16;
  pl.tiles = N / kTileN;
  pl.chunks = K / kChunkK;
  const int stage_bytes = kWBytes + pl.mpad * 128;
  // two CTAs per SM while the ring still holds >= 4 stages, else one
  const int per_sm = (pl.mpad <= 64) ? 2 : 1;
  const int cap = (per_sm == 2 ? kSmemCap / 2 : kSmemCap);
  auto stages_for = [&](int splits) {
    const int per = (M + splits - 1) / splits;
    const int recv = splits > 1 ? splits * per * kTileN * 4 : 0;
    int st = (cap - recv - 1024 - 256) / stage_bytes;
    return st > kMaxStages ? kMaxStages : st;
  };
  // Split k over a cluster of up to 16 CTAs per W tile.  Each split keeps
  // >= 4 chunks at two CTAs per SM (fewer makes the cluster epilogue
  // dominate; measured: K = 1536 at <= 16 rows is fastest with 6 splits and
  // 2x slower with 8), the ring
  // (>= 3 stages) must hold the [mpad][128] fp32 accumulator copy, and the
  // grid must fit one wave: with two CTAs per SM, 90% of the CTA slots
  // (measured on B200: the occupancy API's cluster count is conservative
  // there); with one CTA per SM, the occupancy API's count of co-resident
  // clusters (a cluster too many runs as a second wave at twice the time).
  const int slots = sm_count() * per_sm;
  int smax = (per_sm == 2 ? slots * 9 / 10 : slots) / (pl.tiles > 0 ? pl.tiles : 1);
  if (smax > kMaxSplits) smax = kMaxSplits;
  if (per_sm == 2 && smax > pl.chunks / 4) smax = pl.chunks / 4;
  if (smax > pl.chunks / 2) smax = pl.chunks / 2;
  size_smem(pl, M, 1, stages_for(1));
  pl.splits = 1;
  for (int cand = smax; cand >= 2; --cand) {
    const int st = stages_for(cand);
    if (st < 3 || st * stage_bytes < pl.mpad * kTileN * 4) continue;
    LinearPlan trial = pl;
    size_smem(trial, M, cand, st);
    if (per_sm == 2 || max_clusters(cand, trial.smem_bytes, pl.tiles) >= pl.tiles) {
      pl = trial;
      pl.splits = cand;
      break;
    }
  }
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(pl.mpad)) cols <<= 1;
  pl.tmem_cols = cols;
  return pl;
}

cudaError_t launch_linear(const LinearLaunch& a, const LinearPlan& pl, const CUtensorMap& wmap,
                          const CUtensorMap& xmap, cudaStream_t stream) {
  cudaError_t e = configure_kernel();
  if (e != cudaSuccess) return e;
  LinParams p{};
  p.y = static_cast<__nv_bfloat16*>(a.y);
  p.ldy = a.ldy;
  p.bias = static_cast<const __nv_bfloat16*>(a.bias);
  p.M = a.M;
  p.N = a.N;
  p.chunks = pl.chunks;
  p.splits = pl.splits;
  p.stages = pl.stages;
  p.mpad = pl.mpad;
  p.tmem_cols = pl.tmem_cols;
  p.recv_off = pl.recv_off;
  p.w_tiled = a.w_tiled;
  p.swiglu = a.swiglu;
  p.rope = a.rope;
  // kind::f16 instruction descriptor: fp32 D, bf16 A and B, both K-major,
  // N = mpad (>> 3 at bit 17), M = 128 (>> 4 at bit 24)
  p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((static_cast<uint32_t>(pl.mpad) >> 3) << 17) |
            ((static_cast<uint32_t>(kTileN) >> 4) << 24);
  p.err = a.err;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.tiles, pl.splits);
  cfg.blockDim = dim3(kLinThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(pl.smem_bytes);
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2] = {};
  unsigned n = 0;
  if (pdl_enabled()) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (pl.splits > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = 1;
    attrs[n].val.clusterDim.y = static_cast<unsigned>(pl.splits);
    attrs[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, linear_tc_kernel, p, wmap, xmap);
}

cudaError_t launch_pair_gate_up(const void* w, int64_t ldw, int32_t inter, int32_t k, void* out,
                                cudaStream_t stream) {
  const int64_t total16 = static_cast<int64_t>(2) * inter * k / 8;
  return launch_k(pair_gate_up_kernel, dim3(static_cast<unsigned>((total16 + 255) / 256)),
                  dim3(256), 0, stream, static_cast<const __nv_bfloat16*>(w), ldw,
                  static_cast<int>(inter), static_cast<int>(k), total16,
                  static_cast<__nv_bfloat16*>(out));
}

cudaError_t launch_pack_weight(const void* w, int64_t ldw, int32_t n, int32_t k, void* out,
                               cudaStream_t stream) {
  const int64_t total16 = static_cast<int64_t>(n) * k / 8;
  return launch_k(pack_weight_kernel, dim3(static_cast<unsigned>((total16 + 255) / 256)),
                  dim3(256), 0, stream, static_cast<const __nv_bfloat16*>(w), ldw, k / kChunkK,
                  total16, static_cast<__nv_bfloat16*>(out));
}

}  // namespace pkv
