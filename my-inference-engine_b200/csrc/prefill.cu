// Ragged causal prefill attention over paged (or dense) K/V for sm_100a.
//
// Reference behaviour: kernels/fa2.py:23-162 with is_causal = T > 1
// (model.py:185): query i of row b sits at key position i + kv_len - T
// (bottom-right alignment, fa2.py:110-111), keys at or past kv_len are
// masked (fa2.py:132-136), online softmax in fp32 (fa2.py:117-148), P is
// rounded to the value dtype before the PV product (fa2.py:145).
//
//   grid  = (ceil(T/16), kv_heads * sub_groups, batch)
//   block = nheads consumer warps (one query head of the KV group each,
//           16 query rows) + 1 producer warp that streams 64-token K/V tiles
//           (4 blocks) into an NST-deep ring with TMA.
// All query heads of the group share each K/V tile in shared memory.
#include <math.h>

#include "pkv_device.cuh"
#include "pkv_kernels.h"

namespace pkv {
namespace {

constexpr int kTileBlocks = 4;                                // 64 tokens
constexpr int kTileBytes = kTileBlocks * kHeadBlockBytes;     // K or V: 16 KiB
constexpr int kPrefillStages = 2;
constexpr int kMaxHeadsPerCta = 8;

struct PrefillParams {
  const __nv_bfloat16* q;
  int64_t q_sb, q_sh, q_st;
  __nv_bfloat16* out;
  int64_t o_sb, o_sh, o_st;
  const int32_t* kv_lens;
  const int32_t* tables;
  int64_t pitch;
  const int32_t* rows;
  int32_t num_blocks;
  int32_t T;
  int32_t group;
  int32_t sub_groups;
  int32_t causal;
  float scale_log2;
  int32_t* err;
};

constexpr int prefill_smem_bytes() {
  return kPrefillStages * 2 * kTileBytes + kPrefillStages * 2 * 8 + 1024;
}

template <bool kPaged>
__global__ void __launch_bounds__((kMaxHeadsPerCta + 1) * 32, 1)
    prefill_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap) {
  constexpr int NST = kPrefillStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * 2 * kTileBytes);
  uint64_t* empty = full + NST;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int b = blockIdx.z;
  const int y = blockIdx.y;
  const int kvh = y / p.sub_groups;
  const int sub = y - kvh * p.sub_groups;
  const int head0 = kvh * p.group + sub * kMaxHeadsPerCta;
  const int nheads = min(kMaxHeadsPerCta, p.group - sub * kMaxHeadsPerCta);
  const int q0 = blockIdx.x * 16;
  const int T = p.T;
  const DevErr err{p.err};

  int kv_len = max(p.kv_lens[b], 0);
  const int32_t* trow = nullptr;
  if constexpr (kPaged) {
    const int row = p.rows ? p.rows[b] : b;
    trow = p.tables + static_cast<int64_t>(row) * p.pitch;
    if (kv_len > p.pitch * kBlockTokens) {
      if (tid == 0 && blockIdx.x == 0) err.raise(PKV_DEVERR_POSITION);
      kv_len = static_cast<int>(p.pitch) * kBlockTokens;
    }
  }
  const int offset = kv_len - T;  // query i sits at key position i + offset
  int kv_end = kv_len;
  if (p.causal) kv_end = min(kv_len, min(q0 + 16, T) - 1 + offset + 1);
  kv_end = max(kv_end, 0);
  const int nblk = (kv_end + kBlockTokens - 1) / kBlockTokens;
  const int ntiles = (nblk + kTileBlocks - 1) / kTileBlocks;

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], nheads);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == nheads) {
    // ---------------- producer warp ----------------
    if (lane == 0) {
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
      const uint64_t policy = policy_evict_last();
      for (int i = 0; i < ntiles; ++i) {
        const int st = i % NST;
        if (i >= NST && !mbar_wait(&empty[st], ((i / NST) - 1) & 1, err)) break;
        const int nb = min(kTileBlocks, nblk - i * kTileBlocks);
        uint8_t* kt = smem + st * 2 * kTileBytes;
        uint8_t* vt = kt + kTileBytes;
        mbar_arrive_expect_tx(&full[st], nb * 2 * kHeadBlockBytes);
        for (int jb = 0; jb < nb; ++jb) {
          const int j = i * kTileBlocks + jb;
          uint8_t* kd = kt + jb * kHeadBlockBytes;
          uint8_t* vd = vt + jb * kHeadBlockBytes;
          if constexpr (kPaged) {
            int blk = trow[j];
            if (blk < 0 || blk >= p.num_blocks) {
              err.raise(PKV_DEVERR_BLOCK_ID);
              blk = 0;
            }
            const int slot = blk * kBlockTokens;
            tma_load_3d(kd, &kmap, &full[st], 0, kvh, slot, policy);
            tma_load_3d(kd + kBoxBytes, &kmap, &full[st], 64, kvh, slot, policy);
            tma_load_3d(vd, &vmap, &full[st], 0, kvh, slot, policy);
            tma_load_3d(vd + kBoxBytes, &vmap, &full[st], 64, kvh, slot, policy);
          } else {
            const int tok = j * kBlockTokens;
            tma_load_4d(kd, &kmap, &full[st], 0, tok, kvh, b, policy);
            tma_load_4d(kd + kBoxBytes, &kmap, &full[st], 64, tok, kvh, b, policy);
            tma_load_4d(vd, &vmap, &full[st], 0, tok, kvh, b, policy);
            tma_load_4d(vd + kBoxBytes, &vmap, &full[st], 64, tok, kvh, b, policy);
          }
        }
      }
    }
    return;
  }
  if (warp > nheads) return;

  // ---------------- consumer warp: query head head0 + warp ----------------
  const int hq = head0 + warp;
  const int r0 = q0 + g, r1 = q0 + g + 8;  // query rows of this lane
  uint32_t qa[8][4];
  {
    const __nv_bfloat16* qb = p.q + b * p.q_sb + hq * p.q_sh;
    const __nv_bfloat16* qr0 = qb + static_cast<int64_t>(min(r0, T - 1)) * p.q_st;
    const __nv_bfloat16* qr1 = qb + static_cast<int64_t>(min(r1, T - 1)) * p.q_st;
    const bool v0 = r0 < T, v1 = r1 < T;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int c = kk * 16 + 2 * t;
      qa[kk][0] = v0 ? *reinterpret_cast<const uint32_t*>(qr0 + c) : 0u;
      qa[kk][1] = v1 ? *reinterpret_cast<const uint32_t*>(qr1 + c) : 0u;
      qa[kk][2] = v0 ? *reinterpret_cast<const uint32_t*>(qr0 + c + 8) : 0u;
      qa[kk][3] = v1 ? *reinterpret_cast<const uint32_t*>(qr1 + c + 8) : 0u;
    }
  }
  const int lim0 = p.causal ? min(kv_len, r0 + offset + 1) : kv_len;  // keys < lim visible
  const int lim1 = p.causal ? min(kv_len, r1 + offset + 1) : kv_len;

  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  const int q4 = lane >> 3, r8 = lane & 7;
  bool ok = true;
  for (int i = 0; i < ntiles; ++i) {
    const int st = i % NST;
    ok = __all_sync(0xffffffffu, mbar_wait(&full[st], (i / NST) & 1, err));
    if (!ok) break;
    const uint32_t kt = smem_u32(smem + st * 2 * kTileBytes);
    const uint32_t vt = kt + kTileBytes;
    const int nb = min(kTileBlocks, nblk - i * kTileBlocks);
    const int key0 = i * kTileBlocks * kBlockTokens;

    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int np = 0; np < 4; ++np) {  // pairs of 8-token n-tiles == one block
      if (np < nb) {
        const int tok = np * 16 + (q4 >> 1) * 8 + r8;  // token within tile
        const uint32_t rowbase = kt + np * kHeadBlockBytes;
        const int rib = tok & 15;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const int chunk = 2 * kk + (q4 & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(rowbase + (chunk >> 3) * kBoxBytes + swz128(rib, chunk & 7), b0, b1, b2, b3);
          mma_bf16(s[2 * np], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
          mma_bf16(s[2 * np + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
        }
      }
    }
    // scale, mask, row max
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int key = key0 + n * 8 + 2 * t;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool in_tile = (n >> 1) < nb;
        float a = s[n][e] * p.scale_log2, c = s[n][2 + e] * p.scale_log2;
        if (!in_tile || key + e >= lim0) a = -INFINITY;
        if (!in_tile || key + e >= lim1) c = -INFINITY;
        s[n][e] = a;
        s[n][2 + e] = c;
        mx0 = fmaxf(mx0, a);
        mx1 = fmaxf(mx1, c);
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float base0 = mn0 == -INFINITY ? 0.f : mn0;
    const float base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = ex2(m0 - base0), al1 = ex2(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      s[n][0] = ex2(s[n][0] - base0);
      s[n][1] = ex2(s[n][1] - base0);
      s[n][2] = ex2(s[n][2] - base1);
      s[n][3] = ex2(s[n][3] - base1);
      rs0 += s[n][0] + s[n][1];
      rs1 += s[n][2] + s[n][3];
    }
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= al0;
      o[n][1] *= al0;
      o[n][2] *= al1;
      o[n][3] *= al1;
    }
    // O += P . V, one 16-token k-step per block
#pragma unroll
    for (int kb = 0; kb < 4; ++kb) {
      if (kb < nb) {
        const uint32_t a0 = pack_bf16(s[2 * kb][0], s[2 * kb][1]);
        const uint32_t a1 = pack_bf16(s[2 * kb][2], s[2 * kb][3]);
        const uint32_t a2 = pack_bf16(s[2 * kb + 1][0], s[2 * kb + 1][1]);
        const uint32_t a3 = pack_bf16(s[2 * kb + 1][2], s[2 * kb + 1][3]);
        const uint32_t vb = vt + kb * kHeadBlockBytes;
        const int rib = (q4 & 1) * 8 + r8;  // token within block
#pragma unroll
        for (int nd = 0; nd < 16; nd += 2) {
          const int chunk = nd + (q4 >> 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vb + (chunk >> 3) * kBoxBytes + swz128(rib, chunk & 7), b0, b1, b2, b3);
          mma_bf16(o[nd], a0, a1, a2, a3, b0, b1);
          mma_bf16(o[nd + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  if (!ok) {
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
  }
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;  // 0/0 -> NaN for a row with no keys
  __nv_bfloat16* ob = p.out + b * p.o_sb + hq * p.o_sh;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int c = n * 8 + 2 * t;
    if (r0 < T)
      *reinterpret_cast<uint32_t*>(ob + static_cast<int64_t>(r0) * p.o_st + c) =
          pack_bf16(o[n][0] * inv0, o[n][1] * inv0);
    if (r1 < T)
      *reinterpret_cast<uint32_t*>(ob + static_cast<int64_t>(r1) * p.o_st + c) =
          pack_bf16(o[n][2] * inv1, o[n][3] * inv1);
  }
}

template <bool kPaged>
cudaError_t launch_prefill_t(const PrefillParams& prm, const KVSource& src, dim3 grid, int nheads,
                             cudaStream_t stream) {
  auto kern = prefill_kernel<kPaged>;
  constexpr int smem = prefill_smem_bytes();
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
  kern<<<grid, (nheads + 1) * 32, smem, stream>>>(prm, src.kmap, src.vmap);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill(const PrefillLaunch& a, const KVSource& src, cudaStream_t stream) {
  PrefillParams prm{};
  prm.q = static_cast<const __nv_bfloat16*>(a.q);
  prm.q_sb = a.q_sb;
  prm.q_sh = a.q_sh;
  prm.q_st = a.q_st;
  prm.out = static_cast<__nv_bfloat16*>(a.out);
  prm.o_sb = a.o_sb;
  prm.o_sh = a.o_sh;
  prm.o_st = a.o_st;
  prm.kv_lens = a.kv_lens;
  prm.tables = src.tables;
  prm.pitch = src.pitch;
  prm.rows = src.rows;
  prm.num_blocks = src.num_blocks;
  prm.T = a.seq_len_q;
  prm.group = a.num_q_heads / a.num_kv_heads;
  prm.sub_groups = (prm.group + kMaxHeadsPerCta - 1) / kMaxHeadsPerCta;
  prm.causal = a.causal;
  prm.scale_log2 = a.sm_scale * 1.4426950408889634f;
  prm.err = a.err;
  const int nheads = min(kMaxHeadsPerCta, prm.group);
  dim3 grid((a.seq_len_q + 15) / 16, a.num_kv_heads * prm.sub_groups, a.batch);
  return src.paged ? launch_prefill_t<true>(prm, src, grid, nheads, stream)
                   : launch_prefill_t<false>(prm, src, grid, nheads, stream);
}

}  // namespace pkv
