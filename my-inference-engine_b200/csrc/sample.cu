// Temperature sampling of one token per row on the device (sm_100a).
//
// Contract: chat.py:103-107 of the reference, `softmax(logits.float() / T)`
// followed by `torch.multinomial(probs, 1)`: one id per row drawn from the
// categorical distribution softmax(logits / T).  Here in ONE pass over the
// logits, with no probability tensor: by the Gumbel-max trick,
//     argmax_i ( logits_i / T + G_i ),   G_i = -ln(-ln U_i) i.i.d. Gumbel(0, 1)
// is distributed exactly as that categorical (the softmax normaliser is a
// constant shift of every score).
//
// Uniforms: Philox-4x32-10 (J. Salmon, M. Moraes, R. Dror, D. Shaw, "Parallel
// random numbers: as easy as 1, 2, 3", SC'11), a counter-based generator:
// key = the 64-bit seed, counter = (element quad, row, call low, call high),
// so a draw depends only on (seed, call, row, element) -- reproducible, and
// independent of the grid shape.  Every Gumbel draw is finite (|G| < 17).
//
// Grid (splits, rows) with the `splits` CTAs of a row forming one thread-block
// cluster: each CTA reduces a contiguous slice of the vocabulary to its best
// (score, index), then cluster rank 0 reads the others' results from their
// shared memory.  Ties go to the lower index.  A row without a finite score
// (NaN / -inf logits everywhere) yields -1, which the host turns into the
// reference's RuntimeError.
#include <cooperative_groups.h>
#include <math.h>

#include <map>
#include <mutex>
#include <utility>

#include "pkv_device.cuh"
#include "pkv_kernels.h"

namespace cg = cooperative_groups;

namespace pkv {
namespace {

constexpr int kSampleThreads = 512;
constexpr int kMaxSampleSplits = 8;  // portable cluster size
constexpr int kNoIndex = 0x7fffffff;

// Philox-4x32 round constants from the paper (multipliers and Weyl key
// increments).
constexpr uint32_t kPhiloxM0 = 0xD2511F53u, kPhiloxM1 = 0xCD9E8D57u;
constexpr uint32_t kPhiloxW0 = 0x9E3779B9u, kPhiloxW1 = 0xBB67AE85u;

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(kPhiloxM0, c.x), lo0 = kPhiloxM0 * c.x;
    const uint32_t hi1 = __umulhi(kPhiloxM1, c.z), lo1 = kPhiloxM1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += kPhiloxW0;
    k.y += kPhiloxW1;
  }
  return c;
}

// Gumbel(0, 1) from 32 random bits: G = -ln E with E = -ln(1 - V) ~ Exp(1)
// and V uniform in (0, 1).  V = (23 bits + 0.5) / 2^23 is exact in fp32 and
// never 0 or 1.  Where V < 1/16, 1 - V is so close to 1 that a fast log
// loses relative accuracy in E, so E comes from the series V + V^2/2 + V^3/3
// + V^4/4 there (relative error < V^4/5 < 4e-6); elsewhere from the log.
__device__ __forceinline__ float gumbel(uint32_t bits) {
  const float v = fmaf(static_cast<float>(bits >> 9), 1.0f / 8388608.0f, 1.0f / 16777216.0f);
  const float series = v * fmaf(v, fmaf(v, fmaf(v, 0.25f, 0.33333334f), 0.5f), 1.0f);
  const float e = v < 0.0625f ? series : -__logf(1.0f - v);
  return -__logf(e);
}

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <>
__device__ __forceinline__ float to_f32<float>(float x) {
  return x;
}

// (score, index) order: higher score first, then lower index; NaN scores
// never win (every comparison with NaN is false).
__device__ __forceinline__ bool better(float s, int i, float bs, int bi) {
  return s > bs || (s == bs && i < bi);
}

template <typename T>
__global__ void __launch_bounds__(kSampleThreads)
    sample_kernel(const T* __restrict__ logits, int64_t ld, int vocab, float inv_temp,
                  uint64_t seed, uint64_t call, int vec, int32_t* __restrict__ out) {
  __shared__ float s_best[kSampleThreads / 32];
  __shared__ int s_idx[kSampleThreads / 32];
  pdl_trigger();
  pdl_wait();
  cg::cluster_group cluster = cg::this_cluster();
  const int row = blockIdx.y;
  const int splits = gridDim.x;
  const int rank = blockIdx.x;  // == cluster rank: the cluster spans grid.x
  const int quads = (vocab + 3) >> 2;
  const int per = (quads + splits - 1) / splits;
  const int q_begin = rank * per, q_end = min(quads, q_begin + per);
  const T* x = logits + static_cast<int64_t>(row) * ld;
  const uint2 key = make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));

  float best = -INFINITY;
  int bidx = kNoIndex;
  for (int q = q_begin + static_cast<int>(threadIdx.x); q < q_end; q += kSampleThreads) {
    const uint4 r = philox4x32_10(
        make_uint4(static_cast<uint32_t>(q), static_cast<uint32_t>(row),
                   static_cast<uint32_t>(call), static_cast<uint32_t>(call >> 32)),
        key);
    float v[4];
    const int e0 = q * 4;
    if (vec && e0 + 3 < vocab) {  // 4-wide loads: the host checked row alignment
      if constexpr (sizeof(T) == 2) {
        const uint2 raw = *reinterpret_cast<const uint2*>(x + e0);
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = to_f32(h[e]);
      } else {
        const float4 raw = *reinterpret_cast<const float4*>(x + e0);
        v[0] = raw.x;
        v[1] = raw.y;
        v[2] = raw.z;
        v[3] = raw.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = e0 + e < vocab ? to_f32(x[e0 + e]) : NAN;
    }
    const uint32_t bits[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float s = fmaf(v[e], inv_temp, gumbel(bits[e]));
      if (better(s, e0 + e, best, bidx)) {
        best = s;
        bidx = e0 + e;
      }
    }
  }
  // CTA: warp shuffles, then one warp over the warp results
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float os = __shfl_xor_sync(0xffffffffu, best, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bidx, off);
    if (better(os, oi, best, bidx)) {
      best = os;
      bidx = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_best[warp] = best;
    s_idx[warp] = bidx;
  }
  __syncthreads();
  if (warp == 0) {
    best = lane < kSampleThreads / 32 ? s_best[lane] : -INFINITY;
    bidx = lane < kSampleThreads / 32 ? s_idx[lane] : kNoIndex;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float os = __shfl_xor_sync(0xffffffffu, best, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bidx, off);
      if (better(os, oi, best, bidx)) {
        best = os;
        bidx = oi;
      }
    }
    if (lane == 0) {
      s_best[0] = best;
      s_idx[0] = bidx;
    }
  }
  // cluster: rank 0 merges the other CTAs' results from their shared memory
  cluster.sync();
  if (rank == 0 && threadIdx.x == 0) {
    float b = s_best[0];
    int bi = s_idx[0];
    for (int rr = 1; rr < splits; ++rr) {
      const float os = *cluster.map_shared_rank(&s_best[0], rr);
      const int oi = *cluster.map_shared_rank(&s_idx[0], rr);
      if (better(os, oi, b, bi)) {
        b = os;
        bi = oi;
      }
    }
    // no finite score in the row (all NaN or -inf): -1, reported on the host
    out[row] = (bi == kNoIndex || !(b > -INFINITY) || !(b < INFINITY)) ? -1 : bi;
  }
  cluster.sync();  // every CTA's shared memory stays valid until rank 0 has read it
}

template <typename T>
cudaError_t launch_sample_t(const SampleLaunch& a, cudaStream_t stream) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a.splits, a.rows, 1);
  cfg.blockDim = dim3(kSampleThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = a.splits;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, sample_kernel<T>, static_cast<const T*>(a.logits), a.ld,
                            a.vocab, a.inv_temp, a.seed, a.call, a.vec, a.out);
}

// Co-resident clusters of `s` sampler CTAs on the current device (a cluster
// lives inside one GPC, so this is below slots / s for larger s); cached
// per (device, s).
int sample_clusters(int s) {
  static std::mutex mu;
  static std::map<std::pair<int, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const auto key = std::make_pair(dev, s);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(s), 1, 1);
  cfg.blockDim = dim3(kSampleThreads, 1, 1);
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = static_cast<unsigned>(s);
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, sample_kernel<__nv_bfloat16>, &cfg) != cudaSuccess) {
    cudaGetLastError();  // a failed query leaves no error behind for the next call
    n = 0;
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = n;
  return n;
}

}  // namespace

int sample_splits(int32_t rows, int32_t vocab) {
  // Each of a row's `s` CTAs (one cluster) scans vocab / s logits; the grid
  // runs in ceil(rows / co-resident clusters) waves, so the time goes as
  // waves / s.  Take the smallest s (1..8, >= ~4096 logits per CTA) that
  // minimises it: a split that spills a few clusters into a second wave is
  // slower than one that leaves some SMs idle (measured: 128 rows, 3 splits
  // = 1.3 waves, 48 us).
  const int cap = max(1, min(kMaxSampleSplits, vocab / 4096));
  const int64_t r = rows > 0 ? rows : 1;
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= cap; ++s) {
    const int clusters = sample_clusters(s);
    if (clusters <= 0) continue;
    const int64_t waves = (r + clusters - 1) / clusters;
    const double cost = static_cast<double>(waves) / s;
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

cudaError_t launch_sample(const SampleLaunch& a, cudaStream_t stream) {
  return a.f32 ? launch_sample_t<float>(a, stream) : launch_sample_t<__nv_bfloat16>(a, stream);
}

}  // namespace pkv
