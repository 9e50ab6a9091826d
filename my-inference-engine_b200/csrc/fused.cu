// Fused elementwise kernels of the Qwen2 block around the attention path
// (sm_100a): residual add + RMSNorm, and SiLU(gate) * up.
//
// Reference op sequences (all on bf16 tensors, every torch op rounding its
// fp32 result to bf16):
//   model.py:136-137  x = x + attention_output ; x = x + mlp(...)
//   model.py:49-55    RMSNorm: h = x.float(); v = mean(h*h); h = h * rsqrt(v + eps);
//                     out = weight * h.to(bf16)
//   model.py:120      down_proj(silu(gate_proj(x)) * up_proj(x))
// One CTA per row for the norm (warp + shared-memory reduction of the sum
// of squares); the SiLU product is a flat 8-wide vectorised loop.
#include "pkv_device.cuh"
#include "pkv_kernels.h"

namespace pkv {
namespace {

__device__ __forceinline__ float bf(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 rn(float x) { return __float2bfloat16_rn(x); }

constexpr int kNormThreads = 256;

// One CTA per row: thread i owns elements [8i, 8i+8) (+ 2048 for dim > 2048).
// h = a (+ resid) in bf16; resid_out = h; out = weight * bf16(h * rsqrt(mean(h^2) + eps))
// One warp per row (dim % 256 == 0, dim <= 2048, >= 1024 rows): lane l owns
// the 16-byte chunks l, l+32, ... of the row; the sum of squares is a
// shuffle tree, no shared memory or block barrier, so every row of a
// prefill is in flight at once.  Same arithmetic per element as
// add_rmsnorm_kernel.
constexpr int kNormRowsPerCta = 8;
template <int kChunks>
__global__ void __launch_bounds__(32 * kNormRowsPerCta)
    add_rmsnorm_warp_kernel(const __nv_bfloat16* __restrict__ a, int64_t a_stride,
                            const __nv_bfloat16* resid, int64_t r_stride,
                            __nv_bfloat16* resid_out, int64_t ro_stride,
                            const __nv_bfloat16* __restrict__ weight,
                            __nv_bfloat16* __restrict__ out, int64_t o_stride, int rows, int dim,
                            float eps) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * kNormRowsPerCta + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  uint4 av[kChunks], rv[kChunks], wv[kChunks];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    av[c] = *reinterpret_cast<const uint4*>(a + row * a_stride + (c * 32 + lane) * 8);
    if (resid) rv[c] = *reinterpret_cast<const uint4*>(resid + row * r_stride + (c * 32 + lane) * 8);
    // the norm weight with the row: its load overlaps the sum of squares
    wv[c] = __ldg(reinterpret_cast<const uint4*>(weight + (c * 32 + lane) * 8));
  }
  float h[kChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const __nv_bfloat16* ap = reinterpret_cast<const __nv_bfloat16*>(&av[c]);
    uint4 hv;
    __nv_bfloat16* hp = reinterpret_cast<__nv_bfloat16*>(&hv);
    if (resid) {
      const __nv_bfloat16* rp = reinterpret_cast<const __nv_bfloat16*>(&rv[c]);
#pragma unroll
      for (int e = 0; e < 8; ++e) hp[e] = rn(__fadd_rn(bf(rp[e]), bf(ap[e])));
    } else {
      hv = av[c];
    }
    if (resid_out)
      *reinterpret_cast<uint4*>(resid_out + row * ro_stride + (c * 32 + lane) * 8) = hv;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      h[c][e] = bf(hp[e]);
      ss = __fadd_rn(ss, __fmul_rn(h[c][e], h[c][e]));
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float r = rsqrtf(__fadd_rn(ss * (1.0f / static_cast<float>(dim)), eps));
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = (c * 32 + lane) * 8;
    const __nv_bfloat16* wp = reinterpret_cast<const __nv_bfloat16*>(&wv[c]);
    uint4 ov;
    __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
    for (int e = 0; e < 8; ++e) op[e] = rn(__fmul_rn(bf(wp[e]), bf(rn(__fmul_rn(h[c][e], r)))));
    *reinterpret_cast<uint4*>(out + row * o_stride + col) = ov;
  }
}

__global__ void __launch_bounds__(kNormThreads)
    add_rmsnorm_kernel(const __nv_bfloat16* __restrict__ a, int64_t a_stride,
                       const __nv_bfloat16* resid, int64_t r_stride, __nv_bfloat16* resid_out,
                       int64_t ro_stride, const __nv_bfloat16* __restrict__ weight,
                       __nv_bfloat16* __restrict__ out, int64_t o_stride, int rows, int dim,
                       float eps) {
  __shared__ float warp_ss[kNormThreads / 32];
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  float h[2][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int col = (c * kNormThreads + tid) * 8;
    if (col < dim) {
      const uint4 av = *reinterpret_cast<const uint4*>(a + row * a_stride + col);
      const __nv_bfloat16* ap = reinterpret_cast<const __nv_bfloat16*>(&av);
      uint4 hv;
      __nv_bfloat16* hp = reinterpret_cast<__nv_bfloat16*>(&hv);
      if (resid) {
        const uint4 rv = *reinterpret_cast<const uint4*>(resid + row * r_stride + col);
        const __nv_bfloat16* rp = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
        for (int e = 0; e < 8; ++e) hp[e] = rn(__fadd_rn(bf(rp[e]), bf(ap[e])));
      } else {
        hv = av;
      }
      if (resid_out) *reinterpret_cast<uint4*>(resid_out + row * ro_stride + col) = hv;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        h[c][e] = bf(hp[e]);
        ss = __fadd_rn(ss, __fmul_rn(h[c][e], h[c][e]));
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((tid & 31) == 0) warp_ss[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += warp_ss[w];
  const float r = rsqrtf(__fadd_rn(tot * (1.0f / static_cast<float>(dim)), eps));
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int col = (c * kNormThreads + tid) * 8;
    if (col < dim) {
      const uint4 wv = *reinterpret_cast<const uint4*>(weight + col);
      const __nv_bfloat16* wp = reinterpret_cast<const __nv_bfloat16*>(&wv);
      uint4 ov;
      __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
      for (int e = 0; e < 8; ++e) op[e] = rn(__fmul_rn(bf(wp[e]), bf(rn(__fmul_rn(h[c][e], r)))));
      *reinterpret_cast<uint4*>(out + row * o_stride + col) = ov;
    }
  }
}

// grid (rows, column chunks of kSiluThreads x 8 elements): the row and
// column come straight from the block index, no integer division per thread
constexpr int kSiluThreads = 128;

__global__ void __launch_bounds__(kSiluThreads)
    silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int64_t gu_stride,
                    __nv_bfloat16* __restrict__ out, int64_t o_stride, int rows, int inter) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const int j = blockIdx.y * kSiluThreads + threadIdx.x;
  if (row >= rows || j >= inter / 8) return;
  const int col = j * 8;
  const uint4 gv = *reinterpret_cast<const uint4*>(gu + row * gu_stride + col);
  const uint4 uv = *reinterpret_cast<const uint4*>(gu + row * gu_stride + inter + col);
  const __nv_bfloat16* gp = reinterpret_cast<const __nv_bfloat16*>(&gv);
  const __nv_bfloat16* up = reinterpret_cast<const __nv_bfloat16*>(&uv);
  // F.silu in fp32, rounded to bf16, times up, rounded to bf16; the roundings
  // go two values per cvt.rn.bf16x2 (the conversions share the MUFU/XU pipe
  // with expf and the division, which bounds this kernel)
  uint4 ov;
  __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    const float g0 = bf(gp[e]), g1 = bf(gp[e + 1]);
    const __nv_bfloat162 s = __floats2bfloat162_rn(g0 / (1.0f + expf(-g0)), g1 / (1.0f + expf(-g1)));
    op[e / 2] = __floats2bfloat162_rn(__fmul_rn(__low2float(s), bf(up[e])),
                                      __fmul_rn(__high2float(s), bf(up[e + 1])));
  }
  *reinterpret_cast<uint4*>(out + row * o_stride + col) = ov;
}

}  // namespace

cudaError_t launch_add_rmsnorm(const NormLaunch& p, cudaStream_t stream) {
  // warp per row for prefill-sized launches (all rows in flight at once);
  // a decode step's few rows keep one CTA each, i.e. one SM each
  if (p.dim % 256 == 0 && p.dim <= 2048 && p.rows >= 1024) {
    const dim3 grid((p.rows + kNormRowsPerCta - 1) / kNormRowsPerCta), block(32 * kNormRowsPerCta);
    auto args = [&](auto kern) {
      return launch_k(kern, grid, block, 0, stream, static_cast<const __nv_bfloat16*>(p.a),
                      p.a_stride, static_cast<const __nv_bfloat16*>(p.resid), p.r_stride,
                      static_cast<__nv_bfloat16*>(p.resid_out), p.ro_stride,
                      static_cast<const __nv_bfloat16*>(p.weight),
                      static_cast<__nv_bfloat16*>(p.out), p.o_stride, static_cast<int>(p.rows),
                      static_cast<int>(p.dim), p.eps);
    };
    switch (p.dim / 256) {
      case 1: return args(add_rmsnorm_warp_kernel<1>);
      case 2: return args(add_rmsnorm_warp_kernel<2>);
      case 3: return args(add_rmsnorm_warp_kernel<3>);
      case 4: return args(add_rmsnorm_warp_kernel<4>);
      case 5: return args(add_rmsnorm_warp_kernel<5>);
      case 6: return args(add_rmsnorm_warp_kernel<6>);
      case 7: return args(add_rmsnorm_warp_kernel<7>);
      default: return args(add_rmsnorm_warp_kernel<8>);
    }
  }
  return launch_k(add_rmsnorm_kernel, dim3(p.rows), dim3(kNormThreads), 0, stream,
                  static_cast<const __nv_bfloat16*>(p.a), p.a_stride,
                  static_cast<const __nv_bfloat16*>(p.resid), p.r_stride,
                  static_cast<__nv_bfloat16*>(p.resid_out), p.ro_stride,
                  static_cast<const __nv_bfloat16*>(p.weight), static_cast<__nv_bfloat16*>(p.out),
                  p.o_stride, static_cast<int>(p.rows), static_cast<int>(p.dim), p.eps);
}

cudaError_t launch_silu_mul(const void* gu, int64_t gu_stride, void* out, int64_t o_stride,
                            int32_t rows, int32_t inter, cudaStream_t stream) {
  const int per_row = inter / 8;
  if (rows == 0 || per_row == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>(rows),
                  static_cast<unsigned>((per_row + kSiluThreads - 1) / kSiluThreads));
  return launch_k(silu_mul_kernel, grid, dim3(kSiluThreads), 0, stream,
                  static_cast<const __nv_bfloat16*>(gu), gu_stride,
                  static_cast<__nv_bfloat16*>(out), o_stride, static_cast<int>(rows),
                  static_cast<int>(inter));
}

}  // namespace pkv
