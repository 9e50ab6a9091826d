// Host-side launch interface between the C ABI layer (capi.cu) and the
// kernel translation units.  Not part of the public ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <cuda_bf16.h>

namespace pkv {

// Where K/V rows come from: the paged pool (3-D tensor map over
// [slot][kv_head][128]) or a dense [B][Hkv][S][128] tensor (4-D map).
struct KVSource {
  bool paged;
  CUtensorMap kmap;
  CUtensorMap vmap;
  const int32_t* tables;  // paged only
  int64_t pitch;
  const int32_t* rows;
  int32_t num_blocks;
};

// FP8 (e4m3) KV pool, opt-in: per layer [num_blocks][Hkv][kFp8HeadBlockBytes],
// one chunk per (16-token block, KV head), fetched by one bulk copy:
//   [0, 2048)     K, 16 token rows of 128 bytes; 16-byte chunk c of token t
//                 sits at chunk c ^ (t & 7) (conflict-free ldmatrix); inside
//                 a chunk byte 4i+u holds dim 2i+u (u < 2) or 2i+8+u-2 (u >= 2),
//                 the order an m16n8k16 A fragment wants
//   [2048, 4096)  V transposed, 128 dim rows of 16 bytes; byte 4i+u holds
//                 token 2i+u (u < 2) or 2i+8+u-2 (u >= 2)
//   [4096, 4160)  fp32 dequantisation scale of each token's K row
//   [4160, 4224)  fp32 scale of each token's V row
// value = e4m3 * scale, scale = amax(|row|) / 448 (1 for an all-zero row).
constexpr int kFp8VOff = 2048;
constexpr int kFp8KScaleOff = 4096;
constexpr int kFp8VScaleOff = 4160;
constexpr int kFp8HeadBlockBytes = 4224;

struct DecodeLaunch {
  const void* q;
  int64_t q_sb, q_sh;
  void* out;
  int64_t o_sb, o_sh;
  const int32_t* kv_lens;
  int32_t batch, num_q_heads, num_kv_heads;
  int32_t max_kv_len;
  float sm_scale;
  void* workspace;
  size_t workspace_bytes;
  int32_t* err;
  const uint8_t* kv8 = nullptr;  // FP8 pool of one layer (KVSource.paged tables)
};

struct DecodePlan {
  int32_t sub_groups;       // ceil(group / 8): CTAs sharing one KV head
  int32_t blocks_per_part;  // 16-token blocks per split-K partition
  int32_t max_parts;        // grid.x
  int32_t min_blocks_per_part;  // a row's partitions hold at least this many blocks
  size_t workspace_bytes;   // 0 when max_parts == 1
};

// Fixed head of every split-K workspace: the completion counters.
size_t decode_counter_bytes();
int64_t decode_max_units();  // rows * kv_heads * sub_groups per launch

// fp8: the plan of the FP8-pool kernel (twice the resident CTAs per SM)
DecodePlan plan_decode(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                       int32_t max_kv_len, bool fp8 = false);
cudaError_t launch_decode(const DecodeLaunch& a, const KVSource& src, const DecodePlan& plan,
                          cudaStream_t stream);
// Same launch with the split-K scratch taken from the library's static device
// array (per-device address set up on first use); see decode.cu.
cudaError_t launch_decode_static(const DecodeLaunch& a, const KVSource& src,
                                 const DecodePlan& plan, cudaStream_t stream);

struct PrefillLaunch {
  const void* q;
  int64_t q_sb, q_sh, q_st;
  void* out;
  int64_t o_sb, o_sh, o_st;
  const int32_t* kv_lens;
  const int32_t* q_lens;  // nullable: every row has seq_len_q queries
  int32_t batch, seq_len_q, num_q_heads, num_kv_heads;
  int32_t causal;
  float sm_scale;
  int32_t* err;
};
// tcgen05/TMEM prefill; qmap: 4-D map over q [B][Hq][T][128], box {64,128,1,1}
cudaError_t launch_prefill_tc(const PrefillLaunch& a, const CUtensorMap& qmap, const KVSource& src,
                              cudaStream_t stream);

struct AppendLaunch {
  const void* q;
  int64_t q_sb, q_sh, q_st;
  const void* k;
  int64_t k_sb, k_sh, k_st;
  const void* v;
  int64_t v_sb, v_sh, v_st;
  const void* rope_cos;
  const void* rope_sin;
  int64_t rope_rows;
  void* q_out;
  int64_t qo_sb, qo_sh, qo_st;
  void* k_pool;
  void* v_pool;
  int64_t num_slots;
  const int32_t* tables;
  int64_t pitch;
  const int32_t* rows;
  const int32_t* starts;
  const int32_t* q_lens;  // nullable
  int32_t batch, num_q_heads, num_kv_heads, seq_len_q;
  int32_t* err;
  uint8_t* kv8 = nullptr;  // FP8 pool of one layer: k/v quantised there (k_pool/v_pool unused)
};
cudaError_t launch_append(const AppendLaunch& a, cudaStream_t stream);

// FP8 pool -> dense bf16 K and V [B][Hkv][S][128] (positions < kv_lens[b]).
struct Fp8DequantLaunch {
  const uint8_t* kv8;
  int32_t num_blocks;
  const int32_t* tables;
  int64_t pitch;
  const int32_t* rows;
  const int32_t* kv_lens;
  int32_t batch, num_kv_heads, seq_len;
  void* k_out;
  int64_t k_sb, k_sh, k_ss;
  void* v_out;
  int64_t v_sb, v_sh, v_ss;
  int32_t* err;
};
cudaError_t launch_fp8_dequant(const Fp8DequantLaunch& a, cudaStream_t stream);

struct NormLaunch {
  const void* a;
  int64_t a_stride;
  const void* resid;  // nullable: no residual add
  int64_t r_stride;
  void* resid_out;    // nullable: sum not stored
  int64_t ro_stride;
  const void* weight;
  void* out;
  int64_t o_stride;
  int32_t rows, dim;
  float eps;
};
cudaError_t launch_add_rmsnorm(const NormLaunch& p, cudaStream_t stream);

// Skinny tcgen05 linear (linear_tc.cu): y[M, N] = x[M, K] . W[N, K]^T (+ bias), M <= 256.
struct LinearPlan {
  int32_t mpad;    // M rounded up to a multiple of 16 (the MMA's N)
  int32_t tiles;   // N / 128
  int32_t chunks;  // K / 64
  int32_t splits;  // split-k factor = cluster size (grid.y)
  int32_t stages;  // TMA ring depth
  int32_t smem_bytes;
  int32_t recv_off;  // byte offset of the split-k receive buffer
  uint32_t tmem_cols;
};
// Epilogue of the q/k/v GEMM that does pkv_append_rope's work (linear_tc.cu).
struct RopeAppend {
  __nv_bfloat16* q_out;  // nullptr: not this mode
  int64_t qo_sb, qo_sh, qo_st;
  __nv_bfloat16* k_pool;
  __nv_bfloat16* v_pool;
  int32_t num_blocks;
  const __nv_bfloat16* cos;
  const __nv_bfloat16* sin;
  int64_t rope_rows;
  const int32_t* tables;
  int64_t pitch;
  const int32_t* rows;
  const int32_t* starts;
  const int32_t* q_lens;
  int32_t T, hq, hkv;
};
struct LinearLaunch {
  int32_t M, N;
  void* y;  // bf16 [M][ldy]
  int64_t ldy;
  const void* bias;  // nullable
  int32_t w_tiled;   // wmap is the 3-D map of a PKV_W_TILED weight
  int32_t swiglu;    // W is PKV_W_GATE_UP_PAIRED: y = SwiGLU [M][N/2]
  int32_t* err;
  RopeAppend rope;   // rope.q_out set: RoPE + K/V append epilogue, y unused
};
// Needs a current CUDA device (the split count comes from the occupancy API).
LinearPlan plan_linear(int32_t M, int32_t N, int32_t K);
// wmap: 2-D over W [N][K] bf16, box {64, 128} (or 3-D over a PKV_W_TILED W,
// box {64, 128, 1}); xmap: 2-D over x [M][K], box {64, mpad}
cudaError_t launch_linear(const LinearLaunch& a, const LinearPlan& pl, const CUtensorMap& wmap,
                          const CUtensorMap& xmap, cudaStream_t stream);
cudaError_t launch_pack_weight(const void* w, int64_t ldw, int32_t n, int32_t k, void* out,
                               cudaStream_t stream);
cudaError_t launch_pair_gate_up(const void* w, int64_t ldw, int32_t inter, int32_t k, void* out,
                                cudaStream_t stream);
cudaError_t launch_silu_mul(const void* gu, int64_t gu_stride, void* out, int64_t o_stride,
                            int32_t rows, int32_t inter, cudaStream_t stream);

// Temperature sampling, one token per row (sample.cu).
struct SampleLaunch {
  const void* logits;  // [rows][ld], bf16 or f32
  int64_t ld;
  int32_t rows, vocab;
  int32_t f32;     // logits are float32 (else bf16)
  int32_t vec;     // rows start 4-element aligned: 4-wide loads
  int32_t splits;  // CTAs (= cluster size) per row, sample_splits()
  float inv_temp;
  uint64_t seed, call;
  int32_t* out;  // [rows]; -1 where a row has no finite score
};
int sample_splits(int32_t rows, int32_t vocab);
cudaError_t launch_sample(const SampleLaunch& a, cudaStream_t stream);

// All decoder layers of a small decode step in one persistent launch
// (layers.cu).  Shapes are Qwen2.5-1.5B's: hidden 1536, 12 q / 2 KV heads of
// 128, intermediate 8960.
constexpr int kLayersMax = 32;
struct LayersMaps {
  // per layer: q/k/v [2048][1536], o [1536][1536], gate/up paired
  // [17920][1536], down [1536][8960]; 2-D maps, box {64, 128}, 128B swizzle
  CUtensorMap w[kLayersMax][4];
  // the whole pool [2L][slots][Hkv][128] bf16: 4-D map, box {64, 1, 16, 1}
  CUtensorMap pool;
};
struct LayersParams {
  int32_t L, M, G;      // layers, rows, grid (one CTA per SM)
  int32_t P;            // attention partitions per (row, KV head)
  int32_t min_blocks;   // a row's attention partitions hold at least this many blocks
  int32_t xslots, nw;   // activation slots, W ring stages
  const __nv_bfloat16* qkv_b[kLayersMax];
  const __nv_bfloat16* post_w[kLayersMax];  // post_attention_layernorm
  const __nv_bfloat16* in_w[kLayersMax];    // input_layernorm (layers >= 1)
  const __nv_bfloat16* h0;  // [M][1536] layer 0's normalised input
  __nv_bfloat16* xs;        // [M][1536] residual stream, updated in place
  __nv_bfloat16* m_out;     // [M][1536] the last layer's MLP output
  __nv_bfloat16* pool;      // [2L][slots][Hkv][128]
  int64_t num_slots;
  int32_t num_blocks;
  const int32_t* tables;
  int64_t pitch;
  const int32_t* rows;    // table row of each batch row (nullable: identity)
  const int32_t* starts;  // length before this step; < 0 = inactive row
  const __nv_bfloat16* cos;
  const __nv_bfloat16* sin;
  int64_t rope_rows;
  float eps, scale_log2;
  // workspace pieces (carve_decode_layers)
  uint32_t* sync;     // [0] grid barrier arrivals, [2] abort word
  int32_t* tile_cnt;  // per W tile completion counters
  int32_t* att_cnt;   // per (row, KV head) attention partition counters
  float* part;        // [G][2][32][128] fp32 tile-segment partials
  float* att_o;       // [M * Hkv * P][8][128]
  float* att_lse;     // [M * Hkv * P][8]
  float* ss;          // [12][32] per-tile sums of squares of the residual
  __nv_bfloat16* q_rot;    // [M][12][128]
  __nv_bfloat16* att_out;  // [M][1536]
  __nv_bfloat16* act;      // [M][8960]
  int32_t* err;
};
struct LayersPlan {
  int32_t mpad, grid, partitions, min_blocks, xslots, nw, smem_bytes;
  bool valid;
};
LayersPlan plan_decode_layers(int32_t rows, int32_t sms);
size_t decode_layers_workspace_bytes(int32_t rows, int32_t sms);
size_t decode_layers_sync_bytes();
void carve_decode_layers(LayersParams& p, void* ws, int32_t rows, int32_t sms, int32_t partitions);
cudaError_t launch_decode_layers(const LayersParams& p, const LayersMaps& maps,
                                 const LayersPlan& pl, cudaStream_t stream);

}  // namespace pkv
