/*
 * pagedkv.h -- C ABI of the B200 (sm_100a) paged-KV attention path.
 *
 * The library libpagedkv.so replaces the GPU half of two Python modules of the
 * reference engine (shubhav1/my-inference-engine):
 *
 *   kv_cache.py   KVCache.write()   (kv_cache.py:108-115, index_copy_ scatter)
 *                 KVCache.read()    (kv_cache.py:117-121, dense gather copy)
 *                 apply_rope()      (model.py:58-65, five bf16 elementwise ops)
 *   kernels/fa2.py fa2_forward + FlashAttention2Function.forward
 *                                   (kernels/fa2.py:23-214)
 *
 * Conventions shared by every entry point
 * ---------------------------------------
 *  - All tensor arguments are raw device pointers; strides are in ELEMENTS.
 *    The innermost (head_dim) dimension is always contiguous.
 *  - Element type is bf16 for activations and the pool, int32 for tables and
 *    lengths, fp32 for scratch.  head_dim must be 128 and block_size 16
 *    (the Qwen2.5-1.5B path).
 *  - The KV pool keeps the reference's layout (kv_cache.py:20-22):
 *      buf[layer][k=0|v=1][slot][kv_head][head_dim],  slot = block*16 + pos%16
 *    Entry points take the base of one layer's K plane (buf[layer,0]) and V
 *    plane (buf[layer,1]) plus num_slots = num_blocks*16.
 *  - Block tables are device-resident int32 [rows][table_pitch]; batch row b
 *    uses table row seq_rows[b] (seq_rows may be NULL: row b).  Logical
 *    position p of row b lives at slot table[row][p/16]*16 + p%16.
 *  - Every call is asynchronous on `stream` and returns a pkv_status.  A
 *    nonzero status means nothing was launched.  Memory is owned by the
 *    caller; the library never allocates or frees device memory.
 *  - Kernels are launched with programmatic dependent launch: a kernel may
 *    start while the previous kernel on the stream drains and waits for it
 *    before touching activations, tables or lengths.  The weights of the
 *    pkv_linear* entries are constant operands and are read before that
 *    wait, so they must not be written by the kernel right before the call
 *    on the same stream.
 *    PKV_PDL=0 in the environment launches without it.
 *  - err_flag (nullable, device int32) receives PKV_DEVERR_* bits when a
 *    kernel meets an out-of-range block id / position: the bad access is
 *    skipped (block 0 is read instead) and the flag is OR-ed, never a fault.
 */
#ifndef PAGEDKV_H_
#define PAGEDKV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  PKV_OK = 0,
  PKV_ERR_INVALID = 1,      /* bad shape, null pointer, bad count        */
  PKV_ERR_UNSUPPORTED = 2,  /* head_dim != 128, group too large, ...     */
  PKV_ERR_ALIGN = 3,        /* pointer / stride not 16-byte aligned      */
  PKV_ERR_DRIVER = 4,       /* driver entry point / tensor map encoding  */
  PKV_ERR_LAUNCH = 5,       /* kernel launch failed                      */
  PKV_ERR_WORKSPACE = 6     /* workspace too small                       */
} pkv_status;

/* Bits a kernel ORs into *err_flag. */
#define PKV_DEVERR_BLOCK_ID 1  /* table entry outside [0, num_blocks)      */
#define PKV_DEVERR_POSITION 2  /* position beyond table pitch / rope rows  */
#define PKV_DEVERR_TIMEOUT 4   /* a bounded wait on an mbarrier ran out    */

/* Library version (major*10000 + minor*100 + patch). */
int pkv_version(void);

/* Static text for a status code. */
const char* pkv_status_string(int status);

/* Detail of the most recent failing call on this host thread ("" if none). */
const char* pkv_last_error(void);

/*
 * Fused RoPE + K/V append for one layer and one forward step.
 *
 * Replaces apply_rope (model.py:62-65, with cos/sin from rope_cos_sin
 * model.py:151-155) followed by KVCache.write (kv_cache.py:108-115).
 * For batch row b and step token t the position is pos = starts[b] + t:
 *   - if rope_cos/rope_sin are non-NULL, q and k are rotated with row `pos`
 *     of the bf16 tables [rope_rows][128], rounding to bf16 after every op
 *     exactly like the reference: bf16(bf16(x*cos) + bf16(rotate_half(x)*sin));
 *   - roped q goes to q_out [B][Hq][T][128] (strides q_out_s*), may be NULL;
 *   - roped k and plain v go to the pool slot of (row b, pos).
 * With rope_cos == NULL the call is exactly KVCache.write (k/v copied as-is,
 * q ignored).  q, k, v are [B][H][T][128] with strides (sb, sh, st).
 * A row with starts[b] < 0 is an inactive padding row (e.g. a batch padded
 * to a captured size): nothing is read, rotated or stored for it.
 * q_lens (nullable, device int32 [B]): row b has only q_lens[b] <= T real
 * tokens (right padding); tokens t >= q_lens[b] are skipped.
 */
int pkv_append_rope(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st,
                    const void* k, int64_t k_sb, int64_t k_sh, int64_t k_st,
                    const void* v, int64_t v_sb, int64_t v_sh, int64_t v_st,
                    const void* rope_cos, const void* rope_sin, int64_t rope_rows,
                    void* q_out, int64_t qo_sb, int64_t qo_sh, int64_t qo_st,
                    void* k_pool, void* v_pool, int64_t num_slots,
                    const int32_t* block_tables, int64_t table_pitch,
                    const int32_t* seq_rows, const int32_t* starts, const int32_t* q_lens,
                    int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                    int32_t seq_len_q, int32_t head_dim,
                    int32_t* err_flag, void* stream);

/*
 * Bytes of fp32 scratch pkv_paged_decode (and pkv_paged_decode_fp8) needs
 * for these sizes (split-K partials + per-(row, kv_head) counters).  0 when
 * one pass suffices.
 */
size_t pkv_decode_workspace_size(int32_t batch, int32_t num_q_heads,
                                 int32_t num_kv_heads, int32_t max_kv_len);

/*
 * The split-K plan pkv_paged_decode takes for these sizes, written to
 * plan[0..3] = {blocks_per_part, min_blocks_per_part, max_parts (grid.x),
 * sub_groups}.  Host-only arithmetic (no GPU, no launch); lets a caller or a
 * test see which partition sizing a launch of this shape uses (the FP8
 * kernel, with twice the CTAs resident per SM, plans for twice the CTAs and
 * so may split rows more finely).  Diagnostic,
 * no counterpart in the reference (its kernel has no split-K,
 * kernels/fa2.py:192-207).  Returns PKV_ERR_INVALID for invalid sizes.
 */
int pkv_decode_plan(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                    int32_t max_kv_len, int32_t* plan);

/*
 * Paged decode attention (one query token per row) reading K/V blocks in
 * place through the block table: no dense gather copy.
 *
 * Replaces KVCache.read (kv_cache.py:117-121) + fa2_forward with T=1
 * (kernels/fa2.py:23-162 as launched at :192-207; model.py:103).
 * q  : [B][Hq][128] (strides q_sb, q_sh)      out: [B][Hq][128] (o_sb, o_sh)
 * kv_lens[b] keys are visible to row b (is_causal is irrelevant at T=1,
 * fa2.py:110-111).  max_kv_len >= max(kv_lens) sizes the grid; the host
 * keeps it without a device read.  sm_scale is 1/sqrt(128) in the reference
 * (fa2.py:173).  Rows with kv_len == 0 produce NaN, as 0/0 does in
 * fa2.py:151.  workspace: >= pkv_decode_workspace_size() bytes, zeroed
 * before first use; the kernel leaves its counters at zero on exit.
 */
int pkv_paged_decode(const void* q, int64_t q_sb, int64_t q_sh,
                     const void* k_pool, const void* v_pool, int64_t num_slots,
                     const int32_t* block_tables, int64_t table_pitch,
                     const int32_t* seq_rows, const int32_t* kv_lens,
                     int32_t max_kv_len, int32_t batch, int32_t num_q_heads,
                     int32_t num_kv_heads, int32_t head_dim, float sm_scale,
                     void* out, int64_t o_sb, int64_t o_sh,
                     void* workspace, size_t workspace_bytes,
                     int32_t* err_flag, void* stream);

/*
 * Paged (ragged) prefill / chunked-prefill attention, T >= 1 queries per row.
 *
 * Replaces KVCache.read + fa2_forward with is_causal = T > 1
 * (kernels/fa2.py:23-162; model.py:185).  Query i of row b sits at key
 * position i + kv_lens[b] - T (bottom-right causal, fa2.py:110-111); with
 * causal == 0 every query sees all kv_lens[b] keys.
 * q/out: [B][Hq][T][128] with strides (sb, sh, st).
 * q_lens (nullable, device int32 [B]): row b has q_lens[b] <= T real queries
 * at positions 0..q_lens[b]-1 (right padding); query i then sits at key
 * i + kv_lens[b] - q_lens[b], and output rows i >= q_lens[b] are not written.
 */
int pkv_paged_prefill(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st,
                      const void* k_pool, const void* v_pool, int64_t num_slots,
                      const int32_t* block_tables, int64_t table_pitch,
                      const int32_t* seq_rows, const int32_t* kv_lens, const int32_t* q_lens,
                      int32_t max_kv_len, int32_t batch, int32_t seq_len_q,
                      int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                      int32_t causal, float sm_scale,
                      void* out, int64_t o_sb, int64_t o_sh, int64_t o_st,
                      int32_t* err_flag, void* stream);

/*
 * Attention over dense, padded K/V -- the exact argument contract of
 * FlashAttention2Function.forward (kernels/fa2.py:166-214): K/V are
 * [B][Hkv][S][128] with strides (sb, sh, ss); each stride must be a
 * multiple of 8 elements (16 bytes) and the bases 16-byte aligned.
 * Rows are masked to kv_lens[b] (<= S) and bottom-right causal when
 * causal != 0.  T == 1 uses the decode kernel (and the workspace, sized by
 * pkv_decode_workspace_size with max_kv_len = S), T > 1 the prefill kernel.
 */
int pkv_dense_attention(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st,
                        const void* k, int64_t k_sb, int64_t k_sh, int64_t k_ss,
                        const void* v, int64_t v_sb, int64_t v_sh, int64_t v_ss,
                        const int32_t* kv_lens, int32_t batch, int32_t seq_len_q,
                        int32_t seq_len_k, int32_t num_q_heads, int32_t num_kv_heads,
                        int32_t head_dim, int32_t causal, float sm_scale,
                        void* out, int64_t o_sb, int64_t o_sh, int64_t o_st,
                        void* workspace, size_t workspace_bytes,
                        int32_t* err_flag, void* stream);

/*
 * FP8 (e4m3) KV pool -- opt-in storage format, no counterpart in the
 * reference (whose pool is the activation dtype, kv_cache.py:20-22).  Half
 * the bytes per token (528 B per token and layer instead of 1024), so decode
 * reads half as much; values are rounded to 3 mantissa bits.
 *
 * Layout of one layer: [num_blocks][num_kv_heads][pkv_fp8_block_bytes()]
 * bytes, one chunk per (16-token block, KV head):
 *   [0, 2048)     K: 16 token rows of 128 bytes.  16-byte group c of token t
 *                 is stored at group c ^ (t & 7); inside a group, byte 4i+u
 *                 holds dim 2i+u (u = 0, 1) or dim 2i+8+u-2 (u = 2, 3).
 *   [2048, 4096)  V transposed: 128 dim rows of 16 bytes; byte 4i+u holds
 *                 token 2i+u (u = 0, 1) or token 2i+8+u-2 (u = 2, 3).
 *   [4096, 4160)  fp32 K scale per token, [4160, 4224) fp32 V scale per token.
 * A row x (128 values of one token and head, k after RoPE) is stored as
 * e4m3 = RNE(x * (448 / amax)) with saturation, scale = amax / 448, where
 * amax = max |x| (each quotient one IEEE fp32 division; an all-zero row
 * stores zeros and scale 1); it reads back as e4m3 * scale.
 */
size_t pkv_fp8_block_bytes(void);

/*
 * pkv_append_rope for the FP8 pool: q is rotated into q_out exactly as
 * pkv_append_rope does; k (rotated, the same bf16 bits) and v are quantised
 * into their token's slot of the FP8 pool (kv8_pool = one layer's chunks,
 * num_blocks blocks).  Block tables, starts, q_lens and padding rows as
 * pkv_append_rope.  Replaces apply_rope + KVCache.write (model.py:62-65,
 * kv_cache.py:108-115) for a cache created in FP8 mode.
 */
int pkv_append_rope_fp8(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st,
                        const void* k, int64_t k_sb, int64_t k_sh, int64_t k_st,
                        const void* v, int64_t v_sb, int64_t v_sh, int64_t v_st,
                        const void* rope_cos, const void* rope_sin, int64_t rope_rows,
                        void* q_out, int64_t qo_sb, int64_t qo_sh, int64_t qo_st,
                        void* kv8_pool, int64_t num_blocks,
                        const int32_t* block_tables, int64_t table_pitch,
                        const int32_t* seq_rows, const int32_t* starts, const int32_t* q_lens,
                        int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                        int32_t seq_len_q, int32_t head_dim,
                        int32_t* err_flag, void* stream);

/*
 * pkv_paged_decode over the FP8 pool (same arguments and workspace sizing,
 * kv8_pool/num_blocks in place of the two bf16 planes).  Each block is one
 * bulk copy per KV head; K and V are widened to f16 in registers (exactly),
 * the products are f16 tensor-core MMAs accumulating in fp32, and the
 * per-token scales are applied to the scores and the probabilities.  A
 * probability (at most 2^8 before the row sum divides it out) times its
 * token's V scale (amax / 448) is an f16 operand, so V rows must stay below
 * about 1.1e5 in magnitude.
 * Replaces KVCache.read + fa2_forward at T = 1 (kv_cache.py:117-121,
 * kernels/fa2.py:23-162) for a cache in FP8 mode.
 */
int pkv_paged_decode_fp8(const void* q, int64_t q_sb, int64_t q_sh,
                         const void* kv8_pool, int64_t num_blocks,
                         const int32_t* block_tables, int64_t table_pitch,
                         const int32_t* seq_rows, const int32_t* kv_lens,
                         int32_t max_kv_len, int32_t batch, int32_t num_q_heads,
                         int32_t num_kv_heads, int32_t head_dim, float sm_scale,
                         void* out, int64_t o_sb, int64_t o_sh,
                         void* workspace, size_t workspace_bytes,
                         int32_t* err_flag, void* stream);

/*
 * FP8 pool -> dense bf16 K and V [B][Hkv][seq_len][128] (strides in
 * elements, rows 8-byte aligned): position p < kv_lens[b] of row b becomes
 * bf16(e4m3 * scale); later positions are left untouched.  A prefill step
 * of a cache in FP8 mode attends over these rows with pkv_dense_attention
 * (the compute-bound prefill reads each key once per query tile, so the
 * extra copy is small next to it).  Replaces KVCache.read
 * (kv_cache.py:117-121) for that step.
 */
int pkv_fp8_dequant(const void* kv8_pool, int64_t num_blocks,
                    const int32_t* block_tables, int64_t table_pitch,
                    const int32_t* seq_rows, const int32_t* kv_lens, int32_t batch,
                    int32_t num_kv_heads, int32_t seq_len,
                    void* k_out, int64_t k_sb, int64_t k_sh, int64_t k_ss,
                    void* v_out, int64_t v_sb, int64_t v_sh, int64_t v_ss,
                    int32_t* err_flag, void* stream);

/*
 * Residual add + RMSNorm of the Qwen2 block, one launch.
 *
 * Replaces `x = x + sublayer_out` (model.py:136-137) followed by RMSNorm
 * (model.py:49-55) with the reference's rounding: h = bf16(resid + a);
 * out = bf16(weight * bf16(h * rsqrt(mean(h*h) + eps))), the mean and rsqrt
 * in fp32.  resid == NULL normalises `a` alone; resid_out (nullable, may
 * equal resid) receives h.  Rows of `dim` bf16 (dim % 8 == 0, <= 4096)
 * with element row strides; 16-byte aligned rows.
 */
int pkv_add_rmsnorm(const void* a, int64_t a_stride, const void* resid, int64_t r_stride,
                    void* resid_out, int64_t ro_stride, const void* weight, void* out,
                    int64_t o_stride, int32_t rows, int32_t dim, float eps, void* stream);

/*
 * SwiGLU activation: out = bf16(bf16(silu(gate)) * up) where each row of `gu`
 * is [gate (inter) | up (inter)] -- the output of one merged gate/up GEMM.
 * Replaces F.silu(gate_proj(x)) * up_proj(x) (model.py:120) around the GEMMs.
 * inter % 8 == 0; 16-byte aligned rows.
 */
int pkv_silu_mul(const void* gu, int64_t gu_stride, void* out, int64_t o_stride, int32_t rows,
                 int32_t inter, void* stream);

/*
 * Temperature sampling: one token id per row from softmax(logits / temperature).
 * Replaces chat.py:103-107 (`torch.multinomial(F.softmax(logits.float() / T,
 * dim=-1), num_samples=1)`) with one kernel pass over the logits and no
 * probability tensor (Gumbel-max: argmax of logits / T plus i.i.d. Gumbel
 * noise, an exact draw from that categorical).  The noise comes from
 * Philox-4x32-10 keyed by `seed`, counter (element / 4, row, call): the same
 * (seed, call) always gives the same ids.  logits: [rows][ld], bf16
 * (dtype 0) or float32 (dtype 1), ld >= vocab.  temperature > 0.  out: int32
 * device [rows]; a row with no finite logit gets -1 (the reference raises
 * RuntimeError for such a row; the Python shim does too).
 */
int pkv_sample(const void* logits, int64_t ld, int32_t rows, int32_t vocab, int32_t dtype,
               float temperature, uint64_t seed, uint64_t call, int32_t* out, void* stream);

/*
 * Size of the library-owned scratch used by pkv_paged_decode_static_scratch:
 * one array of this many bytes per GPU that loads the library, held until
 * the process exits.
 */
#define PKV_DECODE_STATIC_SCRATCH_BYTES (8u << 20)

/*
 * pkv_paged_decode without a caller-provided workspace.  No counterpart in
 * the reference: it exists for callers that cannot call cudaMalloc -- code
 * running where the CUDA allocator is not theirs to use (a host that owns
 * all device memory through its own pool, a plugin whose host forbids
 * allocation during a serving step, or code that must not touch the
 * allocator at all).  Inputs, outputs, pool and tables are still passed in;
 * only the split-K scratch comes from a static device array of
 * PKV_DECODE_STATIC_SCRATCH_BYTES inside the library.
 *
 *  - Calls no cudaMalloc/cudaFree or any allocating routine.
 *  - The first call on a device looks up that array's device address (with
 *    the device current), so make the first call on each device before any
 *    stream capture begins.
 *  - Shapes whose split-K scratch (pkv_decode_workspace_size) exceeds
 *    PKV_DECODE_STATIC_SCRATCH_BYTES are rejected with PKV_ERR_WORKSPACE and
 *    nothing is launched.
 *  - Every call on a device shares the one array, which keeps the previous
 *    call's contents; the call clears the counters it needs itself.  Calls
 *    whose kernels overlap on the GPU (different streams without ordering)
 *    race on the array and produce wrong results: order them on one stream.
 */
int pkv_paged_decode_static_scratch(const void* q, int64_t q_sb, int64_t q_sh,
                                    const void* k_pool, const void* v_pool, int64_t num_slots,
                                    const int32_t* block_tables, int64_t table_pitch,
                                    const int32_t* seq_rows, const int32_t* kv_lens,
                                    int32_t max_kv_len, int32_t batch, int32_t num_q_heads,
                                    int32_t num_kv_heads, int32_t head_dim, float sm_scale,
                                    void* out, int64_t o_sb, int64_t o_sh,
                                    int32_t* err_flag, void* stream);

/*
 * Skinny linear layers for decode-sized batches (tcgen05 tensor cores).
 *
 * y[m, n] = x[m, :] . w[n, :] (+ bias[n]) for m < rows <= PKV_LINEAR_MAX_ROWS,
 * the nn.Linear projections of the Qwen2 block (model.py:83-86, :114-116)
 * when a decode step (or a short prefill) feeds them a few rows: the weight
 * matrix is read from HBM once, split over the SMs along n and k.  x, w and
 * y are bf16, rows with element strides (multiples of 8), 16-byte aligned;
 * n % 128 == 0, k % 64 == 0.  Accumulation is fp32; the k-split partial sums
 * are added on chip (thread-block cluster) in a fixed order and rounded to
 * bf16 once, so results are deterministic.
 *
 * pkv_linear needs no workspace (the arguments may be NULL / 0).  The fused
 * variants keep the bf16 GEMM output [rows][n] in the workspace
 * (pkv_linear_workspace_size bytes = rows * n * 2, 16-byte aligned) and then
 * apply exactly the arithmetic of the separate entry they replace:
 *   pkv_linear_add_rmsnorm  GEMM, then pkv_add_rmsnorm (o_proj / down_proj
 *                           followed by the next residual add + RMSNorm)
 *   pkv_linear_silu_mul     merged gate/up GEMM (w rows [0, inter) gate,
 *                           [inter, 2 inter) up), then pkv_silu_mul
 *   pkv_linear_rope_append  merged q/k/v GEMM + bias, then pkv_append_rope
 *                           (rows = batch * seq_len_q, row b*seq_len_q + t);
 *                           done in the GEMM's epilogue (no workspace) when
 *                           q_out is 16-byte aligned with strides that are
 *                           multiples of 8, else as GEMM + append kernel
 * where n is the GEMM's width: dim, 2 * inter, (hq + 2 hkv) * head_dim.
 */
#define PKV_LINEAR_MAX_ROWS 256

/* Weight layouts (w_layout) of the pkv_linear* entries. */
#define PKV_W_ROWMAJOR 0 /* w[n][k], element row stride ldw                        */
#define PKV_W_TILED 1    /* [n/128][k/64][128][64] contiguous (ldw unused): every
                            128x64 tile one 16 KiB run, so the GEMM streams each
                            CTA's share of w as one contiguous range of HBM;
                            made by pkv_linear_pack_weight                         */
#define PKV_W_GATE_UP_PAIRED 2 /* pkv_linear_silu_mul only: merged gate/up rows
                            reordered so rows [128t, 128t+128) are gate rows
                            [64t, 64t+64) then up rows [64t, 64t+64) (row stride
                            ldw); the GEMM then finishes SwiGLU in its epilogue
                            (no workspace, no second kernel); made by
                            pkv_linear_pair_gate_up                               */

size_t pkv_linear_workspace_size(int32_t rows, int32_t n, int32_t k);

/* Reorder a merged gate/up weight ([2*inter][k], gate rows then up rows, row
 * stride ldw) into the PKV_W_GATE_UP_PAIRED layout (2*inter rows of k,
 * contiguous, at w_paired; inter % 64 == 0). */
int pkv_linear_pair_gate_up(const void* w_gate_up, int64_t ldw, int32_t inter, int32_t k,
                            void* w_paired, void* stream);

/* Copy a row-major w[n][k] (row stride ldw) into the PKV_W_TILED layout
 * (n * k bf16 elements at w_tiled, 16-byte aligned). */
int pkv_linear_pack_weight(const void* w, int64_t ldw, int32_t n, int32_t k, void* w_tiled,
                           void* stream);

int pkv_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, int32_t w_layout,
               const void* bias, int32_t rows, int32_t n, int32_t k, void* y, int64_t ldy,
               void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream);

int pkv_linear_add_rmsnorm(const void* x, int64_t ldx, const void* w, int64_t ldw,
                           int32_t w_layout, int32_t rows, int32_t n, int32_t k,
                           const void* resid, int64_t r_stride, void* resid_out,
                           int64_t ro_stride, const void* norm_weight, float eps, void* out,
                           int64_t o_stride, void* workspace, size_t workspace_bytes,
                           int32_t* err_flag, void* stream);

int pkv_linear_silu_mul(const void* x, int64_t ldx, const void* w_gate_up, int64_t ldw,
                        int32_t w_layout, int32_t rows, int32_t inter, int32_t k, void* out,
                        int64_t o_stride, void* workspace, size_t workspace_bytes,
                        int32_t* err_flag, void* stream);

int pkv_linear_rope_append(const void* x, int64_t ldx, const void* w_qkv, int64_t ldw,
                           int32_t w_layout, const void* bias, int32_t k, const void* rope_cos,
                           const void* rope_sin, int64_t rope_rows, void* q_out, int64_t qo_sb,
                           int64_t qo_sh, int64_t qo_st, void* k_pool, void* v_pool,
                           int64_t num_slots, const int32_t* block_tables, int64_t table_pitch,
                           const int32_t* seq_rows, const int32_t* starts, const int32_t* q_lens,
                           int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                           int32_t seq_len_q, int32_t head_dim, void* workspace,
                           size_t workspace_bytes, int32_t* err_flag, void* stream);

/*
 * All decoder layers of one small decode step in ONE persistent launch.
 *
 * Replaces, for a step of 1 <= rows <= PKV_LAYERS_MAX_ROWS rows that each add
 * one token (T = 1), the per-layer loop of model.py:157-207 over
 * QwenBlock.forward (model.py:131-138): q/k/v projections + bias, RoPE, the
 * K/V write into the paged cache (kv_cache.py:86-101), attention over each
 * row's blocks (kernels/fa2.py:164-214 at T = 1), o_proj, residual add +
 * RMSNorm, gate/up + SwiGLU, down_proj, residual add and the next layer's
 * RMSNorm -- the same ops, bf16 rounding points and arithmetic as
 * pkv_linear_rope_append, pkv_paged_decode, pkv_linear_add_rmsnorm and
 * pkv_linear_silu_mul applied layer by layer, up to fp32 summation order in
 * the k-split sums and the RMSNorm sums of squares.  One CTA per SM streams
 * every layer's weights through a TMA ring that keeps filling across the
 * layer's phases; the phases meet at grid-wide barriers (every wait bounded:
 * a timeout sets PKV_DEVERR_TIMEOUT in err_flag and the launch returns).
 *
 * Shapes are Qwen2.5-1.5B's: hidden 1536, 12 query and 2 KV heads of 128,
 * intermediate 8960, num_layers <= PKV_LAYERS_MAX_LAYERS.  Per layer (bf16,
 * row-major, 16-byte aligned, rows contiguous):
 *   qkv_w [2048][1536] (q rows, then k, then v), qkv_b [2048],
 *   o_w [1536][1536], post_norm_w [1536] (post_attention_layernorm),
 *   gate_up_w [17920][1536] in the PKV_W_GATE_UP_PAIRED layout,
 *   down_w [1536][8960], in_norm_w [1536] (input_layernorm; layer 0's is
 *   not read: h0 is already normalised).
 * h0 [rows][1536]: layer 0's normalised input; xs [rows][1536]: the residual
 * stream, updated in place; m_out [rows][1536] receives the last layer's MLP
 * output before its residual add (the caller finishes with the final add +
 * RMSNorm and the LM head).  kv_pool: the whole cache [num_layers][2]
 * [num_slots][2][128] bf16 (K then V plane per layer).  Row b writes its new
 * K/V at position starts[b] (< 0: inactive row, nothing written, its
 * outputs undefined) through block_tables[seq_rows[b]] and attends to
 * positions [0, starts[b]].  rope_cos/rope_sin: bf16 [rope_rows][128].
 * workspace: pkv_decode_layers_workspace_size(rows) bytes, 256-byte aligned,
 * owned by one stream at a time; its first 4 KiB are reset by the call.
 */
#define PKV_LAYERS_MAX_ROWS 32
#define PKV_LAYERS_MAX_LAYERS 32

typedef struct pkv_layer_weights {
  const void* qkv_w;
  const void* qkv_b;
  const void* o_w;
  const void* post_norm_w;
  const void* gate_up_w;
  const void* down_w;
  const void* in_norm_w;
} pkv_layer_weights;

size_t pkv_decode_layers_workspace_size(int32_t rows);

int pkv_decode_layers(const pkv_layer_weights* layers, int32_t num_layers, const void* h0,
                      void* xs, void* m_out, int32_t rows, void* kv_pool, int64_t num_slots,
                      const int32_t* block_tables, int64_t table_pitch, const int32_t* seq_rows,
                      const int32_t* starts, const void* rope_cos, const void* rope_sin,
                      int64_t rope_rows, float eps, void* workspace, size_t workspace_bytes,
                      int32_t* err_flag, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PAGEDKV_H_ */
