// extern "C" entry points of libpagedkv.so (declared in include/pagedkv.h):
// argument validation, TMA tensor-map encoding, dispatch to the kernels.
// Nothing here allocates device memory.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>

#include <mutex>
#include <string>

#include "../../include/pagedkv.h"
#include "pkv_kernels.h"

namespace {

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}
int ok() {
  g_last_error.clear();
  return PKV_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda directly (it loads on machines without one).
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Pool plane [num_slots][Hkv][128] bf16 -> 3-D map, box {64, 1, 16}, 128B swizzle.
int encode_pool(CUtensorMap* m, const void* base, int64_t num_slots, int32_t hkv) {
  EncodeFn fn = encode_fn();
  if (!fn) return fail(PKV_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(hkv), static_cast<cuuint64_t>(num_slots)};
  cuuint64_t strides[2] = {128 * 2, static_cast<cuuint64_t>(hkv) * 128 * 2};
  cuuint32_t box[3] = {64, 1, 16};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PKV_ERR_DRIVER, "pool tensor map encode failed (%d)", (int)r);
  return PKV_OK;
}

// Dense [B][Hkv][S][128] bf16 with element strides -> 4-D map, box {64,16,1,1}.
int encode_dense(CUtensorMap* m, const void* base, int32_t B, int32_t hkv, int32_t S, int64_t sb,
                 int64_t sh, int64_t ss) {
  EncodeFn fn = encode_fn();
  if (!fn) return fail(PKV_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(hkv),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(ss) * 2, static_cast<cuuint64_t>(sh) * 2,
                           static_cast<cuuint64_t>(sb) * 2};
  cuuint32_t box[4] = {64, 16, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PKV_ERR_DRIVER, "dense tensor map encode failed (%d)", (int)r);
  return PKV_OK;
}

// Q [B][Hq][T][128] bf16 -> 4-D map, box {64, 128, 1, 1} (128 query rows).
int encode_q(CUtensorMap* m, const void* base, int32_t B, int32_t hq, int32_t T, int64_t sb,
             int64_t sh, int64_t st) {
  EncodeFn fn = encode_fn();
  if (!fn) return fail(PKV_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(hq),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(st) * 2, static_cast<cuuint64_t>(sh) * 2,
                           static_cast<cuuint64_t>(sb) * 2};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PKV_ERR_DRIVER, "q tensor map encode failed (%d)", (int)r);
  return PKV_OK;
}

int check_heads(int32_t hq, int32_t hkv, int32_t d) {
  if (d != 128) return fail(PKV_ERR_UNSUPPORTED, "head_dim must be 128, got %d", d);
  if (hq <= 0 || hkv <= 0 || hq % hkv != 0)
    return fail(PKV_ERR_INVALID, "num_q_heads (%d) must be a positive multiple of num_kv_heads (%d)",
                hq, hkv);
  return PKV_OK;
}

bool mult8(int64_t s) { return (s % 8) == 0; }

int check_pool(const void* kp, const void* vp, int64_t num_slots, const int32_t* tables,
               int64_t pitch) {
  if (!kp || !vp || !tables) return fail(PKV_ERR_INVALID, "null pool or block-table pointer");
  if (num_slots <= 0 || num_slots % 16 != 0)
    return fail(PKV_ERR_INVALID, "num_slots (%lld) must be a positive multiple of 16",
                (long long)num_slots);
  if (num_slots / 16 > INT32_MAX || num_slots > (int64_t(1) << 31))
    return fail(PKV_ERR_UNSUPPORTED, "pool too large for 32-bit slot coordinates");
  if (pitch <= 0) return fail(PKV_ERR_INVALID, "table_pitch must be positive");
  if (!aligned16(kp) || !aligned16(vp)) return fail(PKV_ERR_ALIGN, "pool planes not 16-byte aligned");
  return PKV_OK;
}

int launch_status(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(PKV_ERR_LAUNCH, "%s launch failed: %s", what, cudaGetErrorString(e));
  return ok();
}

// Rows of a [rows][k] bf16 matrix (element row stride ld) -> 2-D map,
// box {64, box_rows}, 128B swizzle; rows past `rows` read as zeros.
int encode_rows(CUtensorMap* m, const void* base, int64_t rows, int64_t k, int64_t ld,
                int32_t box_rows) {
  EncodeFn fn = encode_fn();
  if (!fn) return fail(PKV_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PKV_ERR_DRIVER, "matrix tensor map encode failed (%d)", (int)r);
  return PKV_OK;
}

// PKV_W_TILED weight [n/128][k/64][128][64] -> 3-D map over {64, 128, tiles*chunks},
// box {64, 128, 1}: one contiguous 16 KiB run per box.
int encode_tiled(CUtensorMap* m, const void* base, int32_t n, int32_t k) {
  EncodeFn fn = encode_fn();
  if (!fn) return fail(PKV_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[3] = {64, 128, static_cast<cuuint64_t>(n / 128) * (k / 64)};
  cuuint64_t strides[2] = {128, 128 * 128};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PKV_ERR_DRIVER, "tiled weight map encode failed (%d)", (int)r);
  return PKV_OK;
}

int check_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, int32_t w_layout,
                 int32_t rows, int32_t n, int32_t k) {
  if (!x || !w) return fail(PKV_ERR_INVALID, "null x or w");
  if (w_layout != PKV_W_ROWMAJOR && w_layout != PKV_W_TILED && w_layout != PKV_W_GATE_UP_PAIRED)
    return fail(PKV_ERR_INVALID, "unknown weight layout %d", w_layout);
  if (w_layout == PKV_W_TILED) ldw = k;
  if (rows < 0 || rows > PKV_LINEAR_MAX_ROWS)
    return fail(PKV_ERR_UNSUPPORTED, "rows must be in [0, %d] (got %d)", PKV_LINEAR_MAX_ROWS, rows);
  if (n <= 0 || n % 128 != 0 || k <= 0 || k % 64 != 0)
    return fail(PKV_ERR_UNSUPPORTED, "n must be a positive multiple of 128 and k of 64 (got %d, %d)",
                n, k);
  if (ldx < k || ldw < k) return fail(PKV_ERR_INVALID, "row strides smaller than k");
  if (!aligned16(x) || !aligned16(w) || !mult8(ldx) || !mult8(ldw))
    return fail(PKV_ERR_ALIGN, "x / w must be 16-byte aligned with strides that are multiples of 8");
  return PKV_OK;
}

// The GEMM half of every pkv_linear* entry: bf16 y (+ bias).
int run_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, int32_t w_layout,
               int32_t rows, int32_t n, int32_t k, void* y, int64_t ldy, const void* bias,
               int32_t* err, cudaStream_t stream, bool swiglu = false,
               const pkv::RopeAppend* rope = nullptr) {
  const pkv::LinearPlan pl = pkv::plan_linear(rows, n, k);
  CUtensorMap wmap, xmap;
  int st = w_layout == PKV_W_TILED ? encode_tiled(&wmap, w, n, k)
                                   : encode_rows(&wmap, w, n, k, ldw, 128);
  if (st) return st;
  if ((st = encode_rows(&xmap, x, rows, k, ldx, pl.mpad))) return st;
  pkv::LinearLaunch a{};
  a.M = rows;
  a.N = n;
  a.y = y;
  a.ldy = ldy;
  a.bias = bias;
  a.w_tiled = w_layout == PKV_W_TILED ? 1 : 0;
  a.swiglu = swiglu ? 1 : 0;
  if (rope) a.rope = *rope;
  a.err = err;
  return launch_status(pkv::launch_linear(a, pl, wmap, xmap, stream), "linear_tc");
}

// The fused entries' intermediate y [rows][n] bf16 lives in the workspace.
int check_linear_ws(void* workspace, size_t workspace_bytes, int32_t rows, int32_t n) {
  const size_t need = static_cast<size_t>(rows) * n * 2;
  if (!workspace || workspace_bytes < need)
    return fail(PKV_ERR_WORKSPACE, "linear needs %zu workspace bytes, got %zu", need,
                workspace ? workspace_bytes : (size_t)0);
  if (!aligned16(workspace)) return fail(PKV_ERR_ALIGN, "workspace not 16-byte aligned");
  return PKV_OK;
}

int launch_prefill_any(const pkv::PrefillLaunch& a, const pkv::KVSource& src, cudaStream_t s) {
  CUtensorMap qmap;
  int st = encode_q(&qmap, a.q, a.batch, a.num_q_heads, a.seq_len_q, a.q_sb, a.q_sh, a.q_st);
  if (st) return st;
  return launch_status(pkv::launch_prefill_tc(a, qmap, src, s), "prefill_tc");
}

}  // namespace

extern "C" {

int pkv_version(void) { return 100; }

const char* pkv_status_string(int status) {
  switch (status) {
    case PKV_OK: return "ok";
    case PKV_ERR_INVALID: return "invalid argument";
    case PKV_ERR_UNSUPPORTED: return "unsupported configuration";
    case PKV_ERR_ALIGN: return "misaligned pointer or stride";
    case PKV_ERR_DRIVER: return "CUDA driver / tensor map error";
    case PKV_ERR_LAUNCH: return "kernel launch failed";
    case PKV_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

const char* pkv_last_error(void) { return g_last_error.c_str(); }

int pkv_append_rope(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st, const void* k,
                    int64_t k_sb, int64_t k_sh, int64_t k_st, const void* v, int64_t v_sb,
                    int64_t v_sh, int64_t v_st, const void* rope_cos, const void* rope_sin,
                    int64_t rope_rows, void* q_out, int64_t qo_sb, int64_t qo_sh, int64_t qo_st,
                    void* k_pool, void* v_pool, int64_t num_slots, const int32_t* block_tables,
                    int64_t table_pitch, const int32_t* seq_rows, const int32_t* starts,
                    const int32_t* q_lens, int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t seq_len_q,
                    int32_t head_dim, int32_t* err_flag, void* stream) {
  int st = check_heads(num_q_heads, num_kv_heads, head_dim);
  if (st) return st;
  if ((st = check_pool(k_pool, v_pool, num_slots, block_tables, table_pitch))) return st;
  if (batch < 0 || seq_len_q < 0) return fail(PKV_ERR_INVALID, "negative batch / seq_len_q");
  if (!k || !v || !starts) return fail(PKV_ERR_INVALID, "null k, v or starts");
  if ((rope_cos == nullptr) != (rope_sin == nullptr))
    return fail(PKV_ERR_INVALID, "rope_cos and rope_sin must both be set or both NULL");
  if (rope_cos && rope_rows <= 0) return fail(PKV_ERR_INVALID, "rope_rows must be positive");
  if (q_out && (!q || !rope_cos)) return fail(PKV_ERR_INVALID, "q_out needs q and rope tables");
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 3u ||
      (q && (reinterpret_cast<uintptr_t>(q) & 3u)) ||
      (q_out && (reinterpret_cast<uintptr_t>(q_out) & 3u)) ||
      (rope_cos && ((reinterpret_cast<uintptr_t>(rope_cos) | reinterpret_cast<uintptr_t>(rope_sin)) & 3u)))
    return fail(PKV_ERR_ALIGN, "append pointers must be 4-byte aligned");
  if ((k_sb | k_sh | k_st | v_sb | v_sh | v_st) & 1 ||
      (q_out && ((q_sb | q_sh | q_st | qo_sb | qo_sh | qo_st) & 1)))
    return fail(PKV_ERR_ALIGN, "append strides must be even (4-byte rows pairs)");
  if (batch == 0 || seq_len_q == 0) return ok();
  pkv::AppendLaunch a{};
  a.q = q; a.q_sb = q_sb; a.q_sh = q_sh; a.q_st = q_st;
  a.k = k; a.k_sb = k_sb; a.k_sh = k_sh; a.k_st = k_st;
  a.v = v; a.v_sb = v_sb; a.v_sh = v_sh; a.v_st = v_st;
  a.rope_cos = rope_cos; a.rope_sin = rope_sin; a.rope_rows = rope_rows;
  a.q_out = q_out; a.qo_sb = qo_sb; a.qo_sh = qo_sh; a.qo_st = qo_st;
  a.k_pool = k_pool; a.v_pool = v_pool; a.num_slots = num_slots;
  a.tables = block_tables; a.pitch = table_pitch; a.rows = seq_rows; a.starts = starts;
  a.q_lens = q_lens;
  a.batch = batch; a.num_q_heads = num_q_heads; a.num_kv_heads = num_kv_heads;
  a.seq_len_q = seq_len_q; a.err = err_flag;
  return launch_status(pkv::launch_append(a, static_cast<cudaStream_t>(stream)), "append_rope");
}

// ---------------------------------------------------------------- FP8 pool
size_t pkv_fp8_block_bytes(void) { return pkv::kFp8HeadBlockBytes; }

static int check_pool8(const void* kv8, int64_t num_blocks, const int32_t* tables, int64_t pitch) {
  if (!kv8 || !tables) return fail(PKV_ERR_INVALID, "null FP8 pool or block-table pointer");
  if (num_blocks <= 0 || num_blocks > INT32_MAX / 16)
    return fail(PKV_ERR_INVALID, "num_blocks (%lld) out of range", (long long)num_blocks);
  if (pitch <= 0) return fail(PKV_ERR_INVALID, "table_pitch must be positive");
  if (!aligned16(kv8)) return fail(PKV_ERR_ALIGN, "FP8 pool not 16-byte aligned");
  return PKV_OK;
}

int pkv_append_rope_fp8(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st, const void* k,
                        int64_t k_sb, int64_t k_sh, int64_t k_st, const void* v, int64_t v_sb,
                        int64_t v_sh, int64_t v_st, const void* rope_cos, const void* rope_sin,
                        int64_t rope_rows, void* q_out, int64_t qo_sb, int64_t qo_sh,
                        int64_t qo_st, void* kv8_pool, int64_t num_blocks,
                        const int32_t* block_tables, int64_t table_pitch, const int32_t* seq_rows,
                        const int32_t* starts, const int32_t* q_lens, int32_t batch,
                        int32_t num_q_heads, int32_t num_kv_heads, int32_t seq_len_q,
                        int32_t head_dim, int32_t* err_flag, void* stream) {
  int st = check_heads(num_q_heads, num_kv_heads, head_dim);
  if (st) return st;
  if ((st = check_pool8(kv8_pool, num_blocks, block_tables, table_pitch))) return st;
  if (batch < 0 || seq_len_q < 0) return fail(PKV_ERR_INVALID, "negative batch / seq_len_q");
  if (!k || !v || !starts) return fail(PKV_ERR_INVALID, "null k, v or starts");
  if ((rope_cos == nullptr) != (rope_sin == nullptr))
    return fail(PKV_ERR_INVALID, "rope_cos and rope_sin must both be set or both NULL");
  if (rope_cos && rope_rows <= 0) return fail(PKV_ERR_INVALID, "rope_rows must be positive");
  if (q_out && (!q || !rope_cos)) return fail(PKV_ERR_INVALID, "q_out needs q and rope tables");
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 3u ||
      (q && (reinterpret_cast<uintptr_t>(q) & 3u)) ||
      (q_out && (reinterpret_cast<uintptr_t>(q_out) & 3u)) ||
      (rope_cos && ((reinterpret_cast<uintptr_t>(rope_cos) | reinterpret_cast<uintptr_t>(rope_sin)) & 3u)))
    return fail(PKV_ERR_ALIGN, "append pointers must be 4-byte aligned");
  if ((k_sb | k_sh | k_st | v_sb | v_sh | v_st) & 1 ||
      (q_out && ((q_sb | q_sh | q_st | qo_sb | qo_sh | qo_st) & 1)))
    return fail(PKV_ERR_ALIGN, "append strides must be even (4-byte rows pairs)");
  if (batch == 0 || seq_len_q == 0) return ok();
  pkv::AppendLaunch a{};
  a.q = q; a.q_sb = q_sb; a.q_sh = q_sh; a.q_st = q_st;
  a.k = k; a.k_sb = k_sb; a.k_sh = k_sh; a.k_st = k_st;
  a.v = v; a.v_sb = v_sb; a.v_sh = v_sh; a.v_st = v_st;
  a.rope_cos = rope_cos; a.rope_sin = rope_sin; a.rope_rows = rope_rows;
  a.q_out = q_out; a.qo_sb = qo_sb; a.qo_sh = qo_sh; a.qo_st = qo_st;
  a.kv8 = static_cast<uint8_t*>(kv8_pool); a.num_slots = num_blocks * 16;
  a.tables = block_tables; a.pitch = table_pitch; a.rows = seq_rows; a.starts = starts;
  a.q_lens = q_lens;
  a.batch = batch; a.num_q_heads = num_q_heads; a.num_kv_heads = num_kv_heads;
  a.seq_len_q = seq_len_q; a.err = err_flag;
  return launch_status(pkv::launch_append(a, static_cast<cudaStream_t>(stream)), "append_rope_fp8");
}

int pkv_fp8_dequant(const void* kv8_pool, int64_t num_blocks, const int32_t* block_tables,
                    int64_t table_pitch, const int32_t* seq_rows, const int32_t* kv_lens,
                    int32_t batch, int32_t num_kv_heads, int32_t seq_len, void* k_out,
                    int64_t k_sb, int64_t k_sh, int64_t k_ss, void* v_out, int64_t v_sb,
                    int64_t v_sh, int64_t v_ss, int32_t* err_flag, void* stream) {
  int st = check_pool8(kv8_pool, num_blocks, block_tables, table_pitch);
  if (st) return st;
  if (num_kv_heads <= 0) return fail(PKV_ERR_INVALID, "num_kv_heads must be positive");
  if (!kv_lens || !k_out || !v_out) return fail(PKV_ERR_INVALID, "null kv_lens, k_out or v_out");
  if (batch < 0 || seq_len < 0) return fail(PKV_ERR_INVALID, "negative batch / seq_len");
  if (((reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(v_out)) & 7u) ||
      ((k_sb | k_sh | k_ss | v_sb | v_sh | v_ss) & 3))
    return fail(PKV_ERR_ALIGN, "dequant outputs need 8-byte aligned rows");
  if (batch == 0 || seq_len == 0) return ok();
  pkv::Fp8DequantLaunch a{};
  a.kv8 = static_cast<const uint8_t*>(kv8_pool);
  a.num_blocks = static_cast<int32_t>(num_blocks);
  a.tables = block_tables; a.pitch = table_pitch; a.rows = seq_rows; a.kv_lens = kv_lens;
  a.batch = batch; a.num_kv_heads = num_kv_heads; a.seq_len = seq_len;
  a.k_out = k_out; a.k_sb = k_sb; a.k_sh = k_sh; a.k_ss = k_ss;
  a.v_out = v_out; a.v_sb = v_sb; a.v_sh = v_sh; a.v_ss = v_ss;
  a.err = err_flag;
  return launch_status(pkv::launch_fp8_dequant(a, static_cast<cudaStream_t>(stream)), "fp8_dequant");
}

size_t pkv_decode_workspace_size(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                 int32_t max_kv_len) {
  if (batch <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0) return 0;
  // enough for either pool format's plan
  const size_t a = pkv::plan_decode(batch, num_q_heads, num_kv_heads, max_kv_len).workspace_bytes;
  const size_t b = pkv::plan_decode(batch, num_q_heads, num_kv_heads, max_kv_len, true).workspace_bytes;
  return a > b ? a : b;
}

int pkv_decode_plan(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t max_kv_len,
                    int32_t* plan) {
  if (!plan || batch <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || max_kv_len < 0 ||
      num_q_heads % num_kv_heads != 0)
    return fail(PKV_ERR_INVALID, "decode_plan: bad sizes");
  const pkv::DecodePlan pl = pkv::plan_decode(batch, num_q_heads, num_kv_heads, max_kv_len);
  plan[0] = pl.blocks_per_part;
  plan[1] = pl.min_blocks_per_part;
  plan[2] = pl.max_parts;
  plan[3] = pl.sub_groups;
  return ok();
}

static int decode_common(const pkv::DecodeLaunch& a, const pkv::KVSource& src, cudaStream_t stream) {
  const pkv::DecodePlan plan =
      pkv::plan_decode(a.batch, a.num_q_heads, a.num_kv_heads, a.max_kv_len, a.kv8 != nullptr);
  if (static_cast<int64_t>(a.batch) * a.num_kv_heads * plan.sub_groups > pkv::decode_max_units())
    return fail(PKV_ERR_UNSUPPORTED, "batch * kv_heads too large for one decode launch (max %lld)",
                (long long)pkv::decode_max_units());
  if (plan.workspace_bytes > 0) {
    if (!a.workspace || a.workspace_bytes < plan.workspace_bytes)
      return fail(PKV_ERR_WORKSPACE, "decode needs %zu workspace bytes, got %zu",
                  plan.workspace_bytes, a.workspace ? a.workspace_bytes : (size_t)0);
    if (!aligned16(a.workspace)) return fail(PKV_ERR_ALIGN, "workspace not 16-byte aligned");
  }
  return launch_status(pkv::launch_decode(a, src, plan, stream), "paged_decode");
}

static int check_qo(const void* q, const void* out, int64_t s0, int64_t s1, int64_t s2, int64_t o0,
                    int64_t o1, int64_t o2) {
  if (!q || !out) return fail(PKV_ERR_INVALID, "null q or out");
  if (!aligned16(q) || !aligned16(out)) return fail(PKV_ERR_ALIGN, "q/out not 16-byte aligned");
  if (!mult8(s0) || !mult8(s1) || !mult8(s2) || !mult8(o0) || !mult8(o1) || !mult8(o2))
    return fail(PKV_ERR_ALIGN, "q/out strides must be multiples of 8 elements");
  return PKV_OK;
}

int pkv_paged_decode(const void* q, int64_t q_sb, int64_t q_sh, const void* k_pool,
                     const void* v_pool, int64_t num_slots, const int32_t* block_tables,
                     int64_t table_pitch, const int32_t* seq_rows, const int32_t* kv_lens,
                     int32_t max_kv_len, int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                     int32_t head_dim, float sm_scale, void* out, int64_t o_sb, int64_t o_sh,
                     void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream) {
  int st = check_heads(num_q_heads, num_kv_heads, head_dim);
  if (st) return st;
  if ((st = check_pool(k_pool, v_pool, num_slots, block_tables, table_pitch))) return st;
  if ((st = check_qo(q, out, q_sb, q_sh, 0, o_sb, o_sh, 0))) return st;
  if (!kv_lens) return fail(PKV_ERR_INVALID, "null kv_lens");
  if (batch < 0 || max_kv_len < 0) return fail(PKV_ERR_INVALID, "negative batch / max_kv_len");
  if (batch == 0) return ok();
  pkv::KVSource src{};
  src.paged = true;
  if ((st = encode_pool(&src.kmap, k_pool, num_slots, num_kv_heads))) return st;
  if ((st = encode_pool(&src.vmap, v_pool, num_slots, num_kv_heads))) return st;
  src.tables = block_tables;
  src.pitch = table_pitch;
  src.rows = seq_rows;
  src.num_blocks = static_cast<int32_t>(num_slots / 16);
  pkv::DecodeLaunch a{};
  a.q = q; a.q_sb = q_sb; a.q_sh = q_sh;
  a.out = out; a.o_sb = o_sb; a.o_sh = o_sh;
  a.kv_lens = kv_lens; a.batch = batch; a.num_q_heads = num_q_heads; a.num_kv_heads = num_kv_heads;
  a.max_kv_len = max_kv_len; a.sm_scale = sm_scale;
  a.workspace = workspace; a.workspace_bytes = workspace_bytes; a.err = err_flag;
  return decode_common(a, src, static_cast<cudaStream_t>(stream));
}

int pkv_paged_decode_fp8(const void* q, int64_t q_sb, int64_t q_sh, const void* kv8_pool,
                         int64_t num_blocks, const int32_t* block_tables, int64_t table_pitch,
                         const int32_t* seq_rows, const int32_t* kv_lens, int32_t max_kv_len,
                         int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                         int32_t head_dim, float sm_scale, void* out, int64_t o_sb, int64_t o_sh,
                         void* workspace, size_t workspace_bytes, int32_t* err_flag,
                         void* stream) {
  int st = check_heads(num_q_heads, num_kv_heads, head_dim);
  if (st) return st;
  if ((st = check_pool8(kv8_pool, num_blocks, block_tables, table_pitch))) return st;
  if ((st = check_qo(q, out, q_sb, q_sh, 0, o_sb, o_sh, 0))) return st;
  if (!kv_lens) return fail(PKV_ERR_INVALID, "null kv_lens");
  if (batch < 0 || max_kv_len < 0) return fail(PKV_ERR_INVALID, "negative batch / max_kv_len");
  if (batch == 0) return ok();
  pkv::KVSource src{};
  src.paged = true;
  src.tables = block_tables;
  src.pitch = table_pitch;
  src.rows = seq_rows;
  src.num_blocks = static_cast<int32_t>(num_blocks);
  pkv::DecodeLaunch a{};
  a.q = q; a.q_sb = q_sb; a.q_sh = q_sh;
  a.out = out; a.o_sb = o_sb; a.o_sh = o_sh;
  a.kv_lens = kv_lens; a.batch = batch; a.num_q_heads = num_q_heads; a.num_kv_heads = num_kv_heads;
  a.max_kv_len = max_kv_len; a.sm_scale = sm_scale;
  a.workspace = workspace; a.workspace_bytes = workspace_bytes; a.err = err_flag;
  a.kv8 = static_cast<const uint8_t*>(kv8_pool);
  return decode_common(a, src, static_cast<cudaStream_t>(stream));
}

int pkv_paged_prefill(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st, const void* k_pool,
                      const void* v_pool, int64_t num_slots, const int32_t* block_tables,
                      int64_t table_pitch, const int32_t* seq_rows, const int32_t* kv_lens,
                      const int32_t* q_lens, int32_t max_kv_len, int32_t batch, int32_t seq_len_q,
                      int32_t num_q_heads,
                      int32_t num_kv_heads, int32_t head_dim, int32_t causal, float sm_scale,
                      void* out, int64_t o_sb, int64_t o_sh, int64_t o_st, int32_t* err_flag,
                      void* stream) {
  (void)max_kv_len;
  int st = check_heads(num_q_heads, num_kv_heads, head_dim);
  if (st) return st;
  if ((st = check_pool(k_pool, v_pool, num_slots, block_tables, table_pitch))) return st;
  if ((st = check_qo(q, out, q_sb, q_sh, q_st, o_sb, o_sh, o_st))) return st;
  if (!kv_lens) return fail(PKV_ERR_INVALID, "null kv_lens");
  if (batch < 0 || seq_len_q < 0) return fail(PKV_ERR_INVALID, "negative batch / seq_len_q");
  if (batch == 0 || seq_len_q == 0) return ok();
  pkv::KVSource src{};
  src.paged = true;
  if ((st = encode_pool(&src.kmap, k_pool, num_slots, num_kv_heads))) return st;
  if ((st = encode_pool(&src.vmap, v_pool, num_slots, num_kv_heads))) return st;
  src.tables = block_tables;
  src.pitch = table_pitch;
  src.rows = seq_rows;
  src.num_blocks = static_cast<int32_t>(num_slots / 16);
  pkv::PrefillLaunch a{};
  a.q = q; a.q_sb = q_sb; a.q_sh = q_sh; a.q_st = q_st;
  a.out = out; a.o_sb = o_sb; a.o_sh = o_sh; a.o_st = o_st;
  a.kv_lens = kv_lens; a.q_lens = q_lens; a.batch = batch; a.seq_len_q = seq_len_q;
  a.num_q_heads = num_q_heads; a.num_kv_heads = num_kv_heads; a.causal = causal ? 1 : 0;
  a.sm_scale = sm_scale; a.err = err_flag;
  return launch_prefill_any(a, src, static_cast<cudaStream_t>(stream));
}

int pkv_dense_attention(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_st, const void* k,
                        int64_t k_sb, int64_t k_sh, int64_t k_ss, const void* v, int64_t v_sb,
                        int64_t v_sh, int64_t v_ss, const int32_t* kv_lens, int32_t batch,
                        int32_t seq_len_q, int32_t seq_len_k, int32_t num_q_heads,
                        int32_t num_kv_heads, int32_t head_dim, int32_t causal, float sm_scale,
                        void* out, int64_t o_sb, int64_t o_sh, int64_t o_st, void* workspace,
                        size_t workspace_bytes, int32_t* err_flag, void* stream) {
  int st = check_heads(num_q_heads, num_kv_heads, head_dim);
  if (st) return st;
  if ((st = check_qo(q, out, q_sb, q_sh, q_st, o_sb, o_sh, o_st))) return st;
  if (!k || !v || !kv_lens) return fail(PKV_ERR_INVALID, "null k, v or kv_lens");
  if (!aligned16(k) || !aligned16(v)) return fail(PKV_ERR_ALIGN, "k/v not 16-byte aligned");
  if (!mult8(k_sb) || !mult8(k_sh) || !mult8(k_ss) || !mult8(v_sb) || !mult8(v_sh) || !mult8(v_ss))
    return fail(PKV_ERR_ALIGN, "k/v strides must be multiples of 8 elements");
  if (batch < 0 || seq_len_q < 0 || seq_len_k < 0)
    return fail(PKV_ERR_INVALID, "negative batch / seq lens");
  if (batch == 0 || seq_len_q == 0) return ok();
  if (seq_len_k == 0) return fail(PKV_ERR_INVALID, "seq_len_k must be positive");
  pkv::KVSource src{};
  src.paged = false;
  if ((st = encode_dense(&src.kmap, k, batch, num_kv_heads, seq_len_k, k_sb, k_sh, k_ss))) return st;
  if ((st = encode_dense(&src.vmap, v, batch, num_kv_heads, seq_len_k, v_sb, v_sh, v_ss))) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (seq_len_q == 1) {
    pkv::DecodeLaunch a{};
    a.q = q; a.q_sb = q_sb; a.q_sh = q_sh;
    a.out = out; a.o_sb = o_sb; a.o_sh = o_sh;
    a.kv_lens = kv_lens; a.batch = batch; a.num_q_heads = num_q_heads;
    a.num_kv_heads = num_kv_heads; a.max_kv_len = seq_len_k; a.sm_scale = sm_scale;
    a.workspace = workspace; a.workspace_bytes = workspace_bytes; a.err = err_flag;
    return decode_common(a, src, s);
  }
  pkv::PrefillLaunch a{};
  a.q = q; a.q_sb = q_sb; a.q_sh = q_sh; a.q_st = q_st;
  a.out = out; a.o_sb = o_sb; a.o_sh = o_sh; a.o_st = o_st;
  a.kv_lens = kv_lens; a.batch = batch; a.seq_len_q = seq_len_q;
  a.num_q_heads = num_q_heads; a.num_kv_heads = num_kv_heads; a.causal = causal ? 1 : 0;
  a.sm_scale = sm_scale; a.err = err_flag;
  return launch_prefill_any(a, src, s);
}

int pkv_add_rmsnorm(const void* a, int64_t a_stride, const void* resid, int64_t r_stride,
                    void* resid_out, int64_t ro_stride, const void* weight, void* out,
                    int64_t o_stride, int32_t rows, int32_t dim, float eps, void* stream) {
  if (!a || !weight || !out) return fail(PKV_ERR_INVALID, "null a, weight or out");
  if (rows < 0 || dim <= 0 || dim % 8 != 0 || dim > 4096)
    return fail(PKV_ERR_UNSUPPORTED, "dim must be a positive multiple of 8 up to 4096 (got %d)", dim);
  if (!aligned16(a) || !aligned16(weight) || !aligned16(out) || (resid && !aligned16(resid)) ||
      (resid_out && !aligned16(resid_out)) || !mult8(a_stride) || !mult8(o_stride) ||
      (resid && !mult8(r_stride)) || (resid_out && !mult8(ro_stride)))
    return fail(PKV_ERR_ALIGN, "add_rmsnorm rows must be 16-byte aligned");
  if (rows == 0) return ok();
  pkv::NormLaunch p{a, a_stride, resid, r_stride, resid_out, ro_stride, weight, out, o_stride,
                    rows, dim, eps};
  return launch_status(pkv::launch_add_rmsnorm(p, static_cast<cudaStream_t>(stream)), "add_rmsnorm");
}

int pkv_sample(const void* logits, int64_t ld, int32_t rows, int32_t vocab, int32_t dtype,
               float temperature, uint64_t seed, uint64_t call, int32_t* out, void* stream) {
  if (!logits || !out) return fail(PKV_ERR_INVALID, "null logits or out");
  if (dtype != 0 && dtype != 1) return fail(PKV_ERR_UNSUPPORTED, "dtype must be 0 (bf16) or 1 (f32)");
  if (rows < 0 || rows > 65535 || vocab <= 0 || ld < vocab)
    return fail(PKV_ERR_INVALID, "bad sample shape: rows %d (<= 65535), vocab %d, ld %lld", rows,
                vocab, static_cast<long long>(ld));
  if (!(temperature > 0.f) || !(temperature < INFINITY))
    return fail(PKV_ERR_INVALID, "temperature must be positive and finite");
  const size_t esz = dtype == 1 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(logits) % esz != 0)
    return fail(PKV_ERR_ALIGN, "logits not aligned to their element size");
  if (rows == 0) return ok();
  pkv::SampleLaunch a{};
  a.logits = logits;
  a.ld = ld;
  a.rows = rows;
  a.vocab = vocab;
  a.f32 = dtype == 1;
  // 4-wide loads when every row starts on a 4-element boundary
  a.vec = (ld % 4 == 0) && (reinterpret_cast<uintptr_t>(logits) % (4 * esz) == 0);
  a.splits = pkv::sample_splits(rows, vocab);
  a.inv_temp = 1.0f / temperature;
  a.seed = seed;
  a.call = call;
  a.out = out;
  return launch_status(pkv::launch_sample(a, static_cast<cudaStream_t>(stream)), "sample");
}

int pkv_silu_mul(const void* gu, int64_t gu_stride, void* out, int64_t o_stride, int32_t rows,
                 int32_t inter, void* stream) {
  if (!gu || !out) return fail(PKV_ERR_INVALID, "null gu or out");
  if (rows < 0 || inter <= 0 || inter % 8 != 0)
    return fail(PKV_ERR_UNSUPPORTED, "inter must be a positive multiple of 8 (got %d)", inter);
  if (!aligned16(gu) || !aligned16(out) || !mult8(gu_stride) || !mult8(o_stride))
    return fail(PKV_ERR_ALIGN, "silu_mul rows must be 16-byte aligned");
  if (rows == 0) return ok();
  return launch_status(pkv::launch_silu_mul(gu, gu_stride, out, o_stride, rows, inter,
                                            static_cast<cudaStream_t>(stream)),
                       "silu_mul");
}

int pkv_paged_decode_static_scratch(const void* q, int64_t q_sb, int64_t q_sh, const void* k_pool,
                                    const void* v_pool, int64_t num_slots,
                                    const int32_t* block_tables, int64_t table_pitch,
                                    const int32_t* seq_rows, const int32_t* kv_lens,
                                    int32_t max_kv_len, int32_t batch, int32_t num_q_heads,
                                    int32_t num_kv_heads, int32_t head_dim, float sm_scale,
                                    void* out, int64_t o_sb, int64_t o_sh, int32_t* err_flag,
                                    void* stream) {
  int st = check_heads(num_q_heads, num_kv_heads, head_dim);
  if (st) return st;
  if ((st = check_pool(k_pool, v_pool, num_slots, block_tables, table_pitch))) return st;
  if ((st = check_qo(q, out, q_sb, q_sh, 0, o_sb, o_sh, 0))) return st;
  if (!kv_lens) return fail(PKV_ERR_INVALID, "null kv_lens");
  if (batch < 0 || max_kv_len < 0) return fail(PKV_ERR_INVALID, "negative batch / max_kv_len");
  if (batch == 0) return ok();
  const pkv::DecodePlan plan = pkv::plan_decode(batch, num_q_heads, num_kv_heads, max_kv_len);
  if (static_cast<int64_t>(batch) * num_kv_heads * plan.sub_groups > pkv::decode_max_units())
    return fail(PKV_ERR_UNSUPPORTED, "batch * kv_heads too large for one decode launch (max %lld)",
                (long long)pkv::decode_max_units());
  if (plan.workspace_bytes > PKV_DECODE_STATIC_SCRATCH_BYTES)
    return fail(PKV_ERR_WORKSPACE,
                "this shape needs %zu bytes of split-K scratch, more than the %u-byte static "
                "array; use pkv_paged_decode with a caller-provided workspace",
                plan.workspace_bytes, (unsigned)PKV_DECODE_STATIC_SCRATCH_BYTES);
  pkv::KVSource src{};
  src.paged = true;
  if ((st = encode_pool(&src.kmap, k_pool, num_slots, num_kv_heads))) return st;
  if ((st = encode_pool(&src.vmap, v_pool, num_slots, num_kv_heads))) return st;
  src.tables = block_tables;
  src.pitch = table_pitch;
  src.rows = seq_rows;
  src.num_blocks = static_cast<int32_t>(num_slots / 16);
  pkv::DecodeLaunch a{};
  a.q = q; a.q_sb = q_sb; a.q_sh = q_sh;
  a.out = out; a.o_sb = o_sb; a.o_sh = o_sh;
  a.kv_lens = kv_lens; a.batch = batch; a.num_q_heads = num_q_heads; a.num_kv_heads = num_kv_heads;
  a.max_kv_len = max_kv_len; a.sm_scale = sm_scale; a.err = err_flag;
  return launch_status(pkv::launch_decode_static(a, src, plan, static_cast<cudaStream_t>(stream)),
                       "paged_decode_static_scratch");
}

size_t pkv_linear_workspace_size(int32_t rows, int32_t n, int32_t k) {
  if (rows <= 0 || rows > PKV_LINEAR_MAX_ROWS || n <= 0 || n % 128 != 0 || k <= 0 || k % 64 != 0)
    return 0;
  return static_cast<size_t>(rows) * n * 2;
}

int pkv_linear_pair_gate_up(const void* w_gate_up, int64_t ldw, int32_t inter, int32_t k,
                            void* w_paired, void* stream) {
  if (!w_gate_up || !w_paired) return fail(PKV_ERR_INVALID, "null w_gate_up or w_paired");
  if (inter <= 0 || inter % 64 != 0 || k <= 0 || k % 64 != 0)
    return fail(PKV_ERR_UNSUPPORTED, "inter and k must be positive multiples of 64 (got %d, %d)",
                inter, k);
  if (ldw < k) return fail(PKV_ERR_INVALID, "row stride smaller than k");
  if (!aligned16(w_gate_up) || !aligned16(w_paired) || !mult8(ldw))
    return fail(PKV_ERR_ALIGN, "weights must be 16-byte aligned, ldw a multiple of 8");
  return launch_status(pkv::launch_pair_gate_up(w_gate_up, ldw, inter, k, w_paired,
                                                static_cast<cudaStream_t>(stream)),
                       "pair_gate_up");
}

int pkv_linear_pack_weight(const void* w, int64_t ldw, int32_t n, int32_t k, void* w_tiled,
                           void* stream) {
  if (!w || !w_tiled) return fail(PKV_ERR_INVALID, "null w or w_tiled");
  if (n <= 0 || n % 128 != 0 || k <= 0 || k % 64 != 0)
    return fail(PKV_ERR_UNSUPPORTED, "n must be a positive multiple of 128 and k of 64 (got %d, %d)",
                n, k);
  if (ldw < k) return fail(PKV_ERR_INVALID, "row stride smaller than k");
  if (!aligned16(w) || !aligned16(w_tiled) || !mult8(ldw))
    return fail(PKV_ERR_ALIGN, "w / w_tiled must be 16-byte aligned, ldw a multiple of 8");
  return launch_status(pkv::launch_pack_weight(w, ldw, n, k, w_tiled,
                                               static_cast<cudaStream_t>(stream)),
                       "pack_weight");
}

int pkv_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, int32_t w_layout,
               const void* bias, int32_t rows, int32_t n, int32_t k, void* y, int64_t ldy,
               void* workspace, size_t workspace_bytes, int32_t* err_flag, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  int st = check_linear(x, ldx, w, ldw, w_layout, rows, n, k);
  if (st) return st;
  if (w_layout == PKV_W_GATE_UP_PAIRED)
    return fail(PKV_ERR_INVALID, "PKV_W_GATE_UP_PAIRED weights are for pkv_linear_silu_mul only");
  if (!y) return fail(PKV_ERR_INVALID, "null y");
  if (!aligned16(y) || !mult8(ldy) || ldy < n || (bias && !aligned16(bias)))
    return fail(PKV_ERR_ALIGN, "y / bias must be 16-byte aligned, ldy a multiple of 8 >= n");
  if (rows == 0) return ok();
  if ((st = run_linear(x, ldx, w, ldw, w_layout, rows, n, k, y, ldy, bias, err_flag,
                       static_cast<cudaStream_t>(stream))))
    return st;
  return ok();
}

int pkv_linear_add_rmsnorm(const void* x, int64_t ldx, const void* w, int64_t ldw,
                           int32_t w_layout, int32_t rows, int32_t n, int32_t k,
                           const void* resid, int64_t r_stride, void* resid_out,
                           int64_t ro_stride, const void* norm_weight, float eps, void* out,
                           int64_t o_stride, void* workspace, size_t workspace_bytes,
                           int32_t* err_flag, void* stream) {
  int st = check_linear(x, ldx, w, ldw, w_layout, rows, n, k);
  if (st) return st;
  if (!norm_weight || !out) return fail(PKV_ERR_INVALID, "null norm weight or out");
  if (n > 4096) return fail(PKV_ERR_UNSUPPORTED, "add_rmsnorm dim must be <= 4096 (got %d)", n);
  if (!aligned16(norm_weight) || !aligned16(out) || (resid && !aligned16(resid)) ||
      (resid_out && !aligned16(resid_out)) || !mult8(o_stride) || (resid && !mult8(r_stride)) ||
      (resid_out && !mult8(ro_stride)))
    return fail(PKV_ERR_ALIGN, "add_rmsnorm rows must be 16-byte aligned");
  if (rows == 0) return ok();
  if ((st = check_linear_ws(workspace, workspace_bytes, rows, n))) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((st = run_linear(x, ldx, w, ldw, w_layout, rows, n, k, workspace, n, nullptr, err_flag, s)))
    return st;
  pkv::NormLaunch p{workspace, n, resid, r_stride, resid_out, ro_stride, norm_weight, out,
                    o_stride, rows, n, eps};
  return launch_status(pkv::launch_add_rmsnorm(p, s), "add_rmsnorm");
}

int pkv_linear_silu_mul(const void* x, int64_t ldx, const void* w_gate_up, int64_t ldw,
                        int32_t w_layout, int32_t rows, int32_t inter, int32_t k, void* out,
                        int64_t o_stride, void* workspace, size_t workspace_bytes,
                        int32_t* err_flag, void* stream) {
  if (inter <= 0 || inter % 64 != 0)
    return fail(PKV_ERR_UNSUPPORTED, "inter must be a positive multiple of 64 (got %d)", inter);
  const int32_t n = 2 * inter;
  int st = check_linear(x, ldx, w_gate_up, ldw, w_layout, rows, n, k);
  if (st) return st;
  if (!out) return fail(PKV_ERR_INVALID, "null out");
  if (!aligned16(out) || !mult8(o_stride)) return fail(PKV_ERR_ALIGN, "silu_mul rows must be 16-byte aligned");
  if (rows == 0) return ok();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (w_layout == PKV_W_GATE_UP_PAIRED) {  // SwiGLU in the GEMM's epilogue
    if ((st = run_linear(x, ldx, w_gate_up, ldw, w_layout, rows, n, k, out, o_stride, nullptr,
                         err_flag, s, true)))
      return st;
    return ok();
  }
  if ((st = check_linear_ws(workspace, workspace_bytes, rows, n))) return st;
  if ((st = run_linear(x, ldx, w_gate_up, ldw, w_layout, rows, n, k, workspace, n, nullptr,
                       err_flag, s)))
    return st;
  return launch_status(pkv::launch_silu_mul(workspace, n, out, o_stride, rows, inter, s),
                       "silu_mul");
}

int pkv_linear_rope_append(const void* x, int64_t ldx, const void* w_qkv, int64_t ldw,
                           int32_t w_layout, const void* bias, int32_t k, const void* rope_cos,
                           const void* rope_sin, int64_t rope_rows, void* q_out, int64_t qo_sb,
                           int64_t qo_sh, int64_t qo_st, void* k_pool, void* v_pool,
                           int64_t num_slots, const int32_t* block_tables, int64_t table_pitch,
                           const int32_t* seq_rows, const int32_t* starts, const int32_t* q_lens,
                           int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                           int32_t seq_len_q, int32_t head_dim, void* workspace,
                           size_t workspace_bytes, int32_t* err_flag, void* stream) {
  int st = check_heads(num_q_heads, num_kv_heads, head_dim);
  if (st) return st;
  if ((st = check_pool(k_pool, v_pool, num_slots, block_tables, table_pitch))) return st;
  if (batch < 0 || seq_len_q < 0) return fail(PKV_ERR_INVALID, "negative batch / seq_len_q");
  const int64_t rows64 = static_cast<int64_t>(batch) * seq_len_q;
  if (rows64 > PKV_LINEAR_MAX_ROWS)
    return fail(PKV_ERR_UNSUPPORTED, "batch * seq_len_q must be <= %d (got %lld)",
                PKV_LINEAR_MAX_ROWS, (long long)rows64);
  const int32_t rows = static_cast<int32_t>(rows64);
  const int32_t n = (num_q_heads + 2 * num_kv_heads) * head_dim;
  if ((st = check_linear(x, ldx, w_qkv, ldw, w_layout, rows, n, k))) return st;
  if (!starts || !q_out || !rope_cos || !rope_sin)
    return fail(PKV_ERR_INVALID, "null starts, q_out or rope tables");
  if (rope_rows <= 0) return fail(PKV_ERR_INVALID, "rope_rows must be positive");
  if ((reinterpret_cast<uintptr_t>(q_out) | reinterpret_cast<uintptr_t>(rope_cos) |
       reinterpret_cast<uintptr_t>(rope_sin)) & 3u ||
      (bias && !aligned16(bias)))
    return fail(PKV_ERR_ALIGN, "append pointers must be 4-byte aligned, bias 16-byte aligned");
  if ((qo_sb | qo_sh | qo_st) & 1) return fail(PKV_ERR_ALIGN, "q_out strides must be even");
  if (rows == 0) return ok();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (aligned16(q_out) && mult8(qo_sb) && mult8(qo_sh) && mult8(qo_st)) {
    // RoPE + append in the GEMM's epilogue (8-byte stores of q_out rows)
    pkv::RopeAppend r{};
    r.q_out = static_cast<__nv_bfloat16*>(q_out);
    r.qo_sb = qo_sb; r.qo_sh = qo_sh; r.qo_st = qo_st;
    r.k_pool = static_cast<__nv_bfloat16*>(k_pool);
    r.v_pool = static_cast<__nv_bfloat16*>(v_pool);
    r.num_blocks = static_cast<int32_t>(num_slots / 16);
    r.cos = static_cast<const __nv_bfloat16*>(rope_cos);
    r.sin = static_cast<const __nv_bfloat16*>(rope_sin);
    r.rope_rows = rope_rows;
    r.tables = block_tables; r.pitch = table_pitch; r.rows = seq_rows; r.starts = starts;
    r.q_lens = q_lens;
    r.T = seq_len_q; r.hq = num_q_heads; r.hkv = num_kv_heads;
    if ((st = run_linear(x, ldx, w_qkv, ldw, w_layout, rows, n, k, nullptr, 0, bias, err_flag, s,
                         false, &r)))
      return st;
    return ok();
  }
  if ((st = check_linear_ws(workspace, workspace_bytes, rows, n))) return st;
  if ((st = run_linear(x, ldx, w_qkv, ldw, w_layout, rows, n, k, workspace, n, bias, err_flag, s)))
    return st;
  // the GEMM output [batch][seq_len_q][q heads | k heads | v heads][128]
  const int64_t tok = n, head = head_dim, row = static_cast<int64_t>(seq_len_q) * n;
  const __nv_bfloat16* qkv = static_cast<const __nv_bfloat16*>(workspace);
  pkv::AppendLaunch a{};
  a.q = qkv; a.q_sb = row; a.q_sh = head; a.q_st = tok;
  a.k = qkv + num_q_heads * head; a.k_sb = row; a.k_sh = head; a.k_st = tok;
  a.v = qkv + (num_q_heads + num_kv_heads) * head; a.v_sb = row; a.v_sh = head; a.v_st = tok;
  a.rope_cos = rope_cos; a.rope_sin = rope_sin; a.rope_rows = rope_rows;
  a.q_out = q_out; a.qo_sb = qo_sb; a.qo_sh = qo_sh; a.qo_st = qo_st;
  a.k_pool = k_pool; a.v_pool = v_pool; a.num_slots = num_slots;
  a.tables = block_tables; a.pitch = table_pitch; a.rows = seq_rows; a.starts = starts;
  a.q_lens = q_lens;
  a.batch = batch; a.num_q_heads = num_q_heads; a.num_kv_heads = num_kv_heads;
  a.seq_len_q = seq_len_q; a.err = err_flag;
  return launch_status(pkv::launch_append(a, s), "append_rope");
}

// ---------------------------------------------------------------- decode layers
static int device_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 0;
  return n;
}

size_t pkv_decode_layers_workspace_size(int32_t rows) {
  const int sms = device_sms();
  if (rows <= 0 || rows > PKV_LAYERS_MAX_ROWS || sms <= 0) return 0;
  return pkv::decode_layers_workspace_bytes(rows, sms);
}

int pkv_decode_layers(const pkv_layer_weights* layers, int32_t num_layers, const void* h0,
                      void* xs, void* m_out, int32_t rows, void* kv_pool, int64_t num_slots,
                      const int32_t* block_tables, int64_t table_pitch, const int32_t* seq_rows,
                      const int32_t* starts, const void* rope_cos, const void* rope_sin,
                      int64_t rope_rows, float eps, void* workspace, size_t workspace_bytes,
                      int32_t* err_flag, void* stream) {
  if (!layers || num_layers <= 0 || num_layers > PKV_LAYERS_MAX_LAYERS)
    return fail(PKV_ERR_UNSUPPORTED, "num_layers must be in [1, %d] (got %d)",
                PKV_LAYERS_MAX_LAYERS, num_layers);
  if (rows < 0 || rows > PKV_LAYERS_MAX_ROWS)
    return fail(PKV_ERR_UNSUPPORTED, "rows must be in [0, %d] (got %d)", PKV_LAYERS_MAX_ROWS, rows);
  if (!h0 || !xs || !m_out || !starts || !rope_cos || !rope_sin)
    return fail(PKV_ERR_INVALID, "null h0, xs, m_out, starts or rope tables");
  if (rope_rows <= 0) return fail(PKV_ERR_INVALID, "rope_rows must be positive");
  int st = check_pool(kv_pool, kv_pool, num_slots, block_tables, table_pitch);
  if (st) return st;
  if (!aligned16(h0) || !aligned16(xs) || !aligned16(m_out) || !aligned16(rope_cos) ||
      !aligned16(rope_sin))
    return fail(PKV_ERR_ALIGN, "h0, xs, m_out and rope tables must be 16-byte aligned");
  for (int l = 0; l < num_layers; ++l) {
    const pkv_layer_weights& w = layers[l];
    if (!w.qkv_w || !w.qkv_b || !w.o_w || !w.post_norm_w || !w.gate_up_w || !w.down_w ||
        (l > 0 && !w.in_norm_w))
      return fail(PKV_ERR_INVALID, "layer %d: null weight", l);
    if (!aligned16(w.qkv_w) || !aligned16(w.qkv_b) || !aligned16(w.o_w) ||
        !aligned16(w.post_norm_w) || !aligned16(w.gate_up_w) || !aligned16(w.down_w) ||
        (l > 0 && !aligned16(w.in_norm_w)))
      return fail(PKV_ERR_ALIGN, "layer %d: weights must be 16-byte aligned", l);
  }
  if (rows == 0) return ok();
  const int sms = device_sms();
  if (sms <= 0) return fail(PKV_ERR_DRIVER, "no current CUDA device");
  const pkv::LayersPlan pl = pkv::plan_decode_layers(rows, sms);
  if (!pl.valid) return fail(PKV_ERR_UNSUPPORTED, "no decode-layers plan for %d SMs", sms);
  const size_t need = pkv::decode_layers_workspace_bytes(rows, sms);
  if (!workspace || workspace_bytes < need)
    return fail(PKV_ERR_WORKSPACE, "decode_layers needs %zu workspace bytes, got %zu", need,
                workspace ? workspace_bytes : (size_t)0);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(PKV_ERR_ALIGN, "workspace not 256-byte aligned");

  // Tensor maps: one per weight matrix of every layer and one over the
  // whole pool; kept for the next call with the same pointers.
  static std::mutex mu;
  static pkv::LayersMaps cached;
  static std::string cached_key;
  std::string key(reinterpret_cast<const char*>(layers), sizeof(pkv_layer_weights) * num_layers);
  key.append(reinterpret_cast<const char*>(&kv_pool), sizeof(kv_pool));
  key.append(reinterpret_cast<const char*>(&num_slots), sizeof(num_slots));
  key.append(reinterpret_cast<const char*>(&num_layers), sizeof(num_layers));
  int dev = 0;
  cudaGetDevice(&dev);
  key.append(reinterpret_cast<const char*>(&dev), sizeof(dev));
  pkv::LayersMaps maps;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (key != cached_key) {
      for (int l = 0; l < num_layers; ++l) {
        const pkv_layer_weights& w = layers[l];
        if ((st = encode_rows(&cached.w[l][0], w.qkv_w, 2048, 1536, 1536, 128)) ||
            (st = encode_rows(&cached.w[l][1], w.o_w, 1536, 1536, 1536, 128)) ||
            (st = encode_rows(&cached.w[l][2], w.gate_up_w, 17920, 1536, 1536, 128)) ||
            (st = encode_rows(&cached.w[l][3], w.down_w, 1536, 8960, 8960, 128))) {
          cached_key.clear();
          return st;
        }
      }
      EncodeFn fn = encode_fn();
      if (!fn) {
        cached_key.clear();
        return fail(PKV_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
      }
      cuuint64_t dims[4] = {128, 2, static_cast<cuuint64_t>(num_slots),
                            static_cast<cuuint64_t>(2 * num_layers)};
      cuuint64_t strides[3] = {128 * 2, 2 * 128 * 2, static_cast<cuuint64_t>(num_slots) * 2 * 128 * 2};
      cuuint32_t box[4] = {64, 1, 16, 1};
      cuuint32_t es[4] = {1, 1, 1, 1};
      CUresult r = fn(&cached.pool, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, kv_pool, dims, strides,
                      box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) {
        cached_key.clear();
        return fail(PKV_ERR_DRIVER, "pool tensor map encode failed (%d)", (int)r);
      }
      cached_key = key;
    }
    maps = cached;
  }

  pkv::LayersParams p{};
  p.L = num_layers;
  p.M = rows;
  p.G = pl.grid;
  p.P = pl.partitions;
  p.min_blocks = pl.min_blocks;
  p.xslots = pl.xslots;
  p.nw = pl.nw;


  for (int l = 0; l < num_layers; ++l) {
    p.qkv_b[l] = static_cast<const __nv_bfloat16*>(layers[l].qkv_b);
    p.post_w[l] = static_cast<const __nv_bfloat16*>(layers[l].post_norm_w);
    p.in_w[l] = static_cast<const __nv_bfloat16*>(layers[l].in_norm_w);
  }
  p.h0 = static_cast<const __nv_bfloat16*>(h0);
  p.xs = static_cast<__nv_bfloat16*>(xs);
  p.m_out = static_cast<__nv_bfloat16*>(m_out);
  p.pool = static_cast<__nv_bfloat16*>(kv_pool);
  p.num_slots = num_slots;
  p.num_blocks = static_cast<int32_t>(num_slots / 16);
  p.tables = block_tables;
  p.pitch = table_pitch;
  p.rows = seq_rows;
  p.starts = starts;
  p.cos = static_cast<const __nv_bfloat16*>(rope_cos);
  p.sin = static_cast<const __nv_bfloat16*>(rope_sin);
  p.rope_rows = rope_rows;
  p.eps = eps;
  // as pkv_paged_decode computes it from sm_scale = 1 / sqrt(128) (fa2.py:168)
  p.scale_log2 = static_cast<float>(1.0 / sqrt(128.0)) * 1.4426950408889634f;
  p.err = err_flag;
  pkv::carve_decode_layers(p, workspace, rows, sms, pl.partitions);
  return launch_status(
      pkv::launch_decode_layers(p, maps, pl, static_cast<cudaStream_t>(stream)), "decode_layers");
}

}  // extern "C"
