// C ABI of liblbq.so (declared in include/lbq.h): argument validation, tensor-map encoding and
// launches. Nothing here allocates device memory or synchronises, except lbq_device_status().
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../include/lbq.h"
#include "lbq_kernels.h"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}
int cuda_fail(cudaError_t e, const char* what) {
  return fail(LBQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// Checks a [B, L, H, 128] bf16 activation: non-null, 16-byte aligned base and strides.
int check_act(const char* name, const void* p, int64_t sb, int64_t sl, int64_t sh) {
  if (p == nullptr) return fail(LBQ_ERR_ARG, "%s is null", name);
  if (!aligned16(p)) return fail(LBQ_ERR_ALIGN, "%s is not 16-byte aligned", name);
  if (sb % 8 || sl % 8 || sh % 8 || sb < 0 || sl < 0 || sh < 0)
    return fail(LBQ_ERR_ALIGN, "%s strides (%lld, %lld, %lld) must be non-negative multiples of 8 elements",
                name, (long long)sb, (long long)sl, (long long)sh);
  return LBQ_OK;
}
int check_ptr(const char* name, const void* p) {
  if (p == nullptr) return fail(LBQ_ERR_ARG, "%s is null", name);
  if (!aligned16(p)) return fail(LBQ_ERR_ALIGN, "%s is not 16-byte aligned", name);
  return LBQ_OK;
}
// Checks a ring layout (len == 0: none) over a buffer whose logical window is `window` tokens.
int check_ring(int64_t sink, int64_t len, int64_t head, int64_t window) {
  if (len == 0) return (sink == 0 && head == 0) ? LBQ_OK : fail(LBQ_ERR_ARG, "ring_sink / ring_head without ring_len");
  if (sink < 0 || len < 0 || head < 0 || head >= len)
    return fail(LBQ_ERR_ARG, "ring (sink %lld, len %lld, head %lld) invalid", (long long)sink, (long long)len,
                (long long)head);
  if (window > sink + len)
    return fail(LBQ_ERR_ARG, "window of %lld tokens exceeds the ring's sink %lld + %lld", (long long)window,
                (long long)sink, (long long)len);
  return LBQ_OK;
}
// Checks a pair of [B, L, 64] float64 RoPE tables (cos, sin): both or neither given, 16-byte aligned,
// strides even (so a thread's 4 angles load as two double2).
int check_rope(const double* cs, const double* sn, int64_t sr_b, int64_t sr_l) {
  if ((cs == nullptr) != (sn == nullptr)) return fail(LBQ_ERR_ARG, "rope_cos and rope_sin: give both or neither");
  if (cs == nullptr) return LBQ_OK;
  if (!aligned16(cs) || !aligned16(sn)) return fail(LBQ_ERR_ALIGN, "rope tables are not 16-byte aligned");
  if (sr_b % 2 || sr_l % 2 || sr_b < 0 || sr_l < 64)
    return fail(LBQ_ERR_ALIGN, "rope table strides (%lld, %lld) must be even, the token stride >= 64", (long long)sr_b,
                (long long)sr_l);
  return LBQ_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D uint8 tensor map with a 128 x 128 box and 128-byte swizzle.
int make_map(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
             uint64_t stride2, const char* name, uint32_t box_rows = 128) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(LBQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1, stride2};
  const cuuint32_t box[3] = {128, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LBQ_ERR_CUDA, "tensor map for %s: CUresult %d", name, int(r));
  return LBQ_OK;
}

}  // namespace

namespace lbq {
int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}
}  // namespace lbq

extern "C" {

int lbq_abi_version(void) { return 101; }

const char* lbq_last_error(void) { return g_err; }

int lbq_device_status(int clear, int* status_out) {
  int* p = lbq::device_status_ptr();
  if (p == nullptr) return fail(LBQ_ERR_CUDA, "device status word unavailable");
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read status");
  if (clear) {
    const int zero = 0;
    e = cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "clear status");
  }
  if (status_out) *status_out = v;
  return LBQ_OK;
}

// The entries below with a `dtype` argument (0: bf16, 1: fp16 activations) are the bodies of the
// public bf16 entries; lbq_quant_qkv passes the caller's dtype through them.
static int kv_block_stats_dt(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b,
                             int64_t sv_l, int64_t sv_h, int batch, int heads, int64_t kv_len, int blk_begin,
                             int blk_end, int64_t max_blocks, double* ksum, float* vamax, int dtype, lbq::Ring ring,
                             void* stream) {
  int r;
  if ((r = check_act("k", k, sk_b, sk_l, sk_h)) || (r = check_act("v", v, sv_b, sv_l, sv_h))) return r;
  if ((r = check_ptr("ksum", ksum)) || (r = check_ptr("vamax", vamax))) return r;
  if (batch <= 0 || heads <= 0 || kv_len <= 0) return fail(LBQ_ERR_ARG, "batch, heads and kv_len must be positive");
  if (blk_begin < 0 || blk_end > (kv_len + 63) / 64 || blk_end > max_blocks)
    return fail(LBQ_ERR_ARG, "block range [%d, %d) outside the window (%lld tokens, %lld table rows)", blk_begin,
                blk_end, (long long)kv_len, (long long)max_blocks);
  if (blk_end <= blk_begin) return LBQ_OK;
  lbq::KvBlockStatsArgs a{static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v),
                          sk_b, sk_l, sk_h, sv_b, sv_l, sv_h, batch, heads, kv_len, blk_begin, blk_end,
                          max_blocks, ksum, vamax, lbq::device_status_ptr(), dtype, ring};
  cudaError_t e = lbq::launch_kv_block_stats(a, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : cuda_fail(e, "kv_block_stats launch");
}

int lbq_kv_block_stats(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b,
                       int64_t sv_l, int64_t sv_h, int batch, int heads, int64_t kv_len, int blk_begin, int blk_end,
                       int64_t max_blocks, double* ksum, float* vamax, int64_t ring_sink, int64_t ring_len,
                       int64_t ring_head, void* stream) {
  int r;
  if ((r = check_ring(ring_sink, ring_len, ring_head, kv_len))) return r;
  return kv_block_stats_dt(k, sk_b, sk_l, sk_h, v, sv_b, sv_l, sv_h, batch, heads, kv_len, blk_begin, blk_end,
                           max_blocks, ksum, vamax, 0, lbq::Ring{ring_sink, ring_len, ring_head}, stream);
}

int lbq_kv_window_sums(const double* ksum, const float* vamax, int batch, int heads, int blk_begin, int blk_end,
                       int64_t max_blocks, double* ksum_total, float* vamax_total, void* stream) {
  int r;
  if ((r = check_ptr("ksum", ksum)) || (r = check_ptr("vamax", vamax)) || (r = check_ptr("ksum_total", ksum_total)) ||
      (r = check_ptr("vamax_total", vamax_total)))
    return r;
  if (batch <= 0 || heads <= 0) return fail(LBQ_ERR_ARG, "batch and heads must be positive");
  if (blk_begin < 0 || blk_end < blk_begin || blk_end > max_blocks)
    return fail(LBQ_ERR_ARG, "block range [%d, %d) invalid for %lld table rows", blk_begin, blk_end,
                (long long)max_blocks);
  lbq::KvWindowSumsArgs a{ksum, vamax, batch, heads, blk_begin, blk_end, max_blocks, ksum_total, vamax_total};
  cudaError_t e = lbq::launch_kv_window_sums(a, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : cuda_fail(e, "kv_window_sums launch");
}

static int quant_q_dt(const void* q, int64_t sq_b, int64_t sq_l, int64_t sq_h, int batch, int heads, int q_len,
                      int8_t* q_codes, float* q_scale, int dtype, void* stream) {
  int r;
  if ((r = check_act("q", q, sq_b, sq_l, sq_h)) || (r = check_ptr("q_codes", q_codes)) ||
      (r = check_ptr("q_scale", q_scale)))
    return r;
  if (batch <= 0 || heads <= 0 || q_len <= 0) return fail(LBQ_ERR_ARG, "batch, heads and q_len must be positive");
  lbq::QuantQArgs a{static_cast<const __nv_bfloat16*>(q), sq_b, sq_l, sq_h, batch, heads, q_len,
                    int(round_up(q_len, 128)), q_codes, q_scale, nullptr, nullptr, 0, 0, dtype};
  cudaError_t e = lbq::launch_quant_q(a, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : cuda_fail(e, "quant_q launch");
}

int lbq_quant_q(const void* q, int64_t sq_b, int64_t sq_l, int64_t sq_h, int batch, int heads, int q_len,
                int8_t* q_codes, float* q_scale, void* stream) {
  return quant_q_dt(q, sq_b, sq_l, sq_h, batch, heads, q_len, q_codes, q_scale, 0, stream);
}

int lbq_rope_quant_q(const void* q, int64_t sq_b, int64_t sq_l, int64_t sq_h, const double* rope_cos,
                     const double* rope_sin, int64_t sr_b, int64_t sr_l, int batch, int heads, int q_len,
                     int8_t* q_codes, float* q_scale, void* stream) {
  int r;
  if ((r = check_act("q", q, sq_b, sq_l, sq_h)) || (r = check_ptr("q_codes", q_codes)) ||
      (r = check_ptr("q_scale", q_scale)) || (r = check_rope(rope_cos, rope_sin, sr_b, sr_l)))
    return r;
  if (rope_cos == nullptr) return fail(LBQ_ERR_ARG, "rope tables are null (use lbq_quant_q for unroped Q)");
  if (batch <= 0 || heads <= 0 || q_len <= 0) return fail(LBQ_ERR_ARG, "batch, heads and q_len must be positive");
  lbq::QuantQArgs a{static_cast<const __nv_bfloat16*>(q), sq_b, sq_l, sq_h, batch, heads, q_len,
                    int(round_up(q_len, 128)), q_codes, q_scale, rope_cos, rope_sin, sr_b, sr_l};
  cudaError_t e = lbq::launch_quant_q(a, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : cuda_fail(e, "rope_quant_q launch");
}

int lbq_cache_write(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b,
                    int64_t sv_l, int64_t sv_h, const double* rope_cos, const double* rope_sin, int64_t sr_b,
                    int64_t sr_l, void* k_cache, int64_t ck_b, int64_t ck_l, int64_t ck_h, void* v_cache,
                    int64_t cv_b, int64_t cv_l, int64_t cv_h, int batch, int heads, int64_t kv_size,
                    int64_t tok_begin, int64_t n_tokens, int64_t max_blocks, double* ksum, float* vamax,
                    int64_t ring_sink, int64_t ring_len, int64_t ring_head, void* stream) {
  int r;
  if ((r = check_ring(ring_sink, ring_len, ring_head, tok_begin + n_tokens))) return r;
  if (ring_len && ring_sink + ring_len > kv_size)
    return fail(LBQ_ERR_ARG, "ring of %lld rows after a %lld-token sink exceeds the %lld-token cache", (long long)ring_len,
                (long long)ring_sink, (long long)kv_size);
  if ((r = check_act("k", k, sk_b, sk_l, sk_h)) || (r = check_act("v", v, sv_b, sv_l, sv_h)) ||
      (r = check_act("k_cache", k_cache, ck_b, ck_l, ck_h)) || (r = check_act("v_cache", v_cache, cv_b, cv_l, cv_h)) ||
      (r = check_ptr("ksum", ksum)) || (r = check_ptr("vamax", vamax)) ||
      (r = check_rope(rope_cos, rope_sin, sr_b, sr_l)))
    return r;
  if (batch <= 0 || heads <= 0 || batch > 65535 || heads > 65535)
    return fail(LBQ_ERR_ARG, "batch %d / heads %d out of range (1..65535)", batch, heads);
  if (n_tokens < 0 || tok_begin < 0 || tok_begin + n_tokens > kv_size)
    return fail(LBQ_ERR_ARG, "tokens [%lld, %lld) outside the %lld-token cache", (long long)tok_begin,
                (long long)(tok_begin + n_tokens), (long long)kv_size);
  if (max_blocks < (kv_size + 63) / 64)
    return fail(LBQ_ERR_ARG, "%lld stats rows for a %lld-token cache", (long long)max_blocks, (long long)kv_size);
  if (n_tokens == 0) return LBQ_OK;
  lbq::CacheWriteArgs a{static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v), sk_b, sk_l, sk_h,
                        sv_b, sv_l, sv_h, static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache),
                        ck_b, ck_l, ck_h, cv_b, cv_l, cv_h, rope_cos, rope_sin, sr_b, sr_l, batch, heads, tok_begin,
                        tok_begin + n_tokens, int(tok_begin / 64), max_blocks, ksum, vamax, lbq::device_status_ptr(),
                        lbq::Ring{ring_sink, ring_len, ring_head}};
  cudaError_t e = lbq::launch_cache_write(a, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : cuda_fail(e, "cache_write launch");
}

static int quant_kv_tiles_dt(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b,
                             int64_t sv_l, int64_t sv_h, int batch, int heads, int64_t tok0, int seg, int num_segments,
                             int seg_valid, int seg_len, int64_t kv_len_total, const double* ksum_total,
                             const float* vamax_total, int8_t* k_codes, float* k_scale, uint8_t* vt_codes,
                             void* km_out, float* v_scale, int write_totals, int tile_begin, int tile_end, int dtype,
                             lbq::Ring ring, void* stream) {
  int r;
  if ((r = check_act("k", k, sk_b, sk_l, sk_h)) || (r = check_act("v", v, sv_b, sv_l, sv_h))) return r;
  if ((r = check_ptr("ksum_total", ksum_total)) || (r = check_ptr("vamax_total", vamax_total)) ||
      (r = check_ptr("k_codes", k_codes)) || (r = check_ptr("k_scale", k_scale)) || (r = check_ptr("vt_codes", vt_codes)))
    return r;
  if (write_totals && (r = check_ptr("v_scale", v_scale))) return r;
  if (batch <= 0 || heads <= 0 || seg_len <= 0 || kv_len_total <= 0 || num_segments <= 0)
    return fail(LBQ_ERR_ARG, "batch, heads, seg_len, kv_len and num_segments must be positive");
  if (seg < 0 || seg >= num_segments) return fail(LBQ_ERR_ARG, "segment %d of %d", seg, num_segments);
  if (seg_len % 64 && num_segments > 1)
    return fail(LBQ_ERR_ARG, "seg_len %d must be a multiple of 64 so K blocks match the whole window's", seg_len);
  if (seg_valid <= 0 || seg_valid > seg_len) return fail(LBQ_ERR_ARG, "seg_valid %d not in (0, %d]", seg_valid, seg_len);
  if (tile_begin < 0 || tile_end < tile_begin || tile_end > (seg_valid + 127) / 128)
    return fail(LBQ_ERR_ARG, "tiles [%d, %d) outside the %d tiles holding valid tokens", tile_begin, tile_end,
                (seg_valid + 127) / 128);
  if (tile_end > tile_begin && tok0 + int64_t(tile_begin) * 128 < 0)
    return fail(LBQ_ERR_ARG, "tile %d maps to source token %lld < 0", tile_begin,
                (long long)(tok0 + int64_t(tile_begin) * 128));
  const int seg_pad = int(round_up(seg_len, 128));
  lbq::QuantKArgs ka{static_cast<const __nv_bfloat16*>(k), sk_b, sk_l, sk_h, batch, heads, tok0, seg, seg_valid,
                     seg_pad, kv_len_total, ksum_total, k_codes, k_scale,
                     static_cast<__nv_bfloat16*>(km_out), write_totals, lbq::device_status_ptr(), dtype, ring};
  lbq::QuantVArgs va{static_cast<const __nv_bfloat16*>(v), sv_b, sv_l, sv_h, batch, heads, tok0, seg, seg_valid,
                     seg_pad, vamax_total, vt_codes, v_scale, write_totals, lbq::device_status_ptr(), dtype, ring};
  cudaError_t e = lbq::launch_quant_kv(ka, va, tile_begin, tile_end - tile_begin, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : cuda_fail(e, "quant_kv launch");
}

int lbq_quant_kv_tiles(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b,
                       int64_t sv_l, int64_t sv_h, int batch, int heads, int64_t tok0, int seg, int num_segments,
                       int seg_valid, int seg_len, int64_t kv_len_total, const double* ksum_total,
                       const float* vamax_total, int8_t* k_codes, float* k_scale, uint8_t* vt_codes, void* km_out,
                       float* v_scale, int write_totals, int tile_begin, int tile_end, void* stream) {
  return quant_kv_tiles_dt(k, sk_b, sk_l, sk_h, v, sv_b, sv_l, sv_h, batch, heads, tok0, seg, num_segments, seg_valid,
                           seg_len, kv_len_total, ksum_total, vamax_total, k_codes, k_scale, vt_codes, km_out,
                           v_scale, write_totals, tile_begin, tile_end, 0, lbq::Ring{0, 0, 0}, stream);
}

int lbq_quant_kv(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b, int64_t sv_l,
                 int64_t sv_h, int batch, int heads, int64_t tok0, int seg, int num_segments, int seg_valid,
                 int seg_len, int64_t kv_len_total, const double* ksum_total, const float* vamax_total,
                 int8_t* k_codes, float* k_scale, uint8_t* vt_codes, void* km_out, float* v_scale, int write_totals,
                 void* stream) {
  if (tok0 < 0) return fail(LBQ_ERR_ARG, "tok0 must be >= 0");
  return lbq_quant_kv_tiles(k, sk_b, sk_l, sk_h, v, sv_b, sv_l, sv_h, batch, heads, tok0, seg, num_segments,
                            seg_valid, seg_len, kv_len_total, ksum_total, vamax_total, k_codes, k_scale, vt_codes,
                            km_out, v_scale, write_totals, 0, seg_valid > 0 ? (seg_valid + 127) / 128 : 0, stream);
}

size_t lbq_quant_qkv_workspace(int batch, int heads, int64_t kv_len) {
  // SIZE_MAX for arguments no launch accepts (batch and heads index grid dimensions of at most 65535,
  // kv_len at most 2^30) or a size that does not fit: every capacity check then rejects the call.
  if (batch <= 0 || heads <= 0 || batch > 65535 || heads > 65535 || kv_len <= 0 || kv_len > (int64_t(1) << 30))
    return SIZE_MAX;
  const uint64_t nblk = uint64_t(kv_len + 63) / 64;
  uint64_t cols, per_col, bytes;
  if (__builtin_mul_overflow(uint64_t(batch) * uint64_t(heads), uint64_t(128), &cols) ||
      __builtin_mul_overflow(nblk + 1, uint64_t(8 + 4), &per_col) || __builtin_mul_overflow(cols, per_col, &bytes) ||
      __builtin_add_overflow(bytes, uint64_t(64), &bytes) || bytes > uint64_t(SIZE_MAX))
    return SIZE_MAX;
  return size_t(bytes);
}

int lbq_quant_qkv(const void* q, int64_t sq_b, int64_t sq_l, int64_t sq_h, int q_len, const void* k, int64_t sk_b,
                  int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b, int64_t sv_l, int64_t sv_h, int64_t kv_len,
                  int batch, int heads, int8_t* q_codes, float* q_scale, int8_t* k_codes, float* k_scale,
                  uint8_t* vt_codes, float* v_scale, void* km_out, void* workspace, size_t workspace_bytes,
                  int dtype, void* stream) {
  if (dtype != LBQ_DTYPE_BF16 && dtype != LBQ_DTYPE_F16) return fail(LBQ_ERR_ARG, "dtype %d is neither bf16 nor fp16", dtype);
  if (kv_len <= 0 || kv_len > (int64_t(1) << 30)) return fail(LBQ_ERR_ARG, "kv_len %lld out of range", (long long)kv_len);
  if (batch <= 0 || heads <= 0 || batch > 65535 || heads > 65535)
    return fail(LBQ_ERR_ARG, "batch %d / heads %d out of range (1..65535)", batch, heads);
  if (workspace == nullptr || workspace_bytes < lbq_quant_qkv_workspace(batch, heads, kv_len))
    return fail(LBQ_ERR_ARG, "workspace of %zu bytes is smaller than the %zu needed", workspace_bytes,
                lbq_quant_qkv_workspace(batch, heads, kv_len));
  if (!aligned16(workspace)) return fail(LBQ_ERR_ALIGN, "workspace is not 16-byte aligned");
  const int nblk = int((kv_len + 63) / 64);
  const int64_t cols = int64_t(batch) * heads * 128;
  double* ksum = static_cast<double*>(workspace);
  double* ksum_total = ksum + int64_t(nblk) * cols;
  float* vamax = reinterpret_cast<float*>(ksum_total + cols);
  float* vamax_total = vamax + int64_t(nblk) * cols;
  int r = kv_block_stats_dt(k, sk_b, sk_l, sk_h, v, sv_b, sv_l, sv_h, batch, heads, kv_len, 0, nblk, nblk, ksum,
                            vamax, dtype, lbq::Ring{0, 0, 0}, stream);
  if (r) return r;
  if ((r = lbq_kv_window_sums(ksum, vamax, batch, heads, 0, nblk, nblk, ksum_total, vamax_total, stream))) return r;
  if ((r = quant_q_dt(q, sq_b, sq_l, sq_h, batch, heads, q_len, q_codes, q_scale, dtype, stream))) return r;
  return quant_kv_tiles_dt(k, sk_b, sk_l, sk_h, v, sv_b, sv_l, sv_h, batch, heads, 0, 0, 1, int(kv_len), int(kv_len),
                           kv_len, ksum_total, vamax_total, k_codes, k_scale, vt_codes, km_out, v_scale, 1, 0,
                           int((kv_len + 127) / 128), dtype, lbq::Ring{0, 0, 0}, stream);
}

int lbq_requant_cache(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b,
                      int64_t sv_l, int64_t sv_h, int batch, int heads, int64_t kv_len, int64_t max_blocks,
                      const double* ksum, const float* vamax, void* sums_ws, int8_t* k_codes, float* k_scale,
                      uint8_t* vt_codes, float* v_scale, void* km_out, int64_t ring_sink, int64_t ring_len,
                      int64_t ring_head, void* stream) {
  int r;
  if ((r = check_ptr("sums_ws", sums_ws)) || (r = check_ring(ring_sink, ring_len, ring_head, kv_len))) return r;
  if (kv_len <= 0 || kv_len > (int64_t(1) << 30)) return fail(LBQ_ERR_ARG, "kv_len %lld out of range", (long long)kv_len);
  const int nblk = int((kv_len + 63) / 64);
  if (nblk > max_blocks) return fail(LBQ_ERR_ARG, "kv_len %lld needs %d stats rows, table has %lld", (long long)kv_len,
                                     nblk, (long long)max_blocks);
  const int64_t cols = int64_t(batch) * heads * 128;
  double* ksum_total = static_cast<double*>(sums_ws);
  float* vamax_total = reinterpret_cast<float*>(ksum_total + cols);
  if ((r = lbq_kv_window_sums(ksum, vamax, batch, heads, 0, nblk, max_blocks, ksum_total, vamax_total, stream))) return r;
  return quant_kv_tiles_dt(k, sk_b, sk_l, sk_h, v, sv_b, sv_l, sv_h, batch, heads, 0, 0, 1, int(kv_len), int(kv_len),
                           kv_len, ksum_total, vamax_total, k_codes, k_scale, vt_codes, km_out, v_scale, 1, 0,
                           int((kv_len + 127) / 128), 0, lbq::Ring{ring_sink, ring_len, ring_head}, stream);
}

int lbq_attn_fwd(const int8_t* q_codes, const float* q_scale, int q_len, const int8_t* k_codes, const float* k_scale,
                 const uint8_t* vt_codes, const float* v_scale, int64_t kv_len, int num_segments, int seg_len,
                 int batch, int heads, float sm_scale, int is_causal, void* out, int64_t so_b, int64_t so_l,
                 int64_t so_h, int num_splits, float* o_part, float* ml_part, int* splits_used, int dtype,
                 void* stream) {
  int r;
  if (is_causal)
    return fail(LBQ_ERR_UNSUPPORTED,
                "causal attention is not implemented by the quantized kernel (the drop-in attention() routes "
                "causal calls to the reference's non-Sage branch)");
  if (dtype != LBQ_DTYPE_BF16 && dtype != LBQ_DTYPE_F16) return fail(LBQ_ERR_ARG, "dtype %d is neither bf16 nor fp16", dtype);
  if ((r = check_ptr("q_codes", q_codes)) || (r = check_ptr("q_scale", q_scale)) || (r = check_ptr("k_codes", k_codes)) ||
      (r = check_ptr("k_scale", k_scale)) || (r = check_ptr("vt_codes", vt_codes)) || (r = check_ptr("v_scale", v_scale)))
    return r;
  if ((r = check_act("out", out, so_b, so_l, so_h))) return r;
  if (batch <= 0 || heads <= 0 || q_len <= 0 || kv_len <= 0 || num_segments <= 0 || seg_len <= 0)
    return fail(LBQ_ERR_ARG, "batch, heads, q_len, kv_len, num_segments and seg_len must be positive");
  if (int64_t(num_segments) * seg_len < kv_len || int64_t(num_segments - 1) * seg_len >= kv_len)
    return fail(LBQ_ERR_ARG, "%d segments of %d tokens do not cover exactly %lld tokens", num_segments, seg_len,
                (long long)kv_len);
  if (num_segments > 1 && seg_len % 64)
    return fail(LBQ_ERR_ARG, "seg_len %d must be a multiple of 64 with several segments", seg_len);
  if (kv_len > (int64_t(1) << 30) || q_len > (1 << 30)) return fail(LBQ_ERR_ARG, "length too large");
  if (int64_t(batch) * heads * num_segments > 65535 * 32) return fail(LBQ_ERR_ARG, "too many batch*heads*segments");
  const int q_pad = int(round_up(q_len, 128));
  const int seg_pad = int(round_up(seg_len, 128));
  const int tiles_per_seg = seg_pad / 128;
  const int last_valid = int(kv_len - int64_t(num_segments - 1) * seg_len);
  const int total_tiles = (num_segments - 1) * tiles_per_seg + (last_valid + 127) / 128;
  if (num_splits < 1) num_splits = 1;
  if (num_splits > total_tiles) num_splits = total_tiles;
  int tiles_per_split = (total_tiles + num_splits - 1) / num_splits;
  num_splits = (total_tiles + tiles_per_split - 1) / tiles_per_split;
  if (num_splits > 1) {
    if ((r = check_ptr("o_part", o_part)) || (r = check_ptr("ml_part", ml_part))) return r;
  }
  if (num_splits > 65535) return fail(LBQ_ERR_ARG, "too many splits");
  if (splits_used) *splits_used = num_splits;
  const uint64_t bhs = uint64_t(batch) * heads;
  CUtensorMap tq, tk, tv;
  if ((r = make_map(&tq, q_codes, 128, q_pad, bhs, 128, uint64_t(q_pad) * 128, "q_codes"))) return r;
  if ((r = make_map(&tk, k_codes, 128, seg_pad, bhs * num_segments, 128, uint64_t(seg_pad) * 128, "k_codes"))) return r;
  if ((r = make_map(&tv, vt_codes, seg_pad, 128, bhs * num_segments, seg_pad, uint64_t(seg_pad) * 128, "vt_codes")))
    return r;
  if (sm_scale <= 0.f) sm_scale = 0.08838834764831845f;   // 128 ** -0.5
  lbq::AttnArgs a{};
  a.dtype = dtype;
  a.wide_out = (reinterpret_cast<uintptr_t>(out) % 32 == 0) && so_b % 16 == 0 && so_l % 16 == 0 && so_h % 16 == 0;
  a.wide_part = o_part != nullptr && reinterpret_cast<uintptr_t>(o_part) % 32 == 0;
  a.q_scale = q_scale;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.so_b = so_b;
  a.so_l = so_l;
  a.so_h = so_h;
  a.o_part = o_part;
  a.ml_part = reinterpret_cast<float2*>(ml_part);
  a.batch = batch;
  a.heads = heads;
  a.q_len = q_len;
  a.q_pad = q_pad;
  a.kv_len = int(kv_len);
  a.nseg = num_segments;
  a.seg_len = seg_len;
  a.seg_pad = seg_pad;
  a.num_splits = num_splits;
  a.tiles_per_split = tiles_per_split;
  a.total_tiles = total_tiles;
  a.sm_log2 = sm_scale * 1.4426950408889634f;
  a.status = lbq::device_status_ptr();
  cudaError_t e = lbq::launch_attn(a, tq, tk, tv, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : cuda_fail(e, "attn_fwd launch");
}

int lbq_fp8_quant_rows(const void* x, int64_t sx, int dtype, int rows, int cols, uint8_t* q, int64_t sq,
                       float* scale, void* stream) {
  int r;
  if ((r = check_ptr("x", x)) || (r = check_ptr("q", q)) || (r = check_ptr("scale", scale))) return r;
  if (dtype < 0 || dtype > 2) return fail(LBQ_ERR_ARG, "dtype %d is not bf16 (0), fp16 (1) or fp32 (2)", dtype);
  if (rows < 0 || cols <= 0 || cols % 16) return fail(LBQ_ERR_ARG, "cols %d must be a positive multiple of 16", cols);
  const int esize = dtype == 2 ? 4 : 2;
  if ((sx * esize) % 16 || sq % 16 || sx < cols || sq < cols)
    return fail(LBQ_ERR_ALIGN, "row strides (%lld elements, %lld bytes) must cover a row and be 16-byte multiples",
                (long long)sx, (long long)sq);
  if (rows == 0) return LBQ_OK;
  lbq::Fp8QuantArgs a{x, sx, esize, dtype, rows, cols, q, sq, scale};
  cudaError_t e = lbq::launch_fp8_quant_rows(a, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : cuda_fail(e, "fp8_quant_rows launch");
}

int lbq_fp8_gemm(const uint8_t* a, int64_t sa, const float* a_scale, const uint8_t* w, int64_t sw,
                 const float* w_scale, const void* bias, int M, int N, int K, void* y, int64_t sy, int num_ctas,
                 void* stream) {
  int r;
  if ((r = check_ptr("a", a)) || (r = check_ptr("a_scale", a_scale)) || (r = check_ptr("w", w)) ||
      (r = check_ptr("w_scale", w_scale)) || (r = check_ptr("y", y)))
    return r;
  if (bias != nullptr && !aligned16(bias)) return fail(LBQ_ERR_ALIGN, "bias is not 16-byte aligned");
  if (M <= 0 || N <= 0 || K <= 0 || N % 32 || K % 16)
    return fail(LBQ_ERR_ARG, "M %d, N %d, K %d: N must be a multiple of 32 and K of 16", M, N, K);
  if (sa % 16 || sw % 16 || sa < K || sw < K || sy % 8 || sy < N)
    return fail(LBQ_ERR_ALIGN, "row strides (a %lld, w %lld bytes; y %lld elements) must cover a row and be 16-byte "
                "multiples", (long long)sa, (long long)sw, (long long)sy);
  CUtensorMap ta, tb;
  if ((r = make_map(&ta, a, uint64_t(K), uint64_t(M), 1, uint64_t(sa), uint64_t(sa) * M, "a", 128))) return r;
  if ((r = make_map(&tb, w, uint64_t(K), uint64_t(N), 1, uint64_t(sw), uint64_t(sw) * N, "w", 256))) return r;
  lbq::Fp8GemmArgs g{};
  g.x_scale = a_scale;
  g.w_scale = w_scale;
  g.bias = static_cast<const __nv_bfloat16*>(bias);
  g.y = static_cast<__nv_bfloat16*>(y);
  g.sy = sy;
  g.M = M;
  g.N = N;
  g.K = K;
  g.tiles_m = (M + 127) / 128;
  g.tiles_n = (N + 255) / 256;
  g.status = lbq::device_status_ptr();
  g.wide_stores = (sy % 16 == 0) && (reinterpret_cast<uintptr_t>(y) % 32 == 0);
  const int tiles = g.tiles_m * g.tiles_n;
  if (num_ctas <= 0) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    num_ctas = sms;
  }
  if (num_ctas > tiles) num_ctas = tiles;
  cudaError_t e = lbq::launch_fp8_gemm(g, ta, tb, num_ctas, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : cuda_fail(e, "fp8_gemm launch");
}

int lbq_splitkv_combine(const float* o_part, const float* ml_part, int num_splits, const float* v_scale, int batch,
                        int heads, int q_len, void* out, int64_t so_b, int64_t so_l, int64_t so_h, int dtype,
                        void* stream) {
  int r;
  if (dtype != LBQ_DTYPE_BF16 && dtype != LBQ_DTYPE_F16) return fail(LBQ_ERR_ARG, "dtype %d is neither bf16 nor fp16", dtype);
  if ((r = check_ptr("o_part", o_part)) || (r = check_ptr("ml_part", ml_part)) || (r = check_ptr("v_scale", v_scale)))
    return r;
  if ((r = check_act("out", out, so_b, so_l, so_h))) return r;
  if (num_splits < 1 || batch <= 0 || heads <= 0 || q_len <= 0)
    return fail(LBQ_ERR_ARG, "num_splits, batch, heads and q_len must be positive");
  lbq::CombineArgs a{o_part, reinterpret_cast<const float2*>(ml_part), v_scale, static_cast<__nv_bfloat16*>(out),
                     so_b, so_l, so_h, batch, heads, q_len, int(round_up(q_len, 128)), num_splits, dtype};
  cudaError_t e = lbq::launch_combine(a, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : cuda_fail(e, "splitkv_combine launch");
}

int lbq_attn_fwd_keys(const int8_t* q_codes, const float* q_scale, int q_len, int q_pad, const int8_t* k_codes,
                      const float* k_scale, const uint8_t* vt_codes, int num_segments, int seg_len, int batch,
                      int heads, float sm_scale, const int* range_lt0, const int* range_tiles, const int* range_valid,
                      const uint64_t* peers, int nranks, int rank, int64_t xchg_off, int part, int64_t recv_o_off,
                      int64_t recv_ml_off, void* stream) {
  int r;
  if ((r = check_ptr("q_codes", q_codes)) || (r = check_ptr("q_scale", q_scale)) || (r = check_ptr("k_codes", k_codes)) ||
      (r = check_ptr("k_scale", k_scale)) || (r = check_ptr("vt_codes", vt_codes)))
    return r;
  if (!range_lt0 || !range_tiles || !range_valid) return fail(LBQ_ERR_ARG, "key ranges are null");
  if (peers == nullptr) return fail(LBQ_ERR_ARG, "peers table is null");
  if (nranks < 1 || nranks > lbq::xchg::kMaxRanks || rank < 0 || rank >= nranks)
    return fail(LBQ_ERR_ARG, "rank %d of %d ranks (at most %d)", rank, nranks, lbq::xchg::kMaxRanks);
  if (xchg_off < 0 || xchg_off % 256 || recv_o_off < 0 || recv_o_off % 16 || recv_ml_off < 0 || recv_ml_off % 16)
    return fail(LBQ_ERR_ALIGN, "xchg_off must be a multiple of 256 and the receive offsets of 16 bytes");
  if (batch <= 0 || heads <= 0 || q_len <= 0 || seg_len <= 0) return fail(LBQ_ERR_ARG, "batch, heads, q_len and seg_len must be positive");
  if (num_segments < 1 || num_segments > 2) return fail(LBQ_ERR_ARG, "num_segments %d not in [1, 2]", num_segments);
  if (num_segments > 1 && seg_len % 64)
    return fail(LBQ_ERR_ARG, "seg_len %d must be a multiple of 64 with several segments", seg_len);
  if (q_pad % 128 || q_pad < q_len || q_pad > (1 << 30)) return fail(LBQ_ERR_ARG, "q_pad %d must be a multiple of 128 >= q_len %d", q_pad, q_len);
  if (part <= 0 || part % 128 || int64_t(part) * nranks < q_len)
    return fail(LBQ_ERR_ARG, "part %d must be a multiple of 128 with part * nranks >= q_len", part);
  if (int64_t(batch) * heads * num_segments > 65535 * 32) return fail(LBQ_ERR_ARG, "too many batch*heads*segments");
  const int seg_pad = int(round_up(seg_len, 128));
  lbq::AttnArgs a{};
  int tiles = 0;
  a.range_tile0[0] = 0;
  for (int s = 0; s < num_segments; ++s) {
    if (range_valid[s] <= 0 || range_valid[s] > seg_len)
      return fail(LBQ_ERR_ARG, "range %d: %d valid keys, segment of %d", s, range_valid[s], seg_len);
    if (range_lt0[s] < 0 || range_tiles[s] < 0 || range_lt0[s] + range_tiles[s] > (range_valid[s] + 127) / 128)
      return fail(LBQ_ERR_ARG, "range %d: tiles [%d, %d) outside the %d tiles holding valid keys", s, range_lt0[s],
                  range_lt0[s] + range_tiles[s], (range_valid[s] + 127) / 128);
    a.range_valid[s] = range_valid[s];
    a.range_lt0[s] = range_lt0[s];
    tiles += range_tiles[s];
    a.range_tile0[s + 1] = tiles;
  }
  for (int s = num_segments; s < 2; ++s) {
    a.range_valid[s] = 0;
    a.range_lt0[s] = 0;
    a.range_tile0[s + 1] = tiles;
  }
  if (tiles <= 0) return fail(LBQ_ERR_ARG, "empty key range: every rank needs at least one key tile");
  const uint64_t bhs = uint64_t(batch) * heads;
  CUtensorMap tq, tk, tv;
  if ((r = make_map(&tq, q_codes, 128, q_pad, bhs, 128, uint64_t(q_pad) * 128, "q_codes"))) return r;
  if ((r = make_map(&tk, k_codes, 128, seg_pad, bhs * num_segments, 128, uint64_t(seg_pad) * 128, "k_codes"))) return r;
  if ((r = make_map(&tv, vt_codes, seg_pad, 128, bhs * num_segments, seg_pad, uint64_t(seg_pad) * 128, "vt_codes")))
    return r;
  if (sm_scale <= 0.f) sm_scale = 0.08838834764831845f;   // 128 ** -0.5
  a.q_scale = q_scale;
  a.k_scale = k_scale;
  a.batch = batch;
  a.heads = heads;
  a.q_len = q_len;
  a.q_pad = q_pad;
  a.kv_len = 0;                 // unused: the ranges carry the valid lengths
  a.nseg = num_segments;
  a.seg_len = seg_len;
  a.seg_pad = seg_pad;
  a.num_splits = 1;
  a.tiles_per_split = tiles;
  a.total_tiles = tiles;
  a.sm_log2 = sm_scale * 1.4426950408889634f;
  a.status = lbq::device_status_ptr();
  a.peers = peers;
  a.nranks = nranks;
  a.rank = rank;
  a.part = part;
  a.xchg_off = xchg_off;
  a.recv_o_off = recv_o_off;
  a.recv_ml_off = recv_ml_off;
  cudaError_t e = lbq::launch_attn_keys(a, tq, tk, tv, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : cuda_fail(e, "attn_fwd (key range) launch");
}

int lbq_keys_combine(const void* recv_o, const float* recv_ml, int nranks, int part, int rows, const float* v_scale,
                     int batch, int heads, void* out, int64_t so_b, int64_t so_l, int64_t so_h, void* stream) {
  int r;
  if (nranks < 1 || nranks > lbq::xchg::kMaxRanks || batch <= 0 || heads <= 0 || rows < 0 || part <= 0 || rows > part)
    return fail(LBQ_ERR_ARG, "nranks %d, batch %d, heads %d, rows %d, part %d out of range", nranks, batch, heads,
                rows, part);
  if (rows == 0) return LBQ_OK;               // an empty query slice: nothing to merge (out may be empty)
  if ((r = check_ptr("recv_o", recv_o)) || (r = check_ptr("recv_ml", recv_ml)) || (r = check_ptr("v_scale", v_scale)))
    return r;
  if ((r = check_act("out", out, so_b, so_l, so_h))) return r;
  lbq::KeysCombineArgs a{static_cast<const __half*>(recv_o), reinterpret_cast<const float2*>(recv_ml), v_scale,
                         static_cast<__nv_bfloat16*>(out), so_b, so_l, so_h, batch, heads, rows, part, nranks};
  cudaError_t e = lbq::launch_keys_combine(a, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : cuda_fail(e, "keys_combine launch");
}

}  // extern "C"
