// Argument blocks and launchers shared between the kernels and the C-ABI layer (internal header).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace lbq {

struct KvBlockStatsArgs {
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t sk_b, sk_l, sk_h;   // element strides of K ([B, L, H, 128], channel stride 1)
  int64_t sv_b, sv_l, sv_h;
  int batch, heads;
  int64_t kv_len;             // valid tokens in the buffer
  int blk_begin, blk_end;     // 64-token blocks to (re)compute
  int64_t max_blocks;         // rows of the stats tables
  double* ksum;               // [B][max_blocks][H][128]
  float* vamax;               // [B][max_blocks][H][128]
};

struct KvWindowSumsArgs {
  const double* ksum;
  const float* vamax;
  int batch, heads;
  int blk_begin, blk_end;
  int64_t max_blocks;
  double* ksum_total;         // [B][H][128]
  float* vamax_total;         // [B][H][128]
};

struct QuantQArgs {
  const __nv_bfloat16* q;
  int64_t sq_b, sq_l, sq_h;
  int batch, heads;
  int q_len, q_pad;
  int8_t* q_codes;            // [B][H][q_pad][128]
  float* q_scale;             // [B][H][q_pad/32]
};

struct QuantKArgs {
  const __nv_bfloat16* k;
  int64_t sk_b, sk_l, sk_h;
  int batch, heads;
  int64_t tok0;               // first token of this segment in `k`
  int seg, seg_valid, seg_pad;
  int64_t kv_len_total;       // tokens of the whole window (mean denominator)
  const double* ksum_total;   // [B][H][128]
  int8_t* k_codes;            // [S][B][H][seg_pad][128]
  float* k_scale;             // [S][B][H][seg_pad/64]
  __nv_bfloat16* km_out;      // [B][H][128] or null
  int write_km;
};

struct QuantVArgs {
  const __nv_bfloat16* v;
  int64_t sv_b, sv_l, sv_h;
  int batch, heads;
  int64_t tok0;
  int seg, seg_valid, seg_pad;
  const float* vamax_total;   // [B][H][128]
  uint8_t* vt_codes;          // [S][B][H][128][seg_pad]
  float* v_scale;             // [B][H][128]
  int write_scale;
};

struct AttnArgs {
  const float* q_scale;       // [B][H][q_pad/32]
  const float* k_scale;       // [S][B][H][seg_pad/64]
  const float* v_scale;       // [B][H][128]
  __nv_bfloat16* out;         // [B, Lq, H, 128] with the strides below
  int64_t so_b, so_l, so_h;
  float* o_part;              // [splits][B*H][q_pad][128] when splits > 1
  float2* ml_part;            // [splits][B*H][q_pad]       (row max in log2 units, row sum)
  int batch, heads;
  int q_len, q_pad;
  int kv_len, nseg, seg_len, seg_pad;
  int num_splits, tiles_per_split, total_tiles;
  float sm_log2;              // softmax scale * log2(e)
  int* status;                // device status word (timeouts)
};

struct CombineArgs {
  const float* o_part;
  const float2* ml_part;
  const float* v_scale;
  __nv_bfloat16* out;
  int64_t so_b, so_l, so_h;
  int batch, heads, q_len, q_pad, num_splits;
};

cudaError_t launch_kv_block_stats(const KvBlockStatsArgs& a, cudaStream_t st);
cudaError_t launch_kv_window_sums(const KvWindowSumsArgs& a, cudaStream_t st);
cudaError_t launch_quant_q(const QuantQArgs& a, cudaStream_t st);
cudaError_t launch_quant_k(const QuantKArgs& a, cudaStream_t st);
cudaError_t launch_quant_vt(const QuantVArgs& a, cudaStream_t st);
cudaError_t launch_attn(const AttnArgs& a, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                        const CUtensorMap& tm_v, cudaStream_t st);
cudaError_t launch_combine(const CombineArgs& a, cudaStream_t st);
int* device_status_ptr();
// Records `code` and a printf-style message as this thread's lbq_last_error(); returns `code`.
int set_error(int code, const char* fmt, ...);

}  // namespace lbq
