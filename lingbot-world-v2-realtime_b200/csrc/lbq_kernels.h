// Argument blocks and launchers shared between the kernels and the C-ABI layer (internal header).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>

namespace lbq {

// Rowwise FP8 quantization (lingbot/layers/linear.py:FP8Linear): x [rows][cols] (row stride sx
// elements, dtype 0 bf16 / 1 fp16 / 2 fp32) -> e4m3 codes q [rows][cols] (row stride sq bytes) and one
// fp32 scale per row.
struct Fp8QuantArgs {
  const void* x;
  int64_t sx;
  int esize, dtype;
  int rows, cols;
  uint8_t* q;
  int64_t sq;
  float* scale;
};
// y [M][N] bf16 (row stride sy) = (q_x [M][K] . q_w [N][K]^T) * x_scale[m] * w_scale[n] + bias[n].
constexpr int kGemmThreads = 320;
struct Fp8GemmArgs {
  const float* x_scale;
  const float* w_scale;
  const __nv_bfloat16* bias;    // [N] or null
  __nv_bfloat16* y;
  int64_t sy;
  int M, N, K;
  int tiles_m, tiles_n;
  int* status;
  int wide_stores;              // y and its row stride are 32-byte aligned: 256-bit stores
};

// Ring layout of a KV-cache buffer: logical token t (the reference's window position) lives at buffer
// row t when t < sink, else at sink + ((t - sink + head) mod len). len == 0: rows are logical tokens.
struct Ring {
  int64_t sink, len, head;
};
__host__ __device__ inline int64_t phys_tok(const Ring& r, int64_t t) {
  if (r.len == 0 || t < r.sink) return t;
  int64_t u = t - r.sink + r.head;
  if (u >= r.len) u -= r.len;
  return r.sink + u;
}

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
  int* status;                // device status word (debug-build index checks)
  int dtype;                  // activations: 0 bf16, 1 fp16
  Ring ring;                  // k / v rows of logical tokens
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
  const double* rope_cos;     // null: no RoPE; else [B][L][64] (strides sr_b, sr_l in elements)
  const double* rope_sin;
  int64_t sr_b, sr_l;
  int dtype;                  // q: 0 bf16, 1 fp16 (RoPE only with bf16)
};

// Store a chunk of K/V into the cache buffer (K optionally roped) and recompute the statistics of
// the 64-token blocks covering [tok_begin, tok_end): tokens of those blocks before tok_begin are read
// back from the cache, tokens from tok_end on count as absent (as kv_block_stats with kv_len =
// tok_end).
struct CacheWriteArgs {
  const __nv_bfloat16* k_src;   // [B][n][H][128] (token tok_begin + i at row i)
  const __nv_bfloat16* v_src;
  int64_t sk_b, sk_l, sk_h, sv_b, sv_l, sv_h;
  __nv_bfloat16* k_cache;       // [B][kv_size][H][128]
  __nv_bfloat16* v_cache;
  int64_t ck_b, ck_l, ck_h, cv_b, cv_l, cv_h;
  const double* rope_cos;       // null: K stored as given; else [B][n][64] for the chunk's tokens
  const double* rope_sin;
  int64_t sr_b, sr_l;
  int batch, heads;
  int64_t tok_begin, tok_end;
  int blk_begin;
  int64_t max_blocks;
  double* ksum;                 // [B][max_blocks][H][128]
  float* vamax;
  int* status;
  Ring ring;                    // cache rows of logical tokens (tok_begin.. are logical)
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
  __nv_bfloat16* km_out;      // [B][H][128] (in k's dtype) or null
  int write_km;
  int* status;                // device status word (debug-build index checks)
  int dtype;                  // k: 0 bf16, 1 fp16
  Ring ring;                  // k rows of logical tokens
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
  int* status;                // device status word (debug-build index checks)
  int dtype;                  // v: 0 bf16, 1 fp16
  Ring ring;                  // v rows of logical tokens
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
  // Key-range mode only (attn_fwd_kernel<true>): the CTA's key tiles are one piece per code segment;
  // piece s is tiles [range_tile0[s], range_tile0[s + 1]) of the tile sequence, i.e. tiles
  // range_lt0[s] + ... of segment s, whose keys >= range_valid[s] are masked. The output is a partial
  // (O / row sum as fp16 V-code units, and the row's (max, sum)) stored into this rank's receive slot
  // at the rank that owns the query tile, through peer memory.
  int range_valid[2];
  int range_tile0[3];
  int range_lt0[2];
  const uint64_t* peers;
  int nranks, rank;
  int part;                   // query rows per owner rank (multiple of 128)
  int64_t xchg_off;
  int64_t recv_o_off;         // heap offset of the receive slots [ranks][B*H][part][128] fp16
  int64_t recv_ml_off;        //                                  [ranks][B*H][part] float2
  int wide_out;               // out's base and row strides are 32-byte aligned: 256-bit stores
  int wide_part;              // o_part is 32-byte aligned: 256-bit stores of the split partials
  int dtype;                  // out: 0 bf16, 1 fp16 (one-pass and split-KV modes)
};

// Merge of the key-range partials a rank received for its query rows (flash-decoding merge).
struct KeysCombineArgs {
  const __half* recv_o;       // [ranks][B*H][part][128]
  const float2* recv_ml;      // [ranks][B*H][part]
  const float* v_scale;       // [B*H][128]
  __nv_bfloat16* out;         // [B, rows, H, 128] with the strides below
  int64_t so_b, so_l, so_h;
  int batch, heads, rows, part, nranks;
};

// This rank's query-slice codes (a [B][H][rows_pad][128] buffer and its [B][H][rows_pad/32] scales)
// into row `row0` of every rank's full query buffers ([B][H][q_pad][128] at heap offset q_off and
// [B][H][q_pad/32] at q_scale_off), this rank's own included.
struct QPushArgs {
  const int8_t* q_codes;
  const float* q_scale;
  int rows_pad, row0, q_pad;
  int batch, heads;
  int64_t q_off, q_scale_off;
  const uint64_t* peers;
  int nranks, rank;
  int64_t xchg_off;
};

struct CombineArgs {
  const float* o_part;
  const float2* ml_part;
  const float* v_scale;
  __nv_bfloat16* out;
  int64_t so_b, so_l, so_h;
  int batch, heads, q_len, q_pad, num_splits;
  int dtype;                  // out: 0 bf16, 1 fp16
};

// Exchange area of a sequence split (byte offsets from its start, inside the peer heap).
namespace xchg {
constexpr int kMaxRanks = 8;
constexpr int64_t kFlagsData = 32;    // u32[8]  share_push signals, raised by the producers
constexpr int64_t kSeenData = 96;     // u32[8]  share signals consumed (local)
constexpr int64_t kCall = 128;        // u32     calls completed: totals tag - 1 and slot parity (local)
constexpr int64_t kDone = 132;        // u32     chunk_totals CTAs finished this call (local)
constexpr int64_t kDonePush = 136;    // u32     share_push CTAs finished this launch (local)
constexpr int64_t kDoneQuant = 140;   // u32     share_quant_push / q_push CTAs finished this launch (local)
constexpr int64_t kDoneAttn = 144;    // u32     key-range attention CTAs finished this launch (local)
constexpr int64_t kSlots = 256;       // u64 tagged words [2 parity][ranks][3][B*H*128]
constexpr int kPushCtas = 148;        // default share_push grid (persistent)
__host__ __device__ inline int64_t slot_word(uint32_t par, int nranks, int r, int w, int64_t cols) {
  return ((int64_t(par) * nranks + r) * 3 + w) * cols;
}
__host__ __device__ inline int64_t bytes(int nranks, int64_t cols) { return kSlots + 2 * int64_t(nranks) * 3 * cols * 8; }
__host__ __device__ inline int push_ctas(int units, int ctas) {
  const int c = ctas > 0 ? ctas : kPushCtas;
  return units < c ? units : c;
}
}  // namespace xchg

struct ShareTotalsArgs {
  const double* ksum;         // this rank's cache tables [B][max_blocks][H][128]
  const float* vamax;
  int64_t max_blocks;
  int row0, nb_valid;         // the share's rows in the tables
  int batch, heads;
  const uint64_t* peers;      // [nranks] heap base of every rank, as mapped in this process
  int nranks, rank;
  int64_t xchg_off;
};

struct ChunkTotalsArgs {
  const uint64_t* peers;
  int nranks, rank;
  int64_t xchg_off;
  int batch, heads;
  const double* mem_ksum;     // [B*H*128] totals of the memory part
  const float* mem_vamax;
  double* tot_ksum;           // [B*H*128] totals of the window
  float* tot_vamax;
  uint64_t timeout_ns;
  int* status;
};

struct SharePushArgs {
  const __nv_bfloat16* k;     // this rank's share [B, part, H, 128]
  const __nv_bfloat16* v;
  int64_t sk_b, sk_l, sk_h, sv_b, sv_l, sv_h;
  int batch, heads;
  int share_valid, nb_part;   // valid tokens; 64-token blocks of a share (the same on every rank)
  const uint64_t* peers;
  int nranks, rank;
  int64_t xchg_off;
  int64_t cache_k_off, cache_v_off;     // heap offsets of this layer's cache K / V [B][cache_tokens][H][128]
  int64_t cache_tokens;
  int64_t dst_tok0;                     // cache token of the share's first token (multiple of 64)
  int64_t tbl_ksum_off, tbl_vamax_off;  // heap offsets of this layer's block tables [B][max_blocks][H][128]
  int64_t tbl_max_blocks;
  int ctas;                             // grid size (the same on every rank)
};

// Copy of this rank's share of the chunk-segment codes into every other rank's code buffers: K codes
// (B*H rows of `len` tokens x 128 bytes), transposed V codes (B*H*128 rows of `len` bytes) and K scales
// (B*H rows of len/64 floats), all starting at token `lo` of segment `seg`.
struct CodePushArgs {
  const int8_t* k_codes;      // this rank's buffers (inside the peer heap)
  const float* k_scale;
  const uint8_t* vt_codes;
  int batch, heads, seg, seg_pad;
  int lo, len;                // tokens, multiples of 128
  const uint64_t* peers;
  int nranks, rank;
  int64_t xchg_off;
};

struct PeerWaitArgs {
  const uint64_t* peers;
  int nranks, rank;
  int64_t xchg_off;
  uint32_t signals;           // signals per rank and call (one per push kernel)
  uint64_t timeout_ns;
  int* status;
};

cudaError_t launch_kv_block_stats(const KvBlockStatsArgs& a, cudaStream_t st);
cudaError_t launch_kv_window_sums(const KvWindowSumsArgs& a, cudaStream_t st);
cudaError_t launch_quant_q(const QuantQArgs& a, cudaStream_t st);
cudaError_t launch_fp8_quant_rows(const Fp8QuantArgs& a, cudaStream_t st);
cudaError_t launch_fp8_gemm(const Fp8GemmArgs& a, const CUtensorMap& tm_a, const CUtensorMap& tm_b, int ctas,
                            cudaStream_t st);
cudaError_t launch_cache_write(const CacheWriteArgs& a, cudaStream_t st);
cudaError_t launch_quant_kv(const QuantKArgs& ka, const QuantVArgs& va, int tile0, int tiles, cudaStream_t st);
cudaError_t launch_attn(const AttnArgs& a, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                        const CUtensorMap& tm_v, cudaStream_t st);
cudaError_t launch_combine(const CombineArgs& a, cudaStream_t st);
cudaError_t launch_attn_keys(const AttnArgs& a, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                             const CUtensorMap& tm_v, cudaStream_t st);
cudaError_t launch_keys_combine(const KeysCombineArgs& a, cudaStream_t st);
cudaError_t launch_q_push(const QPushArgs& a, int ctas, cudaStream_t st);
cudaError_t launch_share_totals_push(const ShareTotalsArgs& a, cudaStream_t st);
cudaError_t launch_chunk_totals(const ChunkTotalsArgs& a, cudaStream_t st);
cudaError_t launch_share_push(const SharePushArgs& a, cudaStream_t st);
cudaError_t launch_peer_wait(const PeerWaitArgs& a, cudaStream_t st);
cudaError_t launch_code_push(const CodePushArgs& a, int ctas, cudaStream_t st);
int* device_status_ptr();

// Sets the largest shared-memory carveout for `Kernel` on the current device (once per device). The
// kernels that need little shared memory prefer it, so that one of them starting on an idle SM does
// not configure it for a small shared-memory split, which would keep a concurrent quantizer CTA off
// that SM until it drains (the split pushes run beside the quantizers).
#ifndef LBQ_CARVEOUT
#define LBQ_CARVEOUT 100   // preferred shared-memory carveout in percent (negative: leave the driver's choice)
#endif
template <auto Kernel>
inline cudaError_t prefer_max_shared() {
  if (LBQ_CARVEOUT < 0) return cudaSuccess;
  // per-device flags; two host threads may both set the (idempotent) attribute, nothing races
  static std::atomic<bool> done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!done[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(Kernel, cudaFuncAttributePreferredSharedMemoryCarveout, int(LBQ_CARVEOUT));
    if (e != cudaSuccess) return e;
    done[dev].store(true, std::memory_order_release);
  }
  return cudaSuccess;
}
// Allows `Kernel` `bytes` of dynamic shared memory on the current device (once per device, as above).
template <auto Kernel>
inline cudaError_t allow_dynamic_smem(int bytes) {
  static std::atomic<bool> done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!done[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    done[dev].store(true, std::memory_order_release);
  }
  return cudaSuccess;
}
// Records `code` and a printf-style message as this thread's lbq_last_error(); returns `code`.
int set_error(int code, const char* fmt, ...);

}  // namespace lbq
