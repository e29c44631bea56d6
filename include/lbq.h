/* lbq — B200 (sm_100a) quantized attention for the LingBot-World causal DiT.
 *
 * C ABI of `liblbq.so`. Every entry point takes plain device pointers, element counts and strides
 * and a `cudaStream_t` (passed as `void*`); it validates its arguments, launches on that stream
 * only (no synchronisation, no allocation), and returns 0 or an LBQ_ERR_* code. On error,
 * `lbq_last_error()` describes the failure (thread-local). The caller allocates every buffer.
 *
 * Tensors follow the reference's "NHD" activations: q/k/v/out are [B, L, H, 128] bf16 with
 * arbitrary element strides for B, L and H (the channel stride must be 1, base addresses and the
 * three strides 16-byte aligned).
 *
 * Quantized window layout (produced by the quantizers, consumed by lbq_attn_fwd):
 *   q_codes  int8 [B][H][q_pad][128]        q_pad   = round_up(q_len, 128)
 *   q_scale  f32  [B][H][q_pad/32]
 *   k_codes  int8 [S][B][H][seg_pad][128]   seg_pad = round_up(seg_len, 128)
 *   k_scale  f32  [S][B][H][seg_pad/64]
 *   vt_codes u8   [S][B][H][128][seg_pad]   (e4m3, keys contiguous per channel)
 *   v_scale  f32  [B][H][128]
 *   km       bf16 [B][H][128]
 * S is the number of KV segments: 1 on one GPU; one per rank after the all-gather of a sequence
 * split (segment s holds tokens [s*seg_len, min((s+1)*seg_len, kv_len)) of the window).
 * Paths in citations are inside the reference project (kaarelkaarelson/lingbot-world-v2-realtime).
 */
#ifndef LBQ_H_
#define LBQ_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LBQ_API __attribute__((visibility("default")))
#else
#define LBQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LBQ_OK 0
#define LBQ_ERR_ARG 1          /* bad shape, stride, length or null pointer */
#define LBQ_ERR_ALIGN 2        /* pointer or stride not 16-byte aligned */
#define LBQ_ERR_CUDA 3         /* CUDA runtime / driver error (launch, tensor map) */
#define LBQ_ERR_UNSUPPORTED 4  /* causal attention in the quantized kernel */

/* Activation types of the drop-in path (lbq_quant_qkv, lbq_quant_qkv_static, lbq_attn_fwd,
 * lbq_splitkv_combine): the `dtype` the reference's attention() casts q/k/v to before Sage
 * (lingbot/layers/attention.py:30,34). The other entries take bf16. */
#define LBQ_DTYPE_BF16 0
#define LBQ_DTYPE_F16 1

/* Version of this ABI (major * 100 + minor). */
LBQ_API int lbq_abi_version(void);

/* Message of the last error on this thread ("" if none). */
LBQ_API const char* lbq_last_error(void);

/* Device status word of the current device: 0, or the code of the first device-side wait that
 * gave up (a pipeline stalled past its time limit; the kernel returned early and its output is
 * invalid). Synchronous. `clear` != 0 resets it to 0 afterwards. */
LBQ_API int lbq_device_status(int clear, int* status_out);

/* Ring layout of a KV-cache buffer (the arguments ring_sink, ring_len, ring_head of the three cache
 * entries below): logical window token t — the reference's cache row after its left-shift eviction
 * (lingbot/layers/kv_cache.py:52-61) — is stored at buffer row t when t < ring_sink, else at
 * ring_sink + ((t - ring_sink + ring_head) mod ring_len). An eviction is then ring_head += evicted
 * (mod ring_len) instead of a copy. ring_len = 0 (with sink and head 0): rows are logical tokens. */

/* Per-64-token-block statistics of a bf16 K/V window: ksum (fp64 sum of K per channel) and vamax
 * (max |V| per channel) for blocks [blk_begin, blk_end) of logical tokens [0, kv_len).
 * Tables are [B][max_blocks][H][128]. Block b covers tokens [64b, min(64b+64, kv_len)).
 * Replaces the per-64-token V min/max table of lingbot/layers/sage_preq.py:36-44,87-98
 * (`_blk_minmax`, `_update`) and extends it with the K sums the mean-smoothing needs. */
LBQ_API int lbq_kv_block_stats(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h,
                       const void* v, int64_t sv_b, int64_t sv_l, int64_t sv_h,
                       int batch, int heads, int64_t kv_len, int blk_begin, int blk_end,
                       int64_t max_blocks, double* ksum, float* vamax, int64_t ring_sink,
                       int64_t ring_len, int64_t ring_head, void* stream);

/* Reduce the block statistics of blocks [blk_begin, blk_end) into per-(batch, head, channel)
 * totals: ksum_total (fp64) and vamax_total. With several ranks, each reduces its own blocks and
 * the totals are all-reduced (sum / max) before quantizing.
 * Replaces the window reductions of sage_preq.py:47-63 (`_v_scale`) and :115 (`k.mean`). */
LBQ_API int lbq_kv_window_sums(const double* ksum, const float* vamax, int batch, int heads, int blk_begin,
                       int blk_end, int64_t max_blocks, double* ksum_total, float* vamax_total,
                       void* stream);

/* Q quantizer: int8 per (batch, head, 32-token group), Lq padded to 128 (rows >= q_len encode 0).
 * Replaces the Q half of sageattention.quant.per_warp_int8(q, k, km, "NHD", BLKQ=128, WARPQ=32,
 * BLKK=64) called at lingbot/layers/sage_preq.py:116 (semantics restated at
 * experiments/modules/sage_kvq.py:57-66,104). */
LBQ_API int lbq_quant_q(const void* q, int64_t sq_b, int64_t sq_l, int64_t sq_h, int batch, int heads,
                int q_len, int8_t* q_codes, float* q_scale, void* stream);

/* RoPE + Q quantizer in one pass: the reference's `causal_rope_apply(q, rope)` (fp64 rotation of each
 * channel pair, cast back to bf16; lingbot/models/lingbot_world/transformer.py:134-146, called at
 * :212) followed by lbq_quant_q's codes of the roped rows, without the roped bf16 Q ever reaching
 * memory. rope_cos / rope_sin: the chunk's float64 tables [B, L, 64] from causal_rope_freqs
 * (transformer.py:53-76; the [B, L, 1, 64] tensors with the head axis dropped), element strides
 * sr_b, sr_l (even), 16-byte aligned. */
LBQ_API int lbq_rope_quant_q(const void* q, int64_t sq_b, int64_t sq_l, int64_t sq_h, const double* rope_cos,
                             const double* rope_sin, int64_t sr_b, int64_t sr_l, int batch, int heads, int q_len,
                             int8_t* q_codes, float* q_scale, void* stream);

/* KV-cache write of one chunk with its block statistics, in one pass: stores K (roped first when
 * rope_cos / rope_sin are given, as the reference's causal_rope_apply(k, rope) at transformer.py:213)
 * and V at tokens [tok_begin, tok_begin + n_tokens) of the cache buffers (kv_cache.write's
 * `kv_cache["k"][:, local_start_index:local_end_index] = k`, lingbot/layers/kv_cache.py:64-75), and
 * recomputes the statistics rows of the 64-token blocks covering those tokens exactly as
 * lbq_kv_block_stats(kv_len = tok_begin + n_tokens) would after the copy (earlier tokens of the first
 * block are read back from the cache). The source must not overlap the cache. Tokens are logical;
 * rows follow the ring layout. */
LBQ_API int lbq_cache_write(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b,
                            int64_t sv_l, int64_t sv_h, const double* rope_cos, const double* rope_sin, int64_t sr_b,
                            int64_t sr_l, void* k_cache, int64_t ck_b, int64_t ck_l, int64_t ck_h, void* v_cache,
                            int64_t cv_b, int64_t cv_l, int64_t cv_h, int batch, int heads, int64_t kv_size,
                            int64_t tok_begin, int64_t n_tokens, int64_t max_blocks, double* ksum, float* vamax,
                            int64_t ring_sink, int64_t ring_len, int64_t ring_head, void* stream);

/* K/V quantizer for one segment of the window: tokens [tok0, tok0 + seg_valid) of k/v become
 * segment `seg` of the code buffers (num_segments segments in total). km = bf16(ksum_total /
 * kv_len_total); K codes per 64-token block of (k - km); V codes e4m3 of v * (2.25/vamax_total).
 * `km_out` (nullable) and `v_scale` are written when `write_totals` != 0.
 * Replaces the K half of per_warp_int8 (sage_preq.py:115-116) and Sage's V
 * transpose/pad/permute + per-channel fp8 quantization (sage_preq.py:67-77, 121-124;
 * sage_kvq.py:69-75). */
LBQ_API int lbq_quant_kv(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h,
                 const void* v, int64_t sv_b, int64_t sv_l, int64_t sv_h,
                 int batch, int heads, int64_t tok0, int seg, int num_segments, int seg_valid,
                 int seg_len, int64_t kv_len_total, const double* ksum_total,
                 const float* vamax_total, int8_t* k_codes, float* k_scale, uint8_t* vt_codes,
                 void* km_out, float* v_scale, int write_totals, void* stream);

/* Scratch bytes lbq_quant_qkv needs for batch x heads and kv_len tokens:
 * batch * heads * (ceil(kv_len/64) + 1) * 1536 + 64. SIZE_MAX when batch or heads is outside
 * 1..65535, kv_len outside 1..2^30, or the size overflows. */
LBQ_API size_t lbq_quant_qkv_workspace(int batch, int heads, int64_t kv_len);

/* The whole per-call quantization of sageattn(q, k, v, "NHD") (lingbot/layers/attention.py:34):
 * block stats -> window sums -> Q, K, V codes, in 5 launches, with a caller-provided workspace of
 * lbq_quant_qkv_workspace() bytes. One segment. */
LBQ_API int lbq_quant_qkv(const void* q, int64_t sq_b, int64_t sq_l, int64_t sq_h, int q_len,
                  const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h,
                  const void* v, int64_t sv_b, int64_t sv_l, int64_t sv_h, int64_t kv_len,
                  int batch, int heads, int8_t* q_codes, float* q_scale, int8_t* k_codes,
                  float* k_scale, uint8_t* vt_codes, float* v_scale, void* km_out,
                  void* workspace, size_t workspace_bytes, int dtype, void* stream);

/* lbq_quant_qkv for callers that cannot give this library device memory: an embedding runtime
 * whose device memory pool is fixed and owned elsewhere (no allocation once serving starts), or an
 * FFI binding that can pass inputs and outputs but not a workspace. Same arguments and results as
 * lbq_quant_qkv without the workspace; the scratch is a 16 MiB array inside the library (one per
 * GPU that loads it, kept until exit), so a call needs lbq_quant_qkv_workspace(batch, heads, kv_len)
 * <= 16 MiB (58176 keys at 12 heads, batch 1) and is rejected with LBQ_ERR_ARG beyond that.
 * The call allocates nothing. All calls on a device share the array: calls whose kernels overlap
 * on the GPU race. The first call on a device looks up the array's address; make it before any
 * stream capture. No counterpart in the reference (its quantizers allocate through torch). */
LBQ_API int lbq_quant_qkv_static(const void* q, int64_t sq_b, int64_t sq_l, int64_t sq_h, int q_len,
                                 const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h,
                                 const void* v, int64_t sv_b, int64_t sv_l, int64_t sv_h, int64_t kv_len,
                                 int batch, int heads, int8_t* q_codes, float* q_scale, int8_t* k_codes,
                                 float* k_scale, uint8_t* vt_codes, float* v_scale, void* km_out,
                                 int dtype, void* stream);

/* Re-quantize a bf16 KV cache window [0, kv_len) whose block statistics are current (kept by
 * lbq_kv_block_stats on every write): window sums + K/V codes, one segment, in 3 launches.
 * `sums_ws` holds B*H*128 doubles followed by B*H*128 floats.
 * Replaces the per-call re-quantization of the cache window done by sageattn / sage_preq.attend
 * (lingbot/layers/sage_preq.py:107-124) and sage_kvq.requant_all (experiments/modules/sage_kvq.py:93-98). */
LBQ_API int lbq_requant_cache(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h,
                      const void* v, int64_t sv_b, int64_t sv_l, int64_t sv_h,
                      int batch, int heads, int64_t kv_len, int64_t max_blocks,
                      const double* ksum, const float* vamax, void* sums_ws,
                      int8_t* k_codes, float* k_scale, uint8_t* vt_codes, float* v_scale,
                      void* km_out, int64_t ring_sink, int64_t ring_len, int64_t ring_head,
                      void* stream);

/* Attention over quantized codes. out [B, q_len, H, 128] in `dtype` (LBQ_DTYPE_BF16 or _F16) with
 * element strides so_*. sm_scale <= 0 means 1/sqrt(128). is_causal != 0 returns LBQ_ERR_UNSUPPORTED:
 * the kernel has no causal mask (the drop-in attention() sends causal calls to the reference's
 * non-Sage branch instead; the DiT never makes one). num_splits > 1 splits the key range (flash-decoding):
 * partial results go to o_part (f32, [splits][B*H][q_pad][128]) and ml_part (f32 pairs,
 * [splits][B*H][q_pad]) and lbq_splitkv_combine finishes them; num_splits is clamped so that no
 * split is empty (the value used is written to *splits_used when non-null).
 * Replaces sm89_compile.qk_int8_sv_f8_accum_f16_fuse_v_scale_attn_inst_buf(q_i8, k_i8, v_fp8, o,
 * q_s, k_s, v_s, 0, 0, 2, sm_scale, 0) called at lingbot/layers/sage_preq.py:126-127 and
 * experiments/modules/sage_kvq.py:107-110, with the split-KV variant designed in
 * experiments/bench_attn/splitkv/README.md. */
LBQ_API int lbq_attn_fwd(const int8_t* q_codes, const float* q_scale, int q_len,
                 const int8_t* k_codes, const float* k_scale, const uint8_t* vt_codes,
                 const float* v_scale, int64_t kv_len, int num_segments, int seg_len,
                 int batch, int heads, float sm_scale, int is_causal, void* out, int64_t so_b,
                 int64_t so_l, int64_t so_h, int num_splits, float* o_part, float* ml_part,
                 int* splits_used, int dtype, void* stream);

/* lbq_quant_kv restricted to the 128-token tiles [tile_begin, tile_end) of the segment (those holding
 * valid tokens: tile_end <= ceil(seg_valid / 128)); segment token t reads source token tok0 + t, and
 * tok0 may be negative as long as tok0 + 128 * tile_begin >= 0 (a share whose first token is segment
 * token -tok0). km_out / v_scale are written by the range's first tile when write_totals != 0. Codes are
 * those of lbq_quant_kv for the same tokens: the key-range split quantizes only its own tiles of the
 * window (the per-rank quantization of sage_preq.py:115-124 after lingbot/parallel/split_dit.py:371-386,
 * cut to the rank's keys). */
LBQ_API int lbq_quant_kv_tiles(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h,
                       const void* v, int64_t sv_b, int64_t sv_l, int64_t sv_h, int batch, int heads,
                       int64_t tok0, int seg, int num_segments, int seg_valid, int seg_len,
                       int64_t kv_len_total, const double* ksum_total, const float* vamax_total,
                       int8_t* k_codes, float* k_scale, uint8_t* vt_codes, void* km_out, float* v_scale,
                       int write_totals, int tile_begin, int tile_end, void* stream);

/* Key-range split attention: every query row (q_codes / q_scale [B][H][q_pad][128] / [B][H][q_pad/32],
 * q_len valid rows) against this rank's keys only — for each code segment s < num_segments (1 or 2,
 * [S][B][H][seg_pad] layouts as lbq_attn_fwd), tiles [range_lt0[s], range_lt0[s] + range_tiles[s]) of
 * segment s, keys >= range_valid[s] of the segment masked (host arrays of num_segments ints; at least
 * one tile in total). Instead of an output, each query tile's partial — O / row sum as fp16 in V-code
 * units ([B*H][part][128]) and the row's (max, sum) as f32 pairs ([B*H][part]) — is stored into slot
 * `rank` of the receive buffers of the rank owning the tile (rows [p*part, (p+1)*part) belong to rank
 * p; heap offsets recv_o_off / recv_ml_off of [nranks] slots each), through peer memory; the last CTA
 * then raises every other rank's data signal once. Ranks combine with lbq_keys_combine after
 * lbq_peer_wait(signals = 1). Replaces the Ulysses head exchange around the attention of
 * lingbot/parallel/split_dit.py:366-445: here heads stay whole and the keys are split. */
LBQ_API int lbq_attn_fwd_keys(const int8_t* q_codes, const float* q_scale, int q_len, int q_pad,
                      const int8_t* k_codes, const float* k_scale, const uint8_t* vt_codes,
                      int num_segments, int seg_len, int batch, int heads, float sm_scale,
                      const int* range_lt0, const int* range_tiles, const int* range_valid,
                      const uint64_t* peers, int nranks, int rank, int64_t xchg_off, int part,
                      int64_t recv_o_off, int64_t recv_ml_off, void* stream);

/* Merge of the key-range partials in this rank's receive buffers (recv_o fp16 [nranks][B*H][part][128],
 * recv_ml f32 pairs [nranks][B*H][part]) for its first `rows` query rows into out [B, rows, H, 128]
 * (bf16, element strides so_*), applying the V scale: the split-KV merge of
 * experiments/bench_attn/splitkv/README.md:60-69 over ranks instead of splits. */
LBQ_API int lbq_keys_combine(const void* recv_o, const float* recv_ml, int nranks, int part, int rows,
                     const float* v_scale, int batch, int heads, void* out, int64_t so_b,
                     int64_t so_l, int64_t so_h, void* stream);

/* Rowwise FP8 quantization of FP8Linear (lingbot/layers/linear.py:16-18 for weights, :24-26 for the
 * activations of each call): per row, s = max(fl(max|x| / 448), 1e-12) and q = e4m3(fl(x / s)) with
 * true fp32 divisions. x [rows][cols], row stride sx elements, dtype 0 bf16 / 1 fp16 / 2 fp32;
 * q [rows][cols] e4m3 bytes, row stride sq; scale [rows] f32. cols a multiple of 16. */
LBQ_API int lbq_fp8_quant_rows(const void* x, int64_t sx, int dtype, int rows, int cols, uint8_t* q, int64_t sq,
                               float* scale, void* stream);

/* FP8 GEMM of FP8Linear.forward (lingbot/layers/linear.py:27-29, torch._scaled_mm with rowwise scales):
 * y [M][N] bf16 (row stride sy elements) = (a [M][K] . w [N][K]^T) * a_scale[m] * w_scale[n] + bias[n]
 * (bias bf16 [N] or null), e4m3 operands with row strides sa / sw bytes, fp32 accumulation on the
 * tensor cores. N a multiple of 32, K of 16. num_ctas <= 0: one CTA per SM (persistent over the
 * 128 x 256 output tiles). */
LBQ_API int lbq_fp8_gemm(const uint8_t* a, int64_t sa, const float* a_scale, const uint8_t* w, int64_t sw,
                         const float* w_scale, const void* bias, int M, int N, int K, void* y, int64_t sy,
                         int num_ctas, void* stream);

/* Flash-decoding merge of lbq_attn_fwd's split partials into out (in `dtype`), applying the V scale.
 * The combine kernel of experiments/bench_attn/splitkv/README.md:67-69 (`splitkv_combine_kernel`). */
LBQ_API int lbq_splitkv_combine(const float* o_part, const float* ml_part, int num_splits,
                        const float* v_scale, int batch, int heads, int q_len, void* out,
                        int64_t so_b, int64_t so_l, int64_t so_h, int dtype, void* stream);

/* ---------------------------------------------------------------- sequence split over peer memory
 * The ranks of one node share a "peer heap": a device buffer per rank, mapped into every other
 * rank's address space through CUDA IPC and carved identically on every rank, so a buffer is named
 * by its byte offset and rank p's copy lives at peers[p] + offset. `peers` is a device array of
 * nranks (<= 8) u64 heap bases as mapped in the calling process (its own heap at [rank]). The
 * exchange area (lbq_exchange_bytes, 256-byte aligned offset `xchg_off`) is zeroed by the caller on
 * every rank, followed by a barrier, before first use. Waits are bounded by `timeout_ns`; a wait
 * that gives up records LBQ status 0x201 / 0x202 (lbq_device_status) instead of hanging.
 * Together these replace the head/token exchange of lingbot/parallel/split_dit.py:366-445 (`_layer`:
 * the q/k/v head exchange `self.xch(...)`, the cache write in `_attend`, the output send-back),
 * which needs the head count divisible by the degree (lingbot/parallel/config.py:13-17). */

/* Interprocess handle of the device allocation holding `ptr` (64 bytes to `handle_out`) and the
 * offset of `ptr` inside it. Synchronous; no stream work. Replaces the CUDA-IPC buffer sharing
 * behind `self.xch` in lingbot/parallel/split_dit.py (ZEROCOPY path). */
LBQ_API int lbq_peer_export(const void* ptr, void* handle_out, uint64_t* offset_out);

/* Maps another process's allocation (handle from lbq_peer_export) into this process; *base_out is
 * the mapped allocation base (add the exported offset to reach the peer's pointer). */
LBQ_API int lbq_peer_open(const void* handle, void** base_out);

/* Unmaps an allocation base returned by lbq_peer_open. */
LBQ_API int lbq_peer_close(void* base);

/* Bytes of the exchange area for nranks ranks and batch x heads. */
LBQ_API int64_t lbq_exchange_bytes(int nranks, int batch, int heads);

/* Per-channel totals (fp64 K sum, max |V|) of this rank's share of the chunk, reduced from its block
 * statistics in this rank's cache tables (ksum/vamax [B][max_blocks][H][128], rows [row0, row0 +
 * nb_valid), written by lbq_kv_block_stats), stored into every rank's exchange area, one signal per
 * CTA. Replaces this rank's part of the window reductions of lingbot/layers/sage_preq.py:47-63,115
 * (`_v_scale`, `k.mean`) under a sequence split. */
LBQ_API int lbq_share_totals_push(const double* ksum, const float* vamax, int64_t max_blocks, int row0,
                          int nb_valid, int batch, int heads, const uint64_t* peers, int nranks, int rank,
                          int64_t xchg_off, void* stream);

/* Waits for every rank's lbq_share_totals_push of this call, then writes the window totals
 * tot_ksum = mem_ksum + the shares' sums in rank order and tot_vamax likewise with max ([B*H*128]),
 * identical on every rank. One per call, after lbq_share_totals_push on the same stream. */
LBQ_API int lbq_chunk_totals(const uint64_t* peers, int nranks, int rank, int64_t xchg_off, int batch,
                     int heads, const double* mem_ksum, const float* mem_vamax, double* tot_ksum,
                     float* tot_vamax, uint64_t timeout_ns, void* stream);

/* Copies this rank's bf16 K/V share (k/v [B, part, H, 128], share_valid valid tokens, nb_part =
 * part / 64 on every rank) into every rank's cache replica (heap offsets cache_k_off / cache_v_off of
 * [B][cache_tokens][H][128] bf16 caches, starting at token dst_tok0, a multiple of 64) and the
 * share's block-statistics rows of this rank's tables into the other ranks' tables (heap offsets
 * tbl_ksum_off / tbl_vamax_off, [B][tbl_max_blocks][H][128]), then signals the other ranks once. Must be
 * ordered after this call's lbq_chunk_totals (which proves that every rank has finished reading its
 * cache in the previous call). `ctas` (0 = 148) CTAs stride over the share, bounding how many SMs the
 * push takes from concurrent kernels; every rank passes the same value, here and to lbq_peer_wait. Replaces the ZEROCOPY K/V write into the peer's buffer and the
 * kv_cache.write of lingbot/parallel/split_dit.py:371-376,425-431. */
LBQ_API int lbq_share_push(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h,
                   const void* v, int64_t sv_b, int64_t sv_l, int64_t sv_h,
                   int batch, int heads, int share_valid, int nb_part,
                   const uint64_t* peers, int nranks, int rank, int64_t xchg_off,
                   int64_t cache_k_off, int64_t cache_v_off, int64_t cache_tokens, int64_t dst_tok0,
                   int64_t tbl_ksum_off, int64_t tbl_vamax_off, int64_t tbl_max_blocks, int ctas,
                   void* stream);

/* Quantizes this rank's share of the chunk (k/v [B, part, H, 128], share_valid valid tokens, chunk
 * tokens [lo, lo + part) with lo and part multiples of 128) with the window totals from
 * lbq_chunk_totals — the same codes lbq_quant_kv gives for those tokens of segment `seg` — into this
 * rank's code buffers (k_codes / k_scale / vt_codes, inside the peer heap at the same offsets on every
 * rank), then copies them into every other rank's buffers with `ctas` CTAs (0 = 32; the same on every
 * rank) and signals the other ranks once. km_out / v_scale (this rank only) are written when
 * write_totals != 0. Must be
 * ordered after this call's lbq_chunk_totals (every rank has then finished its previous attention,
 * the last reader of the code buffers). Replaces the per-rank quantization of the gathered chunk
 * (sage_preq.py:115-124 after the exchange of lingbot/parallel/split_dit.py:371-386). */
LBQ_API int lbq_share_quant_push(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h,
                         const void* v, int64_t sv_b, int64_t sv_l, int64_t sv_h, int batch, int heads,
                         int lo, int share_valid, int part, int seg, int num_segments, int seg_len,
                         int64_t kv_len_total, const double* ksum_total, const float* vamax_total,
                         int8_t* k_codes, float* k_scale, uint8_t* vt_codes, void* km_out, float* v_scale,
                         int write_totals, const uint64_t* peers, int nranks, int rank, int64_t xchg_off,
                         int ctas, void* stream);

/* Key-range split: copies this rank's query-slice codes (q_codes [B][H][rows_pad][128] and q_scale
 * [B][H][rows_pad/32], from lbq_quant_q) to rows [row0, row0 + rows_pad) of every rank's full query
 * buffers (heap offsets q_off / q_scale_off of [B][H][q_pad][128] / [B][H][q_pad/32]), this rank's own
 * included, with `ctas` CTAs (0 = 32), then signals the other ranks once. Must be ordered after this
 * rank's previous wait for the partials (lbq_peer_wait before lbq_keys_combine): every rank signals
 * its partials after its attention's last CTA, so every rank has then finished reading the query
 * buffers. Replaces the q all-to-all of the Ulysses split (lingbot/parallel/split_dit.py:371-386):
 * every rank needs every query row once the keys are split. */
LBQ_API int lbq_q_push(const int8_t* q_codes, const float* q_scale, int rows_pad, int row0, int q_pad,
               int batch, int heads, int64_t q_off, int64_t q_scale_off, const uint64_t* peers,
               int nranks, int rank, int64_t xchg_off, int ctas, void* stream);

/* Waits until every other rank's pushes of this call have landed in this rank's buffers: `signals`
 * (1 or 2) = the push launches every rank makes per call (lbq_share_quant_push, plus lbq_share_push
 * when the call persists its K/V; with the key-range split lbq_q_push [+ lbq_share_push] before the
 * attention, then lbq_attn_fwd_keys before the combine); this rank's own pushes are ordered by the
 * caller's streams.
 * Replaces the `comp[c].wait_event(ev)` on the peer's inbox at lingbot/parallel/split_dit.py:384-386. */
LBQ_API int lbq_peer_wait(const uint64_t* peers, int nranks, int rank, int64_t xchg_off, int signals,
                  uint64_t timeout_ns, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LBQ_H_ */
