// Quantized attention forward for sm_100a: INT8 Q.K^T and FP8 P.V on tcgen05, accumulators in
// tensor memory, operands staged by TMA, warp-specialised, two Q tiles in ping-pong.
//
// Semantics are those of SageAttention-2's `qk_int8_sv_f8_accum_f16_fuse_v_scale_attn_inst_buf`
// as the reference calls it (lingbot/layers/sage_preq.py:126-127 with qk_quant_gran=2, i.e. one
// Q scale per 32 rows; documented in experiments/bench_attn/splitkv/README.md:51-69 and
// h2_tiles/cfg_fixedmax.patch:90-93):
//   s   = (q_i8 . k_i8) * q_scale * k_scale * sm_scale * log2(e)      (int32 dot product, exact)
//   m   = running row max of s, updated once per 128-key tile
//   P   = exp2(s - m + 8.807)  (<= 448), rounded to e4m3 for the P.V product
//   d   = d * exp2(m_old - m) + sum(P)                                (fp32, before rounding)
//   O   = O * exp2(m_old - m) + e4m3(P) . e4m3(V)                      (fp32 in tensor memory)
//   out = O / d * v_scale  -> bf16
// Differences from the sm89 kernel (covered by the tolerance tests): the running max is updated
// per 128 keys instead of 64, P.V accumulates in fp32 rather than fp16 inside a tile, and exp2 is
// the ex2.approx instruction for 3/4 of the keys and an FMA-pipe polynomial (relative error
// < 7.5e-5) for the rest.
//
// CTA = two 128-row Q tiles (A, B) x one (batch, head) x one KV split. Warps: 0 = TMA producer,
// 1 = tcgen05 issuer (one thread), 2..5 = softmax warpgroup A, 6..9 = softmax warpgroup B. Q row r
// of a tile is TMEM lane r; one thread owns one row and all 128 keys of each key tile. While one
// warpgroup computes its softmax the tensor core works for the other.
// Tensor memory (512 columns): S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512) (fp32).
// As soon as a warpgroup has read its scores it refills its S buffer with 0x4B400000, the bits of
// the float 1.5*2^23, and the next Q.K^T accumulates onto it: the int32 accumulator then holds the
// bits of the float 1.5*2^23 + S (|S| <= 128*127*127 < 2^22), so scores need no conversion. P is
// written (e4m3, 128-byte-swizzled K-major rows) to a double-buffered shared-memory tile that the
// P.V product reads as its A operand; the next Q.K^T therefore does not wait for P.V.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "lbq_kernels.h"
#include "lbq_peer.cuh"
#include "lbq_ptx.cuh"

namespace lbq {

constexpr int kStages = 3;
constexpr int kTile = 128 * 128;         // bytes of one 128 x 128 8-bit tile
constexpr int kAttnThreads = 64 + 256;   // producer, issuer, 2 softmax warpgroups
constexpr float kFp8Offset = 8.807f;     // splitkv/README.md:58 (S_FP8_OFFSET)
constexpr float kMagic = 12582912.0f;    // 1.5 * 2^23

#ifndef LBQ_POLY_PAIRS
#define LBQ_POLY_PAIRS 4
#endif
// Of every 16 key pairs, this many take the FMA-pipe polynomial exp2 and the rest MUFU ex2 (MUFU
// issues one exp per 8 clocks per SM sub-partition; 4 of 16 measured best).
constexpr int kPolyPairs = LBQ_POLY_PAIRS;

struct AttnShared {
  uint64_t q_full;
  uint64_t k_full[kStages];
  uint64_t k_empty[kStages];
  uint64_t v_full[kStages];
  uint64_t v_empty[kStages];
  uint64_t s_full[2];                    // per Q tile
  uint64_t s_free[2];
  uint64_t p_full[2];
  uint64_t o_done[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// smem: Q_A, Q_B | P_A[2], P_B[2] | K stages | V stages | barriers
constexpr size_t kAttnSmemBytes = 1024 /*alignment slack*/ + kTile * (6 + 2 * kStages) + sizeof(AttnShared);

__device__ int g_status;

template <bool kKeyRange>
__device__ __forceinline__ int seg_valid(const AttnArgs& a, int seg) {
  if constexpr (kKeyRange) return a.range_valid[seg];
  const int rest = a.kv_len - seg * a.seg_len;
  return rest < a.seg_len ? rest : a.seg_len;
}
// Key tile jt of the call's tile sequence -> (code segment, tile inside the segment).
template <bool kKeyRange>
__device__ __forceinline__ void tile_seg(const AttnArgs& a, int jt, int tiles_per_seg, int& seg, int& lt) {
  if constexpr (kKeyRange) {
    seg = jt >= a.range_tile0[1] ? 1 : 0;
    lt = jt - a.range_tile0[seg] + a.range_lt0[seg];
  } else {
    seg = jt / tiles_per_seg;
    lt = jt - seg * tiles_per_seg;
  }
}

// Softmax of one 128-key tile for the calling thread's row. `sv` holds the scores as the bits of
// 1.5*2^23 + S (see the tensor-memory note above). The e4m3 P is written to this row of the shared
// P tile `prow` (128 bytes, 16-byte chunk c stored at chunk c ^ (row & 7): the 128-byte swizzle the
// MMA descriptor expects) as it is produced; `m` and `dsum` are updated and the factor O must be
// rescaled by, 2^(m_old - m_new), is returned. Keys 0..63 use K scale c1a, keys 64..127 use c1b.
template <bool kMasked>
__device__ __forceinline__ float softmax_tile(uint32_t (&sv)[4][32], int valid, float c1a, float c1b, float& m,
                                              float& dsum, uint8_t* prow, int rsw) {
  if (kMasked) {
#pragma unroll
    for (int c = 0; c < 128; ++c)
      if (c >= valid) sv[c >> 5][c & 31] = 0x4B000000u;     // 1.5*2^23 - 2^22: below every real score
  }
  auto F = [&](int c) { return __uint_as_float(sv[c >> 5][c & 31]); };
  float mh[2];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int b0 = half * 64;
    float r0 = fmaxf(F(b0 + 0), F(b0 + 1)), r1 = fmaxf(F(b0 + 2), F(b0 + 3));
    float r2 = fmaxf(F(b0 + 4), F(b0 + 5)), r3 = fmaxf(F(b0 + 6), F(b0 + 7));
#pragma unroll
    for (int c = b0 + 8; c < b0 + 64; c += 8) {
      r0 = fmax3(r0, F(c + 0), F(c + 1));
      r1 = fmax3(r1, F(c + 2), F(c + 3));
      r2 = fmax3(r2, F(c + 4), F(c + 5));
      r3 = fmax3(r3, F(c + 6), F(c + 7));
    }
    mh[half] = fmax3(r0, r1, fmaxf(r2, r3));
  }
  // tile max in log2 units; (mh - magic) is the exact integer max. A half with no valid key is
  // skipped (its block scale is the 1e-7 floor, so its stand-in score is not low enough).
  float tmax = __fmul_rn(mh[0] - kMagic, c1a);
  if (!kMasked || valid > 64) tmax = fmaxf(tmax, __fmul_rn(mh[1] - kMagic, c1b));
  const float m_new = fmaxf(m, tmax);
  const float alpha = (m == m_new) ? 1.f : ex2_approx(m - m_new);
  m = m_new;
  // x = (f - magic) * c1 + (8.807 - m) = f * c1 + c0, c0 = 8.807 - m - magic * c1 (one rounding; the
  // argument is off by at most half an ulp of |c0|, about 6e-5 for typical scales)
  const float c0a = fmaf(-kMagic, c1a, kFp8Offset - m_new);
  const float c0b = fmaf(-kMagic, c1b, kFp8Offset - m_new);
  const uint64_t c0ax2 = f2_pack(c0a, c0a), c0bx2 = f2_pack(c0b, c0b);
  const uint64_t c1ax2 = f2_pack(c1a, c1a), c1bx2 = f2_pack(c1b, c1b);
  uint64_t acc0 = f2_pack(0.f, 0.f), acc1 = acc0;
  uint32_t pw[4];
#pragma unroll
  for (int w = 0; w < 32; ++w) {
    uint32_t half16[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int c = 4 * w + 2 * e;
      const uint64_t x = f2_fma(f2_pack(F(c), F(c + 1)), c < 64 ? c1ax2 : c1bx2, c < 64 ? c0ax2 : c0bx2);
      float x0, x1;
      f2_unpack(x, x0, x1);
      uint64_t p;
      if (((c >> 1) & 15) >= 16 - kPolyPairs) {
        p = exp2_poly_x2(x0, x1);
      } else {
        p = f2_pack(ex2_approx(x0), ex2_approx(x1));
      }
      float p0, p1;
      f2_unpack(p, p0, p1);
      if (kMasked) {
        if (c >= valid) p0 = 0.f;
        if (c + 1 >= valid) p1 = 0.f;
        p = f2_pack(p0, p1);
      }
      if (e == 0) acc0 = f2_add(acc0, p); else acc1 = f2_add(acc1, p);
      half16[e] = pack_e4m3x2(p0, p1);
    }
    pw[w & 3] = half16[0] | (half16[1] << 16);
    if ((w & 3) == 3)   // 16 keys done: one swizzled 16-byte chunk of the row
      *reinterpret_cast<uint4*>(prow + (((w >> 2) ^ rsw) << 4)) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
  }
  float s0, s1, s2, s3;
  f2_unpack(acc0, s0, s1);
  f2_unpack(acc1, s2, s3);
  dsum = __fmaf_rn(dsum, alpha, (s0 + s1) + (s2 + s3));
  return alpha;
}

// Key-range epilogue of one softmax warp: its 32 rows of O / row sum as fp16 (V-code units, |x| <= 448)
// are staged in the tile's P buffers (free once O is complete; 16-byte chunks of a 256-byte row
// XOR-swizzled by row) and stored to the owner rank's receive slot for this rank as whole rows, two
// rows per warp instruction; the (max, sum) of each row follows. Rows past q_len are not stored.
__device__ __forceinline__ void store_key_partial(const AttnArgs& a, uint32_t tO, uint8_t* stage, int quarter,
                                                  int lane, int qtile, int bh, int bhs, float m, float dsum) {
  const float rd = __frcp_rn(dsum);
  const int rl = quarter * 32 + lane;                    // row inside the tile (TMEM lane)
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t ov[32];
    tmem_ld32(tO + 32 * c, ov);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      uint32_t hw[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const __half2 p = __floats2half2_rn(__fmul_rn(__uint_as_float(ov[8 * e + 2 * k]), rd),
                                            __fmul_rn(__uint_as_float(ov[8 * e + 2 * k + 1]), rd));
        hw[k] = *reinterpret_cast<const uint32_t*>(&p);
      }
      const int chunk = 4 * c + e;
      *reinterpret_cast<uint4*>(stage + rl * 256 + ((chunk ^ (rl & 15)) << 4)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    }
  }
  __syncwarp();
  const int qrow0 = qtile * 128;
  const int owner = qrow0 / a.part;                      // part % 128 == 0: one owner per Q tile
  if (!LBQ_CHECK(owner < a.nranks && qrow0 - owner * a.part + 128 <= a.part, a.status, kDevBadOwner)) return;
  const int64_t slot = (int64_t(a.rank) * bhs + bh) * a.part + (qrow0 - owner * a.part);
  char* dst = reinterpret_cast<char*>(static_cast<uintptr_t>(a.peers[owner]));
  uint8_t* dst_o = reinterpret_cast<uint8_t*>(dst + a.recv_o_off) + slot * 256;
#pragma unroll 4
  for (int i = 0; i < 16; ++i) {
    const int r = quarter * 32 + 2 * i + (lane >> 4), ch = lane & 15;
    if (qrow0 + r < a.q_len)
      *reinterpret_cast<uint4*>(dst_o + r * 256 + ch * 16) =
          *reinterpret_cast<const uint4*>(stage + r * 256 + ((ch ^ (r & 15)) << 4));
  }
  if (qrow0 + rl < a.q_len) reinterpret_cast<float2*>(dst + a.recv_ml_off)[slot + rl] = make_float2(m, dsum);
}

// 320 threads hold registers as 384 (whole warpgroups), so at one CTA per SM a thread gets <= 168.
// kKeyRange: the key-range split's variant (tile pieces of AttnArgs::range_*, partials to the query
// tile's owner rank); false: the whole window in uniform segments.
template <bool kKeyRange>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                              // [2][kTile]
  uint8_t* sP = smem + 2 * kTile;                  // [tile][buffer][kTile]
  uint8_t* sK = smem + 6 * kTile;
  uint8_t* sV = smem + kTile * (6 + kStages);
  AttnShared* sh = reinterpret_cast<AttnShared*>(smem + kTile * (6 + 2 * kStages));
  volatile int* abort_flag = &sh->abort;

  const int qp = blockIdx.x, bh = blockIdx.y, split = blockIdx.z;   // qp: pair of 128-row Q tiles
  const int b = bh / a.heads, h = bh - b * a.heads;
  const int t_begin = split * a.tiles_per_split;
  const int t_end = min(t_begin + a.tiles_per_split, a.total_tiles);
  const int n = t_end - t_begin;
  const int tiles_per_seg = a.seg_pad / 128;
  const int bhs = a.batch * a.heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&sh->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh->k_full[s], 1);
      mbar_init(&sh->k_empty[s], 1);
      mbar_init(&sh->v_full[s], 1);
      mbar_init(&sh->v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sh->s_full[t], 1);
      mbar_init(&sh->s_free[t], 128);
      mbar_init(&sh->p_full[t], 128);
      mbar_init(&sh->o_done[t], 1);
    }
    mbar_init(&sh->drain, 1);
    sh->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sh->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      // Both Q tiles; a tile past q_pad reads the map's out-of-bounds zero fill.
      mbar_arrive_expect_tx(&sh->q_full, 2 * kTile);
      tma_load_3d(sQ, &tm_q, &sh->q_full, 0, (2 * qp) * 128, bh);
      tma_load_3d(sQ + kTile, &tm_q, &sh->q_full, 0, (2 * qp + 1) * 128, bh);
      int issued = 0;
      for (int i = 0; i < n; ++i) {
        const int jt = t_begin + i;
        int seg, lt;
        tile_seg<kKeyRange>(a, jt, tiles_per_seg, seg, lt);
        (void)LBQ_CHECK(seg < a.nseg && lt >= 0 && lt < tiles_per_seg, a.status, kDevBadTile);
        const int s = i % kStages;
        const uint32_t ph = (i / kStages) & 1;
        if (!mbar_wait(&sh->k_empty[s], ph ^ 1, abort_flag, a.status, kDevTimeoutKV)) break;
        mbar_arrive_expect_tx(&sh->k_full[s], kTile);
        tma_load_3d(sK + s * kTile, &tm_k, &sh->k_full[s], 0, lt * 128, seg * bhs + bh);
        if (!mbar_wait(&sh->v_empty[s], ph ^ 1, abort_flag, a.status, kDevTimeoutKV)) {
          issued = i + 1;
          break;
        }
        mbar_arrive_expect_tx(&sh->v_full[s], kTile);
        tma_load_3d(sV + s * kTile, &tm_v, &sh->v_full[s], lt * 128, 0, seg * bhs + bh);
        issued = i + 1;
      }
      if (*abort_flag) {
        // Let copies already in flight land before the CTA's shared memory goes away.
        mbar_drain_wait(&sh->q_full, 0);
        for (int i = (issued > kStages ? issued - kStages : 0); i < issued; ++i) {
          const int s = i % kStages;
          const uint32_t ph = (i / kStages) & 1;
          mbar_drain_wait(&sh->k_full[s], ph);
          mbar_drain_wait(&sh->v_full[s], ph);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ tcgen05 issuer
    if (lane == 0 && n > 0) {
      bool ok = mbar_wait(&sh->q_full, 0, abort_flag, a.status, kDevTimeoutQ);
      tc_fence_after();
      const uint64_t qdesc[2] = {smem_desc_sw128(smem_u32(sQ)), smem_desc_sw128(smem_u32(sQ + kTile))};
      // S_t += Q_t . K(i)^T, onto the magic constant the softmax left in S_t
      auto issue_qk = [&](int t, int i) {
        const uint64_t kdesc = smem_desc_sw128(smem_u32(sK + (i % kStages) * kTile));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) mma_i8_ss(tmem + 128 * t, qdesc[t] + 2 * kk, kdesc + 2 * kk, kIdescQK, 1u);
        tc_commit(&sh->s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint64_t pdesc = smem_desc_sw128(smem_u32(sP + (2 * t + (j & 1)) * kTile));
        const uint64_t vdesc = smem_desc_sw128(smem_u32(sV + (j % kStages) * kTile));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f8_ss(tmem + 256 + 128 * t, pdesc + 2 * kk, vdesc + 2 * kk, kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&sh->o_done[t]);
      };
      if (ok && (ok = mbar_wait(&sh->k_full[0], 0, abort_flag, a.status, kDevTimeoutKV))) {
        for (int t = 0; ok && t < 2; ++t) {
          ok = mbar_wait(&sh->s_free[t], 0, abort_flag, a.status, kDevTimeoutS);   // S_t initialised
          tc_fence_after();
          if (ok) issue_qk(t, 0);
        }
        if (ok) tc_commit(&sh->k_empty[0]);
      }
      for (int j = 0; ok && j < n; ++j) {
        const int s = j % kStages;
        const bool more = j + 1 < n;
        if (more && !mbar_wait(&sh->k_full[(j + 1) % kStages], ((j + 1) / kStages) & 1, abort_flag, a.status,
                               kDevTimeoutKV))
          break;
        if (!mbar_wait(&sh->v_full[s], (j / kStages) & 1, abort_flag, a.status, kDevTimeoutKV)) break;
        for (int t = 0; ok && t < 2; ++t) {
          if (more) {            // S_t(j) read and refilled -> next scores
            if (!(ok = mbar_wait(&sh->s_free[t], (j + 1) & 1, abort_flag, a.status, kDevTimeoutS))) break;
            tc_fence_after();
            issue_qk(t, j + 1);
          }
          if (!(ok = mbar_wait(&sh->p_full[t], j & 1, abort_flag, a.status, kDevTimeoutP))) break;
          tc_fence_after();
          issue_pv(t, j);
        }
        if (!ok) break;
        tc_commit(&sh->v_empty[s]);
        if (more) tc_commit(&sh->k_empty[(j + 1) % kStages]);
      }
      // Drain: every MMA issued above has completed once `drain` flips.
      tc_commit(&sh->drain);
      mbar_drain_wait(&sh->drain, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    const int t = (warp - 2) >> 2;                      // Q tile of this warpgroup
    const int quarter = warp & 3;                       // TMEM lanes [32*quarter, 32*quarter+32)
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const uint32_t tS = tmem + 128 * t + lane_off, tO = tmem + 256 + 128 * t + lane_off;
    const int qtile = 2 * qp + t;
    const int row = qtile * 128 + quarter * 32 + lane;
    const float qs = qtile * 128 < a.q_pad ? a.q_scale[int64_t(bh) * (a.q_pad / 32) + qtile * 4 + quarter] : 0.f;
    const int kspb = a.seg_pad / 64;
    auto kscale_ptr = [&](int i) {
      const int jt = t_begin + i;
      int seg, lt;
      tile_seg<kKeyRange>(a, jt, tiles_per_seg, seg, lt);
      if (!LBQ_CHECK(seg < a.nseg && lt >= 0 && lt * 2 + 1 < kspb, a.status, kDevBadTile)) seg = lt = 0;
      return a.k_scale + int64_t(seg * bhs + bh) * kspb + lt * 2;
    };
    float m = -INFINITY, dsum = 0.f;
    bool ok = n > 0;
    const int prow_off = (quarter * 32 + lane) * 128;
    const int rsw = lane & 7;                               // row & 7 (rows of a warp start at 32k)
    // S_t starts as the magic constant (the first Q.K^T accumulates onto it)
#pragma unroll
    for (int c = 0; c < 16; ++c) tmem_fill8(tS + 8 * c, 0x4B400000u);
    tmem_st_wait();
    tc_fence_before();
    mbar_arrive(&sh->s_free[t]);
    float2 ks_next = ok ? *reinterpret_cast<const float2*>(kscale_ptr(0)) : make_float2(0.f, 0.f);
    for (int i = 0; ok && i < n; ++i) {
      const int jt = t_begin + i;
      int seg, lt;
      tile_seg<kKeyRange>(a, jt, tiles_per_seg, seg, lt);
      const int valid = min(128, seg_valid<kKeyRange>(a, seg) - lt * 128);
      const float2 ks = ks_next;
      if (i + 1 < n) ks_next = *reinterpret_cast<const float2*>(kscale_ptr(i + 1));   // prefetch
      const float c1a = __fmul_rn(__fmul_rn(qs, ks.x), a.sm_log2);
      const float c1b = __fmul_rn(__fmul_rn(qs, ks.y), a.sm_log2);
      if (!mbar_wait(&sh->s_full[t], i & 1, abort_flag, a.status, kDevTimeoutS)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[4][32];
      tmem_ld32(tS + 0, sv[0]);
      tmem_ld32(tS + 32, sv[1]);
      tmem_ld32(tS + 64, sv[2]);
      tmem_ld32(tS + 96, sv[3]);
      tmem_ld_wait();
      // refill S_t with the magic constant and let the next Q.K^T go
#pragma unroll
      for (int c = 0; c < 16; ++c) tmem_fill8(tS + 8 * c, 0x4B400000u);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&sh->s_free[t]);
      // P_t[i & 1] was last read by P.V of tile i - 2, complete since the o_done wait of tile i - 1
      uint8_t* prow = sP + (2 * t + (i & 1)) * kTile + prow_off;
      const float alpha = valid == 128 ? softmax_tile<false>(sv, 128, c1a, c1b, m, dsum, prow, rsw)
                                       : softmax_tile<true>(sv, valid, c1a, c1b, m, dsum, prow, rsw);
      fence_proxy_async_smem();
      if (i > 0) {
        if (!mbar_wait(&sh->o_done[t], (i - 1) & 1, abort_flag, a.status, kDevTimeoutO)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
          const uint64_t a2 = f2_pack(alpha, alpha);
#pragma unroll 1
          for (int c = 0; c < 4; c += 2) {     // two 32-column chunks per load/store round trip
            uint32_t ov[2][32];
            tmem_ld32(tO + 32 * c, ov[0]);
            tmem_ld32(tO + 32 * c + 32, ov[1]);
            tmem_ld_wait();
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
#pragma unroll
              for (int e = 0; e < 32; e += 2) {
                float lo, hi;
                f2_unpack(f2_mul(f2_pack(__uint_as_float(ov[h2][e]), __uint_as_float(ov[h2][e + 1])), a2), lo, hi);
                ov[h2][e] = __float_as_uint(lo);
                ov[h2][e + 1] = __float_as_uint(hi);
              }
            }
            tmem_st32(tO + 32 * c, ov[0]);
            tmem_st32(tO + 32 * c + 32, ov[1]);
          }
          tmem_st_wait();
        }
      }
      tc_fence_before();
      mbar_arrive(&sh->p_full[t]);
    }
    const bool o_ready = ok && mbar_wait(&sh->o_done[t], (n - 1) & 1, abort_flag, a.status, kDevTimeoutO);
    if constexpr (kKeyRange) {
      // warp-uniform: tcgen05.ld is a whole-warp instruction
      if (__all_sync(0xffffffffu, o_ready) && qtile * 128 < a.q_len) {
        tc_fence_after();
        store_key_partial(a, tO, sP + 2 * t * kTile, quarter, lane, qtile, bh, bhs, m, dsum);
      }
    } else if (o_ready) {
      tc_fence_after();
      if (a.num_splits == 1) {
        const float rd = __frcp_rn(dsum);
        const float* vs = a.v_scale + int64_t(bh) * 128;
        __nv_bfloat16* dst = a.out + b * a.so_b + int64_t(row) * a.so_l + h * a.so_h;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld32(tO + 32 * c, ov);
          tmem_ld_wait();
          uint32_t packed[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float o0 = __fmul_rn(__fmul_rn(__uint_as_float(ov[2 * e]), rd), vs[32 * c + 2 * e]);
            const float o1 = __fmul_rn(__fmul_rn(__uint_as_float(ov[2 * e + 1]), rd), vs[32 * c + 2 * e + 1]);
            const __nv_bfloat162 pr = __floats2bfloat162_rn(o0, o1);
            packed[e] = *reinterpret_cast<const uint32_t*>(&pr);
          }
          if (row < a.q_len) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              reinterpret_cast<uint4*>(dst + 32 * c)[e] =
                  make_uint4(packed[4 * e], packed[4 * e + 1], packed[4 * e + 2], packed[4 * e + 3]);
          }
        }
      } else {
        const int64_t prow = (int64_t(split) * bhs + bh) * a.q_pad + row;
        float* dst = a.o_part + prow * 128;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld32(tO + 32 * c, ov);
          tmem_ld_wait();
          if (row < a.q_len) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              reinterpret_cast<uint4*>(dst + 32 * c)[e] =
                  make_uint4(ov[4 * e], ov[4 * e + 1], ov[4 * e + 2], ov[4 * e + 3]);
          }
        }
        if (row < a.q_len) a.ml_part[prow] = make_float2(m, dsum);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
  // the owners of the query tiles may read this rank's partials once every CTA has stored them
  if constexpr (kKeyRange) signal_after_last_cta(a.peers, a.nranks, a.rank, a.xchg_off, xchg::kDoneAttn);
}

// Flash-decoding merge of the per-split partials (splitkv/README.md:60-69): one warp per
// (row, batch*head), 4 channels per lane.
__global__ void __launch_bounds__(128) splitkv_combine_kernel(const CombineArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + warp;
  const int bh = blockIdx.y;
  if (row >= a.q_len) return;
  const int bhs = a.batch * a.heads;
  float mx = -INFINITY;
  for (int s = 0; s < a.num_splits; ++s) mx = fmaxf(mx, a.ml_part[(int64_t(s) * bhs + bh) * a.q_pad + row].x);
  float L = 0.f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < a.num_splits; ++s) {
    const int64_t prow = (int64_t(s) * bhs + bh) * a.q_pad + row;
    const float2 ml = a.ml_part[prow];
    const float w = ml.x == -INFINITY ? 0.f : ex2_approx(ml.x - mx);
    L = fmaf(w, ml.y, L);
    const float4 p = reinterpret_cast<const float4*>(a.o_part + prow * 128)[lane];
    o.x = fmaf(w, p.x, o.x);
    o.y = fmaf(w, p.y, o.y);
    o.z = fmaf(w, p.z, o.z);
    o.w = fmaf(w, p.w, o.w);
  }
  const float rl = __frcp_rn(L);
  const float4 vs = reinterpret_cast<const float4*>(a.v_scale + int64_t(bh) * 128)[lane];
  const int b = bh / a.heads, h = bh - b * a.heads;
  const __nv_bfloat162 p0 = __floats2bfloat162_rn(o.x * rl * vs.x, o.y * rl * vs.y);
  const __nv_bfloat162 p1 = __floats2bfloat162_rn(o.z * rl * vs.z, o.w * rl * vs.w);
  uint2 st;
  st.x = *reinterpret_cast<const uint32_t*>(&p0);
  st.y = *reinterpret_cast<const uint32_t*>(&p1);
  *reinterpret_cast<uint2*>(a.out + b * a.so_b + int64_t(row) * a.so_l + h * a.so_h + lane * 4) = st;
}

// Merge of the key-range partials this rank received for its query rows: slot s holds rank s's
// O / row sum (fp16) and (max, sum) over rank s's keys; out = sum_s w_s o_s / sum_s w_s * v_scale with
// w_s = exp2(max_s - max) * sum_s (the split-KV merge of splitkv/README.md:60-69 on normalised
// partials). One warp per (row, batch*head), 4 channels per lane; every slot's loads are issued before
// any arithmetic (up to kMaxRanks slots).
__global__ void __launch_bounds__(128) keys_combine_kernel(const KeysCombineArgs a) {
  constexpr int kMax = xchg::kMaxRanks;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + warp;
  const int bh = blockIdx.y;
  if (row >= a.rows) return;
  const int64_t slot_rows = int64_t(a.batch) * a.heads * a.part;   // rows of one rank's slot
  const int64_t prow0 = int64_t(bh) * a.part + row;
  float2 ml[kMax];
  uint2 raw[kMax];
#pragma unroll
  for (int s = 0; s < kMax; ++s) {
    if (s < a.nranks) {
      ml[s] = a.recv_ml[s * slot_rows + prow0];
      raw[s] = reinterpret_cast<const uint2*>(a.recv_o + (s * slot_rows + prow0) * 128)[lane];
    } else {
      ml[s] = make_float2(-INFINITY, 0.f);
      raw[s] = make_uint2(0u, 0u);
    }
  }
  float mx = -INFINITY;
#pragma unroll
  for (int s = 0; s < kMax; ++s) mx = fmaxf(mx, ml[s].x);
  float L = 0.f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int s = 0; s < kMax; ++s) {
    const float w = ml[s].x == -INFINITY ? 0.f : ex2_approx(ml[s].x - mx) * ml[s].y;
    L += w;
    const float2 p0 = __half22float2(*reinterpret_cast<const __half2*>(&raw[s].x));
    const float2 p1 = __half22float2(*reinterpret_cast<const __half2*>(&raw[s].y));
    o.x = fmaf(w, p0.x, o.x);
    o.y = fmaf(w, p0.y, o.y);
    o.z = fmaf(w, p1.x, o.z);
    o.w = fmaf(w, p1.y, o.w);
  }
  const float rl = __frcp_rn(L);
  const float4 vs = reinterpret_cast<const float4*>(a.v_scale + int64_t(bh) * 128)[lane];
  const int b = bh / a.heads, h = bh - b * a.heads;
  const __nv_bfloat162 q0 = __floats2bfloat162_rn(o.x * rl * vs.x, o.y * rl * vs.y);
  const __nv_bfloat162 q1 = __floats2bfloat162_rn(o.z * rl * vs.z, o.w * rl * vs.w);
  uint2 st;
  st.x = *reinterpret_cast<const uint32_t*>(&q0);
  st.y = *reinterpret_cast<const uint32_t*>(&q1);
  *reinterpret_cast<uint2*>(a.out + b * a.so_b + int64_t(row) * a.so_l + h * a.so_h + lane * 4) = st;
}

template <bool kKeyRange>
cudaError_t launch_attn_variant(const AttnArgs& a, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                                const CUtensorMap& tm_v, cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(attn_fwd_kernel<kKeyRange>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(kAttnSmemBytes));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid((a.q_pad / 128 + 1) / 2, a.batch * a.heads, a.num_splits);
  if (cudaError_t e0 = prefer_max_shared<attn_fwd_kernel<kKeyRange>>(); e0 != cudaSuccess) return e0;
  attn_fwd_kernel<kKeyRange><<<grid, kAttnThreads, kAttnSmemBytes, st>>>(tm_q, tm_k, tm_v, a);
  return cudaGetLastError();
}

cudaError_t launch_attn(const AttnArgs& a, const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                        cudaStream_t st) {
  return launch_attn_variant<false>(a, tm_q, tm_k, tm_v, st);
}
cudaError_t launch_attn_keys(const AttnArgs& a, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                             const CUtensorMap& tm_v, cudaStream_t st) {
  return launch_attn_variant<true>(a, tm_q, tm_k, tm_v, st);
}

cudaError_t launch_combine(const CombineArgs& a, cudaStream_t st) {
  dim3 grid((a.q_len + 3) / 4, a.batch * a.heads);
  if (cudaError_t e0 = prefer_max_shared<splitkv_combine_kernel>(); e0 != cudaSuccess) return e0;
  splitkv_combine_kernel<<<grid, 128, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_keys_combine(const KeysCombineArgs& a, cudaStream_t st) {
  dim3 grid((a.rows + 3) / 4, a.batch * a.heads);
  if (cudaError_t e0 = prefer_max_shared<keys_combine_kernel>(); e0 != cudaSuccess) return e0;
  keys_combine_kernel<<<grid, 128, 0, st>>>(a);
  return cudaGetLastError();
}

// Address of this device's status word (looked up once per device, with that device current).
int* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  static int* ptrs[64] = {};
  if (ptrs[dev] == nullptr) {
    int* p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_status) != cudaSuccess) return nullptr;
    ptrs[dev] = p;
  }
  return ptrs[dev];
}

}  // namespace lbq
