// Quantized attention forward for sm_100a: INT8 Q.K^T and FP8 P.V on tcgen05, accumulators in
// tensor memory, operands staged by TMA, warp-specialised.
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
// CTA = one 128-row Q tile x one (batch, head) x one KV split. Warps: 0 = TMA producer,
// 1 = tcgen05 issuer (one thread), 2.. = kSoftmaxWGs softmax warpgroups. Q row r of the tile is
// TMEM lane r; warpgroup g handles keys [g*kKeys, (g+1)*kKeys) of every 128-key tile (inside one
// K scale block) and the same columns of O. The threads of a row exchange their partial row maxima
// through shared memory each tile.
// Tensor memory (512 columns): S0 [0,128), S1 [128,256) as int32 scores; columns [0,32) of each S
// buffer are overwritten by that tile's e4m3 P (4 keys per column); O f32 [256,384).
#include <cuda_bf16.h>
#include <cstdint>

#include "lbq_kernels.h"
#include "lbq_ptx.cuh"

namespace lbq {

constexpr int kStages = 4;
constexpr int kTile = 128 * 128;         // bytes of one 128 x 128 8-bit tile
#ifndef LBQ_SOFTMAX_WGS
#define LBQ_SOFTMAX_WGS 2
#endif
constexpr int kSoftmaxWGs = LBQ_SOFTMAX_WGS;   // 2 or 4 warpgroups share each 128-key tile
constexpr int kKeys = 128 / kSoftmaxWGs;       // keys (and O columns) per softmax thread
constexpr int kChunks = kKeys / 32;
constexpr int kAttnThreads = 64 + 128 * kSoftmaxWGs;
constexpr float kFp8Offset = 8.807f;     // splitkv/README.md:58 (S_FP8_OFFSET)
constexpr float kMagic = 12582912.0f;    // 1.5 * 2^23

struct AttnShared {
  uint64_t q_full;
  uint64_t k_full[kStages];
  uint64_t k_empty[kStages];
  uint64_t v_full[kStages];
  uint64_t v_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full;
  uint64_t o_done;
  uint64_t drain;
  uint64_t xchg_bar[4][2];               // per TMEM lane quarter, per tile parity: 64 arrivals
  uint32_t tmem_base;
  int abort;
  float xchg[2][kSoftmaxWGs][128];       // partial row max (tile parity, warpgroup, row); then d
};

constexpr size_t kAttnSmemBytes = 1024 /*alignment slack*/ + kTile * (1 + 2 * kStages) + sizeof(AttnShared);

__device__ int g_status;

__device__ __forceinline__ int seg_valid(const AttnArgs& a, int seg) {
  const int rest = a.kv_len - seg * a.seg_len;
  return rest < a.seg_len ? rest : a.seg_len;
}

// Of every 16 key pairs, this many take the FMA-pipe polynomial exp2 and the rest MUFU ex2:
// MUFU issues one exp per 8 clocks per SM sub-partition, so the split balances the two pipes.
#ifndef LBQ_POLY_PAIRS
#define LBQ_POLY_PAIRS 4
#endif
constexpr int kPolyPairs = LBQ_POLY_PAIRS;

// Scores -> floats by the magic-number add (S + 0x4B400000 is the float 1.5*2^23 + S for
// |S| < 2^22, and |S| <= 128*127*127 here), which keeps the conversion off the MUFU pipe; masked
// keys become -2^22. Returns the partial row max over this thread's keys in log2 units, or -inf
// when none of them is valid.
template <bool kMasked>
__device__ __forceinline__ float softmax_convert_max(uint32_t (&sv)[kChunks][32], int valid, float c1) {
  if (kMasked) {
#pragma unroll
    for (int c = 0; c < kKeys; ++c)
      if (c >= valid) sv[c >> 5][c & 31] = 0xFFC00000u;
  }
#pragma unroll
  for (int c = 0; c < kKeys; ++c) sv[c >> 5][c & 31] += 0x4B400000u;
  auto F = [&](int c) { return __uint_as_float(sv[c >> 5][c & 31]); };
  float r0 = fmaxf(F(0), F(1)), r1 = fmaxf(F(2), F(3)), r2 = fmaxf(F(4), F(5)), r3 = fmaxf(F(6), F(7));
#pragma unroll
  for (int c = 8; c < kKeys; c += 8) {
    r0 = fmax3(r0, F(c + 0), F(c + 1));
    r1 = fmax3(r1, F(c + 2), F(c + 3));
    r2 = fmax3(r2, F(c + 4), F(c + 5));
    r3 = fmax3(r3, F(c + 6), F(c + 7));
  }
  const float mh = fmax3(r0, r1, fmaxf(r2, r3));
  if (kMasked && valid <= 0) return -INFINITY;
  return __fmul_rn(mh - kMagic, c1);          // (mh - magic) is the exact integer max
}

// P = 2^(s*c1 + 8.807 - m) for this thread's keys -> e4m3 words in `pw` (key 4w in the low
// byte); returns the fp32 sum of P (masked keys contribute 0).
template <bool kMasked>
__device__ __forceinline__ float softmax_exp_pack(const uint32_t (&sv)[kChunks][32], int valid, float c1, float m,
                                                  uint32_t (&pw)[kKeys / 4]) {
  auto F = [&](int c) { return __uint_as_float(sv[c >> 5][c & 31]); };
  const float c0 = kFp8Offset - m;
  const uint64_t nmagic = f2_pack(-kMagic, -kMagic);
  const uint64_t c0x2 = f2_pack(c0, c0);
  const uint64_t c1x2 = f2_pack(c1, c1);
  uint64_t acc0 = f2_pack(0.f, 0.f), acc1 = acc0;
#pragma unroll
  for (int w = 0; w < kKeys / 4; ++w) {
    uint32_t half16[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int c = 4 * w + 2 * e;
      const uint64_t t = f2_add(f2_pack(F(c), F(c + 1)), nmagic);   // exact: the integer score
      const uint64_t x = f2_fma(t, c1x2, c0x2);                      // s - m + 8.807 (log2)
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
    pw[w] = half16[0] | (half16[1] << 16);
  }
  float s0, s1, s2, s3;
  f2_unpack(acc0, s0, s1);
  f2_unpack(acc1, s2, s3);
  return (s0 + s1) + (s2 + s3);
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kTile;
  uint8_t* sV = smem + kTile * (1 + kStages);
  AttnShared* sh = reinterpret_cast<AttnShared*>(smem + kTile * (1 + 2 * kStages));
  volatile int* abort_flag = &sh->abort;

  const int qt = blockIdx.x, bh = blockIdx.y, split = blockIdx.z;
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
    mbar_init(&sh->s_full[0], 1);
    mbar_init(&sh->s_full[1], 1);
    mbar_init(&sh->p_full, 128 * kSoftmaxWGs);
    mbar_init(&sh->o_done, 1);
    mbar_init(&sh->drain, 1);
    for (int q = 0; q < 4; ++q) {
      mbar_init(&sh->xchg_bar[q][0], 32 * kSoftmaxWGs);
      mbar_init(&sh->xchg_bar[q][1], 32 * kSoftmaxWGs);
    }
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
  const uint32_t tS0 = tmem, tS1 = tmem + 128, tO = tmem + 256;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&sh->q_full, kTile);
      tma_load_3d(sQ, &tm_q, &sh->q_full, 0, qt * 128, bh);
      int issued = 0;
      for (int i = 0; i < n; ++i) {
        const int jt = t_begin + i;
        const int seg = jt / tiles_per_seg, lt = jt - seg * tiles_per_seg;
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
      const uint64_t qdesc = smem_desc_sw128(smem_u32(sQ));
      auto issue_pv = [&](int j) -> bool {
        if (!mbar_wait(&sh->p_full, j & 1, abort_flag, a.status, kDevTimeoutP)) return false;
        const int s = j % kStages;
        if (!mbar_wait(&sh->v_full[s], (j / kStages) & 1, abort_flag, a.status, kDevTimeoutKV)) return false;
        tc_fence_after();
        const uint64_t vdesc = smem_desc_sw128(smem_u32(sV + s * kTile));
        const uint32_t tp = (j & 1) ? tS1 : tS0;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f8_ts(tO, tp + 8 * kk, vdesc + 2 * kk, kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&sh->v_empty[s]);
        tc_commit(&sh->o_done);
        return true;
      };
      for (int i = 0; ok && i < n; ++i) {
        const int s = i % kStages;
        if (!mbar_wait(&sh->k_full[s], (i / kStages) & 1, abort_flag, a.status, kDevTimeoutKV)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t kdesc = smem_desc_sw128(smem_u32(sK + s * kTile));
        const uint32_t ts = (i & 1) ? tS1 : tS0;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) mma_i8_ss(ts, qdesc + 2 * kk, kdesc + 2 * kk, kIdescQK, kk > 0 ? 1u : 0u);
        tc_commit(&sh->s_full[i & 1]);
        tc_commit(&sh->k_empty[s]);
        if (i > 0) ok = issue_pv(i - 1);
      }
      if (ok) issue_pv(n - 1);
      // Drain: every MMA issued above has completed once `drain` flips.
      tc_commit(&sh->drain);
      mbar_drain_wait(&sh->drain, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    const int wg = (warp - 2) >> 2;                     // key slice / O column slice
    const int quarter = warp & 3;                       // TMEM lanes [32*quarter, 32*quarter+32)
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const int trow = quarter * 32 + lane;               // row inside the Q tile
    const int row = qt * 128 + trow;
    const int col0 = wg * kKeys;
    const float qs = a.q_scale[int64_t(bh) * (a.q_pad / 32) + qt * 4 + quarter];
    const int kspb = a.seg_pad / 64;
    float m = -INFINITY, dsum = 0.f;
    bool ok = n > 0;
    for (int i = 0; ok && i < n; ++i) {
      const int jt = t_begin + i;
      const int seg = jt / tiles_per_seg, lt = jt - seg * tiles_per_seg;
      const int valid = min(128, seg_valid(a, seg) - lt * 128) - col0;   // keys of my slice
      const float c1 =
          __fmul_rn(__fmul_rn(qs, a.k_scale[int64_t(seg * bhs + bh) * kspb + lt * 2 + col0 / 64]), a.sm_log2);
      if (!mbar_wait(&sh->s_full[i & 1], (i >> 1) & 1, abort_flag, a.status, kDevTimeoutS)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t ts = ((i & 1) ? tS1 : tS0) + lane_off;
      uint32_t sv[kChunks][32];
#pragma unroll
      for (int c = 0; c < kChunks; ++c) tmem_ld32(ts + col0 + 32 * c, sv[c]);
      tmem_ld_wait();
      const bool masked = valid < kKeys;
      const float tmax = masked ? softmax_convert_max<true>(sv, valid, c1) : softmax_convert_max<false>(sv, kKeys, c1);
      // exchange the partial row max with the other warpgroup's thread of this row
      sh->xchg[i & 1][wg][trow] = tmax;
      mbar_arrive(&sh->xchg_bar[quarter][i & 1]);
      if (!mbar_wait(&sh->xchg_bar[quarter][i & 1], (i >> 1) & 1, abort_flag, a.status, kDevTimeoutS)) {
        ok = false;
        break;
      }
      float m_new = fmaxf(m, tmax);
#pragma unroll
      for (int g = 0; g < kSoftmaxWGs; ++g) m_new = fmaxf(m_new, sh->xchg[i & 1][g][trow]);
      const float alpha = (m == m_new) ? 1.f : ex2_approx(m - m_new);
      m = m_new;
      uint32_t pw[kKeys / 4];
      const float psum =
          masked ? softmax_exp_pack<true>(sv, valid, c1, m, pw) : softmax_exp_pack<false>(sv, kKeys, c1, m, pw);
      dsum = __fmaf_rn(dsum, alpha, psum);
      tmem_st(((i & 1) ? tS1 : tS0) + lane_off + col0 / 4, pw);
      tmem_st_wait();
      if (i > 0) {
        if (!mbar_wait(&sh->o_done, (i - 1) & 1, abort_flag, a.status, kDevTimeoutO)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < kChunks; ++c) {
            uint32_t ov[32];
            const uint32_t ta = tO + lane_off + col0 + 32 * c;
            tmem_ld32(ta, ov);
            tmem_ld_wait();
            const uint64_t a2 = f2_pack(alpha, alpha);
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              float lo, hi;
              f2_unpack(f2_mul(f2_pack(__uint_as_float(ov[e]), __uint_as_float(ov[e + 1])), a2), lo, hi);
              ov[e] = __float_as_uint(lo);
              ov[e + 1] = __float_as_uint(hi);
            }
            tmem_st32(ta, ov);
          }
          tmem_st_wait();
        }
      }
      tc_fence_before();
      mbar_arrive(&sh->p_full);
    }
    if (ok && mbar_wait(&sh->o_done, (n - 1) & 1, abort_flag, a.status, kDevTimeoutO)) {
      tc_fence_after();
      // row sum = the warpgroups' partial sums (same order in every thread of the row)
      const int par = n & 1;
      sh->xchg[par][wg][trow] = dsum;
      mbar_arrive(&sh->xchg_bar[quarter][par]);
      if (mbar_wait(&sh->xchg_bar[quarter][par], (n >> 1) & 1, abort_flag, a.status, kDevTimeoutS)) {
        float dtot = 0.f;
#pragma unroll
        for (int g = 0; g < kSoftmaxWGs; ++g) dtot += sh->xchg[par][g][trow];
        if (a.num_splits == 1) {
          const float rd = __frcp_rn(dtot);
          const float* vs = a.v_scale + int64_t(bh) * 128 + col0;
          __nv_bfloat16* dst = a.out + b * a.so_b + int64_t(row) * a.so_l + h * a.so_h + col0;
#pragma unroll 1
          for (int c = 0; c < kChunks; ++c) {
            uint32_t ov[32];
            tmem_ld32(tO + lane_off + col0 + 32 * c, ov);
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
          float* dst = a.o_part + prow * 128 + col0;
#pragma unroll 1
          for (int c = 0; c < kChunks; ++c) {
            uint32_t ov[32];
            tmem_ld32(tO + lane_off + col0 + 32 * c, ov);
            tmem_ld_wait();
            if (row < a.q_len) {
#pragma unroll
              for (int e = 0; e < 8; ++e)
                reinterpret_cast<uint4*>(dst + 32 * c)[e] =
                    make_uint4(ov[4 * e], ov[4 * e + 1], ov[4 * e + 2], ov[4 * e + 3]);
            }
          }
          if (wg == 0 && row < a.q_len) a.ml_part[prow] = make_float2(m, dtot);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
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

cudaError_t launch_attn(const AttnArgs& a, const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                        cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kAttnSmemBytes));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid(a.q_pad / 128, a.batch * a.heads, a.num_splits);
  attn_fwd_kernel<<<grid, kAttnThreads, kAttnSmemBytes, st>>>(tm_q, tm_k, tm_v, a);
  return cudaGetLastError();
}

cudaError_t launch_combine(const CombineArgs& a, cudaStream_t st) {
  dim3 grid((a.q_len + 3) / 4, a.batch * a.heads);
  splitkv_combine_kernel<<<grid, 128, 0, st>>>(a);
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
