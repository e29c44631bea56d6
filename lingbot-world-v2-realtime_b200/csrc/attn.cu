// Quantized attention forward for sm_100a: INT8 Q.K^T and FP8 P.V on tcgen05, accumulators in tensor
// memory, operands staged by TMA, warp-specialised, two Q tiles per CTA.
//
// Semantics are those of SageAttention-2's `qk_int8_sv_f8_accum_f16_fuse_v_scale_attn_inst_buf` as
// the reference calls it (lingbot/layers/sage_preq.py:126-127 with qk_quant_gran=2: one Q scale per
// 32 rows; experiments/bench_attn/splitkv/README.md:51-69, h2_tiles/cfg_fusedsoftmax.patch:89-160),
// with its tile size and fp32 arithmetic order. The keys run in 64-key tiles (Sage's CTA_K). For a
// row with Q scale q_s and a tile with K scale k_s, S = q_i8 . k_i8 (exact int32), sm = fl(sm_scale
// * log2 e), dq = fl(q_s * k_s):
//   main tiles:        c = fl(sm * dq);  m_t = fma(max S, c, -8.807);  x = fma(S, c, -m)
//   last two tiles:    r = fl(S * dq);   m_t = fma(max r, sm, -8.807); x = fma(r, sm, -m)
//                      (upstream's last two iterations run on dequantized scores with
//                      original_sm_scale, h2_tiles/cfg_fixedmax.patch:307,329)
//   m = max(m_prev, m_t); alpha = exp2(m_prev - m); P = exp2(x) (<= 448) -> e4m3
//   d = d * alpha + sum(P) (fp32, before rounding);  O = O * alpha + e4m3(P) . e4m3(V)
//   out = O / d * v_scale -> bf16
// exp2 is ex2.approx (upstream's ptx_exp2). Differences from the sm89 kernel: P.V accumulates in fp32 in
// tensor memory where Sage sums each 64-key tile in fp16; and in the bulk tiles (full 128-key tiles
// other than the last two 64-key tiles) x is fma(1.5*2^23 + S, c, fl(-1.5*2^23 * c - m)) where
// 1.5*2^23 * c < 4096 (within 2^-13 of upstream's x), where also 2 of every 16 key pairs take a
// degree-3 polynomial exp2 (relative error 7.5e-5). Both can move a P across an e4m3 rounding midpoint
// only when it lies that close to one; the masked and last two tiles, where few keys carry the row, are
// exact.
//
// CTA = two 128-row Q tiles (A, B) x one (batch, head) x one KV split, 512 threads:
//   warps 0-3   softmax of tile A, warps 4-7 softmax of tile B: one thread per row (= TMEM lane);
//   warps 8-11  correction: O_t *= alpha before each 64-key P.V, then the epilogue of both tiles;
//   warp 12     TMA producer of both Q tiles (once) and of K in 128-key stages through a ring;
//   warp 15     TMA producer of V^T (its own ring, so K can run ahead of V);
//   warp 13     Q.K^T issuer and tensor-memory owner, warp 14 P.V issuer: two issuing warps, so that the
//               scores of the next key tile never wait behind the P.V chain (each issues under
//               elect.sync; they touch disjoint tensor memory and hand buffers back by barrier).
// Q.K^T runs on 128 keys (one MMA of N = 128 per 32 channels); the softmax takes the two 64-key halves
// of the score tile in turn, each against the running max after the previous half, and P.V runs per
// half (K = 64), the correction warps rescaling O between the two products when the second half
// raised a row's max. Tensor memory (512 columns): S_A [0,128), S_B [128,256) int32 scores, O_A
// [256,384), O_B [384,512) fp32. After reading S_t a softmax warp refills it with 0x4B400000, the bits
// of the float 1.5*2^23, and the next Q.K^T accumulates onto that: the int32 accumulator then holds the
// bits of the float 1.5*2^23 + S (|S| <= 128*127*127 < 2^21), so S needs one exact subtraction and no
// conversion. The refill completes during the first half's softmax, after which the Q.K^T of the next
// key tile runs during the second half. P (e4m3) goes to a double-buffered shared-memory tile
// (128-byte-swizzled K-major rows), the A operand of P.V; the P.V issuer hands a P buffer back with its
// own barrier, so Q.K^T may run ahead of the P.V products.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "lbq_kernels.h"
#include "lbq_peer.cuh"
#include "lbq_ptx.cuh"

namespace lbq {

constexpr int kStages = 2;               // K and V^T stages (128 keys each)
constexpr int kPBufs = 3;                // P buffers per Q tile: the P.V of a tile may finish two tiles late
__device__ __forceinline__ int pbuf(int j) { return j % kPBufs; }
__device__ __forceinline__ uint32_t pphase(int j) { return (j / kPBufs) & 1; }
constexpr int kTile = 128 * 128;         // bytes of a Q tile, a P tile and a 128-key K or V^T stage
constexpr int kAttnThreads = 512;
constexpr float kFp8Offset = 8.807f;     // splitkv/README.md:58 (S_FP8_OFFSET)
constexpr float kMagic = 12582912.0f;    // 1.5 * 2^23
constexpr uint32_t kMagicBits = 0x4B400000u;
constexpr uint32_t kMaskedBits = 0x4B000000u;   // 1.5*2^23 - 2^22: below every real score
constexpr uint32_t kColS = 0, kColO = 256;
// Registers per thread after the split (launched with 128; a warpgroup's share times 128 threads, summed
// over the four warpgroups, must stay within 512 x 128 or setmaxnreg.inc would wait for good). One-pass
// kernel: softmax 184, correction 104, producers and issuers 40 — the split at which ptxas reports no
// spills (measured 1179 -> 1189 TOPS against 160/120/72). Key-range kernel: 160/120/72 (184/104/40
// spills 436 bytes there; 168/120/56, measured, is 0.5 % slower).
template <bool kKeyRange>
struct RegSplit {
  static constexpr uint32_t softmax = kKeyRange ? 160 : 184;
  static constexpr uint32_t correction = kKeyRange ? 120 : 104;
  static constexpr uint32_t misc = kKeyRange ? 72 : 40;
  static_assert(128 * (2 * softmax + correction + misc) <= kAttnThreads * 128, "register split");
};

// In the bulk tiles with the folded exp2 argument, of every 16 key pairs this many take the FMA-pipe
// polynomial exp2 (relative error 7.5e-5) instead of MUFU ex2, the busiest unit (measured: 2 of 16 is
// the fastest split; with the exact argument, MUFU for every key is faster).
constexpr int kPolyPairs = 2;

struct AttnShared {
  uint64_t q_full;
  uint64_t k_full[kStages];
  uint64_t k_empty[kStages];
  uint64_t v_full[kStages];
  uint64_t v_empty[kStages];
  uint64_t s_full[2];                    // per Q tile: Q.K^T of the next 128-key tile complete
  uint64_t s_read[2];                    // S read (128 softmax threads): the correction warps refill it
  uint64_t s_free[2];                    // S refilled with the magic constant (128 correction threads)
  uint64_t p_full[2][kPBufs];            // [tile][pbuf(j)]: P of key tile j in shared memory, its alphas
                                         // written (128 softmax threads); one per buffer, since the softmax
                                         // may run key tiles ahead of the correction
  uint64_t o_ready[2];                   // O_t rescaled for the next 64-key P.V (128 correction threads)
  uint64_t o_done[2];                    // P.V complete
  uint64_t ml_full[2];                   // final (m, d) of every row in `ml`
  uint64_t drain_qk, drain_pv;           // each issuer's MMAs complete
  uint32_t tmem_base;
  int abort;
  float alpha[2][kPBufs][2][128];        // [Q tile][pbuf(j)][64-key half][row]
  float2 ml[2][128];                     // [Q tile][row]
};

// smem: Q_A, Q_B | P_A[kPBufs], P_B[kPBufs] | K stages | V stages | AttnShared
constexpr int kSmemTiles = 2 + 2 * kPBufs + 2 * kStages;
constexpr size_t kAttnSmemBytes = 1024 /*alignment slack*/ + kTile * kSmemTiles + sizeof(AttnShared);

__device__ int g_status;

template <bool kKeyRange>
__device__ __forceinline__ int seg_valid(const AttnArgs& a, int seg) {
  if constexpr (kKeyRange) return a.range_valid[seg];
  const int rest = a.kv_len - seg * a.seg_len;
  return rest < a.seg_len ? rest : a.seg_len;
}

// Walks the CTA's 128-key tiles in order, tracking (code segment, tile inside the segment) without a
// division per step. Key-range mode: the tile sequence is the pieces of AttnArgs::range_*.
template <bool kKeyRange>
struct TileWalk {
  int jt, seg, lt;
  __device__ __forceinline__ TileWalk(const AttnArgs& a, int jt0, int tiles_per_seg) : jt(jt0) {
    if constexpr (kKeyRange) {
      seg = jt0 >= a.range_tile0[1] ? 1 : 0;
      lt = jt0 - a.range_tile0[seg] + a.range_lt0[seg];
    } else {
      seg = jt0 / tiles_per_seg;
      lt = jt0 - seg * tiles_per_seg;
    }
  }
  __device__ __forceinline__ void next(const AttnArgs& a, int tiles_per_seg) {
    ++jt;
    if constexpr (kKeyRange) {
      if (jt == a.range_tile0[1]) {
        seg = 1;
        lt = a.range_lt0[1];
      } else {
        ++lt;
      }
    } else if (++lt == tiles_per_seg) {
      ++seg;
      lt = 0;
    }
  }
  // valid keys of this tile (1..128)
  __device__ __forceinline__ int valid(const AttnArgs& a) const {
    return min(128, seg_valid<kKeyRange>(a, seg) - lt * 128);
  }
};

// Softmax of one 64-key tile for the calling thread's row, for the tiles the fused 128-key pass does not
// take: a masked tile (keys >= `valid` are not in the window) or one of upstream's last two (`tail`).
// `sv` holds the scores as the bits of 1.5*2^23 + S. Writes the e4m3 P of the 64 keys to `pw` (word w =
// keys 4w..4w+3, key 4w in the low byte), updates `m` and `dsum`, returns alpha.
__device__ __forceinline__ float softmax_sub(uint32_t* sv, int valid, bool tail, float c, float dq, float sm,
                                             float& m, float& dsum, uint32_t (&pw)[16]) {
#pragma unroll
  for (int j = 0; j < 64; ++j)
    if (j >= valid) sv[j] = kMaskedBits;
  auto F = [&](int j) { return __uint_as_float(sv[j]); };
  float r0 = fmaxf(F(0), F(1)), r1 = fmaxf(F(2), F(3)), r2 = fmaxf(F(4), F(5)), r3 = fmaxf(F(6), F(7));
#pragma unroll
  for (int j = 8; j < 64; j += 8) {
    r0 = fmax3(r0, F(j + 0), F(j + 1));
    r1 = fmax3(r1, F(j + 2), F(j + 3));
    r2 = fmax3(r2, F(j + 4), F(j + 5));
    r3 = fmax3(r3, F(j + 6), F(j + 7));
  }
  const float smax = fmax3(r0, r1, fmaxf(r2, r3)) - kMagic;       // exact integer max score
  // main tiles: x = fma(S, c, -m); the last two: x = fma(fl(S * dq), sm, -m). Both as S * mul, then fma.
  const float mul = tail ? dq : 1.f, scl = tail ? sm : c;
  const float m_t = __fmaf_rn(__fmul_rn(smax, mul), scl, -kFp8Offset);
  const float m_new = fmaxf(m, m_t);
  const float alpha = (m == m_new) ? 1.f : ex2_approx(m - m_new);
  m = m_new;
  const uint64_t negm2 = f2_pack(-m_new, -m_new), nk2 = f2_pack(-kMagic, -kMagic);
  const uint64_t mul2 = f2_pack(mul, mul), scl2 = f2_pack(scl, scl);
  uint64_t acc0 = f2_pack(0.f, 0.f), acc1 = acc0;
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    uint32_t half16[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = 4 * w + 2 * e;
      const uint64_t s2 = f2_add(f2_pack(F(j), F(j + 1)), nk2);   // S, exact
      const uint64_t x = f2_fma(f2_mul(s2, mul2), scl2, negm2);    // S * 1 is exact
      float x0, x1;
      f2_unpack(x, x0, x1);
      float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
      if (j >= valid) p0 = 0.f;
      if (j + 1 >= valid) p1 = 0.f;
      const uint64_t p = f2_pack(p0, p1);
      if (e == 0) acc0 = f2_add(acc0, p); else acc1 = f2_add(acc1, p);
      half16[e] = pack_e4m3x2(p0, p1);
    }
    pw[w] = half16[0] | (half16[1] << 16);
  }
  float s0, s1, s2, s3;
  f2_unpack(acc0, s0, s1);
  f2_unpack(acc1, s2, s3);
  dsum = __fadd_rn(__fmul_rn(dsum, alpha), (s0 + s1) + (s2 + s3));
  return alpha;
}

// One 64-key half of the softmax on the masked / tail path; the P words go to chunks 4h..4h+3 of this row
// of the shared P tile (16-byte chunk c at c ^ (row & 7): the 128-byte swizzle of the MMA operand).
__device__ __forceinline__ float softmax_half(uint32_t* sv, int valid, bool tail, float c, float dq, float sm,
                                              float& m, float& dsum, uint8_t* prow, int h, int rsw) {
  uint32_t pw[16];
  const float alpha = softmax_sub(sv, valid, tail, c, dq, sm, m, dsum, pw);
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<uint4*>(prow + (((4 * h + q) ^ rsw) << 4)) =
        make_uint4(pw[4 * q], pw[4 * q + 1], pw[4 * q + 2], pw[4 * q + 3]);
  return alpha;
}

// Softmax of a whole 128-key tile (two 64-key tiles, neither masked nor in upstream's tail) for the
// calling thread's row, in two steps: tile128_max takes the maxima of both halves, tile128_exp every
// exp2, so that the second half's max does not wait for the first half's exponentials. The arithmetic is
// softmax_sub's on each half in turn (the second against the running max after the first), with the
// folded exp2 argument and the polynomial pairs described at the top of this file. P goes to
// chunks 0..7 of this row of the shared P tile; tile128_exp returns the two alphas.
__device__ __forceinline__ float2 tile128_max(const uint32_t* sv) {
  auto F = [&](int j) { return __uint_as_float(sv[j]); };
  float r[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) r[q] = fmaxf(F(8 * (q >> 2) * 8 + 2 * (q & 3)), F(8 * (q >> 2) * 8 + 2 * (q & 3) + 1));
#pragma unroll
  for (int j = 8; j < 64; j += 8) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      r[q] = fmax3(r[q], F(j + 2 * q), F(j + 2 * q + 1));
      r[4 + q] = fmax3(r[4 + q], F(64 + j + 2 * q), F(64 + j + 2 * q + 1));
    }
  }
  return make_float2(fmax3(r[0], r[1], fmaxf(r[2], r[3])) - kMagic, fmax3(r[4], r[5], fmaxf(r[6], r[7])) - kMagic);
}
// The fold (below) is taken where its argument error is small: 1.5*2^23 * c < kFoldMax bounds |b| near
// 4096, so x is within 2^-13 of upstream's. c is uniform over a warp (one Q scale per 32 rows, one K
// scale per 64 keys), so the choice is too.
constexpr float kFoldMax = 4096.f;

// kFold: x = fma(f, c, b) with f = 1.5*2^23 + S and b = fl(-1.5*2^23 * c - m), the exact subtraction of
// the magic bias folded into the exp2 argument (one FFMA2 per key pair; x is within half an ulp of |b|
// of upstream's fma(S, c, -m)). Otherwise S = f - 1.5*2^23 exactly, then x = fma(S, c, -m) as upstream.
template <bool kFold>
__device__ __forceinline__ float2 tile128_exp(const uint32_t* sv, float2 smax, float c0, float c1, float& m,
                                              float& dsum, uint8_t* prow, int rsw) {
  auto F = [&](int j) { return __uint_as_float(sv[j]); };
  const float m1 = fmaxf(m, __fmaf_rn(smax.x, c0, -kFp8Offset));
  const float m2 = fmaxf(m1, __fmaf_rn(smax.y, c1, -kFp8Offset));
  const float alpha1 = (m == m1) ? 1.f : ex2_approx(m - m1);
  const float alpha2 = (m1 == m2) ? 1.f : ex2_approx(m1 - m2);
  m = m2;
  const float b1 = kFold ? __fmaf_rn(-kMagic, c0, -m1) : -m1, b2 = kFold ? __fmaf_rn(-kMagic, c1, -m2) : -m2;
  const uint64_t nk2 = f2_pack(-kMagic, -kMagic);
  uint64_t acc[4] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f), f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
  uint32_t pw[4];
#pragma unroll
  for (int w = 0; w < 32; ++w) {
    const int hh = w >> 4;
    const uint64_t c2 = hh ? f2_pack(c1, c1) : f2_pack(c0, c0);
    const uint64_t b2x = hh ? f2_pack(b2, b2) : f2_pack(b1, b1);
    uint32_t half16[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = 4 * w + 2 * e;
      const uint64_t f = f2_pack(F(j), F(j + 1));
      const uint64_t x = kFold ? f2_fma(f, c2, b2x) : f2_fma(f2_add(f, nk2), c2, b2x);
      float x0, x1;
      f2_unpack(x, x0, x1);
      uint64_t p;
      if (kFold && ((j >> 1) & 15) >= 16 - kPolyPairs) {
        p = exp2_poly_x2(x0, x1);
      } else {
        p = f2_pack(ex2_approx(x0), ex2_approx(x1));
      }
      float p0, p1;
      f2_unpack(p, p0, p1);
      acc[2 * hh + e] = f2_add(acc[2 * hh + e], p);
      half16[e] = pack_e4m3x2(p0, p1);
    }
    pw[w & 3] = half16[0] | (half16[1] << 16);
    if ((w & 3) == 3)   // 16 keys done: one swizzled 16-byte chunk of the row
      *reinterpret_cast<uint4*>(prow + (((w >> 2) ^ rsw) << 4)) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
  }
  float s[8];
#pragma unroll
  for (int q = 0; q < 4; ++q) f2_unpack(acc[q], s[2 * q], s[2 * q + 1]);
  dsum = __fadd_rn(__fmul_rn(dsum, alpha1), (s[0] + s[1]) + (s[2] + s[3]));
  dsum = __fadd_rn(__fmul_rn(dsum, alpha2), (s[4] + s[5]) + (s[6] + s[7]));
  return make_float2(alpha1, alpha2);
}

// Key-range epilogue of one correction warp: its 32 rows of O / row sum as fp16 (V-code units, |x| <=
// 448) are staged in `stage` (32 KB of free shared memory; 16-byte chunks of a 256-byte row XOR-swizzled
// by row) and stored to the owner rank's receive slot for this rank as whole rows, two rows per warp
// instruction; the (max, sum) of each row follows. Rows past q_len are not stored.
__device__ __forceinline__ void store_key_partial(const AttnArgs& a, uint32_t tO, uint8_t* stage, int quarter,
                                                  int lane, int qtile, int bh, int bhs, float m, float dsum) {
  const float rd = __frcp_rn(dsum);
  const int rl = quarter * 32 + lane;                    // row inside the tile (TMEM lane)
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t ov[32];
    tmem_ld32(tO + 32 * c, ov);
    tmem_ld_wait(ov);
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

// O_t *= alpha for the calling warp's 32 TMEM lanes (two 64-column load/store round trips).
__device__ __forceinline__ void rescale_o(uint32_t tO, float alpha) {
  const uint64_t a2 = f2_pack(alpha, alpha);
#pragma unroll 1
  for (int c = 0; c < 4; c += 2) {
    uint32_t ov[2][32];
    tmem_ld32(tO + 32 * c, ov[0]);
    tmem_ld32(tO + 32 * c + 32, ov[1]);
    tmem_ld_wait(ov[0]);
    reg_anchor(ov[1]);
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
  uint8_t* sK = smem + kTile * (2 + 2 * kPBufs);   // [kStages][kTile]
  uint8_t* sV = sK + kTile * kStages;              // [kStages][kTile]
  AttnShared* sh = reinterpret_cast<AttnShared*>(smem + kTile * kSmemTiles);
  volatile int* abort_flag = &sh->abort;

  const int qp = blockIdx.x, bh = blockIdx.y, split = blockIdx.z;   // qp: pair of 128-row Q tiles
  const int b = bh / a.heads, h = bh - b * a.heads;
  const int t_begin = split * a.tiles_per_split;
  const int t_end = min(t_begin + a.tiles_per_split, a.total_tiles);
  const int n = t_end - t_begin;                   // 128-key tiles of this CTA
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
      mbar_init(&sh->s_read[t], 128);
      mbar_init(&sh->s_free[t], 128);
      for (int pb = 0; pb < kPBufs; ++pb) {
        mbar_init(&sh->p_full[t][pb], 128);
      }
      mbar_init(&sh->o_ready[t], 128);
      mbar_init(&sh->o_done[t], 1);
      mbar_init(&sh->ml_full[t], 128);
    }
    mbar_init(&sh->drain_qk, 1);
    mbar_init(&sh->drain_pv, 1);
    sh->abort = 0;
    fence_mbar_init();
  }
  if (warp == 13) {
    tmem_alloc(&sh->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp >= 12) {
    reg_dealloc<RegSplit<kKeyRange>::misc>();
    if (warp == 12 && n > 0) {
      // ---------------------------------------------------------- TMA producer of Q and K (one lane issues)
      if (elect_one()) {
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        // Both Q tiles; a tile past q_pad reads the map's out-of-bounds zero fill.
        mbar_arrive_expect_tx(&sh->q_full, 2 * kTile);
        tma_load_3d(sQ, &tm_q, &sh->q_full, 0, (2 * qp) * 128, bh);
        tma_load_3d(sQ + kTile, &tm_q, &sh->q_full, 0, (2 * qp + 1) * 128, bh);
      }
      int issued = 0;
      TileWalk<kKeyRange> tw(a, t_begin, tiles_per_seg);
      for (int i = 0; i < n; ++i, tw.next(a, tiles_per_seg)) {
        (void)LBQ_CHECK(tw.seg < a.nseg && tw.lt >= 0 && tw.lt < tiles_per_seg, a.status, kDevBadTile);
        const int s = i % kStages;
        if (!mbar_wait_role(&sh->k_empty[s], ((i / kStages) & 1) ^ 1, abort_flag, a.status, kDevTimeoutKV)) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&sh->k_full[s], kTile);
          tma_load_3d(sK + s * kTile, &tm_k, &sh->k_full[s], 0, tw.lt * 128, tw.seg * bhs + bh);
        }
        __syncwarp();
        issued = i + 1;
      }
      if (*abort_flag) {
        // Let copies already in flight land before the CTA's shared memory goes away.
        mbar_drain_wait(&sh->q_full, 0);
        for (int i = (issued > kStages ? issued - kStages : 0); i < issued; ++i)
          mbar_drain_wait(&sh->k_full[i % kStages], (i / kStages) & 1);
      }
    } else if (warp == 15 && n > 0) {
      // ---------------------------------------------------------- TMA producer of V^T (one lane issues)
      if (elect_one()) tma_prefetch_desc(&tm_v);
      int issued = 0;
      TileWalk<kKeyRange> tw(a, t_begin, tiles_per_seg);
      for (int i = 0; i < n; ++i, tw.next(a, tiles_per_seg)) {
        const int s = i % kStages;
        if (!mbar_wait_role(&sh->v_empty[s], ((i / kStages) & 1) ^ 1, abort_flag, a.status, kDevTimeoutKV)) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&sh->v_full[s], kTile);
          tma_load_3d(sV + s * kTile, &tm_v, &sh->v_full[s], tw.lt * 128, 0, tw.seg * bhs + bh);
        }
        __syncwarp();
        issued = i + 1;
      }
      if (*abort_flag) {
        for (int i = (issued > kStages ? issued - kStages : 0); i < issued; ++i)
          mbar_drain_wait(&sh->v_full[i % kStages], (i / kStages) & 1);
      }
    } else if (warp == 13 && n > 0) {
      // ---------------------------------------------------------- Q.K^T issuer (one lane issues)
      // S_t(k) = Q_t . K(k)^T for both tiles once S_t(k - 1) was read and refilled (k = 0: the initial
      // fill), onto the magic constant the softmax left in S_t. Runs ahead of the P.V products.
      bool ok = mbar_wait_role(&sh->q_full, 0, abort_flag, a.status, kDevTimeoutQ);
      tc_fence_after();
      const uint64_t qdesc[2] = {smem_desc_sw128(smem_u32(sQ)), smem_desc_sw128(smem_u32(sQ + kTile))};
      const uint64_t kdesc0 = smem_desc_sw128(smem_u32(sK));
      constexpr uint64_t kTileDesc = kTile >> 4;        // one tile in descriptor address units
      for (int k = 0; ok && k < n; ++k) {
        const int s = k % kStages;
        if (!(ok = mbar_wait_role(&sh->k_full[s], (k / kStages) & 1, abort_flag, a.status, kDevTimeoutKV))) break;
        const uint64_t kdesc = kdesc0 + s * kTileDesc;
        for (int t = 0; ok && t < 2; ++t) {
          // polled without sleeping: the refill -> Q.K^T hand-off is on the softmax's path
          if (!(ok = mbar_wait(&sh->s_free[t], k & 1, abort_flag, a.status, kDevTimeoutS))) break;
          tc_fence_after();
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_i8_ss(tmem + kColS + 128 * t, qdesc[t] + 2 * kk, kdesc + 2 * kk, kIdescQK, 1u);
            tc_commit(&sh->s_full[t]);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) tc_commit(&sh->k_empty[s]);
        __syncwarp();
      }
      // Drain: every MMA this warp issued has completed once `drain_qk` flips.
      if (elect_one()) tc_commit(&sh->drain_qk);
      __syncwarp();
      mbar_drain_wait(&sh->drain_qk, 0);
    } else if (warp == 14 && n > 0) {
      // ---------------------------------------------------------- P.V issuer (one lane issues)
      // O_t (+)= P_t(j, hh) . V(j, hh) per 64-key half once the softmax wrote P and the correction
      // rescaled O_t; P buffer pbuf(j) and V stage j are handed back after the tile's last product.
      const uint64_t vdesc0 = smem_desc_sw128(smem_u32(sV)), pdesc0 = smem_desc_sw128(smem_u32(sP));
      constexpr uint64_t kTileDesc = kTile >> 4;
      bool ok = true;
      TileWalk<kKeyRange> tw(a, t_begin, tiles_per_seg);
      int u = 0;                                        // P.V products issued per Q tile
      for (int j = 0; ok && j < n; ++j, tw.next(a, tiles_per_seg)) {
        const int ns = tw.valid(a) > 64 ? 2 : 1;       // 64-key halves of tile j
        const int s = j % kStages;
        if (!(ok = mbar_wait_role(&sh->v_full[s], (j / kStages) & 1, abort_flag, a.status, kDevTimeoutKV))) break;
        const uint64_t vdesc = vdesc0 + s * kTileDesc;
        for (int hh = 0; ok && hh < ns; ++hh, ++u) {
          for (int t = 0; t < 2; ++t) {
            // polled without sleeping (measured 1172 -> 1181 TOPS against the 64 ns sleep of the producers)
            if (!(ok = mbar_wait(&sh->o_ready[t], u & 1, abort_flag, a.status, kDevTimeoutP))) break;
            tc_fence_after();
            const uint64_t pdesc = pdesc0 + (kPBufs * t + pbuf(j)) * kTileDesc + 4 * hh;
            if (elect_one()) {
#pragma unroll
              for (int kk = 0; kk < 2; ++kk)
                mma_f8_ss(tmem + kColO + 128 * t, pdesc + 2 * kk, vdesc + 4 * hh + 2 * kk, kIdescPV,
                          (u > 0 || kk > 0) ? 1u : 0u);
              tc_commit(&sh->o_done[t]);
            }
            __syncwarp();
          }
        }
        if (!ok) break;
        if (elect_one()) {
          tc_commit(&sh->v_empty[s]);
        }
        __syncwarp();
      }
      // Drain: every MMA this warp issued has completed once `drain_pv` flips.
      if (elect_one()) tc_commit(&sh->drain_pv);
      __syncwarp();
      mbar_drain_wait(&sh->drain_pv, 0);
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ softmax warpgroups
    reg_alloc<RegSplit<kKeyRange>::softmax>();
    const int t = warp >> 2;                            // Q tile of this warpgroup
    const int quarter = warp & 3;                       // TMEM lanes [32*quarter, 32*quarter+32)
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const uint32_t tS = tmem + kColS + 128 * t + lane_off;
    const int qtile = 2 * qp + t;
    const int rl = quarter * 32 + lane;
    const float qs = qtile * 128 < a.q_pad ? a.q_scale[int64_t(bh) * (a.q_pad / 32) + qtile * 4 + quarter] : 0.f;
    const float sm = a.sm_log2;
    const int kspb = a.seg_pad / 64;
    const int prow_off = rl * 128;
    const int rsw = lane & 7;                           // row & 7 (rows of a warp start at 32k)
    float m = -INFINITY, dsum = 0.f;
    bool ok = n > 0;
    TileWalk<kKeyRange> tw(a, t_begin, tiles_per_seg);
    auto kscale_ptr = [&](const TileWalk<kKeyRange>& w) {
      int seg = w.seg, lt = w.lt;
      if (!LBQ_CHECK(seg < a.nseg && lt >= 0 && lt * 2 + 1 < kspb, a.status, kDevBadTile)) seg = lt = 0;
      return a.k_scale + int64_t(seg * bhs + bh) * kspb + lt * 2;
    };
    // the last two 64-key tiles take upstream's tail arithmetic
    int ns_last = 0;
    if (ok) {
      TileWalk<kKeyRange> tl(a, t_end - 1, tiles_per_seg);
      ns_last = tl.valid(a) > 64 ? 2 : 1;
    }
    float2 ks_next = ok ? *reinterpret_cast<const float2*>(kscale_ptr(tw)) : make_float2(0.f, 0.f);
    for (int j = 0; ok && j < n; ++j) {
      const int tv = tw.valid(a);
      const float2 ks = ks_next;
      if (j + 1 < n) {                                  // prefetch the next tile's K scales
        tw.next(a, tiles_per_seg);
        ks_next = *reinterpret_cast<const float2*>(kscale_ptr(tw));
      }
      if (!mbar_wait(&sh->s_full[t], j & 1, abort_flag, a.status, kDevTimeoutS)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[128];
      auto& sv0 = *reinterpret_cast<uint32_t(*)[32]>(sv);
      auto& sv1 = *reinterpret_cast<uint32_t(*)[32]>(sv + 32);
      auto& sv2 = *reinterpret_cast<uint32_t(*)[32]>(sv + 64);
      auto& sv3 = *reinterpret_cast<uint32_t(*)[32]>(sv + 96);
      tmem_ld32(tS + 0, sv0);
      tmem_ld32(tS + 32, sv1);
      tmem_ld32(tS + 64, sv2);
      tmem_ld32(tS + 96, sv3);
      tmem_ld_wait(sv0);
      reg_anchor(sv1);
      reg_anchor(sv2);
      reg_anchor(sv3);
      tc_fence_before();
      mbar_arrive(&sh->s_read[t]);                     // S_t read: the correction warps refill it
      // P buffer pbuf(j) of this tile and its alphas were last read for tile j - kPBufs, and those reads
      // are complete by now without a wait of their own: S(j) exists only after the correction warps'
      // refill at the top of their iteration j - 1, which follows their stages of tile j - 2, and the
      // first of those waited for the last P.V of tile j - 3 to complete (measured: the P-buffer wait
      // this replaces cost 1184 -> 1216 TOPS).
      const int pb = pbuf(j);
      uint8_t* prow = sP + (kPBufs * t + pb) * kTile + prow_off;
      const bool last1 = j == n - 1, prev1 = j == n - 2 && ns_last == 1;
      if (tv == 128 && !last1 && !prev1) {              // the bulk: both halves in one pass
        const float2 smax = tile128_max(sv);
        const float c0 = __fmul_rn(sm, __fmul_rn(qs, ks.x)), c1 = __fmul_rn(sm, __fmul_rn(qs, ks.y));
        const float2 al = kMagic * fmaxf(c0, c1) < kFoldMax ? tile128_exp<true>(sv, smax, c0, c1, m, dsum, prow, rsw)
                                                            : tile128_exp<false>(sv, smax, c0, c1, m, dsum, prow, rsw);
        sh->alpha[t][pb][0][rl] = al.x;
        sh->alpha[t][pb][1][rl] = al.y;
        fence_proxy_async_smem();
        mbar_arrive(&sh->p_full[t][pb]);
        continue;
      }
      {
        const float dq = __fmul_rn(qs, ks.x);
        const float alpha = softmax_half(sv, min(64, tv), last1 || (prev1 && tv <= 64), __fmul_rn(sm, dq), dq, sm,
                                         m, dsum, prow, 0, rsw);
        sh->alpha[t][pb][0][rl] = alpha;
      }
      if (tv > 64) {
        const float dq = __fmul_rn(qs, ks.y);
        const float alpha = softmax_half(sv + 64, tv - 64, last1 || prev1, __fmul_rn(sm, dq), dq, sm, m, dsum, prow,
                                         1, rsw);
        sh->alpha[t][pb][1][rl] = alpha;
      }
      fence_proxy_async_smem();
      mbar_arrive(&sh->p_full[t][pb]);
    }
    if (ok) {
      sh->ml[t][rl] = make_float2(m, dsum);
      mbar_arrive(&sh->ml_full[t]);
    }
  } else {
    // ------------------------------------------------------------ correction + epilogue
    reg_dealloc<RegSplit<kKeyRange>::correction>();
    const int quarter = warp & 3;
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const int rl = quarter * 32 + lane;
    bool ok = n > 0;
    int u = 0;
    // S_t = magic for the Q.K^T to accumulate onto: once at the start, then each time the softmax has
    // read the scores (16 registers hold the constant, so a refill is eight 16-column stores)
    uint32_t mg[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) mg[c] = kMagicBits;
    auto refill = [&](int t) {
      const uint32_t tS = tmem + kColS + 128 * t + lane_off;
#pragma unroll
      for (int c = 0; c < 8; ++c) tmem_st16(tS + 16 * c, mg);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&sh->s_free[t]);
    };
    if (ok) {
      refill(0);
      refill(1);
    }
    // Order kept on purpose: the refill for tile j + 1 comes after every O stage of tile j - 1, whose
    // first stage waited for the last P.V of tile j - 2; the softmax reuses P buffers on that guarantee.
    TileWalk<kKeyRange> tw(a, t_begin, tiles_per_seg);
    for (int j = 0; ok && j < n; ++j, tw.next(a, tiles_per_seg)) {
      const int ns = tw.valid(a) > 64 ? 2 : 1;
      if (j + 1 < n) {                                  // S_t(j) read -> refill for the Q.K^T of tile j + 1
        for (int t = 0; ok && t < 2; ++t) {
          if (!(ok = mbar_wait(&sh->s_read[t], j & 1, abort_flag, a.status, kDevTimeoutS))) break;
          tc_fence_after();
          refill(t);
        }
      }
      for (int hh = 0; ok && hh < ns; ++hh, ++u) {
        for (int t = 0; t < 2; ++t) {
          if (hh == 0 &&
              !(ok = mbar_wait(&sh->p_full[t][pbuf(j)], pphase(j), abort_flag, a.status, kDevTimeoutP)))
            break;
          if (u > 0) {
            if (!(ok = mbar_wait(&sh->o_done[t], (u - 1) & 1, abort_flag, a.status, kDevTimeoutO))) break;
            tc_fence_after();
            const float alpha = sh->alpha[t][pbuf(j)][hh][rl];
            if (__any_sync(0xffffffffu, alpha != 1.f)) rescale_o(tmem + kColO + 128 * t + lane_off, alpha);
          }
          tc_fence_before();
          mbar_arrive(&sh->o_ready[t]);
        }
      }
    }
    for (int t = 0; t < 2; ++t) {
      const uint32_t tO = tmem + kColO + 128 * t + lane_off;
      const int qtile = 2 * qp + t;
      const int row = qtile * 128 + rl;
      const bool o_ready = ok && mbar_wait(&sh->o_done[t], (u - 1) & 1, abort_flag, a.status, kDevTimeoutO) &&
                           mbar_wait(&sh->ml_full[t], 0, abort_flag, a.status, kDevTimeoutO);
      if (!o_ready) ok = false;
      const float2 ml = o_ready ? sh->ml[t][rl] : make_float2(0.f, 1.f);
      if constexpr (kKeyRange) {
        // warp-uniform: tcgen05.ld is a whole-warp instruction
        if (__all_sync(0xffffffffu, o_ready) && qtile * 128 < a.q_len) {
          tc_fence_after();
          store_key_partial(a, tO, sP + kPBufs * t * kTile, quarter, lane, qtile, bh, bhs, ml.x, ml.y);
        }
      } else if (__all_sync(0xffffffffu, o_ready)) {
        tc_fence_after();
        if (a.num_splits == 1) {
          const float rd = __frcp_rn(ml.y);
          const float* vs = a.v_scale + int64_t(bh) * 128;
          __nv_bfloat16* dst = a.out + b * a.so_b + int64_t(row) * a.so_l + h * a.so_h;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t ov[32];
            tmem_ld32(tO + 32 * c, ov);
            tmem_ld_wait(ov);
            uint32_t packed[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float o0 = __fmul_rn(__fmul_rn(__uint_as_float(ov[2 * e]), rd), vs[32 * c + 2 * e]);
              const float o1 = __fmul_rn(__fmul_rn(__uint_as_float(ov[2 * e + 1]), rd), vs[32 * c + 2 * e + 1]);
              packed[e] = pack_act2(o0, o1, a.dtype);
            }
            if (row < a.q_len && a.wide_out) {         // 32-byte aligned rows: 256-bit stores
              st_global_v8(dst + 32 * c, packed);
              st_global_v8(dst + 32 * c + 16, packed + 8);
            } else if (row < a.q_len) {
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
            tmem_ld_wait(ov);
            if (row < a.q_len && a.wide_part) {
#pragma unroll
              for (int e = 0; e < 4; ++e) st_global_v8(dst + 32 * c + 8 * e, ov + 8 * e);
            } else if (row < a.q_len) {
#pragma unroll
              for (int e = 0; e < 8; ++e)
                reinterpret_cast<uint4*>(dst + 32 * c)[e] =
                    make_uint4(ov[4 * e], ov[4 * e + 1], ov[4 * e + 2], ov[4 * e + 3]);
            }
          }
          if (row < a.q_len) a.ml_part[prow] = ml;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 13) tmem_dealloc(tmem, 512);
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
  uint2 st;
  st.x = pack_act2(o.x * rl * vs.x, o.y * rl * vs.y, a.dtype);
  st.y = pack_act2(o.z * rl * vs.z, o.w * rl * vs.w, a.dtype);
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
  if (cudaError_t e = allow_dynamic_smem<attn_fwd_kernel<kKeyRange>>(int(kAttnSmemBytes)); e != cudaSuccess) return e;
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
