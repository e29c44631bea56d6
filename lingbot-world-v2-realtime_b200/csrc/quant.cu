// Quantizers of the Sage-semantics attention path, sm_100a.
//
// Reference semantics (paths inside the reference project):
//   Q : per (batch, head, 32-token group), Lq padded to 128            sage_kvq.py:57-66,104
//   K : km = mean over the window; per (batch, head, 64-token block)   sage_preq.py:115-116, sage_kvq.py:85
//   V : per (batch, head, channel) e4m3 of v * (2.25 / max|v|)         sage_preq.py:47-77, sage_kvq.py:69-75
// Codes are round-half-even / round-to-nearest of x * fl(fl(1/amax) * 127) (resp. * 2.25) — the way
// torch evaluates the reference's `127.0 / amax` — and scales are amax / 127 (resp. / 2.25) as
// true fp32 divisions.
//
// Layout of the quantized window (all caller-allocated, all per "segment" s of the KV window; one
// segment on one GPU, one per rank after a sequence all-gather):
//   q_codes  int8 [B][H][q_pad][128]            q_pad  = round_up(q_len, 128)
//   q_scale  f32  [B][H][q_pad/32]
//   k_codes  int8 [S][B][H][seg_pad][128]       seg_pad = round_up(seg_len, 128)
//   k_scale  f32  [S][B][H][seg_pad/64]
//   vt_codes e4m3 [S][B][H][128][seg_pad]       (V transposed: keys contiguous per channel)
//   v_scale  f32  [B][H][128]
// Tokens past the valid length, up to the next multiple of 128, are stored as code 0 so that the
// attention kernel's masked keys are finite; key tiles past that are never read and not written.
#include <cuda_bf16.h>
#include <cstdint>

#include "lbq_ptx.cuh"
#include "lbq_kernels.h"

namespace lbq {

__device__ __forceinline__ void bf16x8_to_f32(const uint4 raw, float (&f)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
// 8 activations (dtype 0: bf16, 1: fp16) as floats, exactly.
__device__ __forceinline__ void act8_to_f32(const uint4 raw, int dtype, float (&f)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) act2_to_f32(w[i], dtype, f[2 * i], f[2 * i + 1]);
}

// Four values already in (-127.5, 127.5) to four int8 codes, round to nearest even, packed (the first in
// the low byte): adding 1.5 * 2^23 rounds each to an integer held in the low mantissa bits, so byte 0
// of the sum's bits is the code's two's-complement byte — the result of cvt.rni.sat.s8.f32 (no value
// reaches the saturation bounds) on the FMA pipe instead of the conversion unit, and three byte
// permutes instead of shifts and masks.
__device__ __forceinline__ uint32_t pack_rn_s8x4(float a, float b, float c, float d) {
  const uint32_t ua = __float_as_uint(__fadd_rn(a, 12582912.f)), ub = __float_as_uint(__fadd_rn(b, 12582912.f));
  const uint32_t uc = __float_as_uint(__fadd_rn(c, 12582912.f)), ud = __float_as_uint(__fadd_rn(d, 12582912.f));
  return __byte_perm(__byte_perm(ua, ub, 0x0040), __byte_perm(uc, ud, 0x0040), 0x5410);
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// RoPE of 8 consecutive channels (4 rotation pairs) of one token in the reference's fp64 form
// (lingbot/models/lingbot_world/transformer.py:142-146): (xr, xi) -> (xr cos - xi sin, xr sin + xi cos)
// with every product and sum rounded in fp64 (torch evaluates the expression op by op, no fma), then
// cast to bf16 through fp32 (torch's double -> bfloat16 conversion). cs / sn: the pairs' 4 angles.
__device__ __forceinline__ uint4 rope_bf16x8(const uint4 raw, const double* cs, const double* sn) {
  float f[8];
  bf16x8_to_f32(raw, f);
  const double2 c01 = *reinterpret_cast<const double2*>(cs), c23 = *reinterpret_cast<const double2*>(cs + 2);
  const double2 s01 = *reinterpret_cast<const double2*>(sn), s23 = *reinterpret_cast<const double2*>(sn + 2);
  const double c[4] = {c01.x, c01.y, c23.x, c23.y}, s[4] = {s01.x, s01.y, s23.x, s23.y};
  uint32_t w[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const double xr = f[2 * p], xi = f[2 * p + 1];
    const double re = __dsub_rn(__dmul_rn(xr, c[p]), __dmul_rn(xi, s[p]));
    const double im = __dadd_rn(__dmul_rn(xr, s[p]), __dmul_rn(xi, c[p]));
    const __nv_bfloat16 lo = __float2bfloat16_rn(__double2float_rn(re));
    const __nv_bfloat16 hi = __float2bfloat16_rn(__double2float_rn(im));
    w[p] = uint32_t(__bfloat16_as_ushort(lo)) | (uint32_t(__bfloat16_as_ushort(hi)) << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// The buffer row of logical token t: through the ring map when the cache is a ring (kRing), else t.
template <bool kRing>
__device__ __forceinline__ int64_t ring_row(const Ring& r, int64_t t) {
  if constexpr (kRing) return phys_tok(r, t);
  return t;
}

// ------------------------------------------------------------------ K/V block statistics
// One CTA per (64-token block, head, batch). ksum: fp64 sum of K over the block's tokens that are
// < kv_len; vamax: max |V|. 128 threads = 8 row groups x 16 chunks of 8 channels.
template <int kDt, bool kRing>
__global__ void __launch_bounds__(128) kv_block_stats_kernel(KvBlockStatsArgs a) {
  const int blk = a.blk_begin + blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x, c16 = t & 15, rg = t >> 4;
  double s[8];
  float vm[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) { s[i] = 0.0; vm[i] = 0.f; }
  for (int r = rg; r < 64; r += 8) {
    const int64_t tok = int64_t(blk) * 64 + r;
    if (tok >= a.kv_len) break;
    const int64_t row = ring_row<kRing>(a.ring, tok);
    const uint4 kr = *reinterpret_cast<const uint4*>(a.k + b * a.sk_b + row * a.sk_l + h * a.sk_h + c16 * 8);
    const uint4 vr = *reinterpret_cast<const uint4*>(a.v + b * a.sv_b + row * a.sv_l + h * a.sv_h + c16 * 8);
    float kf[8], vf[8];
    act8_to_f32(kr, kDt, kf);
    act8_to_f32(vr, kDt, vf);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s[i] += double(kf[i]);
      vm[i] = fmaxf(vm[i], fabsf(vf[i]));
    }
  }
  // [row group][channel within chunk][chunk]: a warp's 16 chunks of one slot are consecutive words
  __shared__ double sh_s[8][8][16];
  __shared__ float sh_v[8][8][16];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    sh_s[rg][i][c16] = s[i];
    sh_v[rg][i][c16] = vm[i];
  }
  __syncthreads();
  double tot = 0.0;
  float vmax = 0.f;
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    tot += sh_s[g][t & 7][t >> 3];
    vmax = fmaxf(vmax, sh_v[g][t & 7][t >> 3]);
  }
  const int64_t o = ((int64_t(b) * a.max_blocks + blk) * a.heads + h) * 128 + t;
  if (LBQ_CHECK(blk < a.max_blocks, a.status, kDevBadStatsRow)) {
    a.ksum[o] = tot;
    a.vamax[o] = vmax;
  }
}

// ------------------------------------------------------------------ cache write + block statistics
// One CTA per (64-token block, head, batch) over the blocks covering [tok_begin, tok_end): stores
// the block's new tokens into the cache (K roped when the tables are given) and accumulates the
// block's statistics in exactly kv_block_stats_kernel's order and thread layout, so the tables are
// bit-identical to a copy followed by kv_block_stats. Tokens of the block before tok_begin are read
// back from the cache.
template <bool kRing>
__global__ void __launch_bounds__(128) cache_write_kernel(CacheWriteArgs a) {
  const int blk = a.blk_begin + blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x, c16 = t & 15, rg = t >> 4;
  double s[8];
  float vm[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) { s[i] = 0.0; vm[i] = 0.f; }
  for (int r = rg; r < 64; r += 8) {
    const int64_t tok = int64_t(blk) * 64 + r;
    if (tok >= a.tok_end) break;
    const int64_t row = ring_row<kRing>(a.ring, tok);
    __nv_bfloat16* kc = a.k_cache + b * a.ck_b + row * a.ck_l + h * a.ck_h + c16 * 8;
    __nv_bfloat16* vc = a.v_cache + b * a.cv_b + row * a.cv_l + h * a.cv_h + c16 * 8;
    uint4 kr, vr;
    if (tok < a.tok_begin) {
      kr = *reinterpret_cast<const uint4*>(kc);
      vr = *reinterpret_cast<const uint4*>(vc);
    } else {
      const int64_t i = tok - a.tok_begin;
      kr = *reinterpret_cast<const uint4*>(a.k_src + b * a.sk_b + i * a.sk_l + h * a.sk_h + c16 * 8);
      vr = *reinterpret_cast<const uint4*>(a.v_src + b * a.sv_b + i * a.sv_l + h * a.sv_h + c16 * 8);
      if (a.rope_cos != nullptr) {
        const int64_t o = b * a.sr_b + i * a.sr_l + c16 * 4;
        kr = rope_bf16x8(kr, a.rope_cos + o, a.rope_sin + o);
      }
      *reinterpret_cast<uint4*>(kc) = kr;
      *reinterpret_cast<uint4*>(vc) = vr;
    }
    float kf[8], vf[8];
    bf16x8_to_f32(kr, kf);
    bf16x8_to_f32(vr, vf);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s[i] += double(kf[i]);
      vm[i] = fmaxf(vm[i], fabsf(vf[i]));
    }
  }
  __shared__ double sh_s[8][8][16];
  __shared__ float sh_v[8][8][16];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    sh_s[rg][i][c16] = s[i];
    sh_v[rg][i][c16] = vm[i];
  }
  __syncthreads();
  double tot = 0.0;
  float vmax = 0.f;
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    tot += sh_s[g][t & 7][t >> 3];
    vmax = fmaxf(vmax, sh_v[g][t & 7][t >> 3]);
  }
  const int64_t o = ((int64_t(b) * a.max_blocks + blk) * a.heads + h) * 128 + t;
  if (LBQ_CHECK(blk < a.max_blocks, a.status, kDevBadStatsRow)) {
    a.ksum[o] = tot;
    a.vamax[o] = vmax;
  }
}

// ------------------------------------------------------------------ window sums
// One CTA per (32-channel group, head, batch), 256 threads = 32 channels x 8 block groups: per
// channel, the sum of the block sums (fixed order -> deterministic) and the max of the block maxima
// over blocks [blk_begin, blk_end).
__global__ void __launch_bounds__(256) kv_window_sums_kernel(KvWindowSumsArgs a) {
  const int cg = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int c = cg * 32 + (threadIdx.x & 31), g = threadIdx.x >> 5;
  double s = 0.0;
  float vm = 0.f;
  for (int blk = a.blk_begin + g; blk < a.blk_end; blk += 8) {
    const int64_t o = ((int64_t(b) * a.max_blocks + blk) * a.heads + h) * 128 + c;
    s += a.ksum[o];
    vm = fmaxf(vm, a.vamax[o]);
  }
  __shared__ double sh_s[8][32];
  __shared__ float sh_v[8][32];
  sh_s[g][threadIdx.x & 31] = s;
  sh_v[g][threadIdx.x & 31] = vm;
  __syncthreads();
  if (g == 0) {
    double tot = 0.0;
    float vmax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      tot += sh_s[i][threadIdx.x];
      vmax = fmaxf(vmax, sh_v[i][threadIdx.x]);
    }
    const int64_t o = (int64_t(b) * a.heads + h) * 128 + c;
    a.ksum_total[o] = tot;
    a.vamax_total[o] = vmax;
  }
}

// ------------------------------------------------------------------ Q quantizer
// One CTA (8 warps) per (128-row tile, head, batch); warps 2g and 2g+1 share the 32-row scale group
// g, 16 rows each. Lane l handles rows 2*i + (l >> 4) of its warp's 16, 16-byte chunk (l & 15). The
// raw bf16 stays in registers for the second (quantizing) pass.
__global__ void __launch_bounds__(256) quant_q_kernel(QuantQArgs a) {
  const int tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int g = w >> 1;
  const int row0 = tile * 128 + g * 32 + (w & 1) * 16;
  const int c16 = l & 15;
  __shared__ float sh_max[8];
  uint4 raw[8];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = row0 + 2 * i + (l >> 4);
    raw[i] = row < a.q_len
                 ? *reinterpret_cast<const uint4*>(a.q + b * a.sq_b + int64_t(row) * a.sq_l + h * a.sq_h + c16 * 8)
                 : make_uint4(0u, 0u, 0u, 0u);
  }
  if (a.rope_cos != nullptr) {                  // roped Q: the reference's causal_rope_apply, fused
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = row0 + 2 * i + (l >> 4);
      if (row < a.q_len) {
        const int64_t o = b * a.sr_b + int64_t(row) * a.sr_l + c16 * 4;
        raw[i] = rope_bf16x8(raw[i], a.rope_cos + o, a.rope_sin + o);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float x[8];
    act8_to_f32(raw[i], a.dtype, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(x[j]));
  }
  amax = warp_max(amax);
  if (l == 0) sh_max[w] = amax;
  __syncthreads();
  amax = fmaxf(fmaxf(sh_max[2 * g], sh_max[2 * g + 1]), 1e-7f);
  const float inv = __fmul_rn(__frcp_rn(amax), 127.f);
  const int64_t bh = int64_t(b) * a.heads + h;
  if (threadIdx.x == 64 * g) a.q_scale[bh * (a.q_pad / 32) + tile * 4 + g] = __fdiv_rn(amax, 127.f);
  int8_t* dst = a.q_codes + (bh * a.q_pad + row0) * 128;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float x[8];
    act8_to_f32(raw[i], a.dtype, x);
    uint2 packed;
    packed.x = pack_rn_s8x4(__fmul_rn(x[0], inv), __fmul_rn(x[1], inv), __fmul_rn(x[2], inv), __fmul_rn(x[3], inv));
    packed.y = pack_rn_s8x4(__fmul_rn(x[4], inv), __fmul_rn(x[5], inv), __fmul_rn(x[6], inv), __fmul_rn(x[7], inv));
    *reinterpret_cast<uint2*>(dst + (2 * i + (l >> 4)) * 128 + c16 * 8) = packed;
  }
}

// km for channel c of (b, h): the window mean rounded through fp32 to k's dtype (the rounding torch
// applies when a float64 mean is cast to bfloat16 or float16); its 16 bits in *bits.
__device__ __forceinline__ float window_mean_act(const double* ksum_total, int64_t o, int64_t kv_len, int dtype,
                                                 uint16_t* bits) {
  const float mean = __double2float_rn(ksum_total[o] / double(kv_len));
  if (dtype) {
    const __half hm = __float2half_rn(mean);
    *bits = __half_as_ushort(hm);
    return __half2float(hm);
  }
  const __nv_bfloat16 bm = __float2bfloat16_rn(mean);
  *bits = __bfloat16_as_ushort(bm);
  return __bfloat162float(bm);
}

// ------------------------------------------------------------------ K/V quantizer (one launch)
// One CTA of 256 threads per (128-token tile of this segment, head, batch) and tensor: even
// blockIdx.x = K tile tile0 + x/2, odd = V tile tile0 + x/2, so the K and V halves of the work stream
// through the GPU together. Both stage their bf16 tile [128 tokens][128 channels] in shared memory by
// 16-byte `cp.async` copies (pad tokens zero-filled by a zero source size; row pitch 272 bytes), so
// the loads hold no registers: 40 registers a thread, 6 CTAs per SM (measured 5022 -> 5108 GB/s on
// the 30-layer re-quant against register-held loads at 4 CTAs per SM).
//
// K: the two 64-token blocks of the tile go to the two halves of the CTA; in a half, thread t handles
// the 16-byte chunk (t & 15) of rows (t >> 4) + 8*i of its block, read twice from the staged tile
// (amax, then codes). Codes RNE((k - km) * fl(fl(1/amax) * 127)), scale amax / 127 per block.
//
// V: from the staged tile (its column reads conflict-free with the 272-byte pitch) thread t takes the
// channel pair (2*(t & 63), +1) over 32 tokens (32*(t >> 6) ...), converts to e4m3 and writes, per
// channel, 32 consecutive key bytes of the transposed codes [channel][key].
constexpr int kVtPitch = 272;   // bytes per staged token row

struct QuantKvShared {
  uint8_t v[128 * kVtPitch];
  float km[128];
  float recp[128];
  float red[8];
};

template <int kDt, bool kRing>
__device__ __forceinline__ void quant_k_tile(const QuantKArgs& a, QuantKvShared& sh, int tile, bool first, int h,
                                             int b) {
  const int half = threadIdx.x >> 7, t = threadIdx.x & 127, c16 = t & 15, rg = t >> 4;
  const int blk = tile * 2 + half;
  const int64_t bh = int64_t(b) * a.heads + h;
  if (half == 0) {
    uint16_t km_bits;
    const float km = window_mean_act(a.ksum_total, bh * 128 + t, a.kv_len_total, kDt, &km_bits);
    sh.km[t] = km;
    if (a.km_out != nullptr && first && a.write_km) reinterpret_cast<uint16_t*>(a.km_out)[bh * 128 + t] = km_bits;
  }
  uint8_t* stage = sh.v + (half * 64) * kVtPitch + c16 * 16;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t tok = int64_t(blk) * 64 + rg + 8 * i;      // token index inside this segment
    const bool ok = tok < a.seg_valid && LBQ_CHECK(a.tok0 + tok >= 0, a.status, kDevBadSourceToken);
    const void* src = ok ? static_cast<const void*>(a.k + b * a.sk_b + ring_row<kRing>(a.ring, a.tok0 + tok) * a.sk_l +
                                                    h * a.sk_h + c16 * 8)
                         : static_cast<const void*>(a.k);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(stage + (rg + 8 * i) * kVtPitch)),
                 "l"(src), "r"(ok ? 16 : 0)
                 : "memory");
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  auto raw_at = [&](int i) { return *reinterpret_cast<const uint4*>(stage + (rg + 8 * i) * kVtPitch); };
  float km[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) km[j] = sh.km[c16 * 8 + j];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t tok = int64_t(blk) * 64 + rg + 8 * i;
    if (tok < a.seg_valid) {
      float x[8];
      act8_to_f32(raw_at(i), kDt, x);
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(__fsub_rn(x[j], km[j])));
    }
  }
  amax = warp_max(amax);
  if ((t & 31) == 0) sh.red[half * 4 + (t >> 5)] = amax;
  __syncthreads();
  const float* red = sh.red + half * 4;
  amax = fmaxf(fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3])), 1e-7f);
  const float inv = __fmul_rn(__frcp_rn(amax), 127.f);
  const int64_t seg_bh = (int64_t(a.seg) * a.batch + b) * a.heads + h;
  const float scale = __fdiv_rn(amax, 127.f);
  uint2 packed[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = rg + 8 * i;
    const bool valid = int64_t(blk) * 64 + r < a.seg_valid;   // pad tokens encode 0
    float x[8];
    act8_to_f32(raw_at(i), kDt, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = valid ? __fmul_rn(__fsub_rn(x[j], km[j]), inv) : 0.f;
    packed[i].x = pack_rn_s8x4(x[0], x[1], x[2], x[3]);
    packed[i].y = pack_rn_s8x4(x[4], x[5], x[6], x[7]);
  }
  int8_t* dst = a.k_codes + (seg_bh * a.seg_pad + int64_t(blk) * 64) * 128;
  if (t == 0) a.k_scale[seg_bh * (a.seg_pad / 64) + blk] = scale;
#pragma unroll
  for (int i = 0; i < 8; ++i) *reinterpret_cast<uint2*>(dst + (rg + 8 * i) * 128 + c16 * 8) = packed[i];
}

template <int kDt, bool kRing>
__device__ __forceinline__ void quant_v_tile(const QuantVArgs& a, QuantKvShared& sh, int tile, bool first, int h,
                                             int b) {
  const int t = threadIdx.x;
  const int64_t bh = int64_t(b) * a.heads + h;
  if (t < 128) {
    const float amax = a.vamax_total[bh * 128 + t];
    sh.recp[t] = __fmul_rn(__frcp_rn(amax), 2.25f);
    if (first && a.write_scale) a.v_scale[bh * 128 + t] = __fdiv_rn(amax, 2.25f);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int piece = t + 256 * i;                   // 2048 pieces of 16 bytes
    const int r = piece >> 4, c16 = piece & 15;
    const int64_t tok = int64_t(tile) * 128 + r;
    const bool ok = tok < a.seg_valid && LBQ_CHECK(a.tok0 + tok >= 0, a.status, kDevBadSourceToken);
    const void* src = ok ? static_cast<const void*>(a.v + b * a.sv_b + ring_row<kRing>(a.ring, a.tok0 + tok) * a.sv_l +
                                                    h * a.sv_h + c16 * 8)
                         : static_cast<const void*>(a.v);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(&sh.v[r * kVtPitch + c16 * 16])),
                 "l"(src), "r"(ok ? 16 : 0)
                 : "memory");
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  const int cp = t & 63, tq = t >> 6;
  const float r0 = sh.recp[2 * cp], r1 = sh.recp[2 * cp + 1];
  uint32_t w0[8], w1[8];                             // channel 2cp / 2cp+1: 32 key bytes each
#pragma unroll
  for (int k4 = 0; k4 < 8; ++k4) {
    float lo[4], hi[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = tq * 32 + 4 * k4 + e;
      const uint32_t pair = *reinterpret_cast<const uint32_t*>(&sh.v[r * kVtPitch + cp * 4]);
      float v0, v1;
      act2_to_f32(pair, kDt, v0, v1);
      lo[e] = fminf(fmaxf(__fmul_rn(v0, r0), -2.25f), 2.25f);
      hi[e] = fminf(fmaxf(__fmul_rn(v1, r1), -2.25f), 2.25f);
    }
    // padded tokens were staged as 0 and encode as 0
    w0[k4] = pack_e4m3x2(lo[0], lo[1]) | (pack_e4m3x2(lo[2], lo[3]) << 16);
    w1[k4] = pack_e4m3x2(hi[0], hi[1]) | (pack_e4m3x2(hi[2], hi[3]) << 16);
  }
  const int64_t seg_bh = (int64_t(a.seg) * a.batch + b) * a.heads + h;
  uint8_t* dst = a.vt_codes + seg_bh * 128 * a.seg_pad + int64_t(tile) * 128 + tq * 32;
  uint4* d0 = reinterpret_cast<uint4*>(dst + int64_t(2 * cp) * a.seg_pad);
  uint4* d1 = reinterpret_cast<uint4*>(dst + int64_t(2 * cp + 1) * a.seg_pad);
  d0[0] = make_uint4(w0[0], w0[1], w0[2], w0[3]);
  d0[1] = make_uint4(w0[4], w0[5], w0[6], w0[7]);
  d1[0] = make_uint4(w1[0], w1[1], w1[2], w1[3]);
  d1[1] = make_uint4(w1[4], w1[5], w1[6], w1[7]);
}

template <int kDt, bool kRing>
__global__ void __launch_bounds__(256, 6) quant_kv_kernel(QuantKArgs ka, QuantVArgs va, int tile0) {
  __shared__ __align__(16) QuantKvShared sh;
  const int tile = tile0 + int(blockIdx.x >> 1), h = blockIdx.y, b = blockIdx.z;
  const bool first = (blockIdx.x >> 1) == 0;
  if (blockIdx.x & 1) quant_v_tile<kDt, kRing>(va, sh, tile, first, h, b);
  else quant_k_tile<kDt, kRing>(ka, sh, tile, first, h, b);
}

// ------------------------------------------------------------------ launchers
template <int kDt, bool kRing>
cudaError_t launch_stats(const KvBlockStatsArgs& a, dim3 grid, cudaStream_t st) {
  if (cudaError_t e0 = prefer_max_shared<kv_block_stats_kernel<kDt, kRing>>(); e0 != cudaSuccess) return e0;
  kv_block_stats_kernel<kDt, kRing><<<grid, 128, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_kv_block_stats(const KvBlockStatsArgs& a, cudaStream_t st) {
  dim3 grid(a.blk_end - a.blk_begin, a.heads, a.batch);
  const bool ring = a.ring.len != 0;
  if (a.dtype) return ring ? launch_stats<1, true>(a, grid, st) : launch_stats<1, false>(a, grid, st);
  return ring ? launch_stats<0, true>(a, grid, st) : launch_stats<0, false>(a, grid, st);
}
cudaError_t launch_kv_window_sums(const KvWindowSumsArgs& a, cudaStream_t st) {
  dim3 grid(4, a.heads, a.batch);
  if (cudaError_t e0 = prefer_max_shared<kv_window_sums_kernel>(); e0 != cudaSuccess) return e0;
  kv_window_sums_kernel<<<grid, 256, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_quant_q(const QuantQArgs& a, cudaStream_t st) {
  dim3 grid(a.q_pad / 128, a.heads, a.batch);
  if (cudaError_t e0 = prefer_max_shared<quant_q_kernel>(); e0 != cudaSuccess) return e0;
  quant_q_kernel<<<grid, 256, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_cache_write(const CacheWriteArgs& a, cudaStream_t st) {
  const int blk_end = int((a.tok_end + 63) / 64);
  if (blk_end <= a.blk_begin) return cudaSuccess;
  dim3 grid(blk_end - a.blk_begin, a.heads, a.batch);
  if (a.ring.len != 0) {
    if (cudaError_t e0 = prefer_max_shared<cache_write_kernel<true>>(); e0 != cudaSuccess) return e0;
    cache_write_kernel<true><<<grid, 128, 0, st>>>(a);
  } else {
    if (cudaError_t e0 = prefer_max_shared<cache_write_kernel<false>>(); e0 != cudaSuccess) return e0;
    cache_write_kernel<false><<<grid, 128, 0, st>>>(a);
  }
  return cudaGetLastError();
}
// `tiles` 128-token tiles from tile0, stopping at the last tile holding valid tokens: a short last
// segment does not pay for the padding of its seg_pad, which the attention never reads.
cudaError_t launch_quant_kv(const QuantKArgs& ka, const QuantVArgs& va, int tile0, int tiles, cudaStream_t st) {
  if (tiles <= 0) return cudaSuccess;
  // no carveout preference: the driver's choice measured fastest for this kernel (5.0 TB/s on the
  // 30-layer re-quant, 3.9 TB/s with the largest shared-memory split)
  dim3 grid(tiles * 2, ka.heads, ka.batch);
  const bool ring = ka.ring.len != 0;
  auto kern = ka.dtype ? (ring ? quant_kv_kernel<1, true> : quant_kv_kernel<1, false>)
                       : (ring ? quant_kv_kernel<0, true> : quant_kv_kernel<0, false>);
  kern<<<grid, 256, 0, st>>>(ka, va, tile0);
  return cudaGetLastError();
}

}  // namespace lbq
