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
// Tokens past the valid length are stored as code 0 so that the attention kernel's masked keys are
// finite.
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

__device__ __forceinline__ uint32_t pack_s8x4(int32_t a, int32_t b, int32_t c, int32_t d) {
  return (uint32_t(a) & 0xff) | ((uint32_t(b) & 0xff) << 8) | ((uint32_t(c) & 0xff) << 16) | (uint32_t(d) << 24);
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// ------------------------------------------------------------------ K/V block statistics
// One CTA per (64-token block, head, batch). ksum: fp64 sum of K over the block's tokens that are
// < kv_len; vamax: max |V|. 128 threads = 8 row groups x 16 chunks of 8 channels.
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
    const uint4 kr = *reinterpret_cast<const uint4*>(a.k + b * a.sk_b + tok * a.sk_l + h * a.sk_h + c16 * 8);
    const uint4 vr = *reinterpret_cast<const uint4*>(a.v + b * a.sv_b + tok * a.sv_l + h * a.sv_h + c16 * 8);
    float kf[8], vf[8];
    bf16x8_to_f32(kr, kf);
    bf16x8_to_f32(vr, vf);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s[i] += double(kf[i]);
      vm[i] = fmaxf(vm[i], fabsf(vf[i]));
    }
  }
  __shared__ double sh_s[8][128];
  __shared__ float sh_v[8][128];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    sh_s[rg][c16 * 8 + i] = s[i];
    sh_v[rg][c16 * 8 + i] = vm[i];
  }
  __syncthreads();
  double tot = 0.0;
  float vmax = 0.f;
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    tot += sh_s[g][t];
    vmax = fmaxf(vmax, sh_v[g][t]);
  }
  const int64_t o = ((int64_t(b) * a.max_blocks + blk) * a.heads + h) * 128 + t;
  a.ksum[o] = tot;
  a.vamax[o] = vmax;
}

// ------------------------------------------------------------------ window sums
// One CTA per (head, batch): per channel, sum of the block sums (fixed order -> deterministic) and
// max of the block maxima over blocks [blk_begin, blk_end).
__global__ void __launch_bounds__(1024) kv_window_sums_kernel(KvWindowSumsArgs a) {
  const int h = blockIdx.x, b = blockIdx.y;
  const int c = threadIdx.x & 127, g = threadIdx.x >> 7;   // 8 block groups
  double s = 0.0;
  float vm = 0.f;
  for (int blk = a.blk_begin + g; blk < a.blk_end; blk += 8) {
    const int64_t o = ((int64_t(b) * a.max_blocks + blk) * a.heads + h) * 128 + c;
    s += a.ksum[o];
    vm = fmaxf(vm, a.vamax[o]);
  }
  __shared__ double sh_s[8][128];
  __shared__ float sh_v[8][128];
  sh_s[g][c] = s;
  sh_v[g][c] = vm;
  __syncthreads();
  if (g == 0) {
    double tot = 0.0;
    float vmax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      tot += sh_s[i][c];
      vmax = fmaxf(vmax, sh_v[i][c]);
    }
    const int64_t o = (int64_t(b) * a.heads + h) * 128 + c;
    a.ksum_total[o] = tot;
    a.vamax_total[o] = vmax;
  }
}

// ------------------------------------------------------------------ Q quantizer
// One CTA (4 warps) per (128-row tile, head, batch); warp w owns the 32-row scale group.
// Lane l handles rows 2*i + (l >> 4), 16-byte chunk (l & 15), i = 0..15.
__global__ void __launch_bounds__(128) quant_q_kernel(QuantQArgs a) {
  const int tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int row0 = tile * 128 + w * 32;
  const int c16 = l & 15;
  float x[16][8];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int row = row0 + 2 * i + (l >> 4);
    if (row < a.q_len) {
      const uint4 r = *reinterpret_cast<const uint4*>(a.q + b * a.sq_b + int64_t(row) * a.sq_l + h * a.sq_h + c16 * 8);
      bf16x8_to_f32(r, x[i]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) x[i][j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(x[i][j]));
  }
  amax = fmaxf(warp_max(amax), 1e-7f);
  const float inv = __fmul_rn(__frcp_rn(amax), 127.f);
  const int64_t bh = int64_t(b) * a.heads + h;
  if (l == 0) a.q_scale[bh * (a.q_pad / 32) + tile * 4 + w] = __fdiv_rn(amax, 127.f);
  int8_t* dst = a.q_codes + (bh * a.q_pad + row0) * 128;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int row = 2 * i + (l >> 4);
    uint2 packed;
    packed.x = pack_s8x4(cvt_rni_sat_s8(__fmul_rn(x[i][0], inv)), cvt_rni_sat_s8(__fmul_rn(x[i][1], inv)),
                         cvt_rni_sat_s8(__fmul_rn(x[i][2], inv)), cvt_rni_sat_s8(__fmul_rn(x[i][3], inv)));
    packed.y = pack_s8x4(cvt_rni_sat_s8(__fmul_rn(x[i][4], inv)), cvt_rni_sat_s8(__fmul_rn(x[i][5], inv)),
                         cvt_rni_sat_s8(__fmul_rn(x[i][6], inv)), cvt_rni_sat_s8(__fmul_rn(x[i][7], inv)));
    *reinterpret_cast<uint2*>(dst + row * 128 + c16 * 8) = packed;
  }
}

// km for channel c of (b, h): the window mean rounded through fp32 to bf16 (the rounding torch
// applies when a float64 mean is cast to bfloat16).
__device__ __forceinline__ float window_mean_bf16(const double* ksum_total, int64_t o, int64_t kv_len) {
  const double mean = ksum_total[o] / double(kv_len);
  return __bfloat162float(__float2bfloat16_rn(__double2float_rn(mean)));
}

// ------------------------------------------------------------------ K quantizer
// One CTA per (64-token block of this segment, head, batch). 128 threads: thread t handles the
// 16-byte chunk (t & 15) of rows (t >> 4) + 8*i.
__global__ void __launch_bounds__(128) quant_k_kernel(QuantKArgs a) {
  const int blk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x, c16 = t & 15, rg = t >> 4;
  const int64_t bh = int64_t(b) * a.heads + h;
  __shared__ float sh_km[128];
  __shared__ float sh_red[4];
  {
    const float km = window_mean_bf16(a.ksum_total, bh * 128 + t, a.kv_len_total);
    sh_km[t] = km;
    if (a.km_out != nullptr && blk == 0 && a.write_km) a.km_out[bh * 128 + t] = __float2bfloat16_rn(km);
  }
  __syncthreads();
  float km[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) km[j] = sh_km[c16 * 8 + j];
  float x[8][8];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = rg + 8 * i;
    const int64_t tok = int64_t(blk) * 64 + r;      // token index inside this segment
    if (tok < a.seg_valid) {
      const uint4 raw = *reinterpret_cast<const uint4*>(a.k + b * a.sk_b + (a.tok0 + tok) * a.sk_l + h * a.sk_h + c16 * 8);
      bf16x8_to_f32(raw, x[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        x[i][j] = __fsub_rn(x[i][j], km[j]);
        amax = fmaxf(amax, fabsf(x[i][j]));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) x[i][j] = 0.f;
    }
  }
  amax = warp_max(amax);
  if ((t & 31) == 0) sh_red[t >> 5] = amax;
  __syncthreads();
  amax = fmaxf(fmaxf(fmaxf(sh_red[0], sh_red[1]), fmaxf(sh_red[2], sh_red[3])), 1e-7f);
  const float inv = __fmul_rn(__frcp_rn(amax), 127.f);
  const int64_t seg_bh = (int64_t(a.seg) * a.batch + b) * a.heads + h;
  if (t == 0) a.k_scale[seg_bh * (a.seg_pad / 64) + blk] = __fdiv_rn(amax, 127.f);
  int8_t* dst = a.k_codes + (seg_bh * a.seg_pad + int64_t(blk) * 64) * 128;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = rg + 8 * i;
    uint2 packed;
    packed.x = pack_s8x4(cvt_rni_sat_s8(__fmul_rn(x[i][0], inv)), cvt_rni_sat_s8(__fmul_rn(x[i][1], inv)),
                         cvt_rni_sat_s8(__fmul_rn(x[i][2], inv)), cvt_rni_sat_s8(__fmul_rn(x[i][3], inv)));
    packed.y = pack_s8x4(cvt_rni_sat_s8(__fmul_rn(x[i][4], inv)), cvt_rni_sat_s8(__fmul_rn(x[i][5], inv)),
                         cvt_rni_sat_s8(__fmul_rn(x[i][6], inv)), cvt_rni_sat_s8(__fmul_rn(x[i][7], inv)));
    *reinterpret_cast<uint2*>(dst + r * 128 + c16 * 8) = packed;
  }
}

// ------------------------------------------------------------------ V quantizer (transposing)
// One CTA per (128-token tile of this segment, head, batch), 256 threads. Reads [128 tok][128 ch]
// bf16, writes e4m3 codes transposed to [128 ch][128 tok] through shared memory.
__global__ void __launch_bounds__(256) quant_vt_kernel(QuantVArgs a) {
  const int tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x;
  const int64_t bh = int64_t(b) * a.heads + h;
  __shared__ float sh_recp[128];
  __shared__ __align__(16) uint8_t sh_t[128][128 + 16];   // [channel][token], padded rows
  if (t < 128) {
    const float amax = a.vamax_total[bh * 128 + t];
    sh_recp[t] = __fmul_rn(__frcp_rn(amax), 2.25f);
    if (tile == 0 && a.write_scale) a.v_scale[bh * 128 + t] = __fdiv_rn(amax, 2.25f);
  }
  __syncthreads();
  const int c16 = t & 15;
  float rc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) rc[j] = sh_recp[c16 * 8 + j];
#pragma unroll 4
  for (int i = 0; i < 8; ++i) {
    const int r = (t >> 4) + 16 * i;                 // token row inside the tile
    const int64_t tok = int64_t(tile) * 128 + r;
    float x[8];
    if (tok < a.seg_valid) {
      const uint4 raw = *reinterpret_cast<const uint4*>(a.v + b * a.sv_b + (a.tok0 + tok) * a.sv_l + h * a.sv_h + c16 * 8);
      bf16x8_to_f32(raw, x);
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = fminf(fmaxf(__fmul_rn(x[j], rc[j]), -2.25f), 2.25f);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      const uint32_t p = pack_e4m3x2(x[j], x[j + 1]);
      sh_t[c16 * 8 + j][r] = uint8_t(p & 0xff);
      sh_t[c16 * 8 + j + 1][r] = uint8_t(p >> 8);
    }
  }
  __syncthreads();
  // 128 channel rows x 128 bytes: each thread stores 16-byte pieces.
  const int64_t seg_bh = (int64_t(a.seg) * a.batch + b) * a.heads + h;
  uint8_t* dst = a.vt_codes + seg_bh * 128 * a.seg_pad + int64_t(tile) * 128;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int piece = t + 256 * i;                   // 1024 pieces of 16 bytes
    const int ch = piece >> 3, off = (piece & 7) * 16;
    *reinterpret_cast<uint4*>(dst + int64_t(ch) * a.seg_pad + off) = *reinterpret_cast<const uint4*>(&sh_t[ch][off]);
  }
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_kv_block_stats(const KvBlockStatsArgs& a, cudaStream_t st) {
  dim3 grid(a.blk_end - a.blk_begin, a.heads, a.batch);
  kv_block_stats_kernel<<<grid, 128, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_kv_window_sums(const KvWindowSumsArgs& a, cudaStream_t st) {
  dim3 grid(a.heads, a.batch);
  kv_window_sums_kernel<<<grid, 1024, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_quant_q(const QuantQArgs& a, cudaStream_t st) {
  dim3 grid(a.q_pad / 128, a.heads, a.batch);
  quant_q_kernel<<<grid, 128, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_quant_k(const QuantKArgs& a, cudaStream_t st) {
  dim3 grid(a.seg_pad / 64, a.heads, a.batch);
  quant_k_kernel<<<grid, 128, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_quant_vt(const QuantVArgs& a, cudaStream_t st) {
  dim3 grid(a.seg_pad / 128, a.heads, a.batch);
  quant_vt_kernel<<<grid, 256, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace lbq
