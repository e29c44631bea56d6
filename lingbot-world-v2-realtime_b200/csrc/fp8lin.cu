// FP8 linear layers for sm_100a: the rowwise FP8Linear of lingbot/layers/linear.py:10-31.
//
//   quantization (weights once, activations per call):  s = max(fl(max_k |x[r,k]| * fl(1/448)), 1e-12),
//                                                      q[r,k] = e4m3_rn(fl(x[r,k] / s))   (true division)
//   — the reference's `amax.float() / FMAX` and `x.float() / scale` as torch evaluates them on the GPU,
//   where a division by a Python scalar is a multiply by the scalar's fp32 reciprocal and a division by a
//   tensor is an IEEE division.
//   GEMM:  y[m,n] = bf16( (sum_k q_x[m,k] q_w[n,k]) * s_x[m] * s_w[n] + bias[n] )
//
// The reference runs the GEMM as torch._scaled_mm (cuBLASLt) with rowwise scales; here it is a
// persistent tcgen05 kernel: 128 x 256 output tiles, e4m3 x e4m3 -> fp32 in tensor memory (kind::f8f6f4,
// M = 128, N = 256, K = 32 per instruction), operands staged by TMA (128-byte swizzle, 128-byte K steps,
// 4 stages of 48 KB), two 256-column accumulators so the epilogue of one tile overlaps the main loop of
// the next. 320 threads: warp 0 TMA producer, warp 1 MMA issuer and tensor-memory owner, warps 2-9 the
// epilogue (warp w reads TMEM lanes 32 * (w % 4) .. +31, one output row per thread, and columns
// 128 * ((w - 2) / 4) .. +127 of the tile: two warps per lane quarter double the store issue rate,
// which limits the epilogue; with 32-byte aligned output rows each thread writes its 64 bytes of a
// 32-column chunk as two 256-bit stores, half the store instructions of 16-byte stores).
#include <cuda_bf16.h>
#include <cstdint>

#include "lbq_kernels.h"
#include "lbq_ptx.cuh"

namespace lbq {

// ------------------------------------------------------------------ rowwise FP8 quantizer
// One CTA of 256 threads per row: the row's absmax (block reduction), then the codes of x / s.
__global__ void __launch_bounds__(256) fp8_quant_rows_kernel(Fp8QuantArgs a) {
  const int row = blockIdx.x;
  const int t = threadIdx.x;
  const int chunks = a.cols / 8;                     // 8 values (16 bytes of bf16/fp16, 32 of fp32) each
  const unsigned char* src = static_cast<const unsigned char*>(a.x) + (int64_t(row) * a.sx) * a.esize;
  auto load8 = [&](int c, float (&f)[8]) {
    if (a.dtype == 2) {
      const float4 u = *reinterpret_cast<const float4*>(src + int64_t(c) * 32);
      const float4 w = *reinterpret_cast<const float4*>(src + int64_t(c) * 32 + 16);
      f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w; f[4] = w.x; f[5] = w.y; f[6] = w.z; f[7] = w.w;
    } else {
      const uint4 r = *reinterpret_cast<const uint4*>(src + int64_t(c) * 16);
      const uint32_t ws[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) act2_to_f32(ws[i], a.dtype, f[2 * i], f[2 * i + 1]);
    }
  };
  float am = 0.f;
  for (int c = t; c < chunks; c += 256) {
    float f[8];
    load8(c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(f[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  __shared__ float red[8];
  if ((t & 31) == 0) red[t >> 5] = am;
  __syncthreads();
  am = fmaxf(fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3])), fmaxf(fmaxf(red[4], red[5]), fmaxf(red[6], red[7])));
  const float s = fmaxf(__fmul_rn(am, 1.f / 448.f), 1e-12f);
  if (t == 0) a.scale[row] = s;
  uint8_t* dst = a.q + int64_t(row) * a.sq;
  for (int c = t; c < chunks; c += 256) {
    float f[8];
    load8(c, f);
    uint2 out;
    out.x = pack_e4m3x2(__fdiv_rn(f[0], s), __fdiv_rn(f[1], s)) | (pack_e4m3x2(__fdiv_rn(f[2], s), __fdiv_rn(f[3], s)) << 16);
    out.y = pack_e4m3x2(__fdiv_rn(f[4], s), __fdiv_rn(f[5], s)) | (pack_e4m3x2(__fdiv_rn(f[6], s), __fdiv_rn(f[7], s)) << 16);
    *reinterpret_cast<uint2*>(dst + int64_t(c) * 8) = out;
  }
}

// ------------------------------------------------------------------ tcgen05 GEMM
constexpr int kGemmStages = 4;
constexpr int kGemmABytes = 128 * 128;           // A stage: 128 rows x 128 K-bytes
constexpr int kGemmBBytes = 256 * 128;           // B stage: 256 rows x 128 K-bytes
constexpr uint32_t kIdescGemm = idesc_m128(256, 1, 0, 0);   // f32 <- e4m3 x e4m3, N = 256
constexpr int kDevGemmTimeout = 0x401;

struct GemmShared {
  uint64_t full[kGemmStages], empty[kGemmStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
constexpr size_t kGemmSmemBytes = 1024 + kGemmStages * (kGemmABytes + kGemmBBytes) + sizeof(GemmShared);

__global__ void __launch_bounds__(kGemmThreads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const Fp8GemmArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + kGemmStages * kGemmABytes;
  GemmShared* sh = reinterpret_cast<GemmShared*>(sB + kGemmStages * kGemmBBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb_total = (a.K + 127) / 128;
  const int total = a.tiles_m * a.tiles_n;
  volatile int* abort_flag = &sh->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh->acc_full[b], 1);
      mbar_init(&sh->acc_empty[b], 256);
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
    // ------------------------------------------------ TMA producer
    if (elect_one()) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
    }
    __syncwarp();
    int it = 0, issued = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
      const int tm = tile / a.tiles_n, tn = tile - tm * a.tiles_n;
      for (int kb = 0; kb < kb_total; ++kb, ++it) {
        const int s = it % kGemmStages;
        if (!(ok = mbar_wait_role(&sh->empty[s], ((it / kGemmStages) & 1) ^ 1, abort_flag, a.status, kDevGemmTimeout)))
          break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&sh->full[s], kGemmABytes + kGemmBBytes);
          tma_load_3d(sA + s * kGemmABytes, &tm_a, &sh->full[s], kb * 128, tm * 128, 0);
          tma_load_3d(sB + s * kGemmBBytes, &tm_b, &sh->full[s], kb * 128, tn * 256, 0);
        }
        __syncwarp();
        issued = it + 1;
      }
    }
    if (*abort_flag) {                                // let the copies in flight land before exiting
      for (int i = (issued > kGemmStages ? issued - kGemmStages : 0); i < issued; ++i)
        mbar_drain_wait(&sh->full[i % kGemmStages], (i / kGemmStages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    const uint64_t adesc0 = smem_desc_sw128(smem_u32(sA)), bdesc0 = smem_desc_sw128(smem_u32(sB));
    int it = 0, lt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x, ++lt) {
      const int buf = lt & 1;
      if (!(ok = mbar_wait_role(&sh->acc_empty[buf], ((lt >> 1) & 1) ^ 1, abort_flag, a.status, kDevGemmTimeout)))
        break;
      tc_fence_after();
      for (int kb = 0; kb < kb_total; ++kb, ++it) {
        const int s = it % kGemmStages;
        if (!(ok = mbar_wait_role(&sh->full[s], (it / kGemmStages) & 1, abort_flag, a.status, kDevGemmTimeout)))
          break;
        tc_fence_after();
        if (elect_one()) {
          const uint64_t ad = adesc0 + uint64_t(s) * (kGemmABytes >> 4), bd = bdesc0 + uint64_t(s) * (kGemmBBytes >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)                 // 32 e4m3 (32 bytes) per instruction
            mma_f8_ss(tmem + 256 * buf, ad + 2 * kk, bd + 2 * kk, kIdescGemm, (kb > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&sh->empty[s]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (elect_one()) tc_commit(&sh->acc_full[buf]);
      __syncwarp();
    }
    if (elect_one()) tc_commit(&sh->drain);             // every MMA issued here has completed once it flips
    __syncwarp();
    mbar_drain_wait(&sh->drain, 0);
  } else {
    // ------------------------------------------------ epilogue: TMEM -> scales, bias -> bf16 (8 warps)
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    int lt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x, ++lt) {
      const int tm = tile / a.tiles_n, tn = tile - tm * a.tiles_n;
      const int buf = lt & 1;
      if (!(ok = mbar_wait(&sh->acc_full[buf], (lt >> 1) & 1, abort_flag, a.status, kDevGemmTimeout))) break;
      tc_fence_after();
      const int row = tm * 128 + quarter * 32 + lane;
      const bool row_ok = row < a.M;
      const float xs = row_ok ? a.x_scale[row] : 0.f;
      __nv_bfloat16* dst = a.y + int64_t(row) * a.sy + tn * 256;
#pragma unroll 1
      for (int c = 4 * half; c < 4 * half + 4; ++c) {
        const int col0 = tn * 256 + c * 32;
        uint32_t v[32];
        tmem_ld32(tmem + 256 * buf + 32 * c + lane_off, v);
        tmem_ld_wait(v);
        if (col0 >= a.N) continue;                      // warp-uniform
        uint32_t packed[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int n = col0 + 2 * e;
          float o0 = __fmul_rn(__fmul_rn(__uint_as_float(v[2 * e]), xs), __ldg(a.w_scale + n));
          float o1 = __fmul_rn(__fmul_rn(__uint_as_float(v[2 * e + 1]), xs), __ldg(a.w_scale + n + 1));
          if (a.bias != nullptr) {
            o0 = __fadd_rn(o0, __bfloat162float(a.bias[n]));
            o1 = __fadd_rn(o1, __bfloat162float(a.bias[n + 1]));
          }
          packed[e] = pack_act2(o0, o1, 0);
        }
        if (row_ok && a.wide_stores) {                 // 32-byte aligned rows: two 256-bit stores
#pragma unroll
          for (int q = 0; q < 2; ++q) st_global_v8(dst + c * 32 + 16 * q, packed + 8 * q);
        } else if (row_ok) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            reinterpret_cast<uint4*>(dst + c * 32)[q] =
                make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&sh->acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

cudaError_t launch_fp8_quant_rows(const Fp8QuantArgs& a, cudaStream_t st) {
  if (a.rows <= 0) return cudaSuccess;
  fp8_quant_rows_kernel<<<a.rows, 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_fp8_gemm(const Fp8GemmArgs& a, const CUtensorMap& tm_a, const CUtensorMap& tm_b, int ctas,
                            cudaStream_t st) {
  if (cudaError_t e = allow_dynamic_smem<fp8_gemm_kernel>(int(kGemmSmemBytes)); e != cudaSuccess) return e;
  fp8_gemm_kernel<<<ctas, kGemmThreads, kGemmSmemBytes, st>>>(tm_a, tm_b, a);
  return cudaGetLastError();
}

}  // namespace lbq
