// lbq_quant_qkv_static: the per-call Q/K/V quantization of lbq_quant_qkv, for callers that cannot
// give this library any device memory of its own — an embedding runtime that owns a fixed,
// pre-sized device memory pool and forbids allocation once serving has started, or an FFI binding
// that can pass the call's inputs and outputs but has no way to hand over a workspace. Its scratch
// (the per-64-token block statistics and the per-channel window totals) lives in the file-scope
// array below, so the call itself allocates nothing.
//
// Limits and sharing rules:
//  * The array holds kStaticScratchBytes (16 MiB). A call needs lbq_quant_qkv_workspace(batch,
//    heads, kv_len) bytes of it, batch * heads * (ceil(kv_len / 64) + 1) * 1536 + 64 — e.g. up to
//    58176 keys at 12 heads and batch 1 — and is rejected with LBQ_ERR_ARG beyond that.
//  * Every GPU that loads the library keeps its own copy of the array until the process exits.
//  * All calls on a device share that copy and it keeps the last call's contents. No part of it
//    has to start at zero: each call writes every entry it reads before reading it. Two calls
//    whose kernels overlap on the GPU (different streams without ordering) race on the array.
//  * The first call on a device looks up the array's device address (cudaGetSymbolAddress, with
//    that device current) and caches it; make that first call before any stream capture begins.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/lbq.h"
#include "lbq_kernels.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;

// Device-side scratch. In host code this name is only a stand-in for the symbol: its device
// address comes from cudaGetSymbolAddress below, never from taking the address here.
static __device__ __align__(256) unsigned char g_quant_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;

// Looks up (once per device, with that device current) the device address of g_quant_scratch.
cudaError_t scratch_address(void** out) {
  static void* addr[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_quant_scratch);
    if (e != cudaSuccess) return e;
    addr[dev] = p;
  }
  *out = addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" {

int lbq_quant_qkv_static(const void* q, int64_t sq_b, int64_t sq_l, int64_t sq_h, int q_len, const void* k,
                         int64_t sk_b, int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b, int64_t sv_l,
                         int64_t sv_h, int64_t kv_len, int batch, int heads, int8_t* q_codes, float* q_scale,
                         int8_t* k_codes, float* k_scale, uint8_t* vt_codes, float* v_scale, void* km_out,
                         int dtype, void* stream) {
  if (batch <= 0 || heads <= 0 || batch > 65535 || heads > 65535 || kv_len <= 0 || kv_len > (int64_t(1) << 30))
    return lbq::set_error(LBQ_ERR_ARG, "batch and heads must be in 1..65535 and kv_len in 1..2^30");
  const size_t need = lbq_quant_qkv_workspace(batch, heads, kv_len);
  if (need > kStaticScratchBytes)
    return lbq::set_error(LBQ_ERR_ARG,
                          "lbq_quant_qkv_static: batch %d x heads %d x kv_len %lld needs %zu bytes of scratch, "
                          "more than its static %zu bytes; use lbq_quant_qkv with a workspace",
                          batch, heads, (long long)kv_len, need, kStaticScratchBytes);
  void* scratch = nullptr;
  const cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess)
    return lbq::set_error(LBQ_ERR_CUDA, "lbq_quant_qkv_static: address of the static scratch: %s",
                          cudaGetErrorString(e));
  return lbq_quant_qkv(q, sq_b, sq_l, sq_h, q_len, k, sk_b, sk_l, sk_h, v, sv_b, sv_l, sv_h, kv_len, batch, heads,
                       q_codes, q_scale, k_codes, k_scale, vt_codes, v_scale, km_out, scratch,
                       kStaticScratchBytes, dtype, stream);
}

}  // extern "C"
