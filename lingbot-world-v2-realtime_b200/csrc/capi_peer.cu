// C ABI of the sequence-split exchange (declared in include/lbq.h): peer-heap mapping through CUDA IPC
// and the four exchange launches. Validation mirrors capi.cu; errors go to lbq_last_error().
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/lbq.h"
#include "lbq_kernels.h"

namespace {

using lbq::set_error;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_share(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b, int64_t sv_l,
                int64_t sv_h) {
  if (k == nullptr || v == nullptr) return set_error(LBQ_ERR_ARG, "share k/v is null");
  if (!aligned16(k) || !aligned16(v)) return set_error(LBQ_ERR_ALIGN, "share k/v not 16-byte aligned");
  for (int64_t s : {sk_b, sk_l, sk_h, sv_b, sv_l, sv_h})
    if (s < 0 || s % 8) return set_error(LBQ_ERR_ALIGN, "share strides must be non-negative multiples of 8 elements");
  return LBQ_OK;
}

int check_group(const uint64_t* peers, int nranks, int rank, int64_t xchg_off) {
  if (peers == nullptr) return set_error(LBQ_ERR_ARG, "peers table is null");
  if (nranks < 1 || nranks > lbq::xchg::kMaxRanks)
    return set_error(LBQ_ERR_ARG, "nranks %d outside [1, %d]", nranks, lbq::xchg::kMaxRanks);
  if (rank < 0 || rank >= nranks) return set_error(LBQ_ERR_ARG, "rank %d outside [0, %d)", rank, nranks);
  if (xchg_off < 0 || xchg_off % 256) return set_error(LBQ_ERR_ALIGN, "xchg_off must be a non-negative multiple of 256");
  return LBQ_OK;
}

int check_dims(int batch, int heads, int nb_part) {
  if (batch <= 0 || heads <= 0 || nb_part <= 0) return set_error(LBQ_ERR_ARG, "batch, heads and nb_part must be positive");
  if (heads > 65535 || batch > 65535 || nb_part > (1 << 20)) return set_error(LBQ_ERR_ARG, "grid too large");
  return LBQ_OK;
}

PFN_cuMemGetAddressRange_v3020 range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}

}  // namespace

extern "C" {

int lbq_peer_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return set_error(LBQ_ERR_ARG, "ptr, handle_out and offset_out must be non-null");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  auto fn = range_fn();
  if (fn == nullptr) return set_error(LBQ_ERR_CUDA, "cuMemGetAddressRange unavailable from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult cr = fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (cr != CUDA_SUCCESS) return set_error(LBQ_ERR_CUDA, "cuMemGetAddressRange: CUresult %d", int(cr));
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return set_error(LBQ_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = uint64_t(reinterpret_cast<uintptr_t>(ptr) - uintptr_t(base));
  return LBQ_OK;
}

int lbq_peer_open(const void* handle, void** base_out) {
  if (handle == nullptr || base_out == nullptr) return set_error(LBQ_ERR_ARG, "handle and base_out must be non-null");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(LBQ_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  return LBQ_OK;
}

int lbq_peer_close(void* base) {
  if (base == nullptr) return set_error(LBQ_ERR_ARG, "base is null");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return set_error(LBQ_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return LBQ_OK;
}

int64_t lbq_exchange_bytes(int nranks, int batch, int heads) {
  if (nranks < 1 || nranks > lbq::xchg::kMaxRanks || batch <= 0 || heads <= 0) return -1;
  return lbq::xchg::bytes(nranks, int64_t(batch) * heads * 128);
}

int lbq_share_totals_push(const double* ksum, const float* vamax, int64_t max_blocks, int row0, int nb_valid,
                          int batch, int heads, const uint64_t* peers, int nranks, int rank, int64_t xchg_off,
                          void* stream) {
  int r;
  if ((r = check_group(peers, nranks, rank, xchg_off)) || (r = check_dims(batch, heads, 1))) return r;
  if (ksum == nullptr || vamax == nullptr) return set_error(LBQ_ERR_ARG, "block tables are null");
  if (row0 < 0 || nb_valid < 0 || row0 + nb_valid > max_blocks)
    return set_error(LBQ_ERR_ARG, "rows [%d, %d) outside tables of %lld rows", row0, row0 + nb_valid,
                     (long long)max_blocks);
  lbq::ShareTotalsArgs a{ksum, vamax, max_blocks, row0, nb_valid, batch, heads, peers, nranks, rank, xchg_off};
  cudaError_t e = lbq::launch_share_totals_push(a, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : set_error(LBQ_ERR_CUDA, "share_totals_push launch: %s", cudaGetErrorString(e));
}

int lbq_chunk_totals(const uint64_t* peers, int nranks, int rank, int64_t xchg_off, int batch, int heads,
                     const double* mem_ksum, const float* mem_vamax, double* tot_ksum, float* tot_vamax,
                     uint64_t timeout_ns, void* stream) {
  int r;
  if ((r = check_group(peers, nranks, rank, xchg_off)) || (r = check_dims(batch, heads, 1))) return r;
  if (!mem_ksum || !mem_vamax || !tot_ksum || !tot_vamax)
    return set_error(LBQ_ERR_ARG, "memory and window totals must be non-null");
  int* status = lbq::device_status_ptr();
  if (status == nullptr) return set_error(LBQ_ERR_CUDA, "device status word unavailable");
  lbq::ChunkTotalsArgs a{peers, nranks, rank, xchg_off, batch, heads, mem_ksum, mem_vamax, tot_ksum, tot_vamax,
                         timeout_ns, status};
  cudaError_t e = lbq::launch_chunk_totals(a, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : set_error(LBQ_ERR_CUDA, "chunk_totals launch: %s", cudaGetErrorString(e));
}

int lbq_share_push(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b, int64_t sv_l,
                   int64_t sv_h, int batch, int heads, int share_valid, int nb_part, const uint64_t* peers, int nranks,
                   int rank, int64_t xchg_off, int64_t cache_k_off, int64_t cache_v_off, int64_t cache_tokens,
                   int64_t dst_tok0, int64_t tbl_ksum_off, int64_t tbl_vamax_off, int64_t tbl_max_blocks,
                   int ctas, void* stream) {
  int r;
  if ((r = check_share(k, sk_b, sk_l, sk_h, v, sv_b, sv_l, sv_h)) || (r = check_group(peers, nranks, rank, xchg_off)) ||
      (r = check_dims(batch, heads, nb_part)))
    return r;
  if (share_valid < 0 || share_valid > nb_part * 64)
    return set_error(LBQ_ERR_ARG, "share_valid %d not in [0, %d]", share_valid, nb_part * 64);
  if (cache_k_off < 0 || cache_v_off < 0 || cache_k_off % 16 || cache_v_off % 16 || tbl_ksum_off < 0 ||
      tbl_vamax_off < 0 || tbl_ksum_off % 16 || tbl_vamax_off % 16)
    return set_error(LBQ_ERR_ALIGN, "heap offsets must be non-negative multiples of 16 bytes");
  if (dst_tok0 < 0 || dst_tok0 % 64 || dst_tok0 + share_valid > cache_tokens)
    return set_error(LBQ_ERR_ARG, "share [%lld, %lld) must start on a 64-token block inside a cache of %lld tokens",
                     (long long)dst_tok0, (long long)(dst_tok0 + share_valid), (long long)cache_tokens);
  if (dst_tok0 / 64 + (share_valid + 63) / 64 > tbl_max_blocks)
    return set_error(LBQ_ERR_ARG, "share blocks past the %lld rows of the block tables", (long long)tbl_max_blocks);
  if (int64_t(nb_part) * heads * batch > (int64_t(1) << 31) - 1) return set_error(LBQ_ERR_ARG, "too many share units");
  if (ctas < 0 || ctas > 65535) return set_error(LBQ_ERR_ARG, "ctas %d outside [0, 65535]", ctas);
  lbq::SharePushArgs a{static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v), sk_b, sk_l, sk_h,
                       sv_b, sv_l, sv_h, batch, heads, share_valid, nb_part, peers, nranks, rank, xchg_off,
                       cache_k_off, cache_v_off, cache_tokens, dst_tok0, tbl_ksum_off, tbl_vamax_off, tbl_max_blocks,
                       lbq::xchg::push_ctas(nb_part * heads * batch, ctas)};
  cudaError_t e = lbq::launch_share_push(a, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : set_error(LBQ_ERR_CUDA, "share_push launch: %s", cudaGetErrorString(e));
}

int lbq_share_quant_push(const void* k, int64_t sk_b, int64_t sk_l, int64_t sk_h, const void* v, int64_t sv_b,
                         int64_t sv_l, int64_t sv_h, int batch, int heads, int lo, int share_valid, int part, int seg,
                         int num_segments, int seg_len, int64_t kv_len_total, const double* ksum_total,
                         const float* vamax_total, int8_t* k_codes, float* k_scale, uint8_t* vt_codes, void* km_out,
                         float* v_scale, int write_totals, const uint64_t* peers, int nranks, int rank,
                         int64_t xchg_off, int ctas, void* stream) {
  int r;
  if ((r = check_share(k, sk_b, sk_l, sk_h, v, sv_b, sv_l, sv_h)) || (r = check_group(peers, nranks, rank, xchg_off)) ||
      (r = check_dims(batch, heads, 1)))
    return r;
  if (!ksum_total || !vamax_total || !k_codes || !k_scale || !vt_codes)
    return set_error(LBQ_ERR_ARG, "totals and code buffers must be non-null");
  if (!aligned16(k_codes) || !aligned16(vt_codes)) return set_error(LBQ_ERR_ALIGN, "code buffers not 16-byte aligned");
  if (write_totals && v_scale == nullptr) return set_error(LBQ_ERR_ARG, "v_scale is null");
  if (part <= 0 || part % 128 || lo < 0 || lo % 128)
    return set_error(LBQ_ERR_ARG, "share start %d and size %d must be multiples of 128", lo, part);
  if (share_valid < 0 || share_valid > part) return set_error(LBQ_ERR_ARG, "share_valid %d not in [0, %d]", share_valid, part);
  if (num_segments <= 0 || seg < 0 || seg >= num_segments || seg_len <= 0)
    return set_error(LBQ_ERR_ARG, "segment %d of %d (%d tokens)", seg, num_segments, seg_len);
  if (num_segments > 1 && seg_len % 64) return set_error(LBQ_ERR_ARG, "seg_len %d must be a multiple of 64", seg_len);
  if (int64_t(lo) + share_valid > seg_len)
    return set_error(LBQ_ERR_ARG, "share [%d, %d) past the %d-token segment", lo, lo + share_valid, seg_len);
  if (kv_len_total <= 0) return set_error(LBQ_ERR_ARG, "kv_len_total must be positive");
  if (ctas < 0 || ctas > 65535) return set_error(LBQ_ERR_ARG, "ctas %d outside [0, 65535]", ctas);
  const int seg_pad = int((int64_t(seg_len) + 127) / 128 * 128);
  const int tile0 = lo / 128;
  int tile_end = (lo + share_valid + 127) / 128;
  if (tile_end > seg_pad / 128) tile_end = seg_pad / 128;
  if (share_valid == 0) tile_end = tile0;
  const int64_t tok0 = -int64_t(lo);   // segment token t is share token t - lo
  lbq::QuantKArgs ka{static_cast<const __nv_bfloat16*>(k), sk_b, sk_l, sk_h, batch, heads, tok0, seg, lo + share_valid,
                     seg_pad, kv_len_total, ksum_total, k_codes, k_scale, static_cast<__nv_bfloat16*>(km_out),
                     write_totals, lbq::device_status_ptr()};
  lbq::QuantVArgs va{static_cast<const __nv_bfloat16*>(v), sv_b, sv_l, sv_h, batch, heads, tok0, seg, lo + share_valid,
                     seg_pad, vamax_total, vt_codes, v_scale, write_totals, lbq::device_status_ptr()};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = lbq::launch_quant_kv(ka, va, tile0, tile_end - tile0, st);
  if (e != cudaSuccess) return set_error(LBQ_ERR_CUDA, "share quant launch: %s", cudaGetErrorString(e));
  if (nranks == 1) return LBQ_OK;
  lbq::CodePushArgs ca{k_codes, k_scale, vt_codes, batch, heads, seg, seg_pad, lo, (tile_end - tile0) * 128,
                       peers, nranks, rank, xchg_off};
  e = lbq::launch_code_push(ca, ctas > 0 ? ctas : 32, st);
  return e == cudaSuccess ? LBQ_OK : set_error(LBQ_ERR_CUDA, "code push launch: %s", cudaGetErrorString(e));
}

int lbq_q_push(const int8_t* q_codes, const float* q_scale, int rows_pad, int row0, int q_pad, int batch, int heads,
               int64_t q_off, int64_t q_scale_off, const uint64_t* peers, int nranks, int rank, int64_t xchg_off,
               int ctas, void* stream) {
  int r;
  if ((r = check_group(peers, nranks, rank, xchg_off)) || (r = check_dims(batch, heads, 1))) return r;
  if (q_codes == nullptr || q_scale == nullptr) return set_error(LBQ_ERR_ARG, "query codes are null");
  if (!aligned16(q_codes) || !aligned16(q_scale)) return set_error(LBQ_ERR_ALIGN, "query codes not 16-byte aligned");
  if (rows_pad < 0 || rows_pad % 128 || row0 < 0 || row0 % 128 || q_pad % 128 || row0 + rows_pad > q_pad)
    return set_error(LBQ_ERR_ARG, "rows [%d, %d) of %d: all multiples of 128 and inside", row0, row0 + rows_pad, q_pad);
  if (q_off < 0 || q_off % 16 || q_scale_off < 0 || q_scale_off % 16)
    return set_error(LBQ_ERR_ALIGN, "heap offsets must be non-negative multiples of 16 bytes");
  if (ctas < 0 || ctas > 65535) return set_error(LBQ_ERR_ARG, "ctas %d outside [0, 65535]", ctas);
  lbq::QPushArgs a{q_codes, q_scale, rows_pad, row0, q_pad, batch, heads, q_off, q_scale_off, peers, nranks, rank,
                   xchg_off};
  cudaError_t e = lbq::launch_q_push(a, ctas > 0 ? ctas : 32, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : set_error(LBQ_ERR_CUDA, "q_push launch: %s", cudaGetErrorString(e));
}

int lbq_peer_wait(const uint64_t* peers, int nranks, int rank, int64_t xchg_off, int signals, uint64_t timeout_ns,
                  void* stream) {
  int r;
  if ((r = check_group(peers, nranks, rank, xchg_off))) return r;
  if (signals < 1 || signals > 2) return set_error(LBQ_ERR_ARG, "signals %d not in [1, 2]", signals);
  int* status = lbq::device_status_ptr();
  if (status == nullptr) return set_error(LBQ_ERR_CUDA, "device status word unavailable");
  lbq::PeerWaitArgs a{peers, nranks, rank, xchg_off, uint32_t(signals), timeout_ns, status};
  cudaError_t e = lbq::launch_peer_wait(a, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? LBQ_OK : set_error(LBQ_ERR_CUDA, "peer_wait launch: %s", cudaGetErrorString(e));
}

}  // extern "C"
