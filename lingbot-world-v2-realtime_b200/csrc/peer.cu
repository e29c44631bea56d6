// Sequence-split exchange over NVLink peer memory, sm_100a.
//
// Every rank of a sequence split holds a replica of the layer KV caches and an exchange area, all
// inside one "peer heap" (a device buffer that every other rank of the node has mapped through CUDA
// IPC). All ranks carve the heap identically, so a buffer is named by its byte offset and rank p's
// copy lives at peers[p] + offset. The kernels below replace the all-reduce of the chunk statistics
// and the all-gather of the chunk's K/V (lingbot/parallel/split_dit.py:366-445 exchanges heads and
// tokens through host-staged copies instead):
//
//   share_totals_push  per-channel totals (fp64 K sum, max |V|) of this rank's share, from the block
//                      statistics lbq_kv_block_stats wrote into this rank's cache tables, stored
//                      into every rank's slot for this rank as tagged 8-byte words.
//   chunk_totals       waits for every rank's tagged totals and adds the memory totals and the
//                      shares' in rank order (bit-identical on every rank).
//   code_push          copies this rank's share of the chunk-segment codes (quantized locally by
//                      quant_kv_kernel) into every other rank's code buffers, then one signal per rank.
//   share_push         copies this rank's bf16 K/V share and its block statistics into every rank's
//                      cache replica and tables (calls whose K/V persist), then one signal per rank.
//   peer_wait          waits for every other rank's signals of this call.
//   q_push             (key-range split) this rank's query-slice codes into every rank's full query
//                      buffers, then one signal per rank; the partials come back from the attention
//                      kernel itself (attn.cu, key-range variant) and are merged by keys_combine.
//
// The totals travel as tagged words: each 8-byte store carries 32 data bits and the call's tag (call
// counter + 1, kept on the device by every rank in lockstep), so the receiver polls the data itself.
// The pushes signal with monotonic u32 counters in the receiver's exchange area: every CTA fences its
// stores at system scope and counts itself done, and the last one raises each receiver's counter with
// a system-scope release add; the receiver keeps how many it has consumed ("seen") in its own area.
// No host-side epoch is needed, so the launches can be replayed from a CUDA graph. Every wait is
// bounded (time limit in the arguments) and records a status code instead of hanging.
//
// Reuse without overwriting what a rank still reads: totals slots are double-buffered by call parity,
// and rank r writes its call-c+1 totals only after it read every rank's call-c totals, which each rank
// sends after finishing its call c-1 reads. The pushes of call c into another rank's code buffers and
// cache start after this rank's call-c window totals, i.e. after every rank sent its call-c totals,
// which each rank does after its call c-1 attention, the last reader of those buffers.
#include <cuda_bf16.h>
#include <cstdint>

#include "lbq_ptx.cuh"
#include "lbq_kernels.h"
#include "lbq_peer.cuh"

namespace lbq {


// ------------------------------------------------------------------ share totals -> every rank
// One CTA per (32-channel group, head, batch), 256 threads = 32 channels x 8 block groups: per
// channel, the fp64 sum of the share's block sums and the max of its block maxima (this rank's cache
// tables, rows [row0, row0 + nb_valid), written by lbq_kv_block_stats). Each rank's slot receives three
// tagged words per channel (the two halves of the sum and the max), each an 8-byte store of 32 data bits
// and the call's tag, so the receiver needs no fence or separate signal: a word is complete when its
// tag is this call's.
__global__ void __launch_bounds__(256) share_totals_push_kernel(ShareTotalsArgs a) {
  const int cg = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int c = cg * 32 + (threadIdx.x & 31), g = threadIdx.x >> 5;
  double s = 0.0;
  float vm = 0.f;
#pragma unroll 4
  for (int blk = g; blk < a.nb_valid; blk += 8) {
    const int64_t o = ((int64_t(b) * a.max_blocks + a.row0 + blk) * a.heads + h) * 128 + c;
    s += a.ksum[o];
    vm = fmaxf(vm, a.vamax[o]);
  }
  __shared__ double sh_s[8][32];
  __shared__ float sh_v[8][32];
  sh_s[g][threadIdx.x & 31] = s;
  sh_v[g][threadIdx.x & 31] = vm;
  __syncthreads();
  if (g != 0) return;
  double tot = 0.0;
  float vmax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    tot += sh_s[i][threadIdx.x];
    vmax = fmaxf(vmax, sh_v[i][threadIdx.x]);
  }
  const char* mine = heap(a.peers, a.rank) + a.xchg_off;
  const uint32_t call = *reinterpret_cast<const volatile uint32_t*>(mine + xchg::kCall);
  const uint64_t tag = uint64_t(call + 1u) << 32;
  const int64_t cols = int64_t(a.batch) * a.heads * 128;
  const int64_t col = (int64_t(b) * a.heads + h) * 128 + c;
  const uint64_t w0 = tag | uint32_t(__double2loint(tot));
  const uint64_t w1 = tag | uint32_t(__double2hiint(tot));
  const uint64_t w2 = tag | __float_as_uint(vmax);
  for (int q = 0; q < a.nranks; ++q) {
    uint64_t* slot = reinterpret_cast<uint64_t*>(heap(a.peers, (a.rank + 1 + q) % a.nranks) + a.xchg_off +
                                                 xchg::kSlots) +
                     xchg::slot_word(call & 1u, a.nranks, a.rank, 0, cols) + col;
    st_relaxed_sys_u64(slot, w0);
    st_relaxed_sys_u64(slot + cols, w1);
    st_relaxed_sys_u64(slot + 2 * cols, w2);
  }
}

// ------------------------------------------------------------------ window totals of the split window
// One CTA per (head, batch), one channel per thread: waits for every rank's three tagged words of its
// channel, then tot = memory totals + the ranks' share totals in rank order (the same sum on every
// rank). The last CTA to finish advances the call counter (the tag and the slot parity).
__global__ void __launch_bounds__(128) chunk_totals_kernel(ChunkTotalsArgs a) {
  const int h = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
  char* mine = heap(a.peers, a.rank) + a.xchg_off;
  const uint32_t call = *reinterpret_cast<const volatile uint32_t*>(mine + xchg::kCall);
  const uint32_t tag = call + 1u;
  const int64_t cols = int64_t(a.batch) * a.heads * 128;
  const int64_t col = (int64_t(b) * a.heads + h) * 128 + t;
  const uint64_t* slots = reinterpret_cast<const uint64_t*>(mine + xchg::kSlots);
  __shared__ int sh_fail;
  if (t == 0) sh_fail = 0;
  __syncthreads();
  double s = a.mem_ksum[col];
  float vm = a.mem_vamax[col];
  bool ok = true;
  const uint64_t t0 = globaltimer_ns();
  for (int r = 0; r < a.nranks && ok; ++r) {
    const uint64_t* w = slots + xchg::slot_word(call & 1u, a.nranks, r, 0, cols) + col;
    uint64_t v0, v1, v2;
    for (uint32_t i = 0;; ++i) {
      v0 = ld_relaxed_sys_u64(w);
      v1 = ld_relaxed_sys_u64(w + cols);
      v2 = ld_relaxed_sys_u64(w + 2 * cols);
      if (uint32_t(v0 >> 32) == tag && uint32_t(v1 >> 32) == tag && uint32_t(v2 >> 32) == tag) break;
      if (i >= LBQ_SPIN_LIMIT || ((i & 63) == 63 && globaltimer_ns() - t0 > a.timeout_ns)) {
        ok = false;
        break;
      }
      __nanosleep(32);
    }
    if (ok) {
      s += __hiloint2double(int(uint32_t(v1)), int(uint32_t(v0)));
      vm = fmaxf(vm, __uint_as_float(uint32_t(v2)));
    }
  }
  if (!ok) {
    sh_fail = 1;
    atomicCAS(a.status, 0, kDevTimeoutPeerStats);
  }
  __syncthreads();
  if (sh_fail) return;
  a.tot_ksum[col] = s;
  a.tot_vamax[col] = vm;
  __syncthreads();
  if (t == 0) {
    __threadfence();
    uint32_t* done = reinterpret_cast<uint32_t*>(mine + xchg::kDone);
    if (atomicAdd(done, 1u) == gridDim.x * gridDim.y - 1) {
      *reinterpret_cast<uint32_t*>(mine + xchg::kCall) = call + 1u;
      *done = 0;
      __threadfence();
    }
  }
}

// ------------------------------------------------------------------ share -> every rank's cache
// Persistent: `ctas` CTAs stride over the units (64-token block of the share, head,
// batch). Thread = (row group of 4 rows, 16-byte chunk); a unit's K/V rows are read once into
// registers and stored to every rank (CTAs start on different ranks), with the block's statistics row (already in
// this rank's tables) copied to the other ranks' tables. One signal per peer after the last CTA.
__global__ void __launch_bounds__(256) share_push_kernel(SharePushArgs a) {
  const int t = threadIdx.x, c16 = t & 15, rg = t >> 4;
  const int units = a.nb_part * a.heads * a.batch;
  const int nb_valid = (a.share_valid + 63) / 64;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int blk = u % a.nb_part;
    const int h = (u / a.nb_part) % a.heads;
    const int b = u / (a.nb_part * a.heads);
    if (blk >= nb_valid) continue;
    uint4 kr[4], vr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t tok = int64_t(blk) * 64 + rg + 16 * i;
      if (tok < a.share_valid) {
        kr[i] = *reinterpret_cast<const uint4*>(a.k + b * a.sk_b + tok * a.sk_l + h * a.sk_h + c16 * 8);
        vr[i] = *reinterpret_cast<const uint4*>(a.v + b * a.sv_b + tok * a.sv_l + h * a.sv_h + c16 * 8);
      }
    }
    const int64_t row = a.dst_tok0 / 64 + blk;
    const int64_t so = ((int64_t(b) * a.tbl_max_blocks + row) * a.heads + h) * 128 + (t & 127);
    const char* mine = heap(a.peers, a.rank);
    double bs = 0.0;
    float bv = 0.f;
    if (t < 128) bs = reinterpret_cast<const double*>(mine + a.tbl_ksum_off)[so];
    else bv = reinterpret_cast<const float*>(mine + a.tbl_vamax_off)[so];
    for (int q = 0; q < a.nranks; ++q) {
      const int p = (a.rank + 1 + q + blockIdx.x) % a.nranks;   // CTAs start on different ranks
      char* base = heap(a.peers, p);
      __nv_bfloat16* dk = reinterpret_cast<__nv_bfloat16*>(base + a.cache_k_off);
      __nv_bfloat16* dv = reinterpret_cast<__nv_bfloat16*>(base + a.cache_v_off);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t tok = int64_t(blk) * 64 + rg + 16 * i;
        if (tok < a.share_valid) {
          const int64_t o = ((int64_t(b) * a.cache_tokens + a.dst_tok0 + tok) * a.heads + h) * 128 + c16 * 8;
          *reinterpret_cast<uint4*>(dk + o) = kr[i];
          *reinterpret_cast<uint4*>(dv + o) = vr[i];
        }
      }
      if (p != a.rank) {
        if (t < 128) reinterpret_cast<double*>(base + a.tbl_ksum_off)[so] = bs;
        else reinterpret_cast<float*>(base + a.tbl_vamax_off)[so] = bv;
      }
    }
  }
  signal_after_last_cta(a.peers, a.nranks, a.rank, a.xchg_off, xchg::kDonePush);
}

// ------------------------------------------------------------------ share codes -> every other rank
// `ctas` CTAs stride over the 16-byte pieces of this rank's share of the chunk-segment codes (K rows of
// len*128 bytes, then V channel rows of len bytes); each piece is read once and stored to every other
// rank at the same heap offset. CTA 0 also copies the K scales. One signal per rank after the last CTA.
__global__ void __launch_bounds__(256) code_push_kernel(CodePushArgs a) {
  const int64_t bh_rows = int64_t(a.batch) * a.heads;
  const int64_t k_row = int64_t(a.len) * 8;            // 16-byte pieces per K row
  const int64_t v_row = a.len / 16;                    // 16-byte pieces per V channel row
  const int64_t pk = bh_rows * k_row, total = pk + bh_rows * 128 * v_row;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const char* mine = heap(a.peers, a.rank);
  const char* kbase = reinterpret_cast<const char*>(a.k_codes);
  const char* vbase = reinterpret_cast<const char*>(a.vt_codes);
  for (int64_t g0 = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g0 < total; g0 += 4 * stride) {
    uint4 val[4];
    int64_t off[4];                                    // byte offset from this rank's heap base
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t g = g0 + i * stride;
      off[i] = -1;
      if (g < total) {
        const char* src;
        if (g < pk) {
          const int64_t row = g / k_row, col = g - row * k_row;
          src = kbase + ((a.seg * bh_rows + row) * a.seg_pad + a.lo) * 128 + col * 16;
        } else {
          const int64_t gv = g - pk, row = gv / v_row, col = gv - row * v_row;   // row = bh * 128 + channel
          src = vbase + (a.seg * bh_rows * 128 + row) * a.seg_pad + a.lo + col * 16;
        }
        off[i] = src - mine;
        val[i] = *reinterpret_cast<const uint4*>(src);
      }
    }
    for (int q = 0; q + 1 < a.nranks; ++q) {
      // every other rank once, CTAs starting on different ones
      char* dst = heap(a.peers, (a.rank + 1 + (q + int(blockIdx.x)) % (a.nranks - 1)) % a.nranks);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (off[i] >= 0) *reinterpret_cast<uint4*>(dst + off[i]) = val[i];
    }
  }
  if (blockIdx.x == 0) {
    const int per = a.len / 64;
    for (int64_t i = threadIdx.x; i < bh_rows * per; i += blockDim.x) {
      const int64_t row = i / per;
      const float* src = a.k_scale + (a.seg * bh_rows + row) * (a.seg_pad / 64) + a.lo / 64 + (i - row * per);
      const int64_t off = reinterpret_cast<const char*>(src) - mine;
      const float v = *src;
      for (int q = 1; q < a.nranks; ++q)
        *reinterpret_cast<float*>(heap(a.peers, (a.rank + q) % a.nranks) + off) = v;
    }
  }
  signal_after_last_cta(a.peers, a.nranks, a.rank, a.xchg_off, xchg::kDoneQuant);
}

// ------------------------------------------------------------------ query-slice codes -> every rank
// Key-range split: every rank attends every query row against its own keys, so each rank's query-slice
// codes (quantized locally into a [B][H][rows_pad][128] buffer) and scales go to rows [row0, row0 +
// rows_pad) of every rank's full query buffers, this rank's own included, in 16-byte pieces (CTAs start
// on different ranks); then one signal per other rank.
__global__ void __launch_bounds__(256) q_push_kernel(QPushArgs a) {
  const int64_t bh_rows = int64_t(a.batch) * a.heads;
  const int64_t code_row = int64_t(a.rows_pad) * 8;    // 16-byte pieces of one (b, h) block of codes
  const int64_t scale_row = a.rows_pad / 128;          // 16-byte pieces of its rows_pad / 32 scales
  const int64_t pc = bh_rows * code_row, total = pc + bh_rows * scale_row;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const char* codes = reinterpret_cast<const char*>(a.q_codes);
  const char* scales = reinterpret_cast<const char*>(a.q_scale);
  for (int64_t g0 = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g0 < total; g0 += 4 * stride) {
    uint4 val[4];
    int64_t off[4];                                    // byte offset of the destination in every heap
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t g = g0 + i * stride;
      off[i] = -1;
      if (g < total) {
        const char* src;
        if (g < pc) {
          const int64_t row = g / code_row, col = g - row * code_row;
          src = codes + row * a.rows_pad * 128 + col * 16;
          off[i] = a.q_off + (row * a.q_pad + a.row0) * 128 + col * 16;
        } else {
          const int64_t gs = g - pc, row = gs / scale_row, col = gs - row * scale_row;
          src = scales + row * (a.rows_pad / 8) + col * 16;
          off[i] = a.q_scale_off + row * (a.q_pad / 8) + a.row0 / 8 + col * 16;
        }
        val[i] = *reinterpret_cast<const uint4*>(src);
      }
    }
    for (int q = 0; q < a.nranks; ++q) {
      char* dst = heap(a.peers, (a.rank + q + int(blockIdx.x)) % a.nranks);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (off[i] >= 0) *reinterpret_cast<uint4*>(dst + off[i]) = val[i];
    }
  }
  signal_after_last_cta(a.peers, a.nranks, a.rank, a.xchg_off, xchg::kDoneQuant);
}

// ------------------------------------------------------------------ wait for the other ranks' shares
__global__ void __launch_bounds__(32) peer_wait_kernel(PeerWaitArgs a) {
  const int t = threadIdx.x;
  char* mine = heap(a.peers, a.rank) + a.xchg_off;
  uint32_t* seen = reinterpret_cast<uint32_t*>(mine + xchg::kSeenData);
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(mine + xchg::kFlagsData);
  if (t < a.nranks && t != a.rank) {
    const uint32_t target = seen[t] + a.signals;
    if (wait_counter(flags + t, target, a.timeout_ns)) {
      seen[t] = target;
    } else {
      atomicCAS(a.status, 0, kDevTimeoutPeerData);
    }
  }
  __threadfence_system();
}

cudaError_t launch_share_totals_push(const ShareTotalsArgs& a, cudaStream_t st) {
  if (cudaError_t e0 = prefer_max_shared<share_totals_push_kernel>(); e0 != cudaSuccess) return e0;
  share_totals_push_kernel<<<dim3(4, a.heads, a.batch), 256, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_chunk_totals(const ChunkTotalsArgs& a, cudaStream_t st) {
  if (cudaError_t e0 = prefer_max_shared<chunk_totals_kernel>(); e0 != cudaSuccess) return e0;
  chunk_totals_kernel<<<dim3(a.heads, a.batch), 128, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_share_push(const SharePushArgs& a, cudaStream_t st) {
  if (cudaError_t e0 = prefer_max_shared<share_push_kernel>(); e0 != cudaSuccess) return e0;
  share_push_kernel<<<a.ctas, 256, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_code_push(const CodePushArgs& a, int ctas, cudaStream_t st) {
  if (cudaError_t e0 = prefer_max_shared<code_push_kernel>(); e0 != cudaSuccess) return e0;
  code_push_kernel<<<ctas, 256, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_q_push(const QPushArgs& a, int ctas, cudaStream_t st) {
  if (cudaError_t e0 = prefer_max_shared<q_push_kernel>(); e0 != cudaSuccess) return e0;
  q_push_kernel<<<ctas, 256, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_peer_wait(const PeerWaitArgs& a, cudaStream_t st) {
  if (cudaError_t e0 = prefer_max_shared<peer_wait_kernel>(); e0 != cudaSuccess) return e0;
  peer_wait_kernel<<<1, 32, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace lbq
