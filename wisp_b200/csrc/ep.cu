// ep.cu -- device-side plumbing of the expert-parallel exchange.
//
// The reference engine runs on one GPU and has no expert parallelism; these
// kernels serve the multi-GPU path (wisp_b200/ep.py), where routed experts
// are sharded in contiguous blocks of E/N over N ranks and token rows travel
// to their experts' owner and back through fixed-size NCCL all-to-all
// exchanges. Fixed sizes keep every count on the device: no host round trip
// sits between routing and the expert FFN.
//
// Layout of the exchange buffers: rank r's send buffer holds, for each
// destination q, a block of `cap` rows (cap = tokens * top_k, the most any
// one destination can receive); the rows for q occupy the block's first
// rows in expert order. After the all-to-all, the receive buffer holds the
// source blocks in rank order, so source s's rows for local expert e start
// at s*cap + (rows s sends for experts before e). Before the expert FFN the
// received rows are gathered expert-contiguous, so each local expert is ONE
// segment (its weights are streamed once, whatever the number of ranks,
// and it runs on the same kernel as in a single-GPU call); the results are
// scattered back into the source blocks for the return trip.
//
//   ep_send_pack_kernel     row p of the dispatch plan (sorted by expert)
//                           -> send slot q*cap + (p - first row for q),
//                           bf16 -> fp16 in interleaved K order.
//   ep_recv_plan_kernel     per-source receive counts -> one segment per
//                           local expert over the gathered rows, and the
//                           receive position of every gathered row.
//   ep_move_rows_kernel     gather (fp16 rows) / scatter back (fp32 rows).
//   ep_combine_kernel       out[token(p)] += w_p * y_back[slot(p)].
#include <cuda_bf16.h>

#include "common.cuh"
#include "internal.h"

using namespace wb;

namespace {

constexpr int kMaxWorld = 64;

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// One block per plan row.
__global__ void ep_send_pack_kernel(const uint16_t* __restrict__ x, int M,
                                    const int* __restrict__ row_token,
                                    const WispSegment* __restrict__ plan_segs, int e_loc,
                                    int n_rows, int world, int cap, uint16_t* __restrict__ xsend,
                                    int* __restrict__ slot) {
  __shared__ int dst_row;
  const int p = blockIdx.x;
  if (threadIdx.x == 0) {
    // destination rank: the last q whose first row is <= p
    int q = 0;
    for (int r = 1; r < world; r++)
      if (__ldg(&plan_segs[r * e_loc].row_begin) <= p) q = r;
    const int d = q * cap + (p - __ldg(&plan_segs[q * e_loc].row_begin));
    slot[p] = d;
    dst_row = d;
  }
  __syncthreads();
  const uint16_t* xr = x + (size_t)__ldg(row_token + p) * M;
  uint16_t* orow = xsend + (size_t)dst_row * M;
  for (int k8 = threadIdx.x * 8; k8 < M; k8 += blockDim.x * 8) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(xr + k8));
    const uint32_t a[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      f[2 * j] = bf16_bits_to_f32(a[j] & 0xffffu);
      f[2 * j + 1] = bf16_bits_to_f32(a[j] >> 16);
    }
    // logical slot j holds physical offset {0,4,1,5,2,6,3,7}[j]
    const __half2 h0 = __floats2half2_rn(f[0], f[4]);
    const __half2 h1 = __floats2half2_rn(f[1], f[5]);
    const __half2 h2 = __floats2half2_rn(f[2], f[6]);
    const __half2 h3 = __floats2half2_rn(f[3], f[7]);
    *reinterpret_cast<uint4*>(orow + k8) = make_uint4(h22u(h0), h22u(h1), h22u(h2), h22u(h3));
  }
}

// Single block. rc[s][e] = rows source s sends for local expert e (s <
// world, e < e_loc, world * e_loc <= 1024). Gathered order: expert-major,
// then source, then the source's own order.
__global__ void __launch_bounds__(1024) ep_recv_plan_kernel(const int* __restrict__ rc, int world,
                                                            int e_loc, int cap,
                                                            WispSegment* __restrict__ segs,
                                                            int* __restrict__ src_pos,
                                                            int* __restrict__ total_out) {
  __shared__ int src_off[1024];  // [s][e]: receive position of the chunk
  __shared__ int dst_off[1024];  // [s][e]: gathered position of the chunk
  __shared__ int cnt[1024];
  const int n = world * e_loc;
  for (int i = threadIdx.x; i < n; i += blockDim.x) cnt[i] = __ldg(rc + i);
  __syncthreads();
  if (threadIdx.x < world) {  // prefix over the experts of one source
    const int s = threadIdx.x;
    int off = s * cap;
    for (int e = 0; e < e_loc; e++) {
      src_off[s * e_loc + e] = off;
      off += cnt[s * e_loc + e];
    }
  }
  if (threadIdx.x == 32) {  // gathered order (another warp than the above)
    int off = 0;
    for (int e = 0; e < e_loc; e++) {
      WispSegment sg;
      sg.expert = e;
      sg.row_begin = off;
      sg.reserved = 0;
      for (int s = 0; s < world; s++) {
        dst_off[s * e_loc + e] = off;
        off += cnt[s * e_loc + e];
      }
      sg.rows = off - sg.row_begin;
      segs[e] = sg;
    }
    *total_out = off;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    for (int j = 0; j < cnt[i]; j++) src_pos[dst_off[i] + j] = src_off[i] + j;
}

// One block per gathered row j < *total: GATHER copies fp16 row src_pos[j]
// of `a` to row j of `b`; otherwise fp32 row j of `b` goes back to row
// src_pos[j] of `a`.
template <bool GATHER>
__global__ void ep_move_rows_kernel(void* __restrict__ a, void* __restrict__ b,
                                    const int* __restrict__ src_pos,
                                    const int* __restrict__ total, int row_bytes) {
  const int j = blockIdx.x;
  if (j >= __ldg(total)) return;
  const size_t r = (size_t)__ldg(src_pos + j);
  const uint4* src = reinterpret_cast<const uint4*>(
      GATHER ? static_cast<const uint8_t*>(a) + r * row_bytes
             : static_cast<const uint8_t*>(b) + (size_t)j * row_bytes);
  uint4* dst = reinterpret_cast<uint4*>(GATHER ? static_cast<uint8_t*>(b) + (size_t)j * row_bytes
                                               : static_cast<uint8_t*>(a) + r * row_bytes);
  for (int i = threadIdx.x; i < row_bytes / 16; i += blockDim.x) dst[i] = __ldg(src + i);
}

__global__ void ep_combine_kernel(const float* __restrict__ y, const int* __restrict__ slot,
                                  const int* __restrict__ row_token,
                                  const float* __restrict__ row_weight, int M,
                                  float* __restrict__ out) {
  const int p = blockIdx.x;
  const float w = __ldg(row_weight + p);
  const float* yr = y + (size_t)__ldg(slot + p) * M;
  float* orow = out + (size_t)__ldg(row_token + p) * M;
  for (int i = threadIdx.x * 4; i < M; i += blockDim.x * 4) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(yr + i));
    red_add_f32(orow + i, w * v.x);
    red_add_f32(orow + i + 1, w * v.y);
    red_add_f32(orow + i + 2, w * v.z);
    red_add_f32(orow + i + 3, w * v.w);
  }
}

}  // namespace

extern "C" WispError wisp_b200_ep_send_pack(const uint16_t* d_x, int hidden, const int* d_row_token,
                                            const WispSegment* d_plan_segs, int n_experts,
                                            int n_rows, int world, int cap, uint16_t* d_xsend,
                                            int* d_slot, cudaStream_t stream, WispErrCtx* err) {
  if (!d_x || !d_row_token || !d_plan_segs || !d_xsend || !d_slot)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_send_pack: null pointer argument");
  if (world < 1 || world > kMaxWorld || n_experts % world || hidden % 8 || n_rows < 0 ||
      n_rows > cap)
    return WB_FAIL(WISP_ERR_INVALID_ARG,
                   "ep_send_pack: world=%d experts=%d hidden=%d rows=%d cap=%d", world,
                   n_experts, hidden, n_rows, cap);
  if (((uintptr_t)d_x | (uintptr_t)d_xsend) & 15)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_send_pack: row buffers must be 16-byte aligned");
  if (n_rows == 0) return WISP_OK;
  wb::launch_k(ep_send_pack_kernel, n_rows, 128, 0, stream, d_x, hidden, d_row_token,
               d_plan_segs, n_experts / world, n_rows, world, cap, d_xsend, d_slot);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

extern "C" WispError wisp_b200_ep_recv_plan(const int* d_recv_counts, int world, int e_loc,
                                            int cap, WispSegment* d_segs, int* d_src_pos,
                                            int* d_total, cudaStream_t stream, WispErrCtx* err) {
  if (!d_recv_counts || !d_segs || !d_src_pos || !d_total)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_recv_plan: null pointer argument");
  if (world < 1 || world > kMaxWorld || e_loc < 1 || world * e_loc > 1024 || cap < 0)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_recv_plan: world=%d e_loc=%d cap=%d (world*e_loc <= 1024)",
                   world, e_loc, cap);
  wb::launch_k(ep_recv_plan_kernel, 1, 1024, 0, stream, d_recv_counts, world, e_loc, cap, d_segs,
               d_src_pos, d_total);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

extern "C" WispError wisp_b200_ep_gather_rows(const uint16_t* d_recv, const int* d_src_pos,
                                             const int* d_total, int max_rows, int hidden,
                                             uint16_t* d_sorted, cudaStream_t stream,
                                             WispErrCtx* err) {
  if (!d_recv || !d_src_pos || !d_total || !d_sorted)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_gather_rows: null pointer argument");
  if (hidden % 8 || max_rows < 0 || (((uintptr_t)d_recv | (uintptr_t)d_sorted) & 15))
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_gather_rows: hidden=%d (rows 16-byte aligned)", hidden);
  if (max_rows == 0) return WISP_OK;
  wb::launch_k(ep_move_rows_kernel<true>, max_rows, 128, 0, stream,
               const_cast<uint16_t*>(d_recv), d_sorted, d_src_pos, d_total, hidden * 2);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

extern "C" WispError wisp_b200_ep_scatter_rows(const float* d_sorted, const int* d_src_pos,
                                              const int* d_total, int max_rows, int hidden,
                                              float* d_recv, cudaStream_t stream,
                                              WispErrCtx* err) {
  if (!d_sorted || !d_src_pos || !d_total || !d_recv)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_scatter_rows: null pointer argument");
  if (hidden % 4 || max_rows < 0 || (((uintptr_t)d_recv | (uintptr_t)d_sorted) & 15))
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_scatter_rows: hidden=%d (rows 16-byte aligned)", hidden);
  if (max_rows == 0) return WISP_OK;
  wb::launch_k(ep_move_rows_kernel<false>, max_rows, 256, 0, stream, d_recv,
               const_cast<float*>(d_sorted), d_src_pos, d_total, hidden * 4);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

extern "C" WispError wisp_b200_ep_combine(const float* d_y, const int* d_slot,
                                         const int* d_row_token, const float* d_row_weight,
                                         int n_rows, int hidden, float* d_out, cudaStream_t stream,
                                         WispErrCtx* err) {
  if (!d_y || !d_slot || !d_row_token || !d_row_weight || !d_out)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_combine: null pointer argument");
  if (hidden % 4 || n_rows < 0 || ((uintptr_t)d_y & 15))
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_combine: hidden=%d rows=%d (y 16-byte aligned)",
                   hidden, n_rows);
  if (n_rows == 0) return WISP_OK;
  wb::launch_k(ep_combine_kernel, n_rows, 256, 0, stream, d_y, d_slot, d_row_token, d_row_weight,
               hidden, d_out);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}
