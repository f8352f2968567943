// ep.cu -- device-side plumbing of the expert-parallel exchange.
//
// The reference engine runs on one GPU and has no expert parallelism; these
// kernels serve the multi-GPU path (wisp_b200/ep.py), where routed experts
// are sharded in contiguous blocks of E/N over N ranks and token rows travel
// to their experts' owners and back through fixed-size NCCL all-to-all
// exchanges. Fixed sizes keep every count on the device: no host round trip
// sits between routing and the expert FFN.
//
// A token goes to an owner rank once, whatever the number of its experts
// there: rank r's send buffer holds one block per destination q, with
//   n_rows                 rows in the block (the tokens with >= 1 expert on q,
//                          in token order)
//   cnt[e_loc]             routed (token, expert) entries per local expert of q
//   ent_row[cap*k]         the entries, expert-major (then token order): block
//   ent_w[cap*k]           row and routing weight
//   rows[cap][hidden]      the token rows, fp16 in interleaved K order
// with cap = the most tokens any rank holds (a token fills at most one row
// per block). One all-to-all moves the blocks; the owner gathers the rows
// expert-contiguous (each local expert is ONE segment, as on one GPU), runs
// the grouped FFN with the routing weights, which adds every expert's
// weighted output into an fp32 row per received token, and one all-to-all
// returns those rows; the home rank adds its rows from each owner.
//
//   ep_dispatch_kernel   one block: per destination (one warp each) the
//                        token -> row slots (a ballot scan over tokens), the
//                        block headers and the entries from the dispatch
//                        plan.
//   ep_pack_kernel       token rows (bf16 -> fp16 interleaved) into every
//                        block that holds them (and into the rank's own rows
//                        for the shared expert).
//   ep_recv_plan_kernel  one block: from the received headers and entries,
//                        one segment per local expert over the gathered
//                        rows, the receive row and weight of each.
//   ep_gather_kernel     gathered fp16 rows from the receive blocks (and the
//                        rank's own rows for the shared expert).
//   ep_to_half_kernel    the owner's fp32 return rows rounded to fp16 (the
//                        return exchange carries half the bytes).
//   ep_combine_kernel    out[t] += the returned rows of token t, in rank order.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"

using namespace wb;

namespace {

constexpr int kMaxWorld = 64;

struct Layout {
  size_t off_ent, off_w, off_rows, bytes;
  int cap;
};

__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~(size_t)15; }

// Byte layout of one exchange block (elem = bytes per row element).
__host__ __device__ inline Layout ep_layout(int hidden, int e_loc, int cap, int top_k, int elem) {
  Layout L;
  L.cap = cap;
  L.off_ent = align16(16 + 4 * (size_t)e_loc);
  L.off_w = L.off_ent + 4 * (size_t)cap * top_k;
  L.off_rows = align16(L.off_w + 4 * (size_t)cap * top_k);
  L.bytes = align16(L.off_rows + (size_t)cap * hidden * elem);
  return L;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// Exclusive scan of one flag per thread over the block; returns the prefix
// and leaves the block total in *total (all threads must call).
__device__ int block_scan(int f, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int v = f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += y;
  }
  if (lane == 31) warp_tot[w] = v;
  __syncthreads();
  if (w == 0) {
    int tv = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, tv, o);
      if (lane >= o) tv += y;
    }
    warp_tot[lane] = tv;
  }
  __syncthreads();
  const int incl = v + (w > 0 ? warp_tot[w - 1] : 0);
  *total = warp_tot[(blockDim.x >> 5) - 1];
  __syncthreads();
  return incl - f;
}

// Single block. idx [T x k] (global experts); the plan (plan_segs over the E
// global experts, row_token / row_weight sorted by expert then token) comes
// from the dispatch plan of the same routing. slot[t * world + q] = row of
// token t in block q, or -1. The routing, the plan's segments and the slots
// are staged in shared memory (when they fit), so every phase is one round
// of parallel loads: slots by one warp per destination, then the entries by
// one thread per plan row.
constexpr int kDispStage = 4096;   // idx / slot entries staged in shared memory

__global__ void __launch_bounds__(1024) ep_dispatch_kernel(
    const int* __restrict__ idx, const WispSegment* __restrict__ plan_segs,
    const int* __restrict__ row_token, const float* __restrict__ row_weight, int T, int k, int E,
    int world, Layout L, uint8_t* __restrict__ send, int* __restrict__ slot) {
  __shared__ int s_idx[kDispStage];
  __shared__ int s_slot[kDispStage];
  __shared__ int s_begin[1024];
  __shared__ int s_rows[1024];
  const int e_loc = E / world;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool idx_sm = T * k <= kDispStage, slot_sm = T * world <= kDispStage;
  if (idx_sm)
    for (int i = threadIdx.x; i < T * k; i += blockDim.x) s_idx[i] = __ldg(idx + i);
  for (int g = threadIdx.x; g < E; g += blockDim.x) {
    s_begin[g] = __ldg(&plan_segs[g].row_begin);
    s_rows[g] = __ldg(&plan_segs[g].rows);
  }
  __syncthreads();
  const int* ix = idx_sm ? s_idx : idx;
  // one warp per destination q: a token's slot in q's block is the number
  // of earlier tokens with an expert on q (ballot prefix over 32-token runs)
  for (int q = warp; q < world; q += blockDim.x >> 5) {
    int carry = 0;
    for (int base = 0; base < T; base += 32) {
      const int t = base + lane;
      bool f = false;
      if (t < T)
        for (int j = 0; j < k; j++) {
          const int e = ix[(size_t)t * k + j];
          if (e >= 0 && e < E && e / e_loc == q) f = true;
        }
      const unsigned m = __ballot_sync(0xffffffffu, f);
      if (t < T) {
        const int v = f ? carry + __popc(m & ((1u << lane) - 1u)) : -1;
        slot[(size_t)t * world + q] = v;
        if (slot_sm) s_slot[t * world + q] = v;
      }
      carry += __popc(m);
    }
    if (lane == 0) reinterpret_cast<int*>(send + q * L.bytes)[0] = carry;
  }
  for (int g = threadIdx.x; g < E; g += blockDim.x) {
    const int q = g / e_loc;
    reinterpret_cast<int*>(send + q * L.bytes + 16)[g - q * e_loc] = s_rows[g];
  }
  __syncthreads();  // the slots above are read back below
  // entries: plan row p (expert g = the last segment starting at or before
  // p) goes to block q = g / e_loc at position p - (q's first plan row)
  const int nrows = s_begin[E - 1] + s_rows[E - 1];
  for (int p = threadIdx.x; p < nrows; p += blockDim.x) {
    int lo = 0, hi = E - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_begin[mid] <= p) lo = mid; else hi = mid - 1;
    }
    const int q = lo / e_loc;
    const int first = s_begin[q * e_loc];
    int* ent = reinterpret_cast<int*>(send + q * L.bytes + L.off_ent);
    float* ew = reinterpret_cast<float*>(send + q * L.bytes + L.off_w);
    const int t = __ldg(row_token + p);
    ent[p - first] = slot_sm ? s_slot[t * world + q] : slot[(size_t)t * world + q];
    ew[p - first] = __ldg(row_weight + p);
  }
}

// One block per token: its bf16 row, converted once, into each block that
// holds it.
// With own_rows, the converted row also goes there (this rank's own rows for
// the shared expert's segment).
__global__ void ep_pack_kernel(const uint16_t* __restrict__ x, int M, const int* __restrict__ slot,
                               int world, Layout L, uint8_t* __restrict__ send,
                               uint16_t* __restrict__ own_rows) {
  __shared__ int sl[kMaxWorld];
  const int t = blockIdx.x;
  if (threadIdx.x < world) sl[threadIdx.x] = slot[(size_t)t * world + threadIdx.x];
  __syncthreads();
  const uint16_t* xr = x + (size_t)t * M;
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
    const uint4 o = make_uint4(h22u(__floats2half2_rn(f[0], f[4])), h22u(__floats2half2_rn(f[1], f[5])),
                               h22u(__floats2half2_rn(f[2], f[6])), h22u(__floats2half2_rn(f[3], f[7])));
    for (int q = 0; q < world; q++) {
      const int s = sl[q];
      if (s >= 0)
        *reinterpret_cast<uint4*>(send + q * L.bytes + L.off_rows + ((size_t)s * M + k8) * 2) = o;
    }
    if (own_rows) *reinterpret_cast<uint4*>(own_rows + (size_t)t * M + k8) = o;
  }
}

// Single block of 1024 threads (world * e_loc <= 1024 chunks, chunk (s, e) =
// the entries of local expert e in source block s). Gathered order: local
// expert, then source rank, then the source's entry order; with own > 0 the
// rank's own own token rows follow as segment e_loc (the shared expert). src_pos[j] =
// receive row (s * cap + block row) of gathered row j, weight[j] its routing
// weight; a source's entries are clamped to its block's capacity (cap * k)
// in expert order. Two block scans give every chunk its source offset and
// its gathered offset; warps then copy the chunks' entries.
__global__ void __launch_bounds__(1024) ep_recv_plan_kernel(const uint8_t* __restrict__ recv,
                                                            int world, int e_loc, int k, Layout L,
                                                            int own,
                                                            WispSegment* __restrict__ segs,
                                                            int* __restrict__ src_pos,
                                                            float* __restrict__ weight,
                                                            int* __restrict__ total_out) {
  __shared__ int src_off[1024];  // [s][e]: first entry of the chunk in block s
  __shared__ int dst_off[1024];  // [s][e]: gathered position of the chunk
  __shared__ int cnt[1024];      // [s][e]: entries of the chunk (clamped)
  __shared__ int warp_tot[32];
  const int n = world * e_loc;
  const int max_ent = L.cap * k;
  const int i = threadIdx.x;
  // 1. counts, clamped per source: chunk (s, e) starts at min(sum of the
  //    source's earlier counts, cap * k) and ends at min(that + its count,
  //    cap * k) -- a scan over the source-major order minus the source's base
  int c = 0;
  if (i < n) {
    const int s = i / e_loc, e = i - s * e_loc;
    c = min(max(reinterpret_cast<const int*>(recv + s * L.bytes + 16)[e], 0), max_ent);
  }
  int tot;
  const int ex = block_scan(c, warp_tot, &tot);   // exclusive, source-major
  if (i < n) cnt[i] = ex;                          // staged: the prefix
  __syncthreads();
  if (i < n) {
    const int s = i / e_loc;
    const int base = cnt[s * e_loc];               // the source's first prefix
    const int b = min(ex - base, max_ent), e2 = min(ex - base + c, max_ent);
    src_off[i] = b;
    dst_off[i] = e2 - b;                           // staged: the clamped count
  }
  __syncthreads();
  if (i < n) cnt[i] = dst_off[i];
  __syncthreads();
  // 2. gathered offsets: a scan over the expert-major order (e, s)
  int ct = 0, s_t = 0, e_t = 0;
  if (i < n) {
    e_t = i / world;
    s_t = i - e_t * world;
    ct = cnt[s_t * e_loc + e_t];
  }
  const int ex2 = block_scan(ct, warp_tot, &tot);
  if (i < n) dst_off[s_t * e_loc + e_t] = ex2;
  if (i == 0) *total_out = tot;
  // this rank's own token rows for the shared expert (local entry e_loc):
  // one more segment after the received rows, source row world * cap + t
  if (own > 0) {
    if (i == 0) {
      WispSegment sg;
      sg.expert = e_loc;
      sg.row_begin = tot;
      sg.rows = own;
      sg.reserved = 0;
      segs[e_loc] = sg;
    }
    for (int t = i; t < own; t += blockDim.x) {
      src_pos[tot + t] = world * L.cap + t;
      weight[tot + t] = 1.f;
    }
  }
  __syncthreads();
  if (i < e_loc) {
    int rows = 0;
    for (int s = 0; s < world; s++) rows += cnt[s * e_loc + i];
    WispSegment sg;
    sg.expert = i;
    sg.row_begin = dst_off[i];   // source 0 of expert i
    sg.rows = rows;
    sg.reserved = 0;
    segs[i] = sg;
  }
  // 3. the entries, one warp per chunk
  const int warp = i >> 5, lane = i & 31;
  for (int q = warp; q < n; q += blockDim.x >> 5) {
    const int s = q / e_loc;
    const int* ent = reinterpret_cast<const int*>(recv + s * L.bytes + L.off_ent);
    const float* ew = reinterpret_cast<const float*>(recv + s * L.bytes + L.off_w);
    const int so = src_off[q], d = dst_off[q], m = cnt[q];
    for (int j = lane; j < m; j += 32) {
      const int row = ent[so + j];
      src_pos[d + j] = s * L.cap + min(max(row, 0), L.cap - 1);
      weight[d + j] = ew[so + j];
    }
  }
}

// One block per gathered row j < *total + own: sorted[j] = receive row
// src_pos[j], or, for src_pos[j] >= world * cap, own row src_pos[j] - world *
// cap (fp16 rows of this rank's tokens, already in the interleaved order).
__global__ void ep_gather_kernel(const uint8_t* __restrict__ recv, Layout L, int M, int world,
                                 const int* __restrict__ src_pos, const int* __restrict__ total,
                                 const uint16_t* __restrict__ own_rows, int own,
                                 uint16_t* __restrict__ sorted) {
  const int j = blockIdx.x;
  if (j >= __ldg(total) + own) return;
  const int r = __ldg(src_pos + j);
  const uint4* src;
  if (r >= world * L.cap) {
    src = reinterpret_cast<const uint4*>(own_rows + (size_t)(r - world * L.cap) * M);
  } else {
    const int s = r / L.cap, row = r - s * L.cap;
    src = reinterpret_cast<const uint4*>(recv + s * L.bytes + L.off_rows + (size_t)row * M * 2);
  }
  uint4* dst = reinterpret_cast<uint4*>(sorted + (size_t)j * M);
  for (int i = threadIdx.x; i < M / 8; i += blockDim.x) dst[i] = __ldg(src + i);
}

// Four consecutive values of a returned row as floats (fp32 or fp16 rows).
__device__ __forceinline__ float4 load4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 load4(const __half* p) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// Block (t, c): out[t] += yback[q * cap + slot[t][q]] for q = 0..world-1 over
// the c-th run of 1024 values of the row.
// With `local` (fp32 [T x M]), out[t] = local[t] + the returned rows instead.
template <typename T>
__global__ void ep_combine_kernel(const T* __restrict__ y, const int* __restrict__ slot,
                                  const float* __restrict__ local, int world, int cap, int M,
                                  float* __restrict__ out) {
  __shared__ int sl[kMaxWorld];
  const int t = blockIdx.x;
  if (threadIdx.x < world) sl[threadIdx.x] = slot[(size_t)t * world + threadIdx.x];
  __syncthreads();
  float* orow = out + (size_t)t * M;
  const int end = min(M, ((int)blockIdx.y + 1) * (int)blockDim.x * 4);
  for (int i = blockIdx.y * blockDim.x * 4 + threadIdx.x * 4; i < end; i += blockDim.x * 4) {
    float4 acc = local ? __ldg(reinterpret_cast<const float4*>(local + (size_t)t * M + i))
                       : *reinterpret_cast<const float4*>(orow + i);
    for (int q = 0; q < world; q++) {
      if (sl[q] < 0) continue;
      const float4 v = load4(y + ((size_t)q * cap + sl[q]) * M + i);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    *reinterpret_cast<float4*>(orow + i) = acc;
  }
}

// The owner's fp32 return rows rounded to fp16 for the return exchange
// (half its bytes); four values per thread.
__global__ void ep_to_half_kernel(const float* __restrict__ y, size_t n4, __half* __restrict__ o) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
       i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(y) + i);
    const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    reinterpret_cast<uint2*>(o)[i] = u;
  }
}

bool bad_shape(int world, int e_loc, int cap, int top_k, int hidden) {
  return world < 1 || world > kMaxWorld || e_loc < 1 || world * e_loc > 1024 || cap < 1 ||
         top_k < 1 || top_k > 32 || hidden < 8 || hidden % 8;
}

}  // namespace

extern "C" size_t wisp_b200_ep_block_bytes(int hidden, int e_loc, int cap, int top_k) {
  if (bad_shape(1, e_loc, cap, top_k, hidden)) return 0;
  return ep_layout(hidden, e_loc, cap, top_k, 2).bytes;
}

extern "C" WispError wisp_b200_ep_dispatch(const uint16_t* d_x, int tokens, int hidden,
                                           const int* d_topk_idx, int top_k,
                                           const WispSegment* d_plan_segs, const int* d_row_token,
                                           const float* d_row_weight, int n_experts, int world,
                                           int cap, uint8_t* d_send, int* d_slot,
                                           uint16_t* d_own, cudaStream_t stream,
                                           WispErrCtx* err) {
  if (!d_x || !d_topk_idx || !d_plan_segs || !d_row_token || !d_row_weight || !d_send || !d_slot)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_dispatch: null pointer argument");
  if (world < 1 || n_experts % world || bad_shape(world, n_experts / world, cap, top_k, hidden) ||
      tokens < 0 || tokens > cap)
    return WB_FAIL(WISP_ERR_INVALID_ARG,
                   "ep_dispatch: world=%d experts=%d hidden=%d tokens=%d cap=%d top_k=%d", world,
                   n_experts, hidden, tokens, cap, top_k);
  if (((uintptr_t)d_x | (uintptr_t)d_send | (uintptr_t)d_own) & 15)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_dispatch: x and the send buffer must be 16-byte aligned");
  const Layout L = ep_layout(hidden, n_experts / world, cap, top_k, 2);
  wb::launch_k(ep_dispatch_kernel, 1, 1024, 0, stream, d_topk_idx, d_plan_segs, d_row_token,
               d_row_weight, tokens, top_k, n_experts, world, L, d_send, d_slot);
  if (tokens > 0)
    wb::launch_k(ep_pack_kernel, tokens, 128, 0, stream, d_x, hidden, d_slot, world, L, d_send,
                 d_own);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

extern "C" WispError wisp_b200_ep_recv_plan(const uint8_t* d_recv, int world, int e_loc, int cap,
                                            int top_k, int hidden, int own_rows,
                                            WispSegment* d_segs, int* d_src_pos, float* d_weight,
                                            int* d_total, cudaStream_t stream, WispErrCtx* err) {
  if (!d_recv || !d_segs || !d_src_pos || !d_weight || !d_total)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_recv_plan: null pointer argument");
  if (bad_shape(world, e_loc, cap, top_k, hidden) || own_rows < 0 || own_rows > cap)
    return WB_FAIL(WISP_ERR_INVALID_ARG,
                   "ep_recv_plan: world=%d e_loc=%d cap=%d top_k=%d hidden=%d own_rows=%d "
                   "(world*e_loc <= 1024, own_rows <= cap)",
                   world, e_loc, cap, top_k, hidden, own_rows);
  const Layout L = ep_layout(hidden, e_loc, cap, top_k, 2);
  wb::launch_k(ep_recv_plan_kernel, 1, 1024, 0, stream, d_recv, world, e_loc, top_k, L, own_rows,
               d_segs, d_src_pos, d_weight, d_total);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

extern "C" WispError wisp_b200_ep_gather_rows(const uint8_t* d_recv, int world, int e_loc, int cap,
                                             int top_k, int hidden, const int* d_src_pos,
                                             const int* d_total, const uint16_t* d_own,
                                             int own_rows, int max_rows, uint16_t* d_sorted,
                                             cudaStream_t stream, WispErrCtx* err) {
  if (!d_recv || !d_src_pos || !d_total || !d_sorted || (own_rows > 0 && !d_own))
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_gather_rows: null pointer argument");
  if (bad_shape(world, e_loc, cap, top_k, hidden) || max_rows < 0 || own_rows < 0 ||
      own_rows > cap || (((uintptr_t)d_recv | (uintptr_t)d_sorted | (uintptr_t)d_own) & 15))
    return WB_FAIL(WISP_ERR_INVALID_ARG,
                   "ep_gather_rows: hidden=%d max_rows=%d own_rows=%d (16-byte aligned rows)",
                   hidden, max_rows, own_rows);
  if (max_rows == 0) return WISP_OK;
  const Layout L = ep_layout(hidden, e_loc, cap, top_k, 2);
  wb::launch_k(ep_gather_kernel, max_rows, 128, 0, stream, d_recv, L, hidden, world, d_src_pos,
               d_total, d_own, own_rows, d_sorted);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

extern "C" WispError wisp_b200_ep_combine(const float* d_yback, const int* d_slot, int tokens,
                                         int world, int cap, int hidden, float* d_out,
                                         cudaStream_t stream, WispErrCtx* err) {
  if (!d_yback || !d_slot || !d_out)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_combine: null pointer argument");
  if (world < 1 || world > kMaxWorld || cap < 1 || tokens < 0 || tokens > cap || hidden % 4 ||
      (((uintptr_t)d_yback | (uintptr_t)d_out) & 15))
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_combine: world=%d tokens=%d cap=%d hidden=%d", world,
                   tokens, cap, hidden);
  if (tokens == 0) return WISP_OK;
  wb::launch_k(ep_combine_kernel<float>, dim3(tokens, (hidden + 1023) / 1024), 256, 0, stream,
               d_yback, d_slot, static_cast<const float*>(nullptr), world, cap, hidden, d_out);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

extern "C" WispError wisp_b200_ep_combine_f16(const uint16_t* d_yback, const int* d_slot,
                                             const float* d_local, int tokens, int world, int cap,
                                             int hidden, float* d_out, cudaStream_t stream,
                                             WispErrCtx* err) {
  if (!d_yback || !d_slot || !d_out)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_combine_f16: null pointer argument");
  if (world < 1 || world > kMaxWorld || cap < 1 || tokens < 0 || tokens > cap || hidden % 4 ||
      ((uintptr_t)d_yback & 7) || (((uintptr_t)d_out | (uintptr_t)d_local) & 15))
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_combine_f16: world=%d tokens=%d cap=%d hidden=%d",
                   world, tokens, cap, hidden);
  if (tokens == 0) return WISP_OK;
  wb::launch_k(ep_combine_kernel<__half>, dim3(tokens, (hidden + 1023) / 1024), 256, 0, stream,
               reinterpret_cast<const __half*>(d_yback), d_slot, d_local, world, cap, hidden, d_out);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

extern "C" WispError wisp_b200_ep_return_rows(const float* d_y, int rows, int hidden,
                                             uint16_t* d_y16, cudaStream_t stream,
                                             WispErrCtx* err) {
  if (!d_y || !d_y16) return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_return_rows: null pointer argument");
  if (rows < 0 || hidden < 4 || hidden % 4 || ((uintptr_t)d_y & 15) || ((uintptr_t)d_y16 & 7))
    return WB_FAIL(WISP_ERR_INVALID_ARG, "ep_return_rows: rows=%d hidden=%d", rows, hidden);
  const size_t n4 = (size_t)rows * hidden / 4;
  if (n4 == 0) return WISP_OK;
  const int blocks = (int)std::min<size_t>((n4 + 255) / 256, (size_t)4 * 148);
  wb::launch_k(ep_to_half_kernel, blocks, 256, 0, stream, d_y, n4,
               reinterpret_cast<__half*>(d_y16));
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}
