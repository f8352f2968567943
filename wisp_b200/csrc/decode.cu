// decode.cu -- fused int4 expert FFN for one token at the reference's
// precision (fp32 activations), replacing gpu_expert_ffn's per-expert chain
// of 3 dequant launches + swiglu_ffn + gemv + scale_accum
// (csrc/core/wisp_engine.c:1507-1531) with two launches for ALL experts:
//
//   gateup_kernel: h_j[i] = silu(gate_j[i] . x) * (up_j[i] . x)
//   down_kernel:   acc[m] += sum_j w_j * (down_j[m] . h_j)
//
// The int4 weights are read straight from the reference's expert blobs with
// coalesced 16-byte (or 8-byte, for blobs that sit 8 bytes off a 16-byte
// boundary) loads; nibbles become exact (n - 8) values through the fp16
// magic-number conversion and are accumulated in fp32 against fp32
// activations staged in shared memory (bank-conflict-free swizzle). The
// per-group scale (and zero, when present) is applied once per 32 weights.
// The down kernel gives each output row to one warp across all experts, so
// the weighted combine is deterministic and needs no atomics.
#include <algorithm>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "internal.h"

using namespace wb;

namespace {

constexpr int kMaxBlobs = 16;

struct MatPtrs {
  const uint8_t* packed;
  const __half* scales;
  const __half* zeros;  // nullptr: symmetric
};

struct DecodeParams {
  MatPtrs mat[kMaxBlobs][3];
  float weight[kMaxBlobs];
  int n;
  int hidden, inter, gs;
};

// Chunk c of VEC packed bytes covers 2*VEC activations. Activations live in
// shared memory in chunks of 2*VEC floats whose float4 pieces are permuted
// (piece p stored at p ^ swz(c)) so that a warp reading 32 consecutive
// chunks hits all 32 banks.
template <int VEC>
__device__ __forceinline__ int piece_swz(int c) {
  return VEC == 16 ? (c & 7) : ((c >> 1) & 3);
}

template <int VEC>
__device__ void stage_vector(const float* __restrict__ src, float* __restrict__ dst, int n) {
  constexpr int P = VEC / 2;  // float4 pieces per chunk
  for (int q = threadIdx.x; q < n / 4; q += blockDim.x) {
    const int c = q / P, p = q % P;
    const float4 v = reinterpret_cast<const float4*>(src)[q];
    reinterpret_cast<float4*>(dst)[c * P + (p ^ piece_swz<VEC>(c))] = v;
  }
}

template <int VEC>
__device__ __forceinline__ void load_chunk(const uint8_t* p, uint32_t (&w)[VEC / 4]) {
  if constexpr (VEC == 16) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    w[0] = v.x;
    w[1] = v.y;
    w[2] = v.z;
    w[3] = v.w;
  } else {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    w[0] = v.x;
    w[1] = v.y;
  }
}

// dot of one chunk of nibbles with the matching activations, plus the
// activation sum (for the zero point).
template <int VEC>
__device__ __forceinline__ float chunk_dot(const uint32_t (&w)[VEC / 4], const float (&xv)[2 * VEC]) {
  float acc = 0.f;
#pragma unroll
  for (int wd = 0; wd < VEC / 4; wd++) {
    __half2 c[4];
    nib8_centered(w[wd], c);
    // c[j] holds K offsets (j, j+4) of this word.
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float2 f = __half22float2(c[j]);
      acc = fmaf(f.x, xv[8 * wd + j], acc);
      acc = fmaf(f.y, xv[8 * wd + j + 4], acc);
    }
  }
  return acc;
}

template <int VEC>
__device__ __forceinline__ void read_chunk_x(const float* xs, int c, float (&xv)[2 * VEC]) {
  constexpr int P = VEC / 2;
  const int sw = piece_swz<VEC>(c);
#pragma unroll
  for (int p = 0; p < P; p++) {
    const float4 v = reinterpret_cast<const float4*>(xs)[c * P + (p ^ sw)];
    xv[4 * p + 0] = v.x;
    xv[4 * p + 1] = v.y;
    xv[4 * p + 2] = v.z;
    xv[4 * p + 3] = v.w;
  }
}

// R weight rows (all of length `cols`) against the staged vector xs.
template <int VEC, int R>
__device__ void rows_dot(const MatPtrs* const (&mats)[R], const int (&rows)[R], int cols, int gs,
                         const float* xs, float (&out)[R]) {
  const int lane = threadIdx.x & 31;
  const int nchunks = cols / (2 * VEC);
  const int gpr = cols / gs;  // groups per row
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; r++) acc[r] = 0.f;
  for (int c = lane; c < nchunks; c += 32) {
    uint32_t w[R][VEC / 4];
#pragma unroll
    for (int r = 0; r < R; r++)
      load_chunk<VEC>(mats[r]->packed + (size_t)rows[r] * (cols / 2) + (size_t)c * VEC, w[r]);
    float xv[2 * VEC];
    read_chunk_x<VEC>(xs, c, xv);
    float xsum = 0.f;
#pragma unroll
    for (int j = 0; j < 2 * VEC; j++) xsum += xv[j];
    const int g_in_row = (c * 2 * VEC) / gs;
#pragma unroll
    for (int r = 0; r < R; r++) {
      const size_t g = (size_t)rows[r] * gpr + g_in_row;
      const float s = __half2float(mats[r]->scales[g]);
      const float d = chunk_dot<VEC>(w[r], xv);
      acc[r] = fmaf(s, d, acc[r]);
      if (mats[r]->zeros) acc[r] = fmaf(__half2float(mats[r]->zeros[g]), xsum, acc[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < R; r++) {
    float v = acc[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    out[r] = v;
  }
}

// grid (ceil(I/16), n): each warp computes two intermediate rows of one
// expert: gate and up for rows i and i+1 share every activation load.
template <int VEC>
__global__ void __launch_bounds__(256) gateup_kernel(const __grid_constant__ DecodeParams p,
                                                     const float* __restrict__ x,
                                                     float* __restrict__ h) {
  extern __shared__ float4 smem_f4[];
  float* xs = reinterpret_cast<float*>(smem_f4);
  stage_vector<VEC>(x, xs, p.hidden);
  __syncthreads();
  const int j = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int i0 = blockIdx.x * 16 + warp * 2;
  if (i0 >= p.inter) return;
  const int i1 = min(i0 + 1, p.inter - 1);
  const MatPtrs* const mats[4] = {&p.mat[j][0], &p.mat[j][1], &p.mat[j][0], &p.mat[j][1]};
  const int rows[4] = {i0, i0, i1, i1};
  float d[4];
  rows_dot<VEC, 4>(mats, rows, p.hidden, p.gs, xs, d);
  if ((threadIdx.x & 31) == 0) {
    h[(size_t)j * p.inter + i0] = silu(d[0]) * d[1];
    if (i1 != i0) h[(size_t)j * p.inter + i1] = silu(d[2]) * d[3];
  }
}

// grid ceil(M/16): each warp owns output rows m, m+1 across all experts.
template <int VEC>
__global__ void __launch_bounds__(256) down_kernel(const __grid_constant__ DecodeParams p,
                                                   const float* __restrict__ h,
                                                   float* __restrict__ acc) {
  extern __shared__ float4 smem_f4[];
  float* hs = reinterpret_cast<float*>(smem_f4);
  for (int j = 0; j < p.n; j++) stage_vector<VEC>(h + (size_t)j * p.inter, hs + (size_t)j * p.inter, p.inter);
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  const int m0 = blockIdx.x * 16 + warp * 2;
  if (m0 >= p.hidden) return;
  const int m1 = min(m0 + 1, p.hidden - 1);
  float y0 = 0.f, y1 = 0.f;
  for (int j = 0; j < p.n; j++) {
    const MatPtrs* const mats[2] = {&p.mat[j][2], &p.mat[j][2]};
    const int rows[2] = {m0, m1};
    float d[2];
    rows_dot<VEC, 2>(mats, rows, p.inter, p.gs, hs + (size_t)j * p.inter, d);
    y0 = fmaf(p.weight[j], d[0], y0);
    y1 = fmaf(p.weight[j], d[1], y1);
  }
  if ((threadIdx.x & 31) == 0) {
    acc[m0] += y0;
    if (m1 != m0) acc[m1] += y1;
  }
}


}  // namespace

extern "C" size_t wisp_b200_expert_ffn_scratch_bytes(const WispExpertMeta* meta, int n_blobs) {
  if (!meta || n_blobs <= 0) return 0;
  return (size_t)n_blobs * meta->rows[0] * sizeof(float);
}

extern "C" WispError wisp_b200_expert_ffn(const WispExpertMeta* meta, const void* const* d_blobs,
                                          const float* weights, int n_blobs, const float* d_x,
                                          float* d_acc, void* d_scratch, size_t scratch_bytes,
                                          cudaStream_t stream, WispErrCtx* err) {
  if (!meta || !meta->valid) return WB_FAIL(WISP_ERR_INVALID_ARG, "expert_ffn: invalid meta");
  if (!d_blobs || !weights || !d_x || !d_acc || !d_scratch)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "expert_ffn: null pointer argument");
  if (n_blobs < 1 || n_blobs > kMaxBlobs)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "expert_ffn: n_blobs=%d (1..%d)", n_blobs, kMaxBlobs);
  const int inter = (int)meta->rows[0], hidden = (int)meta->cols[0], gs = (int)meta->group_size;
  if (meta->rows[1] != (uint32_t)inter || meta->cols[1] != (uint32_t)hidden ||
      meta->rows[2] != (uint32_t)hidden || meta->cols[2] != (uint32_t)inter)
    return WB_FAIL(WISP_ERR_MODEL, "expert_ffn: inconsistent shapes gate %ux%u up %ux%u down %ux%u",
                   meta->rows[0], meta->cols[0], meta->rows[1], meta->cols[1], meta->rows[2],
                   meta->cols[2]);
  if (inter <= 0 || hidden <= 0 || gs <= 0 || hidden % gs || inter % gs || gs % 16)
    return WB_FAIL(WISP_ERR_INVALID_ARG,
                   "expert_ffn: need hidden, inter multiples of group_size and group_size %% 16 == 0 "
                   "(hidden=%d inter=%d gs=%d)", hidden, inter, gs);
  if (scratch_bytes < wisp_b200_expert_ffn_scratch_bytes(meta, n_blobs))
    return WB_FAIL(WISP_ERR_INVALID_ARG, "expert_ffn: scratch too small (%zu < %zu)",
                   scratch_bytes, wisp_b200_expert_ffn_scratch_bytes(meta, n_blobs));
  if (((uintptr_t)d_x | (uintptr_t)d_scratch) & 15)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "expert_ffn: x and scratch must be 16-byte aligned");

  DecodeParams p;
  memset(&p, 0, sizeof p);
  p.n = n_blobs;
  p.hidden = hidden;
  p.inter = inter;
  p.gs = gs;
  bool al16 = (gs % 32 == 0);
  for (int j = 0; j < n_blobs; j++) {
    const uint8_t* base = (const uint8_t*)d_blobs[j];
    if (!base) return WB_FAIL(WISP_ERR_INVALID_ARG, "expert_ffn: blob %d is NULL", j);
    for (int m = 0; m < 3; m++) {
      p.mat[j][m].packed = base + meta->packed_off[m];
      p.mat[j][m].scales = (const __half*)(base + meta->scales_off[m]);
      // The blob carries zero points when bytes remain between zeros_off and
      // the start of the next matrix (or the end of the blob).
      const size_t end = m < 2 ? meta->packed_off[m + 1] : meta->total_bytes;
      p.mat[j][m].zeros =
          end > meta->zeros_off[m] ? (const __half*)(base + meta->zeros_off[m]) : nullptr;
      const uintptr_t a = (uintptr_t)p.mat[j][m].packed;
      if (a & 7)
        return WB_FAIL(WISP_ERR_INVALID_ARG,
                       "expert_ffn: blob %d matrix %d packed data not 8-byte aligned", j, m);
      if (a & 15) al16 = false;
      if (meta->scales_off[m] & 1)
        return WB_FAIL(WISP_ERR_INVALID_ARG, "expert_ffn: blob %d scales misaligned", j);
    }
    p.weight[j] = weights[j];
  }
  float* h = (float*)d_scratch;
  const size_t smem_gu = (size_t)hidden * sizeof(float);
  const size_t smem_dn = (size_t)n_blobs * inter * sizeof(float);
  if (smem_gu > 227 * 1024 || smem_dn > 227 * 1024)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "expert_ffn: activations exceed shared memory "
                   "(hidden=%d, n*inter=%d)", hidden, n_blobs * inter);
  dim3 g1((inter + 15) / 16, n_blobs), g2((hidden + 15) / 16);
  if (al16) {
    cudaFuncSetAttribute(gateup_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_gu);
    cudaFuncSetAttribute(down_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_dn);
    gateup_kernel<16><<<g1, 256, smem_gu, stream>>>(p, d_x, h);
    down_kernel<16><<<g2, 256, smem_dn, stream>>>(p, h, d_acc);
  } else {
    cudaFuncSetAttribute(gateup_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_gu);
    cudaFuncSetAttribute(down_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_dn);
    gateup_kernel<8><<<g1, 256, smem_gu, stream>>>(p, d_x, h);
    down_kernel<8><<<g2, 256, smem_dn, stream>>>(p, h, d_acc);
  }
  const cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) return WB_FAIL(WISP_ERR_CUDA, "expert_ffn launch: %s", cudaGetErrorString(ce));
  return WISP_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot call cudaMalloc: an engine whose VRAM budget is fully
// committed to the expert tier cache (a new allocation there fails, or forces
// evicting cached experts), or a host callback in a decode loop where a
// cudaMalloc / cudaFree would implicitly synchronise the device. For them the
// intermediate activations live in a fixed per-device array compiled into
// this library: 58112 floats (227 KB, the most the down kernel can stage in
// shared memory, so every size that fits the array also fits the kernel),
// held by every GPU that loads the library until the process exits.
// n_blobs * inter must fit in it.
//
// The array's host-side name is only a stand-in, so its device address is
// looked up once per device (cudaGetSymbolAddress, with that device current)
// on the first call made on that device; make that first call before any
// stream capture. The cached address belongs to the device's primary
// context (the runtime's): callers that switch to another driver context on
// the device, or call cudaDeviceReset, must not use this entry afterwards.
// Every call shares the array: the gate/up kernel writes all of the slots
// the down kernel reads, so nothing needs clearing, but calls whose kernels
// overlap on the GPU (different streams, no ordering between them) race on
// it.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocScratchFloats = 227 * 1024 / sizeof(float);
__device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {nullptr};
}  // namespace

extern "C" WispError wisp_b200_expert_ffn_noalloc(const WispExpertMeta* meta,
                                                  const void* const* d_blobs,
                                                  const float* weights, int n_blobs,
                                                  const float* d_x, float* d_acc,
                                                  cudaStream_t stream, WispErrCtx* err) {
  if (!meta || !meta->valid) return WB_FAIL(WISP_ERR_INVALID_ARG, "expert_ffn_noalloc: invalid meta");
  if (n_blobs < 1 || n_blobs > kMaxBlobs)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "expert_ffn_noalloc: n_blobs=%d (1..%d)", n_blobs, kMaxBlobs);
  const size_t need = (size_t)n_blobs * meta->rows[0];
  if (need > kNoAllocScratchFloats)
    return WB_FAIL(WISP_ERR_INVALID_ARG,
                   "expert_ffn_noalloc: n_blobs * inter = %zu exceeds the built-in scratch of %zu "
                   "floats; use wisp_b200_expert_ffn with a caller buffer",
                   need, kNoAllocScratchFloats);
  int dev = -1;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce != cudaSuccess || dev < 0 || dev >= 64)
    return WB_FAIL(WISP_ERR_CUDA, "expert_ffn_noalloc: cudaGetDevice: %s", cudaGetErrorString(ce));
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
      void* ptr = nullptr;
      ce = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (ce != cudaSuccess || !ptr)
        return WB_FAIL(WISP_ERR_CUDA, "expert_ffn_noalloc: cudaGetSymbolAddress: %s",
                       cudaGetErrorString(ce));
      g_noalloc_addr[dev] = ptr;
    }
    scratch = g_noalloc_addr[dev];
  }
  return wisp_b200_expert_ffn(meta, d_blobs, weights, n_blobs, d_x, d_acc, scratch,
                              kNoAllocScratchFloats * sizeof(float), stream, err);
}
