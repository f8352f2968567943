// dropin.cu -- the reference engine's GPU launcher ABI, re-implemented for
// sm_100a. Same symbol names, signatures, argument meaning and error
// behaviour as the reference (csrc/core/wisp_engine.h:496-583), so a build of
// the reference engine can link this library in place of its csrc/cuda/*.cu.
//
//   launch_dequant_expert  csrc/cuda/expert_loader.cu:46-63
//   async_load_expert      csrc/cuda/expert_loader.cu:67-97
//   wisp_gpu_gemv_f16      csrc/cuda/matmul.cu:43-65
//   wisp_gpu_swiglu        csrc/cuda/matmul.cu:133-148
//   wisp_gpu_swiglu_ffn    csrc/cuda/matmul.cu:169-205
//   wisp_gpu_scale_accum   csrc/cuda/matmul.cu:150-161
//   wisp_gpu_router_topk   csrc/cuda/router.cu:140-171
//
// The void launchers return silently on non-positive sizes, exactly as the
// reference does. The fused int4 path that supersedes the dequant -> gemv
// chain lives in decode.cu / grouped.cu.
#include <mutex>

#include "common.cuh"
#include "wisp_b200.h"

using namespace wb;

namespace {

// ---------------------------------------------------------------------------
// int4 -> fp16 dequantisation: one packed byte (two elements) per thread
// iteration, fp32 math then one rounding to fp16, as the reference kernel.
// ---------------------------------------------------------------------------
__global__ void dequant_int4_f16_kernel(const uint8_t* __restrict__ packed,
                                        const __half* __restrict__ scales,
                                        const __half* __restrict__ zeros,
                                        __half* __restrict__ out, long long n, int gs) {
  const long long nbytes = (n + 1) >> 1;
  for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < nbytes;
       b += (long long)gridDim.x * blockDim.x) {
    const uint8_t byte = __ldg(packed + b);
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const long long i = 2 * b + h;
      if (i >= n) break;
      const int nib = h ? (byte >> 4) : (byte & 0x0f);
      const long long g = i / gs;
      const float s = __half2float(scales[g]);
      const float z = __half2float(zeros[g]);
      out[i] = __float2half((float)(nib - 8) * s + z);
    }
  }
}

int grid_for(long long work, int threads) {
  long long b = (work + threads - 1) / threads;
  const long long cap = 148LL * 16;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

// ---------------------------------------------------------------------------
// fp16-weight GEMV, fp32 x/y: one warp per row, 16-byte weight loads when
// the row is 16-byte aligned, fp32 accumulation, shuffle reduction.
// ---------------------------------------------------------------------------
__device__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ float row_dot_f16(const __half* __restrict__ row, const float* __restrict__ x,
                             int cols) {
  const int lane = threadIdx.x & 31;
  float acc = 0.f;
  const bool vec = ((reinterpret_cast<uintptr_t>(row) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && (cols % 8 == 0);
  if (vec) {
    for (int c = lane * 8; c < cols; c += 256) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(row + c));
      const float4 x0 = __ldg(reinterpret_cast<const float4*>(x + c));
      const float4 x1 = __ldg(reinterpret_cast<const float4*>(x + c + 4));
      const float2 w0 = __half22float2(u2h2(w.x)), w1 = __half22float2(u2h2(w.y));
      const float2 w2 = __half22float2(u2h2(w.z)), w3 = __half22float2(u2h2(w.w));
      acc += w0.x * x0.x + w0.y * x0.y + w1.x * x0.z + w1.y * x0.w;
      acc += w2.x * x1.x + w2.y * x1.y + w3.x * x1.z + w3.y * x1.w;
    }
  } else {
    for (int c = lane; c < cols; c += 32) acc += __half2float(row[c]) * x[c];
  }
  return warp_sum(acc);
}

__global__ void gemv_f16_kernel(const __half* __restrict__ W, const float* __restrict__ x,
                                float* __restrict__ y, int rows, int cols) {
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float acc = row_dot_f16(W + (size_t)r * cols, x, cols);
  if ((threadIdx.x & 31) == 0) y[r] = acc;
}

__global__ void swiglu_ffn_f16_kernel(const __half* __restrict__ Wg, const __half* __restrict__ Wu,
                                      const float* __restrict__ x, float* __restrict__ h,
                                      int inter, int cols) {
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= inter) return;
  const float g = row_dot_f16(Wg + (size_t)r * cols, x, cols);
  const float u = row_dot_f16(Wu + (size_t)r * cols, x, cols);
  if ((threadIdx.x & 31) == 0) h[r] = silu(g) * u;
}

__global__ void swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u,
                              float* __restrict__ o, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    o[i] = silu(g[i]) * u[i];
}

__global__ void scale_accum_kernel(float* __restrict__ acc, const float* __restrict__ x, float w,
                                   int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    acc[i] += w * x[i];
}

// ---------------------------------------------------------------------------
// Router: logits[e] = W[e] . x + bias[e]  (4 warps per row split the hidden
// dimension), then one block does softmax + top-k + renormalisation.
// ---------------------------------------------------------------------------
constexpr int kRouterMaxTopK = 64;

__global__ void router_gemv_kernel(const __half* __restrict__ W, const __half* __restrict__ bias,
                                   const float* __restrict__ x, float* __restrict__ logits,
                                   int n_experts, int hidden) {
  __shared__ float part[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 2 + (warp >> 2);
  const int q = warp & 3;  // quarter of the hidden dimension
  float acc = 0.f;
  if (e < n_experts) {
    const __half* row = W + (size_t)e * hidden;
    for (int c = q * 32 + lane; c < hidden; c += 128) acc += __half2float(row[c]) * x[c];
  }
  acc = warp_sum(acc);
  if (lane == 0) part[warp] = acc;
  __syncthreads();
  if ((warp & 3) == 0 && lane == 0 && e < n_experts) {
    const float s = part[warp] + part[warp + 1] + part[warp + 2] + part[warp + 3];
    logits[e] = s + (bias ? __half2float(bias[e]) : 0.f);
  }
}

// Block-wide argmax with the lower index winning ties.
__device__ void block_argmax(float v, int idx, float* sv, int* si, float& bv, int& bi) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi >= 0 && (idx < 0 || oi < idx))) {
      v = ov;
      idx = oi;
    }
  }
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = sv[0];
    int i = si[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) {
      if (sv[w] > b || (sv[w] == b && si[w] >= 0 && (i < 0 || si[w] < i))) {
        b = sv[w];
        i = si[w];
      }
    }
    sv[0] = b;
    si[0] = i;
  }
  __syncthreads();
  bv = sv[0];
  bi = si[0];
  __syncthreads();
}

// Softmax over all experts, k rounds of "largest untaken probability, lower
// index on ties" (initial best value -1 and index -1 as in the reference),
// then renormalise the winners. n_experts <= 1024 (4 per thread).
__global__ void router_topk_kernel(const float* __restrict__ logits, int n_experts, int top_k,
                                   int* __restrict__ out_idx, float* __restrict__ out_w) {
  __shared__ float sv[8];
  __shared__ int si[8];
  float p[4];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int e = threadIdx.x + j * 256;
    p[j] = e < n_experts ? logits[e] : -INFINITY;
    mx = fmaxf(mx, p[j]);
  }
  float bv;
  int bi;
  block_argmax(mx, 0, sv, si, bv, bi);
  const float gmax = bv;
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int e = threadIdx.x + j * 256;
    p[j] = e < n_experts ? expf(p[j] - gmax) : 0.f;
    s += p[j];
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) sv[threadIdx.x >> 5] = s;
  __syncthreads();
  float den = 0.f;
  for (int w = 0; w < 8; w++) den += sv[w];
  __syncthreads();
  const float inv = 1.f / (den > 0.f ? den : 1.f);
#pragma unroll
  for (int j = 0; j < 4; j++) p[j] *= inv;
  bool taken[4] = {false, false, false, false};
  float wsum = 0.f;
  for (int k = 0; k < top_k; k++) {
    float v = -1.f;
    int i = -1;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int e = threadIdx.x + j * 256;
      if (e < n_experts && !taken[j] && p[j] > v) {
        v = p[j];
        i = e;
      }
    }
    block_argmax(v, i, sv, si, bv, bi);
#pragma unroll
    for (int j = 0; j < 4; j++)
      if (threadIdx.x + j * 256 == bi) taken[j] = true;
    if (threadIdx.x == 0) {
      out_idx[k] = bi;
      out_w[k] = bv;
    }
    wsum += bv;
  }
  if (threadIdx.x == 0 && wsum > 0.f)
    for (int k = 0; k < top_k; k++) out_w[k] /= wsum;
}

// Any number of experts: the same selection with the scratch row as working
// memory, as the reference does (its softmax leaves exp(logit - max) in the
// scratch). Each of the k rounds takes the largest remaining exp value (lower
// index on ties, initial best -1) and marks the winner's slot -inf so no
// later round can pick it; weights are value / sum, renormalised over the
// winners.
__global__ void router_topk_any_kernel(float* __restrict__ logits, int n_experts, int top_k,
                                       int* __restrict__ out_idx, float* __restrict__ out_w) {
  __shared__ float sv[8];
  __shared__ int si[8];
  float mx = -INFINITY;
  for (int e = threadIdx.x; e < n_experts; e += blockDim.x) mx = fmaxf(mx, logits[e]);
  float bv;
  int bi;
  block_argmax(mx, 0, sv, si, bv, bi);
  const float gmax = bv;
  float s = 0.f;
  for (int e = threadIdx.x; e < n_experts; e += blockDim.x) {
    const float v = expf(logits[e] - gmax);
    logits[e] = v;
    s += v;
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) sv[threadIdx.x >> 5] = s;
  __syncthreads();
  float den = 0.f;
  for (int w = 0; w < 8; w++) den += sv[w];
  __syncthreads();
  const float inv = 1.f / (den > 0.f ? den : 1.f);
  float wsum = 0.f;
  for (int k = 0; k < top_k; k++) {
    float v = -1.f;
    int i = -1;
    for (int e = threadIdx.x; e < n_experts; e += blockDim.x) {
      const float q = logits[e];
      if (q > v) {   // ascending e per thread: the lower index keeps a tie
        v = q;
        i = e;
      }
    }
    block_argmax(v, i, sv, si, bv, bi);
    if (threadIdx.x == 0) {
      out_idx[k] = bi;
      out_w[k] = bv * inv;
      if (bi >= 0) logits[bi] = -INFINITY;
    }
    wsum += bv * inv;
    __syncthreads();
  }
  if (threadIdx.x == 0 && wsum > 0.f)
    for (int k = 0; k < top_k; k++) out_w[k] /= wsum;
}

// Per-device staging for the router result (process-wide, as in the
// reference: the engine runs one router per layer on one stream).
std::mutex g_stage_mu;
int* g_stage_idx[64] = {nullptr};
float* g_stage_w[64] = {nullptr};

}  // namespace

extern "C" cudaError_t launch_dequant_expert(const uint8_t* d_packed, const wisp_half* d_scales,
                                             const wisp_half* d_zeros, wisp_half* d_output,
                                             int n_elements, int group_size,
                                             cudaStream_t stream) {
  if (n_elements <= 0 || group_size <= 0) return cudaErrorInvalidValue;
  const long long nbytes = ((long long)n_elements + 1) / 2;
  dequant_int4_f16_kernel<<<grid_for(nbytes, 256), 256, 0, stream>>>(
      d_packed, reinterpret_cast<const __half*>(d_scales),
      reinterpret_cast<const __half*>(d_zeros), reinterpret_cast<__half*>(d_output),
      n_elements, group_size);
  return cudaGetLastError();
}

extern "C" cudaError_t async_load_expert(const uint8_t* h_packed, const wisp_half* h_scales,
                                         const wisp_half* h_zeros, uint8_t* d_packed_tmp,
                                         wisp_half* d_scales_tmp, wisp_half* d_zeros_tmp,
                                         wisp_half* d_output, int n_elements, int group_size,
                                         cudaStream_t stream) {
  if (n_elements <= 0 || group_size <= 0) return cudaErrorInvalidValue;
  const size_t n_groups = ((size_t)n_elements + group_size - 1) / group_size;
  const size_t packed_bytes = ((size_t)n_elements + 1) / 2;
  const size_t scale_bytes = n_groups * 2;
  cudaError_t e = cudaMemcpyAsync(d_packed_tmp, h_packed, packed_bytes, cudaMemcpyHostToDevice,
                                  stream);
  if (e != cudaSuccess) return e;
  e = cudaMemcpyAsync(d_scales_tmp, h_scales, scale_bytes, cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return e;
  e = cudaMemcpyAsync(d_zeros_tmp, h_zeros, scale_bytes, cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return e;
  return launch_dequant_expert(d_packed_tmp, d_scales_tmp, d_zeros_tmp, d_output, n_elements,
                               group_size, stream);
}

extern "C" void wisp_gpu_gemv_f16(const wisp_half* W, const float* x, float* y, int rows,
                                  int cols, cudaStream_t s) {
  if (rows <= 0 || cols <= 0) return;
  gemv_f16_kernel<<<(rows + 7) / 8, 256, 0, s>>>(reinterpret_cast<const __half*>(W), x, y, rows,
                                                 cols);
}

extern "C" void wisp_gpu_swiglu(const float* gate, const float* up, float* out, int n,
                                cudaStream_t s) {
  if (n <= 0) return;
  swiglu_kernel<<<grid_for(n, 256), 256, 0, s>>>(gate, up, out, n);
}

extern "C" void wisp_gpu_swiglu_ffn(const wisp_half* Wg, const wisp_half* Wu, const float* x,
                                    float* h, int inter, int cols, cudaStream_t s) {
  if (inter <= 0 || cols <= 0) return;
  swiglu_ffn_f16_kernel<<<(inter + 7) / 8, 256, 0, s>>>(reinterpret_cast<const __half*>(Wg),
                                                       reinterpret_cast<const __half*>(Wu), x,
                                                       h, inter, cols);
}

extern "C" void wisp_gpu_scale_accum(float* acc, const float* x, float w, int n,
                                     cudaStream_t s) {
  if (n <= 0) return;
  scale_accum_kernel<<<grid_for(n, 256), 256, 0, s>>>(acc, x, w, n);
}

extern "C" void wisp_gpu_router_topk(const wisp_half* W, const wisp_half* bias, const float* x,
                                     float* logits_scratch, int n_experts, int hidden,
                                     int top_k, int* out_idx, float* out_w, cudaStream_t s) {
  if (n_experts <= 0 || top_k <= 0) return;
  if (top_k > kRouterMaxTopK) top_k = kRouterMaxTopK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
  {
    std::lock_guard<std::mutex> lock(g_stage_mu);
    if (!g_stage_idx[dev]) {
      if (cudaMalloc(&g_stage_idx[dev], kRouterMaxTopK * sizeof(int)) != cudaSuccess) return;
      if (cudaMalloc(&g_stage_w[dev], kRouterMaxTopK * sizeof(float)) != cudaSuccess) return;
    }
  }
  router_gemv_kernel<<<(n_experts + 1) / 2, 256, 0, s>>>(reinterpret_cast<const __half*>(W),
                                                         reinterpret_cast<const __half*>(bias),
                                                         x, logits_scratch, n_experts, hidden);
  if (n_experts <= 1024)   // one block of 256 threads holds 4 experts each in registers
    router_topk_kernel<<<1, 256, 0, s>>>(logits_scratch, n_experts, top_k, g_stage_idx[dev],
                                         g_stage_w[dev]);
  else
    router_topk_any_kernel<<<1, 256, 0, s>>>(logits_scratch, n_experts, top_k, g_stage_idx[dev],
                                             g_stage_w[dev]);
  cudaMemcpyAsync(out_idx, g_stage_idx[dev], (size_t)top_k * sizeof(int), cudaMemcpyDeviceToHost,
                  s);
  cudaMemcpyAsync(out_w, g_stage_w[dev], (size_t)top_k * sizeof(float), cudaMemcpyDeviceToHost,
                  s);
  // The caller synchronises the stream before reading out_idx / out_w.
}
