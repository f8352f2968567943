// route.cu -- batched routing and token -> expert dispatch for T tokens.
//
//   router_logits_kernel  logits = x W^T (+ bias), bf16 inputs, fp32 sums.
//                         Tiled 64x64 with a deterministic split-K so small
//                         token counts still fill the GPU (the top-k kernel
//                         sums the partials in a fixed order).
//   router_mma_kernel     the same with a bf16 router weight on the tensor
//                         cores (mma.sync m16n8k16 bf16, fp32 accumulate):
//                         64x64 tiles, 64-K stages double-buffered by
//                         cp.async into swizzled shared memory, ldmatrix
//                         fragments; the same split-K partials.
//   router_gemv_kernel    the same logits for T <= 4 tokens: one warp per
//                         (expert, K quarter) with all of its weight loads
//                         in flight, quarters summed in a fixed order.
//   topk_kernel           one warp per token. Softmax scoring follows the
//                         reference exactly (csrc/core/wisp_engine.c:782-818,
//                         csrc/cuda/router.cu:67-138): softmax, k rounds of
//                         "largest untaken probability, lower index on a
//                         tie", renormalise. Sigmoid group-limited scoring
//                         (DeepSeek-V3 convention; absent in the reference):
//                         group score = sum of the top-2 sigmoid scores,
//                         keep topk_groups groups, pick k experts among
//                         them, w = s / sum(s) * routed_scaling.
//   count / fill kernels  one block per expert; its warps scan consecutive
//                         ranges of the (token, slot) pairs, count, take
//                         their ranges' offsets in order and compact their
//                         matches with a ballot, so every expert's rows are
//                         sorted by token and the permutation is
//                         deterministic. An always-on shared expert is one
//                         more segment holding every token.
//   pack_rows_kernel      gathers bf16 token rows into fp16 rows in the
//                         interleaved K order the tensor-core kernel expects.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "skinny.h"

using namespace wb;

namespace {

constexpr int kRT = 64;   // router tile: tokens
constexpr int kRE = 64;   // router tile: experts
constexpr int kRK = 32;   // K chunk

__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

__device__ __forceinline__ float f16f(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// grid (ceil(E/64), ceil(T/64), splits); 256 threads compute 4x4 each.
// W_FP16 selects the router weight dtype (bf16 or fp16); x is bf16.
template <bool W_FP16>
__global__ void __launch_bounds__(256) router_logits_kernel(const uint16_t* __restrict__ x,
                                                            const uint16_t* __restrict__ W,
                                                            float* __restrict__ part, int T, int E,
                                                            int M, int kspan) {
  // read as float4 below: 16-byte alignment must not depend on the layout
  // of the kernel's other shared variables
  __shared__ __align__(16) float xs[kRK][kRT + 4];
  __shared__ __align__(16) float ws[kRK][kRE + 4];
  const int e0 = blockIdx.x * kRE, t0 = blockIdx.y * kRT;
  const int kb = blockIdx.z * kspan, ke = min(M, kb + kspan);
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 16 x 16 threads
  float acc[4][4] = {};
  for (int k0 = kb; k0 < ke; k0 += kRK) {
    // 64 rows x 32 K per operand: 256 threads x 8 values.
    {
      const int row = threadIdx.x >> 2, kq = (threadIdx.x & 3) * 8;
      const int t = t0 + row, e = e0 + row;
      uint4 xv = make_uint4(0, 0, 0, 0), wv = make_uint4(0, 0, 0, 0);
      if (t < T && k0 + kq < ke) xv = __ldg(reinterpret_cast<const uint4*>(x + (size_t)t * M + k0 + kq));
      if (e < E && k0 + kq < ke) wv = __ldg(reinterpret_cast<const uint4*>(W + (size_t)e * M + k0 + kq));
      const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        xs[kq + 2 * j][row] = bf16f((uint16_t)(xa[j] & 0xffff));
        xs[kq + 2 * j + 1][row] = bf16f((uint16_t)(xa[j] >> 16));
        ws[kq + 2 * j][row] = W_FP16 ? f16f((uint16_t)(wa[j] & 0xffff)) : bf16f((uint16_t)(wa[j] & 0xffff));
        ws[kq + 2 * j + 1][row] = W_FP16 ? f16f((uint16_t)(wa[j] >> 16)) : bf16f((uint16_t)(wa[j] >> 16));
      }
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < kRK; k++) {
      const float4 a = *reinterpret_cast<const float4*>(&xs[k][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&ws[k][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  float* out = part + (size_t)blockIdx.z * T * E;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int t = t0 + ty * 4 + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int e = e0 + tx * 4 + j;
      if (e < E) out[(size_t)t * E + e] = acc[i][j];
    }
  }
}

constexpr int kMT = 64, kME = 64, kMK = 64;   // tensor-core router tile: tokens, experts, K

__device__ __forceinline__ void cp_async_16_zfill(void* smem_dst, const void* gsrc, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc),
               "r"(valid ? 16 : 0)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// grid (ceil(E/64), ceil(T/64), splits), 128 threads; bf16 x [T x M] and W
// [E x M] (M and kspan multiples of 64). Warp (wm, wn) owns tokens 32 wm..
// and experts 32 wn.. of the tile. Shared rows are 64 K (128 bytes) with
// 16-byte chunk c of row r stored at c ^ (r & 7), so each ldmatrix phase
// reads eight distinct bank groups.
__global__ void __launch_bounds__(128) router_mma_kernel(const uint16_t* __restrict__ x,
                                                         const uint16_t* __restrict__ W,
                                                         float* __restrict__ part, int T, int E,
                                                         int M, int kspan) {
  __shared__ __align__(128) uint16_t sa[2][kMT * kMK];
  __shared__ __align__(128) uint16_t sb[2][kME * kMK];
  const int e0 = blockIdx.x * kME, t0 = blockIdx.y * kMT;
  const int kb = blockIdx.z * kspan, ke = min(M, kb + kspan);
  const int nst = max(0, (ke - kb) / kMK);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wm = warp & 1, wn = warp >> 1;
  auto load = [&](int st, int buf) {
    const int k0 = kb + st * kMK;
    for (int c = tid; c < kMT * 8; c += blockDim.x) {
      const int r = c >> 3, ch = c & 7;
      const int sw = (r * kMK) + ((ch ^ (r & 7)) << 3);
      const bool vt = t0 + r < T, ve = e0 + r < E;
      cp_async_16_zfill(&sa[buf][sw], x + (size_t)(vt ? t0 + r : 0) * M + k0 + ch * 8, vt);
      cp_async_16_zfill(&sb[buf][sw], W + (size_t)(ve ? e0 + r : 0) * M + k0 + ch * 8, ve);
    }
    cp_async_commit();
  };
  float c[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; i++)
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int v = 0; v < 4; v++) c[i][j][v] = 0.f;
  if (nst > 0) load(0, 0);
  const int mat = lane >> 3, lr = lane & 7;
  for (int st = 0; st < nst; st++) {
    const int buf = st & 1;
    if (st + 1 < nst) {
      load(st + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t abase = smem_u32(&sa[buf][0]), bbase = smem_u32(&sb[buf][0]);
#pragma unroll
    for (int kk = 0; kk < kMK / 16; kk++) {
      uint32_t a[2][4], b[4][2];
#pragma unroll
      for (int mi = 0; mi < 2; mi++) {
        // matrices: rows 0-7 / 8-15 x k 0-7, then the same x k 8-15
        const int row = wm * 32 + mi * 16 + (mat & 1) * 8 + lr;
        const int ch = kk * 2 + (mat >> 1);
        ldsm_x4(abase + (uint32_t)(row * kMK + ((ch ^ (row & 7)) << 3)) * 2, a[mi][0], a[mi][1],
                a[mi][2], a[mi][3]);
      }
#pragma unroll
      for (int nj = 0; nj < 2; nj++) {
        // matrices: experts 0-7 x k 0-7 / 8-15, then experts 8-15 likewise
        const int row = wn * 32 + nj * 16 + (mat >> 1) * 8 + lr;
        const int ch = kk * 2 + (mat & 1);
        ldsm_x4(bbase + (uint32_t)(row * kMK + ((ch ^ (row & 7)) << 3)) * 2, b[2 * nj][0],
                b[2 * nj][1], b[2 * nj + 1][0], b[2 * nj + 1][1]);
      }
#pragma unroll
      for (int mi = 0; mi < 2; mi++)
#pragma unroll
        for (int ni = 0; ni < 4; ni++) mma_bf16_16816(c[mi][ni], a[mi], b[ni][0], b[ni][1]);
    }
    __syncthreads();  // the next iteration's copy overwrites this buffer
  }
  float* out = part + (size_t)blockIdx.z * T * E;
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int mi = 0; mi < 2; mi++)
#pragma unroll
    for (int ni = 0; ni < 4; ni++)
#pragma unroll
      for (int v = 0; v < 4; v++) {
        const int tok = t0 + wm * 32 + mi * 16 + g + (v >> 1) * 8;
        const int e = e0 + wn * 32 + ni * 8 + 2 * t4 + (v & 1);
        if (tok < T && e < E) out[(size_t)tok * E + e] = c[mi][ni][v];
      }
}

constexpr int kGemvMaxT = 4;   // tokens per launch of the GEMV router
constexpr int kGemvQ = 4;      // K quarters per expert (one warp each)
constexpr int kGemvU = 8;      // 16-byte weight loads in flight per lane

template <bool W_FP16>
__device__ __forceinline__ float dot8(uint4 w, uint4 x, float acc) {
  const uint32_t wa[4] = {w.x, w.y, w.z, w.w}, xa[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const float w0 = W_FP16 ? f16f((uint16_t)(wa[j] & 0xffff)) : bf16f((uint16_t)(wa[j] & 0xffff));
    const float w1 = W_FP16 ? f16f((uint16_t)(wa[j] >> 16)) : bf16f((uint16_t)(wa[j] >> 16));
    acc = fmaf(bf16f((uint16_t)(xa[j] & 0xffff)), w0, acc);
    acc = fmaf(bf16f((uint16_t)(xa[j] >> 16)), w1, acc);
  }
  return acc;
}

// grid ceil(E/2) x 256 threads: warp w covers expert 2*blockIdx.x + w/4 over
// K quarter w%4 (M a multiple of 8). Writes logits [T x E] (no bias).
template <bool W_FP16>
__global__ void __launch_bounds__(256) router_gemv_kernel(const uint16_t* __restrict__ x,
                                                          const uint16_t* __restrict__ W,
                                                          float* __restrict__ logits, int T, int E,
                                                          int M) {
  __shared__ float red[8][kGemvMaxT];
  pdl_trigger();   // the decode planner may start; it waits for these logits
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 2 + warp / kGemvQ, q = warp % kGemvQ;
  const int n8 = M / 8;
  const int qb = q * n8 / kGemvQ, qe = (q + 1) * n8 / kGemvQ;
  float acc[kGemvMaxT];
#pragma unroll
  for (int t = 0; t < kGemvMaxT; t++) acc[t] = 0.f;
  if (e < E) {
    const uint4* wr = reinterpret_cast<const uint4*>(W + (size_t)e * M);
    for (int c0 = qb; c0 < qe; c0 += 32 * kGemvU) {
      uint4 wv[kGemvU];
#pragma unroll
      for (int i = 0; i < kGemvU; i++) {
        const int c = c0 + lane + 32 * i;
        wv[i] = c < qe ? __ldg(wr + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int t = 0; t < kGemvMaxT; t++) {
        if (t >= T) break;
        const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)t * M);
        uint4 xv[kGemvU];
#pragma unroll
        for (int i = 0; i < kGemvU; i++) {
          const int c = c0 + lane + 32 * i;
          xv[i] = c < qe ? __ldg(xr + c) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < kGemvU; i++) acc[t] = dot8<W_FP16>(wv[i], xv[i], acc[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kGemvMaxT; t++) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int t = 0; t < kGemvMaxT; t++) red[warp][t] = acc[t];
  }
  __syncthreads();
  if (threadIdx.x < 2 * kGemvMaxT) {
    const int el = threadIdx.x / kGemvMaxT, t = threadIdx.x % kGemvMaxT;
    const int ee = blockIdx.x * 2 + el;
    if (ee < E && t < T) {
      float s = red[el * kGemvQ][t];
#pragma unroll
      for (int j = 1; j < kGemvQ; j++) s += red[el * kGemvQ + j][t];
      logits[(size_t)t * E + ee] = s;
    }
  }
}

// Warp argmax with the lower index winning ties; (v, i) = (-inf/-1, -1) for
// an empty lane.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (oi >= 0 && (i < 0 || ov > v || (ov == v && oi < i))) {
      v = ov;
      i = oi;
    }
  }
}

// The routing of token t by one warp; lane l holds experts l + 32 j for
// j < PER (E <= 32 PER). Writes idx/w [T x k] (global or shared memory) and,
// optionally, the fp32 logits.
template <int PER>
__device__ __forceinline__ void topk_token(const float* __restrict__ part, int splits,
                                           const float* __restrict__ bias, int T, int t, int E,
                                           int k, int scoring, int n_groups, int topk_groups,
                                           float scaling, int* idx, float* wout,
                                           float* logits_out, int lane,
                                           const float* presum = nullptr) {
  const int per = (E + 31) / 32;
  float v[PER];
#pragma unroll
  for (int j = 0; j < PER; j++) v[j] = 0.f;
  if (presum) {
    // the logits were summed over the splits already (topk_kernel's helper
    // warps): one value per expert from shared memory
#pragma unroll
    for (int j = 0; j < PER; j++) {
      const int e = lane + 32 * j;
      if (j < per && e < E) v[j] = presum[e];
    }
  } else {
    // Split-K partials: split-major, all of a split's loads in flight
    // together (a per-expert loop over the splits would wait one L2 round
    // trip per split and expert).
    for (int z = 0; z < splits; z++) {
      const float* pz = part + ((size_t)z * T + t) * E;
#pragma unroll
      for (int j = 0; j < PER; j++) {
        const int e = lane + 32 * j;
        if (j < per && e < E) v[j] += __ldg(pz + e);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < PER; j++) {
    const int e = lane + 32 * j;
    if (j < per && e < E) {
      if (bias) v[j] += bias[e];
      if (logits_out) logits_out[(size_t)t * E + e] = v[j];
    } else {
      v[j] = -INFINITY;
    }
  }
  uint32_t taken = 0;  // bit j: expert lane + 32 j already chosen

  if (scoring == WISP_SCORE_SOFTMAX) {
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < PER; j++) mx = fmaxf(mx, v[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
      v[j] = (j < per && lane + 32 * j < E) ? expf(v[j] - mx) : -1.f;
      sum += v[j] > 0.f ? v[j] : 0.f;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.f / sum;
#pragma unroll
    for (int j = 0; j < PER; j++)
      if (v[j] >= 0.f) v[j] *= inv;
    float wsum = 0.f;
    float myw = 0.f;
    int myi = -1;
    for (int r = 0; r < k; r++) {
      float bv = -1.f;
      int bi = -1;
#pragma unroll
      for (int j = 0; j < PER; j++) {
        const int e = lane + 32 * j;
        if (j < per && e < E && !((taken >> j) & 1u) && v[j] > bv) {
          bv = v[j];
          bi = e;
        }
      }
      warp_argmax(bv, bi);
      if (bi >= 0 && (bi & 31) == lane) taken |= 1u << (bi >> 5);
      if (lane == r) {
        myw = bv;
        myi = bi;
      }
      wsum += bv;
    }
    if (lane < k) {
      idx[(size_t)t * k + lane] = myi;
      wout[(size_t)t * k + lane] = wsum > 0.f ? myw / wsum : myw;
    }
  } else {
    // Sigmoid group-limited.
    const int gsz = E / n_groups;
#pragma unroll
    for (int j = 0; j < PER; j++)
      if (j < per && lane + 32 * j < E) v[j] = 1.f / (1.f + expf(-v[j]));
    // Group scores, in registers: per group, every lane's top two of its
    // experts in the group, then a warp-wide top-2 merge; lane g keeps group
    // g's score (the sum of its two largest scores, ties counted twice).
    int gid[PER];
#pragma unroll
    for (int j = 0; j < PER; j++) gid[j] = (j < per && lane + 32 * j < E) ? (lane + 32 * j) / gsz : -1;
    float gscore = -INFINITY;
    for (int g = 0; g < n_groups; g++) {
      float a = -INFINITY, b = -INFINITY;
#pragma unroll
      for (int j = 0; j < PER; j++) {
        if (gid[j] == g) {
          const float s = v[j];
          b = fmaxf(b, fminf(a, s));
          a = fmaxf(a, s);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, a, o);
        const float ob = __shfl_xor_sync(0xffffffffu, b, o);
        b = fmaxf(fminf(a, oa), fmaxf(b, ob));
        a = fmaxf(a, oa);
      }
      if (lane == g) gscore = a + (gsz > 1 ? b : 0.f);
    }
    bool gsel = false;  // lane g: is group g kept
    for (int r = 0; r < topk_groups; r++) {
      float bv = (lane < n_groups && !gsel) ? gscore : -INFINITY;
      int bi = (lane < n_groups && !gsel) ? lane : -1;
      warp_argmax(bv, bi);
      if (bi == lane) gsel = true;
    }
    const unsigned gmask = __ballot_sync(0xffffffffu, gsel);
    uint32_t allow = 0;  // bit j: expert lane + 32 j lies in a kept group
#pragma unroll
    for (int j = 0; j < PER; j++) {
      const int e = lane + 32 * j;
      if (j < per && e < E && ((gmask >> (e / gsz)) & 1u)) allow |= 1u << j;
    }
    float ssum = 0.f, myw = 0.f;
    int myi = -1;
    for (int r = 0; r < k; r++) {
      float bv = -INFINITY;
      int bi = -1;
#pragma unroll
      for (int j = 0; j < PER; j++) {
        const int e = lane + 32 * j;
        if (((allow & ~taken) >> j) & 1u && (bi < 0 || v[j] > bv)) {
          bv = v[j];
          bi = e;
        }
      }
      warp_argmax(bv, bi);
      if (bi >= 0 && (bi & 31) == lane) taken |= 1u << (bi >> 5);
      if (lane == r) {
        myw = bv;
        myi = bi;
      }
      ssum += bi >= 0 ? bv : 0.f;
    }
    if (lane < k) {
      idx[(size_t)t * k + lane] = myi;
      wout[(size_t)t * k + lane] = myw / ssum * scaling;
    }
  }
}

// Block of 64 threads = two tokens x one warp, or, for many split partials,
// of kTopkQ warps for one token: warp q sums splits q, q + kTopkQ, ...
// (loads of a split in flight together) and warp 0 adds the kTopkQ sums in
// order, so the token waits for ceil(splits / kTopkQ) L2 round trips, not
// splits; warp 0 then routes the token.
constexpr int kTopkQ = 8;

template <int PER>
__global__ void __launch_bounds__(kTopkQ * 32) topk_kernel(
    const float* __restrict__ part, int splits, const float* __restrict__ bias, int T, int E, int k,
    int scoring, int n_groups, int topk_groups, float scaling, int* __restrict__ idx,
    float* __restrict__ wout, float* __restrict__ logits_out) {
  __shared__ float sums[kTopkQ][PER * 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool split_warps = blockDim.x == kTopkQ * 32;
  const int t = split_warps ? (int)blockIdx.x : (int)blockIdx.x * 2 + warp;
  const int q = split_warps ? warp : 0;
  const int per = (E + 31) / 32;
  if (split_warps) {
    if (t < T) {
      float v[PER];
#pragma unroll
      for (int j = 0; j < PER; j++) v[j] = 0.f;
      for (int z = q; z < splits; z += kTopkQ) {
        const float* pz = part + ((size_t)z * T + t) * E;
#pragma unroll
        for (int j = 0; j < PER; j++) {
          const int e = lane + 32 * j;
          if (j < per && e < E) v[j] += __ldg(pz + e);
        }
      }
#pragma unroll
      for (int j = 0; j < PER; j++) sums[q][lane + 32 * j] = v[j];
    }
    __syncthreads();
    if (q == 0 && t < T) {
#pragma unroll
      for (int j = 0; j < PER; j++) {
        float a = sums[0][lane + 32 * j];
        for (int qq = 1; qq < kTopkQ; qq++) a += sums[qq][lane + 32 * j];
        sums[0][lane + 32 * j] = a;
      }
    }
    __syncwarp();
  }
  if (q != 0 || t >= T) return;
  topk_token<PER>(part, splits, bias, T, t, E, k, scoring, n_groups, topk_groups, scaling, idx,
                  wout, logits_out, lane, split_warps ? &sums[0][0] : nullptr);
}

// One block of kPlanWarps warps per expert v: warp w scans the w-th
// contiguous range of the T*k (token, slot) pairs (a multiple of 32 long).
constexpr int kPlanWarps = 8;

__device__ __forceinline__ int plan_range(int nslots) {
  return ((nslots + kPlanWarps - 1) / kPlanWarps + 31) & ~31;
}

// Matches of expert v among slots [b, e) counted by one warp.
__device__ __forceinline__ int warp_count(const int* __restrict__ idx, int b, int e, int v, int lane) {
  int c = 0;
  for (int base = b; base < e; base += 32) {
    const int s = base + lane;
    c += __popc(__ballot_sync(0xffffffffu, s < e && __ldg(idx + s) == v));
  }
  return c;
}

// counts[v] for the routed experts (the shared expert, v == E, has T rows).
__global__ void __launch_bounds__(kPlanWarps * 32) count_kernel(const int* __restrict__ idx,
                                                                int nslots, int E, int T,
                                                                int* __restrict__ counts) {
  __shared__ int part[kPlanWarps];
  const int v = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (v == E) {
    if (threadIdx.x == 0) counts[v] = T;
    return;
  }
  const int L = plan_range(nslots);
  const int b = min(nslots, warp * L), e = min(nslots, b + L);
  const int c = warp_count(idx, b, e, v, lane);
  if (lane == 0) part[warp] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < kPlanWarps; w++) t += part[w];
    counts[v] = t;
  }
}

// Exclusive scan of counts into segments (single block).
__global__ void segments_kernel(const int* __restrict__ counts, int V, WispSegment* __restrict__ segs) {
  __shared__ int warp_tot[32];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int base = 0; base < V; base += blockDim.x) {
    const int v = base + threadIdx.x;
    const int n = v < V ? counts[v] : 0;
    int x = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[w] = x;
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
    const int incl = x + (w > 0 ? warp_tot[w - 1] : 0) + carry;
    if (v < V) {
      WispSegment s;
      s.expert = v;
      s.row_begin = incl - n;
      s.rows = n;
      s.reserved = 0;
      segs[v] = s;
    }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = incl;
    __syncthreads();
  }
}

// Rows of expert v sorted by (token, slot): row_token / row_weight. Each
// warp counts its range, the ranges' offsets follow in range order, then each
// warp compacts its matches with a ballot.
__global__ void __launch_bounds__(kPlanWarps * 32) fill_kernel(
    const int* __restrict__ idx, const float* __restrict__ w, int nslots, int k, int E, int T,
    const WispSegment* __restrict__ segs, int* __restrict__ row_token,
    float* __restrict__ row_weight) {
  __shared__ int part[kPlanWarps];
  const int v = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int begin = segs[v].row_begin;
  if (v == E) {
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
      row_token[begin + t] = t;
      row_weight[begin + t] = 1.f;
    }
    return;
  }
  const int L = plan_range(nslots);
  const int b = min(nslots, warp * L), e = min(nslots, b + L);
  const int c = warp_count(idx, b, e, v, lane);
  if (lane == 0) part[warp] = c;
  __syncthreads();
  int pos = begin;
  for (int q = 0; q < warp; q++) pos += part[q];
  for (int base = b; base < e; base += 32) {
    const int s = base + lane;
    const bool hit = s < e && __ldg(idx + s) == v;
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    if (hit) {
      const int p = pos + __popc(m & ((1u << lane) - 1u));
      row_token[p] = s / k;
      row_weight[p] = w[s];
    }
    pos += __popc(m);
  }
}

// The plan for up to kPlanMaxV experts (routed + shared) in two launches.
// count_segments_kernel (one block): per-expert counters in shared memory,
// filled with one atomic per (warp, expert) (__match_any_sync groups the
// lanes that hold the same expert), then the exclusive scan into segments.
// fill_ordered_kernel (one block per chunk of slots): the rows of expert v
// are its slots in (token, slot) order, so a slot's row is v's first row +
// the matches of v before the chunk (counted by the block) + the matches
// before it inside the chunk (per-warp counts, then ranks within each
// 32-slot group).
constexpr int kPlanMaxV = 1025;
constexpr int kChunkedPlanMin = 8192;   // slots above which the chunked plan runs
constexpr int kFillWarps = 8;

__device__ __forceinline__ void count_groups(int e, int lane, int* cnt) {
  const unsigned m = __match_any_sync(0xffffffffu, e);
  if (e >= 0 && (m & ((1u << lane) - 1u)) == 0) atomicAdd(&cnt[e], __popc(m));
}

__global__ void __launch_bounds__(1024) count_segments_kernel(const int* __restrict__ idx,
                                                              int nslots, int E, int T, int V,
                                                              int* __restrict__ counts,
                                                              WispSegment* __restrict__ segs) {
  __shared__ int cnt[kPlanMaxV];
  __shared__ int warp_tot[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int v = threadIdx.x; v < V; v += blockDim.x) cnt[v] = 0;
  __syncthreads();
  for (int base = 0; base < nslots; base += blockDim.x) {
    const int s = base + threadIdx.x;
    int e = s < nslots ? __ldg(idx + s) : -1;
    if (e >= E) e = -1;   // out-of-range indices match no expert
    count_groups(e, lane, cnt);
  }
  __syncthreads();
  if (V > E && threadIdx.x == 0) cnt[E] = T;   // the shared expert holds every token
  __syncthreads();
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < V; base += blockDim.x) {
    const int v = base + threadIdx.x;
    const int n = v < V ? cnt[v] : 0;
    int x = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[w] = x;
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
    const int incl = x + (w > 0 ? warp_tot[w - 1] : 0) + carry;
    if (v < V) {
      WispSegment sg;
      sg.expert = v;
      sg.row_begin = incl - n;
      sg.rows = n;
      sg.reserved = 0;
      segs[v] = sg;
      counts[v] = n;
    }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = incl;
    __syncthreads();
  }
}

// With `base` (the chunked plan), base[blockIdx.x * E + v] is the first row
// of expert v's rows from this chunk (segment start + the expert's matches in
// earlier chunks) and the scan of the earlier slots is skipped.
__global__ void __launch_bounds__(kFillWarps * 32) fill_ordered_kernel(
    const int* __restrict__ idx, const float* __restrict__ w, int nslots, int chunk, int k, int E,
    int T, int V, const WispSegment* __restrict__ segs, int* __restrict__ row_token,
    float* __restrict__ row_weight, const int* __restrict__ base) {
  __shared__ int before[kPlanMaxV];
  __shared__ int wcnt[kFillWarps][kPlanMaxV];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = blockIdx.x * chunk;
  const int per_warp = chunk / kFillWarps;            // a multiple of 32
  const int wb = c0 + warp * per_warp;
  // the shared expert's rows: every token once, in token order
  if (V > E) {
    const int begin = segs[E].row_begin;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
      row_token[begin + t] = t;
      row_weight[begin + t] = 1.f;
    }
  }
  for (int v = threadIdx.x; v < E; v += blockDim.x) {
    before[v] = 0;
#pragma unroll
    for (int q = 0; q < kFillWarps; q++) wcnt[q][v] = 0;
  }
  __syncthreads();
  // matches before the chunk (c0 is a multiple of the block size)
  for (int s = threadIdx.x; s < (base ? 0 : c0); s += blockDim.x) {
    int e = __ldg(idx + s);
    if (e >= E) e = -1;
    count_groups(e, lane, before);
  }
  // this warp's matches in its range
  for (int g = 0; g < per_warp; g += 32) {
    const int s = wb + g + lane;
    int e = s < nslots ? __ldg(idx + s) : -1;
    if (e >= E) e = -1;
    const unsigned m = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && (m & ((1u << lane) - 1u)) == 0) wcnt[warp][e] += __popc(m);
    __syncwarp();
  }
  __syncthreads();
  // first row of each (warp, expert) run
  for (int v = threadIdx.x; v < E; v += blockDim.x) {
    int run = base ? __ldg(base + (size_t)blockIdx.x * E + v) : segs[v].row_begin + before[v];
#pragma unroll
    for (int q = 0; q < kFillWarps; q++) {
      const int t = wcnt[q][v];
      wcnt[q][v] = run;
      run += t;
    }
  }
  __syncthreads();
  for (int g = 0; g < per_warp; g += 32) {
    const int s = wb + g + lane;
    int e = s < nslots ? __ldg(idx + s) : -1;
    if (e >= E) e = -1;
    const unsigned m = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(m & ((1u << lane) - 1u));
    const int base = e >= 0 ? wcnt[warp][e] : 0;
    __syncwarp();
    if (e >= 0) {
      row_token[base + rank] = s / k;
      row_weight[base + rank] = w[s];
      if (rank == 0) wcnt[warp][e] = base + __popc(m);
    }
    __syncwarp();
  }
}

// Chunked plan for many slots (prefill): one block per chunk of kChunkSlots
// slots counts its chunk per expert; one block then turns the counts into
// the segments and, per chunk and expert, the first row of the chunk's
// matches; fill_ordered_kernel places the rows with those bases. Three
// launches, each one pass over its data, instead of every fill block
// rescanning all slots before its chunk.
constexpr int kChunkSlots = 1024;

__global__ void __launch_bounds__(kChunkSlots) chunk_count_kernel(const int* __restrict__ idx,
                                                                  int nslots, int E,
                                                                  int* __restrict__ ccount) {
  __shared__ int cnt[kPlanMaxV];
  for (int v = threadIdx.x; v < E; v += blockDim.x) cnt[v] = 0;
  __syncthreads();
  const int s = blockIdx.x * kChunkSlots + threadIdx.x;
  int e = s < nslots ? __ldg(idx + s) : -1;
  if (e >= E) e = -1;
  count_groups(e, threadIdx.x & 31, cnt);
  __syncthreads();
  for (int v = threadIdx.x; v < E; v += blockDim.x) ccount[(size_t)blockIdx.x * E + v] = cnt[v];
}

// One block: totals per expert (chunk order), segments by a block scan (the
// shared expert, v = E, holds every token), then the per-chunk bases, in
// place of the counts.
__global__ void __launch_bounds__(1024) chunk_scan_kernel(int* __restrict__ ccount, int nchunk,
                                                          int E, int T, int V,
                                                          int* __restrict__ counts,
                                                          WispSegment* __restrict__ segs) {
  __shared__ int warp_tot[32];
  __shared__ int carry;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int b0 = 0; b0 < V; b0 += blockDim.x) {
    const int v = b0 + threadIdx.x;
    int n = 0;
    if (v < E) {
      for (int c = 0; c < nchunk; c++) n += ccount[(size_t)c * E + v];
    } else if (v < V) {
      n = T;
    }
    int x = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[w] = x;
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
    const int begin = x + (w > 0 ? warp_tot[w - 1] : 0) + carry - n;
    if (v < V) {
      WispSegment sg;
      sg.expert = v;
      sg.row_begin = begin;
      sg.rows = n;
      sg.reserved = 0;
      segs[v] = sg;
      counts[v] = n;
    }
    if (v < E) {   // chunk bases: the expert's first row of each chunk's matches
      int run = begin;
      for (int c = 0; c < nchunk; c++) {
        const int m = ccount[(size_t)c * E + v];
        ccount[(size_t)c * E + v] = run;
        run += m;
      }
    }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = begin + n;
    __syncthreads();
  }
}

// xp[p] = fp16(x[src[p]]) in interleaved K order; each thread moves 8 values.
__global__ void pack_rows_kernel(const uint16_t* __restrict__ x, const int* __restrict__ src, int n_rows,
                                 int M, uint16_t* __restrict__ xp) {
  const int p = blockIdx.x;
  if (p >= n_rows) return;
  const int s = src ? src[p] : p;
  const uint16_t* xr = x + (size_t)s * M;
  uint16_t* orow = xp + (size_t)p * M;
  for (int k8 = threadIdx.x * 8; k8 < M; k8 += blockDim.x * 8) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(xr + k8));
    const uint32_t a[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      f[2 * j] = bf16f((uint16_t)(a[j] & 0xffff));
      f[2 * j + 1] = bf16f((uint16_t)(a[j] >> 16));
    }
    // logical slot j holds physical offset {0,4,1,5,2,6,3,7}[j]
    const __half2 h0 = __floats2half2_rn(f[0], f[4]);
    const __half2 h1 = __floats2half2_rn(f[1], f[5]);
    const __half2 h2 = __floats2half2_rn(f[2], f[6]);
    const __half2 h3 = __floats2half2_rn(f[3], f[7]);
    *reinterpret_cast<uint4*>(orow + k8) = make_uint4(h22u(h0), h22u(h1), h22u(h2), h22u(h3));
  }
}

// The same rows gathered into the operand form of the kernel that computes
// them: xp[p] as above for rows of segments larger than sk_rows (tensor-core
// kernel), xq[p] as a q16 row (layout in skinny.h) for the others (register
// path). The row's segment is found by binary search over the segments'
// first rows. One block of 128 threads per row; a thread owns one
// packed-weight word (8 consecutive K) per 1024-K pass, so each half-warp
// holds one 128-K block: its max |x| (four shuffles) sets the block's scale,
// and every thread writes its word's 16 bytes. Half-warps past the row's
// end take part in the shuffles with zeros and store nothing.
__global__ void __launch_bounds__(128) pack_rows_q16_kernel(const uint16_t* __restrict__ x,
                                                            const int* __restrict__ src, int n_rows,
                                                            int M, uint16_t* __restrict__ xp,
                                                            uint8_t* __restrict__ xq,
                                                            const WispSegment* __restrict__ segs,
                                                            int nseg, int sk_rows) {
  const int p = blockIdx.x;
  if (p >= n_rows) return;
  // last segment whose first row is <= p (empty segments share a first row
  // with the next one and are skipped)
  int lo = 0, hi = nseg - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(&segs[mid].row_begin) <= p) lo = mid; else hi = mid - 1;
  }
  const WispSegment sg = segs[lo];
  if (p >= sg.row_begin + sg.rows) return;   // a padding row of no segment
  const bool want_q16 = sg.rows <= sk_rows;
  const int s = src ? src[p] : p;
  const uint16_t* xr = x + (size_t)s * M;
  uint16_t* orow = xp + (size_t)p * M;
  uint8_t* qrow = xq + (size_t)p * q16_row_bytes(M);
  const int lane = threadIdx.x & 31;
  for (int k0 = 0; k0 < M; k0 += 1024) {
    const int w = k0 / 8 + threadIdx.x;          // packed word of this thread
    const bool in = 8 * w < M;
    float f[8];
    if (in) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(xr + 8 * w));
      const uint32_t a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        f[2 * j] = bf16f((uint16_t)(a[j] & 0xffff));
        f[2 * j + 1] = bf16f((uint16_t)(a[j] >> 16));
      }
      const __half2 h0 = __floats2half2_rn(f[0], f[4]);
      const __half2 h1 = __floats2half2_rn(f[1], f[5]);
      const __half2 h2 = __floats2half2_rn(f[2], f[6]);
      const __half2 h3 = __floats2half2_rn(f[3], f[7]);
      if (!want_q16)
        *reinterpret_cast<uint4*>(orow + 8 * w) = make_uint4(h22u(h0), h22u(h1), h22u(h2), h22u(h3));
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) f[j] = 0.f;
    }
    if (!want_q16) continue;   // block-uniform
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) m = fmaxf(m, fabsf(f[j]));
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float inv = m > 0.f ? 32767.f / m : 0.f;
    int v[8], sum = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      v[j] = max(-32767, min(32767, __float2int_rn(f[j] * inv)));
      sum += v[j];
    }
    auto hi = [](int q) { return (uint32_t)((q >> 8) & 0xFF); };
    auto lo = [](int q) { return (uint32_t)(q & 0xFF); };
    const uint4 chunk = make_uint4(hi(v[0]) | hi(v[2]) << 8 | hi(v[4]) << 16 | hi(v[6]) << 24,
                                   hi(v[1]) | hi(v[3]) << 8 | hi(v[5]) << 16 | hi(v[7]) << 24,
                                   lo(v[0]) | lo(v[2]) << 8 | lo(v[4]) << 16 | lo(v[6]) << 24,
                                   lo(v[1]) | lo(v[3]) << 8 | lo(v[5]) << 16 | lo(v[7]) << 24);
    // sums over the block's K 0-63 (its first 8 threads) and 64-127
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const int sum1 = __shfl_sync(0xffffffffu, sum, (lane & 16) | 8);
    if (in) {
      *reinterpret_cast<uint4*>(qrow + q16_word_offset(w)) = chunk;
      if ((lane & 15) == 0) {
        const float sc = m / 32767.f;
        *reinterpret_cast<float4*>(qrow + q16_meta_offset(w / 16)) =
            make_float4(sc * 0.0625f, sc * (float)sum, sc * (float)sum1, 0.f);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Decode planner: for a batch of at most kGemvMaxT tokens, everything between
// the router logits and the register-path FFN in one block of 1024 threads
// (the general path takes six launches and two memsets for the same work,
// each a few microseconds of fixed cost at batch 1). Apart from the logits
// and the token rows, which are read at the start, it works in shared memory:
//   1. the routing into shared memory -- softmax: warps 0..T-1, one per
//      token (the code of topk_kernel); sigmoid group-limited: the first 256
//      threads together (route_sigmoid_block) -- while the other warps
//      quantise the T token rows to q16 rows in (dynamic) shared memory (a
//      row's q16 form depends only on its token) and zero the output rows
//      and the error word;
//   2. per-expert counts and segments (a block scan over the V experts), the
//      shared expert holding every token;
//   3. the register path's unit plans for gate/up and down, from the chunk
//      prefix the scan of step 2 carried along; the rows: slot s of expert e
//      lands at begin[e] + (earlier slots of e), so each expert's rows are in
//      token order, as in the general plan;
//   4. every row's q16 row, copied from its token's (coalesced 16-byte
//      stores); with one token, row 0 alone.
// Every segment has at most T <= 4 rows, so all of them run on the register
// path and no fp16 rows or tensor-core plans are needed.
// ---------------------------------------------------------------------------
struct DecodePlan {
  const float* logits;   // [T x E] from router_gemv_kernel (no bias)
  const float* bias;
  int T, E, k, scoring, n_groups, topk_groups;
  float scaling;
  int V;                 // E, + 1 with a shared expert
  int* idx;
  float* w;
  int* counts;
  WispSegment* segs;
  int* row_token;
  float* row_weight;
  const uint16_t* x;
  int M;
  uint8_t* xq;
  float* out;
  int* error_flag;
  int32_t* units_gu;
  int32_t* units_dn;
  int per_gu, per_dn, cols, sk_rows, ks_dn, nk_dn, target;
};

constexpr int kDecodeMaxSlots = kGemvMaxT * 32;         // tokens x top_k (k <= 32)
constexpr int kDecodeMaxRows = kDecodeMaxSlots + kGemvMaxT;

// Quantises one 128-K block of a bf16 row to q16 (layout in skinny.h) with
// a half-warp: lane hl of the half owns packed word 16 b + hl. All 32 lanes
// of the warp call it together; `valid` false contributes zeros and stores
// nothing.
__device__ __forceinline__ void q16_block(const uint16_t* __restrict__ xr, int b, bool valid,
                                          int lane, uint8_t* qrow) {
  const int hl = lane & 15;
  const int wd = b * (kQ16Block / 8) + hl;
  float f[8];
  if (valid) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(xr + 8 * wd));
    const uint32_t a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      f[2 * j] = bf16f((uint16_t)(a[j] & 0xffff));
      f[2 * j + 1] = bf16f((uint16_t)(a[j] >> 16));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; j++) f[j] = 0.f;
  }
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < 8; j++) m = fmaxf(m, fabsf(f[j]));
#pragma unroll
  for (int o = 1; o < 16; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float inv = m > 0.f ? 32767.f / m : 0.f;
  int v[8], sum = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    v[j] = max(-32767, min(32767, __float2int_rn(f[j] * inv)));
    sum += v[j];
  }
  auto hi = [](int q) { return (uint32_t)((q >> 8) & 0xFF); };
  auto lo = [](int q) { return (uint32_t)(q & 0xFF); };
  const uint4 chunk = make_uint4(hi(v[0]) | hi(v[2]) << 8 | hi(v[4]) << 16 | hi(v[6]) << 24,
                                 hi(v[1]) | hi(v[3]) << 8 | hi(v[5]) << 16 | hi(v[7]) << 24,
                                 lo(v[0]) | lo(v[2]) << 8 | lo(v[4]) << 16 | lo(v[6]) << 24,
                                 lo(v[1]) | lo(v[3]) << 8 | lo(v[5]) << 16 | lo(v[7]) << 24);
  // sums over the block's K 0-63 (its first 8 lanes) and 64-127
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const int sum1 = __shfl_sync(0xffffffffu, sum, (lane & 16) | 8);
  if (valid) {
    *reinterpret_cast<uint4*>(qrow + q16_word_offset(wd)) = chunk;
    if (hl == 0) {
      const float sc = m / 32767.f;
      *reinterpret_cast<float4*>(qrow + q16_meta_offset(b)) =
          make_float4(sc * 0.0625f, sc * (float)sum, sc * (float)sum1, 0.f);
    }
  }
}

// Sigmoid group-limited routing of T <= kGemvMaxT tokens by the first
// kRouteThreads threads of the block (named barrier 1), in parallel instead
// of one warp's serial rounds: scores, then one warp per (token, group) for
// the group scores (sum of the top two), then ranks -- a group is kept when
// fewer than topk_groups groups beat it, an expert in a kept group is picked
// at position r when r experts of the kept groups beat it, where "beat"
// means a higher score or an equal score at a lower index. That is exactly
// the order of topk_token's rounds (largest first, lower index on a tie), so
// indices and weights are identical to it. The picks land in s_sel / s_sels
// (32 per token, in order); sigmoid_slot turns them into a slot's index and
// weight after the block's next barrier, one thread per slot.
constexpr int kRouteThreads = 256;

__device__ __forceinline__ void route_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kRouteThreads) : "memory");
}

__device__ void route_sigmoid_block(const DecodePlan& p, float (*s_score)[1024],
                                    float (*s_gscore)[32], uint32_t* s_gkeep, int* s_sel,
                                    float* s_sels) {
  const int rt = threadIdx.x, lane = rt & 31, w = rt >> 5;
  const int T = p.T, E = p.E, k = p.k, G = p.n_groups, gsz = E / G;
  if (rt < T) s_gkeep[rt] = 0u;
  for (int i = rt; i < T * E; i += kRouteThreads) {
    const int t = i / E, e = i - t * E;
    float v = p.logits[i];
    if (p.bias) v += p.bias[e];
    s_score[t][e] = 1.f / (1.f + expf(-v));
  }
  route_bar();
  for (int pr = w; pr < T * G; pr += kRouteThreads / 32) {
    const int t = pr / G, g = pr - t * G;
    float a = -INFINITY, b = -INFINITY;
    for (int q = lane; q < gsz; q += 32) {
      const float v = s_score[t][g * gsz + q];
      b = fmaxf(b, fminf(a, v));
      a = fmaxf(a, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float oa = __shfl_xor_sync(0xffffffffu, a, o);
      const float ob = __shfl_xor_sync(0xffffffffu, b, o);
      b = fmaxf(fminf(a, oa), fmaxf(b, ob));
      a = fmaxf(a, oa);
    }
    if (lane == 0) s_gscore[t][g] = a + (gsz > 1 ? b : 0.f);
  }
  route_bar();
  for (int pr = rt; pr < T * G; pr += kRouteThreads) {
    const int t = pr / G, g = pr - t * G;
    const float gs = s_gscore[t][g];
    int rank = 0;
    for (int q = 0; q < G; q++) {
      const float o = s_gscore[t][q];
      rank += (o > gs) || (o == gs && q < g);
    }
    if (rank < p.topk_groups) atomicOr(&s_gkeep[t], 1u << g);
  }
  route_bar();
  for (int i = rt; i < T * E; i += kRouteThreads) {
    const int t = i / E, e = i - t * E;
    const uint32_t keep = s_gkeep[t];
    if (!((keep >> (e / gsz)) & 1u)) continue;
    const float v = s_score[t][e];
    int rank = 0;
    for (uint32_t m = keep; m; m &= m - 1) {
      const int g = __ffs(m) - 1;
      const float* row = &s_score[t][g * gsz];
      for (int q = 0; q < gsz; q++) {
        const float o = row[q];
        rank += (o > v) || (o == v && g * gsz + q < e);
      }
    }
    if (rank < k) {
      s_sel[t * 32 + rank] = e;
      s_sels[t * 32 + rank] = v;
    }
  }
  // (the weights are normalised by the caller, one thread per slot)
}

// Slot s of a sigmoid-routed token: its expert and its weight, the selected
// scores normalised over the token's k picks (summed in pick order) times
// routed_scaling.
__device__ __forceinline__ void sigmoid_slot(const DecodePlan& p, const int* s_sel,
                                             const float* s_sels, int s, int& e, float& w) {
  const int t = s / p.k, r = s - t * p.k;
  float ssum = 0.f;
  for (int q = 0; q < p.k; q++) ssum += s_sels[t * 32 + q];
  e = s_sel[t * 32 + r];
  w = s_sels[t * 32 + r] / ssum * p.scaling;
}

template <int PER>
__global__ void __launch_bounds__(1024) decode_plan_kernel(const DecodePlan p) {
  extern __shared__ __align__(16) uint8_t s_q16[];   // T q16 token rows
  __shared__ int s_idx[kDecodeMaxSlots];
  __shared__ float s_w[kDecodeMaxSlots];
  __shared__ __align__(16) WispSegment s_segs[kPlanMaxV];
  __shared__ int s_cpre[kPlanMaxV];   // register-path chunks before each segment
  __shared__ int s_tok[kDecodeMaxRows];
  __shared__ int warp_tot[32];
  __shared__ int carry;
  // sigmoid routing
  __shared__ float s_score[kGemvMaxT][1024];
  __shared__ float s_gscore[kGemvMaxT][32];
  __shared__ uint32_t s_gkeep[kGemvMaxT];
  __shared__ int s_sel[kGemvMaxT * 32];
  __shared__ float s_sels[kGemvMaxT * 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = blockDim.x >> 5;
  const int T = p.T, k = p.k, E = p.E, V = p.V, M = p.M, nslots = T * k;
  const size_t qbytes = q16_row_bytes(M);
  const int nblk = M / kQ16Block;
  // Launched as a programmatic dependent of the router: the routing warps
  // wait for the logits; the others only read the token rows, which the
  // kernels before the router wrote, and write buffers the router does not
  // touch.
  // 1. routing | token rows to q16, output zeroed. Softmax: one warp per
  // token; sigmoid group-limited: the first 256 threads together.
  const bool sigmoid = p.scoring == WISP_SCORE_SIGMOID_GROUPED;
  const int nrw = sigmoid ? kRouteThreads / 32 : T;   // routing warps
  if (warp < nrw) {
    pdl_wait();
    if (sigmoid)
      route_sigmoid_block(p, s_score, s_gscore, s_gkeep, s_sel, s_sels);
    else
      topk_token<PER>(p.logits, 1, p.bias, T, warp, E, k, p.scoring, p.n_groups, p.topk_groups,
                      p.scaling, s_idx, s_w, nullptr, lane);
  } else {
    const int ntask = T * nblk, half = (lane >> 4) & 1;
    // warp-uniform rounds: both halves of a warp run the same number
    for (int base = 2 * (warp - nrw); base < ntask; base += 2 * (nwarp - nrw)) {
      const int task = base + half;
      const bool valid = task < ntask;
      const int t = valid ? task / nblk : 0;
      q16_block(p.x + (size_t)t * M, valid ? task % nblk : 0, valid, lane, s_q16 + t * qbytes);
    }
    for (int i = tid - 32 * nrw; i < T * M; i += blockDim.x - 32 * nrw) p.out[i] = 0.f;
    if (tid == blockDim.x - 1) *p.error_flag = 0;
  }
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int s = tid; s < nslots; s += blockDim.x) {
    if (sigmoid) sigmoid_slot(p, s_sel, s_sels, s, s_idx[s], s_w[s]);
    p.idx[s] = s_idx[s];
    p.w[s] = s_w[s];
    if (s_idx[s] < 0 || s_idx[s] >= E) s_idx[s] = -1;
  }
  __syncthreads();
  // 2. counts and segments; the same scan counts each segment's register-path
  // chunks (low 16 bits: rows, high bits: chunks; rows <= 132, chunks <= V)
  for (int base = 0; base < V; base += blockDim.x) {
    const int v = base + tid;
    int n = 0;
    if (v < E) {
      for (int q = 0; q < nslots; q++) n += s_idx[q] == v;
    } else if (v < V) {
      n = T;
    }
    const int c = (n > 0 && n <= p.sk_rows) ? (n + p.cols - 1) / p.cols : 0;
    int xs = n | (c << 16);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, xs, o);
      if (lane >= o) xs += y;
    }
    if (lane == 31) warp_tot[warp] = xs;
    __syncthreads();
    if (warp == 0) {
      int tv = lane < nwarp ? warp_tot[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, tv, o);
        if (lane >= o) tv += y;
      }
      warp_tot[lane] = tv;
    }
    __syncthreads();
    const int incl = xs + (warp > 0 ? warp_tot[warp - 1] : 0) + carry;
    if (v < V) {
      WispSegment sg;
      sg.expert = v;
      sg.row_begin = (incl & 0xFFFF) - n;
      sg.rows = n;
      sg.reserved = 0;
      s_segs[v] = sg;
      p.segs[v] = sg;
      p.counts[v] = n;
      s_cpre[v] = (incl >> 16) - c;
    }
    __syncthreads();
    if (tid == blockDim.x - 1) carry = incl;
    __syncthreads();
  }
  const int rows = carry & 0xFFFF, chunks = carry >> 16;
  // 3. the register path's unit plans (the grouped call's plan_units: per
  // segment its chunks times the row blocks per chunk; the down projection's
  // K split when its units would not reach the target), and the rows in
  // token order within each expert
  {
    const int tot_dn = chunks * p.per_dn;
    int ks = 1;
    if (tot_dn > 0 && tot_dn < p.target)
      ks = min(min(p.ks_dn, p.nk_dn), (p.target + tot_dn - 1) / tot_dn);
    if (ks < 1) ks = 1;
    for (int v = tid; v < V; v += blockDim.x) {
      p.units_gu[v] = s_cpre[v] * p.per_gu;
      p.units_dn[v] = s_cpre[v] * p.per_dn * ks;
    }
    if (tid == 0) {
      p.units_gu[V] = chunks * p.per_gu;
      p.units_gu[V + 1] = 1;
      p.units_dn[V] = tot_dn * ks;
      p.units_dn[V + 1] = ks;
    }
  }
  for (int s = tid; s < nslots; s += blockDim.x) {
    const int e = s_idx[s];
    if (e < 0) continue;
    int r = 0;
    for (int q = 0; q < s; q++) r += s_idx[q] == e;
    const int pos = s_segs[e].row_begin + r;
    p.row_token[pos] = s / k;
    p.row_weight[pos] = s_w[s];
    s_tok[pos] = s / k;
  }
  if (V > E) {
    for (int t = tid; t < T; t += blockDim.x) {
      const int pos = s_segs[E].row_begin + t;
      p.row_token[pos] = t;
      p.row_weight[pos] = 1.f;
      s_tok[pos] = t;
    }
  }
  __syncthreads();
  // 4. every row's q16 row, copied from its token's. With one token every row
  // is token 0: only row 0 is written, and the gate/up kernel reads its token
  // rows there (SkLaunch::tok_row0).
  const int wpr = (int)(qbytes / 16);   // 16-byte words per q16 row
  const int ncopy = T == 1 ? min(rows, 1) : rows;
  for (int row = 0; row < ncopy; row++) {
    const uint4* src = reinterpret_cast<const uint4*>(s_q16 + (size_t)s_tok[row] * qbytes);
    uint4* dst = reinterpret_cast<uint4*>(p.xq + (size_t)row * qbytes);
    for (int wd = tid; wd < wpr; wd += blockDim.x) dst[wd] = src[wd];
  }
}

// y[t] = bf16(x[t] / rms(x[t])): per-token RMS normalisation (no weight)
// between stacked MoE layers. One block per token.
__global__ void rms_rescale_kernel(const float* __restrict__ x, uint16_t* __restrict__ y, int M,
                                   float eps) {
  __shared__ float red[32];
  const float* xr = x + (size_t)blockIdx.x * M;
  float s = 0.f;
  for (int i = threadIdx.x; i < M; i += blockDim.x) s += xr[i] * xr[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / M + eps);
  uint16_t* yr = y + (size_t)blockIdx.x * M;
  for (int i = threadIdx.x; i < M; i += blockDim.x)
    yr[i] = __bfloat16_as_ushort(__float2bfloat16_rn(xr[i] * inv));
}

// out[row_token[p]] += row_weight[p] * y[p] for p < n_rows (fp32 atomics):
// the combine of rows returned by the expert-parallel all-to-all.
__global__ void combine_rows_kernel(const float* __restrict__ y, const int* __restrict__ row_token,
                                    const float* __restrict__ row_weight, int M,
                                    float* __restrict__ out) {
  const int p = blockIdx.x;
  const int t = row_token[p];
  const float w = row_weight[p];
  const float* yr = y + (size_t)p * M;
  float* orow = out + (size_t)t * M;
  for (int i = threadIdx.x; i < M; i += blockDim.x) red_add_f32(orow + i, w * yr[i]);
}

int g_sms_cached = 0;

}  // namespace

namespace wb {

// Workspace carving shared with moe.cu.
size_t router_splits(int T, int E, int M) {
  if (!g_sms_cached) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms_cached, cudaDevAttrMultiProcessorCount, dev);
    if (g_sms_cached <= 0) g_sms_cached = 148;
  }
  if (T <= kGemvMaxT) return 1;
  const long long tiles = (long long)((E + kRE - 1) / kRE) * ((T + kRT - 1) / kRT);
  long long splits = (2LL * g_sms_cached + tiles - 1) / tiles;
  const long long max_splits = std::max(1, M / 256);
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  return (size_t)splits;
}

WispError launch_route(const WispMoeConfig* c, const uint16_t* x, const uint16_t* W,
                       const float* bias, float* part, size_t splits, float* logits_out, int* idx,
                       float* w, cudaStream_t st, WispErrCtx* err) {
  const int T = c->tokens, E = c->n_experts, M = c->hidden;
  int nsplit = 1;
  if (T <= kGemvMaxT) {
    const int g = (E + 1) / 2;
    if (c->router_fp16)
      wb::launch_k(router_gemv_kernel<true>, g, 256, 0, st, x, W, part, T, E, M);
    else
      wb::launch_k(router_gemv_kernel<false>, g, 256, 0, st, x, W, part, T, E, M);
  } else {
    // fp16 weights stay on the fp32 SIMT kernel (the tensor cores would need
    // the bf16 activations rounded to fp16).
    const int gran = c->router_fp16 ? kRK : kMK;
    int kspan = (M + (int)splits - 1) / (int)splits;
    kspan = (kspan + gran - 1) / gran * gran;
    nsplit = (M + kspan - 1) / kspan;
    dim3 g1((E + kRE - 1) / kRE, (T + kRT - 1) / kRT, nsplit);
    if (c->router_fp16)
      wb::launch_k(router_logits_kernel<true>, g1, 256, 0, st, x, W, part, T, E, M, kspan);
    else
      wb::launch_k(router_mma_kernel, g1, 128, 0, st, x, W, part, T, E, M, kspan);
  }
  auto topk = E <= 32 ? topk_kernel<1> : E <= 64 ? topk_kernel<2> : E <= 128 ? topk_kernel<4>
            : E <= 256 ? topk_kernel<8> : E <= 512 ? topk_kernel<16> : topk_kernel<32>;
  // two tokens per block (one warp each), so a few hundred tokens still
  // spread over the SMs; kTopkQ warps per token to sum more than two splits
  const bool split_warps = nsplit > 2;
  wb::launch_k(topk, split_warps ? T : (T + 1) / 2, split_warps ? kTopkQ * 32 : 64, 0, st, part,
               nsplit,
               bias, T, E, c->top_k, c->scoring, c->n_groups, c->topk_groups, c->routed_scaling,
               idx, w, logits_out);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

// Scratch of the chunked plan (ints), 0 when the two-launch plan is used.
size_t plan_scratch_ints(const WispMoeConfig* c) {
  const int nslots = c->tokens * c->top_k;
  const int V = c->n_experts + (c->has_shared ? 1 : 0);
  if (nslots <= kChunkedPlanMin || V > kPlanMaxV) return 0;
  return (size_t)((nslots + kChunkSlots - 1) / kChunkSlots) * c->n_experts;
}

WispError launch_plan(const WispMoeConfig* c, const int* idx, const float* w, int* counts,
                      WispSegment* segs, int* row_token, float* row_weight, cudaStream_t st,
                      WispErrCtx* err, int* scratch) {
  const int T = c->tokens, E = c->n_experts, k = c->top_k, sh = c->has_shared ? 1 : 0;
  const int V = E + sh;
  const int nslots = T * k;
  if (scratch && plan_scratch_ints(c) > 0) {
    const int nchunk = (nslots + kChunkSlots - 1) / kChunkSlots;
    wb::launch_k(chunk_count_kernel, nchunk, kChunkSlots, 0, st, idx, nslots, E, scratch);
    wb::launch_k(chunk_scan_kernel, 1, 1024, 0, st, scratch, nchunk, E, T, V, counts, segs);
    wb::launch_k(fill_ordered_kernel, nchunk, kFillWarps * 32, 0, st, idx, w, nslots,
                 kChunkSlots, k, E, T, V, segs, row_token, row_weight,
                 static_cast<const int*>(scratch));
  } else if (V <= kPlanMaxV) {
    // chunks of 1024 slots, larger for large batches so that at most 32
    // blocks count the slots before their chunk
    const int chunk = 1024 * std::max(1, (nslots + 32 * 1024 - 1) / (32 * 1024));
    wb::launch_k(count_segments_kernel, 1, 1024, 0, st, idx, nslots, E, T, V, counts, segs);
    wb::launch_k(fill_ordered_kernel, (nslots + chunk - 1) / chunk, kFillWarps * 32, 0, st, idx, w,
                 nslots, chunk, k, E, T, V, segs, row_token, row_weight,
                 static_cast<const int*>(nullptr));
  } else {
    wb::launch_k(count_kernel, V, kPlanWarps * 32, 0, st, idx, nslots, E, T, counts);
    wb::launch_k(segments_kernel, 1, 1024, 0, st, counts, V, segs);
    wb::launch_k(fill_kernel, V, kPlanWarps * 32, 0, st, idx, w, nslots, k, E, T, segs, row_token,
                 row_weight);
  }
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

WispError launch_pack_q16(const uint16_t* x, const int* src, int n_rows, int M, uint16_t* xp,
                          uint8_t* xq, const WispSegment* segs, int nseg, int sk_rows,
                          cudaStream_t st, WispErrCtx* err) {
  if (n_rows <= 0) return WISP_OK;
  wb::launch_k(pack_rows_q16_kernel, n_rows, 128, 0, st, x, src, n_rows, M, xp, xq, segs, nseg,
               sk_rows);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

WispError launch_router_gemv(const WispMoeConfig* c, const uint16_t* x, const uint16_t* W,
                             float* logits, cudaStream_t st, WispErrCtx* err) {
  const int g = (c->n_experts + 1) / 2;
  if (c->router_fp16)
    wb::launch_k(router_gemv_kernel<true>, g, 256, 0, st, x, W, logits, c->tokens, c->n_experts,
                 c->hidden);
  else
    wb::launch_k(router_gemv_kernel<false>, g, 256, 0, st, x, W, logits, c->tokens, c->n_experts,
                 c->hidden);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

// Dynamic shared memory of the decode planner: the T tokens' q16 rows.
static size_t decode_plan_smem(const WispMoeConfig* c) {
  return (size_t)c->tokens * q16_row_bytes(c->hidden);
}

bool decode_plan_fits(const WispMoeConfig* c, int sk_rows) {
  const int V = c->n_experts + (c->has_shared ? 1 : 0);
  // the q16 token rows next to ~36 KB of static shared memory
  return c->tokens >= 1 && c->tokens <= kGemvMaxT && c->tokens <= sk_rows && V <= kPlanMaxV &&
         c->top_k <= 32 && c->n_experts <= 1024 && decode_plan_smem(c) <= 160 * 1024;
}

WispError launch_decode_plan(const WispMoeConfig* c, const float* logits, const float* bias,
                             int* idx, float* w, int* counts, WispSegment* segs, int* row_token,
                             float* row_weight, const uint16_t* x, float* out, int* error_flag,
                             const DecodeUnits& du, cudaStream_t st, WispErrCtx* err) {
  DecodePlan p;
  p.logits = logits;
  p.bias = bias;
  p.T = c->tokens;
  p.E = c->n_experts;
  p.k = c->top_k;
  p.scoring = c->scoring;
  p.n_groups = c->n_groups;
  p.topk_groups = c->topk_groups;
  p.scaling = c->routed_scaling;
  p.V = c->n_experts + (c->has_shared ? 1 : 0);
  p.idx = idx;
  p.w = w;
  p.counts = counts;
  p.segs = segs;
  p.row_token = row_token;
  p.row_weight = row_weight;
  p.x = x;
  p.M = c->hidden;
  p.xq = du.xq;
  p.out = out;
  p.error_flag = error_flag;
  p.units_gu = du.units_gu;
  p.units_dn = du.units_dn;
  p.per_gu = du.per_gu;
  p.per_dn = du.per_dn;
  p.cols = du.cols;
  p.sk_rows = du.sk_rows;
  p.ks_dn = du.ks_dn;
  p.nk_dn = du.nk_dn;
  p.target = du.target;
  const int E = c->n_experts;
  auto kern = E <= 32 ? decode_plan_kernel<1> : E <= 64 ? decode_plan_kernel<2>
            : E <= 128 ? decode_plan_kernel<4> : E <= 256 ? decode_plan_kernel<8>
            : E <= 512 ? decode_plan_kernel<16> : decode_plan_kernel<32>;
  const size_t smem = decode_plan_smem(c);
  WB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  wb::launch_k_pdl(kern, 1, 1024, smem, st, p);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

WispError launch_pack(const uint16_t* x, const int* src, int n_rows, int M, uint16_t* xp,
                      cudaStream_t st, WispErrCtx* err) {
  if (n_rows <= 0) return WISP_OK;
  wb::launch_k(pack_rows_kernel, n_rows, 128, 0, st, x, src, n_rows, M, xp);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

}  // namespace wb

extern "C" WispError wisp_b200_pack_rows(const uint16_t* d_x, const int* d_src, int n_rows,
                                         int hidden, uint16_t* d_xp, cudaStream_t stream,
                                         WispErrCtx* err) {
  if (!d_x || !d_xp || hidden <= 0 || hidden % 8)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "pack_rows: bad arguments (hidden=%d)", hidden);
  if (((uintptr_t)d_x | (uintptr_t)d_xp) & 15)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "pack_rows: buffers must be 16-byte aligned");
  return wb::launch_pack(d_x, d_src, n_rows, hidden, d_xp, stream, err);
}

extern "C" WispError wisp_b200_dispatch_plan(const WispMoeConfig* cfg, const int* d_idx,
                                             const float* d_w, int* d_counts, WispSegment* d_segs,
                                             int* d_row_token, float* d_row_weight,
                                             cudaStream_t stream, WispErrCtx* err) {
  if (!cfg || !d_idx || !d_w || !d_counts || !d_segs || !d_row_token || !d_row_weight)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "dispatch_plan: null pointer argument");
  if (cfg->tokens <= 0 || cfg->top_k <= 0 || cfg->n_experts <= 0)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "dispatch_plan: tokens=%d top_k=%d n_experts=%d",
                   cfg->tokens, cfg->top_k, cfg->n_experts);
  return wb::launch_plan(cfg, d_idx, d_w, d_counts, d_segs, d_row_token, d_row_weight, stream, err,
                         nullptr);
}

extern "C" WispError wisp_b200_rms_rescale(const float* d_in, uint16_t* d_out, int tokens,
                                           int hidden, float eps, cudaStream_t stream,
                                           WispErrCtx* err) {
  if (!d_in || !d_out || tokens <= 0 || hidden <= 0)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "rms_rescale: bad arguments");
  wb::launch_k(rms_rescale_kernel, tokens, 256, 0, stream, d_in, d_out, hidden, eps);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

extern "C" WispError wisp_b200_combine_rows(const float* d_y, const int* d_row_token,
                                            const float* d_row_weight, int n_rows, int hidden,
                                            float* d_out, cudaStream_t stream, WispErrCtx* err) {
  if (n_rows < 0 || hidden <= 0 || (n_rows > 0 && (!d_y || !d_row_token || !d_row_weight || !d_out)))
    return WB_FAIL(WISP_ERR_INVALID_ARG, "combine_rows: bad arguments");
  if (n_rows == 0) return WISP_OK;
  wb::launch_k(combine_rows_kernel, n_rows, 256, 0, stream, d_y, d_row_token, d_row_weight, hidden,
               d_out);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}
