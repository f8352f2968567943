// skinny.cu -- grouped int4 expert FFN for small token groups (decode).
//
// When an expert sees at most 16 tokens (batch decode: ~5 per expert in the
// 256-token / 384-expert configuration), the work per weight is one int4
// conversion plus a handful of multiply-adds. A tcgen05.mma (M=128, K=16)
// costs a fixed ~60-95 SM cycles whatever N <= 128 is (measured on B200), so
// at N <= 16 the 5th-generation path tops out near 2048 weights per ~60
// cycles per SM. This kernel keeps the dequantised operand in registers:
// every warp streams its own weight rows from HBM, converts each 32-bit word
// of nibbles to exact (n - 8) fp16 pairs, and feeds them as A fragments to
// m16n8k16 tensor-core MMAs (~1.6 per cycle per SM) against the tokens' B
// fragments, accumulating fp32 per 64-K half group and applying the group's
// scale (and zero point) to the fp32 partial sums. No shared memory, no
// cross-warp synchronisation.
//
// Work unit = (segment, row block); 4 warps per unit:
//   GATEUP: 64 intermediate rows i, each warp 16 gate rows + the same 16 up
//           rows -> h = silu(g) * u written to H (fp16, interleaved K order).
//   DOWN:   128 output rows m, each warp 32 rows -> out[token] += w * y
//           (mode 0, fp32 atomics) or y rows (mode 1).
// Segments with more than 16 rows are left to the tcgen05 kernel.
//
// Fragment mapping. m16n8k16 gives thread (g = lane/4, t = lane%4) the A
// pairs (row g, k 2t..2t+1), (row g+8, same), (row g, k 2t+8..2t+9),
// (row g+8, same) and the B pairs (k 2t..2t+1, col g), (k 2t+8..2t+9, col g).
// The logical k of one MMA may map to any physical K as long as A and B
// agree. Per 64-K half group, thread t owns packed words 2t and 2t+1 (bytes
// 8t..8t+7); nib8_centered turns a word into the pairs (k0,k4) (k1,k5)
// (k2,k6) (k3,k7). MMA m (0..3) of the half takes word m/2 and pair p =
// 2(m&1) as its (2t,2t+1) slot and pair p+1 as its (2t+8,2t+9) slot. The
// activation rows are stored interleaved (within 8 K: 0,4,1,5,2,6,3,7), so
// pair q of word w is 32-bit element q of that word's 16 bytes: B slot 0 is
// element p and B slot 1 element p+1 of the same activation word.
#include "common.cuh"
#include "internal.h"

using namespace wb;

namespace {

constexpr int kSkMaxRows = 16;
constexpr int kSkWarps = 4;
enum { SK_GATEUP = 0, SK_DOWN = 1 };

struct SkParams {
  const uint8_t* prepared;
  size_t p_flags, p_scales, p_zeros, p_mat_sc_bytes;
  const WispInt4Expert* experts;   // packed nibble pointers
  const WispSegment* segs;
  const int32_t* units;            // [0,S]: unit prefix (no units for large segments)
  int nseg;
  int M, I, gs;
  const __half* act;               // GATEUP: Xp rows [R x M]; DOWN: H rows [R x I]
  __half* h_out;                   // GATEUP output
  const int* row_token;
  const float* row_weight;
  float* out;
  int mode;
};

__device__ __forceinline__ void hmma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint2 ldg_stream_64(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

__device__ __forceinline__ int find_seg(const int32_t* pre, int nseg, int unit) {
  int lo = 0, hi = nseg - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(pre + mid) <= unit) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// The packed words of one 16-row tile this thread needs for one 128-K group:
// rows g and g+8, both 64-K halves (2 words each).
struct RawTile {
  uint2 w[2][2];  // [half][row g / g+8]
};

__device__ __forceinline__ void load_tile(RawTile& r, const uint8_t* packed, int row0,
                                          int kbytes_row, int kg, int g, int t) {
  const uint8_t* p0 = packed + (size_t)(row0 + g) * kbytes_row + kg * 64 + 8 * t;
  const uint8_t* p8 = p0 + (size_t)8 * kbytes_row;
  r.w[0][0] = ldg_stream_64(p0);
  r.w[0][1] = ldg_stream_64(p8);
  r.w[1][0] = ldg_stream_64(p0 + 32);
  r.w[1][1] = ldg_stream_64(p8 + 32);
}

// Activation words of one 128-K group for token column g of each n8 tile:
// [half][word 2t / 2t+1][nt]; zero for columns beyond the segment.
template <int NT>
struct BFrag {
  uint4 v[2][2][NT];
};

template <int NT>
__device__ __forceinline__ void load_b(BFrag<NT>& b, const __half* const (&rows)[NT],
                                       const bool (&valid)[NT], int kg, int t) {
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const uint4* src = reinterpret_cast<const uint4*>(rows[nt] + kg * 128 + h * 64 + 16 * t);
      b.v[h][0][nt] = valid[nt] ? __ldg(src) : make_uint4(0, 0, 0, 0);
      b.v[h][1][nt] = valid[nt] ? __ldg(src + 1) : make_uint4(0, 0, 0, 0);
    }
  }
}

__device__ __forceinline__ uint32_t u4_get(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// acc[nt] += s * (A x B) for one 16-row tile over one 128-K group; scales
// per half group and row (g, g+8).
template <int NT>
__device__ __forceinline__ void tile_group(float (&acc)[NT][4], const RawTile& w,
                                           const BFrag<NT>& b, const float (&sg)[2],
                                           const float (&s8)[2]) {
#pragma unroll
  for (int h = 0; h < 2; h++) {
    __half2 ag[2][4], a8[2][4];
    nib8_centered(w.w[h][0].x, ag[0]);
    nib8_centered(w.w[h][0].y, ag[1]);
    nib8_centered(w.w[h][1].x, a8[0]);
    nib8_centered(w.w[h][1].y, a8[1]);
    float ct[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int q = 0; q < 4; q++) ct[nt][q] = 0.f;
#pragma unroll
    for (int m = 0; m < 4; m++) {
      const int wd = m >> 1, p = 2 * (m & 1);
      const uint32_t a0 = h22u(ag[wd][p]), a2 = h22u(ag[wd][p + 1]);
      const uint32_t a1 = h22u(a8[wd][p]), a3 = h22u(a8[wd][p + 1]);
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
        hmma16816(ct[nt], a0, a1, a2, a3, u4_get(b.v[h][wd][nt], p), u4_get(b.v[h][wd][nt], p + 1));
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      acc[nt][0] = fmaf(sg[h], ct[nt][0], acc[nt][0]);
      acc[nt][1] = fmaf(sg[h], ct[nt][1], acc[nt][1]);
      acc[nt][2] = fmaf(s8[h], ct[nt][2], acc[nt][2]);
      acc[nt][3] = fmaf(s8[h], ct[nt][3], acc[nt][3]);
    }
  }
}

// Zero points: acc[row, col] += z[row] * sum_k x[col, k] over each half
// group. xs[h][nt][j]: activation sum of column 2t+j of tile nt.
template <int NT>
__device__ __forceinline__ void half_sums(const BFrag<NT>& b, float (&xs)[2][NT][2], int t) {
#pragma unroll
  for (int h = 0; h < 2; h++)
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      float s = 0.f;
#pragma unroll
      for (int wd = 0; wd < 2; wd++) {
        const uint4 v = b.v[h][wd][nt];
        const uint32_t e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float2 f = __half22float2(u2h2(e[i]));
          s += f.x + f.y;
        }
      }
      // the quad (same column g, t = 0..3) holds the 64 K of the half
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      // column 2t+j lives in quad 2t+j
      xs[h][nt][0] = __shfl_sync(0xffffffffu, s, (2 * t) * 4);
      xs[h][nt][1] = __shfl_sync(0xffffffffu, s, (2 * t + 1) * 4);
    }
}

template <int NT>
__device__ __forceinline__ void add_zeros(float (&acc)[NT][4], const float (&xs)[2][NT][2],
                                          const float (&zg)[2], const float (&z8)[2]) {
#pragma unroll
  for (int h = 0; h < 2; h++)
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      acc[nt][0] = fmaf(zg[h], xs[h][nt][0], acc[nt][0]);
      acc[nt][1] = fmaf(zg[h], xs[h][nt][1], acc[nt][1]);
      acc[nt][2] = fmaf(z8[h], xs[h][nt][0], acc[nt][2]);
      acc[nt][3] = fmaf(z8[h], xs[h][nt][1], acc[nt][3]);
    }
}

// Scale (or zero point) of rows (row, row+8) for both half groups of group kg,
// from the prepared tile-transposed copy [tile][group][128 rows].
__device__ __forceinline__ void group_scales(const __half* st, int gpr, int gs, int row, int kg,
                                             float (&a)[2], float (&b)[2]) {
  const int tile = row >> 7, r = row & 127;
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int grp = (kg * 128 + h * 64) / gs;
    const __half* base = st + ((size_t)tile * gpr + grp) * 128;
    a[h] = __half2float(base[r]);
    b[h] = __half2float(base[r + 8]);
  }
}

template <int MODE, int NT>
__device__ void sk_unit(const SkParams& p, const WispSegment& sg, int rb, int warp, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const int K = MODE == SK_GATEUP ? p.M : p.I;
  const int ngroups = K / 128;
  const int gpr = K / p.gs;
  const int kbytes_row = K / 2;
  const int n = sg.rows;
  const WispInt4Expert ex = p.experts[sg.expert];
  const int32_t* flags = reinterpret_cast<const int32_t*>(p.prepared + p.p_flags);
  const int e3 = sg.expert * 3;

  const __half* rows[NT];
  bool valid[NT];
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const int tok = nt * 8 + g;
    valid[nt] = tok < n;
    rows[nt] = p.act + (size_t)(sg.row_begin + (valid[nt] ? tok : 0)) * K;
  }

  // Two 16-row tiles per warp: GATEUP: (gate, up) of rows i0..i0+15;
  // DOWN: rows m0..m0+15 and m0+16..m0+31.
  const int r0 = MODE == SK_GATEUP ? rb * 64 + warp * 16 : rb * 128 + warp * 32;
  const int r1 = MODE == SK_GATEUP ? r0 : r0 + 16;
  const uint8_t* pk0 = MODE == SK_GATEUP ? ex.gate.packed : ex.down.packed;
  const uint8_t* pk1 = MODE == SK_GATEUP ? ex.up.packed : ex.down.packed;
  const int m0 = MODE == SK_GATEUP ? 0 : 2, m1 = MODE == SK_GATEUP ? 1 : 2;
  const __half* sc0 = reinterpret_cast<const __half*>(p.prepared + p.p_scales + (size_t)(e3 + m0) * p.p_mat_sc_bytes);
  const __half* sc1 = reinterpret_cast<const __half*>(p.prepared + p.p_scales + (size_t)(e3 + m1) * p.p_mat_sc_bytes);
  const bool hz0 = __ldg(flags + e3 + m0) & 1, hz1 = __ldg(flags + e3 + m1) & 1;
  const __half* zr0 = reinterpret_cast<const __half*>(p.prepared + p.p_zeros + (size_t)(e3 + m0) * p.p_mat_sc_bytes);
  const __half* zr1 = reinterpret_cast<const __half*>(p.prepared + p.p_zeros + (size_t)(e3 + m1) * p.p_mat_sc_bytes);

  float acc0[NT][4], acc1[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int q = 0; q < 4; q++) acc0[nt][q] = acc1[nt][q] = 0.f;

  RawTile nx0, nx1;
  load_tile(nx0, pk0, r0, kbytes_row, 0, g, t);
  load_tile(nx1, pk1, r1, kbytes_row, 0, g, t);
  for (int kg = 0; kg < ngroups; kg++) {
    const RawTile w0 = nx0, w1 = nx1;
    if (kg + 1 < ngroups) {
      load_tile(nx0, pk0, r0, kbytes_row, kg + 1, g, t);
      load_tile(nx1, pk1, r1, kbytes_row, kg + 1, g, t);
    }
    BFrag<NT> b;
    load_b<NT>(b, rows, valid, kg, t);
    float sa[2], sb[2], sc[2], sd[2];
    group_scales(sc0, gpr, p.gs, r0 + g, kg, sa, sb);
    group_scales(sc1, gpr, p.gs, r1 + g, kg, sc, sd);
    tile_group<NT>(acc0, w0, b, sa, sb);
    tile_group<NT>(acc1, w1, b, sc, sd);
    if (hz0 | hz1) {
      float xs[2][NT][2];
      half_sums<NT>(b, xs, t);
      if (hz0) {
        float za[2], zb[2];
        group_scales(zr0, gpr, p.gs, r0 + g, kg, za, zb);
        add_zeros<NT>(acc0, xs, za, zb);
      }
      if (hz1) {
        float za[2], zb[2];
        group_scales(zr1, gpr, p.gs, r1 + g, kg, za, zb);
        add_zeros<NT>(acc1, xs, za, zb);
      }
    }
  }

  // Epilogue. acc[nt][0..1]: row g, columns 2t, 2t+1; [2..3]: row g+8.
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int col = nt * 8 + 2 * t + (q & 1);
      if (col >= n) continue;
      const int rr = (q >> 1) ? 8 : 0;
      const int prow = sg.row_begin + col;
      if (MODE == SK_GATEUP) {
        const int i = r0 + g + rr;
        const float hv = silu(acc0[nt][q]) * acc1[nt][q];
        p.h_out[(size_t)prow * p.I + k_interleave_slot(i)] = __float2half(hv);
      } else {
        const float y0 = acc0[nt][q], y1 = acc1[nt][q];
        const int ma = r0 + g + rr, mb = r1 + g + rr;
        if (p.mode == 0) {
          const int tok = __ldg(p.row_token + prow);
          const float wgt = __ldg(p.row_weight + prow);
          red_add_f32(p.out + (size_t)tok * p.M + ma, wgt * y0);
          red_add_f32(p.out + (size_t)tok * p.M + mb, wgt * y1);
        } else {
          p.out[(size_t)prow * p.M + ma] = y0;
          p.out[(size_t)prow * p.M + mb] = y1;
        }
      }
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(kSkWarps * 32, 4) skinny_ffn_kernel(const __grid_constant__ SkParams p) {
  const int total = __ldg(p.units + p.nseg);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int unit = blockIdx.x; unit < total; unit += gridDim.x) {
    const int s = find_seg(p.units, p.nseg, unit);
    const int rb = unit - __ldg(p.units + s);
    const WispSegment sg = p.segs[s];
    if (sg.rows > 8)
      sk_unit<MODE, 2>(p, sg, rb, warp, lane);
    else
      sk_unit<MODE, 1>(p, sg, rb, warp, lane);
  }
}

}  // namespace

namespace wb {

struct SkLaunch {
  const uint8_t* prepared;
  size_t p_flags, p_scales, p_zeros, p_mat_sc_bytes;
  const WispInt4Expert* experts;
  const WispSegment* segs;
  int nseg;
  const int32_t* units_gu;
  const int32_t* units_dn;
  int M, I, gs;
  const __half* xp;
  __half* h;
  const int* row_token;
  const float* row_weight;
  float* out;
  int mode;
};  // mirrored in grouped.cu

int skinny_max_rows() { return kSkMaxRows; }

void launch_skinny(const SkLaunch& L, int phase, cudaStream_t st) {
  SkParams p;
  p.prepared = L.prepared;
  p.p_flags = L.p_flags;
  p.p_scales = L.p_scales;
  p.p_zeros = L.p_zeros;
  p.p_mat_sc_bytes = L.p_mat_sc_bytes;
  p.experts = L.experts;
  p.segs = L.segs;
  p.nseg = L.nseg;
  p.M = L.M;
  p.I = L.I;
  p.gs = L.gs;
  p.h_out = L.h;
  p.row_token = L.row_token;
  p.row_weight = L.row_weight;
  p.out = L.out;
  p.mode = L.mode;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = sms * 4;
  if (phase == 0) {
    p.units = L.units_gu;
    p.act = L.xp;
    skinny_ffn_kernel<SK_GATEUP><<<grid, kSkWarps * 32, 0, st>>>(p);
  } else {
    p.units = L.units_dn;
    p.act = L.h;
    skinny_ffn_kernel<SK_DOWN><<<grid, kSkWarps * 32, 0, st>>>(p);
  }
}

}  // namespace wb
