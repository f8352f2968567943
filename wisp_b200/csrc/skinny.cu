// skinny.cu -- grouped int4 expert FFN for small token groups (decode).
//
// When an expert sees a few tokens (batch decode: ~5 per expert in the
// 256-token / 384-expert configuration), the work per weight is one int4
// conversion plus a handful of multiply-adds, and the kernel's only job is
// to stream the packed weights at HBM speed. A tcgen05.mma (M=128, K=16)
// costs a fixed ~60-95 SM cycles whatever N <= 128 is (measured on B200), so
// at small N the 5th-generation path tops out far below HBM speed; this
// kernel feeds m16n8k16 tensor-core MMAs (~1.6 per cycle per SM) from
// registers instead.
//
// One persistent CTA per SM, warp-specialised:
//   warp 8      producer: per 256-K stage, one TMA box of packed nibbles per
//               128-row weight block (128 rows x 128 bytes, 128-byte
//               swizzle: a box row is one 128-byte request; narrower boxes
//               left the TMA unit, not HBM, as the limit), one TMA box per
//               64-K quarter of the unit's token rows (fp16, 128-byte
//               swizzle), and bulk copies of the stage's scales (and zero
//               points) from the prepared tile-transposed copy, into a
//               5-deep shared-memory ring (44 KB per stage, up to 160 KB of
//               weights in flight per SM: under full load a copy takes
//               several microseconds from issue to arrival, so the bytes in
//               flight per SM set the bandwidth). Units are looked up in a
//               shared-memory copy of the unit prefix; the next unit's
//               segment record is fetched one unit ahead.
//   warps 0-7   consumers, each with two 16-row MMA tiles. Per 64-K quarter
//               a warp reads its nibbles
//               (conflict-free 8-byte loads: MMA row g lives in box row
//               sigma(g) = 2(g%4) + g/4 (mod 8), so each half-warp's rows
//               fall in distinct swizzle chunks) and the tokens' B fragments
//               (conflict-free 16-byte loads), converts each 32-bit word of
//               nibbles to exact (n - 8) fp16 pairs, runs a 4-MMA chain, and
//               folds it into fp32 accumulators times the group's scale (and
//               adds the zero-point term). The stage is released once its
//               last quarter has been read; units of at most 8 tokens
//               read a whole stage into registers and release it at once.
//               (Sixteen one-tile warps, four per scheduler, measured
//               slower: every warp re-reads the token fragments.)
//
// Work unit = (segment, weight row block, chunk of up to 16 tokens, and for
// a weighted down projection with fewer than two units per SM a part of a K
// split, whose partial sums the epilogue adds atomically):
//   GATEUP: 128 intermediate rows i of gate and of up; warp w takes rows
//           16w..16w+15 of both -> h = silu(g) * u written to H (fp16,
//           interleaved K order).
//   DOWN:   256 output rows m (two 128-row blocks); warp w takes 32 rows ->
//           out[token] += w * y (mode 0, fp32 atomics) or y rows (mode 1).
// Chunks of one row block are consecutive units, so CTAs that run them at
// the same time share the weight tile through L2. Every token runs the same
// arithmetic in the same order whatever chunk it lands in, so a token's
// result does not depend on the batch around it. Segments larger than the
// routing threshold go to the tcgen05 kernel.
//
// Fragment mapping. m16n8k16 gives thread (g = lane/4, t = lane%4) the A
// pairs (row g, k 2t..2t+1), (row g+8, same), (row g, k 2t+8..2t+9),
// (row g+8, same) and the B pairs (k 2t..2t+1, col g), (k 2t+8..2t+9, col g).
// The logical k of one MMA may map to any physical K as long as A and B
// agree. Per 64-K quarter, thread t owns packed words 2t and 2t+1 (bytes
// 8t..8t+7); nib8_centered turns a word into the pairs (k0,k4) (k1,k5)
// (k2,k6) (k3,k7). MMA m (0..3) of the quarter takes word m/2 and pair p =
// 2(m&1) as its (2t,2t+1) slot and pair p+1 as its (2t+8,2t+9) slot. The
// activation rows are stored interleaved (within 8 K: 0,4,1,5,2,6,3,7), so
// pair q of word w is 32-bit element q of that word's 16 bytes: B slot 0 is
// element p and B slot 1 element p+1 of the same activation word.
#include "common.cuh"
#include "internal.h"

using namespace wb;

namespace {

constexpr int kCW = 8;                        // consumer warps, two 16-row tiles each
constexpr int kThreads = (kCW + 1) * 32;      // + one producer warp
constexpr int kStages = 5;
constexpr int kCols = 16;                     // tokens per unit
// Default routing threshold: segments of up to 16 rows run here, larger ones
// on the tcgen05 kernel (a larger segment costs this kernel one weight pass
// per 16-token chunk; measured crossover on B200: prefill-shaped layers run
// 1.5x faster at 16 than at 256, decode layers are within 3 %).
constexpr int kSkMaxRows = 16;
constexpr int kKS = 256;                      // K per stage
constexpr int kQ = kKS / 64;                  // 64-K quarters per stage
constexpr int kBoxRows = 128;
constexpr int kBoxBytes = kBoxRows * 128;     // one weight block of a stage
constexpr int kBQBytes = kCols * 128;         // one 64-K quarter of 16 token rows
constexpr int kScRun = 4 * kBoxRows * 2;      // up to 4 scale groups x 128 rows
// Stage layout (bytes): [weights 2 blocks][tokens 4 quarters]
// [scales 2 blocks][zeros 2 blocks]; the stage headers live apart, so a
// stage is a whole number of KB and every TMA box keeps 1024-byte alignment.
constexpr int kOffB = 2 * kBoxBytes;
constexpr int kOffS = kOffB + kQ * kBQBytes;
constexpr int kOffZ = kOffS + 2 * kScRun;
constexpr int kStageBytes = kOffZ + 2 * kScRun;
static_assert(kStageBytes % 1024 == 0, "stages must keep 1024-byte alignment");
constexpr int kMaxSegs = 1040;                // segments per launch (experts + shared)
constexpr int kMaxEntries = 1536;             // prepared expert entries
enum { SK_GATEUP = 0, SK_DOWN = 1 };
enum { HF_HZ0 = 1, HF_HZ1 = 2, HF_V1 = 4 };

struct __align__(16) StageHdr {
  int prow0;  // first activation row of the unit
  int n;      // tokens in the unit (1..16)
  int row0;   // first weight row of the unit
  int flags;  // HF_*: zero points of block 0 / 1, block 1 inside the matrix
  int kg0;    // first 256-K stage of the unit's K range
  int nst;    // stages in the unit (the whole K, or one part of a K split)
  int pad[2];
};

struct SkSmem {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  StageHdr hdr[kStages];
  int abort;
  int32_t units[kMaxSegs + 2];           // unit prefix per segment, then the K split
  uint32_t zbits[kMaxEntries * 3 / 32];  // zero-point flag per matrix entry
};

struct SkParams {
  CUtensorMap act_map[2];  // token rows, boxes {64 halves, 8/16 rows}, 128-byte swizzle
  const uint8_t* prepared;
  size_t p_maps_sk, p_zbits, p_scales, p_zeros, p_mat_sc_bytes;
  const WispSegment* segs;
  const int32_t* units;  // [0, S]: unit prefix per segment
  int nseg;
  int n_entries;
  int M, I, gs;
  __half* h_out;
  const int* row_token;
  const float* row_weight;
  float* out;
  int mode;
  int* error_flag;
  unsigned long long* counters;  // optional wait-cycle counters (diagnostics)
};

// Diagnostic counters (cycles summed over warps): consumers' waits for a
// full stage and their total time, the producer's waits for a free stage
// and its total time.
enum { SC_FULL_WAIT, SC_CONS_TOTAL, SC_EMPTY_WAIT, SC_PROD_TOTAL, SC_COUNT };

__device__ __forceinline__ void hmma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The same with a zero accumulator input (the first MMA of a chain).
__device__ __forceinline__ void hmma16816_z(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                            uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// Waits without the abort shortcut: used to let issued copies land before
// the CTA exits.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, long long limit) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - t0 > limit) return;
}

// Nibbles of one 16-row tile for one 64-K quarter: MMA rows g and g+8.
struct RawTile {
  uint2 w[2];  // [row g / g+8]
};

// Token words of one 64-K quarter: [word 2t / 2t+1][n8 tile].
template <int NT>
struct BQuarter {
  uint4 v[2][NT];
};

__device__ __forceinline__ uint32_t u4_get(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// acc[nt] += s * (A x B) for one 16-row tile over one 64-K quarter; scales
// of MMA rows g (sg) and g+8 (s8).
template <int NT>
__device__ __forceinline__ void tile_quarter(float (&acc)[2][4], const RawTile& w,
                                             const BQuarter<NT>& b, float sg, float s8) {
  __half2 ag[2][4], a8[2][4];
  nib8_centered(w.w[0].x, ag[0]);
  nib8_centered(w.w[0].y, ag[1]);
  nib8_centered(w.w[1].x, a8[0]);
  nib8_centered(w.w[1].y, a8[1]);
  float ct[NT][4];
#pragma unroll
  for (int m = 0; m < 4; m++) {
    const int wd = m >> 1, p = 2 * (m & 1);
    const uint32_t a0 = h22u(ag[wd][p]), a2 = h22u(ag[wd][p + 1]);
    const uint32_t a1 = h22u(a8[wd][p]), a3 = h22u(a8[wd][p + 1]);
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      if (m == 0)
        hmma16816_z(ct[nt], a0, a1, a2, a3, u4_get(b.v[wd][nt], p), u4_get(b.v[wd][nt], p + 1));
      else
        hmma16816(ct[nt], a0, a1, a2, a3, u4_get(b.v[wd][nt], p), u4_get(b.v[wd][nt], p + 1));
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    acc[nt][0] = fmaf(sg, ct[nt][0], acc[nt][0]);
    acc[nt][1] = fmaf(sg, ct[nt][1], acc[nt][1]);
    acc[nt][2] = fmaf(s8, ct[nt][2], acc[nt][2]);
    acc[nt][3] = fmaf(s8, ct[nt][3], acc[nt][3]);
  }
}

// Zero points: acc[row, col] += z[row] * sum_k x[col, k] over the 64-K
// quarter. xs[nt][j]: activation sum of column 2t+j of tile nt.
template <int NT>
__device__ __forceinline__ void quarter_sums(const BQuarter<NT>& b, float (&xs)[NT][2], int t) {
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    float s = 0.f;
#pragma unroll
    for (int wd = 0; wd < 2; wd++) {
      const uint4 v = b.v[wd][nt];
      const uint32_t e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float2 f = __half22float2(u2h2(e[i]));
        s += f.x + f.y;
      }
    }
    // the quad (same column g, t = 0..3) holds the 64 K of the quarter
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    // column 2t+j lives in quad 2t+j
    xs[nt][0] = __shfl_sync(0xffffffffu, s, (2 * t) * 4);
    xs[nt][1] = __shfl_sync(0xffffffffu, s, (2 * t + 1) * 4);
  }
}

template <int NT>
__device__ __forceinline__ void add_zeros(float (&acc)[2][4], const float (&xs)[NT][2], float zg,
                                          float z8) {
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    acc[nt][0] = fmaf(zg, xs[nt][0], acc[nt][0]);
    acc[nt][1] = fmaf(zg, xs[nt][1], acc[nt][1]);
    acc[nt][2] = fmaf(z8, xs[nt][0], acc[nt][2]);
    acc[nt][3] = fmaf(z8, xs[nt][1], acc[nt][3]);
  }
}

// MMA rows g and g+8 of a tile for 64-K quarter q: box rows ra (block ba)
// and rb (block bb), both = sigma(g) (mod 8). Thread t reads bytes
// 8t..8t+7 of the quarter's 32 bytes, i.e. 16-byte chunk 2q + t/2, stored at
// chunk ^ (row & 7).
__device__ __forceinline__ void load_tile(RawTile& r, const uint8_t* st, int ba, int ra, int bb,
                                          int rb, int q, int t) {
  const int off = (((2 * q + (t >> 1)) ^ (ra & 7)) << 4) + 8 * (t & 1);
  r.w[0] = *reinterpret_cast<const uint2*>(st + ba * kBoxBytes + ra * 128 + off);
  r.w[1] = *reinterpret_cast<const uint2*>(st + bb * kBoxBytes + rb * 128 + off);
}

// Scale (or zero point) of box row `row` of a block for scale group grp.
__device__ __forceinline__ float row_scale(const uint8_t* st, int off, int block, int grp,
                                           int row) {
  return __half2float(
      reinterpret_cast<const __half*>(st + off + block * kScRun)[grp * kBoxRows + row]);
}

// Token row r's 16-byte chunk c of a 64-K quarter: the 128-byte swizzle puts
// it at chunk c ^ (r & 7).
template <int NT>
__device__ __forceinline__ void load_b(BQuarter<NT>& b, const uint8_t* st, int q, int g, int t) {
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const int r = nt * 8 + g;
    const uint8_t* row = st + kOffB + q * kBQBytes + r * 128;
#pragma unroll
    for (int wd = 0; wd < 2; wd++)
      b.v[wd][nt] = *reinterpret_cast<const uint4*>(row + (((2 * t + wd) ^ (r & 7)) << 4));
  }
}

// ---------------------------------------------------------------------------
// Producer warp.
// ---------------------------------------------------------------------------
template <int MODE>
__device__ void sk_producer(const SkParams& p, uint8_t* ring, SkSmem* L, int total, int lane) {
  volatile int* abort = &L->abort;
  const int K = MODE == SK_GATEUP ? p.M : p.I;
  const int nk = (K + kKS - 1) / kKS;
  const int gpr = K / p.gs;
  const int ksplit = L->units[p.nseg + 1];
  if (lane < 2) tma_prefetch_desc(&p.act_map[lane]);
  int slot = 0, item = 0;
  uint32_t phase = 0;
  const long long t_start = p.counters ? clock64() : 0;
  long long wait_cycles = 0;
  bool ok = true;
  // Units are resolved from the shared-memory prefix; the segment record of
  // the next unit is requested one unit ahead so its latency hides behind
  // the current unit's stages.
  int seg = 0;
  while (L->units[seg + 1] <= (int)blockIdx.x) seg++;
  WispSegment sg_next = p.segs[seg];
  int seg_next = seg;
  for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
    const WispSegment sg = sg_next;
    seg = seg_next;
    const int un = u + gridDim.x;
    if (un < total) {
      while (L->units[seg_next + 1] <= un) seg_next++;
      sg_next = p.segs[seg_next];
    }
    const int chunks = (sg.rows + kCols - 1) / kCols;
    const int l = u - L->units[seg];
    // l = (row block * ksplit + K part) * chunks + chunk: the chunks of one
    // weight tile are consecutive units
    const int ch = l % chunks, rest = l / chunks;
    const int ks = rest % ksplit, rbk = rest / ksplit;
    const int kg0 = ks * nk / ksplit, kg1 = (ks + 1) * nk / ksplit;
    const int col0 = ch * kCols;
    const int n = min(kCols, sg.rows - col0);
    const int mi = n <= 8 ? 0 : 1;               // token box of 8 / 16 rows
    const uint32_t bq = (8u << mi) * 128;        // bytes of one token quarter box
    const int row0 = rbk * (MODE == SK_GATEUP ? kBoxRows : 2 * kBoxRows);
    const int row1 = MODE == SK_GATEUP ? row0 : row0 + kBoxRows;
    const bool v1 = MODE == SK_GATEUP || row1 < p.M;
    const int e0 = sg.expert * 3 + (MODE == SK_GATEUP ? 0 : 2);
    const int e1 = MODE == SK_GATEUP ? e0 + 1 : e0;
    const bool hz0 = (L->zbits[e0 >> 5] >> (e0 & 31)) & 1;
    const bool hz1 = v1 && ((L->zbits[e1 >> 5] >> (e1 & 31)) & 1);
    const CUtensorMap* map0 =
        reinterpret_cast<const CUtensorMap*>(p.prepared + p.p_maps_sk + (size_t)e0 * sizeof(CUtensorMap));
    const CUtensorMap* map1 =
        reinterpret_cast<const CUtensorMap*>(p.prepared + p.p_maps_sk + (size_t)e1 * sizeof(CUtensorMap));
    const size_t t0off = (size_t)(row0 / kBoxRows) * gpr * kBoxRows * 2;
    const size_t t1off = (size_t)(row1 / kBoxRows) * gpr * kBoxRows * 2;
    const uint8_t* sc0 = p.prepared + p.p_scales + (size_t)e0 * p.p_mat_sc_bytes + t0off;
    const uint8_t* sc1 = p.prepared + p.p_scales + (size_t)e1 * p.p_mat_sc_bytes + t1off;
    const uint8_t* zr0 = p.prepared + p.p_zeros + (size_t)e0 * p.p_mat_sc_bytes + t0off;
    const uint8_t* zr1 = p.prepared + p.p_zeros + (size_t)e1 * p.p_mat_sc_bytes + t1off;
    StageHdr hdr;
    hdr.prow0 = sg.row_begin + col0;
    hdr.n = n;
    hdr.row0 = row0;
    hdr.flags = (hz0 ? HF_HZ0 : 0) | (hz1 ? HF_HZ1 : 0) | (v1 ? HF_V1 : 0);
    hdr.kg0 = kg0;
    hdr.nst = kg1 - kg0;
    if (lane == 0) {
      tma_prefetch_desc(map0);
      if (MODE == SK_GATEUP) tma_prefetch_desc(map1);
    }
    for (int kg = kg0; kg < kg1; kg++, item++) {
      // quarters in this stage (the last one holds 2 when K % 256 == 128)
      const int nq = min(kQ, (K - kg * kKS) / 64);
      const uint32_t scb = (uint32_t)(nq * 64 / p.gs) * kBoxRows * 2;
      const uint32_t bytes = (v1 ? 2 : 1) * kBoxBytes + nq * bq +
                             scb * (1 + (v1 ? 1 : 0) + (hz0 ? 1 : 0) + (hz1 ? 1 : 0));
      if (lane == 0 && item >= kStages) {
        const long long tw = p.counters ? clock64() : 0;
        ok = mbar_wait(&L->empty[slot], phase ^ 1, abort);
        if (p.counters) wait_cycles += clock64() - tw;
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      uint8_t* st = ring + slot * kStageBytes;
      uint64_t* fb = &L->full[slot];
      if (lane == 0) {
        L->hdr[slot] = hdr;
        mbar_arrive_expect_tx(fb, bytes);
      }
      __syncwarp();
      const size_t goff = (size_t)(kg * kKS / p.gs) * kBoxRows * 2;
      if (lane < 2) {
        if (lane == 0 || v1)
          tma_load_2d(st + lane * kBoxBytes, lane ? map1 : map0, fb, kg * (kKS / 2),
                      lane ? row1 : row0);
      } else if (lane < 2 + kQ) {
        const int q = lane - 2;
        if (q < nq)
          tma_load_2d(st + kOffB + q * kBQBytes, &p.act_map[mi], fb, kg * kKS + q * 64, hdr.prow0);
      } else if (lane == 2 + kQ) {
        bulk_load(st + kOffS, sc0 + goff, scb, fb);
        if (v1) bulk_load(st + kOffS + kScRun, sc1 + goff, scb, fb);
      } else if (lane == 3 + kQ) {
        if (hz0) bulk_load(st + kOffZ, zr0 + goff, scb, fb);
        if (hz1) bulk_load(st + kOffZ + kScRun, zr1 + goff, scb, fb);
      }
      if (++slot == kStages) { slot = 0; phase ^= 1; }
    }
  }
  // Let every issued copy land before the CTA can exit: slot i was last
  // filled by item j = the largest j < item with j % kStages == i.
  if (lane == 0)
    for (int i = 0; i < kStages && i < item; i++) {
      const int j = i + (item - 1 - i) / kStages * kStages;
      drain_wait(&L->full[i], (uint32_t)((j / kStages) & 1), 200000000LL);
    }
  if (p.counters && lane == 0) {
    atomicAdd(p.counters + SC_EMPTY_WAIT, (unsigned long long)wait_cycles);
    atomicAdd(p.counters + SC_PROD_TOTAL, (unsigned long long)(clock64() - t_start));
  }
}

// One full stage for a unit of at most 8 tokens (the decode case): all of
// the warp's nibbles, token fragments and scales are read first and the
// stage is released before any conversion, so the producer can refill it
// while the MMAs run (G scale groups per 256-K stage). Per quarter and tile
// a 4-MMA chain (alternating register sets, so the next quarter's MMAs need
// not wait for this quarter's fold) is folded into the accumulator times its
// group's scale, then the zero-point term is added: the arithmetic, in the
// same order, of the general path in sk_unit, so a token's result does not
// depend on which path its unit took.
template <int G>
__device__ __forceinline__ void stage_single(float (&acc0)[2][4], float (&acc1)[2][4],
                                             const uint8_t* st, int b0, int b1, int r0, int r1,
                                             int g, int t, bool hz0, bool hz1, SkSmem* L, int slot,
                                             int lane) {
  constexpr int QPG = kQ / G;  // quarters per scale group
  RawTile w0[kQ], w1[kQ];
  BQuarter<1> bq[kQ];
#pragma unroll
  for (int q = 0; q < kQ; q++) {
    load_tile(w0[q], st, b0, r0, b0, r0 + 8, q, t);
    load_tile(w1[q], st, b1, r1, b1, r1 + 8, q, t);
    load_b<1>(bq[q], st, q, g, t);
  }
  // scales and zero points of MMA rows g (low half) and g+8 (high half)
  float2 s0[G], s1[G];
  __half2 z0[G], z1[G];
#pragma unroll
  for (int j = 0; j < G; j++) {
    s0[j] = make_float2(row_scale(st, kOffS, b0, j, r0), row_scale(st, kOffS, b0, j, r0 + 8));
    s1[j] = make_float2(row_scale(st, kOffS, b1, j, r1), row_scale(st, kOffS, b1, j, r1 + 8));
    z0[j] = hz0 ? __floats2half2_rn(row_scale(st, kOffZ, b0, j, r0), row_scale(st, kOffZ, b0, j, r0 + 8))
                : __half2{};
    z1[j] = hz1 ? __floats2half2_rn(row_scale(st, kOffZ, b1, j, r1), row_scale(st, kOffZ, b1, j, r1 + 8))
                : __half2{};
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(&L->empty[slot]);

  float c0[2][4], c1[2][4];
#pragma unroll
  for (int q = 0; q < kQ; q++) {
    const int j = q / QPG, ci = q & 1;
    __half2 ag0[2][4], a80[2][4], ag1[2][4], a81[2][4];
    nib8_centered(w0[q].w[0].x, ag0[0]);
    nib8_centered(w0[q].w[0].y, ag0[1]);
    nib8_centered(w0[q].w[1].x, a80[0]);
    nib8_centered(w0[q].w[1].y, a80[1]);
    nib8_centered(w1[q].w[0].x, ag1[0]);
    nib8_centered(w1[q].w[0].y, ag1[1]);
    nib8_centered(w1[q].w[1].x, a81[0]);
    nib8_centered(w1[q].w[1].y, a81[1]);
#pragma unroll
    for (int m = 0; m < 4; m++) {
      const int wd = m >> 1, pp = 2 * (m & 1);
      const uint32_t b0v = u4_get(bq[q].v[wd][0], pp), b1v = u4_get(bq[q].v[wd][0], pp + 1);
      if (m == 0) {
        hmma16816_z(c0[ci], h22u(ag0[wd][pp]), h22u(a80[wd][pp]), h22u(ag0[wd][pp + 1]),
                    h22u(a80[wd][pp + 1]), b0v, b1v);
        hmma16816_z(c1[ci], h22u(ag1[wd][pp]), h22u(a81[wd][pp]), h22u(ag1[wd][pp + 1]),
                    h22u(a81[wd][pp + 1]), b0v, b1v);
      } else {
        hmma16816(c0[ci], h22u(ag0[wd][pp]), h22u(a80[wd][pp]), h22u(ag0[wd][pp + 1]),
                  h22u(a80[wd][pp + 1]), b0v, b1v);
        hmma16816(c1[ci], h22u(ag1[wd][pp]), h22u(a81[wd][pp]), h22u(ag1[wd][pp + 1]),
                  h22u(a81[wd][pp + 1]), b0v, b1v);
      }
    }
    const float2 f0 = s0[j], f1 = s1[j];
    acc0[0][0] = fmaf(f0.x, c0[ci][0], acc0[0][0]);
    acc0[0][1] = fmaf(f0.x, c0[ci][1], acc0[0][1]);
    acc0[0][2] = fmaf(f0.y, c0[ci][2], acc0[0][2]);
    acc0[0][3] = fmaf(f0.y, c0[ci][3], acc0[0][3]);
    acc1[0][0] = fmaf(f1.x, c1[ci][0], acc1[0][0]);
    acc1[0][1] = fmaf(f1.x, c1[ci][1], acc1[0][1]);
    acc1[0][2] = fmaf(f1.y, c1[ci][2], acc1[0][2]);
    acc1[0][3] = fmaf(f1.y, c1[ci][3], acc1[0][3]);
    if (hz0 | hz1) {
      float xs[1][2];
      quarter_sums<1>(bq[q], xs, t);
      const float2 g0 = __half22float2(z0[j]), g1 = __half22float2(z1[j]);
      if (hz0) add_zeros<1>(acc0, xs, g0.x, g0.y);
      if (hz1) add_zeros<1>(acc1, xs, g1.x, g1.y);
    }
  }
}

// ---------------------------------------------------------------------------
// Consumer warps: one unit with NT n8 token tiles.
// ---------------------------------------------------------------------------
template <int MODE, int NT>
__device__ bool sk_unit(const SkParams& p, uint8_t* ring, SkSmem* L, const StageHdr& hdr,
                        int warp, int lane, int& slot, uint32_t& phase,
                        long long& wait_cycles) {
  volatile int* abort = &L->abort;
  const int g = lane >> 2, t = lane & 3;
  const int sig = ((g & 3) << 1) | (g >> 2);  // box row (mod 8) of MMA row g
  const int K = MODE == SK_GATEUP ? p.M : p.I;
  const int qpg = p.gs / 64;  // quarters per scale group (1 or 2)
  // Two tiles per warp; a tile's MMA rows g and g+8 are box rows r and r+8.
  // GATEUP: gate rows 16w + sig (block 0) and the same up rows (block 1);
  // DOWN: rows 32(w%4) + sig and +16 of block w/4.
  const int b0 = MODE == SK_GATEUP ? 0 : warp >> 2;
  const int b1 = MODE == SK_GATEUP ? 1 : warp >> 2;
  const int r0 = (MODE == SK_GATEUP ? 16 * warp : 32 * (warp & 3)) + sig;
  const int r1 = MODE == SK_GATEUP ? r0 : r0 + 16;
  const bool active = MODE == SK_GATEUP || b0 == 0 || (hdr.flags & HF_V1);
  const bool hz0 = hdr.flags & (b0 ? HF_HZ1 : HF_HZ0);
  const bool hz1 = hdr.flags & (b1 ? HF_HZ1 : HF_HZ0);

  float acc0[2][4], acc1[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; nt++)
#pragma unroll
    for (int e = 0; e < 4; e++) acc0[nt][e] = acc1[nt][e] = 0.f;

  // The down epilogue's token indices and router weights, requested now so
  // that their latency hides behind the unit's stages.
  int tok[NT][2];
  float wgt[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int col = nt * 8 + 2 * t + j;
      const bool need = MODE == SK_DOWN && p.mode == 0 && active && col < hdr.n;
      tok[nt][j] = need ? __ldg(p.row_token + hdr.prow0 + col) : 0;
      wgt[nt][j] = need ? __ldg(p.row_weight + hdr.prow0 + col) : 0.f;
    }

  for (int kk = 0; kk < hdr.nst; kk++) {
    if (kk > 0) {
      const long long tw = p.counters ? clock64() : 0;
      if (!mbar_wait(&L->full[slot], phase, abort)) return false;
      if (p.counters) wait_cycles += clock64() - tw;
    }
    const uint8_t* st = ring + slot * kStageBytes;
    const int nq = min(kQ, (K - (hdr.kg0 + kk) * kKS) / 64);
    if (active && NT == 1 && nq == kQ) {
      if (p.gs == 128)
        stage_single<2>(acc0, acc1, st, b0, b1, r0, r1, g, t, hz0, hz1, L, slot, lane);
      else
        stage_single<4>(acc0, acc1, st, b0, b1, r0, r1, g, t, hz0, hz1, L, slot, lane);
    } else if (active) {
#pragma unroll
      for (int q = 0; q < kQ; q++) {
        if (q < nq) {
          RawTile w0, w1;
          load_tile(w0, st, b0, r0, b0, r0 + 8, q, t);
          load_tile(w1, st, b1, r1, b1, r1 + 8, q, t);
          BQuarter<NT> bq;
          load_b<NT>(bq, st, q, g, t);
          const int grp = q / qpg;
          const float sa = row_scale(st, kOffS, b0, grp, r0), sb = row_scale(st, kOffS, b0, grp, r0 + 8);
          const float sc = row_scale(st, kOffS, b1, grp, r1), sd = row_scale(st, kOffS, b1, grp, r1 + 8);
          const float za = hz0 ? row_scale(st, kOffZ, b0, grp, r0) : 0.f;
          const float zb = hz0 ? row_scale(st, kOffZ, b0, grp, r0 + 8) : 0.f;
          const float zc = hz1 ? row_scale(st, kOffZ, b1, grp, r1) : 0.f;
          const float zd = hz1 ? row_scale(st, kOffZ, b1, grp, r1 + 8) : 0.f;
          if (q == nq - 1) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&L->empty[slot]);
          }
          tile_quarter<NT>(acc0, w0, bq, sa, sb);
          tile_quarter<NT>(acc1, w1, bq, sc, sd);
          if (hz0 | hz1) {
            float xs[NT][2];
            quarter_sums<NT>(bq, xs, t);
            if (hz0) add_zeros<NT>(acc0, xs, za, zb);
            if (hz1) add_zeros<NT>(acc1, xs, zc, zd);
          }
        }
      }
    } else {
      __syncwarp();
      if (lane == 0) mbar_arrive(&L->empty[slot]);
    }
    if (++slot == kStages) { slot = 0; phase ^= 1; }
  }
  if (!active) return true;

  // Epilogue. acc[nt][0..1]: MMA row g (box row r), columns 2t, 2t+1;
  // [2..3]: MMA row g+8 (box row r+8).
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int j = e & 1, col = nt * 8 + 2 * t + j;
      if (col >= hdr.n) continue;
      const int rr = (e >> 1) ? 8 : 0;
      const int prow = hdr.prow0 + col;
      if (MODE == SK_GATEUP) {
        const int i = hdr.row0 + r0 + rr;
        const float hv = silu(acc0[nt][e]) * acc1[nt][e];
        p.h_out[(size_t)prow * p.I + k_interleave_slot(i)] = __float2half(hv);
      } else {
        const int base = hdr.row0 + b0 * kBoxRows;
        const int ma = base + r0 + rr, mb = base + r1 + rr;
        const float y0 = acc0[nt][e], y1 = acc1[nt][e];
        if (p.mode == 0) {
          red_add_f32(p.out + (size_t)tok[nt][j] * p.M + ma, wgt[nt][j] * y0);
          red_add_f32(p.out + (size_t)tok[nt][j] * p.M + mb, wgt[nt][j] * y1);
        } else {
          p.out[(size_t)prow * p.M + ma] = y0;
          p.out[(size_t)prow * p.M + mb] = y1;
        }
      }
    }
  }
  return true;
}

template <int MODE>
__device__ void sk_consumer(const SkParams& p, uint8_t* ring, SkSmem* L, int total, int warp,
                            int lane) {
  volatile int* abort = &L->abort;
  int slot = 0;
  uint32_t phase = 0;
  const long long t_start = p.counters ? clock64() : 0;
  long long wait_cycles = 0;
  for (int u = blockIdx.x; u < total; u += gridDim.x) {
    const long long tw = p.counters ? clock64() : 0;
    if (!mbar_wait(&L->full[slot], phase, abort)) return;
    if (p.counters) wait_cycles += clock64() - tw;
    const StageHdr hdr = L->hdr[slot];
    bool ok;
    if (hdr.n <= 8) ok = sk_unit<MODE, 1>(p, ring, L, hdr, warp, lane, slot, phase, wait_cycles);
    else ok = sk_unit<MODE, 2>(p, ring, L, hdr, warp, lane, slot, phase, wait_cycles);
    if (!ok) return;
  }
  if (p.counters && lane == 0) {
    atomicAdd(p.counters + SC_FULL_WAIT, (unsigned long long)wait_cycles);
    atomicAdd(p.counters + SC_CONS_TOTAL, (unsigned long long)(clock64() - t_start));
  }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) skinny_ffn_kernel(const __grid_constant__ SkParams p) {
  extern __shared__ uint8_t smem_raw[];
  const int total = __ldg(p.units + p.nseg);
  if ((int)blockIdx.x >= total) return;
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  SkSmem* L = reinterpret_cast<SkSmem*>(ring + kStages * kStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; i++) {
      mbar_init(&L->full[i], 1);
      mbar_init(&L->empty[i], kCW);
    }
    L->abort = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i <= p.nseg + 1; i += blockDim.x) L->units[i] = __ldg(p.units + i);
  const uint32_t* zb = reinterpret_cast<const uint32_t*>(p.prepared + p.p_zbits);
  for (int w = threadIdx.x; w < (p.n_entries * 3 + 31) / 32; w += blockDim.x) L->zbits[w] = __ldg(zb + w);
  __syncthreads();
  if (warp == kCW)
    sk_producer<MODE>(p, ring, L, total, lane);
  else
    sk_consumer<MODE>(p, ring, L, total, warp, lane);
  __syncthreads();
  if (threadIdx.x == 0 && L->abort && p.error_flag) atomicExch(p.error_flag, 1);
}

constexpr size_t kSmemBytes = 1024 + (size_t)kStages * kStageBytes + sizeof(SkSmem);
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

}  // namespace

namespace wb {

struct SkLaunch {
  const uint8_t* prepared;
  size_t p_maps_sk, p_zbits, p_scales, p_zeros, p_mat_sc_bytes;
  const WispSegment* segs;
  int nseg;
  int n_entries;
  const int32_t* units_gu;
  const int32_t* units_dn;
  int M, I, gs;
  const CUtensorMap* xp_maps;  // [2]: boxes of 8 / 16 rows
  const CUtensorMap* h_maps;   // [2]
  __half* h;
  const int* row_token;
  const float* row_weight;
  float* out;
  int mode;
  int* error_flag;
  unsigned long long* counters;
};  // mirrored in grouped.cu

int skinny_max_rows() { return kSkMaxRows; }
int skinny_max_segs() { return kMaxSegs; }
int skinny_max_entries() { return kMaxEntries; }
int skinny_cols() { return kCols; }
int skinny_stages(int K) { return (K + kKS - 1) / kKS; }
int skinny_units_gateup(int I) { return I / kBoxRows; }
int skinny_units_down(int M) { return (M + 2 * kBoxRows - 1) / (2 * kBoxRows); }

cudaError_t launch_skinny(const SkLaunch& L, int phase, int grid, cudaStream_t st) {
  // The attribute belongs to the current device's context: set it per launch.
  cudaError_t ce = phase == 0
      ? cudaFuncSetAttribute(skinny_ffn_kernel<SK_GATEUP>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes)
      : cudaFuncSetAttribute(skinny_ffn_kernel<SK_DOWN>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (ce != cudaSuccess) return ce;
  SkParams p;
  memset(&p, 0, sizeof p);
  p.prepared = L.prepared;
  p.p_maps_sk = L.p_maps_sk;
  p.p_zbits = L.p_zbits;
  p.p_scales = L.p_scales;
  p.p_zeros = L.p_zeros;
  p.p_mat_sc_bytes = L.p_mat_sc_bytes;
  p.segs = L.segs;
  p.nseg = L.nseg;
  p.n_entries = L.n_entries;
  p.M = L.M;
  p.I = L.I;
  p.gs = L.gs;
  p.h_out = L.h;
  p.row_token = L.row_token;
  p.row_weight = L.row_weight;
  p.out = L.out;
  p.mode = L.mode;
  p.error_flag = L.error_flag;
  p.counters = L.counters ? L.counters + phase * SC_COUNT : nullptr;
  const CUtensorMap* maps = phase == 0 ? L.xp_maps : L.h_maps;
  for (int i = 0; i < 2; i++) p.act_map[i] = maps[i];
  if (phase == 0) {
    p.units = L.units_gu;
    wb::launch_k(skinny_ffn_kernel<SK_GATEUP>, grid, kThreads, kSmemBytes, st, p);
  } else {
    p.units = L.units_dn;
    wb::launch_k(skinny_ffn_kernel<SK_DOWN>, grid, kThreads, kSmemBytes, st, p);
  }
  return cudaGetLastError();
}

}  // namespace wb
