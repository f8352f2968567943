// grouped.cu -- grouped int4 expert FFN on the 5th-generation tensor cores.
//
// Replaces, for batched and prefill tokens, the reference's per-token loop
// of dequant -> fp16 GEMV -> scale_accum (csrc/core/wisp_engine.c:1507-1531
// called from run_moe :1563-1674 and, for prefill, decode_step per token
// :2292-2307). Rows of activations are pre-grouped by expert ("segments");
// the kernel runs as persistent pairs of CTAs (clusters of 2) whose tiles
// compute 256 weight rows (the pair MMA's M; 128 per CTA, one TMEM lane
// each) x BN token rows (its N):
//
//   GATEUP: H[p, i] = silu(gate[i] . x_p) * (up[i] . x_p)   (fp16 H out)
//           over 128 intermediate rows, 64 per CTA: in a CTA, A rows
//           16j..16j+7 are gate rows 8j..8j+7 of its block, A rows
//           16j+8..16j+15 the matching up rows, so a gate lane's partner is
//           lane ^ 8 of the same warp.
//   DOWN:   out[token(p), m] += w_p * (down[m] . H_p)        (fp32 atomics)
//           or y[p, m] = down[m] . H_p                        (mode 1)
//
// BN is chosen per segment: the fewest tiles of at most 192 rows, each a
// multiple of 32 (an M=128 tcgen05.mma costs ~96 SM cycles at N=128 and
// ~141 at N=256 on B200, so wide tiles use the tensor pipe best; the cap
// leaves room for two accumulators). The pair MMA (cta_group::2, issued by
// the even CTA) reads each CTA's A from its own tensor memory and the token
// rows half from each CTA's shared memory, so every SM loads half of a
// tile's activations and one issuing thread drives two tensor cores. Roles
// inside each CTA:
//   warp 26     weight producer: per 128-K raw stage, one TMA box of this
//               CTA's packed nibbles per matrix (64 or 128 rows x 64 bytes,
//               64-byte swizzle) and bulk copies of the scales (and zero
//               points) of the stage's groups from the prepared copy.
//   warps 0-15  dequantise: warp w converts, for TMEM lane quadrant w % 4,
//               32 K of every other A stage (64 K) -- one 16-byte read of its
//               row from the raw stage, (n-8)*s + z in fp16 with one
//               rounding, written straight into tensor memory with
//               tcgen05.st -- and reports the stage to the even CTA's
//               barrier as soon as the store has completed.
//   warp 24     TMA producer for this CTA's half of the activation rows
//               (128-byte swizzle), one A stage per ring slot.
//   warp 25     even CTA: MMA issuer (tcgen05.mma kind::f16, A from TMEM, B
//               from smem, fp32 accumulators in TMEM; tcgen05.commit
//               multicast to both CTAs' barriers). Odd CTA: forwards each
//               landed activation stage to the even CTA's barrier.
//   warps 16-23 epilogue, two warps per lane quadrant (alternate 16- or
//               32-column chunks): tcgen05.ld of the accumulators, SwiGLU
//               (GATEUP) or the weighted scatter-combine (DOWN).
// TMEM columns (the same in both CTAs): [0,192) and [192,384) two
// accumulator buffers (the epilogue of one tile runs while the next
// accumulates), [384,512) four 32-column A stages. Every wait is bounded; a
// wait that gives up raises a CTA-wide abort and the device error word.
//
// The K order inside every group of 8 activations is 0,4,1,5,2,6,3,7: that
// is the order the nibble conversion produces the weights in, so the
// activation operands (Xp, H) are stored in the same interleaved order.
#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "plan.cuh"
#include "skinny.h"

using namespace wb;

namespace {

constexpr int kDqWarps = 16;
constexpr int kEpiWarps = 8;
constexpr int kEpiWarp0 = kDqWarps;
constexpr int kTmaBWarp = kDqWarps + kEpiWarps;
constexpr int kMmaWarp = kTmaBWarp + 1;
constexpr int kTmaWWarp = kTmaBWarp + 2;
constexpr int kThreads = (kTmaWWarp + 1) * 32;
constexpr int BM = 128;                      // A rows per tile (TMEM lanes)
constexpr int kGuRows = 64;                  // intermediate rows per gate/up tile
#ifndef WB_TC_BN
#define WB_TC_BN 192
#endif
constexpr int kBNMax = WB_TC_BN;             // token rows per tile
constexpr int KA = 128;                      // K per stage (A stage = raw stage = B stage)
constexpr int kAStageCols = KA / 2;          // 128 K of fp16 per lane
constexpr int kAColBase = 2 * kBNMax;
constexpr int kTmemCols = 512;
constexpr int kAStages = (kTmemCols - kAColBase) / kAStageCols;
static_assert(kAStages >= 2, "TMEM columns");
constexpr int kRawK = KA;
// raw stage: [nibbles: gate box, up box (4 KB each) | down box (8 KB)]
//            [scales: 2 runs of up to 512 B][zero points: the same]
constexpr int kRawStages = 6;
constexpr int kScRun = 512;
constexpr int kScOff = 8192;
constexpr int kZOff = kScOff + 2 * kScRun;
constexpr int kRawStageBytes = kZOff + 2 * kScRun;
static_assert(kRawStageBytes % 1024 == 0, "raw stages keep 1024-byte alignment");
constexpr int kBStages = 5;
// one CTA's token rows of a stage: two 64-K halves of kBNMax/2 rows x 128 B
constexpr int kBStageBytes = kBNMax / 2 * 256;
// Stage j is ready when full[j % kRing] completes (in the even CTA: both
// CTAs' dequant warps and both halves of the token rows; in the odd CTA: its
// own token rows, which a relay forwards) and consumed when done[j % kRing]
// completes (one commit per stage), which frees A slot j % kAStages and B
// slot j % kBStages: one ring whose length both divide.
constexpr int kRing = kAStages * kBStages;
// Split K: a call with fewer tiles than half the SMs cuts each tile's K into
// up to kMaxSplit ranges (work items) so more SMs take part; the down
// projection's parts add into the output with its usual atomics, gate/up
// parts go to a scratch buffer and the last part of a tile's lane quadrant
// sums them in order and applies SwiGLU. At most kMaxSplitItems items.
constexpr int kMaxSplit = 8;
constexpr int kMaxSplitItems = 128;
constexpr int kMaxFix = 16;   // quadrants one CTA may complete (<= 4 per item, <= 2 items per pair)
constexpr size_t kPartialFloats = (size_t)kBNMax * BM;   // one CTA's part of a gate/up work item

enum { GATEUP = 0, DOWN = 1 };

// Prepared weights: per matrix entry (expert v, matrix m in gate/up/down) two
// TMA descriptors of its packed nibbles (64-byte boxes of 64 rows for gate
// and up, 128 rows for down, with the 64-byte swizzle for this kernel;
// 128-byte boxes of 128 rows with the 128-byte swizzle for the register-path
// kernel), a zero-point flag, and its scales and zero points
// transposed to [row tile][group][128 rows] so that the scales of one stage
// are one contiguous run. For the register-path kernel, per expert a second
// copy of the scales (and zero points) in its unit order: the gate/up pair
// as [128-row block][256-K stage][gate, up][groups of the stage][128 rows]
// and down as [256-row block][256-K stage][first, second 128 rows][groups]
// [128 rows], so each stage of a unit takes one contiguous copy (slots
// outside the matrix hold zeros).
struct PreparedLayout {
  size_t maps, maps_sk, flags, zbits, scales, zeros, mat_sc_bytes;
  size_t sk_scales, sk_zeros, sk_gu_bytes, sk_dn_bytes, sk_stage_bytes;
  size_t total;
};

PreparedLayout prepared_layout(const WispMoeConfig* c, int n) {
  PreparedLayout L;
  const size_t entries = (size_t)n * 3;
  const int M = c->hidden, I = c->inter;
  L.mat_sc_bytes = (size_t)M * I / c->group_size * 2;
  L.maps = 0;
  L.maps_sk = entries * sizeof(CUtensorMap);
  L.flags = L.maps_sk + entries * sizeof(CUtensorMap);
  L.zbits = L.flags + entries * 4;  // the same flags, one bit per entry
  L.scales = (L.zbits + (entries + 31) / 32 * 4 + 255) & ~(size_t)255;
  L.zeros = L.scales + entries * L.mat_sc_bytes;
  const int G = 256 / c->group_size;
  L.sk_stage_bytes = (size_t)2 * G * BM * 2;
  L.sk_gu_bytes = (size_t)(I / BM) * ((M + 255) / 256) * L.sk_stage_bytes;
  L.sk_dn_bytes = (size_t)((M + 255) / 256) * ((I + 255) / 256) * L.sk_stage_bytes;
  L.sk_scales = (L.zeros + entries * L.mat_sc_bytes + 255) & ~(size_t)255;
  L.sk_zeros = L.sk_scales + (size_t)n * (L.sk_gu_bytes + L.sk_dn_bytes);
  L.total = L.sk_zeros + (size_t)n * (L.sk_gu_bytes + L.sk_dn_bytes);
  return L;
}


struct GemmParams {
  CUtensorMap tmap[6];  // activation rows as {64 K, rows, K / 64}: boxes {64, 16 (i + 1), 2}
  const uint8_t* prepared;
  size_t p_flags, p_scales, p_zeros, p_mat_sc_bytes;
  const WispSegment* segs;
  const int32_t* tiles;  // [0, S]: tile prefix; [S+1, 2S+1): bn per segment; [2S+1]: K split
  float* partial;        // split gate/up: per work item [column][128 A rows] floats
  int* tickets;          // split gate/up: arrivals per (tile, lane quadrant)
  int nseg;
  int M, I, gs;
  __half* h_out;
  const int* row_token;
  const float* row_weight;
  float* out;
  int mode;
  int* error_flag;
  unsigned long long* counters;  // optional wait-cycle counters (diagnostics)
};

// Diagnostic counters (cycles, summed over CTAs; one recording thread per
// warp): which wait each role spends its time in.
enum {
  C_DQ_RFULL, C_DQ_AEMPTY, C_DQ_WAITST, C_DQ_TOTAL,
  C_MMA_AFULL, C_MMA_BFULL, C_MMA_ACCEMPTY, C_MMA_TOTAL,
  C_TW_REMPTY, C_TW_TOTAL, C_TB_BEMPTY, C_TB_TOTAL,
  C_EPI_ACCFULL, C_EPI_TOTAL, C_TILES, C_COUNT
};

struct Prof {
  unsigned long long* out;
  unsigned long long acc[4];
  long long t_start;
  __device__ explicit Prof(unsigned long long* o) : out(o), acc{0, 0, 0, 0} {
    t_start = out ? clock64() : 0;
  }
  __device__ __forceinline__ long long now() const { return out ? clock64() : 0; }
  __device__ __forceinline__ void add(int i, long long t0) {
    if (out) acc[i] += (unsigned long long)(clock64() - t0);
  }
  __device__ void flush(const int (&slots)[4], int total_slot, bool recorder) {
    if (!out || !recorder) return;
    for (int i = 0; i < 4; i++)
      if (slots[i] >= 0) atomicAdd(out + slots[i], acc[i]);
    atomicAdd(out + total_slot, (unsigned long long)(clock64() - t_start));
  }
};

struct SmemLayout {
  uint64_t rfull[kRawStages], rempty[kRawStages];
  uint64_t full[kRing];
  uint64_t done[kRing];
  uint64_t accfull[2], accempty[2], final_bar;
  uint32_t tmem_base;
  int abort;
  int fix_n;            // split gate/up: lane quadrants this CTA completes
  int fix[kMaxFix];     // tile * 4 + quadrant
};

struct TileInfo {
  int seg, expert, row0, nvalid, bn, mblk;
};

// Tiles are ordered (segment, weight row block, token block) with the token
// blocks of one weight block adjacent, so CTAs that run them at the same
// time share the weight tile through L2.
__device__ __forceinline__ TileInfo decode_tile(const GemmParams& p, int tile) {
  // Largest segment s with tiles[s] <= tile (segments with no tiles are
  // skipped because their prefix equals the next one).
  int lo = 0, hi = p.nseg - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(p.tiles + mid) <= tile) lo = mid; else hi = mid - 1;
  }
  const int s = lo;
  const WispSegment sg = p.segs[s];
  const int bn = __ldg(p.tiles + p.nseg + 1 + s);
  const int nblk = (sg.rows + bn - 1) / bn;
  const int local = tile - __ldg(p.tiles + s);
  TileInfo t;
  t.seg = s;
  t.expert = sg.expert;
  t.mblk = local / nblk;
  const int nb = local % nblk;
  t.bn = bn;
  t.row0 = sg.row_begin + nb * bn;
  t.nvalid = min(bn, sg.rows - nb * bn);
  return t;
}

// A row r of a gate/up tile: matrix (0 gate, 1 up) and row within the tile's
// 64 intermediate rows.
__device__ __forceinline__ int gu_matrix(int r) { return (r >> 3) & 1; }
__device__ __forceinline__ int gu_row(int r) { return ((r >> 4) << 3) | (r & 7); }

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) grouped_ffn_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (base_u32 & 1023)) & 1023);
  uint8_t* raw_ring = smem;                                   // kRawStages * kRawStageBytes
  uint8_t* b_ring = raw_ring + kRawStages * kRawStageBytes;   // kBStages * kBStageBytes
  SmemLayout* L = reinterpret_cast<SmemLayout*>(b_ring + kBStages * kBStageBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = (int)cluster_rank();      // 0: issues the pair's MMAs
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int ntiles = __ldg(p.tiles + p.nseg);
  const int split = __ldg(p.tiles + 2 * p.nseg + 1);
  const int nitems = ntiles * split;  // work item = (tile, K part), parts of a tile adjacent
  // A pair without work leaves before any set-up, tensor memory included
  // (both CTAs of the pair take the same branch).
  if (pair >= nitems) return;
  const int K = MODE == GATEUP ? p.M : p.I;
  const int nR = K / KA;              // stages of the whole K
  // Stages [r0, r1) of K part ks (each item has at least one).
  auto part_range = [&](int ks, int& r0, int& r1) {
    r0 = ks * nR / split;
    r1 = (ks + 1) * nR / split;
  };
  // This CTA's weight-row block of a pair tile: 64 intermediate rows
  // (gate/up) or 128 output rows (down).
  auto cta_block = [&](const TileInfo& ti) { return 2 * ti.mblk + rank; };
  volatile int* abort = &L->abort;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRawStages; i++) {
      mbar_init(&L->rfull[i], 1);
      mbar_init(&L->rempty[i], kDqWarps);       // every dequant warp reads every raw stage
    }
    // even CTA: both CTAs' dequant warps + its token copy + the odd CTA's
    // relay; odd CTA: its token copy
    for (int i = 0; i < kRing; i++) {
      mbar_init(&L->full[i], rank == 0 ? 2 * kDqWarps + 2 : 1);
      mbar_init(&L->done[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&L->accfull[i], 1);
      mbar_init(&L->accempty[i], 2 * kEpiWarps);  // both CTAs' epilogue warps (even CTA's)
    }
    mbar_init(&L->final_bar, 1);
    L->abort = 0;
    L->fix_n = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc_pair(&L->tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = L->tmem_base;
  const int32_t* flags = reinterpret_cast<const int32_t*>(p.prepared + p.p_flags);

  if (warp < kDqWarps) {
    // ------------------------------------------------------------------
    // Dequantisation: warp w converts K quarter w >> 2 (32 K) of every
    // stage for TMEM lanes 32 (w % 4) .. +31, one A row per thread, and
    // reports the stage to the even CTA's MMA issuer as soon as its store
    // has completed.
    // ------------------------------------------------------------------
    const int qd = warp & 3, kq = warp >> 2;
    const int r = qd * 32 + lane;
    const int beta = MODE == GATEUP ? gu_matrix(r) : 0;
    const int rho = MODE == GATEUP ? gu_row(r) : r;
    // 16-byte chunk kq of this thread's 64-byte row under the box's 64-byte
    // swizzle: conflict-free, the 8 threads of a quarter-warp read 8 rows of
    // one box.
    const uint32_t rd_off = (uint32_t)(beta * 4096 + rho * 64 + ((kq ^ ((rho >> 1) & 3)) << 4));
    const int gl = (kq * 32) / p.gs;             // scale group inside the stage
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t st_col = kAColBase + kq * 16;
    const uint32_t full_remote = rank ? cluster_addr(&L->full[0], 0) : 0u;
    int ir = 0;          // stages this CTA has consumed
    bool ok = true;
    Prof pf(p.counters);
    for (int it = pair; it < nitems && ok && !*abort; it += npairs) {
      const int tile = it / split;
      int r0, r1;
      part_range(it - tile * split, r0, r1);
      const TileInfo ti = decode_tile(p, tile);
      const int cb = cta_block(ti);
      const int mat = MODE == GATEUP ? beta : 2;
      const bool has_zero = __ldg(flags + ti.expert * 3 + mat) & 1;
      // row inside the stage's scale run (the 128-row tile of the prepared copy)
      const int srow = MODE == GATEUP ? (cb & 1) * kGuRows + rho : rho;
      const uint32_t s_off = (uint32_t)(kScOff + beta * kScRun + (gl * BM + srow) * 2);
      for (int rs = r0; rs < r1; rs++, ir++) {
        const int rslot = ir % kRawStages;
        long long t0 = pf.now();
        if (!mbar_wait(&L->rfull[rslot], (uint32_t)(ir / kRawStages) & 1, abort)) { ok = false; break; }
        pf.add(0, t0);
        const uint8_t* rsb = raw_ring + rslot * kRawStageBytes;
        const uint4 qv = *reinterpret_cast<const uint4*>(rsb + rd_off);
        const __half s = *reinterpret_cast<const __half*>(rsb + s_off);
        const __half z = has_zero ? *reinterpret_cast<const __half*>(rsb + s_off + (kZOff - kScOff))
                                  : __float2half(0.f);
        __syncwarp();
        if (lane == 0) mbar_arrive(&L->rempty[rslot]);
        const __half2 s2 = __halves2half2(s, s), z2 = __halves2half2(z, z);
        uint32_t v[16];
        const uint32_t words[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
        for (int w = 0; w < 4; w++) {
          uint32_t o[4];
          nib8_dequant(words[w], s2, z2, o);
          v[4 * w + 0] = o[0];
          v[4 * w + 1] = o[1];
          v[4 * w + 2] = o[2];
          v[4 * w + 3] = o[3];
        }
        const int sa = ir % kAStages;
        t0 = pf.now();
        if (ir >= kAStages) {
          const int j = ir - kAStages;   // the stage whose completion frees this slot
          if (!mbar_wait(&L->done[j % kRing], (uint32_t)(j / kRing) & 1, abort)) {
            ok = false;
            break;
          }
        }
        pf.add(1, t0);
        tc_fence_after();
        tmem_st16(tmem + lane_base + st_col + (uint32_t)(sa * kAStageCols), v);
        t0 = pf.now();
        tmem_wait_st();
        pf.add(2, t0);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          const int f = ir % kRing;
          if (rank == 0) mbar_arrive(&L->full[f]);
          else mbar_arrive_remote(full_remote + (uint32_t)(f * sizeof(uint64_t)));
        }
      }
    }
    {
      const int slots[4] = {C_DQ_RFULL, C_DQ_AEMPTY, C_DQ_WAITST, -1};
      pf.flush(slots, C_DQ_TOTAL, lane == 0);
    }
  } else if (warp == kTmaWWarp) {
    // ------------------------------------------------------------------
    // Weight producer: this CTA's nibble boxes + scale / zero runs per
    // stage (a down block past the matrix's last row loads nothing).
    // ------------------------------------------------------------------
    if (lane == 0) {
      const int ng = KA / p.gs;           // scale groups per stage (1 or 2)
      const int gpr = K / p.gs;           // groups per weight row
      const int nm = MODE == GATEUP ? 2 : 1;
      const uint32_t run = (uint32_t)(ng * BM * 2);
      int ir = 0;
      bool ok = true;
      Prof pf(p.counters);
      for (int it = pair; it < nitems && ok && !*abort; it += npairs) {
        const int tile = it / split;
        int r0, r1;
        part_range(it - tile * split, r0, r1);
        const TileInfo ti = decode_tile(p, tile);
        const int cb = cta_block(ti);
        const int tile128 = MODE == GATEUP ? cb >> 1 : cb;
        const int wrow = MODE == GATEUP ? cb * kGuRows : cb * BM;
        const bool in = MODE == GATEUP || wrow < p.M;
        uint32_t bytes = 0;
        bool hz[2] = {false, false};
        const CUtensorMap* map[2] = {nullptr, nullptr};
        const uint8_t* sc[2] = {nullptr, nullptr};
        const uint8_t* zr[2] = {nullptr, nullptr};
        for (int j = 0; j < nm && in; j++) {
          const int e = ti.expert * 3 + (MODE == GATEUP ? j : 2);
          hz[j] = __ldg(flags + e) & 1;
          map[j] = reinterpret_cast<const CUtensorMap*>(p.prepared + (size_t)e * sizeof(CUtensorMap));
          sc[j] = p.prepared + p.p_scales + (size_t)e * p.p_mat_sc_bytes + (size_t)tile128 * gpr * BM * 2;
          zr[j] = p.prepared + p.p_zeros + (size_t)e * p.p_mat_sc_bytes + (size_t)tile128 * gpr * BM * 2;
          bytes += (MODE == GATEUP ? 4096u : 8192u) + run * (hz[j] ? 2u : 1u);
        }
        for (int rs = r0; rs < r1; rs++, ir++) {
          const int rslot = ir % kRawStages;
          const long long t0 = pf.now();
          if (ir >= kRawStages &&
              !mbar_wait(&L->rempty[rslot], (uint32_t)(ir / kRawStages - 1) & 1, abort)) {
            ok = false;
            break;
          }
          pf.add(0, t0);
          uint8_t* dst = raw_ring + rslot * kRawStageBytes;
          mbar_arrive_expect_tx(&L->rfull[rslot], bytes);
          const size_t goff = (size_t)rs * ng * BM * 2;
          for (int j = 0; j < nm && in; j++) {
            tma_load_2d(dst + j * 4096, map[j], &L->rfull[rslot], rs * (KA / 2), wrow);
            bulk_load(dst + kScOff + j * kScRun, sc[j] + goff, run, &L->rfull[rslot]);
            if (hz[j]) bulk_load(dst + kZOff + j * kScRun, zr[j] + goff, run, &L->rfull[rslot]);
          }
        }
      }
      {
        const int slots[4] = {C_TW_REMPTY, -1, -1, -1};
        pf.flush(slots, C_TW_TOTAL, true);
      }
      // Let every issued copy land before the CTA can exit.
      for (int j = max(0, ir - kRawStages); j < ir; j++)
        mbar_wait(&L->rfull[j % kRawStages], (uint32_t)(j / kRawStages) & 1, abort, 200000000LL);
    }
  } else if (warp == kTmaBWarp) {
    // ------------------------------------------------------------------
    // Activation producer: per stage, this CTA's half of the tile's token
    // rows (the even CTA the first bn/2, the odd one the rest) x 128 K, as
    // one 3D box laid out [64-K half][row][128 B] in one ring slot.
    // ------------------------------------------------------------------
    if (lane == 0) {
      for (int i = 0; i < 6; i++) tma_prefetch_desc(&p.tmap[i]);
      int ia = 0;
      bool ok = true;
      Prof pf(p.counters);
      for (int it = pair; it < nitems && ok && !*abort; it += npairs) {
        const int tile = it / split;
        int r0, r1;
        part_range(it - tile * split, r0, r1);
        const TileInfo ti = decode_tile(p, tile);
        const int half = ti.bn >> 1;
        const CUtensorMap* tm = &p.tmap[(half >> 4) - 1];
        const int row0 = ti.row0 + rank * half;
        for (int ka = r0; ka < r1; ka++, ia++) {
          const int sb = ia % kBStages;
          const long long t0 = pf.now();
          if (ia >= kBStages) {
            const int j = ia - kBStages;   // the stage whose completion frees this slot
            if (!mbar_wait(&L->done[j % kRing], (uint32_t)(j / kRing) & 1, abort)) {
              ok = false;
              break;
            }
          }
          pf.add(0, t0);
          uint64_t* fb = &L->full[ia % kRing];
          mbar_arrive_expect_tx(fb, (uint32_t)(half * 256));
          tma_load_3d(b_ring + sb * kBStageBytes, tm, fb, 0, row0, 2 * ka);
        }
      }
      {
        const int slots[4] = {C_TB_BEMPTY, -1, -1, -1};
        pf.flush(slots, C_TB_TOTAL, true);
      }
      // Let this CTA's last copies land before it can exit (the even CTA's
      // phases also need the dequant warps and the odd CTA's relay).
      for (int j = max(0, ia - kBStages); j < ia; j++)
        mbar_wait(&L->full[j % kRing], (uint32_t)(j / kRing) & 1, abort, 200000000LL);
    }
  } else if (warp == kMmaWarp) {
    if (rank == 0) {
      // ----------------------------------------------------------------
      // MMA issuer (one thread of the even CTA): per stage eight M=256 x
      // N=bn x K=16 pair MMAs into the item's accumulator buffer (items
      // alternate buffers) and one commit that frees the stage's A and B
      // slots in both CTAs. Ring positions advance without divisions.
      // ----------------------------------------------------------------
      if (lane == 0) {
        const uint32_t b0 = smem_u32(b_ring);
        const uint32_t a0 = tmem + (uint32_t)kAColBase;
        // ring positions of the next stage, advanced without divisions
        int sa = 0, sb = 0, sf = 0, nloc = 0;
        uint32_t pf_phase = 0;
        bool ok = true;
        Prof pf(p.counters);
        for (int it = pair; it < nitems && ok && !*abort; it += npairs, nloc++) {
          const int tile = it / split;
          int r0, r1;
          part_range(it - tile * split, r0, r1);
          const TileInfo ti = decode_tile(p, tile);
          const uint32_t idesc = idesc_f16_m256(ti.bn);
          const uint32_t khalf = (uint32_t)((ti.bn >> 1) * 128) >> 4;   // second 64-K half
          const int ab = nloc & 1;
          const uint32_t d_tmem = tmem + (uint32_t)(ab * kBNMax);
          long long t0 = pf.now();
          if (nloc >= 2 && !mbar_wait(&L->accempty[ab], (uint32_t)((nloc >> 1) - 1) & 1, abort)) break;
          pf.add(2, t0);
          tc_fence_after();
          for (int a = r0; a < r1; a++) {
            t0 = pf.now();
            if (!mbar_wait(&L->full[sf], pf_phase, abort)) { ok = false; break; }
            pf.add(0, t0);
            tc_fence_after();
            const uint32_t a_col = a0 + (uint32_t)(sa * kAStageCols);
            const uint64_t bd = smem_desc_sw128(b0 + (uint32_t)(sb * kBStageBytes));
            if (a == r0) mma_f16_ts_pair<0>(d_tmem, a_col, bd, idesc);
            else mma_f16_ts_pair<1>(d_tmem, a_col, bd, idesc);
#pragma unroll
            for (int kk = 1; kk < 8; kk++)
              mma_f16_ts_pair<1>(d_tmem, a_col + kk * 8, bd + (kk >> 2) * khalf + 2 * (kk & 3), idesc);
            mma_commit_pair(&L->done[sf]);
            sa = sa + 1 == kAStages ? 0 : sa + 1;
            sb = sb + 1 == kBStages ? 0 : sb + 1;
            if (++sf == kRing) { sf = 0; pf_phase ^= 1; }
          }
          if (!ok) break;
          mma_commit_pair(&L->accfull[ab]);
        }
        {
          const int slots[4] = {C_MMA_AFULL, C_MMA_BFULL, C_MMA_ACCEMPTY, -1};
          pf.flush(slots, C_MMA_TOTAL, true);
          if (p.counters) atomicAdd(p.counters + C_TILES, (unsigned long long)nloc);
        }
        // Drain: make sure no MMA is still running before either CTA moves
        // on to release its tensor memory.
        mma_commit_pair(&L->final_bar);
        mbar_wait(&L->final_bar, 0, abort, 200000000LL);
      }
    } else if (lane == 0) {
      // ----------------------------------------------------------------
      // Relay (odd CTA): forward each of this CTA's landed activation
      // stages to the even CTA's barrier, in stage order.
      // ----------------------------------------------------------------
      const uint32_t full_remote = cluster_addr(&L->full[0], 0);
      int sf = 0;
      uint32_t pf_phase = 0;
      bool ok = true;
      for (int it = pair; it < nitems && ok && !*abort; it += npairs) {
        const int tile = it / split;
        int r0, r1;
        part_range(it - tile * split, r0, r1);
        for (int ka = r0; ka < r1; ka++) {
          if (!mbar_wait(&L->full[sf], pf_phase, abort)) { ok = false; break; }
          mbar_arrive_remote(full_remote + (uint32_t)(sf * sizeof(uint64_t)));
          if (++sf == kRing) { sf = 0; pf_phase ^= 1; }
        }
      }
    }
  } else {
    // ------------------------------------------------------------------
    // Epilogue warps 16-23: warp w reads accumulator lanes 32 (w % 4) ..
    // +31 of this CTA's rows; the two warps of a quadrant take alternate
    // column chunks. Both CTAs report a drained buffer to the even CTA.
    // ------------------------------------------------------------------
    const int qd = warp & 3, ch = (warp - kEpiWarp0) >> 2;
    const int r = qd * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(qd * 32) << 16);
    int nloc = 0;
    Prof pf(p.counters);
    for (int it = pair; it < nitems && !*abort; it += npairs, nloc++) {
      const int tile = it / split;
      const TileInfo ti = decode_tile(p, tile);
      const int cb = cta_block(ti);
      const int ab = nloc & 1;
      const long long t0 = pf.now();
      if (!mbar_wait(&L->accfull[ab], (uint32_t)(nloc >> 1) & 1, abort)) break;
      pf.add(0, t0);
      tc_fence_after();
      const uint32_t acc = lane_addr + (uint32_t)(ab * kBNMax);
      bool released = false;
      if (MODE == GATEUP) {
        const int beta = gu_matrix(r);
        if (split == 1) {
          const int islot = k_interleave_slot(cb * kGuRows + gu_row(r));
          for (int c0 = 16 * ch; c0 < ti.bn; c0 += 32) {
            uint32_t a[16];
            tmem_ld16(acc + c0, a);
            tmem_wait_ld();
            // Column pair (j, j+1): the gate lane finishes column j, its up
            // partner (lane ^ 8) column j+1; one exchange serves both.
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
              const float mine_lo = __uint_as_float(a[j]), mine_hi = __uint_as_float(a[j + 1]);
              const float got = __shfl_xor_sync(0xffffffffu, beta ? mine_lo : mine_hi, 8);
              const float g = beta ? got : mine_lo;
              const float u = beta ? mine_hi : got;
              const int col = c0 + j + beta;
              if (col < ti.nvalid)
                p.h_out[(size_t)(ti.row0 + col) * p.I + islot] = __float2half(silu(g) * u);
            }
          }
        } else {
          // This K part's sums go to the scratch item of this CTA, laid out
          // [column][A row]; the CTA whose arrival completes the quadrant
          // (both of its warps, every part) sums all parts in order after
          // its last item.
          float* pit = p.partial + (size_t)(2 * it + rank) * kPartialFloats + r;
          for (int c0 = 16 * ch; c0 < ti.bn; c0 += 32) {
            uint32_t a[16];
            tmem_ld16(acc + c0, a);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; j++) pit[(size_t)(c0 + j) * BM] = __uint_as_float(a[j]);
          }
          tc_fence_before();
          __threadfence();
          __syncwarp();
          if (lane == 0) {
            if (rank == 0) mbar_arrive(&L->accempty[ab]);
            else mbar_arrive_remote(cluster_addr(&L->accempty[ab], 0));
          }
          released = true;
          int old = 0;
          if (lane == 0) {
            __threadfence();
            old = atomicAdd(p.tickets + (2 * tile + rank) * 4 + qd, 1);
            __threadfence();
          }
          old = __shfl_sync(0xffffffffu, old, 0);
          if (old == 2 * split - 1 && lane == 0) {
            const int slot = atomicAdd(&L->fix_n, 1);
            if (slot < kMaxFix) L->fix[slot] = tile * 4 + qd;
            else atomicExch(&L->abort, 1);  // cannot happen: items per pair are bounded
          }
        }
      } else {
        const int m = cb * BM + r;
        const bool row_in = m < p.M;
        for (int c0 = 32 * ch; c0 < ti.bn; c0 += 64) {
          // tokens and router weights of these 32 columns: one per lane,
          // broadcast below (no dependent loads inside the store loop)
          const int myrow = ti.row0 + c0 + lane;
          const bool mine = c0 + lane < ti.nvalid;
          const int tok_l = (p.mode == 0 && mine) ? __ldg(p.row_token + myrow) : 0;
          const float w_l = (p.mode == 0 && mine) ? __ldg(p.row_weight + myrow) : 0.f;
          uint32_t ya[16], yb[16];
          tmem_ld16(acc + c0, ya);
          if (c0 + 16 < ti.bn) tmem_ld16(acc + c0 + 16, yb);
          else {
#pragma unroll
            for (int j = 0; j < 16; j++) yb[j] = 0u;
          }
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const int tt = c0 + j;
            const int tok = __shfl_sync(0xffffffffu, tok_l, j);
            const float wgt = __shfl_sync(0xffffffffu, w_l, j);
            if (tt < ti.nvalid && row_in) {
              const float yv = __uint_as_float(j < 16 ? ya[j] : yb[j - 16]);
              if (p.mode == 0)
                red_add_f32(p.out + (size_t)tok * p.M + m, wgt * yv);
              else
                p.out[(size_t)(ti.row0 + tt) * p.M + m] = yv;
            }
          }
        }
      }
      if (!released) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) mbar_arrive(&L->accempty[ab]);
          else mbar_arrive_remote(cluster_addr(&L->accempty[ab], 0));
        }
      }
    }
    const int slots[4] = {C_EPI_ACCFULL, -1, -1, -1};
    pf.flush(slots, C_EPI_TOTAL, lane == 0);
  }

  tc_fence_before();
  // Neither CTA leaves (or frees tensor memory) while the pair's MMAs or
  // the other CTA's arrivals may still touch it.
  cluster_sync();
  // Split gate/up: every thread of the CTA sums the parts of the quadrants
  // it completes (K parts in order), applies SwiGLU and writes H; the partial
  // sums were published before the arrival counts (fence, then the count;
  // the completing warp fenced after reading it, then the cluster barrier).
  if (MODE == GATEUP && split > 1 && !L->abort) {
    const int nfix = min(L->fix_n, kMaxFix);
    for (int f = 0; f < nfix; f++) {
      const int tile = L->fix[f] >> 2, qd = L->fix[f] & 3;
      const TileInfo ti = decode_tile(p, tile);
      const int cb = cta_block(ti);
      // 16 (gate, up) row pairs per quadrant; part ks of this CTA's rows is
      // scratch item 2 (tile * split + ks) + rank
      for (int i = threadIdx.x; i < 16 * ti.nvalid; i += blockDim.x) {
        const int pr = i & 15, c = i >> 4;
        const int rg = qd * 32 + ((pr >> 3) << 4) + (pr & 7);   // gate lane; up lane rg + 8
        float g = 0.f, u = 0.f;
        for (int ks = 0; ks < split; ks++) {
          const float* pc = p.partial + (size_t)(2 * (tile * split + ks) + rank) * kPartialFloats +
                            (size_t)c * BM + rg;
          g += __ldcg(pc);
          u += __ldcg(pc + 8);
        }
        const int row = cb * kGuRows + gu_row(rg);
        p.h_out[(size_t)(ti.row0 + c) * p.I + k_interleave_slot(row)] = __float2half(silu(g) * u);
      }
    }
  }
  if (threadIdx.x == 0 && L->abort && p.error_flag) atomicExch(p.error_flag, 1);
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

// Per segment: BN (the fewest tiles of at most kBNMax rows, rounded up to
// a multiple of 16) and the
// prefix sum of tiles; then the K split (tiles[2 nseg + 1]): when the tiles
// fill fewer than half of `target` SMs, each is cut into up to max_split K
// parts of at least one raw stage (nraw stages in all), at most
// kMaxSplitItems parts in all. `tickets` (split gate/up arrivals, 4 per
// tile) are zeroed. Segments of at most skip_rows rows belong to the
// register-path kernel and get no tiles here.
__device__ void plan_tiles(const WispSegment* __restrict__ segs, int nseg, int mblocks,
                           int skip_rows, int max_split, int target, int nraw,
                           int32_t* __restrict__ tiles, int32_t* __restrict__ tickets) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < nseg; base += blockDim.x) {
    const int s = base + threadIdx.x;
    int n = 0, bn = 16;
    if (s < nseg) {
      const int rows = segs[s].rows;
      const int nt = (max(rows, 1) + kBNMax - 1) / kBNMax;
      bn = ((max(rows, 1) + nt - 1) / nt + 31) & ~31;   // pair MMAs: N % 32 == 0
      n = rows > skip_rows ? ((rows + bn - 1) / bn) * mblocks : 0;
      tiles[nseg + 1 + s] = bn;
    }
    int v = n;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
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
    const int incl = v + (w > 0 ? warp_tot[w - 1] : 0) + carry;
    if (s < nseg) tiles[s] = incl - n;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const int nt = carry;
    int split = 1;
    if (nt > 0 && 2 * nt <= target)
      split = min(min(max_split, target / nt), min(nraw, kMaxSplitItems / nt));
    tiles[nseg] = nt;
    tiles[2 * nseg + 1] = max(split, 1);
  }
  if (tickets)
    for (int i = threadIdx.x; i < 8 * kMaxSplitItems; i += blockDim.x) tickets[i] = 0;
}

// Rows of the register-path segments (0 < rows <= sk_rows): fp16 rows in
// interleaved K order (within 8 K: 0,4,1,5,2,6,3,7) -> q16 rows (layout in
// skinny.h). Block (s, r) converts row r of segment s with 128 threads: a
// thread owns one packed-weight word (8 consecutive K) per 1024-K pass, so
// each half-warp holds one 128-K block, whose max |x| (four shuffles) sets
// its scale. Half-warps past the row's end take part in the shuffles with
// zeros and store nothing.
__global__ void __launch_bounds__(128) quant_rows_kernel(const WispSegment* __restrict__ segs,
                                                         int sk_rows, const __half* __restrict__ xp,
                                                         int M, uint8_t* __restrict__ xq) {
  const WispSegment sg = segs[blockIdx.x];
  const int r = blockIdx.y;
  if (sg.rows <= 0 || sg.rows > sk_rows || r >= sg.rows) return;
  const size_t p = (size_t)(sg.row_begin + r);
  const __half* xr = xp + p * M;
  uint8_t* qrow = xq + p * q16_row_bytes(M);
  const int lane = threadIdx.x & 31;
  for (int k0 = 0; k0 < M; k0 += 1024) {
    const int w = k0 / 8 + threadIdx.x;
    const bool in = 8 * w < M;
    float f[8];   // physical K order
    if (in) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + 8 * w);
      const float2 s04 = __half22float2(u2h2(v.x)), s15 = __half22float2(u2h2(v.y));
      const float2 s26 = __half22float2(u2h2(v.z)), s37 = __half22float2(u2h2(v.w));
      f[0] = s04.x; f[4] = s04.y; f[1] = s15.x; f[5] = s15.y;
      f[2] = s26.x; f[6] = s26.y; f[3] = s37.x; f[7] = s37.y;
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

// The four plans of one call in one launch: blocks 0 and 1 tile gate/up and
// down for the tensor-core kernel, blocks 2 and 3 cut them into register-path
// units.
struct PlanArgs {
  const WispSegment* segs;
  int nseg, sk_rows;
  int mb_gu, mb_dn;
  int split_gu, split_dn, nraw_gu, nraw_dn, sms;
  int32_t* tickets;
  int per_gu, per_dn, cols, ks_dn, nk_dn, target;
  int32_t *tiles_gu, *tiles_dn, *units_gu, *units_dn;
};

__global__ void __launch_bounds__(1024) plan_all_kernel(const __grid_constant__ PlanArgs a) {
  switch (blockIdx.x) {
    case 0:
      plan_tiles(a.segs, a.nseg, a.mb_gu, a.sk_rows, a.split_gu, a.sms, a.nraw_gu,
                 a.tiles_gu, a.tickets);
      break;
    case 1:
      plan_tiles(a.segs, a.nseg, a.mb_dn, a.sk_rows, a.split_dn, a.sms, a.nraw_dn,
                 a.tiles_dn, nullptr);
      break;
    case 2: plan_units(a.segs, a.nseg, a.per_gu, a.cols, a.sk_rows, 1, 1, 0, a.units_gu); break;
    default:
      plan_units(a.segs, a.nseg, a.per_dn, a.cols, a.sk_rows, a.ks_dn, a.nk_dn, a.target,
                 a.units_dn);
  }
}

// Scales (and zero points) of every prepared matrix, transposed from
// [rows][groups] to [row tile][group][128 rows].
// With experts == nullptr the launch covers the one entry `one`, written as
// entry `slot` of the prepared set (gridDim.y = 3).
__global__ void transpose_scales_kernel(const WispInt4Expert* __restrict__ experts, int n, int M,
                                        int I, int gs, uint8_t* __restrict__ prepared,
                                        size_t off_scales, size_t off_zeros, size_t mat_bytes,
                                        WispInt4Expert one, int slot) {
  const int m = blockIdx.y % 3;
  const int v = experts ? (int)blockIdx.y / 3 : slot;
  const int e = v * 3 + m;  // matrix entry
  const WispInt4Expert ex = experts ? experts[v] : one;
  const WispInt4Mat mt = m == 0 ? ex.gate : m == 1 ? ex.up : ex.down;
  const int rows = m == 2 ? M : I;
  const int gpr = (m == 2 ? I : M) / gs;
  const size_t total = (size_t)rows * gpr;
  const uint16_t* s = reinterpret_cast<const uint16_t*>(mt.scales);
  const uint16_t* z = reinterpret_cast<const uint16_t*>(mt.zeros);
  uint16_t* so = reinterpret_cast<uint16_t*>(prepared + off_scales + (size_t)e * mat_bytes);
  uint16_t* zo = reinterpret_cast<uint16_t*>(prepared + off_zeros + (size_t)e * mat_bytes);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    // destination index i = (tile * gpr + g) * 128 + r
    const size_t r = i % BM, rest = i / BM;
    const size_t g = rest % gpr, tile = rest / gpr;
    const size_t src = (tile * BM + r) * gpr + g;
    so[i] = s[src];
    if (z) zo[i] = z[src];
  }
}

// The register-path kernel's per-stage runs of scales and zero points (see
// PreparedLayout): blockIdx.y = expert * 2 + (0: gate/up pair, 1: down).
// With experts == nullptr: the one entry `one` as entry `slot` (gridDim.y = 2).
__global__ void skinny_scales_kernel(const WispInt4Expert* __restrict__ experts, int M, int I,
                                     int gs, uint8_t* __restrict__ prepared, size_t off_scales,
                                     size_t off_zeros, size_t gu_bytes, size_t dn_bytes,
                                     WispInt4Expert one, int slot) {
  const int v = experts ? (int)(blockIdx.y >> 1) : slot, part = blockIdx.y & 1;
  const WispInt4Expert ex = experts ? experts[v] : one;
  const int G = 256 / gs;
  const size_t base = (size_t)v * (gu_bytes + dn_bytes) + (part ? gu_bytes : 0);
  uint16_t* so = reinterpret_cast<uint16_t*>(prepared + off_scales + base);
  uint16_t* zo = reinterpret_cast<uint16_t*>(prepared + off_zeros + base);
  const size_t total = (part ? dn_bytes : gu_bytes) / 2;
  const int K = part ? I : M;
  const int nk = (K + 255) / 256, gpr = K / gs;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    // i = (((block * nk + kg) * 2 + half) * G + grp) * 128 + r
    const int r = (int)(i % BM);
    size_t rest = i / BM;
    const int grp = (int)(rest % G);
    rest /= G;
    const int half = (int)(rest % 2);
    rest /= 2;
    const int kg = (int)(rest % nk);
    const int blk = (int)(rest / nk);
    const WispInt4Mat mt = part ? ex.down : (half ? ex.up : ex.gate);
    const int row = part ? blk * 2 * BM + half * BM + r : blk * BM + r;
    const int group = kg * G + grp;
    const bool in = row < (part ? M : I) && group < gpr;
    const size_t src = (size_t)row * gpr + group;
    so[i] = in ? reinterpret_cast<const uint16_t*>(mt.scales)[src] : 0;
    zo[i] = (in && mt.zeros) ? reinterpret_cast<const uint16_t*>(mt.zeros)[src] : 0;
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// fp16 activation rows [rows x cols] as a 3D tensor {64 K, rows, K / 64} for
// the tensor-core kernel: one box = box_rows rows x 128 K, stored as two [box_rows][128 B]
// halves (one per 64 K) with the 128-byte swizzle -- the MMA's B operand of
// one stage in a single copy.
bool encode_rows_map3(CUtensorMap* m, const void* base, int rows, int cols, int box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)cols / 64};
  cuuint64_t strides[2] = {(cuuint64_t)cols * 2, 128};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 2};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// q16 rows (layout in skinny.h) as a 3D tensor {128 bytes, rows, lines}:
// one box = box_rows rows x the five lines of one 256-K stage, stored in
// shared memory as [line][row][128 bytes] with the 128-byte swizzle.
bool encode_q16_map(CUtensorMap* m, const void* base, int rows, int cols, int box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  const cuuint64_t rb = q16_row_bytes(cols);
  cuuint64_t dims[3] = {(cuuint64_t)kQ16LineBytes, (cuuint64_t)rows, rb / kQ16LineBytes};
  cuuint64_t strides[2] = {rb, (cuuint64_t)kQ16LineBytes};
  cuuint32_t box[3] = {(cuuint32_t)kQ16LineBytes, (cuuint32_t)box_rows, (cuuint32_t)kQ16Lines};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// Packed nibbles of one matrix [rows x cols/2 bytes] for the tensor-core
// kernel: boxes of 64 bytes x box_rows rows (64 for gate and up, 128 for
// down) with the 64-byte swizzle (conflict-free 16-byte reads per row).
bool encode_packed_map(CUtensorMap* m, const void* base, int rows, int cols, int box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols / 2, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols / 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// The same nibbles in 128-byte (256-K) x 128-row boxes with the 128-byte
// swizzle, for the register-path kernel: a box row is one 128-byte request.
bool encode_packed_map_sk(CUtensorMap* m, const void* base, int rows, int cols) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols / 2, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols / 2};
  cuuint32_t box[2] = {128, (cuuint32_t)BM};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

size_t smem_bytes() {
  return 1024 + (size_t)kRawStages * kRawStageBytes + (size_t)kBStages * kBStageBytes +
         sizeof(SmemLayout);
}

int num_sms();

// The tensor-core kernels run as persistent CTA pairs (clusters of 2), as
// many pairs as can be resident at once on this device (a GPC with an odd
// number of free SMs leaves one idle).
template <int MODE>
cudaLaunchConfig_t pair_config(int npairs, cudaStream_t st, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * npairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes();
  cfg.stream = st;
  attr->id = cudaLaunchAttributeClusterDimension;
  attr->val.clusterDim.x = 2;
  attr->val.clusterDim.y = 1;
  attr->val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

int grouped_pairs() {
  static int pairs[64] = {0};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  std::lock_guard<std::mutex> lock(mu);
  if (!pairs[dev]) {
    int n = 0;
    cudaFuncSetAttribute(grouped_ffn_kernel<GATEUP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem_bytes());
    cudaFuncSetAttribute(grouped_ffn_kernel<DOWN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem_bytes());
    cudaLaunchAttribute attr;
    cudaLaunchConfig_t cfg = pair_config<GATEUP>(num_sms() / 2, nullptr, &attr);
    if (cudaOccupancyMaxActiveClusters(&n, grouped_ffn_kernel<GATEUP>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms() / 2;
    }
    pairs[dev] = std::min(n, num_sms() / 2);
  }
  return pairs[dev];
}

template <int MODE>
cudaError_t launch_pairs(int npairs, cudaStream_t st, const GemmParams& p) {
  cudaLaunchAttribute attr;
  cudaLaunchConfig_t cfg = pair_config<MODE>(npairs, st, &attr);
  return cudaLaunchKernelEx(&cfg, grouped_ffn_kernel<MODE>, p);
}

int num_sms() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return sms[dev] > 0 ? sms[dev] : 148;
}

WispError check_shapes(const WispMoeConfig* cfg, WispErrCtx* err) {
  const int M = cfg->hidden, I = cfg->inter, gs = cfg->group_size;
  if (M <= 0 || I <= 0 || M % 128 || I % 128)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "grouped_ffn: hidden (%d) and inter (%d) must be multiples of 128", M, I);
  if (gs != 64 && gs != 128)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "grouped_ffn: group_size must be 64 or 128 (got %d)", gs);
  return WISP_OK;
}

unsigned long long* g_counters = nullptr;
int g_skinny_rows = -1;  // -1: library default

}  // namespace


extern "C" void wisp_b200_set_skinny_max_rows(int rows) { g_skinny_rows = rows; }

extern "C" void wisp_b200_debug_set_counters(unsigned long long* d_counters) {
  g_counters = d_counters;
}

namespace {
// Host side of one entry's preparation: its three matrices' TMA descriptors
// (tensor-core and register-path boxes) and zero-point flags.
WispError encode_entry(const WispInt4Expert& x, int M, int I, int v, CUtensorMap* maps,
                       CUtensorMap* maps_sk, int32_t* flags, WispErrCtx* err) {
  const WispInt4Mat* mats[3] = {&x.gate, &x.up, &x.down};
  for (int m = 0; m < 3; m++) {
    const int rows = m == 2 ? M : I, cols = m == 2 ? I : M;
    const WispInt4Mat& mt = *mats[m];
    if (!mt.packed || !mt.scales)
      return WB_FAIL(WISP_ERR_INVALID_ARG, "prepare_experts: entry %d matrix %d has no data", v, m);
    if (((uintptr_t)mt.packed & 15) || ((uintptr_t)mt.scales & 1) || ((uintptr_t)mt.zeros & 1))
      return WB_FAIL(WISP_ERR_INVALID_ARG,
                     "prepare_experts: entry %d matrix %d: packed must be 16-byte aligned", v, m);
    if (!encode_packed_map(&maps[m], mt.packed, rows, cols, m == 2 ? BM : kGuRows) ||
        !encode_packed_map_sk(&maps_sk[m], mt.packed, rows, cols))
      return WB_FAIL(WISP_ERR_CUDA, "prepare_experts: cuTensorMapEncodeTiled failed (entry %d)", v);
    flags[m] = mt.zeros ? 1 : 0;
  }
  return WISP_OK;
}

// One slot's descriptors and flags, passed by value, written into the
// prepared set: 6 x 128-byte descriptors copied as 16-byte words, the three
// flag words, and the slot's three bits of the flag bitmap (atomic, since a
// bitmap word is shared with neighbouring slots).
struct SlotMeta {
  CUtensorMap maps[3];
  CUtensorMap maps_sk[3];
  int32_t flags[3];
};

__global__ void write_slot_kernel(const __grid_constant__ SlotMeta sm, uint8_t* __restrict__ prepared,
                                  size_t off_maps, size_t off_maps_sk, size_t off_flags,
                                  size_t off_zbits, int slot) {
  const int t = threadIdx.x;  // 48 threads: 8 words per descriptor
  const uint4* src = reinterpret_cast<const uint4*>(t < 24 ? sm.maps : sm.maps_sk);
  uint4* dst = reinterpret_cast<uint4*>(prepared + (t < 24 ? off_maps : off_maps_sk) +
                                        (size_t)slot * 3 * sizeof(CUtensorMap));
  const int w = t % 24;
  dst[w] = src[w];
  if (t < 3) {
    const int i = slot * 3 + t;
    reinterpret_cast<int32_t*>(prepared + off_flags)[i] = sm.flags[t];
    unsigned int* zb = reinterpret_cast<unsigned int*>(prepared + off_zbits) + i / 32;
    if (sm.flags[t]) atomicOr(zb, 1u << (i % 32));
    else atomicAnd(zb, ~(1u << (i % 32)));
  }
}
}  // namespace

extern "C" size_t wisp_b200_prepared_bytes(const WispMoeConfig* cfg, int n_entries) {
  if (!cfg || n_entries <= 0 || check_shapes(cfg, nullptr) != WISP_OK) return 0;
  return prepared_layout(cfg, n_entries).total;
}

extern "C" WispError wisp_b200_prepare_experts(const WispMoeConfig* cfg,
                                               const WispInt4Expert* d_experts, int n_entries,
                                               void* d_prepared, size_t prepared_bytes,
                                               cudaStream_t stream, WispErrCtx* err) {
  if (!cfg || !d_experts || !d_prepared || n_entries <= 0)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "prepare_experts: bad arguments");
  WispError e = check_shapes(cfg, err);
  if (e != WISP_OK) return e;
  const PreparedLayout PL = prepared_layout(cfg, n_entries);
  if (prepared_bytes < PL.total)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "prepare_experts: buffer %zu < required %zu", prepared_bytes, PL.total);
  if ((uintptr_t)d_prepared & 255)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "prepare_experts: buffer must be 256-byte aligned");
  const int M = cfg->hidden, I = cfg->inter;
  std::vector<WispInt4Expert> h(n_entries);
  WB_CUDA_CHECK(cudaMemcpyAsync(h.data(), d_experts, sizeof(WispInt4Expert) * n_entries,
                                cudaMemcpyDeviceToHost, stream));
  WB_CUDA_CHECK(cudaStreamSynchronize(stream));
  std::vector<CUtensorMap> maps((size_t)n_entries * 3), maps_sk((size_t)n_entries * 3);
  std::vector<int32_t> flags((size_t)n_entries * 3);
  for (int v = 0; v < n_entries; v++) {
    e = encode_entry(h[v], M, I, v, &maps[(size_t)v * 3], &maps_sk[(size_t)v * 3],
                     &flags[(size_t)v * 3], err);
    if (e != WISP_OK) return e;
  }
  uint8_t* base = static_cast<uint8_t*>(d_prepared);
  WB_CUDA_CHECK(cudaMemcpyAsync(base + PL.maps, maps.data(), maps.size() * sizeof(CUtensorMap),
                                cudaMemcpyHostToDevice, stream));
  WB_CUDA_CHECK(cudaMemcpyAsync(base + PL.maps_sk, maps_sk.data(),
                                maps_sk.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice,
                                stream));
  WB_CUDA_CHECK(cudaMemcpyAsync(base + PL.flags, flags.data(), flags.size() * 4,
                                cudaMemcpyHostToDevice, stream));
  std::vector<uint32_t> zbits((flags.size() + 31) / 32, 0u);
  for (size_t i = 0; i < flags.size(); i++)
    if (flags[i]) zbits[i / 32] |= 1u << (i % 32);
  WB_CUDA_CHECK(cudaMemcpyAsync(base + PL.zbits, zbits.data(), zbits.size() * 4,
                                cudaMemcpyHostToDevice, stream));
  dim3 grid(64, n_entries * 3);
  transpose_scales_kernel<<<grid, 256, 0, stream>>>(d_experts, n_entries, M, I, cfg->group_size,
                                                    base, PL.scales, PL.zeros, PL.mat_sc_bytes,
                                                    WispInt4Expert{}, 0);
  WB_CUDA_CHECK(cudaGetLastError());
  skinny_scales_kernel<<<dim3(64, n_entries * 2), 256, 0, stream>>>(
      d_experts, M, I, cfg->group_size, base, PL.sk_scales, PL.sk_zeros, PL.sk_gu_bytes,
      PL.sk_dn_bytes, WispInt4Expert{}, 0);
  WB_CUDA_CHECK(cudaGetLastError());
  // The host vectors are read by the copies above before they are freed.
  WB_CUDA_CHECK(cudaStreamSynchronize(stream));
  return WISP_OK;
}

extern "C" WispError wisp_b200_prepare_expert_slot(const WispMoeConfig* cfg, int n_entries,
                                                   int slot, const WispInt4Expert* entry,
                                                   void* d_prepared, size_t prepared_bytes,
                                                   cudaStream_t stream, WispErrCtx* err) {
  if (!cfg || !entry || !d_prepared || n_entries <= 0 || slot < 0 || slot >= n_entries)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "prepare_expert_slot: bad arguments (slot %d of %d)",
                   slot, n_entries);
  WispError e = check_shapes(cfg, err);
  if (e != WISP_OK) return e;
  const PreparedLayout PL = prepared_layout(cfg, n_entries);
  if (prepared_bytes < PL.total)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "prepare_expert_slot: buffer %zu < required %zu",
                   prepared_bytes, PL.total);
  if ((uintptr_t)d_prepared & 255)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "prepare_expert_slot: buffer must be 256-byte aligned");
  const int M = cfg->hidden, I = cfg->inter;
  SlotMeta sm;
  memset(&sm, 0, sizeof sm);
  e = encode_entry(*entry, M, I, slot, sm.maps, sm.maps_sk, sm.flags, err);
  if (e != WISP_OK) return e;
  uint8_t* base = static_cast<uint8_t*>(d_prepared);
  write_slot_kernel<<<1, 48, 0, stream>>>(sm, base, PL.maps, PL.maps_sk, PL.flags, PL.zbits, slot);
  WB_CUDA_CHECK(cudaGetLastError());
  transpose_scales_kernel<<<dim3(64, 3), 256, 0, stream>>>(nullptr, n_entries, M, I,
                                                           cfg->group_size, base, PL.scales,
                                                           PL.zeros, PL.mat_sc_bytes, *entry, slot);
  WB_CUDA_CHECK(cudaGetLastError());
  skinny_scales_kernel<<<dim3(64, 2), 256, 0, stream>>>(
      nullptr, M, I, cfg->group_size, base, PL.sk_scales, PL.sk_zeros, PL.sk_gu_bytes,
      PL.sk_dn_bytes, *entry, slot);
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}

// Workspace of one grouped-FFN call: tensor-core gate/up and down tables
// [prefix S+1 | bn S | K split] each, the register path's gate/up and down
// unit prefixes [S+2] each, the split gate/up arrival counts [4 x
// kMaxSplitItems] (int32 words); then, 256-byte aligned, the split gate/up
// partial sums [kMaxSplitItems x 192 columns x 128 A rows floats], and the q16 rows
// (layout in skinny.h) of the register-path segments' input and of their
// SwiGLU output H.
namespace {
struct GroupedWs {
  int32_t* tiles_gu;
  int32_t* tiles_dn;
  int32_t* units_gu;
  int32_t* units_dn;
  int32_t* tickets;
  float* partial;
  uint8_t* xq;
  uint8_t* hq;
  size_t bytes;
};

GroupedWs carve_grouped(int n_segs, int rows, int M, int I, void* base) {
  GroupedWs w;
  size_t off = 0;
  auto take = [&](size_t bytes) -> uint8_t* {
    off = (off + 255) & ~(size_t)255;
    uint8_t* q = base ? static_cast<uint8_t*>(base) + off : nullptr;
    off += bytes;
    return q;
  };
  const size_t tw = (size_t)(2 * n_segs + 2);
  int32_t* words = reinterpret_cast<int32_t*>(
      take(4 * (2 * tw + (size_t)2 * (n_segs + 2) + 8 * (size_t)kMaxSplitItems)));
  w.tiles_gu = words;
  w.tiles_dn = words ? words + tw : nullptr;
  w.units_gu = words ? words + 2 * tw : nullptr;
  w.units_dn = words ? w.units_gu + (n_segs + 2) : nullptr;
  w.tickets = words ? w.units_dn + (n_segs + 2) : nullptr;
  w.partial = reinterpret_cast<float*>(take((size_t)2 * kMaxSplitItems * kPartialFloats * 4));
  w.xq = take((size_t)rows * q16_row_bytes(M));
  w.hq = take((size_t)rows * q16_row_bytes(I));
  w.bytes = (off + 255) & ~(size_t)255;
  return w;
}
}  // namespace

extern "C" size_t wisp_b200_grouped_workspace_bytes(const WispMoeConfig* cfg, int n_segs,
                                                    int rows_capacity) {
  if (!cfg || n_segs <= 0 || rows_capacity <= 0 || check_shapes(cfg, nullptr) != WISP_OK) return 0;
  return carve_grouped(n_segs, rows_capacity, cfg->hidden, cfg->inter, nullptr).bytes;
}

namespace wb {
// The routing threshold of a grouped-FFN call: segments of at most this many
// rows run on the register path. The register-path kernel keeps the
// zero-point flags in shared memory; larger launches run on the tensor-core
// kernel alone.
int grouped_sk_rows(int n_segs, int n_entries) {
  if (n_segs > skinny_max_segs() || n_entries > skinny_max_entries()) return 0;
  return g_skinny_rows >= 0 ? g_skinny_rows : skinny_max_rows();
}
// Where the q16 rows of the gate/up input live inside a grouped-FFN
// workspace (a caller that packs them itself passes xq_ready to
// grouped_ffn_impl).
uint8_t* grouped_xq(void* d_workspace, int n_segs, int rows_capacity, int M, int I) {
  return carve_grouped(n_segs, rows_capacity, M, I, d_workspace).xq;
}
WispError grouped_ffn_impl(const WispMoeConfig* cfg, const void* d_prepared,
                           const WispInt4Expert* d_experts, int n_entries,
                           const WispSegment* d_segs, int n_segs, int rows_capacity,
                           const uint16_t* d_xp, uint16_t* d_h, int mode, const int* d_row_token,
                           const float* d_row_weight, float* d_out, void* d_workspace,
                           size_t workspace_bytes, int* d_error_flag, bool xq_ready,
                           int max_seg_rows, cudaStream_t stream, WispErrCtx* err,
                           bool plans_ready = false);
void decode_units(const WispMoeConfig* cfg, int n_segs, int n_entries, int rows_capacity, int mode,
                  void* d_workspace, DecodeUnits* du);
}  // namespace wb

// The register path's plan arrays and plan numbers of a grouped call in mode
// `mode` over n_segs segments, for a planner that runs before the call
// (grouped_ffn_impl with plans_ready); the same numbers the call's own
// planner uses.
void wb::decode_units(const WispMoeConfig* cfg, int n_segs, int n_entries, int rows_capacity,
                      int mode, void* d_workspace, DecodeUnits* du) {
  const GroupedWs ws = carve_grouped(n_segs, rows_capacity, cfg->hidden, cfg->inter, d_workspace);
  du->units_gu = ws.units_gu;
  du->units_dn = ws.units_dn;
  du->xq = ws.xq;
  du->per_gu = wb::skinny_units_gateup(cfg->inter);
  du->per_dn = wb::skinny_units_down(cfg->hidden);
  du->cols = wb::skinny_cols();
  du->sk_rows = wb::grouped_sk_rows(n_segs, n_entries);
  du->ks_dn = mode == 0 ? 8 : 1;
  du->nk_dn = wb::skinny_stages(cfg->inter);
  du->target = 2 * num_sms();
}

extern "C" WispError wisp_b200_grouped_ffn(const WispMoeConfig* cfg, const void* d_prepared,
                                           const WispInt4Expert* d_experts,
                                           int n_entries, const WispSegment* d_segs, int n_segs,
                                           int rows_capacity, const uint16_t* d_xp, uint16_t* d_h,
                                           int mode, const int* d_row_token,
                                           const float* d_row_weight, float* d_out,
                                           void* d_workspace, size_t workspace_bytes,
                                           int* d_error_flag, cudaStream_t stream,
                                           WispErrCtx* err) {
  return wb::grouped_ffn_impl(cfg, d_prepared, d_experts, n_entries, d_segs, n_segs,
                              rows_capacity, d_xp, d_h, mode, d_row_token, d_row_weight, d_out,
                              d_workspace, workspace_bytes, d_error_flag, false, rows_capacity,
                              stream, err);
}

WispError wb::grouped_ffn_impl(const WispMoeConfig* cfg, const void* d_prepared,
                               const WispInt4Expert* d_experts, int n_entries,
                               const WispSegment* d_segs, int n_segs, int rows_capacity,
                               const uint16_t* d_xp, uint16_t* d_h, int mode,
                               const int* d_row_token, const float* d_row_weight, float* d_out,
                               void* d_workspace, size_t workspace_bytes, int* d_error_flag,
                               bool xq_ready, int max_seg_rows, cudaStream_t stream,
                               WispErrCtx* err, bool plans_ready) {
  if (!cfg || !d_prepared || !d_experts || !d_segs || !d_xp || !d_h || !d_out || !d_workspace ||
      n_entries <= 0)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "grouped_ffn: null pointer argument");
  WispError e = check_shapes(cfg, err);
  if (e != WISP_OK) return e;
  const int M = cfg->hidden, I = cfg->inter, gs = cfg->group_size;
  if (n_segs <= 0 || rows_capacity <= 0)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "grouped_ffn: n_segs=%d rows=%d", n_segs, rows_capacity);
  if (mode == 0 && (!d_row_token || !d_row_weight))
    return WB_FAIL(WISP_ERR_INVALID_ARG, "grouped_ffn: mode 0 needs row_token and row_weight");
  if (((uintptr_t)d_xp | (uintptr_t)d_h) & 15)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "grouped_ffn: activation buffers must be 16-byte aligned");
  if ((uintptr_t)d_prepared & 255)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "grouped_ffn: prepared weights must be 256-byte aligned");
  if ((uintptr_t)d_workspace & 255)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "grouped_ffn: workspace must be 256-byte aligned");
  const GroupedWs ws = carve_grouped(n_segs, rows_capacity, M, I, d_workspace);
  if (workspace_bytes < ws.bytes)
    return WB_FAIL(WISP_ERR_INVALID_ARG, "grouped_ffn: workspace %zu < required %zu",
                   workspace_bytes, ws.bytes);

  const PreparedLayout PL = prepared_layout(cfg, n_entries);
  GemmParams gu, dn;
  memset(&gu, 0, sizeof gu);
  for (int i = 0; i < 6; i++) {
    if (!encode_rows_map3(&gu.tmap[i], d_xp, rows_capacity, M, 16 * (i + 1)))
      return WB_FAIL(WISP_ERR_CUDA, "grouped_ffn: cuTensorMapEncodeTiled failed (activations)");
  }
  gu.prepared = static_cast<const uint8_t*>(d_prepared);
  gu.p_flags = PL.flags;
  gu.p_scales = PL.scales;
  gu.p_zeros = PL.zeros;
  gu.p_mat_sc_bytes = PL.mat_sc_bytes;
  gu.segs = d_segs;
  gu.nseg = n_segs;
  gu.M = M;
  gu.I = I;
  gu.gs = gs;
  gu.h_out = reinterpret_cast<__half*>(d_h);
  gu.error_flag = d_error_flag;
  gu.counters = g_counters;
  dn = gu;
  dn.counters = g_counters ? g_counters + C_COUNT : nullptr;
  for (int i = 0; i < 6; i++) {
    if (!encode_rows_map3(&dn.tmap[i], d_h, rows_capacity, I, 16 * (i + 1)))
      return WB_FAIL(WISP_ERR_CUDA, "grouped_ffn: cuTensorMapEncodeTiled failed (H)");
  }
  dn.row_token = d_row_token;
  dn.row_weight = d_row_weight;
  dn.out = d_out;
  dn.mode = mode;

  const int sk_rows = wb::grouped_sk_rows(n_segs, n_entries);
  gu.tiles = ws.tiles_gu;
  dn.tiles = ws.tiles_dn;
  gu.tickets = ws.tickets;
  gu.partial = ws.partial;
  // Register path: gate/up cannot split K (SwiGLU needs whole sums), nor can
  // mode 1 (plain row stores); the weighted down projection splits K when it
  // has fewer than two units per SM. Tensor-core path: both projections split
  // K when their tiles fill fewer than half the SMs (gate/up through the
  // partial sums, the weighted down projection through its atomics; mode 1
  // does not split).
  PlanArgs pa;
  pa.segs = d_segs;
  pa.nseg = n_segs;
  pa.sk_rows = sk_rows;
  pa.mb_gu = I / (2 * kGuRows);           // pair tiles: 128 intermediate rows
  pa.mb_dn = (M + 2 * BM - 1) / (2 * BM);  // pair tiles: 256 output rows
  pa.per_gu = wb::skinny_units_gateup(I);
  pa.per_dn = wb::skinny_units_down(M);
  pa.cols = wb::skinny_cols();
  pa.ks_dn = mode == 0 ? 8 : 1;
  pa.nk_dn = wb::skinny_stages(I);
  pa.target = 2 * num_sms();
  const int npairs = grouped_pairs();
  pa.sms = npairs;   // the tensor-core kernels' K split fills the CTA pairs
  pa.split_gu = kMaxSplit;
  pa.split_dn = mode == 0 ? kMaxSplit : 1;
  pa.nraw_gu = M / kRawK;
  pa.nraw_dn = I / kRawK;
  pa.tickets = ws.tickets;
  pa.tiles_gu = ws.tiles_gu;
  pa.tiles_dn = ws.tiles_dn;
  pa.units_gu = ws.units_gu;
  pa.units_dn = ws.units_dn;
  // (the decode planner has written the register path's plans already)
  if (!plans_ready) wb::launch_k(plan_all_kernel, 4, 1024, 0, stream, pa);
  if (sk_rows > 0 && !xq_ready)
    wb::launch_k(quant_rows_kernel, dim3(n_segs, sk_rows), 128, 0, stream, d_segs, sk_rows,
                 reinterpret_cast<const __half*>(d_xp), M, ws.xq);
  CUtensorMap sk_xq[2], sk_hq[2];
  for (int i = 0; i < 2; i++) {
    if (!encode_q16_map(&sk_xq[i], ws.xq, rows_capacity, M, 8 << i) ||
        !encode_q16_map(&sk_hq[i], ws.hq, rows_capacity, I, 8 << i))
      return WB_FAIL(WISP_ERR_CUDA, "grouped_ffn: cuTensorMapEncodeTiled failed (token rows)");
  }
  wb::SkLaunch sk;
  sk.prepared = gu.prepared;
  sk.p_maps_sk = PL.maps_sk;
  sk.p_zbits = PL.zbits;
  sk.p_sk_scales = PL.sk_scales;
  sk.p_sk_zeros = PL.sk_zeros;
  sk.sk_gu_bytes = PL.sk_gu_bytes;
  sk.sk_dn_bytes = PL.sk_dn_bytes;
  sk.segs = d_segs;
  sk.nseg = n_segs;
  sk.n_entries = n_entries;
  sk.units_gu = ws.units_gu;
  sk.units_dn = ws.units_dn;
  sk.M = M;
  sk.I = I;
  sk.gs = gs;
  sk.xq_maps = sk_xq;
  sk.hq_maps = sk_hq;
  sk.hq = ws.hq;
  sk.row_token = d_row_token;
  sk.row_weight = d_row_weight;
  sk.out = d_out;
  sk.mode = mode;
  sk.error_flag = d_error_flag;
  // a one-token decode call: the decode planner wrote only q16 row 0
  sk.tok_row0 = (plans_ready && cfg->tokens == 1) ? 1 : 0;
  // diagnostics: the register-path kernel's counters follow the two
  // tensor-core kernels' blocks
  sk.counters = g_counters ? g_counters + 2 * C_COUNT : nullptr;

  // (the kernel itself balances its units over the CTAs it keeps)
  const int grid_gu = num_sms(), grid_dn = num_sms();
  // When no segment can exceed the routing threshold (max_seg_rows, an upper
  // bound the caller knows, e.g. the token count of a decode batch), the
  // tensor-core kernels would find no tiles: they are not launched.
  const bool tc = max_seg_rows > sk_rows;
  if (sk_rows > 0) WB_CUDA_CHECK(wb::launch_skinny(sk, 0, grid_gu, stream));
  if (tc) WB_CUDA_CHECK(launch_pairs<GATEUP>(npairs, stream, gu));
  if (sk_rows > 0) WB_CUDA_CHECK(wb::launch_skinny(sk, 1, grid_dn, stream));
  if (tc) WB_CUDA_CHECK(launch_pairs<DOWN>(npairs, stream, dn));
  WB_CUDA_CHECK(cudaGetLastError());
  return WISP_OK;
}
