// skinny.h -- interface between the grouped-FFN host code (grouped.cu) and
// the register-path kernel for small token groups (skinny.cu).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "wisp_b200.h"

namespace wb {

// Register-path activation rows ("q16 rows"). Per 128-K block of a row a
// 16-bit integer v with x ~= v * s, s = the block's max |x| / 32767. The row
// is stored stage by stage (256 K per stage) as five 128-byte lines:
//   lines 0-3: the stage's 256 values, 16 bytes per 8 consecutive K (one
//              packed weight word):
//     [hi(v0) hi(v2) hi(v4) hi(v6) | hi(v1) hi(v3) hi(v5) hi(v7) |
//      lo(v0) lo(v2) lo(v4) lo(v6) | lo(v1) lo(v3) lo(v5) lo(v7)]
//     with hi(v) = v >> 8 (signed byte), lo(v) = v & 255 (unsigned), so
//     v = 256 hi + lo; block b of the stage (b = 0, 1) is lines 2b, 2b+1;
//   line 4:    per block b, 16 bytes at 16 b: {s / 16, s * sum(v of its K
//              0-63), s * sum(v of K 64-127), 0} (the sums serve weights with
//              zero points); the rest of the line is unused.
// One 3D TMA box (128 bytes x rows x 5 lines) then brings a stage's token
// rows and their scales in a single copy.
constexpr int kQ16Block = 128;
constexpr int kQ16MetaFloats = 4;
constexpr int kQ16StageK = 256;
constexpr int kQ16LineBytes = 128;
constexpr int kQ16Lines = 5;
constexpr int kQ16StageBytes = kQ16Lines * kQ16LineBytes;

__host__ __device__ inline size_t q16_row_bytes(int K) {
  return (size_t)((K + kQ16StageK - 1) / kQ16StageK) * kQ16StageBytes;
}
// Byte offset, inside a q16 row, of the 16-byte chunk of packed word w
// (K 8w..8w+7 of the row).
__host__ __device__ inline size_t q16_word_offset(int w) {
  const int k = 8 * w;
  return (size_t)(k / kQ16StageK) * kQ16StageBytes + (size_t)(k % kQ16StageK) * 2;
}
// Byte offset of block b's metadata inside a q16 row.
__host__ __device__ inline size_t q16_meta_offset(int b) {
  return (size_t)(b / 2) * kQ16StageBytes + 4 * kQ16LineBytes + (size_t)(b % 2) * 16;
}

struct SkLaunch {
  const uint8_t* prepared;
  size_t p_maps_sk, p_zbits;
  size_t p_sk_scales, p_sk_zeros;   // per-unit-stage weight scales / zero points
  size_t sk_gu_bytes, sk_dn_bytes;  // per expert: its gate/up pair's and its down runs
  const WispSegment* segs;
  int nseg;
  int n_entries;
  const int32_t* units_gu;
  const int32_t* units_dn;
  int M, I, gs;
  const CUtensorMap* xq_maps;  // [2]: q16 rows of the gate/up input, boxes of 8 / 16 rows
  const CUtensorMap* hq_maps;  // [2]: q16 rows of H
  uint8_t* hq;                 // q16 H rows written by the gate/up phase
  const int* row_token;
  const float* row_weight;
  float* out;
  int mode;
  int* error_flag;
  unsigned long long* counters;
  // 1: a single-token decode call, whose rows all hold token 0; the gate/up
  // phase reads its token rows from row 0 of the q16 input, the only row the
  // decode planner writes.
  int tok_row0;
};

int skinny_max_rows();
int skinny_max_segs();
int skinny_max_entries();
int skinny_cols();
int skinny_stages(int K);
int skinny_units_gateup(int I);
int skinny_units_down(int M);
cudaError_t launch_skinny(const SkLaunch& L, int phase, int grid, cudaStream_t st);

}  // namespace wb
