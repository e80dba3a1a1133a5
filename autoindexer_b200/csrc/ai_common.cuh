// Shared device helpers of the chain-of-edits attention kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/ai_attn.h"

namespace ai {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Decoded block record (see AI_BLOCK_* in ai_attn.h).
struct Block {
  int row, s, e, key_off, kv_lo, flags, abs_lo, abs_hi;
  // Whether keys [j0, j1) include one of the block's abs keys.
  __device__ __forceinline__ bool abs_in(int j0, int j1) const {
    if (!(flags & AI_BLOCKF_ABS)) return false;
    if (abs_hi <= abs_lo) return true;
    return j0 < abs_hi && abs_lo < j1;
  }
};

__device__ __forceinline__ Block load_block(const int32_t* blocks, int id) {
  const int32_t* p = blocks + (int64_t)id * AI_BLOCK_FIELDS;
  Block b;
  b.row = p[AI_BLOCK_ROW];
  b.s = p[AI_BLOCK_START];
  b.e = p[AI_BLOCK_END];
  b.key_off = p[AI_BLOCK_KEY_OFF];
  b.kv_lo = p[AI_BLOCK_KV_LO];
  b.flags = p[AI_BLOCK_FLAGS];
  b.abs_lo = p[AI_BLOCK_ABS_LO];
  b.abs_hi = p[AI_BLOCK_ABS_HI];
  return b;
}

// First error wins; later errors do not overwrite it.
__device__ __forceinline__ void report(int32_t* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// Rotary table row of key_info, clamped into the table.  An out-of-range row
// is reported (AI_ERR_DEV_BOUNDS) and replaced by row 0.
__device__ __forceinline__ int key_row(uint32_t info, int n_pos, int32_t* status) {
  int r = (int)(info & AI_KEY_ROW_MASK);
  if (r >= n_pos) {
    report(status, AI_ERR_DEV_BOUNDS);
    r = 0;
  }
  return r;
}

// Work unit of the k-th round of a persistent CTA: rounds of gridDim.x units
// alternate direction (snake order), so that with units sorted longest first
// every CTA's total stays close to the mean.  A value >= the unit count ends
// the CTA's walk (only the last round can be partial).
__device__ __forceinline__ int snake_unit(int k) {
  const int G = (int)gridDim.x, c = (int)blockIdx.x;
  return k * G + ((k & 1) ? G - 1 - c : c);
}

// Query heads of one GQA group (G heads) packed into one 128-row tile for a
// work item of `rows` query rows: four heads of 32 rows, two of 64, or one.
__device__ __forceinline__ int pack_heads(int rows, int G) {
  if (G % 4 == 0 && rows <= 32) return 4;
  if (G % 2 == 0 && rows <= 64) return 2;
  return 1;
}

// Work units of one launch of the persistent forward / dQ kernels: the work
// items from item_base on, the first n_pack_items of them (items of at most
// 64 rows) as n_pack_units four-head units, the others as two-head units;
// n_units in all.  The abs split launches them once for the abs-block items
// (item_base 0; their key tiles without abs keys) and once for the rest.
struct UnitPlan {
  int item_base, n_pack_items, n_pack_units, n_units;
};

// Key tiles [ja, jb) (tiles of bn keys from kv_lo, the last one ending at
// kv_hi) that hold one of the block's abs keys: exactly the tiles for which
// Block::abs_in(k0, min(k0 + bn, kv_hi)) holds (a contiguous range, since the
// abs keys lie in [abs_lo, abs_hi)); ja = jb = 0 when there are none.
__device__ __forceinline__ void abs_tiles(const Block& blk, int kv_lo, int kv_hi, int bn, int& ja, int& jb) {
  ja = jb = 0;
  const int n = kv_hi > kv_lo ? (kv_hi - kv_lo + bn - 1) / bn : 0;
  if (!(blk.flags & AI_BLOCKF_ABS) || n == 0) return;
  if (blk.abs_hi <= blk.abs_lo) {
    jb = n;
    return;
  }
  if (blk.abs_lo >= kv_hi || blk.abs_hi <= kv_lo) return;
  const int a0 = blk.abs_lo < kv_lo ? 0 : (blk.abs_lo - kv_lo) / bn;
  const int a1 = min(n, (blk.abs_hi - kv_lo + bn - 1) / bn);
  if (a0 < a1) {
    ja = a0;
    jb = a1;
  }
}

// Number of CTAs that share the n abs tiles of a short abs item whose tile
// packs P heads (P CTAs per head group are launched): up to P chunks of at
// least min_tiles tiles each, 1 when the range is shorter (that CTA writes
// the final rows itself).  Chunk c takes tiles [n c / k, n (c + 1) / k).
__device__ __forceinline__ int abs_chunks(int n, int P, int min_tiles) {
  const int k = n / min_tiles;
  return k < 1 ? 1 : (k < P ? k : P);
}

// First chunk_cls entry of a block's rotation classes, or -1 when the block
// has none or the rotated copies are not in the workspace (`prerot` false).
__device__ __forceinline__ int block_classes(const AiAttnLayout& L, int block, bool prerot) {
  if (!prerot || L.n_rot_classes <= 0 || !L.blk_cls) return -1;
  return __ldg(L.blk_cls + block);
}

// Rotation class of chunk i of a block whose entries start at `base`; an
// index or class outside the tables is reported (AI_ERR_DEV_BOUNDS) and
// gives -1, which sends the chunk down the rotate-in-shared-memory path.
__device__ __forceinline__ int chunk_class(const AiAttnLayout& L, int base, int i, int32_t* status) {
  const int idx = base + i;
  if (base < 0 || idx >= L.n_chunk_cls) {
    if (base >= 0) report(status, AI_ERR_DEV_BOUNDS);
    return -1;
  }
  const int c = __ldg(L.chunk_cls + idx);
  if (c < 0 || c >= L.n_rot_classes) {
    report(status, AI_ERR_DEV_BOUNDS);
    return -1;
  }
  return c;
}

__device__ __forceinline__ int clamp_row(int r, int n_pos, int32_t* status) {
  if (r < 0 || r >= n_pos) {
    report(status, AI_ERR_DEV_BOUNDS);
    return 0;
  }
  return r;
}

}  // namespace ai
