// Forward of the chain-of-edits attention on sm_100a tensor cores
// (tcgen05.mma with TMEM accumulators, TMA tile loads), bf16 in / fp32
// accumulate, head_dim 128.
//
// One CTA computes one work item (block b, query rows [q0, q1) with
// q1 - q0 <= 128) for one query head, or for two or four heads of the same
// GQA group when the item has at most 64 or 32 rows (their rows share the
// 128 TMEM lanes and every K / V tile):
//   * Q rows are loaded by their owning thread, rotated by the row's query
//     position (fp32 cos/sin table) and written as bf16 into a 128-byte
//     swizzled K-major tile; the unrotated rows go to a second tile when the
//     block has abs keys.
//   * For every 128-key tile of the block's key range [kv_lo, min(e, q1)):
//     TMA brings K and V (128-byte swizzle); each thread rotates its key row in
//     place by the key's position *in this block* (key_info -> table row);
//     one thread issues S = Qrot.Krot^T (and S_abs = Q.Krot^T when the block
//     has abs keys) into TMEM; every thread owns one TMEM lane = one query row
//     and applies the abs select, the attention / causal mask and the online
//     softmax without cross-thread reductions; P (bf16) goes to a swizzled
//     smem tile and one thread issues O += P.V into TMEM.
//   * The running max is only moved (and O rescaled in TMEM) when it grows by
//     more than 2^8, so most tiles need no TMEM read-modify-write of O.
//
// Semantics restated from attention/reference.py:11-64, :96-141 (reference):
// logits of block rows use that block's key positions, abs columns use the
// unrotated query, a global causal mask, scale, softmax, P.V.  Rows past q1
// are computed on zero queries and discarded.
//
// Every wait on an mbarrier is bounded (~2 s of SM clocks); on expiry the
// kernel records AI_ERR_DEV_TIMEOUT in the status word, skips the remaining
// work, frees its TMEM and returns.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <math_constants.h>

#include "ai_common.cuh"
#include "ai_kernels.h"
#include "sm100_ptx.cuh"
#include "sm100_tile.cuh"

namespace ai {
namespace sm100 {

constexpr int D = 128;
constexpr int BM = 128;  // query rows per CTA = TMEM lanes
constexpr int BN = 128;  // keys per tile
constexpr int kThreads = 128;
constexpr uint32_t kHalf = BM * 128;  // one 64-element (128-byte) column block of a 128-row bf16 tile
constexpr uint32_t kTile = 2 * kHalf;  // 128 rows x 128 bf16
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColSabs = 128, kColO = 256;
constexpr long long kWaitCycles = 4000000000LL;
// Fewest 128-key abs tiles a chunk of a short abs item takes (a chunk costs
// its CTA's set-up and a partial row on top of its tiles).
constexpr int kFwdChunkTiles = 3;

struct Smem {
  static constexpr uint32_t Q = 0;
  static constexpr uint32_t QA = Q + kTile;
  static constexpr uint32_t K = QA + kTile;  // K / V buffer 0
  static constexpr uint32_t V = K + kTile;
  static constexpr uint32_t P = V + kTile;
  static constexpr uint32_t K1 = P + kTile;  // K / V buffer 1: tile j + 1 loads while tile j runs
  static constexpr uint32_t V1 = K1 + kTile;
  static constexpr uint32_t INFO = V1 + kTile;
  static constexpr uint32_t BAR_TMA = INFO + 4 * BN;  // two barriers, one per K / V buffer
  static constexpr uint32_t BAR_MMA = BAR_TMA + 16;
  static constexpr uint32_t TMEM_SLOT = BAR_MMA + 8;
  static constexpr uint32_t ABORT = TMEM_SLOT + 4;
  static constexpr uint32_t TOTAL = ABORT + 4;
};
constexpr size_t kSmemBytes = Smem::TOTAL + 1024;

using tile::pack8;
using tile::rotate8;

__device__ __forceinline__ uint32_t chunk_off(int r, int c) { return tile::chunk_off<BM>(r, c); }

__global__ void __launch_bounds__(kThreads, 1)
    fwd_kernel(const AiAttnFwdArgs a, const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
               const __grid_constant__ CUtensorMap tm_kc, const int prerot, float* __restrict__ part_o,
               float* __restrict__ part_lse) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = tile::align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid / 32;
  uint32_t* s_info = reinterpret_cast<uint32_t*>(sm + Smem::INFO);
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + Smem::ABORT);
  const uint32_t bar_tma = sbase + Smem::BAR_TMA, bar_mma = sbase + Smem::BAR_MMA;

  const AiAttnLayout& L = a.layout;
  const int32_t* item = L.fwd_items + 4 * (int64_t)blockIdx.x;
  const Block blk = load_block(L.blocks, item[0]);
  const int q0 = item[1], q1 = item[2];
  // A short item packs P heads of the group into the tile: thread tid is row
  // tid % (128 / P) of head y * P + tid / (128 / P).  Without the abs split
  // the CTAs y >= Hq / P return at once.  With it (part_o given), the P CTAs
  // y, y + Hq / P, ... of a head group each take one of up to P consecutive
  // chunks of the item's abs tiles (abs_chunks) and leave a partial row in
  // the workspace at row chunk * (128 / P) + r of the (item, head) slab,
  // which fwd_abs_combine_kernel merges: the longest abs ranges (up to a
  // whole edit chain's keys) no longer run serially on one SM.
  // An abs range shorter than two chunks of kFwdChunkTiles stays whole on
  // chunk 0's CTA (the others return at once).
  const int G = a.num_q_heads / a.num_kv_heads, P = pack_heads(q1 - q0, G), slot = BM / P;
  const int kv_hi = min(blk.e, q1);
  int y = (int)blockIdx.y, chunk = 0, n_chunks = 1;
  if (part_o != nullptr && P > 1) {
    chunk = y / (a.num_q_heads / P);
    y %= a.num_q_heads / P;
    int ja, jb;
    abs_tiles(blk, blk.kv_lo, kv_hi, BN, ja, jb);
    n_chunks = abs_chunks(jb - ja, P, kFwdChunkTiles);
    if (chunk >= n_chunks) return;
  } else if (y * P >= a.num_q_heads) {
    return;
  }
  const bool chunked = n_chunks > 1;
  const int h = y * P + tid / slot, hk = (y * P) / G, b = blk.row;
  const bool has_abs = (blk.flags & AI_BLOCKF_ABS) != 0;
  // The block's rotation classes: K tiles whose two chunks have one come rotated.
  const int cls = block_classes(L, item[0], prerot != 0);

  // Key tiles of this CTA: the block's, or with the abs split only those
  // holding abs keys (chunk 0 of a chunked item starts from the persistent
  // kernel's partial, the other chunks from nothing).
  const bool o_init = part_o != nullptr && chunk == 0;
  int j_begin = 0, j_end = kv_hi > blk.kv_lo ? (kv_hi - blk.kv_lo + BN - 1) / BN : 0;
  if (part_o != nullptr) {
    abs_tiles(blk, blk.kv_lo, kv_hi, BN, j_begin, j_end);
    if (chunked) {
      const int n = j_end - j_begin, jb = j_begin;
      j_begin = jb + n * chunk / n_chunks;
      j_end = jb + n * (chunk + 1) / n_chunks;
    }
  }

  // K and V of tile jt into buffer `buf` by TMA (K from its chunks' rotated
  // copies when it has them).  Tile jt + 1 loads while tile jt runs; its
  // buffer was last read by tile jt - 1's MMAs, complete by then.
  auto issue_tile = [&](int jt, int buf) {
    const int k0 = blk.kv_lo + jt * BN;
    const int c0 = cls >= 0 ? chunk_class(L, cls, 2 * jt, a.status) : -1;
    const int c1 = c0 >= 0 ? chunk_class(L, cls, 2 * jt + 1, a.status) : -1;
    const uint32_t kb = sbase + (buf ? Smem::K1 : Smem::K), vb = sbase + (buf ? Smem::V1 : Smem::V);
    const uint32_t bt = bar_tma + 8u * (uint32_t)buf;
    ptx::fence_proxy_async_smem();
    ptx::mbar_arrive_expect_tx(bt, 2 * kTile);
    if (c0 >= 0 && c1 >= 0) {
      ptx::tma_load_4d(kb, &tm_kc, bt, 0, 0, hk, c0);
      ptx::tma_load_4d(kb + kHalf / 2, &tm_kc, bt, 0, 0, hk, c1);
      ptx::tma_load_4d(kb + kHalf, &tm_kc, bt, 64, 0, hk, c0);
      ptx::tma_load_4d(kb + kHalf + kHalf / 2, &tm_kc, bt, 64, 0, hk, c1);
    } else {
      ptx::tma_load_4d(kb, &tm_k, bt, 0, k0, hk, b);
      ptx::tma_load_4d(kb + kHalf, &tm_k, bt, 64, k0, hk, b);
    }
    ptx::tma_load_4d(vb, &tm_v, bt, 0, k0, hk, b);
    ptx::tma_load_4d(vb + kHalf, &tm_v, bt, 64, k0, hk, b);
  };

  if (tid == 0) {
    ptx::mbar_init(bar_tma, 1);
    ptx::mbar_init(bar_tma + 8, 1);
    ptx::mbar_init(bar_mma, 1);
    *s_abort = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tm_k);
    ptx::prefetch_tmap(&tm_v);
    // The first tile loads while the query rows are set up.
    if (j_begin < j_end) issue_tile(j_begin, 0);
  }
  if (warp == 0) {
    ptx::tmem_alloc(sbase + Smem::TMEM_SLOT, kTmemCols);
    ptx::tmem_relinquish();
  }

  // Query row `tid`: rotated into Q, raw into QA (abs blocks only).
  {
    const int i = q0 + tid % slot;
    const __nv_bfloat16* Qrow =
        static_cast<const __nv_bfloat16*>(a.q.ptr) + b * a.q.stride_b + h * a.q.stride_h + (int64_t)i * a.q.stride_t;
    int p = 0;
    if (i < q1) p = clamp_row(L.q_pos[(int64_t)b * a.seq_len + i], L.n_pos, a.status);
    const float* cs = L.rope_cos + (int64_t)p * (D / 2);
    const float* sn = L.rope_sin + (int64_t)p * (D / 2);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 x1 = make_uint4(0, 0, 0, 0), x2 = x1, y1, y2;
      if (i < q1) {
        x1 = __ldg(reinterpret_cast<const uint4*>(Qrow + 8 * c));
        x2 = __ldg(reinterpret_cast<const uint4*>(Qrow + 64 + 8 * c));
      }
      rotate8(x1, x2, cs + 8 * c, sn + 8 * c, y1, y2);
      *reinterpret_cast<uint4*>(sm + Smem::Q + chunk_off(tid, c)) = y1;
      *reinterpret_cast<uint4*>(sm + Smem::Q + chunk_off(tid, c + 8)) = y2;
      if (has_abs) {
        *reinterpret_cast<uint4*>(sm + Smem::QA + chunk_off(tid, c)) = x1;
        *reinterpret_cast<uint4*>(sm + Smem::QA + chunk_off(tid, c + 8)) = x2;
      }
    }
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + Smem::TMEM_SLOT);
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  const float sl2 = a.scale * kLog2e;
  constexpr uint32_t idesc_qk = ptx::idesc_bf16_f32(BM, BN, false, false);
  constexpr uint32_t idesc_pv = ptx::idesc_bf16_f32(BM, D, false, true);
  const int i = q0 + tid % slot;
  float m_use = -CUDART_INF_F, l = 0.f;
  uint32_t ph_tma = 0, ph_mma = 0;  // ph_tma: bit b = phase of K / V buffer b
  int n_tiles = 0;
  bool aborted = false;

  // With the abs split the persistent kernel has run this item's key tiles
  // without abs keys and left each row's (O / l, log2-sum) partial: start
  // the online softmax from it (m = that sum, l = 1, O = the partial) and
  // run the tiles that hold abs keys only.
  if (o_init) {
    const int64_t prow = ((int64_t)blockIdx.x * a.num_q_heads + h) * BM + (i - q0);
    const bool have = i < q1;
    const float lp = have ? part_lse[prow] : -CUDART_INF_F;
    m_use = lp;
    l = lp > -CUDART_INF_F ? 1.f : 0.f;
#pragma unroll
    for (int cc = 0; cc < D / 32; ++cc) {
      uint32_t r[32];
#pragma unroll
      for (int x = 0; x < 32; x += 4) {
        const float4 v = (have && l > 0.f) ? *reinterpret_cast<const float4*>(part_o + prow * D + 32 * cc + x)
                                           : make_float4(0.f, 0.f, 0.f, 0.f);
        r[x] = __float_as_uint(v.x);
        r[x + 1] = __float_as_uint(v.y);
        r[x + 2] = __float_as_uint(v.z);
        r[x + 3] = __float_as_uint(v.w);
      }
      ptx::tmem_st32(tmem + lane_base + kColO + 32 * cc, r);
    }
    ptx::tmem_wait_st();
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
  }

  for (int jt = j_begin, k0 = blk.kv_lo + j_begin * BN; jt < j_end; ++jt, k0 += BN) {
    const int buf = (jt - j_begin) & 1;
    const uint32_t kcur = buf ? Smem::K1 : Smem::K, vcur = buf ? Smem::V1 : Smem::V;
    // Only a tile that holds one of the block's abs keys needs S_abs.
    const bool tabs = blk.abs_in(k0, min(k0 + BN, kv_hi));
    const int c0 = cls >= 0 ? chunk_class(L, cls, 2 * jt, a.status) : -1;
    const int c1 = c0 >= 0 ? chunk_class(L, cls, 2 * jt + 1, a.status) : -1;
    const bool ctile = c0 >= 0 && c1 >= 0;
    // 1. The next tile's K and V start loading; this tile's have been
    // requested one tile ago.  Key row `tid`'s flags are read meanwhile.
    if (tid == 0 && jt + 1 < j_end) issue_tile(jt + 1, buf ^ 1);
    const int j = k0 + tid;
    const uint32_t info = j < kv_hi ? (uint32_t)L.key_info[blk.key_off + j] : 0u;
    if (!ptx::mbar_wait(bar_tma + 8u * (uint32_t)buf, (ph_tma >> buf) & 1u, kWaitCycles)) {
      report(a.status, AI_ERR_DEV_TIMEOUT);
      *s_abort = 1;
    }
    ph_tma ^= 1u << buf;
    __syncthreads();
    if (*s_abort) {
      aborted = true;
      break;
    }

    // 2. Rotate key row `tid` in place by its position in this block (the
    // fp16 (cos, sin) table, as the rotated copies are made).
    {
      if (j < kv_hi) {
        if (!ctile) {
          const int p = key_row(info, L.n_pos, a.status);
          const uint4* tp = static_cast<const uint4*>(L.rope_cs16) + (int64_t)p * (D / 8);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint4* pa = reinterpret_cast<uint4*>(sm + kcur + chunk_off(tid, c));
            uint4* pb = reinterpret_cast<uint4*>(sm + kcur + chunk_off(tid, c + 8));
            uint4 y1, y2;
            tile::rotate8h(*pa, *pb, __ldg(tp + 2 * c), __ldg(tp + 2 * c + 1), y1, y2);
            *pa = y1;
            *pb = y2;
          }
        }
      }
      s_info[tid] = info;
    }
    ptx::fence_proxy_async_smem();
    __syncthreads();

    // 3. S = Qrot . Krot^T (and S_abs = Q . Krot^T) into TMEM.
    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (uint32_t)(kk >> 2) * kHalf + (uint32_t)(kk & 3) * 32u;
        ptx::mma_ss(tmem + kColS, ptx::sdesc_sw128(sbase + Smem::Q + off, 16, 1024),
                    ptx::sdesc_sw128(sbase + kcur + off, 16, 1024), idesc_qk, kk > 0);
      }
      if (tabs) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(kk >> 2) * kHalf + (uint32_t)(kk & 3) * 32u;
          ptx::mma_ss(tmem + kColSabs, ptx::sdesc_sw128(sbase + Smem::QA + off, 16, 1024),
                      ptx::sdesc_sw128(sbase + kcur + off, 16, 1024), idesc_qk, kk > 0);
        }
      }
      ptx::mma_commit(bar_mma);
    }
    if (!ptx::mbar_wait(bar_mma, ph_mma, kWaitCycles)) {
      report(a.status, AI_ERR_DEV_TIMEOUT);
      *s_abort = 1;
    }
    ph_mma ^= 1;
    __syncthreads();
    if (*s_abort) {
      aborted = true;
      break;
    }
    ptx::tc_fence_after();

    // 4. Online softmax of row i (TMEM lane tid).
    float s[BN];
#pragma unroll
    for (int cc = 0; cc < BN / 32; ++cc) {
      uint32_t r[32];
      ptx::tmem_ld32(tmem + lane_base + kColS + 32 * cc, r);
      ptx::tmem_wait_ld();
#pragma unroll
      for (int x = 0; x < 32; ++x) s[32 * cc + x] = __uint_as_float(r[x]);
      if (tabs) {
        ptx::tmem_ld32(tmem + lane_base + kColSabs + 32 * cc, r);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int x = 0; x < 32; ++x)
          if (s_info[32 * cc + x] & AI_KEY_ABS) s[32 * cc + x] = __uint_as_float(r[x]);
      }
    }
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int c = 0; c < BN; ++c) {
      const uint32_t info = s_info[c];
      const bool valid = (info & AI_KEY_ATTN) && (k0 + c <= i) && (i < q1);
      s[c] = valid ? s[c] * sl2 : -CUDART_INF_F;
      mx = fmaxf(mx, s[c]);
    }
    const float m_new = fmaxf(m_use, mx);
    float alpha = 1.f;
    bool rescale = false;
    if (m_new > m_use + 8.f) {
      if ((n_tiles > 0 || o_init) && l > 0.f) {
        alpha = ptx::ex2(m_use - m_new);
        rescale = true;
      }
      m_use = m_new;
    }
    // TMEM ld/st are warp-collective: rescale the whole warp if any lane needs it.
    if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t r[32];
        ptx::tmem_ld32(tmem + lane_base + kColO + 32 * cc, r);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int x = 0; x < 32; ++x) r[x] = __float_as_uint(__uint_as_float(r[x]) * alpha);
        ptx::tmem_st32(tmem + lane_base + kColO + 32 * cc, r);
      }
      ptx::tmem_wait_st();
    }
    l *= alpha;
    float sum = 0.f;
#pragma unroll
    for (int c8 = 0; c8 < BN / 8; ++c8) {
      float pv[8];
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        const float v = s[8 * c8 + x];
        pv[x] = (v == -CUDART_INF_F) ? 0.f : ptx::ex2(v - m_use);
        sum += pv[x];
      }
      *reinterpret_cast<uint4*>(sm + Smem::P + chunk_off(tid, c8)) = pack8(pv);
    }
    l += sum;
    ptx::fence_proxy_async_smem();
    ptx::tc_fence_before();
    __syncthreads();

    // 5. O += P . V (P K-major from smem, V MN-major from smem).
    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        const uint32_t aoff = (uint32_t)(kk >> 2) * kHalf + (uint32_t)(kk & 3) * 32u;
        const uint32_t boff = (uint32_t)kk * 2048u;  // 16 key rows of 128 bytes
        ptx::mma_ss(tmem + kColO, ptx::sdesc_sw128(sbase + Smem::P + aoff, 16, 1024),
                    ptx::sdesc_sw128(sbase + vcur + boff, kHalf, 1024), idesc_pv,
                    (n_tiles > 0 || o_init || kk > 0) ? 1u : 0u);
      }
      ptx::mma_commit(bar_mma);
    }
    if (!ptx::mbar_wait(bar_mma, ph_mma, kWaitCycles)) {
      report(a.status, AI_ERR_DEV_TIMEOUT);
      *s_abort = 1;
    }
    ph_mma ^= 1;
    __syncthreads();
    if (*s_abort) {
      aborted = true;
      break;
    }
    ptx::tc_fence_after();
    ++n_tiles;
  }

  // Epilogue: O / l -> bf16 row, lse; a chunk leaves its partial row
  // (O / l in fp32, log2-sum) for fwd_abs_combine_kernel instead.
  if (!aborted && chunked) {
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int64_t prow = ((int64_t)blockIdx.x * a.num_q_heads + h) * BM + chunk * slot + (i - q0);
#pragma unroll
    for (int cc = 0; cc < D / 32; ++cc) {
      uint32_t r[32];
      if (n_tiles > 0 || o_init) {
        ptx::tmem_ld32(tmem + lane_base + kColO + 32 * cc, r);
        ptx::tmem_wait_ld();
      } else {
#pragma unroll
        for (int x = 0; x < 32; ++x) r[x] = 0u;
      }
      if (i < q1) {
#pragma unroll
        for (int x = 0; x < 32; x += 4)
          *reinterpret_cast<float4*>(part_o + prow * D + 32 * cc + x) =
              make_float4(__uint_as_float(r[x]) * inv, __uint_as_float(r[x + 1]) * inv,
                          __uint_as_float(r[x + 2]) * inv, __uint_as_float(r[x + 3]) * inv);
      }
    }
    if (i < q1) part_lse[prow] = l > 0.f ? m_use + log2f(l) : -CUDART_INF_F;
  } else if (!aborted) {
    __nv_bfloat16* Orow =
        static_cast<__nv_bfloat16*>(a.out.ptr) + b * a.out.stride_b + h * a.out.stride_h + (int64_t)i * a.out.stride_t;
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int cc = 0; cc < D / 32; ++cc) {
      uint32_t r[32];
      if (n_tiles > 0 || o_init) {
        ptx::tmem_ld32(tmem + lane_base + kColO + 32 * cc, r);
        ptx::tmem_wait_ld();
      } else {
#pragma unroll
        for (int x = 0; x < 32; ++x) r[x] = 0u;
      }
      if (i < q1) {
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float f[8];
#pragma unroll
          for (int x = 0; x < 8; ++x) f[x] = __uint_as_float(r[8 * c8 + x]) * inv;
          *reinterpret_cast<uint4*>(Orow + 32 * cc + 8 * c8) = pack8(f);
        }
      }
    }
    if (i < q1)
      a.lse[((int64_t)b * a.num_q_heads + h) * a.seq_len + i] =
          l > 0.f ? (m_use + log2f(l)) * kLn2 : -CUDART_INF_F;
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// Merges the chunk partials fwd_kernel left for the abs items it ran
// chunked (P = heads packed per tile > 1, more than one chunk): per row, in
// chunk order (so the result does not depend on the launch order of the
// chunks),
//   lse2 = log2 sum_c 2^lse2_c,  O = sum_c 2^(lse2_c - lse2) (O / l)_c,
// then the bf16 output row and lse.  Grid (abs items, query heads); thread d
// owns dimension d of every row of the item.
__global__ void __launch_bounds__(D) fwd_abs_combine_kernel(const AiAttnFwdArgs a, const float* __restrict__ part_o,
                                                             const float* __restrict__ part_lse) {
  const AiAttnLayout& L = a.layout;
  const int it = (int)blockIdx.x, h = (int)blockIdx.y, d = (int)threadIdx.x;
  const int32_t* item = L.fwd_items + 4 * (int64_t)it;
  const Block blk = load_block(L.blocks, item[0]);
  const int b = blk.row, q0 = item[1], q1 = item[2];
  const int G = a.num_q_heads / a.num_kv_heads, P = pack_heads(q1 - q0, G), slot = BM / P;
  if (P == 1) return;  // run whole by fwd_kernel
  int ja, jb;
  abs_tiles(blk, blk.kv_lo, min(blk.e, q1), BN, ja, jb);
  const int nc = abs_chunks(jb - ja, P, kFwdChunkTiles);
  if (nc == 1) return;  // finished by its one CTA
  const int64_t base = ((int64_t)it * a.num_q_heads + h) * BM;
  for (int r = 0; r < q1 - q0; ++r) {
    float l2[4], m = -CUDART_INF_F;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      l2[c] = c < nc ? part_lse[base + c * slot + r] : -CUDART_INF_F;
      m = fmaxf(m, l2[c]);
    }
    float o = 0.f, w_sum = 0.f;
    if (m > -CUDART_INF_F) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (c < nc && l2[c] > -CUDART_INF_F) {
          const float w = exp2f(l2[c] - m);
          w_sum += w;
          o += w * part_o[(base + c * slot + r) * D + d];
        }
      }
    }
    const int i = q0 + r;
    __nv_bfloat16* Orow =
        static_cast<__nv_bfloat16*>(a.out.ptr) + b * a.out.stride_b + h * a.out.stride_h + (int64_t)i * a.out.stride_t;
    Orow[d] = __float2bfloat16_rn(w_sum > 0.f ? o / w_sum : 0.f);
    if (d == 0)
      a.lse[((int64_t)b * a.num_q_heads + h) * a.seq_len + i] =
          w_sum > 0.f ? (m + log2f(w_sum)) * kLn2 : -CUDART_INF_F;
  }
}

// ---------------------------------------------------------------------------
// Warp-specialised forward for blocks without abs keys (fwd_pers_kernel).
//
// Work unit = one work item (block, <= 128 query rows) x two query heads of
// the same GQA group, so every rotated K tile and every V tile feeds 256 query
// rows.  384 threads in roles:
//   warps 0-3   softmax of head 2y     (thread = query row = TMEM lane)
//   warps 4-7   softmax of head 2y + 1
//   warp  8     TMA producer: K and V tiles into a 2-deep ring
//   warp  9     MMA issuer and TMEM owner
//   warps 10-11 rotate each K tile in place by its keys' block positions
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
// Softmax t reads S_t, writes P_t (bf16, two per column) over the first 64
// columns of S_t, and the PV MMA takes P_t straight from TMEM.  MMA order
// per key tile j: PV0(j), S0(j+1), PV1(j), S1(j+1): while one softmax group
// works the tensor core runs the other group's MMAs.  S_t(j+1) overwrites
// P_t right after PV_t(j) read it: tcgen05.mma ops issued by one thread
// execute in issue order, so no wait on PV_t(j) is needed, and the S_t(j+1)
// commit (which tracks every earlier MMA) also tells softmax t that PV_t(j)
// is done with O_t before it may rescale O_t.
// The MMA warp runs converged: descriptors are computed by all 32 lanes (so
// they stay warp-uniform) and elect.sync picks the lane that issues.
// ---------------------------------------------------------------------------
namespace ws {
constexpr uint32_t Q0 = 0, Q1 = kTile, KB = 2 * kTile, VB = 4 * kTile;  // K ring at KB, V ring at VB
constexpr uint32_t INFO = 6 * kTile;                                    // [2][128] u32
constexpr uint32_t C_S0 = 0, C_S1 = 128, C_O0 = 256, C_O1 = 384;
}  // namespace ws

// ---------------------------------------------------------------------------
// Persistence: one CTA per SM walks the work units in a snake order (unit =
// work item x pair of query heads; items are longest first, and the snake
// evens out the sum of unit lengths per CTA).  Roles and tiles as above;
// what carries across units:
//   * tile barriers (K/V ring, S, P, O commits) count phases by the CTA's
//     running tile index g, unit barriers by its running unit index k;
//   * the next unit's Q tiles are loaded as soon as the current unit's last
//     S MMAs are done (Q_EMPTY), and its K/V tiles stream into the ring
//     behind the current unit's — the load latency of a unit start hides
//     behind the end of the previous unit;
//   * the first PV of a unit (accumulate = 0) overwrites O_t, so it waits
//     until softmax group t has read the previous unit's O_t (O_FREE);
//   * barriers, TMEM allocation and tensor-map prefetch happen once per CTA.
// ---------------------------------------------------------------------------
namespace pf {
using ws::Q0;
using ws::Q1;
using ws::KB;
using ws::VB;
using ws::INFO;
using ws::C_S0;
using ws::C_S1;
using ws::C_O0;
using ws::C_O1;
// 384 threads = three whole warpgroups (the register split below is per
// warpgroup): warps 0-7 softmax, 8 TMA producer, 9 MMA, 10-11 K rotation (two
// key rows per thread).  Launched at 168 registers a thread (64,512 for the
// block), the softmax warpgroups raise theirs to 200 (a row's 128 scores stay
// in registers) and warpgroup 2 lowers its to 104: 256 x 200 + 128 x 104.
constexpr int kThreads = 384;
constexpr uint32_t kRegLaunch = 168, kRegSoftmax = 200, kRegOther = 104;
static_assert(256 * kRegSoftmax + 128 * kRegOther <= kThreads * kRegLaunch, "register split");
// Output staging (128 rows x 64 bf16, 128-byte swizzle, 16 KB) per softmax
// group: a full unit's O_t leaves as two 64-column TMA stores through its
// group's own buffer, so neither group waits for the other's stores.
constexpr uint32_t OSTAGE = INFO + 2 * 4 * BN;
constexpr uint32_t BARS = OSTAGE + kTile;
// K and V tiles have their own full / empty barriers: a K slot is released
// when the second head's S MMAs of its tile are done and a V slot when the
// second head's PV MMAs are, so the K load of tile j + 2 starts about a
// thousand cycles before the V load and has as long to land as the V load.
enum Bar { K_FULL = 0, K_READY = 2, K_EMPTY = 4, S_FULL = 6, P_READY = 8, O_DONE = 10, O_FREE = 12, Q_READY = 14,
           Q_EMPTY = 15, SFREE0 = 16, SFREE1 = 17, STG0 = 18, STG1 = 19, FINAL = 20, V_FULL = 21, V_EMPTY = 23,
           N_BARS = 25 };
// Key flags (1 = the key may be attended) of the last four K tiles, slot
// g % 4 for tile g: the rotation warps fill tile g + 2's while the softmax
// may still read tile g's and g + 1's.
constexpr int kInfoSlots = 4;
static_assert(kInfoSlots * BN <= 2 * 4 * BN, "key flags fit the INFO area");
constexpr uint32_t TMEM_SLOT = BARS + 8 * N_BARS;
constexpr uint32_t ABORT = TMEM_SLOT + 4;
constexpr uint32_t TOTAL = ABORT + 4;
constexpr size_t kSmem = TOTAL + 1024;
constexpr long long kWait = 1000000000LL;
static_assert(kSmem <= 227 * 1024, "shared memory budget");

// One work unit: rows [q0, q1) of a block x four query heads h0 .. h0 + 3 of
// one GQA group (pk = 2: an item of at most 64 rows, tile t holds heads
// h0 + 2t in lanes 0-63 and h0 + 2t + 1 in lanes 64-127) or x two query heads
// h0, h0 + 1 (pk = 1: tile t holds head h0 + t in all 128 lanes).  The
// n_pack_units packed units come first (the short items follow the abs items
// in the work list), then the two-head units of the remaining items.
struct Unit {
  Block blk;
  int it;   // work item
  int q0, q1, h0, pk, hk, kv_lo, kv_hi, n;
  int ja, jb;  // an abs-block unit skips key tiles [ja, jb) (they hold abs keys); n counts the others
  int cls;  // the block's first rotation-class entry (chunk_cls), -1: none
  bool masked, k_pre, abs;
};

// Key tile of the unit's j-th tile (abs-block units skip [ja, jb)).
__device__ __forceinline__ int unit_tile(const Unit& w, int j) { return j < w.ja ? j : j + (w.jb - w.ja); }

// Rotation classes of the two 64-key chunks of K tile j of a unit: a tile
// whose chunks both have a class is read rotated from the class copies.
__device__ __forceinline__ bool class_tile(const AiAttnLayout& L, const Unit& w, int j, int32_t* status, int& c0,
                                           int& c1) {
  if (w.cls < 0) return false;
  const int jt = unit_tile(w, j);
  c0 = chunk_class(L, w.cls, 2 * jt, status);
  c1 = chunk_class(L, w.cls, 2 * jt + 1, status);
  return c0 >= 0 && c1 >= 0;
}

// Head and query row of TMEM lane r of tile t.
__device__ __forceinline__ int unit_head(const Unit& w, int t, int r) {
  return w.pk == 2 ? w.h0 + 2 * t + (r >> 6) : w.h0 + t;
}
__device__ __forceinline__ int unit_row(const Unit& w, int r) { return w.q0 + (w.pk == 2 ? (r & 63) : r); }

template <bool kAbs>
__device__ __forceinline__ Unit load_unit(const AiAttnFwdArgs& a, int u, int prerot, const UnitPlan& up) {
  const AiAttnLayout& L = a.layout;
  const int hpairs = a.num_q_heads / 2, hquads = a.num_q_heads / 4, G = a.num_q_heads / a.num_kv_heads;
  int it;
  Unit w;
  w.abs = kAbs;
  if (u < up.n_pack_units) {
    it = up.item_base + u / hquads;
    w.h0 = 4 * (u % hquads);
    w.pk = 2;
  } else {
    const int v = u - up.n_pack_units;
    it = up.item_base + up.n_pack_items + v / hpairs;
    w.h0 = 2 * (v % hpairs);
    w.pk = 1;
  }
  w.it = it;
  const int32_t* item = L.fwd_items + 4 * (int64_t)it;
  w.blk = load_block(L.blocks, item[0]);
  w.q0 = item[1];
  w.q1 = item[2];
  w.hk = w.h0 / G;
  w.kv_lo = w.blk.kv_lo;
  w.kv_hi = min(w.blk.e, w.q1);
  w.n = w.kv_hi > w.kv_lo ? (w.kv_hi - w.kv_lo + BN - 1) / BN : 0;
  w.ja = w.jb = 0;
  if (kAbs) {
    abs_tiles(w.blk, w.kv_lo, w.kv_hi, BN, w.ja, w.jb);
    w.n -= w.jb - w.ja;
  }
  w.masked = (w.blk.flags & AI_BLOCKF_MASKED) != 0;
  w.k_pre = prerot && (w.blk.flags & AI_BLOCKF_OWNPOS);
  w.cls = w.k_pre ? -1 : block_classes(L, item[0], prerot != 0);
  return w;
}
}  // namespace pf

// kAbs: the units are the abs-block items' key tiles without abs keys
// (partial rows into part_o / part_lse); otherwise the other items, whole.
template <bool kAbs>
__global__ void __launch_bounds__(pf::kThreads, 1)
    fwd_pers_kernel(const AiAttnFwdArgs a, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_qr,
                    const __grid_constant__ CUtensorMap tm_kr, const __grid_constant__ CUtensorMap tm_o,
                    const __grid_constant__ CUtensorMap tm_qr64, const __grid_constant__ CUtensorMap tm_kc,
                    const int prerot, const UnitPlan up, float* __restrict__ part_o, float* __restrict__ part_lse) {
  using namespace pf;
  // The launch after this one (the other persistent launch of the split)
  // reads nothing this one writes: let its CTAs take the SMs these leave.
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int n_units = up.n_units;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = tile::align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  uint8_t* s_flag = sm + INFO;
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + ABORT);
  auto bar = [&](int i) { return sbase + BARS + 8u * (uint32_t)i; };
  const AiAttnLayout& L = a.layout;

  if (tid == 0) {
    for (int i = 0; i < N_BARS; ++i) {
      uint32_t count = 1;
      if (i == K_READY || i == K_READY + 1) count = 64;
      if (i == P_READY || i == P_READY + 1 || i == O_FREE || i == O_FREE + 1 ||
          i == STG0 || i == STG1)
        count = 128;
      if (i == Q_READY) count = prerot ? 1 : 256;
      ptx::mbar_init(bar(i), count);
    }
    *s_abort = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 9) {
    ptx::tmem_alloc(sbase + TMEM_SLOT, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + TMEM_SLOT);
  if (warp < 8)
    ptx::setmaxnreg_inc<kRegSoftmax>();
  else
    ptx::setmaxnreg_dec<kRegOther>();

  auto wait = [&](int i, uint32_t parity) -> bool {
    if (*s_abort) return false;
    if (!ptx::mbar_wait(bar(i), parity, kWait)) {
      report(a.status, AI_ERR_DEV_TIMEOUT);
      *s_abort = 1;
      return false;
    }
    return true;
  };

  if (warp < 8) {
    // ------------------------------------------------------------ softmax
    const int t = warp / 4, r = tid % 128;
    const uint32_t lane_base = (uint32_t)((warp % 4) * 32) << 16;
    const uint32_t c_s = t ? C_S1 : C_S0, c_o = t ? C_O1 : C_O0;
    const float sl2 = a.scale * kLog2e;
    const float2 sl2x2 = make_float2(sl2, sl2);
    int g = 0, k = 0, ko = 0;  // ko: units with key tiles so far (O_DONE phases)
    int nst = 0;               // this group's staging-buffer uses
    // The next unit's description is read from global memory while this
    // unit's last PV MMAs run (before the epilogue's O_DONE wait).
    Unit w_next{};
    if (snake_unit(0) < n_units) w_next = load_unit<kAbs>(a, snake_unit(0), prerot, up);
    bool store_pending = false;  // thread 0: the last TMA store's smem read not yet waited for
    for (int u = snake_unit(k); u < n_units && !*s_abort; u = snake_unit(++k)) {
      const Unit w = w_next;
      const int i = unit_row(w, r), h = unit_head(w, t, r), b = w.blk.row;
      if (!prerot) {
        // Q rows of this unit (rotated): the previous unit's S MMAs must be
        // done reading Q_t.
        if (k > 0 && !wait(Q_EMPTY, (k - 1) & 1)) break;
        const __nv_bfloat16* Qrow = static_cast<const __nv_bfloat16*>(a.q.ptr) + b * a.q.stride_b +
                                    h * a.q.stride_h + (int64_t)i * a.q.stride_t;
        int p = 0;
        if (i < w.q1) p = clamp_row(L.q_pos[(int64_t)b * a.seq_len + i], L.n_pos, a.status);
        const uint4* tab =
            reinterpret_cast<const uint4*>(static_cast<const __half2*>(L.rope_cs16) + (int64_t)p * (D / 2));
        const uint32_t qt = t ? Q1 : Q0;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint4 x1[4], x2[4], cs[8];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int cc = 4 * hf + c;
            x1[c] = i < w.q1 ? __ldg(reinterpret_cast<const uint4*>(Qrow + 8 * cc)) : make_uint4(0, 0, 0, 0);
            x2[c] = i < w.q1 ? __ldg(reinterpret_cast<const uint4*>(Qrow + 64 + 8 * cc)) : make_uint4(0, 0, 0, 0);
            cs[2 * c] = __ldg(tab + 2 * cc);
            cs[2 * c + 1] = __ldg(tab + 2 * cc + 1);
          }
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int cc = 4 * hf + c;
            uint4 y1, y2;
            tile::rotate8h(x1[c], x2[c], cs[2 * c], cs[2 * c + 1], y1, y2);
            *reinterpret_cast<uint4*>(sm + qt + chunk_off(r, cc)) = y1;
            *reinterpret_cast<uint4*>(sm + qt + chunk_off(r, cc + 8)) = y2;
          }
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(bar(Q_READY));
      }
      float m_use = -CUDART_INF_F, l = 0.f;
      int done = 0;
      for (int j = 0; j < w.n; ++j) {
        const int gj = g + j, k0 = w.kv_lo + unit_tile(w, j) * BN;
        if (!wait(S_FULL + t, gj & 1)) break;
        ptx::tc_fence_after();
        const bool fast = !w.masked && (k0 + BN <= w.kv_hi) && (k0 + BN - 1 <= w.q0);
        const int lim = min(i - k0, w.kv_hi - 1 - k0);
        const uint8_t* info = s_flag + (gj & (kInfoSlots - 1)) * BN;
        // The row's 128 scores, read from TMEM once (cols 32 q + x in sq[x]).
        uint32_t s0[32], s1[32], s2[32], s3[32];
        ptx::tmem_ld32(tmem + lane_base + c_s, s0);
        ptx::tmem_ld32(tmem + lane_base + c_s + 32, s1);
        ptx::tmem_ld32(tmem + lane_base + c_s + 64, s2);
        ptx::tmem_ld32(tmem + lane_base + c_s + 96, s3);
        ptx::tmem_wait_ld();
        if (!fast && !w.masked) {
#pragma unroll
          for (int x = 0; x < 32; ++x) {
            if (x > lim) s0[x] = 0xff800000u;  // -inf
            if (x + 32 > lim) s1[x] = 0xff800000u;
            if (x + 64 > lim) s2[x] = 0xff800000u;
            if (x + 96 > lim) s3[x] = 0xff800000u;
          }
        } else if (w.masked) {
#pragma unroll
          for (int x = 0; x < 32; ++x) {
            if (!(info[x] && x <= lim)) s0[x] = 0xff800000u;
            if (!(info[x + 32] && x + 32 <= lim)) s1[x] = 0xff800000u;
            if (!(info[x + 64] && x + 64 <= lim)) s2[x] = 0xff800000u;
            if (!(info[x + 96] && x + 96 <= lim)) s3[x] = 0xff800000u;
          }
        }
        float mxa = -CUDART_INF_F, mxb = -CUDART_INF_F, mxc = -CUDART_INF_F, mxd = -CUDART_INF_F;
#pragma unroll
        for (int x = 0; x < 32; x += 2) {
          mxa = ptx::fmax3(mxa, __uint_as_float(s0[x]), __uint_as_float(s0[x + 1]));
          mxb = ptx::fmax3(mxb, __uint_as_float(s1[x]), __uint_as_float(s1[x + 1]));
          mxc = ptx::fmax3(mxc, __uint_as_float(s2[x]), __uint_as_float(s2[x + 1]));
          mxd = ptx::fmax3(mxd, __uint_as_float(s3[x]), __uint_as_float(s3[x + 1]));
        }
        const float mx = fmaxf(fmaxf(mxa, mxb), fmaxf(mxc, mxd));
        const float m_new = fmaxf(m_use, mx * sl2);
        float alpha = 1.f;
        bool rescale = false;
        if (m_new > m_use + 8.f) {
          if (j > 0 && l > 0.f) {
            alpha = ptx::ex2(m_use - m_new);
            rescale = true;
          }
          m_use = m_new;
        }
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int cc = 0; cc < D / 16; ++cc) {
            uint32_t rr[16];
            ptx::tmem_ld16(tmem + lane_base + c_o + 16 * cc, rr);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int x = 0; x < 16; ++x) rr[x] = __float_as_uint(__uint_as_float(rr[x]) * alpha);
            ptx::tmem_st16(tmem + lane_base + c_o + 16 * cc, rr);
          }
        }
        l *= alpha;
        const float msub = m_use == -CUDART_INF_F ? 0.f : m_use;
        const float2 nm2 = make_float2(-msub, -msub);
        float2 suma = make_float2(0.f, 0.f), sumb = make_float2(0.f, 0.f);
        // P (bf16 pairs) over S columns [0, 64): column 16 q + x holds keys
        // 32 q + 2 x and 32 q + 2 x + 1 (the PV MMA's A operand); each score
        // array is done with once its 16 columns are stored.
        auto emit = [&](const uint32_t (&ra)[32], uint32_t col, float2& sum) {
          uint32_t pk[16];
#pragma unroll
          for (int x = 0; x < 16; ++x) {
            const float2 a01 =
                __ffma2_rn(make_float2(__uint_as_float(ra[2 * x]), __uint_as_float(ra[2 * x + 1])), sl2x2, nm2);
            const float2 p01 = make_float2(ptx::ex2(a01.x), ptx::ex2(a01.y));
            sum = __fadd2_rn(sum, p01);
            pk[x] = tile::pack2(p01.x, p01.y);
          }
          ptx::tmem_st16(tmem + lane_base + c_s + col, pk);
        };
        emit(s0, 0, suma);
        emit(s1, 16, sumb);
        emit(s2, 32, suma);
        emit(s3, 48, sumb);
        l += (suma.x + suma.y) + (sumb.x + sumb.y);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(P_READY + t));
        done = j + 1;
      }
      if (done != w.n) break;
      if (snake_unit(k + 1) < n_units) w_next = load_unit<kAbs>(a, snake_unit(k + 1), prerot, up);
      // Epilogue: O_t / l.  O_t is read into registers, then released to the
      // next unit's first PV before the global stores.
      bool have_o = false;
      if (w.n > 0) {
        have_o = wait(O_DONE + t, (uint32_t)ko & 1u);
        ++ko;
        if (!have_o) break;
      }
      ptx::tc_fence_after();
      __nv_bfloat16* Orow = static_cast<__nv_bfloat16*>(a.out.ptr) + b * a.out.stride_b + h * a.out.stride_h +
                            (int64_t)i * a.out.stride_t;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      // An abs-block unit leaves its rows' partial (O / l in fp32, log2-sum)
      // for the abs pass, which adds the tiles holding abs keys.
      const int64_t prow = ((int64_t)w.it * a.num_q_heads + h) * BM + (i - w.q0);
      float* po = (w.abs && i < w.q1) ? part_o + prow * D : nullptr;
      uint4 packed[D / 8];
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t rr[32];
        if (have_o) {
          ptx::tmem_ld32(tmem + lane_base + c_o + 32 * cc, rr);
          ptx::tmem_wait_ld();
        } else {
#pragma unroll
          for (int x = 0; x < 32; ++x) rr[x] = 0u;
        }
        if (po) {
#pragma unroll
          for (int x = 0; x < 32; x += 4)
            *reinterpret_cast<float4*>(po + 32 * cc + x) =
                make_float4(__uint_as_float(rr[x]) * inv, __uint_as_float(rr[x + 1]) * inv,
                            __uint_as_float(rr[x + 2]) * inv, __uint_as_float(rr[x + 3]) * inv);
        }
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float fo[8];
#pragma unroll
          for (int x = 0; x < 8; ++x) fo[x] = __uint_as_float(rr[8 * c8 + x]) * inv;
          packed[4 * cc + c8] = pack8(fo);
        }
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar(O_FREE + t));
      // Output rows: a full unit goes through the group's staging buffer, one
      // 64-column half at a time (its threads hand their rows to thread 0
      // through STG_t; thread 0 frees the buffer through SFREE_t once the TMA
      // store has read it, for the second half only at the group's next staged
      // epilogue, so no thread waits for that read before the next unit's
      // scores); a unit whose item ends early is stored row by row
      // (the TMA box would spill into the next block's rows).  A unit without
      // key tiles stores its zero rows directly: its thread 0 has not waited
      // for the group's other threads in O_DONE.
      const bool full = !w.abs && w.pk == 1 && w.q1 == w.q0 + BM && w.n > 0;
      const uint32_t buf = OSTAGE + (uint32_t)t * kHalf;
      bool ok_st = true;
      if (full) {
        if (r == 0 && store_pending) {
          // The previous unit's second half: its store has long read the
          // buffer by now.
          ptx::bulk_wait_read_all();
          ptx::mbar_arrive(bar(SFREE0 + t));
          store_pending = false;
        }
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          if (nst > 0 && !wait(SFREE0 + t, (uint32_t)(nst - 1) & 1u)) {
            ok_st = false;
            break;
          }
#pragma unroll
          for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(sm + buf + chunk_off(r, c)) = packed[8 * hf + c];
          ptx::fence_proxy_async_smem();
          ptx::mbar_arrive(bar(STG0 + t));
          if (r == 0) {
            if (!wait(STG0 + t, (uint32_t)nst & 1u)) {
              ok_st = false;
              break;
            }
            ptx::tma_store_4d(&tm_o, sbase + buf, 64 * hf, w.q0, h, b);
            ptx::bulk_commit_group();
            if (hf == 0) {
              ptx::bulk_wait_read_all();
              ptx::mbar_arrive(bar(SFREE0 + t));
            } else {
              store_pending = true;  // released at the group's next staged epilogue
            }
          }
          ++nst;
        }
      } else if (i < w.q1 && !w.abs) {
#pragma unroll
        for (int c = 0; c < D / 8; ++c) *reinterpret_cast<uint4*>(Orow + 8 * c) = packed[c];
      }
      if (!ok_st) break;
      if (i < w.q1 && w.abs)
        part_lse[prow] = l > 0.f ? m_use + log2f(l) : -CUDART_INF_F;
      else if (i < w.q1)
        a.lse[((int64_t)b * a.num_q_heads + h) * a.seq_len + i] = l > 0.f ? (m_use + log2f(l)) * kLn2 : -CUDART_INF_F;
      g += w.n;
    }
    if (r == 0) ptx::bulk_wait_all();  // this thread's output stores have landed
  } else if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      ptx::prefetch_tmap(&tm_k);
      ptx::prefetch_tmap(&tm_v);
      if (prerot) {
        ptx::prefetch_tmap(&tm_qr);
        ptx::prefetch_tmap(&tm_qr64);
        ptx::prefetch_tmap(&tm_kr);
      }
      // Loads in the order their slots are released: K(g), V(g), ... with a
      // unit's Q after its first K and V tiles (Q is released by the previous
      // unit's last S MMAs, after that unit's second-to-last K and V).
      int g = 0, k = 0;
      bool ok = true;
      for (int u = snake_unit(k); ok && u < n_units; u = snake_unit(++k)) {
        const Unit w = load_unit<kAbs>(a, u, prerot, up);
        const int b = w.blk.row;
        const CUtensorMap* mk = w.k_pre ? &tm_kr : &tm_k;
        for (int j = 0; j <= w.n && ok; ++j) {
          if (j == min(1, w.n) && prerot) {
            if (k > 0 && !wait(Q_EMPTY, (k - 1) & 1)) {
              ok = false;
              break;
            }
            const int h0 = w.h0;
            ptx::mbar_arrive_expect_tx(bar(Q_READY), 2 * kTile);
            if (w.pk == 1) {
              ptx::tma_load_4d(sbase + Q0, &tm_qr, bar(Q_READY), 0, w.q0, h0, b);
              ptx::tma_load_4d(sbase + Q0 + kHalf, &tm_qr, bar(Q_READY), 64, w.q0, h0, b);
              ptx::tma_load_4d(sbase + Q1, &tm_qr, bar(Q_READY), 0, w.q0, h0 + 1, b);
              ptx::tma_load_4d(sbase + Q1 + kHalf, &tm_qr, bar(Q_READY), 64, w.q0, h0 + 1, b);
            } else {
              // Four heads, 64 rows each: head h0 + 2t + x into rows [64x, 64x + 64) of tile t.
#pragma unroll
              for (int hh = 0; hh < 4; ++hh) {
                const uint32_t dst = sbase + Q0 + (uint32_t)(hh >> 1) * kTile + (uint32_t)(hh & 1) * (kHalf / 2);
                ptx::tma_load_4d(dst, &tm_qr64, bar(Q_READY), 0, w.q0, h0 + hh, b);
                ptx::tma_load_4d(dst + kHalf, &tm_qr64, bar(Q_READY), 64, w.q0, h0 + hh, b);
              }
            }
          }
          if (j == w.n) break;
          const int slot = g & 1, k0 = w.kv_lo + unit_tile(w, j) * BN;
          const uint32_t kb = sbase + KB + (uint32_t)slot * kTile, vb = sbase + VB + (uint32_t)slot * kTile;
          if (g >= 2 && !wait(K_EMPTY + slot, ((g >> 1) - 1) & 1)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(bar(K_FULL + slot), kTile);
          int c0, c1;
          if (class_tile(L, w, j, a.status, c0, c1)) {
            // Rows 0-63 from chunk c0's copy, rows 64-127 from c1's (64-row
            // boxes land in the same 128-byte-swizzled layout as one 128-row box).
            ptx::tma_load_4d(kb, &tm_kc, bar(K_FULL + slot), 0, 0, w.hk, c0);
            ptx::tma_load_4d(kb + kHalf / 2, &tm_kc, bar(K_FULL + slot), 0, 0, w.hk, c1);
            ptx::tma_load_4d(kb + kHalf, &tm_kc, bar(K_FULL + slot), 64, 0, w.hk, c0);
            ptx::tma_load_4d(kb + kHalf + kHalf / 2, &tm_kc, bar(K_FULL + slot), 64, 0, w.hk, c1);
          } else {
            ptx::tma_load_4d(kb, mk, bar(K_FULL + slot), 0, k0, w.hk, b);
            ptx::tma_load_4d(kb + kHalf, mk, bar(K_FULL + slot), 64, k0, w.hk, b);
          }
          if (g >= 2 && !wait(V_EMPTY + slot, ((g >> 1) - 1) & 1)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(bar(V_FULL + slot), kTile);
          ptx::tma_load_4d(vb, &tm_v, bar(V_FULL + slot), 0, k0, w.hk, b);
          ptx::tma_load_4d(vb + kHalf, &tm_v, bar(V_FULL + slot), 64, k0, w.hk, b);
          ++g;
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    // Whole warp (warp-uniform descriptors); one elected lane issues.
    // The tensor core's instruction queue holds only a couple of MMAs, so the
    // warp's time between two MMA groups idles the tensor core almost one for
    // one: a barrier that has already completed is recognised by one try_wait
    // of the whole warp, before the bounded polling path.
    auto wait_u = [&](int i, uint32_t parity) -> bool {
      if (__all_sync(0xffffffffu, ptx::mbar_try_wait(bar(i), parity))) return true;
      return __shfl_sync(0xffffffffu, wait(i, parity), 0);
    };
    constexpr uint32_t idesc_qk = ptx::idesc_bf16_f32(BM, BN, false, false);
    constexpr uint32_t idesc_pv = ptx::idesc_bf16_f32(BM, D, false, true);
    // Every operand tile sits at a constant offset from a base descriptor, and
    // a descriptor's low 14 bits are the shared address / 16 (addresses stay
    // below 256 KB, so no carry leaves that field): each MMA's descriptor is
    // one add.
    const uint64_t d_q = ptx::sdesc_sw128(sbase + Q0, 16, 1024);
    const uint64_t d_k = ptx::sdesc_sw128(sbase + KB, 16, 1024);
    const uint64_t d_v = ptx::sdesc_sw128(sbase + VB, kHalf, 1024);
    constexpr uint64_t kT = kTile >> 4;
    static_assert(Q1 == Q0 + kTile, "Q tiles adjacent");
    auto issue_s = [&](int t, int slot) {
      const uint64_t dq = d_q + kT * (uint64_t)t, dk = d_k + kT * (uint64_t)slot;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t off = (uint64_t)(((kk >> 2) * kHalf + (kk & 3) * 32) >> 4);
        ptx::mma_ss_w(tmem + (t ? C_S1 : C_S0), dq + off, dk + off, idesc_qk, kk > 0);
      }
      ptx::mma_commit_w(bar(S_FULL + t));
    };
    // O_DONE is committed after a unit's last PV only (the epilogue's wait);
    // the softmax's rescale of O_t is ordered by the S_t commit that follows
    // each PV_t.
    auto issue_pv = [&](int t, int slot, bool first, bool last) {
      const uint64_t dv = d_v + kT * (uint64_t)slot;
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        ptx::mma_ts_w(tmem + (t ? C_O1 : C_O0), tmem + (t ? C_S1 : C_S0) + 8u * (uint32_t)kk,
                      dv + (uint64_t)((kk * 2048) >> 4), idesc_pv, (!first || kk > 0) ? 1u : 0u);
      }
      if (last) ptx::mma_commit_w(bar(O_DONE + t));
    };
    int g = 0, k = 0;
    bool ok = true;
    for (int u = snake_unit(k); ok && u < n_units; u = snake_unit(++k)) {
      const Unit w = load_unit<kAbs>(a, u, prerot, up);
      if (!wait_u(Q_READY, k & 1)) break;
      if (w.n == 0) {
        ptx::mma_commit_w(bar(Q_EMPTY));
        continue;
      }
      if (!wait_u(K_READY + (g & 1), (g >> 1) & 1)) break;
      ptx::tc_fence_after();
      issue_s(0, g & 1);
      issue_s(1, g & 1);
      ptx::mma_commit_w(bar(K_EMPTY + (g & 1)));
      if (w.n == 1) ptx::mma_commit_w(bar(Q_EMPTY));  // the unit's last reads of Q
      for (int j = 0; j < w.n; ++j) {
        const int gj = g + j, slot = gj & 1, nslot = (gj + 1) & 1;
        const bool more = j + 1 < w.n;
        if (!wait_u(P_READY, gj & 1) || (j == 0 && k > 0 && !wait_u(O_FREE, (k - 1) & 1)) ||
            !wait_u(V_FULL + slot, (gj >> 1) & 1)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        issue_pv(0, slot, j == 0, !more);
        if (more) {
          if (!wait_u(K_READY + nslot, ((gj + 1) >> 1) & 1)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          issue_s(0, nslot);
        }
        if (!wait_u(P_READY + 1, gj & 1) || (j == 0 && k > 0 && !wait_u(O_FREE + 1, (k - 1) & 1))) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        issue_pv(1, slot, j == 0, !more);
        ptx::mma_commit_w(bar(V_EMPTY + slot));
        if (more) {
          issue_s(1, nslot);
          ptx::mma_commit_w(bar(K_EMPTY + nslot));
          if (j + 2 == w.n) ptx::mma_commit_w(bar(Q_EMPTY));
        }
      }
      g += w.n;
    }
    // Drain: every MMA issued so far has completed before TMEM is released.
    ptx::mma_commit_w(bar(FINAL));
    ptx::mbar_wait(bar(FINAL), 0, kWait);
  } else {
    // ------------------------------------------------------------ K rotation (warps 10-11)
    // Thread rt rotates key rows rt and rt + 64 of each K tile in place by
    // the keys' block positions (nothing to do for a pre-rotated copy) and
    // records their key_info words.
    const int rt = tid - 320;
    const __half2* cs16 = static_cast<const __half2*>(L.rope_cs16);
    int g = 0;
    for (int kr = 0, u = snake_unit(0); u < n_units && !*s_abort; u = snake_unit(++kr)) {
      const Unit w = load_unit<kAbs>(a, u, prerot, up);
      for (int j = 0; j < w.n; ++j, ++g) {
        const int slot = g & 1;
        int c0, c1;
        const bool pre_tile = w.k_pre || class_tile(L, w, j, a.status, c0, c1);
        if (!wait(K_FULL + slot, (g >> 1) & 1)) break;
        const uint32_t kt = KB + (uint32_t)slot * kTile;
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int row = rt + 64 * hr, key = w.kv_lo + unit_tile(w, j) * BN + row;
          uint32_t info = 0;
          if (key < w.kv_hi) {
            info = (uint32_t)__ldg(L.key_info + w.blk.key_off + key);
            if (!pre_tile) {
              const int p = key_row(info, L.n_pos, a.status);
              const uint4* tp = reinterpret_cast<const uint4*>(cs16 + (int64_t)p * (D / 2));
#pragma unroll
              for (int qt = 0; qt < 4; ++qt) {
                uint4 tab[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) tab[c] = __ldg(tp + 4 * qt + c);
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                  uint4* pa = reinterpret_cast<uint4*>(sm + kt + chunk_off(row, 2 * qt + c));
                  uint4* pb = reinterpret_cast<uint4*>(sm + kt + chunk_off(row, 2 * qt + c + 8));
                  uint4 y1, y2;
                  tile::rotate8h(*pa, *pb, tab[2 * c], tab[2 * c + 1], y1, y2);
                  *pa = y1;
                  *pb = y2;
                }
              }
            }
          }
          s_flag[(g & (kInfoSlots - 1)) * BN + row] = (info & AI_KEY_ATTN) ? 1 : 0;
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(bar(K_READY + slot));
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool strides_ok(const AiTensor4& t) {
  return ((uintptr_t)t.ptr % 16 == 0) && (t.stride_b % 8 == 0) && (t.stride_h % 8 == 0) && (t.stride_t % 8 == 0);
}

}  // namespace sm100

// 4-D map over a (B, H, T, 128) bf16 tensor; box = 64 dims x box_rows rows,
// 128-byte swizzle, zero fill past T.
bool sm100_make_map(CUtensorMap* map, const AiTensor4& t, int B, int H, int T, int box_rows) {
  auto enc = sm100::get_encode();
  if (!enc) return false;
  cuuint64_t dims[4] = {(cuuint64_t)sm100::D, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)t.stride_t * 2, (cuuint64_t)t.stride_h * 2, (cuuint64_t)t.stride_b * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, t.ptr, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool sm100_fwd_supported(int dtype, int head_dim) { return dtype == AI_DTYPE_BF16 && head_dim == sm100::D; }

int sm100_fwd_tile_rows() { return sm100::BM; }

size_t sm100_fwd_abs_part_bytes(const AiAttnFwdArgs& a) {
  const int G = a.num_kv_heads > 0 ? a.num_q_heads / a.num_kv_heads : 0;
  if (!sm100_fwd_supported(a.dtype, a.head_dim) || G % 2 != 0 || a.layout.n_fwd_abs_items <= 0) return 0;
  const size_t rows = (size_t)a.layout.n_fwd_abs_items * a.num_q_heads * sm100::BM;
  return (rows * (sm100::D + 1) * sizeof(float) + 255) & ~size_t(255);
}

int sm100_fwd(const AiAttnFwdArgs& a, cudaStream_t st, cudaError_t* cuda_err) {
  using namespace sm100;
  if (!strides_ok(a.q) || !strides_ok(a.k) || !strides_ok(a.v) || !strides_ok(a.out)) return AI_ERR_STRIDE;
  cudaError_t e = cudaSuccess;
  // With enough workspace, Q and K are rotated once (HBM-bound) and the
  // warp-specialised kernel reads the rotated copies.  They are written
  // whenever the workspace holds them, so that the backward can reuse them.
  const size_t pb = prerot_bytes(a, nullptr);
  const bool pre = a.workspace && a.workspace_bytes >= pb;
  AiTensor4 qr{}, kr{}, kc{};
  if (pre) {
    if (!sm100_rotated_views(a, a.workspace, &qr, &kr, &kc)) return AI_ERR_ALIGN;
    e = prerot(a, a.workspace, st);
  }
  if (e == cudaSuccess && a.layout.n_fwd_items > 0) {
    CUtensorMap tm_k, tm_v;
    if (!sm100_make_map(&tm_k, a.k, a.batch, a.num_kv_heads, a.seq_len, BN)) return AI_ERR_TMA;
    if (!sm100_make_map(&tm_v, a.v, a.batch, a.num_kv_heads, a.seq_len, BN)) return AI_ERR_TMA;
    // Items of blocks with abs keys (and every item when a GQA group has an
    // odd number of query heads) run on the one-head kernel; the rest run two
    // or four heads per unit on the warp-specialised persistent kernel.  With
    // room in the workspace for the abs split, the persistent kernel also
    // runs the abs-block items' key tiles that hold no abs key, leaving
    // partial rows that the one-head kernel finishes with the other tiles.
    const int G = a.num_q_heads / a.num_kv_heads;
    const int n_single = (G % 2 == 0) ? a.layout.n_fwd_abs_items : a.layout.n_fwd_items;
    const int n_pair = a.layout.n_fwd_items - n_single;
    const size_t part_bytes = sm100_fwd_abs_part_bytes(a);
    const bool split = pre && part_bytes > 0 && a.workspace_bytes >= pb + part_bytes;
    float* part_o = split ? reinterpret_cast<float*>(static_cast<char*>(a.workspace) + pb) : nullptr;
    float* part_lse = split ? part_o + (size_t)a.layout.n_fwd_abs_items * a.num_q_heads * BM * D : nullptr;
    // Units of the persistent launches: the items after the abs ones, and
    // (split) the abs items' key tiles without abs keys.
    UnitPlan up{a.layout.n_fwd_abs_items, 0, 0, 0}, up_abs{0, 0, 0, 0};
    if (G % 2 == 0) {
      up.n_pack_items = (G % 4 == 0) ? a.layout.n_fwd_short_items : 0;
      up.n_pack_units = up.n_pack_items * (a.num_q_heads / 4);
      up.n_units = up.n_pack_units + (n_pair - up.n_pack_items) * (a.num_q_heads / 2);
      if (split) {
        up_abs.n_pack_items = (G % 4 == 0) ? a.layout.n_fwd_abs_short_items : 0;
        up_abs.n_pack_units = up_abs.n_pack_items * (a.num_q_heads / 4);
        up_abs.n_units = up_abs.n_pack_units + (a.layout.n_fwd_abs_items - up_abs.n_pack_items) * (a.num_q_heads / 2);
      }
    }
    CUtensorMap tm_kc = tm_k;
    if (pre && a.layout.n_rot_classes > 0 &&
        !sm100_make_map(&tm_kc, kc, a.layout.n_rot_classes, a.num_kv_heads, AI_ROT_CLASS_KEYS, AI_ROT_CLASS_KEYS))
      return AI_ERR_TMA;
    auto launch_single = [&]() -> int {
      if (n_single <= 0) return AI_OK;
      e = cudaFuncSetAttribute(fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
      if (e == cudaSuccess) {
        ProfScope ps(AI_PROF_FWD, st);
        fwd_kernel<<<dim3(n_single, a.num_q_heads), kThreads, kSmemBytes, st>>>(a, tm_k, tm_v, tm_kc, pre ? 1 : 0,
                                                                                part_o, part_lse);
        e = cudaGetLastError();
      }
      return AI_OK;
    };
    CUtensorMap tm_qr = tm_k, tm_kr = tm_k, tm_qr64 = tm_k, tm_o;
    if (pre && (!sm100_make_map(&tm_qr, qr, a.batch, a.num_q_heads, a.seq_len, BM) ||
                !sm100_make_map(&tm_qr64, qr, a.batch, a.num_q_heads, a.seq_len, BM / 2) ||
                !sm100_make_map(&tm_kr, kr, a.batch, a.num_kv_heads, a.seq_len, BN)))
      return AI_ERR_TMA;
    if (!sm100_make_map(&tm_o, a.out, a.batch, a.num_q_heads, a.seq_len, BM)) return AI_ERR_TMA;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    auto launch_pers = [&](auto kernel, const UnitPlan& p, bool after_pers) {
      if (p.n_units <= 0 || e != cudaSuccess) return;
      const int grid = p.n_units < sms ? p.n_units : sms;
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf::kSmem);
      if (e == cudaSuccess) {
        ProfScope ps(AI_PROF_FWD, st);
        // Right after the other persistent launch (which reads and writes
        // nothing this one touches) it starts by programmatic dependent
        // launch on the SMs that one leaves.
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(pf::kThreads);
        cfg.dynamicSmemBytes = pf::kSmem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = after_pers ? 1 : 0;
        e = cudaLaunchKernelEx(&cfg, kernel, a, tm_k, tm_v, tm_qr, tm_kr, tm_o, tm_qr64, tm_kc, pre ? 1 : 0, p, part_o,
                               part_lse);
        if (e == cudaSuccess) e = cudaGetLastError();
      }
    };
    // The split's partial rows come from the abs launch of the persistent
    // kernel (first: its units are short, the other launch fills in behind
    // it); the one-head kernel runs after both.
    if (split) launch_pers(fwd_pers_kernel<true>, up_abs, false);
    launch_pers(fwd_pers_kernel<false>, up, split && up_abs.n_units > 0);
    if (e == cudaSuccess) launch_single();
    // With the split, short abs items ran chunked: merge their partial rows.
    if (e == cudaSuccess && split && n_single > 0) {
      ProfScope ps(AI_PROF_FWD, st);
      fwd_abs_combine_kernel<<<dim3(n_single, a.num_q_heads), D, 0, st>>>(a, part_o, part_lse);
      e = cudaGetLastError();
    }
  }
  if (cuda_err) *cuda_err = e;
  return e == cudaSuccess ? AI_OK : AI_ERR_LAUNCH;
}

bool sm100_rotated_views(const AiAttnFwdArgs& a, void* buf, AiTensor4* qr, AiTensor4* kr, AiTensor4* kc) {
  if (!buf || ((uintptr_t)buf % 256)) return false;
  size_t qb = 0, qkb = 0;
  prerot_bytes(a, &qb, &qkb);
  const int64_t T = a.seq_len, Dm = sm100::D;
  qr->ptr = buf;
  qr->stride_t = Dm;
  qr->stride_h = T * Dm;
  qr->stride_b = (int64_t)a.num_q_heads * T * Dm;
  kr->ptr = static_cast<char*>(buf) + qb;
  kr->stride_t = Dm;
  kr->stride_h = T * Dm;
  kr->stride_b = (int64_t)a.num_kv_heads * T * Dm;
  if (kc) {
    kc->ptr = static_cast<char*>(buf) + qkb;
    kc->stride_t = Dm;
    kc->stride_h = (int64_t)AI_ROT_CLASS_KEYS * Dm;
    kc->stride_b = (int64_t)a.num_kv_heads * AI_ROT_CLASS_KEYS * Dm;
  }
  return true;
}

}  // namespace ai
