// Backward of the chain-of-edits attention on sm_100a tensor cores
// (tcgen05.mma, TMEM accumulators, TMA), bf16 in / fp32 accumulate,
// head_dim 128.  Two kernels, no atomics (deterministic):
//
// dq_kernel  (Q-stationary; one CTA = one forward work item x one query head,
//             or two / four heads of a GQA group for items of at most 64 / 32
//             rows, thread = query row = TMEM lane):
//   for each 64-key tile of the block's key range: S = Qrot.Krot^T (and
//   S_abs = Q.Krot^T on abs blocks) and dP = dO.V^T into TMEM; P =
//   exp(S*scale - lse); dS = P (dP - delta) scale; dS goes to smem split by key
//   into the rotated part and the abs part; dQrot += dS_rot.Krot and
//   dQabs += dS_abs.Krot accumulate in TMEM.  Epilogue:
//   dQ = R(qpos)^T dQrot + dQabs (the inverse rotation fused into the store).
//
// dkdv_kernel (KV-stationary; one CTA = 128 keys of one batch row x one KV
//             head, thread = key = TMEM lane):
//   V is loaded once; for every block that sees these keys the raw K tile is
//   re-loaded and rotated by the keys' positions *in that block*; then for
//   every 64-row query tile of the block and every query head of the GQA
//   group (or once for all G heads when the block has at most 64 / G rows,
//   their rows packed side by side): S^T = Krot.Qrot^T (abs keys take Krot.Q^T: a per-thread choice,
//   since abs is a property of the key), dP^T = V.dO^T, P^T, dS^T; dV += P^T.dO
//   and dKrot += dS^T.Qrot (+ dS^T_abs.Q) in TMEM.  When a block is done its
//   dKrot is rotated back by the block's key positions and added to the dK
//   accumulator (TMEM), so a key that several blocks see is summed without
//   atomics.
//
// Gradient algebra restated from the reference's eager function
// (attention/reference.py:46-62: s = Qrot.Krot + abs * (Q - Qrot).Krot) and
// its autograd; the row sums delta = sum(dO * O) come from the caller's
// scratch.  Every mbarrier wait is bounded; on expiry the status word gets
// AI_ERR_DEV_TIMEOUT and the CTA frees its TMEM and returns.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <math_constants.h>

#include "ai_common.cuh"
#include "ai_kernels.h"
#include "sm100_ptx.cuh"
#include "sm100_tile.cuh"

namespace ai {
namespace sm100bwd {

constexpr int D = 128;
constexpr int kThreads = 128;
constexpr uint32_t kTmemCols = 512;
constexpr long long kWaitCycles = 4000000000LL;
// Fewest 64-key abs tiles a chunk of a short abs item takes in dq_kernel.
constexpr int kDqChunkTiles = 6;

using tile::chunk_off;
using tile::pack8;
using tile::rotate8;

__device__ __forceinline__ float lse_log2(float lse) { return lse == -CUDART_INF_F ? CUDART_INF_F : lse * kLog2e; }

// Bounded wait shared by all threads; any thread that times out flags the CTA.
__device__ __forceinline__ void wait_or_flag(uint32_t bar, uint32_t& phase, volatile int* s_abort, int32_t* status) {
  if (!ptx::mbar_wait(bar, phase, kWaitCycles)) {
    report(status, AI_ERR_DEV_TIMEOUT);
    *s_abort = 1;
  }
  phase ^= 1;
}

__device__ __forceinline__ void store_bf16_row32(__nv_bfloat16* dst, const float* f) {
#pragma unroll
  for (int c8 = 0; c8 < 4; ++c8) {
    float v[8];
#pragma unroll
    for (int x = 0; x < 8; ++x) v[x] = f[8 * c8 + x];
    *reinterpret_cast<uint4*>(dst + 8 * c8) = pack8(v);
  }
}

// The same with two 32-byte stores (each a full sector); dst 32-byte aligned.
__device__ __forceinline__ void store_bf16_row32_v8(__nv_bfloat16* dst, const float* f) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t w[8];
#pragma unroll
    for (int x = 0; x < 8; ++x) w[x] = tile::pack2(f[16 * h + 2 * x], f[16 * h + 2 * x + 1]);
    ptx::st_global_v8(dst + 16 * h, w);
  }
}

// Whether every row of t starts on a 32-byte boundary.
__device__ __forceinline__ bool rows_32b(const AiTensor4& t) {
  return ((uintptr_t)t.ptr % 32 == 0) && (t.stride_b % 16 == 0) && (t.stride_h % 16 == 0) && (t.stride_t % 16 == 0);
}

// ===========================================================================
// dQ
// ===========================================================================
namespace dq {
constexpr int BM = 128;  // query rows (TMEM lanes)
constexpr int BN = 64;   // keys per tile
constexpr uint32_t QR = 0;            // 128 x 128 bf16, rotated Q
constexpr uint32_t QA = QR + 32768;   // unrotated Q (abs blocks)
constexpr uint32_t DO = QA + 32768;   // dO rows
constexpr uint32_t KR = DO + 32768;   // 64 keys x 128, rotated in place
constexpr uint32_t VV = KR + 16384;   // 64 keys x 128
constexpr uint32_t DS = VV + 16384;   // 128 rows x 64 keys: dS on non-abs keys
constexpr uint32_t DSA = DS + 16384;  // dS on abs keys
constexpr uint32_t KR1 = DSA + 16384;  // second K / V buffer: tile j + 1 loads while tile j runs
constexpr uint32_t VV1 = KR1 + 16384;
constexpr uint32_t INFO = VV1 + 16384;
constexpr uint32_t BAR_TMA = INFO + 4 * BN;  // two barriers, one per K / V buffer
constexpr uint32_t BAR_MMA = BAR_TMA + 16;
constexpr uint32_t TMEM_SLOT = BAR_MMA + 8;
constexpr uint32_t ABORT = TMEM_SLOT + 4;
constexpr uint32_t TOTAL = ABORT + 4;
constexpr size_t kSmem = TOTAL + 1024;
constexpr uint32_t C_S = 0, C_DP = 64, C_DQR = 128, C_DQA = 256, C_SA = 384;
}  // namespace dq

__global__ void __launch_bounds__(kThreads, 1)
    dq_kernel(const AiAttnBwdArgs a, const float* __restrict__ delta, const __grid_constant__ CUtensorMap tm_k,
              const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_kc, const int prerot,
              float* __restrict__ part_dq) {
  using namespace dq;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = tile::align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid / 32;
  uint32_t* s_info = reinterpret_cast<uint32_t*>(sm + INFO);
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + ABORT);
  const uint32_t bar_tma = sbase + BAR_TMA, bar_mma = sbase + BAR_MMA;

  const AiAttnFwdArgs& f = a.fwd;
  const AiAttnLayout& L = f.layout;
  const int32_t* item = L.fwd_items + 4 * (int64_t)blockIdx.x;
  const Block blk = load_block(L.blocks, item[0]);
  const int q0 = item[1], q1 = item[2];
  // A short item packs P heads of the group into the tile (as the forward).
  // With the abs split (part_dq given) the P CTAs y, y + Hq / P, ... of a
  // head group each take one of up to P consecutive chunks of the item's abs
  // tiles (abs_chunks) and leave their rows' dQ (fp32, rotated back) at row
  // chunk * (128 / P) + r of the (item, head) slab, which
  // dq_abs_combine_kernel sums.
  // An abs range shorter than two chunks of kDqChunkTiles stays whole on
  // chunk 0's CTA (the others return at once).
  const int G = f.num_q_heads / f.num_kv_heads, P = pack_heads(q1 - q0, G), slot = BM / P;
  const int kv_hi = min(blk.e, q1);
  int y = (int)blockIdx.y, chunk = 0, n_chunks = 1;
  if (part_dq != nullptr && P > 1) {
    chunk = y / (f.num_q_heads / P);
    y %= f.num_q_heads / P;
    int ja, jb;
    abs_tiles(blk, blk.kv_lo, kv_hi, BN, ja, jb);
    n_chunks = abs_chunks(jb - ja, P, kDqChunkTiles);
    if (chunk >= n_chunks) return;
  } else if (y * P >= f.num_q_heads) {
    return;
  }
  const bool chunked = n_chunks > 1;
  const int h = y * P + tid / slot, hk = (y * P) / G, b = blk.row;
  const bool has_abs = (blk.flags & AI_BLOCKF_ABS) != 0;
  const int i = q0 + tid % slot;
  // The block's rotation classes: a 64-key tile with one comes rotated.
  const int cls = block_classes(L, item[0], prerot != 0);

  // Key tiles of this CTA: the block's, or with the abs split only those
  // holding abs keys (chunk 0 of a chunked item starts from the persistent
  // kernel's partial, the other chunks from zero).
  const bool o_init = part_dq != nullptr && chunk == 0;
  int j_begin = 0, j_end = kv_hi > blk.kv_lo ? (kv_hi - blk.kv_lo + BN - 1) / BN : 0;
  if (part_dq != nullptr) {
    abs_tiles(blk, blk.kv_lo, kv_hi, BN, j_begin, j_end);
    if (chunked) {
      const int n = j_end - j_begin, jb = j_begin;
      j_begin = jb + n * chunk / n_chunks;
      j_end = jb + n * (chunk + 1) / n_chunks;
    }
  }

  // K and V of tile jt into buffer `buf` by TMA (K from its class copy when
  // it has one).  Tile jt + 1 loads while tile jt runs; its buffer was last
  // read by tile jt - 1's MMAs, complete by then.
  auto issue_tile = [&](int jt, int buf) {
    const int k0 = blk.kv_lo + jt * BN;
    const int kc = cls >= 0 ? chunk_class(L, cls, jt, f.status) : -1;
    const uint32_t kb = sbase + (buf ? KR1 : KR), vb = sbase + (buf ? VV1 : VV);
    const uint32_t bt = bar_tma + 8u * (uint32_t)buf;
    ptx::fence_proxy_async_smem();
    ptx::mbar_arrive_expect_tx(bt, 2 * 16384);
    if (kc >= 0) {
      ptx::tma_load_4d(kb, &tm_kc, bt, 0, 0, hk, kc);
      ptx::tma_load_4d(kb + 8192, &tm_kc, bt, 64, 0, hk, kc);
    } else {
      ptx::tma_load_4d(kb, &tm_k, bt, 0, k0, hk, b);
      ptx::tma_load_4d(kb + 8192, &tm_k, bt, 64, k0, hk, b);
    }
    ptx::tma_load_4d(vb, &tm_v, bt, 0, k0, hk, b);
    ptx::tma_load_4d(vb + 8192, &tm_v, bt, 64, k0, hk, b);
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
    ptx::tmem_alloc(sbase + TMEM_SLOT, kTmemCols);
    ptx::tmem_relinquish();
  }

  // Row i: rotated Q, raw Q (abs blocks), dO, lse, delta.
  int qrow = 0;
  float lse2 = 0.f, dl = 0.f;
  {
    const int64_t st_off = (int64_t)i;
    const __nv_bfloat16* Qrow = static_cast<const __nv_bfloat16*>(f.q.ptr) + b * f.q.stride_b + h * f.q.stride_h +
                                st_off * f.q.stride_t;
    const __nv_bfloat16* dOrow = static_cast<const __nv_bfloat16*>(a.dout.ptr) + b * a.dout.stride_b +
                                 h * a.dout.stride_h + st_off * a.dout.stride_t;
    if (i < q1) {
      qrow = clamp_row(L.q_pos[(int64_t)b * f.seq_len + i], L.n_pos, f.status);
      const int64_t idx = ((int64_t)b * f.num_q_heads + h) * f.seq_len + i;
      lse2 = lse_log2(f.lse[idx]);
      dl = delta[idx];
    }
    const float* cs = L.rope_cos + (int64_t)qrow * (D / 2);
    const float* sn = L.rope_sin + (int64_t)qrow * (D / 2);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 x1 = make_uint4(0, 0, 0, 0), x2 = x1, g1 = x1, g2 = x1, y1, y2;
      if (i < q1) {
        x1 = __ldg(reinterpret_cast<const uint4*>(Qrow + 8 * c));
        x2 = __ldg(reinterpret_cast<const uint4*>(Qrow + 64 + 8 * c));
        g1 = __ldg(reinterpret_cast<const uint4*>(dOrow + 8 * c));
        g2 = __ldg(reinterpret_cast<const uint4*>(dOrow + 64 + 8 * c));
      }
      rotate8(x1, x2, cs + 8 * c, sn + 8 * c, y1, y2);
      *reinterpret_cast<uint4*>(sm + QR + chunk_off<BM>(tid, c)) = y1;
      *reinterpret_cast<uint4*>(sm + QR + chunk_off<BM>(tid, c + 8)) = y2;
      *reinterpret_cast<uint4*>(sm + DO + chunk_off<BM>(tid, c)) = g1;
      *reinterpret_cast<uint4*>(sm + DO + chunk_off<BM>(tid, c + 8)) = g2;
      if (has_abs) {
        *reinterpret_cast<uint4*>(sm + QA + chunk_off<BM>(tid, c)) = x1;
        *reinterpret_cast<uint4*>(sm + QA + chunk_off<BM>(tid, c + 8)) = x2;
      }
    }
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + TMEM_SLOT);
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  constexpr uint32_t idesc_s = ptx::idesc_bf16_f32(BM, BN, false, false);
  constexpr uint32_t idesc_dq = ptx::idesc_bf16_f32(BM, D, false, true);
  const float sl2 = f.scale * kLog2e;
  uint32_t ph_tma = 0, ph_mma = 0;  // ph_tma: bit b = phase of K / V buffer b
  int n_tiles = 0;
  bool aborted = false, dqa_started = false;

  // With the abs split the persistent kernel has run this item's key tiles
  // without abs keys and left each row's dQrot (fp32): start the rotated
  // accumulator from it and run the tiles that hold abs keys only.
  if (o_init) {
    const bool have = i < q1;
    const float* prow = part_dq + (((int64_t)blockIdx.x * f.num_q_heads + h) * BM + (i - q0)) * D;
#pragma unroll
    for (int cc = 0; cc < D / 32; ++cc) {
      uint32_t r[32];
#pragma unroll
      for (int x = 0; x < 32; x += 4) {
        const float4 v = have ? *reinterpret_cast<const float4*>(prow + 32 * cc + x) : make_float4(0.f, 0.f, 0.f, 0.f);
        r[x] = __float_as_uint(v.x);
        r[x + 1] = __float_as_uint(v.y);
        r[x + 2] = __float_as_uint(v.z);
        r[x + 3] = __float_as_uint(v.w);
      }
      ptx::tmem_st32(tmem + lane_base + C_DQR + 32 * cc, r);
    }
    ptx::tmem_wait_st();
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
  }

  for (int jt = j_begin, k0 = blk.kv_lo + j_begin * BN; jt < j_end; ++jt, k0 += BN) {
    // Only a tile that holds one of the block's abs keys needs S_abs and dQabs.
    const bool tabs = blk.abs_in(k0, min(k0 + BN, kv_hi));
    const int kc = cls >= 0 ? chunk_class(L, cls, jt, f.status) : -1;
    const int buf = (jt - j_begin) & 1;
    const uint32_t KC = buf ? KR1 : KR, VC = buf ? VV1 : VV;
    // The next tile's K and V start loading (this tile's were requested one
    // tile ago); key row r's flags are read meanwhile.
    if (tid == 0 && jt + 1 < j_end) issue_tile(jt + 1, buf ^ 1);
    const int r = tid & 63, cg = tid >> 6, j = k0 + r;
    const uint32_t info = j < kv_hi ? (uint32_t)L.key_info[blk.key_off + j] : 0u;
    uint32_t ph = (ph_tma >> buf) & 1u;
    wait_or_flag(bar_tma + 8u * (uint32_t)buf, ph, s_abort, f.status);
    ph_tma ^= 1u << buf;
    __syncthreads();
    if (*s_abort) { aborted = true; break; }

    // Rotate key rows in place (fp16 (cos, sin) table, as the rotated copies
    // are made): thread -> (row tid % 64, chunk pairs 4*(tid/64) .. +3).
    {
      if (j < kv_hi) {
        if (kc < 0) {
          const int p = key_row(info, L.n_pos, f.status);
          const uint4* tp = static_cast<const uint4*>(L.rope_cs16) + (int64_t)p * (D / 8);
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int c = 4 * cg + cc;
            uint4* pa = reinterpret_cast<uint4*>(sm + KC + chunk_off<BN>(r, c));
            uint4* pb = reinterpret_cast<uint4*>(sm + KC + chunk_off<BN>(r, c + 8));
            uint4 y1, y2;
            tile::rotate8h(*pa, *pb, __ldg(tp + 2 * c), __ldg(tp + 2 * c + 1), y1, y2);
            *pa = y1;
            *pb = y2;
          }
        }
      }
      if (cg == 0) s_info[r] = info;
    }
    ptx::fence_proxy_async_smem();
    __syncthreads();

    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t ao = (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u;
        const uint32_t bo = (uint32_t)(kk >> 2) * 8192u + (uint32_t)(kk & 3) * 32u;
        ptx::mma_ss(tmem + C_S, ptx::sdesc_sw128(sbase + QR + ao, 16, 1024), ptx::sdesc_sw128(sbase + KC + bo, 16, 1024),
                    idesc_s, kk > 0);
        ptx::mma_ss(tmem + C_DP, ptx::sdesc_sw128(sbase + DO + ao, 16, 1024),
                    ptx::sdesc_sw128(sbase + VC + bo, 16, 1024), idesc_s, kk > 0);
        if (tabs)
          ptx::mma_ss(tmem + C_SA, ptx::sdesc_sw128(sbase + QA + ao, 16, 1024),
                      ptx::sdesc_sw128(sbase + KC + bo, 16, 1024), idesc_s, kk > 0);
      }
      ptx::mma_commit(bar_mma);
    }
    wait_or_flag(bar_mma, ph_mma, s_abort, f.status);
    __syncthreads();
    if (*s_abort) { aborted = true; break; }
    ptx::tc_fence_after();

    // dS of row i over the 64 keys, split by abs.
#pragma unroll
    for (int cc = 0; cc < BN / 32; ++cc) {
      uint32_t rs[32], rp[32], ra[32];
      ptx::tmem_ld32(tmem + lane_base + C_S + 32 * cc, rs);
      ptx::tmem_ld32(tmem + lane_base + C_DP + 32 * cc, rp);
      if (tabs) ptx::tmem_ld32(tmem + lane_base + C_SA + 32 * cc, ra);
      ptx::tmem_wait_ld();
      float dsr[32], dsa[32];
#pragma unroll
      for (int x = 0; x < 32; ++x) {
        const int c = 32 * cc + x;
        const uint32_t info = s_info[c];
        const bool is_abs = tabs && (info & AI_KEY_ABS);
        const float s = is_abs ? __uint_as_float(ra[x]) : __uint_as_float(rs[x]);
        const bool valid = (info & AI_KEY_ATTN) && (k0 + c <= i) && (i < q1);
        const float p = valid ? ptx::ex2(s * sl2 - lse2) : 0.f;
        const float ds = p * (__uint_as_float(rp[x]) - dl) * f.scale;
        dsr[x] = is_abs ? 0.f : ds;
        dsa[x] = is_abs ? ds : 0.f;
      }
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        float v[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) v[x] = dsr[8 * c8 + x];
        *reinterpret_cast<uint4*>(sm + DS + chunk_off<BM>(tid, 4 * cc + c8)) = pack8(v);
        if (tabs) {
#pragma unroll
          for (int x = 0; x < 8; ++x) v[x] = dsa[8 * c8 + x];
          *reinterpret_cast<uint4*>(sm + DSA + chunk_off<BM>(tid, 4 * cc + c8)) = pack8(v);
        }
      }
    }
    ptx::fence_proxy_async_smem();
    ptx::tc_fence_before();
    __syncthreads();

    if (tid == 0) {
      ptx::tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        const uint32_t ao = (uint32_t)kk * 32u;
        const uint32_t bo = (uint32_t)kk * 2048u;  // 16 key rows of 128 bytes
        const uint32_t acc = (n_tiles > 0 || o_init || kk > 0) ? 1u : 0u;
        ptx::mma_ss(tmem + C_DQR, ptx::sdesc_sw128(sbase + DS + ao, 16, 1024),
                    ptx::sdesc_sw128(sbase + KC + bo, 8192, 1024), idesc_dq, acc);
        if (tabs)
          ptx::mma_ss(tmem + C_DQA, ptx::sdesc_sw128(sbase + DSA + ao, 16, 1024),
                      ptx::sdesc_sw128(sbase + KC + bo, 8192, 1024), idesc_dq, (dqa_started || kk > 0) ? 1u : 0u);
      }
      ptx::mma_commit(bar_mma);
    }
    wait_or_flag(bar_mma, ph_mma, s_abort, f.status);
    __syncthreads();
    if (*s_abort) { aborted = true; break; }
    ptx::tc_fence_after();
    ++n_tiles;
    dqa_started = dqa_started || tabs;
  }

  // dQ = R(qpos)^T dQrot + dQabs.
  if (!aborted) {
    __nv_bfloat16* dQrow = static_cast<__nv_bfloat16*>(a.dq.ptr) + b * a.dq.stride_b + h * a.dq.stride_h +
                           (int64_t)i * a.dq.stride_t;
    const float* cs = L.rope_cos + (int64_t)qrow * (D / 2);
    const float* sn = L.rope_sin + (int64_t)qrow * (D / 2);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t g1[32], g2[32], a1[32], a2[32];
      const bool have_r = n_tiles > 0 || o_init;
      if (have_r) {
        ptx::tmem_ld32(tmem + lane_base + C_DQR + 32 * half, g1);
        ptx::tmem_ld32(tmem + lane_base + C_DQR + 64 + 32 * half, g2);
        if (dqa_started) {
          ptx::tmem_ld32(tmem + lane_base + C_DQA + 32 * half, a1);
          ptx::tmem_ld32(tmem + lane_base + C_DQA + 64 + 32 * half, a2);
        }
        ptx::tmem_wait_ld();
      }
      float o1[32], o2[32];
#pragma unroll
      for (int x = 0; x < 32; ++x) {
        const int d = 32 * half + x;
        float y1 = 0.f, y2 = 0.f;
        if (have_r) {
          const float c = cs[d], s = sn[d];
          const float v1 = __uint_as_float(g1[x]), v2 = __uint_as_float(g2[x]);
          y1 = v1 * c + v2 * s;
          y2 = v2 * c - v1 * s;
          if (dqa_started) {
            y1 += __uint_as_float(a1[x]);
            y2 += __uint_as_float(a2[x]);
          }
        }
        o1[x] = y1;
        o2[x] = y2;
      }
      if (i < q1 && chunked) {
        float* prow = part_dq + (((int64_t)blockIdx.x * f.num_q_heads + h) * BM + chunk * slot + (i - q0)) * D;
#pragma unroll
        for (int x = 0; x < 32; x += 4) {
          *reinterpret_cast<float4*>(prow + 32 * half + x) = make_float4(o1[x], o1[x + 1], o1[x + 2], o1[x + 3]);
          *reinterpret_cast<float4*>(prow + 64 + 32 * half + x) = make_float4(o2[x], o2[x + 1], o2[x + 2], o2[x + 3]);
        }
      } else if (i < q1) {
        store_bf16_row32(dQrow + 32 * half, o1);
        store_bf16_row32(dQrow + 64 + 32 * half, o2);
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// Sums the chunk rows dq_kernel left for the abs items it ran chunked
// (P = heads packed per tile > 1, more than one chunk), in chunk order, into
// the bf16 dQ rows.
// Grid (abs items, query heads); thread d owns dimension d of every row.
__global__ void __launch_bounds__(D) dq_abs_combine_kernel(const AiAttnBwdArgs a, const float* __restrict__ part_dq) {
  const AiAttnFwdArgs& f = a.fwd;
  const AiAttnLayout& L = f.layout;
  const int it = (int)blockIdx.x, h = (int)blockIdx.y, d = (int)threadIdx.x;
  const int32_t* item = L.fwd_items + 4 * (int64_t)it;
  const Block blk = load_block(L.blocks, item[0]);
  const int b = blk.row, q0 = item[1], q1 = item[2];
  const int G = f.num_q_heads / f.num_kv_heads, P = pack_heads(q1 - q0, G), slot = dq::BM / P;
  if (P == 1) return;  // written whole by dq_kernel
  int ja, jb;
  abs_tiles(blk, blk.kv_lo, min(blk.e, q1), dq::BN, ja, jb);
  const int nc = abs_chunks(jb - ja, P, kDqChunkTiles);
  if (nc == 1) return;  // finished by its one CTA
  const int64_t base = ((int64_t)it * f.num_q_heads + h) * dq::BM;
  for (int r = 0; r < q1 - q0; ++r) {
    float g = 0.f;
    for (int c = 0; c < nc; ++c) g += part_dq[(base + c * slot + r) * D + d];
    __nv_bfloat16* dQrow = static_cast<__nv_bfloat16*>(a.dq.ptr) + b * a.dq.stride_b + h * a.dq.stride_h +
                           (int64_t)(q0 + r) * a.dq.stride_t;
    dQrow[d] = __float2bfloat16_rn(g);
  }
}

// ===========================================================================
// dK / dV
// ===========================================================================
namespace kv {
constexpr int BN = 128;  // keys per CTA (TMEM lanes)
constexpr int BQ = 64;   // query rows per step
constexpr uint32_t KR = 0;               // 128 keys x 128 d, rotated per block
constexpr uint32_t VV = KR + 32768;
constexpr uint32_t QR = VV + 32768;      // 64 rows x 128 d, rotated
constexpr uint32_t QA = QR + 16384;      // 64 rows, unrotated (abs blocks)
constexpr uint32_t DO = QA + 16384;      // 64 rows of dO
constexpr uint32_t PT = DO + 16384;      // 128 keys x 64 rows: P^T
constexpr uint32_t DST = PT + 16384;     // dS^T of non-abs keys
constexpr uint32_t DSTA = DST + 16384;   // dS^T of abs keys
constexpr uint32_t LSE = DSTA + 16384;   // 64 floats (log2 units)
constexpr uint32_t DEL = LSE + 4 * BQ;   // 64 floats
constexpr uint32_t QPOS = DEL + 4 * BQ;  // 64 ints
constexpr uint32_t BAR_K = QPOS + 4 * BQ;
constexpr uint32_t BAR_Q = BAR_K + 8;
constexpr uint32_t BAR_MMA = BAR_Q + 8;
constexpr uint32_t TMEM_SLOT = BAR_MMA + 8;
constexpr uint32_t ABORT = TMEM_SLOT + 4;
constexpr uint32_t TOTAL = ABORT + 4;
constexpr size_t kSmem = TOTAL + 1024;
constexpr uint32_t C_ST = 0, C_DPT = 64, C_DV = 128, C_DKR = 256, C_DK = 384;
}  // namespace kv

__global__ void __launch_bounds__(kThreads, 1)
    dkdv_kernel(const AiAttnBwdArgs a, const float* __restrict__ delta, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_q,
                const __grid_constant__ CUtensorMap tm_do, const __grid_constant__ CUtensorMap tm_qp,
                const __grid_constant__ CUtensorMap tm_dop, const __grid_constant__ CUtensorMap tm_kc,
                const __grid_constant__ CUtensorMap tm_qr, const __grid_constant__ CUtensorMap tm_qrp,
                const int prerot, const int abs_only) {
  using namespace kv;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = tile::align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid / 32;
  float* s_lse = reinterpret_cast<float*>(sm + LSE);
  float* s_del = reinterpret_cast<float*>(sm + DEL);
  int* s_qpos = reinterpret_cast<int*>(sm + QPOS);
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + ABORT);
  const uint32_t bar_k = sbase + BAR_K, bar_q = sbase + BAR_Q, bar_mma = sbase + BAR_MMA;

  const AiAttnFwdArgs& f = a.fwd;
  const AiAttnLayout& L = f.layout;
  // One-dimensional grid, KV head fastest (entries costliest first).
  const int32_t* item = L.kv_items + 4 * (int64_t)(blockIdx.x / (unsigned)f.num_kv_heads);
  const int b = item[0], j0 = item[1], j1 = item[2];
  const int hk = (int)(blockIdx.x % (unsigned)f.num_kv_heads), G = f.num_q_heads / f.num_kv_heads;
  const int j = j0 + tid;  // this thread's key

  if (tid == 0) {
    ptx::mbar_init(bar_k, 1);
    ptx::mbar_init(bar_q, 1);
    ptx::mbar_init(bar_mma, 1);
    *s_abort = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tm_k);
    ptx::prefetch_tmap(&tm_v);
    ptx::prefetch_tmap(&tm_q);
    ptx::prefetch_tmap(&tm_do);
  }
  if (warp == 0) {
    ptx::tmem_alloc(sbase + TMEM_SLOT, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + TMEM_SLOT);
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  uint32_t ph_k = 0, ph_q = 0, ph_mma = 0;
  bool aborted = false, dv_started = false, dk_started = false;
  constexpr uint32_t idesc_st = ptx::idesc_bf16_f32(BN, BQ, false, false);
  constexpr uint32_t idesc_acc = ptx::idesc_bf16_f32(BN, D, false, true);
  const float sl2 = f.scale * kLog2e;

  // V tile, once.
  if (tid == 0) {
    ptx::mbar_arrive_expect_tx(bar_k, 32768);
    ptx::tma_load_4d(sbase + VV, &tm_v, bar_k, 0, j0, hk, b);
    ptx::tma_load_4d(sbase + VV + 16384, &tm_v, bar_k, 64, j0, hk, b);
  }
  wait_or_flag(bar_k, ph_k, s_abort, f.status);
  __syncthreads();
  if (*s_abort) aborted = true;

  // Query / dO rows of one step by TMA: the 64 rows from q0 of head h, or
  // (P > 1) 64 / P rows of each of the P heads of the group from hk * G.
  auto issue_q = [&](bool has_abs, int P, int sr, int q0, int h) {
    const uint32_t qdst = has_abs ? QA : QR;
    ptx::fence_proxy_async_smem();
    ptx::mbar_arrive_expect_tx(bar_q, (prerot && has_abs ? 6u : 4u) * 8192u);
    if (P == 1) {
      if (!prerot || has_abs) {
        ptx::tma_load_4d(sbase + qdst, &tm_q, bar_q, 0, q0, h, b);
        ptx::tma_load_4d(sbase + qdst + 8192, &tm_q, bar_q, 64, q0, h, b);
      }
      if (prerot) {
        ptx::tma_load_4d(sbase + QR, &tm_qr, bar_q, 0, q0, h, b);
        ptx::tma_load_4d(sbase + QR + 8192, &tm_qr, bar_q, 64, q0, h, b);
      }
      ptx::tma_load_4d(sbase + DO, &tm_do, bar_q, 0, q0, h, b);
      ptx::tma_load_4d(sbase + DO + 8192, &tm_do, bar_q, 64, q0, h, b);
    } else {
      for (int x = 0; x < P; ++x) {
        const uint32_t ro = (uint32_t)(x * sr) * 128u;
        if (!prerot || has_abs) {
          ptx::tma_load_4d(sbase + qdst + ro, &tm_qp, bar_q, 0, q0, hk * G + x, b);
          ptx::tma_load_4d(sbase + qdst + 8192 + ro, &tm_qp, bar_q, 64, q0, hk * G + x, b);
        }
        if (prerot) {
          ptx::tma_load_4d(sbase + QR + ro, &tm_qrp, bar_q, 0, q0, hk * G + x, b);
          ptx::tma_load_4d(sbase + QR + 8192 + ro, &tm_qrp, bar_q, 64, q0, hk * G + x, b);
        }
        ptx::tma_load_4d(sbase + DO + ro, &tm_dop, bar_q, 0, q0, hk * G + x, b);
        ptx::tma_load_4d(sbase + DO + 8192 + ro, &tm_dop, bar_q, 64, q0, hk * G + x, b);
      }
    }
  };

  for (int bi = L.row_blocks[b]; bi < L.row_blocks[b + 1] && !aborted; ++bi) {
    const Block blk = load_block(L.blocks, bi);
    if (blk.e <= j0 || blk.kv_lo >= j1) continue;
    const int qs = max(blk.s, j0);
    if (qs >= blk.e) continue;
    const bool has_abs = (blk.flags & AI_BLOCKF_ABS) != 0;
    if (abs_only && !blk.abs_in(j0, j1)) continue;
    // A block of at most 64 / G rows packs the rows of all G heads of the
    // group into one step: column c is row q0 + c % (64 / G) of head
    // hk * G + c / (64 / G) (tm_qp / tm_dop have boxes of 64 / G rows).
    const int P = ((G == 2 || G == 4 || G == 8) && blk.e - qs <= BQ / G) ? G : 1, sr = BQ / P;
    const int kmax = min(j1, blk.e);
    // The tile's two 64-key chunks in this block's rotation classes, if any.
    int c0 = -1, c1 = -1;
    {
      const int base = block_classes(L, bi, prerot != 0);
      if (base >= 0 && j0 >= blk.kv_lo && !(blk.flags & AI_BLOCKF_OWNPOS)) {
        const int ci = (j0 - blk.kv_lo) / AI_ROT_CLASS_KEYS;
        const int n = 2 * ((blk.e - blk.kv_lo + 2 * AI_ROT_CLASS_KEYS - 1) / (2 * AI_ROT_CLASS_KEYS));
        c0 = chunk_class(L, base, ci, f.status);
        c1 = ci + 1 < n ? chunk_class(L, base, ci + 1, f.status) : c0;
      }
    }
    const bool ctile = c0 >= 0 && c1 >= 0;

    // K tile: the rotated class copies, or raw and rotated in place by this
    // block's key positions.
    if (tid == 0) {
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive_expect_tx(bar_k, 32768);
      if (ctile) {
        ptx::tma_load_4d(sbase + KR, &tm_kc, bar_k, 0, 0, hk, c0);
        ptx::tma_load_4d(sbase + KR + 8192, &tm_kc, bar_k, 0, 0, hk, c1);
        ptx::tma_load_4d(sbase + KR + 16384, &tm_kc, bar_k, 64, 0, hk, c0);
        ptx::tma_load_4d(sbase + KR + 16384 + 8192, &tm_kc, bar_k, 64, 0, hk, c1);
      } else {
        ptx::tma_load_4d(sbase + KR, &tm_k, bar_k, 0, j0, hk, b);
        ptx::tma_load_4d(sbase + KR + 16384, &tm_k, bar_k, 64, j0, hk, b);
      }
      // The block's first step's query / dO rows load alongside (the previous
      // block's MMAs, the last readers of those buffers, are complete).
      issue_q(has_abs, P, sr, qs, hk * G);
    }
    const uint32_t my_info = j < kmax ? (uint32_t)L.key_info[blk.key_off + j] : 0u;
    wait_or_flag(bar_k, ph_k, s_abort, f.status);
    __syncthreads();
    if (*s_abort) { aborted = true; break; }
    int my_row = 0;
    if (j < kmax) {
      my_row = key_row(my_info, L.n_pos, f.status);
      if (!ctile) {
        const uint4* tp = static_cast<const uint4*>(L.rope_cs16) + (int64_t)my_row * (D / 8);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4* pa = reinterpret_cast<uint4*>(sm + KR + chunk_off<BN>(tid, c));
          uint4* pb = reinterpret_cast<uint4*>(sm + KR + chunk_off<BN>(tid, c + 8));
          uint4 y1, y2;
          tile::rotate8h(*pa, *pb, __ldg(tp + 2 * c), __ldg(tp + 2 * c + 1), y1, y2);
          *pa = y1;
          *pb = y2;
        }
      }
    }
    const bool key_ok = (my_info & AI_KEY_ATTN) != 0;
    const bool key_abs = has_abs && (my_info & AI_KEY_ABS);
    ptx::fence_proxy_async_smem();
    __syncthreads();

    bool dkr_started = false;
    bool first_step = true;
    for (int q0 = qs; q0 < blk.e && !aborted; q0 += BQ) {
      const int q1 = min(q0 + BQ, blk.e);
      for (int g = 0; g < G; g += P) {
        const int h = hk * G + g;
        // Raw query rows go to QA (abs blocks) or straight to QR to be rotated
        // there; with the rotated copies the rotated rows come by TMA as well.
        // The block's first step was requested with its K tile.
        const uint32_t qdst = has_abs ? QA : QR;
        if (tid == 0 && !first_step) issue_q(has_abs, P, sr, q0, h);
        first_step = false;
        if (tid < BQ) {
          const int r = q0 + tid % sr, hc = P == 1 ? h : hk * G + tid / sr;
          float l2 = CUDART_INF_F, dlt = 0.f;
          int qp = 0;
          if (r < q1) {
            const int64_t idx = ((int64_t)b * f.num_q_heads + hc) * f.seq_len + r;
            l2 = lse_log2(f.lse[idx]);
            dlt = delta[idx];
            qp = clamp_row(L.q_pos[(int64_t)b * f.seq_len + r], L.n_pos, f.status);
          }
          s_lse[tid] = l2;
          s_del[tid] = dlt;
          s_qpos[tid] = qp;
        }
        wait_or_flag(bar_q, ph_q, s_abort, f.status);
        __syncthreads();
        if (*s_abort) { aborted = true; break; }

        // Rotate the query rows: thread -> (row tid % 64, chunk pairs 4*(tid/64) .. +3).
        if (!prerot) {
          const int r = tid & 63, cg = tid >> 6;
          const int p = s_qpos[r];
          const float* cs = L.rope_cos + (int64_t)p * (D / 2);
          const float* sn = L.rope_sin + (int64_t)p * (D / 2);
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int c = 4 * cg + cc;
            const uint4 xa = *reinterpret_cast<const uint4*>(sm + qdst + chunk_off<BQ>(r, c));
            const uint4 xb = *reinterpret_cast<const uint4*>(sm + qdst + chunk_off<BQ>(r, c + 8));
            uint4 y1, y2;
            rotate8(xa, xb, cs + 8 * c, sn + 8 * c, y1, y2);
            *reinterpret_cast<uint4*>(sm + QR + chunk_off<BQ>(r, c)) = y1;
            *reinterpret_cast<uint4*>(sm + QR + chunk_off<BQ>(r, c + 8)) = y2;
          }
        }
        ptx::fence_proxy_async_smem();
        __syncthreads();

        // S^T (and S^T_abs) ; dP^T.
        if (tid == 0) {
          ptx::tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t ao = (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u;
            const uint32_t bo = (uint32_t)(kk >> 2) * 8192u + (uint32_t)(kk & 3) * 32u;
            ptx::mma_ss(tmem + C_ST, ptx::sdesc_sw128(sbase + KR + ao, 16, 1024),
                        ptx::sdesc_sw128(sbase + QR + bo, 16, 1024), idesc_st, kk > 0);
            if (has_abs)
              ptx::mma_ss(tmem + C_DPT, ptx::sdesc_sw128(sbase + KR + ao, 16, 1024),
                          ptx::sdesc_sw128(sbase + QA + bo, 16, 1024), idesc_st, kk > 0);
            else
              ptx::mma_ss(tmem + C_DPT, ptx::sdesc_sw128(sbase + VV + ao, 16, 1024),
                          ptx::sdesc_sw128(sbase + DO + bo, 16, 1024), idesc_st, kk > 0);
          }
          ptx::mma_commit(bar_mma);
        }
        wait_or_flag(bar_mma, ph_mma, s_abort, f.status);
        __syncthreads();
        if (*s_abort) { aborted = true; break; }
        ptx::tc_fence_after();

        float s[BQ];
#pragma unroll
        for (int cc = 0; cc < BQ / 32; ++cc) {
          uint32_t r0[32], r1[32];
          ptx::tmem_ld32(tmem + lane_base + C_ST + 32 * cc, r0);
          if (has_abs) ptx::tmem_ld32(tmem + lane_base + C_DPT + 32 * cc, r1);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < 32; ++x) s[32 * cc + x] = key_abs ? __uint_as_float(r1[x]) : __uint_as_float(r0[x]);
        }
        if (has_abs) {
          // The abs scores used the dP^T columns; now compute dP^T there.
          ptx::tc_fence_before();
          __syncthreads();
          if (tid == 0) {
            ptx::tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t ao = (uint32_t)(kk >> 2) * 16384u + (uint32_t)(kk & 3) * 32u;
              const uint32_t bo = (uint32_t)(kk >> 2) * 8192u + (uint32_t)(kk & 3) * 32u;
              ptx::mma_ss(tmem + C_DPT, ptx::sdesc_sw128(sbase + VV + ao, 16, 1024),
                          ptx::sdesc_sw128(sbase + DO + bo, 16, 1024), idesc_st, kk > 0);
            }
            ptx::mma_commit(bar_mma);
          }
          wait_or_flag(bar_mma, ph_mma, s_abort, f.status);
          __syncthreads();
          if (*s_abort) { aborted = true; break; }
          ptx::tc_fence_after();
        }

        // P^T and dS^T of key j over the 64 rows.
#pragma unroll
        for (int cc = 0; cc < BQ / 32; ++cc) {
          uint32_t rp[32];
          ptx::tmem_ld32(tmem + lane_base + C_DPT + 32 * cc, rp);
          ptx::tmem_wait_ld();
          float pv[32], dsv[32];
#pragma unroll
          for (int x = 0; x < 32; ++x) {
            const int c = 32 * cc + x, r = q0 + c % sr;
            const bool valid = key_ok && (j <= r) && (r < q1) && (j < kmax);
            const float p = valid ? ptx::ex2(s[c] * sl2 - s_lse[c]) : 0.f;
            pv[x] = p;
            dsv[x] = p * (__uint_as_float(rp[x]) - s_del[c]) * f.scale;
          }
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            float v[8], w[8], z[8];
#pragma unroll
            for (int x = 0; x < 8; ++x) {
              v[x] = pv[8 * c8 + x];
              w[x] = dsv[8 * c8 + x];
              z[x] = 0.f;
            }
            const uint32_t off = chunk_off<BN>(tid, 4 * cc + c8);
            *reinterpret_cast<uint4*>(sm + PT + off) = pack8(v);
            if (has_abs) {
              *reinterpret_cast<uint4*>(sm + DST + off) = key_abs ? pack8(z) : pack8(w);
              *reinterpret_cast<uint4*>(sm + DSTA + off) = key_abs ? pack8(w) : pack8(z);
            } else {
              *reinterpret_cast<uint4*>(sm + DST + off) = pack8(w);
            }
          }
        }
        ptx::fence_proxy_async_smem();
        ptx::tc_fence_before();
        __syncthreads();

        // dV += P^T dO ; dKrot += dS^T Qrot (+ dS^T_abs Q).
        if (tid == 0) {
          ptx::tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk) {
            const uint32_t ao = (uint32_t)kk * 32u;
            const uint32_t bo = (uint32_t)kk * 2048u;  // 16 query rows of 128 bytes
            ptx::mma_ss(tmem + C_DV, ptx::sdesc_sw128(sbase + PT + ao, 16, 1024),
                        ptx::sdesc_sw128(sbase + DO + bo, 8192, 1024), idesc_acc, (dv_started || kk > 0) ? 1u : 0u);
            ptx::mma_ss(tmem + C_DKR, ptx::sdesc_sw128(sbase + DST + ao, 16, 1024),
                        ptx::sdesc_sw128(sbase + QR + bo, 8192, 1024), idesc_acc, (dkr_started || kk > 0) ? 1u : 0u);
          }
          if (has_abs) {
#pragma unroll
            for (int kk = 0; kk < BQ / 16; ++kk) {
              ptx::mma_ss(tmem + C_DKR, ptx::sdesc_sw128(sbase + DSTA + (uint32_t)kk * 32u, 16, 1024),
                          ptx::sdesc_sw128(sbase + QA + (uint32_t)kk * 2048u, 8192, 1024), idesc_acc, 1u);
            }
          }
          ptx::mma_commit(bar_mma);
        }
        wait_or_flag(bar_mma, ph_mma, s_abort, f.status);
        __syncthreads();
        if (*s_abort) { aborted = true; break; }
        ptx::tc_fence_after();
        dv_started = true;
        dkr_started = true;
      }
    }
    if (aborted) break;

    // dK += R(key position in this block)^T dKrot.
    if (dkr_started) {
      const float* cs = L.rope_cos + (int64_t)my_row * (D / 2);
      const float* sn = L.rope_sin + (int64_t)my_row * (D / 2);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t g1[32], g2[32], k1[32], k2[32];
        ptx::tmem_ld32(tmem + lane_base + C_DKR + 32 * half, g1);
        ptx::tmem_ld32(tmem + lane_base + C_DKR + 64 + 32 * half, g2);
        if (dk_started) {
          ptx::tmem_ld32(tmem + lane_base + C_DK + 32 * half, k1);
          ptx::tmem_ld32(tmem + lane_base + C_DK + 64 + 32 * half, k2);
        }
        ptx::tmem_wait_ld();
#pragma unroll
        for (int x = 0; x < 32; ++x) {
          const int d = 32 * half + x;
          const float c = cs[d], sn_ = sn[d];
          const float v1 = __uint_as_float(g1[x]), v2 = __uint_as_float(g2[x]);
          float y1 = v1 * c + v2 * sn_, y2 = v2 * c - v1 * sn_;
          if (dk_started) {
            y1 += __uint_as_float(k1[x]);
            y2 += __uint_as_float(k2[x]);
          }
          k1[x] = __float_as_uint(y1);
          k2[x] = __float_as_uint(y2);
        }
        ptx::tmem_st32(tmem + lane_base + C_DK + 32 * half, k1);
        ptx::tmem_st32(tmem + lane_base + C_DK + 64 + 32 * half, k2);
      }
      ptx::tmem_wait_st();
      dk_started = true;
      ptx::tc_fence_before();
      __syncthreads();
      ptx::tc_fence_after();
    }
  }

  // Epilogue: dK and dV rows of this CTA's keys.
  if (!aborted) {
    __nv_bfloat16* dKrow = static_cast<__nv_bfloat16*>(a.dk.ptr) + b * a.dk.stride_b + hk * a.dk.stride_h +
                           (int64_t)j * a.dk.stride_t;
    __nv_bfloat16* dVrow = static_cast<__nv_bfloat16*>(a.dv.ptr) + b * a.dv.stride_b + hk * a.dv.stride_h +
                           (int64_t)j * a.dv.stride_t;
#pragma unroll
    for (int cc = 0; cc < D / 32; ++cc) {
      uint32_t rk[32], rv[32];
      if (dk_started) ptx::tmem_ld32(tmem + lane_base + C_DK + 32 * cc, rk);
      if (dv_started) ptx::tmem_ld32(tmem + lane_base + C_DV + 32 * cc, rv);
      ptx::tmem_wait_ld();
      float fk[32], fv[32];
#pragma unroll
      for (int x = 0; x < 32; ++x) {
        fk[x] = dk_started ? __uint_as_float(rk[x]) : 0.f;
        fv[x] = dv_started ? __uint_as_float(rv[x]) : 0.f;
      }
      if (j < j1) {
        if (abs_only) {
          // The warp-specialised pass already wrote the other blocks' part
          // of these rows (stream order): add to it.
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            const uint4 ok_ = *reinterpret_cast<const uint4*>(dKrow + 32 * cc + 8 * c8);
            const uint4 ov_ = *reinterpret_cast<const uint4*>(dVrow + 32 * cc + 8 * c8);
            const __nv_bfloat162* pk2 = reinterpret_cast<const __nv_bfloat162*>(&ok_);
            const __nv_bfloat162* pv2 = reinterpret_cast<const __nv_bfloat162*>(&ov_);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float2 k2 = __bfloat1622float2(pk2[u]), v2 = __bfloat1622float2(pv2[u]);
              fk[8 * c8 + 2 * u] += k2.x;
              fk[8 * c8 + 2 * u + 1] += k2.y;
              fv[8 * c8 + 2 * u] += v2.x;
              fv[8 * c8 + 2 * u + 1] += v2.y;
            }
          }
        }
        store_bf16_row32(dKrow + 32 * cc, fk);
        store_bf16_row32(dVrow + 32 * cc, fv);
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// ===========================================================================
// dQ, warp-specialised (work items of blocks without abs keys)
//
// Work unit = one forward work item x two query heads of one GQA group.  384
// threads: warps 0-3 / 4-7 score groups of head 2y / 2y+1 (thread = query
// row = TMEM lane); warp 8 TMA producer (64-key K and V tiles, 3-deep ring);
// warp 9 MMA issuer; warps 10-11 rotate each K tile by the keys' block
// positions.  TMEM per head t: S_t [128t .. +64), dP_t [+64 .. +128), dQ_t
// accumulator [256 + 128t .. +128).  dS_t (bf16 pairs) overwrites the first 32
// columns of S_t and is the A operand of dQ_t += dS_t.Krot; the next S_t
// follows that MMA directly (MMAs of one thread execute in issue order).  MMA
// order per key tile j: dQ0(j), S0/dP0(j+1), dQ1(j), S1/dP1(j+1).  The MMA
// warp runs converged and elects one lane per MMA.
// ===========================================================================
namespace dqw {
// 384 threads = three whole warpgroups (the register split is per
// warpgroup): warps 0-7 score groups, 8 TMA producer, 9 MMA, 10-11 K rotation
// (one key row per thread).  Launched at 168 registers a thread, the score
// warpgroups raise theirs to 184 (a tile's S and dP columns are read from
// TMEM at once) and warpgroup 2 lowers its to 136: 256 x 184 + 128 x 136.
constexpr int BM = 128, BN = 64, kThreads = 384;
constexpr uint32_t kRegScore = 184, kRegOther = 136;
static_assert(256 * kRegScore + 128 * kRegOther <= kThreads * 168, "register split");
constexpr int kKS = 3;  // K / V ring depth (the refill of tile g + kKS starts when tile g is done)
constexpr uint32_t Q0 = 0, Q1 = 32768, DO0 = 65536, DO1 = 98304;  // 128 x 128 bf16 each
constexpr uint32_t KB = 131072, VB = KB + kKS * 16384;            // rings of kKS x (64 x 128 bf16)
constexpr uint32_t INFO = VB + kKS * 16384;                       // [kKS][64] u32
constexpr uint32_t BARS = INFO + kKS * 4 * BN;
enum Bar { KV_FULL = 0, K_READY = kKS, KV_EMPTY = 2 * kKS, S_FULL = 3 * kKS, DS_READY = S_FULL + 2,
           DQ_DONE = DS_READY + 2, DQ_FREE = DQ_DONE + 2, Q_READY = DQ_FREE + 2, Q_EMPTY, FINAL, N_BARS };
constexpr uint32_t TMEM_SLOT = BARS + 8 * N_BARS;
constexpr uint32_t ABORT = TMEM_SLOT + 4;
constexpr uint32_t TOTAL = ABORT + 4;
constexpr size_t kSmem = TOTAL + 1024;
static_assert(kSmem <= 227 * 1024, "shared memory budget");
constexpr long long kWait = 1000000000LL;

// One work unit: rows [q0, q1) of a block x four query heads h0 .. h0 + 3 of
// one GQA group (pk = 2: an item of at most 64 rows, tile t holds heads
// h0 + 2t in lanes 0-63 and h0 + 2t + 1 in lanes 64-127) or x two query heads
// h0, h0 + 1 (pk = 1: tile t holds head h0 + t), as in the persistent forward.
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

// Rotation class of the unit's j-th K tile (64 keys: one class chunk), -1:
// the tile is rotated in shared memory (or comes from k_rot when k_pre).
__device__ __forceinline__ int tile_class(const AiAttnLayout& L, const Unit& w, int j, int32_t* status) {
  return w.cls < 0 ? -1 : chunk_class(L, w.cls, unit_tile(w, j), status);
}

__device__ __forceinline__ int unit_head(const Unit& w, int t, int r) {
  return w.pk == 2 ? w.h0 + 2 * t + (r >> 6) : w.h0 + t;
}
__device__ __forceinline__ int unit_row(const Unit& w, int r) { return w.q0 + (w.pk == 2 ? (r & 63) : r); }

template <bool kAbs>
__device__ __forceinline__ Unit load_unit(const AiAttnFwdArgs& f, int u, int prerot, const UnitPlan& up) {
  const AiAttnLayout& L = f.layout;
  const int hpairs = f.num_q_heads / 2, hquads = f.num_q_heads / 4, G = f.num_q_heads / f.num_kv_heads;
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
}  // namespace dqw

// ===========================================================================
// dQ, warp-specialised and persistent (work items of blocks without abs keys)
//
// One CTA per SM walks the work units u = blockIdx.x, blockIdx.x + gridDim.x,
// ... (unit = forward work item x two query heads of one GQA group; items
// longest first).  384 threads: warps 0-3 / 4-7 score groups of heads 2 hp /
// 2 hp + 1 (thread = query row = TMEM lane); warp 8 TMA producer (64-key K and
// V tiles, 3-deep ring); warp 9 MMA issuer; warps 10-11 rotate each K tile by
// the keys' block positions.  TMEM per head t: S_t [128t .. +64), dP_t
// [+64 .. +128), dQ_t accumulator [256 + 128t .. +128).  dS_t (bf16 pairs)
// overwrites the first 32 columns of S_t and is the A operand of dQ_t +=
// dS_t.Krot; the next S_t follows that MMA directly (MMAs of one thread
// execute in issue order).  MMA order per key tile j: dQ0(j), S0/dP0(j+1),
// dQ1(j), S1/dP1(j+1).  The MMA warp runs converged and elects one lane per
// MMA.  Across units (as in the persistent forward): tile barriers count by
// the running tile index, unit barriers by the running unit index; the next
// unit's Q / dO load starts once the current unit's last S / dP MMAs are done
// (Q_EMPTY); a unit's first dQ MMA waits until the previous unit's dQ_t has
// been read (DQ_FREE).
// ===========================================================================
// kAbs: the units are the abs-block items' key tiles without abs keys
// (their dQrot into part_dq); otherwise the other items, whole.
template <bool kAbs>
__global__ void __launch_bounds__(dqw::kThreads, 1)
    dq_pers_kernel(const AiAttnBwdArgs a, const float* __restrict__ delta, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_qr,
                   const __grid_constant__ CUtensorMap tm_do, const __grid_constant__ CUtensorMap tm_kr,
                   const __grid_constant__ CUtensorMap tm_qr64, const __grid_constant__ CUtensorMap tm_do64,
                   const __grid_constant__ CUtensorMap tm_kc, const int prerot, const UnitPlan up,
                   float* __restrict__ part_dq) {
  using namespace dqw;
  const int n_units = up.n_units;
  // The dK/dV kernel launched after this one reads nothing it writes: let it
  // start as soon as every CTA here has started, so its CTAs take each SM as
  // this kernel's CTA there finishes.
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = tile::align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  uint32_t* s_info = reinterpret_cast<uint32_t*>(sm + INFO);
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + ABORT);
  auto bar = [&](int i) { return sbase + BARS + 8u * (uint32_t)i; };

  const AiAttnFwdArgs& f = a.fwd;
  const AiAttnLayout& L = f.layout;
  const __half2* cs16 = static_cast<const __half2*>(L.rope_cs16);

  if (tid == 0) {
    for (int i = 0; i < N_BARS; ++i) {
      uint32_t count = 1;
      if (i == DS_READY || i == DS_READY + 1 || i == DQ_FREE || i == DQ_FREE + 1) count = 128;
      if (i >= K_READY && i < K_READY + kKS) count = 64;
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
    ptx::setmaxnreg_inc<kRegScore>();
  else
    ptx::setmaxnreg_dec<kRegOther>();

  auto wait = [&](int i, uint32_t parity) -> bool {
    if (*s_abort) return false;
    if (!ptx::mbar_wait(bar(i), parity, kWait)) {
      report(f.status, AI_ERR_DEV_TIMEOUT);
      *s_abort = 1;
      return false;
    }
    return true;
  };

  if (warp < 8) {
    // ------------------------------------------------------------ score groups
    const int t = warp / 4, r = tid % 128;
    const uint32_t lane_base = (uint32_t)((warp % 4) * 32) << 16;
    const uint32_t c_s = 128u * (uint32_t)t, c_dq = 256u + 128u * (uint32_t)t;
    const bool v8 = rows_32b(a.dq);
    const float sl2 = f.scale * kLog2e, scale = f.scale;
    const float2 sl2x2 = make_float2(sl2, sl2), scalex2 = make_float2(scale, scale);
    int g = 0, k = 0, ko = 0;  // ko: units with key tiles so far (DQ_DONE phases)
    for (int u = snake_unit(k); u < n_units && !*s_abort; u = snake_unit(++k)) {
      const Unit w = load_unit<kAbs>(f, u, prerot, up);
      const int i = unit_row(w, r), h = unit_head(w, t, r), b = w.blk.row, q1 = w.q1;
      int qrow = 0;
      float lse2 = 0.f, dl = 0.f;
      if (i < q1) {
        qrow = clamp_row(L.q_pos[(int64_t)b * f.seq_len + i], L.n_pos, f.status);
        const int64_t idx = ((int64_t)b * f.num_q_heads + h) * f.seq_len + i;
        lse2 = lse_log2(f.lse[idx]);
        dl = delta[idx];
      }
      if (!prerot) {
        // Q rows (rotated) and dO rows of this unit into shared memory, once
        // the previous unit's S / dP MMAs are done reading them.
        if (k > 0 && !wait(Q_EMPTY, (k - 1) & 1)) break;
        const __nv_bfloat16* Qrow = static_cast<const __nv_bfloat16*>(f.q.ptr) + b * f.q.stride_b +
                                    h * f.q.stride_h + (int64_t)i * f.q.stride_t;
        const __nv_bfloat16* dOrow = static_cast<const __nv_bfloat16*>(a.dout.ptr) + b * a.dout.stride_b +
                                     h * a.dout.stride_h + (int64_t)i * a.dout.stride_t;
        const uint4* tab = reinterpret_cast<const uint4*>(cs16 + (int64_t)qrow * (D / 2));
        const uint32_t qt = t ? Q1 : Q0, ot = t ? DO1 : DO0;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint4 x1[4], x2[4], g1[4], g2[4], cs[8];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int cc = 4 * hf + c;
            const uint4 z = make_uint4(0, 0, 0, 0);
            x1[c] = i < q1 ? __ldg(reinterpret_cast<const uint4*>(Qrow + 8 * cc)) : z;
            x2[c] = i < q1 ? __ldg(reinterpret_cast<const uint4*>(Qrow + 64 + 8 * cc)) : z;
            g1[c] = i < q1 ? __ldg(reinterpret_cast<const uint4*>(dOrow + 8 * cc)) : z;
            g2[c] = i < q1 ? __ldg(reinterpret_cast<const uint4*>(dOrow + 64 + 8 * cc)) : z;
            cs[2 * c] = __ldg(tab + 2 * cc);
            cs[2 * c + 1] = __ldg(tab + 2 * cc + 1);
          }
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int cc = 4 * hf + c;
            uint4 y1, y2;
            tile::rotate8h(x1[c], x2[c], cs[2 * c], cs[2 * c + 1], y1, y2);
            *reinterpret_cast<uint4*>(sm + qt + chunk_off<BM>(r, cc)) = y1;
            *reinterpret_cast<uint4*>(sm + qt + chunk_off<BM>(r, cc + 8)) = y2;
            *reinterpret_cast<uint4*>(sm + ot + chunk_off<BM>(r, cc)) = g1[c];
            *reinterpret_cast<uint4*>(sm + ot + chunk_off<BM>(r, cc + 8)) = g2[c];
          }
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(bar(Q_READY));
      }
      // Rows past q1 (another block's rows) get lse = +inf: their P is 0 with
      // no per-element test on the unmasked path.
      const float lse2r = i < q1 ? lse2 : CUDART_INF_F, dls = dl * scale;
      const float2 nlse2 = make_float2(-lse2r, -lse2r), ndls = make_float2(-dls, -dls);
      int done = 0;
      for (int j = 0; j < w.n; ++j) {
        const int gj = g + j, slot = gj % kKS, k0 = w.kv_lo + unit_tile(w, j) * BN;
        if (!wait(S_FULL + t, gj & 1)) break;
        ptx::tc_fence_after();
        // Tiles wholly below the diagonal of a block without masked keys take
        // the unmasked loop; the test sits outside the unrolled element loops.
        const bool fast = !w.masked && (k0 + BN <= w.kv_hi) && (k0 + BN - 1 <= w.q0);
        const int lim = min(i - k0, w.kv_hi - 1 - k0);
        const uint32_t* info = s_info + slot * BN;
        uint32_t pk[32];
        // The tile's 64 S and 64 dP columns, read from TMEM at once.
        uint32_t rs2[2][32], rp2[2][32];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          ptx::tmem_ld32(tmem + lane_base + c_s + 32 * hf, rs2[hf]);
          ptx::tmem_ld32(tmem + lane_base + c_s + 64 + 32 * hf, rp2[hf]);
        }
        ptx::tmem_wait_ld();
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const uint32_t(&rs)[32] = rs2[hf];
          const uint32_t(&rp)[32] = rp2[hf];
          // Pairs of keys on the packed f32x2 pipe.
          auto pair = [&](int x2, bool ok0, bool ok1) {
            float2 arg = __ffma2_rn(make_float2(__uint_as_float(rs[2 * x2]), __uint_as_float(rs[2 * x2 + 1])), sl2x2,
                                    nlse2);
            arg.x = ok0 ? arg.x : -CUDART_INF_F;
            arg.y = ok1 ? arg.y : -CUDART_INF_F;
            const float2 pp = make_float2(ptx::ex2(arg.x), ptx::ex2(arg.y));
            const float2 ds = __fmul2_rn(
                pp, __ffma2_rn(make_float2(__uint_as_float(rp[2 * x2]), __uint_as_float(rp[2 * x2 + 1])), scalex2,
                               ndls));
            pk[16 * hf + x2] = tile::pack2(ds.x, ds.y);
          };
          if (fast) {
#pragma unroll
            for (int x2 = 0; x2 < 16; ++x2) pair(x2, true, true);
          } else if (!w.masked) {
            // causal / key-range limit only: column c valid iff c <= lim
#pragma unroll
            for (int x2 = 0; x2 < 16; ++x2) {
              const int c = 32 * hf + 2 * x2;
              pair(x2, c <= lim, c + 1 <= lim);
            }
          } else {
#pragma unroll
            for (int x2 = 0; x2 < 16; ++x2) {
              const int c = 32 * hf + 2 * x2;
              pair(x2, (info[c] & AI_KEY_ATTN) && c <= lim, (info[c + 1] & AI_KEY_ATTN) && c + 1 <= lim);
            }
          }
        }
        ptx::tmem_st32(tmem + lane_base + c_s, pk);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(DS_READY + t));
        done = j + 1;
      }
      if (done != w.n) break;
      // Epilogue: dQ = R(qpos)^T dQrot; dQ_t is released to the next unit's
      // first dQ MMA once it has been read.  The row's rotary entries are
      // requested before the wait for the last dQ MMAs: each of these loads
      // touches 32 table rows, and their latency (thousands of cycles with
      // every warp of the CTA loading at once) would otherwise hold up the
      // next unit's first tile.
      uint4 tv_row[16];
      if (!kAbs) {
        const uint4* tab = reinterpret_cast<const uint4*>(cs16 + (int64_t)qrow * (D / 2));
#pragma unroll
        for (int q = 0; q < 16; ++q) tv_row[q] = __ldg(tab + q);
      }
      bool have = false;
      if (w.n > 0) {
        have = wait(DQ_DONE + t, (uint32_t)ko & 1u);
        ++ko;
        if (!have) break;
      }
      ptx::tc_fence_after();
      __nv_bfloat16* dQrow = static_cast<__nv_bfloat16*>(a.dq.ptr) + b * a.dq.stride_b + h * a.dq.stride_h +
                             (int64_t)i * a.dq.stride_t;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t g1[32], g2[32];
        if (have) {
          ptx::tmem_ld32(tmem + lane_base + c_dq + 32 * hf, g1);
          ptx::tmem_ld32(tmem + lane_base + c_dq + 64 + 32 * hf, g2);
          ptx::tmem_wait_ld();
        } else {
#pragma unroll
          for (int x = 0; x < 32; ++x) g1[x] = g2[x] = 0u;
        }
        if (hf == 1) {  // dQ_t has been read
          ptx::tc_fence_before();
          ptx::mbar_arrive(bar(DQ_FREE + t));
        }
        if (w.abs) {
          // An abs-block unit leaves its rows' dQrot (fp32, not rotated back)
          // for the abs pass, which adds the tiles holding abs keys.
          if (i < q1) {
            float* po = part_dq + (((int64_t)w.it * f.num_q_heads + h) * BM + (i - w.q0)) * D;
#pragma unroll
            for (int x = 0; x < 32; x += 4) {
              *reinterpret_cast<float4*>(po + 32 * hf + x) =
                  make_float4(__uint_as_float(g1[x]), __uint_as_float(g1[x + 1]), __uint_as_float(g1[x + 2]),
                              __uint_as_float(g1[x + 3]));
              *reinterpret_cast<float4*>(po + 64 + 32 * hf + x) =
                  make_float4(__uint_as_float(g2[x]), __uint_as_float(g2[x + 1]), __uint_as_float(g2[x + 2]),
                              __uint_as_float(g2[x + 3]));
            }
          }
          continue;
        }
        float o1[32], o2[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint4 tv = tv_row[8 * hf + q];
          const __half2* h2 = reinterpret_cast<const __half2*>(&tv);
#pragma unroll
          for (int uu = 0; uu < 4; ++uu) {
            const int xx = 4 * q + uu;
            const float2 csn = __half22float2(h2[uu]);
            const float v1 = __uint_as_float(g1[xx]), v2 = __uint_as_float(g2[xx]);
            o1[xx] = v1 * csn.x + v2 * csn.y;
            o2[xx] = v2 * csn.x - v1 * csn.y;
          }
        }
        if (i < q1) {
          // Rows 8 KB apart: each store instruction touches 32 rows, so full
          // 32-byte sectors halve the L1 / L2 write requests.
          if (v8) {
            store_bf16_row32_v8(dQrow + 32 * hf, o1);
            store_bf16_row32_v8(dQrow + 64 + 32 * hf, o2);
          } else {
            store_bf16_row32(dQrow + 32 * hf, o1);
            store_bf16_row32(dQrow + 64 + 32 * hf, o2);
          }
        }
      }
      g += w.n;
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      ptx::prefetch_tmap(&tm_k);
      ptx::prefetch_tmap(&tm_v);
      if (prerot) {
        ptx::prefetch_tmap(&tm_kr);
        ptx::prefetch_tmap(&tm_qr);
        ptx::prefetch_tmap(&tm_do);
        ptx::prefetch_tmap(&tm_qr64);
        ptx::prefetch_tmap(&tm_do64);
      }
      int g = 0, k = 0;
      bool ok = true;
      for (int u = snake_unit(k); ok && u < n_units; u = snake_unit(++k)) {
        const Unit w = load_unit<kAbs>(f, u, prerot, up);
        const int b = w.blk.row;
        if (prerot) {
          if (k > 0 && !wait(Q_EMPTY, (k - 1) & 1)) break;
          const int h0 = w.h0;
          ptx::mbar_arrive_expect_tx(bar(Q_READY), 4 * 32768);
          if (w.pk == 1) {
            ptx::tma_load_4d(sbase + Q0, &tm_qr, bar(Q_READY), 0, w.q0, h0, b);
            ptx::tma_load_4d(sbase + Q0 + 16384, &tm_qr, bar(Q_READY), 64, w.q0, h0, b);
            ptx::tma_load_4d(sbase + Q1, &tm_qr, bar(Q_READY), 0, w.q0, h0 + 1, b);
            ptx::tma_load_4d(sbase + Q1 + 16384, &tm_qr, bar(Q_READY), 64, w.q0, h0 + 1, b);
            ptx::tma_load_4d(sbase + DO0, &tm_do, bar(Q_READY), 0, w.q0, h0, b);
            ptx::tma_load_4d(sbase + DO0 + 16384, &tm_do, bar(Q_READY), 64, w.q0, h0, b);
            ptx::tma_load_4d(sbase + DO1, &tm_do, bar(Q_READY), 0, w.q0, h0 + 1, b);
            ptx::tma_load_4d(sbase + DO1 + 16384, &tm_do, bar(Q_READY), 64, w.q0, h0 + 1, b);
          } else {
            // Four heads, 64 rows each: head h0 + 2t + x into rows [64x, 64x + 64) of tile t.
#pragma unroll
            for (int hh = 0; hh < 4; ++hh) {
              const uint32_t off = (uint32_t)(hh >> 1) * 32768u + (uint32_t)(hh & 1) * 8192u;
              ptx::tma_load_4d(sbase + Q0 + off, &tm_qr64, bar(Q_READY), 0, w.q0, h0 + hh, b);
              ptx::tma_load_4d(sbase + Q0 + off + 16384, &tm_qr64, bar(Q_READY), 64, w.q0, h0 + hh, b);
              ptx::tma_load_4d(sbase + DO0 + off, &tm_do64, bar(Q_READY), 0, w.q0, h0 + hh, b);
              ptx::tma_load_4d(sbase + DO0 + off + 16384, &tm_do64, bar(Q_READY), 64, w.q0, h0 + hh, b);
            }
          }
        }
        const CUtensorMap* mk = w.k_pre ? &tm_kr : &tm_k;
        for (int j = 0; j < w.n; ++j, ++g) {
          const int slot = g % kKS, k0 = w.kv_lo + unit_tile(w, j) * BN;
          if (g >= kKS && !wait(KV_EMPTY + slot, ((g / kKS) - 1) & 1)) {
            ok = false;
            break;
          }
          const uint32_t kb = sbase + KB + 16384u * (uint32_t)slot, vb = sbase + VB + 16384u * (uint32_t)slot;
          ptx::mbar_arrive_expect_tx(bar(KV_FULL + slot), 32768);
          const int kc = tile_class(L, w, j, f.status);
          if (kc >= 0) {
            ptx::tma_load_4d(kb, &tm_kc, bar(KV_FULL + slot), 0, 0, w.hk, kc);
            ptx::tma_load_4d(kb + 8192, &tm_kc, bar(KV_FULL + slot), 64, 0, w.hk, kc);
          } else {
            ptx::tma_load_4d(kb, mk, bar(KV_FULL + slot), 0, k0, w.hk, b);
            ptx::tma_load_4d(kb + 8192, mk, bar(KV_FULL + slot), 64, k0, w.hk, b);
          }
          ptx::tma_load_4d(vb, &tm_v, bar(KV_FULL + slot), 0, k0, w.hk, b);
          ptx::tma_load_4d(vb + 8192, &tm_v, bar(KV_FULL + slot), 64, k0, w.hk, b);
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
    constexpr uint32_t idesc_s = ptx::idesc_bf16_f32(BM, BN, false, false);
    constexpr uint32_t idesc_dq = ptx::idesc_bf16_f32(BM, D, false, true);
    // Every operand tile sits at a constant offset from a base descriptor, and
    // a descriptor's low 14 bits are the shared address / 16 (addresses stay
    // below 256 KB, so no carry leaves that field): each MMA's descriptor is
    // one add.
    static_assert(Q1 == Q0 + 32768 && DO0 == Q0 + 65536 && DO1 == Q0 + 98304, "Q / dO tile layout");
    const uint64_t d_q = ptx::sdesc_sw128(sbase + Q0, 16, 1024);
    const uint64_t d_k = ptx::sdesc_sw128(sbase + KB, 16, 1024);
    const uint64_t d_ka = ptx::sdesc_sw128(sbase + KB, 8192, 1024);  // K as the MN-major B of dQ += dS.K
    constexpr uint64_t kSlot = 16384u >> 4, kHead = 32768u >> 4, kDo = 65536u >> 4, kV = (uint64_t)(VB - KB) >> 4;
    auto issue_s = [&](int t, int slot) {
      const uint64_t dq = d_q + kHead * (uint64_t)t, dk = d_k + kSlot * (uint64_t)slot;
      const uint32_t cs = tmem + 128u * (uint32_t)t;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t ao = (uint64_t)(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
        const uint64_t bo = (uint64_t)(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4);
        ptx::mma_ss_w(cs, dq + ao, dk + bo, idesc_s, kk > 0);
        ptx::mma_ss_w(cs + 64, dq + kDo + ao, dk + kV + bo, idesc_s, kk > 0);
      }
      ptx::mma_commit_w(bar(S_FULL + t));
    };
    // DQ_DONE is committed after a unit's last dQ MMAs only (the epilogue's
    // wait).
    auto issue_dq = [&](int t, int slot, bool first, bool last) {
      const uint64_t dk = d_ka + kSlot * (uint64_t)slot;
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk)
        ptx::mma_ts_w(tmem + 256u + 128u * (uint32_t)t, tmem + 128u * (uint32_t)t + 8u * (uint32_t)kk,
                      dk + (uint64_t)((2048 * kk) >> 4), idesc_dq, (!first || kk > 0) ? 1u : 0u);
      if (last) ptx::mma_commit_w(bar(DQ_DONE + t));
    };
    int g = 0, k = 0;
    bool ok = true;
    for (int u = snake_unit(k); ok && u < n_units; u = snake_unit(++k)) {
      const Unit w = load_unit<kAbs>(f, u, prerot, up);
      if (!wait_u(Q_READY, k & 1)) break;
      if (w.n == 0) {
        ptx::mma_commit_w(bar(Q_EMPTY));
        continue;
      }
      if (!wait_u(K_READY + g % kKS, (g / kKS) & 1)) break;
      ptx::tc_fence_after();
      issue_s(0, g % kKS);
      issue_s(1, g % kKS);
      if (w.n == 1) ptx::mma_commit_w(bar(Q_EMPTY));  // the unit's last reads of Q and dO
      for (int j = 0; j < w.n; ++j) {
        const int gj = g + j, slot = gj % kKS, nslot = (gj + 1) % kKS;
        const bool more = j + 1 < w.n;
        if (!wait_u(DS_READY, gj & 1) || (j == 0 && k > 0 && !wait_u(DQ_FREE, (k - 1) & 1))) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        issue_dq(0, slot, j == 0, !more);
        if (more) {
          if (!wait_u(K_READY + nslot, ((gj + 1) / kKS) & 1)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          issue_s(0, nslot);
        }
        if (!wait_u(DS_READY + 1, gj & 1) || (j == 0 && k > 0 && !wait_u(DQ_FREE + 1, (k - 1) & 1))) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        issue_dq(1, slot, j == 0, !more);
        ptx::mma_commit_w(bar(KV_EMPTY + slot));
        if (more) {
          issue_s(1, nslot);
          if (j + 2 == w.n) ptx::mma_commit_w(bar(Q_EMPTY));
        }
      }
      g += w.n;
    }
    ptx::mma_commit_w(bar(FINAL));
    ptx::mbar_wait(bar(FINAL), 0, kWait);
  } else {
    // ------------------------------------------------------------ K rotation (warps 10-11)
    const int row = tid - 320;  // 0..63: key row of the tile
    int g = 0;
    for (int kr = 0, u = snake_unit(0); u < n_units && !*s_abort; u = snake_unit(++kr)) {
      const Unit w = load_unit<kAbs>(f, u, prerot, up);
      for (int j = 0; j < w.n; ++j, ++g) {
        const int slot = g % kKS, key = w.kv_lo + unit_tile(w, j) * BN + row;
        uint32_t info = 0;
        int p = 0;
        if (key < w.kv_hi) {
          info = (uint32_t)__ldg(L.key_info + w.blk.key_off + key);
          p = key_row(info, L.n_pos, f.status);
        }
        const bool pre_tile = w.k_pre || tile_class(L, w, j, f.status) >= 0;
        if (!wait(KV_FULL + slot, (g / kKS) & 1)) break;
        const uint32_t kt = KB + 16384u * (uint32_t)slot;
        if (!pre_tile && key < w.kv_hi) {
          const uint4* tp = reinterpret_cast<const uint4*>(cs16 + (int64_t)p * (D / 2));
#pragma unroll
          for (int cg = 0; cg < 2; ++cg) {
            uint4 tab[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) tab[c] = __ldg(tp + 8 * cg + c);
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
              const int c = 4 * cg + cc;
              uint4* pa = reinterpret_cast<uint4*>(sm + kt + chunk_off<BN>(row, c));
              uint4* pb = reinterpret_cast<uint4*>(sm + kt + chunk_off<BN>(row, c + 8));
              uint4 y1, y2;
              tile::rotate8h(*pa, *pb, tab[2 * cc], tab[2 * cc + 1], y1, y2);
              *pa = y1;
              *pb = y2;
            }
          }
        }
        s_info[slot * BN + row] = info;
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

// ===========================================================================
// dK / dV, warp-specialised (key tiles whose blocks have no abs keys)
//
// One CTA = 128 keys of one batch row x one KV head.  A "step" is one
// 64-row query tile of a block x one query head of the GQA group.  640
// threads in roles:
//   warps 0-15      four score groups of four warps, group t taking query
//                   columns [16t, 16t + 16) of every step (thread = key =
//                   TMEM lane): P^T = exp(S^T - lse), dS^T = P^T (dP^T - delta)
//                   scale, written back into TMEM as bf16 pairs;
//   warp 16         TMA producer (V once, raw K per block, Q and dO per step)
//   warp 17         MMA issuer and TMEM owner
//   warps 18-19     rotate K per block (two keys a thread) and each Q tile in
//                   place (one row a thread); stage the step's lse / delta
//                   rows in smem.
// TMEM: S^T / dP^T double-buffered by step parity (4 x 64 columns), dV and
// dKrot accumulators (128 each).  dV += P^T dO and dKrot += dS^T Qrot take
// their A operands from TMEM; the scores of step s + 2 reuse that buffer
// right after those MMAs (one thread's MMAs execute in issue order), and the
// producer alone waits for them before refilling the Q / dO slot.  The MMA
// warp runs converged and elects one lane per MMA.  At the end of a block the
// score groups rotate dKrot back by the keys' block positions (group t the
// rotation pairs (d, d + 64), d in [16t, 16t + 16)) into an fp32 dK
// accumulator in smem, so keys seen by several blocks are summed without
// atomics.
// ===========================================================================
namespace kvw {
// 640 threads (five whole warpgroups): warps 0-15 four score groups of 16
// query columns each, 16 TMA producer, 17 MMA issuer, 18-19 rotation.
constexpr int BN = 128, BQ = 64, kThreads = 640, kGroups = 4, kCols = BQ / kGroups;
constexpr int kRot = kThreads - 32 * (4 * kGroups + 2);  // rotation threads
static_assert(kRot == 64 && BQ == kRot && BN == 2 * kRot, "rotation: one Q row, two K rows per thread");
// Q / dO ring depth: the load of step s + kQS starts when step s's dV / dK
// MMAs are done, so with 3 stages it has about two steps of MMA time to land.
constexpr int kQS = 3;
constexpr uint32_t K = 0;                   // 128 keys x 128 d (rotated per block)
constexpr uint32_t V = 32768;
constexpr uint32_t Q = 65536;               // ring of kQS x (64 rows x 128 d), rotated in place
constexpr uint32_t DO = Q + kQS * 16384;    // ring of kQS x (64 rows x 128 d)
constexpr uint32_t DK = DO + kQS * 16384;   // fp32 [128 d][128 keys]
constexpr uint32_t STATS = DK + 65536;      // [kQS slots][lse2 64 | delta 64] fp32
constexpr uint32_t BARS = STATS + kQS * 2 * 4 * BQ;
enum Bar { V_FULL = 0, K_FULL, K_READY, BLK_DONE, FOLD_DONE, Q_FULL = 5, Q_READY = Q_FULL + kQS,
           Q_EMPTY = Q_READY + kQS, S_FULL = Q_EMPTY + kQS, P_READY = S_FULL + 2, FINAL = P_READY + 2, N_BARS };
constexpr uint32_t TMEM_SLOT = BARS + 8 * N_BARS;
constexpr uint32_t ABORT = TMEM_SLOT + 4;
constexpr uint32_t TOTAL = ABORT + 4;
constexpr size_t kSmem = TOTAL + 1024;
static_assert(kSmem <= 227 * 1024, "shared memory budget");
// TMEM columns: buffer x at 128 x: S^T [0,64) (P^T packed in [0,32)), dP^T [64,128) (dS^T packed in [64,96)).
constexpr uint32_t C_BUF = 0, C_DV = 256, C_DKR = 384;
constexpr long long kWait = 1000000000LL;
}  // namespace kvw

// Iterates the blocks of row b that see keys [j0, j1) (same order in every
// role); with skip_abs, only the blocks with no abs key among [j0, j1)
// (the others go to the abs pass, dkdv_kernel with abs_only, which adds its
// part afterwards).
//
// The 64-row query tiles of the blocks it yields are numbered in order; with
// a chunk [qt0, qt1) only the blocks holding some of those tiles are yielded,
// and [lq0, lq1) are the block's own tiles of the chunk.
struct BlockIter {
  const AiAttnLayout* L;
  int b, j0, j1, bi, end, qt0, qt1, qcum = 0, lq0 = 0, lq1 = 0;
  bool skip_abs;
  __device__ BlockIter(const AiAttnLayout* L_, int b_, int j0_, int j1_, bool skip_abs_, int qt0_, int qt1_)
      : L(L_), b(b_), j0(j0_), j1(j1_), qt0(qt0_), qt1(qt1_), skip_abs(skip_abs_) {
    bi = L->row_blocks[b] - 1;
    end = L->row_blocks[b + 1];
  }
  __device__ bool next(Block& blk) {
    while (++bi < end) {
      blk = load_block(L->blocks, bi);
      if (blk.e <= j0 || blk.kv_lo >= j1 || max(blk.s, j0) >= blk.e) continue;
      if (skip_abs && blk.abs_in(j0, j1)) continue;
      const int nq = (blk.e - max(blk.s, j0) + kvw::BQ - 1) / kvw::BQ, c0 = qcum;
      qcum += nq;
      lq0 = max(qt0, c0) - c0;
      lq1 = min(qt1, c0 + nq) - c0;
      if (lq0 >= lq1) continue;
      return true;
    }
    return false;
  }
};

// BlockIter with one block of lookahead, grouping consecutive blocks into
// segments that give the key tile the same rotation: both 64-key chunks of
// [j0, j0 + 128) in the same rotation classes (the keys every block of the
// segment attends sit at the same positions).  Within a segment the rotated
// K tile is loaded once and dKrot accumulates in TMEM; it is folded into dK
// at the segment's end.  A block without classes for the tile is a segment
// of its own.
struct SegIter {
  BlockIter it, ahead;
  Block nxt;
  int2 sig = make_int2(-1, -1), sig_nxt = make_int2(-1, -1);
  bool has_nxt = false, started = false, seg_first = true, seg_last = true;
  bool prerot;
  int32_t* status;
  __device__ SegIter(const AiAttnLayout* L_, int b_, int j0_, int j1_, bool skip_abs_, int qt0_, int qt1_,
                     bool prerot_, int32_t* status_)
      : it(L_, b_, j0_, j1_, skip_abs_, qt0_, qt1_), ahead(it), prerot(prerot_), status(status_) {}
  // Rotation classes of the tile's two chunks in block bi, (-1, -1): none.
  __device__ int2 sig_of(int bi, const Block& blk) const {
    const AiAttnLayout& L = *it.L;
    const int base = block_classes(L, bi, prerot);
    if (base < 0 || it.j0 < blk.kv_lo || (blk.flags & AI_BLOCKF_OWNPOS)) return make_int2(-1, -1);
    const int i = (it.j0 - blk.kv_lo) / AI_ROT_CLASS_KEYS;
    const int n = 2 * ((blk.e - blk.kv_lo + 2 * AI_ROT_CLASS_KEYS - 1) / (2 * AI_ROT_CLASS_KEYS));
    const int c0 = chunk_class(L, base, i, status);
    const int c1 = i + 1 < n ? chunk_class(L, base, i + 1, status) : c0;  // past the block's keys
    return (c0 >= 0 && c1 >= 0) ? make_int2(c0, c1) : make_int2(-1, -1);
  }
  __device__ bool next(Block& blk) {
    if (!started) {
      started = true;
      has_nxt = ahead.next(nxt);
      if (has_nxt) sig_nxt = sig_of(ahead.bi, nxt);
    }
    if (!has_nxt) return false;
    const int2 prev = sig;
    it = ahead;
    blk = nxt;
    sig = sig_nxt;
    seg_first = !(sig.x >= 0 && sig.x == prev.x && sig.y == prev.y);
    has_nxt = ahead.next(nxt);
    sig_nxt = has_nxt ? sig_of(ahead.bi, nxt) : make_int2(-1, -1);
    seg_last = !(has_nxt && sig_nxt.x >= 0 && sig_nxt.x == sig.x && sig_nxt.y == sig.y);
    return true;
  }
};

__global__ void __launch_bounds__(kvw::kThreads, 1)
    dkdv_ws_kernel(const AiAttnBwdArgs a, const float* __restrict__ delta, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_q,
                   const __grid_constant__ CUtensorMap tm_do, const __grid_constant__ CUtensorMap tm_kr,
                   const __grid_constant__ CUtensorMap tm_kc, const int prerot, const int item_base,
                   const int skip_abs, const int32_t* __restrict__ chunks, float* __restrict__ partials,
                   const int hg) {
  using namespace kvw;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = tile::align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + ABORT);
  float* s_dk = reinterpret_cast<float*>(sm + DK);
  float* s_stats = reinterpret_cast<float*>(sm + STATS);
  auto bar = [&](int i) { return sbase + BARS + 8u * (uint32_t)i; };

  const AiAttnFwdArgs& f = a.fwd;
  const AiAttnLayout& L = f.layout;
  // A CTA runs one key tile whole, or one chunk of its query tiles when the
  // tile is split (kv_chunks): then it writes fp32 partial sums to `partials`.
  // CTA order (one-dimensional grid): the KV heads in groups of hg, one
  // group after the other; within a group the entries in their order
  // (costliest first) with the group's heads varying fastest.  A group's
  // CTAs read the query / dO rows of its heads only, which then stay in L2,
  // and its costliest entries start first, so its last wave holds short CTAs.
  const unsigned per_grp = (gridDim.x / (unsigned)a.fwd.num_kv_heads) * (unsigned)hg;
  const unsigned grp = blockIdx.x / per_grp, rem = blockIdx.x % per_grp;
  const int ent = (int)(rem / (unsigned)hg);
  int it_idx = item_base + ent, qt0 = 0, qt1 = 0x7fffffff, slot = -1;
  if (chunks) {
    const int32_t* c = chunks + 4 * (int64_t)ent;
    it_idx = c[0];
    qt0 = c[1];
    qt1 = c[2];
    slot = c[3];
  }
  const int32_t* item = L.kv_items + 4 * (int64_t)it_idx;
  const int b = item[0], j0 = item[1], j1 = item[2];
  const int hk = (int)(grp * (unsigned)hg + rem % (unsigned)hg), G = f.num_q_heads / f.num_kv_heads;
  const __half2* cs16 = static_cast<const __half2*>(L.rope_cs16);

  if (tid == 0) {
    for (int i = 0; i < N_BARS; ++i) {
      uint32_t count = 1;
      if (i == K_READY || (i >= Q_READY && i < Q_READY + kQS)) count = kRot;
      if (i == P_READY || i == P_READY + 1 || i == FOLD_DONE) count = 32 * 4 * kGroups;
      ptx::mbar_init(bar(i), count);
    }
    *s_abort = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 4 * kGroups + 1) {
    ptx::tmem_alloc(sbase + TMEM_SLOT, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + TMEM_SLOT);

  auto wait = [&](int i, uint32_t parity) -> bool {
    if (*s_abort) return false;
    if (!ptx::mbar_wait(bar(i), parity, kWait)) {
      report(f.status, AI_ERR_DEV_TIMEOUT);
      *s_abort = 1;
      return false;
    }
    return true;
  };
  // Steps of the current block of an iterator: its query tiles in the chunk x the group's heads.
  auto n_steps_of = [&](const BlockIter& bit) { return (bit.lq1 - bit.lq0) * G; };

  if (warp < 4 * kGroups) {
    // ------------------------------------------------------------ score groups
    const int t = warp / 4, lrow = tid % 128, j = j0 + lrow;
    // The fp32 dK accumulator entries this thread folds into and writes out
    // (key lrow, d in [16t, 16t + 16) and [64 + 16t, 80 + 16t)) are its own:
    // it clears them here, while the first tiles load.
#pragma unroll
    for (int x = 0; x < kCols; ++x) {
      s_dk[(kCols * t + x) * BN + lrow] = 0.f;
      s_dk[(64 + kCols * t + x) * BN + lrow] = 0.f;
    }
    const uint32_t lane_base = (uint32_t)((warp % 4) * 32) << 16;
    const float sl2 = f.scale * kLog2e, scale = f.scale;
    const float2 sl2x2 = make_float2(sl2, sl2), scalex2 = make_float2(scale, scale);
    SegIter sit(&L, b, j0, j1, skip_abs != 0, qt0, qt1, prerot != 0, f.status);
    const BlockIter& it = sit.it;
    Block blk;
    int s = 0, seg = -1;
    bool any = false;
    while (!*s_abort && sit.next(blk)) {
      any = true;
      seg += sit.seg_first ? 1 : 0;
      const int kmax = min(j1, blk.e), qs = max(blk.s, j0);
      uint32_t info = 0;
      if (j < kmax) info = (uint32_t)__ldg(L.key_info + blk.key_off + j);
      const bool key_ok = (info & AI_KEY_ATTN) != 0;
      const int nsteps = n_steps_of(it);
      for (int st = 0; st < nsteps; ++st, ++s) {
        const int x = s & 1, qslot = s % kQS, q0 = qs + (it.lq0 + st / G) * BQ, q1 = min(q0 + BQ, blk.e);
        if (!wait(Q_READY + qslot, (s / kQS) & 1) || !wait(S_FULL + x, (s >> 1) & 1)) break;
        ptx::tc_fence_after();
        // This group's 16 query columns of the step: c0 + [0, 16).
        const int c0 = kCols * t;
        const float* nlse2 = s_stats + qslot * 2 * BQ + c0;  // -lse2 per query row
        const float* ndlt = nlse2 + BQ;                       // -scale * delta per query row
        const uint32_t cb = tmem + lane_base + C_BUF + 128u * (uint32_t)x + (uint32_t)c0;
        uint32_t rs[kCols], rp[kCols];
        ptx::tmem_ld16(cb, rs);
        ptx::tmem_ld16(cb + 64, rp);
        // Whole-step masks: causal (j <= i) holds for every pair when the tile
        // lies wholly above the query rows, and every row is in the block when
        // the tile is full.
        const bool no_causal = j0 + BN - 1 <= q0, rows_full = q1 == q0 + BQ;
        // The step-uniform test sits outside the unrolled element loops (a
        // per-element branch there costs as much as the rest of the step).
        const bool plain = no_causal && rows_full;
        const int clo = j - q0 - c0, chi = q1 - q0 - c0;  // general path: clo <= c < chi
        uint32_t pk[kCols / 2], dk[kCols / 2];
        ptx::tmem_wait_ld();
        auto pair = [&](int x2, bool ok0, bool ok1) {
          const int c = 2 * x2;
          const float2 nl = *reinterpret_cast<const float2*>(nlse2 + c);
          const float2 nd = *reinterpret_cast<const float2*>(ndlt + c);
          float2 arg = __ffma2_rn(make_float2(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1])), sl2x2, nl);
          arg.x = ok0 ? arg.x : -CUDART_INF_F;
          arg.y = ok1 ? arg.y : -CUDART_INF_F;
          const float2 pp = make_float2(ptx::ex2(arg.x), ptx::ex2(arg.y));
          const float2 ds =
              __fmul2_rn(pp, __ffma2_rn(make_float2(__uint_as_float(rp[c]), __uint_as_float(rp[c + 1])), scalex2, nd));
          pk[x2] = tile::pack2(pp.x, pp.y);
          dk[x2] = tile::pack2(ds.x, ds.y);
        };
        if (plain) {
#pragma unroll
          for (int x2 = 0; x2 < kCols / 2; ++x2) pair(x2, key_ok, key_ok);
        } else {
#pragma unroll
          for (int x2 = 0; x2 < kCols / 2; ++x2) {
            const int c = 2 * x2;
            pair(x2, key_ok && c >= clo && c < chi, key_ok && c + 1 >= clo && c + 1 < chi);
          }
        }
        // P^T / dS^T of these columns go over the first 8 of the group's own
        // 16 score columns (bf16 pairs), where the dV / dK MMAs read them.
        ptx::tmem_st8(cb, pk);
        ptx::tmem_st8(cb + 64, dk);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(P_READY + x));
      }
      if (*s_abort) break;
      if (sit.seg_last) {
        // Fold the segment's dKrot into dK: dK += R(key position)^T dKrot;
        // group t takes the rotation pairs (d, d + 64) with d in [16t, 16t + 16).
        if (!wait(BLK_DONE, seg & 1)) break;
        ptx::tc_fence_after();
        const int p = key_row(info, L.n_pos, f.status);
        const uint4* tp = reinterpret_cast<const uint4*>(cs16 + (int64_t)p * (D / 2));
        {
          uint32_t g1[kCols], g2[kCols];
          ptx::tmem_ld16(tmem + lane_base + C_DKR + kCols * t, g1);
          ptx::tmem_ld16(tmem + lane_base + C_DKR + 64 + kCols * t, g2);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < kCols / 4; ++q) {
            const uint4 tv = __ldg(tp + (kCols / 4) * t + q);
            const __half2* h2 = reinterpret_cast<const __half2*>(&tv);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int xx = 4 * q + u, d = kCols * t + xx;
              const float2 csn = __half22float2(h2[u]);
              const float v1 = __uint_as_float(g1[xx]), v2 = __uint_as_float(g2[xx]);
              s_dk[d * BN + lrow] += v1 * csn.x + v2 * csn.y;
              s_dk[(d + 64) * BN + lrow] += v2 * csn.x - v1 * csn.y;
            }
          }
        }
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(FOLD_DONE));
      }
    }
    // Epilogue: group t writes the columns it folded, d in [16t, 16t + 16)
    // and [64 + 16t, 80 + 16t), of dK (smem) and dV (TMEM; the last block's
    // MMAs are done, its fold waited for them).
    if (!*s_abort) {
      ptx::tc_fence_after();
      __nv_bfloat16* dk_row =
          static_cast<__nv_bfloat16*>(a.dk.ptr) + b * a.dk.stride_b + hk * a.dk.stride_h + (int64_t)j * a.dk.stride_t;
      __nv_bfloat16* dv_row =
          static_cast<__nv_bfloat16*>(a.dv.ptr) + b * a.dv.stride_b + hk * a.dv.stride_h + (int64_t)j * a.dv.stride_t;
      // A chunk of a split key tile leaves fp32 partial sums instead:
      // [slot][kv head][dK, dV][key][d].
      float* part = slot >= 0 ? partials + (((int64_t)slot * f.num_kv_heads + hk) * 2) * (BN * D) + lrow * D : nullptr;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int d0 = kCols * t + 64 * h2;
        float v[kCols];
#pragma unroll
        for (int x = 0; x < kCols; ++x) v[x] = s_dk[(d0 + x) * BN + lrow];
        if (j < j1 && part) {
#pragma unroll
          for (int x = 0; x < kCols; x += 4)
            *reinterpret_cast<float4*>(part + d0 + x) = make_float4(v[x], v[x + 1], v[x + 2], v[x + 3]);
        } else if (j < j1) {
          *reinterpret_cast<uint4*>(dk_row + d0) = tile::pack8(*reinterpret_cast<const float(*)[8]>(v));
          *reinterpret_cast<uint4*>(dk_row + d0 + 8) = tile::pack8(*reinterpret_cast<const float(*)[8]>(v + 8));
        }
        uint32_t rr[kCols];
        if (any) {
          ptx::tmem_ld16(tmem + lane_base + C_DV + d0, rr);
          ptx::tmem_wait_ld();
        }
#pragma unroll
        for (int x = 0; x < kCols; ++x) v[x] = any ? __uint_as_float(rr[x]) : 0.f;
        if (j < j1 && part) {
#pragma unroll
          for (int x = 0; x < kCols; x += 4)
            *reinterpret_cast<float4*>(part + BN * D + d0 + x) = make_float4(v[x], v[x + 1], v[x + 2], v[x + 3]);
        } else if (j < j1) {
          *reinterpret_cast<uint4*>(dv_row + d0) = tile::pack8(*reinterpret_cast<const float(*)[8]>(v));
          *reinterpret_cast<uint4*>(dv_row + d0 + 8) = tile::pack8(*reinterpret_cast<const float(*)[8]>(v + 8));
        }
      }
    }
  } else if (warp == 4 * kGroups) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      ptx::prefetch_tmap(&tm_k);
      ptx::prefetch_tmap(&tm_v);
      ptx::prefetch_tmap(&tm_q);
      ptx::prefetch_tmap(&tm_do);
      ptx::mbar_arrive_expect_tx(bar(V_FULL), 32768);
      ptx::tma_load_4d(sbase + V, &tm_v, bar(V_FULL), 0, j0, hk, b);
      ptx::tma_load_4d(sbase + V + 16384, &tm_v, bar(V_FULL), 64, j0, hk, b);
      SegIter sit(&L, b, j0, j1, skip_abs != 0, qt0, qt1, prerot != 0, f.status);
      const BlockIter& it = sit.it;
      Block blk;
      int s = 0, seg = -1;
      bool ok = true;
      while (ok && sit.next(blk)) {
        if (sit.seg_first) {
          // A new segment's K tile, once the previous segment's MMAs are done.
          if (++seg > 0 && !wait(BLK_DONE, (seg - 1) & 1)) break;
          ptx::mbar_arrive_expect_tx(bar(K_FULL), 32768);
          if (sit.sig.x >= 0) {
            // rows 0-63 and 64-127 from the two chunks' rotated copies
            ptx::tma_load_4d(sbase + K, &tm_kc, bar(K_FULL), 0, 0, hk, sit.sig.x);
            ptx::tma_load_4d(sbase + K + 8192, &tm_kc, bar(K_FULL), 0, 0, hk, sit.sig.y);
            ptx::tma_load_4d(sbase + K + 16384, &tm_kc, bar(K_FULL), 64, 0, hk, sit.sig.x);
            ptx::tma_load_4d(sbase + K + 16384 + 8192, &tm_kc, bar(K_FULL), 64, 0, hk, sit.sig.y);
          } else {
            const CUtensorMap* mk = (prerot && (blk.flags & AI_BLOCKF_OWNPOS)) ? &tm_kr : &tm_k;
            ptx::tma_load_4d(sbase + K, mk, bar(K_FULL), 0, j0, hk, b);
            ptx::tma_load_4d(sbase + K + 16384, mk, bar(K_FULL), 64, j0, hk, b);
          }
        }
        const int qs = max(blk.s, j0), nsteps = n_steps_of(it);
        for (int st = 0; st < nsteps; ++st, ++s) {
          const int qslot = s % kQS, q0 = qs + (it.lq0 + st / G) * BQ, h = hk * G + st % G;
          if (s >= kQS && !wait(Q_EMPTY + qslot, ((s / kQS) - 1) & 1)) {
            ok = false;
            break;
          }
          const uint32_t qb = sbase + Q + 16384u * (uint32_t)qslot, ob = sbase + DO + 16384u * (uint32_t)qslot;
          ptx::mbar_arrive_expect_tx(bar(Q_FULL + qslot), 32768);
          ptx::tma_load_4d(qb, &tm_q, bar(Q_FULL + qslot), 0, q0, h, b);
          ptx::tma_load_4d(qb + 8192, &tm_q, bar(Q_FULL + qslot), 64, q0, h, b);
          ptx::tma_load_4d(ob, &tm_do, bar(Q_FULL + qslot), 0, q0, h, b);
          ptx::tma_load_4d(ob + 8192, &tm_do, bar(Q_FULL + qslot), 64, q0, h, b);
        }
      }
    }
  } else if (warp == 4 * kGroups + 1) {
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
    constexpr uint32_t idesc_st = ptx::idesc_bf16_f32(BN, BQ, false, false);
    constexpr uint32_t idesc_acc = ptx::idesc_bf16_f32(BN, D, false, true);
    // Every operand tile sits at a constant offset from one of four base
    // descriptors, and a descriptor's low 14 bits are the shared address / 16
    // (addresses stay below 256 KB, so no carry leaves that field): each MMA's
    // descriptor is one add, and a step's slot one more.
    const uint64_t d_k = ptx::sdesc_sw128(sbase + K, 16, 1024);
    const uint64_t d_v = ptx::sdesc_sw128(sbase + V, 16, 1024);
    const uint64_t d_q = ptx::sdesc_sw128(sbase + Q, 16, 1024);     // Q / dO K-major (scores)
    const uint64_t d_qa = ptx::sdesc_sw128(sbase + Q, 8192, 1024);  // Q / dO MN-major (dV / dK)
    constexpr uint64_t kSlot = 16384u >> 4, kDo = (uint64_t)(DO - Q) >> 4;
    auto issue_scores = [&](int x, int slot) {
      const uint64_t dq = d_q + kSlot * (uint64_t)slot;
      const uint32_t cb = tmem + C_BUF + 128u * (uint32_t)x;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t ao = (uint64_t)(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
        const uint64_t bo = (uint64_t)(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4);
        ptx::mma_ss_w(cb, d_k + ao, dq + bo, idesc_st, kk > 0);
        ptx::mma_ss_w(cb + 64, d_v + ao, dq + kDo + bo, idesc_st, kk > 0);
      }
      ptx::mma_commit_w(bar(S_FULL + x));
    };
    // Q / dO slot and Q_READY parity of a step, advanced one step at a time.
    auto advance = [](int& slot, uint32_t& phase) {
      if (++slot == kQS) {
        slot = 0;
        phase ^= 1u;
      }
    };
    bool ok = wait_u(V_FULL, 0);
    SegIter sit(&L, b, j0, j1, skip_abs != 0, qt0, qt1, prerot != 0, f.status);
    const BlockIter& it = sit.it;
    Block blk;
    int s = 0, seg = -1, sl = 0;
    uint32_t ph = 0;
    bool dv_started = false;
    while (ok && sit.next(blk)) {
      const int nsteps = n_steps_of(it);
      const bool seg_first = sit.seg_first;
      if (seg_first) {
        ++seg;
        if (!wait_u(K_READY, seg & 1)) break;
      }
      ptx::tc_fence_after();
      const int sb = s;
      // scores of the block's first step
      if (!wait_u(Q_READY + sl, ph)) break;
      ptx::tc_fence_after();
      issue_scores(s & 1, sl);
      int sl1 = sl;  // step s + 1
      uint32_t ph1 = ph;
      advance(sl1, ph1);
      for (; s < sb + nsteps; ++s) {
        const int x = s & 1;
        if (s + 1 < sb + nsteps) {
          if (!wait_u(Q_READY + sl1, ph1)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          issue_scores(x ^ 1, sl1);
        }
        if (!wait_u(P_READY + x, (s >> 1) & 1)) {
          ok = false;
          break;
        }
        if (s == sb && seg_first && seg > 0 && !wait_u(FOLD_DONE, (seg - 1) & 1)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint64_t dqa = d_qa + kSlot * (uint64_t)sl;
        const uint32_t cb = tmem + C_BUF + 128u * (uint32_t)x;
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          // query rows 16 kk .. 16 kk + 15: packed by score group kk
          const uint32_t ca = cb + (uint32_t)(kCols * kk);
          const uint64_t ko = (uint64_t)(2048 * kk) >> 4;
          ptx::mma_ts_w(tmem + C_DV, ca, dqa + kDo + ko, idesc_acc, (dv_started || kk > 0) ? 1u : 0u);
          ptx::mma_ts_w(tmem + C_DKR, ca + 64u, dqa + ko, idesc_acc, (s > sb || kk > 0 || !seg_first) ? 1u : 0u);
        }
        ptx::mma_commit_w(bar(Q_EMPTY + sl));
        dv_started = true;
        sl = sl1;
        ph = ph1;
        advance(sl1, ph1);
      }
      if (!ok) break;
      if (sit.seg_last) ptx::mma_commit_w(bar(BLK_DONE));
    }
    ptx::mma_commit_w(bar(FINAL));
    ptx::mbar_wait(bar(FINAL), 0, kWait);
  } else {
    // ------------------------------------------------------------ rotation (warps 18-19)
    const int rt = tid - 32 * (4 * kGroups + 2);  // 0..63: Q row rt, K rows rt and rt + 64
    SegIter sit(&L, b, j0, j1, skip_abs != 0, qt0, qt1, prerot != 0, f.status);
    const BlockIter& it = sit.it;
    Block blk;
    int s = 0, seg = -1;
    while (!*s_abort && sit.next(blk)) {
      // K rows of a new segment by its key positions (already rotated when
      // they come from k_rot or the rotation-class copies).
      if (sit.seg_first) {
        ++seg;
        const bool k_pre = (prerot && (blk.flags & AI_BLOCKF_OWNPOS)) || sit.sig.x >= 0;
        const int kend = min(j1, blk.e);
        int p[2] = {0, 0};
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int key = j0 + rt + kRot * u;
          if (key < kend) p[u] = key_row((uint32_t)__ldg(L.key_info + blk.key_off + key), L.n_pos, f.status);
        }
        if (!wait(K_FULL, seg & 1)) break;
#pragma unroll 1
        for (int u = 0; u < 2; ++u) {
          const int kr = rt + kRot * u;
          if (k_pre || j0 + kr >= kend) continue;
          // (a quarter of the row at a time: these warps have 96 registers)
          const uint4* tp = reinterpret_cast<const uint4*>(cs16 + (int64_t)(u ? p[1] : p[0]) * (D / 2));
#pragma unroll
          for (int qt = 0; qt < 4; ++qt) {
            uint4 tab[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) tab[c] = __ldg(tp + 4 * qt + c);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              uint4* pa = reinterpret_cast<uint4*>(sm + K + chunk_off<BN>(kr, 2 * qt + c));
              uint4* pb = reinterpret_cast<uint4*>(sm + K + chunk_off<BN>(kr, 2 * qt + c + 8));
              uint4 y1, y2;
              tile::rotate8h(*pa, *pb, tab[2 * c], tab[2 * c + 1], y1, y2);
              *pa = y1;
              *pb = y2;
            }
          }
        }
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(bar(K_READY));
      }
      const int qs = max(blk.s, j0), nsteps = n_steps_of(it);
      const int r = rt;
      for (int st = 0; st < nsteps; ++st, ++s) {
        const int qslot = s % kQS, q0 = qs + (it.lq0 + st / G) * BQ, q1 = min(q0 + BQ, blk.e), h = hk * G + st % G;
        const int i = q0 + r;
        // Row position and row statistics are fetched before the TMA wait.
        int p = 0;
        float l2 = CUDART_INF_F, dl = 0.f;
        if (i < q1) {
          p = clamp_row(__ldg(L.q_pos + (int64_t)b * f.seq_len + i), L.n_pos, f.status);
          const int64_t idx = ((int64_t)b * f.num_q_heads + h) * f.seq_len + i;
          l2 = lse_log2(__ldg(f.lse + idx));
          dl = __ldg(delta + idx);
        }
        if (!wait(Q_FULL + qslot, (s / kQS) & 1)) break;
        const uint32_t qb = Q + 16384u * (uint32_t)qslot;
        if (!prerot) {
          const uint4* tp = reinterpret_cast<const uint4*>(cs16 + (int64_t)p * (D / 2));
#pragma unroll
          for (int qt = 0; qt < 4; ++qt) {
            uint4 tab[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) tab[c] = __ldg(tp + 4 * qt + c);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              uint4* pa = reinterpret_cast<uint4*>(sm + qb + chunk_off<BQ>(r, 2 * qt + c));
              uint4* pb = reinterpret_cast<uint4*>(sm + qb + chunk_off<BQ>(r, 2 * qt + c + 8));
              uint4 y1, y2;
              tile::rotate8h(*pa, *pb, tab[2 * c], tab[2 * c + 1], y1, y2);
              *pa = y1;
              *pb = y2;
            }
          }
        }
        s_stats[qslot * 2 * BQ + r] = -l2;
        s_stats[qslot * 2 * BQ + BQ + r] = -(dl * f.scale);
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(bar(Q_READY + qslot));
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 4 * kGroups + 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

bool strides_ok(const AiTensor4& t) {
  return ((uintptr_t)t.ptr % 16 == 0) && (t.stride_b % 8 == 0) && (t.stride_h % 8 == 0) && (t.stride_t % 8 == 0);
}

// Sums the partial dK / dV of a split key tile in chunk order and writes the
// bf16 rows: one CTA per (split key tile, KV head), a warp per key, four d a lane.
__global__ void __launch_bounds__(256) dkdv_reduce_kernel(const AiAttnBwdArgs a, const float* __restrict__ partials) {
  const AiAttnFwdArgs& f = a.fwd;
  const AiAttnLayout& L = f.layout;
  const int32_t* red = L.kv_reduce + 4 * (int64_t)blockIdx.x;
  const int32_t* item = L.kv_items + 4 * (int64_t)red[0];
  const int b = item[0], j0 = item[1], j1 = item[2], first = red[1], n = red[2];
  const int hk = blockIdx.y, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr int BN = kvw::BN;
  for (int kk = warp; kk < BN && j0 + kk < j1; kk += 8) {
    float4 dk = make_float4(0.f, 0.f, 0.f, 0.f), dv = dk;
    for (int c = 0; c < n; ++c) {
      const float* part = partials + (((int64_t)(first + c) * f.num_kv_heads + hk) * 2) * (BN * D) + kk * D + 4 * lane;
      const float4 x = *reinterpret_cast<const float4*>(part);
      const float4 y = *reinterpret_cast<const float4*>(part + BN * D);
      dk.x += x.x; dk.y += x.y; dk.z += x.z; dk.w += x.w;
      dv.x += y.x; dv.y += y.y; dv.z += y.z; dv.w += y.w;
    }
    const int j = j0 + kk;
    __nv_bfloat16* dk_row =
        static_cast<__nv_bfloat16*>(a.dk.ptr) + b * a.dk.stride_b + hk * a.dk.stride_h + (int64_t)j * a.dk.stride_t;
    __nv_bfloat16* dv_row =
        static_cast<__nv_bfloat16*>(a.dv.ptr) + b * a.dv.stride_b + hk * a.dv.stride_h + (int64_t)j * a.dv.stride_t;
    __nv_bfloat162 k2[2] = {__floats2bfloat162_rn(dk.x, dk.y), __floats2bfloat162_rn(dk.z, dk.w)};
    __nv_bfloat162 v2[2] = {__floats2bfloat162_rn(dv.x, dv.y), __floats2bfloat162_rn(dv.z, dv.w)};
    *reinterpret_cast<uint2*>(dk_row + 4 * lane) = *reinterpret_cast<const uint2*>(k2);
    *reinterpret_cast<uint2*>(dv_row + 4 * lane) = *reinterpret_cast<const uint2*>(v2);
  }
}

}  // namespace sm100bwd

bool sm100_bwd_supported(int dtype, int head_dim) { return dtype == AI_DTYPE_BF16 && head_dim == sm100bwd::D; }

int sm100_kv_tile_rows() { return sm100bwd::kv::BN; }

size_t sm100_kv_partial_bytes(const AiAttnFwdArgs& f) {
  const AiAttnLayout& L = f.layout;
  if (L.n_kv_chunks <= 0 || L.n_kv_partials <= 0 || !L.kv_chunks || !L.kv_reduce) return 0;
  // Split the key tiles only when the costliest one outweighs the average
  // work of an SM (one CTA per key tile and KV head otherwise sets the pace).
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const double avg = (double)L.kv_cost_total * f.num_kv_heads / (sms > 0 ? sms : 148);
  if ((double)L.kv_cost_max <= 1.25 * avg) return 0;
  const size_t n = (size_t)L.n_kv_partials * f.num_kv_heads * 2 * sm100bwd::kvw::BN * sm100bwd::D * sizeof(float);
  return (n + 255) & ~size_t(255);
}

size_t sm100_dq_abs_part_bytes(const AiAttnFwdArgs& f) {
  const int G = f.num_kv_heads > 0 ? f.num_q_heads / f.num_kv_heads : 0;
  if (!sm100_bwd_supported(f.dtype, f.head_dim) || G % 2 != 0 || f.layout.n_fwd_abs_items <= 0) return 0;
  const size_t n = (size_t)f.layout.n_fwd_abs_items * f.num_q_heads * sm100bwd::dq::BM * sm100bwd::D * sizeof(float);
  return (n + 255) & ~size_t(255);
}

int sm100_bwd(const AiAttnBwdArgs& a, float* delta, void* rot, bool rot_ready, float* partials, float* dq_part,
              int parts, cudaStream_t st, cudaError_t* cuda_err) {
  using namespace sm100bwd;
  const AiAttnFwdArgs& f = a.fwd;
  const bool do_dq = (parts & AI_BWD_DQ) != 0, do_kv = (parts & AI_BWD_DKDV) != 0;
  if (!strides_ok(f.q) || !strides_ok(f.k) || !strides_ok(f.v) || !strides_ok(a.dout) || !strides_ok(a.dq) ||
      !strides_ok(a.dk) || !strides_ok(a.dv))
    return AI_ERR_STRIDE;
  // With `rot` scratch, Q and K are rotated once (HBM-bound) and the
  // warp-specialised kernels read the rotated copies.
  AiTensor4 qr{}, kr{}, kc{};
  const bool pre = rot != nullptr;
  if (pre && !sm100_rotated_views(f, rot, &qr, &kr, &kc)) return AI_ERR_ALIGN;
  cudaError_t e = cudaSuccess;
  if (do_dq) {  // (a dK/dV-only call reads what the dQ call left in the workspace)
    {
      ProfScope ps(AI_PROF_DELTA, st);
      e = bwd_delta(a, delta, st);
    }
    if (e == cudaSuccess && pre && !rot_ready) e = prerot(f, rot, st);
  }
  // The abs split (with the rotated copies and room for dq_part): the
  // persistent dQ kernel also runs the abs-block items' key tiles that hold
  // no abs key and leaves their dQrot in dq_part; the one-head kernel, later
  // in the stream, adds the tiles with abs keys and writes those rows.
  const int Gq = f.num_q_heads / f.num_kv_heads;
  const bool dq_split = pre && dq_part && Gq % 2 == 0 && f.layout.n_fwd_abs_items > 0;
  CUtensorMap dq_tk, dq_tv, dq_tkc;  // maps of the deferred one-head dQ launch
  bool dq_deferred = false;
  if (e == cudaSuccess && do_dq && f.layout.n_fwd_items > 0) {
    CUtensorMap tk, tv, tqr, tdo, tkr;
    if (!sm100_make_map(&tk, f.k, f.batch, f.num_kv_heads, f.seq_len, dq::BN) ||
        !sm100_make_map(&tv, f.v, f.batch, f.num_kv_heads, f.seq_len, dq::BN) ||
        !sm100_make_map(&tdo, a.dout, f.batch, f.num_q_heads, f.seq_len, dq::BM))
      return AI_ERR_TMA;
    tqr = tk;
    tkr = tk;
    if (pre && (!sm100_make_map(&tqr, qr, f.batch, f.num_q_heads, f.seq_len, dq::BM) ||
                !sm100_make_map(&tkr, kr, f.batch, f.num_kv_heads, f.seq_len, dq::BN)))
      return AI_ERR_TMA;
    // Items of blocks with abs keys (all items when a GQA group has an odd
    // number of heads) on the one-head kernel, the rest two heads per CTA.
    const int G = f.num_q_heads / f.num_kv_heads;
    const int n_single = (G % 2 == 0) ? f.layout.n_fwd_abs_items : f.layout.n_fwd_items;
    const int n_pair = f.layout.n_fwd_items - n_single;
    CUtensorMap tkc = tk;
    if (pre && f.layout.n_rot_classes > 0 &&
        !sm100_make_map(&tkc, kc, f.layout.n_rot_classes, f.num_kv_heads, AI_ROT_CLASS_KEYS, AI_ROT_CLASS_KEYS))
      return AI_ERR_TMA;
    if (n_single > 0 && dq_split) {
      dq_tk = tk;
      dq_tv = tv;
      dq_tkc = tkc;
      dq_deferred = true;
    } else if (n_single > 0) {
      e = cudaFuncSetAttribute(dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dq::kSmem);
      if (e == cudaSuccess) {
        ProfScope ps(AI_PROF_DQ, st);
        dq_kernel<<<dim3(n_single, f.num_q_heads), kThreads, dq::kSmem, st>>>(a, delta, tk, tv, tkc, pre ? 1 : 0,
                                                                              nullptr);
        e = cudaGetLastError();
      }
    }
    CUtensorMap tqr64 = tk, tdo64 = tk;
    if (!sm100_make_map(&tdo64, a.dout, f.batch, f.num_q_heads, f.seq_len, dq::BM / 2)) return AI_ERR_TMA;
    if (pre && !sm100_make_map(&tqr64, qr, f.batch, f.num_q_heads, f.seq_len, dq::BM / 2)) return AI_ERR_TMA;
    // Persistent: one CTA per SM walks the units (the forward's order): with
    // the split, the abs-block items' units first, then four-head units of
    // the short items when a GQA group has a multiple of four query heads,
    // then two-head units of the other items.
    UnitPlan up{f.layout.n_fwd_abs_items, 0, 0, 0}, up_abs{0, 0, 0, 0};
    if (G % 2 == 0) {
      up.n_pack_items = (G % 4 == 0) ? f.layout.n_fwd_short_items : 0;
      up.n_pack_units = up.n_pack_items * (f.num_q_heads / 4);
      up.n_units = up.n_pack_units + (n_pair - up.n_pack_items) * (f.num_q_heads / 2);
      if (dq_split) {
        up_abs.n_pack_items = (G % 4 == 0) ? f.layout.n_fwd_abs_short_items : 0;
        up_abs.n_pack_units = up_abs.n_pack_items * (f.num_q_heads / 4);
        up_abs.n_units =
            up_abs.n_pack_units + (f.layout.n_fwd_abs_items - up_abs.n_pack_items) * (f.num_q_heads / 2);
      }
    }
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    auto launch_pers = [&](auto kernel, const UnitPlan& p, bool after_pers) {
      if (p.n_units <= 0 || e != cudaSuccess) return;
      const int grid = p.n_units < sms ? p.n_units : sms;
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dqw::kSmem);
      if (e == cudaSuccess) {
        ProfScope ps(AI_PROF_DQ, st);
        // Right after the other persistent launch (which shares no data with
        // this one) it starts by programmatic dependent launch.
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(dqw::kThreads);
        cfg.dynamicSmemBytes = dqw::kSmem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = after_pers ? 1 : 0;
        e = cudaLaunchKernelEx(&cfg, kernel, a, delta, tk, tv, tqr, tdo, tkr, tqr64, tdo64, tkc, pre ? 1 : 0, p,
                               dq_split ? dq_part : (float*)nullptr);
        if (e == cudaSuccess) e = cudaGetLastError();
      }
    };
    // The abs launch first: the other launch, then the dK/dV pass below,
    // start their CTAs under the tail of the launch right before them
    // (programmatic dependent launch).
    if (dq_split) launch_pers(dq_pers_kernel<true>, up_abs, false);
    launch_pers(dq_pers_kernel<false>, up, dq_split && up_abs.n_units > 0);
  }
  // The deferred one-head dQ launch (after the dK/dV pass below, so that the
  // dK/dV CTAs start under the persistent dQ as before).
  auto launch_dq_deferred = [&]() {
    if (!dq_deferred || e != cudaSuccess) return;
    dq_deferred = false;
    e = cudaFuncSetAttribute(dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dq::kSmem);
    if (e == cudaSuccess) {
      ProfScope ps(AI_PROF_DQ, st);
      dq_kernel<<<dim3(f.layout.n_fwd_abs_items, f.num_q_heads), kThreads, dq::kSmem, st>>>(
          a, delta, dq_tk, dq_tv, dq_tkc, 1, dq_part);
      e = cudaGetLastError();
      // The short abs items ran chunked: sum their chunks' rows.
      if (e == cudaSuccess) {
        dq_abs_combine_kernel<<<dim3(f.layout.n_fwd_abs_items, f.num_q_heads), D, 0, st>>>(a, dq_part);
        e = cudaGetLastError();
      }
    }
  };
  if (e == cudaSuccess && do_kv && f.layout.n_kv_items > 0) {
    CUtensorMap tk, tv, tq, tdo, tqr, tkr;
    if (!sm100_make_map(&tk, f.k, f.batch, f.num_kv_heads, f.seq_len, kv::BN) ||
        !sm100_make_map(&tv, f.v, f.batch, f.num_kv_heads, f.seq_len, kv::BN) ||
        !sm100_make_map(&tq, f.q, f.batch, f.num_q_heads, f.seq_len, kv::BQ) ||
        !sm100_make_map(&tdo, a.dout, f.batch, f.num_q_heads, f.seq_len, kv::BQ))
      return AI_ERR_TMA;
    tqr = tq;
    tkr = tk;
    if (pre && (!sm100_make_map(&tqr, qr, f.batch, f.num_q_heads, f.seq_len, kv::BQ) ||
                !sm100_make_map(&tkr, kr, f.batch, f.num_kv_heads, f.seq_len, kv::BN)))
      return AI_ERR_TMA;
    CUtensorMap tkc = tk;
    if (pre && f.layout.n_rot_classes > 0 &&
        !sm100_make_map(&tkc, kc, f.layout.n_rot_classes, f.num_kv_heads, AI_ROT_CLASS_KEYS, AI_ROT_CLASS_KEYS))
      return AI_ERR_TMA;
    // Every key tile runs on the warp-specialised kernel for the blocks
    // without abs keys; then the key tiles that blocks with abs keys see
    // run on the one-warpgroup kernel for those blocks only, adding their
    // part to the rows the first pass wrote (stream order, no atomics).
    const int n_abs = f.layout.n_kv_abs_items, n_plain = f.layout.n_kv_items;
    if (n_plain > 0) {
      e = cudaFuncSetAttribute(dkdv_ws_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kvw::kSmem);
      if (e == cudaSuccess) {
        ProfScope ps(AI_PROF_DKDV, st);
        // Programmatic dependent launch: the kernel before this one (the
        // persistent dQ, which reads nothing this one writes and writes
        // nothing it reads) signals at the start of each CTA, so these CTAs
        // fill the SMs its CTAs leave; everything before that kernel is done.
        cudaLaunchConfig_t cfg = {};
        const bool split = partials != nullptr;
        const unsigned n_ent = (unsigned)(split ? f.layout.n_kv_chunks : n_plain);
        // Head groups as small as keep one and a half waves of CTAs in a
        // group: smaller groups keep a group's query / dO rows in L2, larger
        // ones shorten the tail of each group's last wave (measured on B200:
        // config 1 takes groups of two KV heads, 0.424 ms against 0.435 ms
        // with four; config 4 one head, 2.10 ms against 2.16 ms with two;
        // configs 2a and 3 run alike with groups of 4 or 8, 1 or 2).
        int hg = 1, dev = 0, sms = 148;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        while (hg < f.num_kv_heads && f.num_kv_heads % (2 * hg) == 0 && (int64_t)n_ent * hg * 2 < 3 * (int64_t)sms)
          hg *= 2;
        cfg.gridDim = dim3(n_ent * (unsigned)f.num_kv_heads);
        cfg.blockDim = dim3(kvw::kThreads);
        cfg.dynamicSmemBytes = kvw::kSmem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, dkdv_ws_kernel, a, (const float*)delta, tk, tv, pre ? tqr : tq, tdo, tkr, tkc,
                               pre ? 1 : 0, 0, n_abs > 0 ? 1 : 0, split ? f.layout.kv_chunks : (const int32_t*)nullptr,
                               partials, hg);
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e == cudaSuccess && split && f.layout.n_kv_reduce > 0) {
          dkdv_reduce_kernel<<<dim3(f.layout.n_kv_reduce, f.num_kv_heads), 256, 0, st>>>(a, partials);
          e = cudaGetLastError();
        }
      }
    }
    launch_dq_deferred();
    if (e == cudaSuccess && n_abs > 0) {
      // Boxes of 64 / G rows for the steps that pack a group's heads.
      const int Gk = f.num_q_heads / f.num_kv_heads;
      CUtensorMap tqp = tq, tdop = tdo, tqrp = tqr;
      if ((Gk == 2 || Gk == 4 || Gk == 8) &&
          (!sm100_make_map(&tqp, f.q, f.batch, f.num_q_heads, f.seq_len, kv::BQ / Gk) ||
           !sm100_make_map(&tdop, a.dout, f.batch, f.num_q_heads, f.seq_len, kv::BQ / Gk) ||
           (pre && !sm100_make_map(&tqrp, qr, f.batch, f.num_q_heads, f.seq_len, kv::BQ / Gk))))
        return AI_ERR_TMA;
      e = cudaFuncSetAttribute(dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kv::kSmem);
      if (e == cudaSuccess) {
        ProfScope ps(AI_PROF_DKDV, st);
        dkdv_kernel<<<dim3((unsigned)n_abs * (unsigned)f.num_kv_heads), kThreads, kv::kSmem, st>>>(a, delta, tk, tv, tq, tdo, tqp, tdop,
                                                                               tkc, tqr, tqrp, pre ? 1 : 0, 1);
        e = cudaGetLastError();
      }
    }
  }
  launch_dq_deferred();  // (a dQ-only call, or no key tiles: not launched above)
  if (e == cudaSuccess && do_dq && !f.layout.all_rows_owned) {
    ProfScope ps(AI_PROF_BWD_FILL, st);
    e = bwd_fill(a, st);
  }
  if (cuda_err) *cuda_err = e;
  return e == cudaSuccess ? AI_OK : AI_ERR_LAUNCH;
}

}  // namespace ai
