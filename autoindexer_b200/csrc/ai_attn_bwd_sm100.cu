// Backward of the chain-of-edits attention on sm_100a tensor cores
// (tcgen05.mma, TMEM accumulators, TMA), bf16 in / fp32 accumulate,
// head_dim 128.  Two kernels, no atomics (deterministic):
//
// dq_kernel  (Q-stationary; one CTA = one forward work item x one query head,
//             thread = query row = TMEM lane):
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
//   group: S^T = Krot.Qrot^T (abs keys take Krot.Q^T: a per-thread choice,
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
constexpr uint32_t INFO = DSA + 16384;
constexpr uint32_t BAR_TMA = INFO + 4 * BN;
constexpr uint32_t BAR_MMA = BAR_TMA + 8;
constexpr uint32_t TMEM_SLOT = BAR_MMA + 8;
constexpr uint32_t ABORT = TMEM_SLOT + 4;
constexpr uint32_t TOTAL = ABORT + 4;
constexpr size_t kSmem = TOTAL + 1024;
constexpr uint32_t C_S = 0, C_DP = 64, C_DQR = 128, C_DQA = 256, C_SA = 384;
}  // namespace dq

__global__ void __launch_bounds__(kThreads, 1)
    dq_kernel(const AiAttnBwdArgs a, const float* __restrict__ delta, const __grid_constant__ CUtensorMap tm_k,
              const __grid_constant__ CUtensorMap tm_v) {
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
  const int h = blockIdx.y, G = f.num_q_heads / f.num_kv_heads, hk = h / G, b = blk.row;
  const bool has_abs = (blk.flags & AI_BLOCKF_ABS) != 0;
  const int kv_hi = min(blk.e, q1);
  const int i = q0 + tid;

  if (tid == 0) {
    ptx::mbar_init(bar_tma, 1);
    ptx::mbar_init(bar_mma, 1);
    *s_abort = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tm_k);
    ptx::prefetch_tmap(&tm_v);
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
  uint32_t ph_tma = 0, ph_mma = 0;
  int n_tiles = 0;
  bool aborted = false;

  for (int k0 = blk.kv_lo; k0 < kv_hi; k0 += BN) {
    if (tid == 0) {
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive_expect_tx(bar_tma, 2 * 16384);
      ptx::tma_load_4d(sbase + KR, &tm_k, bar_tma, 0, k0, hk, b);
      ptx::tma_load_4d(sbase + KR + 8192, &tm_k, bar_tma, 64, k0, hk, b);
      ptx::tma_load_4d(sbase + VV, &tm_v, bar_tma, 0, k0, hk, b);
      ptx::tma_load_4d(sbase + VV + 8192, &tm_v, bar_tma, 64, k0, hk, b);
    }
    wait_or_flag(bar_tma, ph_tma, s_abort, f.status);
    __syncthreads();
    if (*s_abort) { aborted = true; break; }

    // Rotate key rows in place: thread -> (row tid % 64, chunk pairs 4*(tid/64) .. +3).
    {
      const int r = tid & 63, cg = tid >> 6, j = k0 + r;
      uint32_t info = 0;
      if (j < kv_hi) {
        info = (uint32_t)L.key_info[blk.key_off + j];
        const int p = key_row(info, L.n_pos, f.status);
        const float* cs = L.rope_cos + (int64_t)p * (D / 2);
        const float* sn = L.rope_sin + (int64_t)p * (D / 2);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = 4 * cg + cc;
          uint4* pa = reinterpret_cast<uint4*>(sm + KR + chunk_off<BN>(r, c));
          uint4* pb = reinterpret_cast<uint4*>(sm + KR + chunk_off<BN>(r, c + 8));
          uint4 y1, y2;
          rotate8(*pa, *pb, cs + 8 * c, sn + 8 * c, y1, y2);
          *pa = y1;
          *pb = y2;
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
        ptx::mma_ss(tmem + C_S, ptx::sdesc_sw128(sbase + QR + ao, 16, 1024), ptx::sdesc_sw128(sbase + KR + bo, 16, 1024),
                    idesc_s, kk > 0);
        ptx::mma_ss(tmem + C_DP, ptx::sdesc_sw128(sbase + DO + ao, 16, 1024),
                    ptx::sdesc_sw128(sbase + VV + bo, 16, 1024), idesc_s, kk > 0);
        if (has_abs)
          ptx::mma_ss(tmem + C_SA, ptx::sdesc_sw128(sbase + QA + ao, 16, 1024),
                      ptx::sdesc_sw128(sbase + KR + bo, 16, 1024), idesc_s, kk > 0);
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
      if (has_abs) ptx::tmem_ld32(tmem + lane_base + C_SA + 32 * cc, ra);
      ptx::tmem_wait_ld();
      float dsr[32], dsa[32];
#pragma unroll
      for (int x = 0; x < 32; ++x) {
        const int c = 32 * cc + x;
        const uint32_t info = s_info[c];
        const bool is_abs = has_abs && (info & AI_KEY_ABS);
        const float s = is_abs ? __uint_as_float(ra[x]) : __uint_as_float(rs[x]);
        const bool valid = (info & AI_KEY_ATTN) && (k0 + c <= i) && (i < q1);
        const float p = valid ? exp2f(s * sl2 - lse2) : 0.f;
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
        if (has_abs) {
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
        const uint32_t acc = (n_tiles > 0 || kk > 0) ? 1u : 0u;
        ptx::mma_ss(tmem + C_DQR, ptx::sdesc_sw128(sbase + DS + ao, 16, 1024),
                    ptx::sdesc_sw128(sbase + KR + bo, 8192, 1024), idesc_dq, acc);
        if (has_abs)
          ptx::mma_ss(tmem + C_DQA, ptx::sdesc_sw128(sbase + DSA + ao, 16, 1024),
                      ptx::sdesc_sw128(sbase + KR + bo, 8192, 1024), idesc_dq, acc);
      }
      ptx::mma_commit(bar_mma);
    }
    wait_or_flag(bar_mma, ph_mma, s_abort, f.status);
    __syncthreads();
    if (*s_abort) { aborted = true; break; }
    ptx::tc_fence_after();
    ++n_tiles;
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
      if (n_tiles > 0) {
        ptx::tmem_ld32(tmem + lane_base + C_DQR + 32 * half, g1);
        ptx::tmem_ld32(tmem + lane_base + C_DQR + 64 + 32 * half, g2);
        if (has_abs) {
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
        if (n_tiles > 0) {
          const float c = cs[d], s = sn[d];
          const float v1 = __uint_as_float(g1[x]), v2 = __uint_as_float(g2[x]);
          y1 = v1 * c + v2 * s;
          y2 = v2 * c - v1 * s;
          if (has_abs) {
            y1 += __uint_as_float(a1[x]);
            y2 += __uint_as_float(a2[x]);
          }
        }
        o1[x] = y1;
        o2[x] = y2;
      }
      if (i < q1) {
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
                const __grid_constant__ CUtensorMap tm_do) {
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
  const int32_t* item = L.kv_items + 4 * (int64_t)blockIdx.x;
  const int b = item[0], j0 = item[1], j1 = item[2];
  const int hk = blockIdx.y, G = f.num_q_heads / f.num_kv_heads;
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

  for (int bi = L.row_blocks[b]; bi < L.row_blocks[b + 1] && !aborted; ++bi) {
    const Block blk = load_block(L.blocks, bi);
    if (blk.e <= j0 || blk.kv_lo >= j1) continue;
    const int qs = max(blk.s, j0);
    if (qs >= blk.e) continue;
    const bool has_abs = (blk.flags & AI_BLOCKF_ABS) != 0;
    const int kmax = min(j1, blk.e);

    // Raw K tile, rotated in place by this block's key positions.
    if (tid == 0) {
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive_expect_tx(bar_k, 32768);
      ptx::tma_load_4d(sbase + KR, &tm_k, bar_k, 0, j0, hk, b);
      ptx::tma_load_4d(sbase + KR + 16384, &tm_k, bar_k, 64, j0, hk, b);
    }
    wait_or_flag(bar_k, ph_k, s_abort, f.status);
    __syncthreads();
    if (*s_abort) { aborted = true; break; }
    uint32_t my_info = 0;
    int my_row = 0;
    if (j < kmax) {
      my_info = (uint32_t)L.key_info[blk.key_off + j];
      my_row = key_row(my_info, L.n_pos, f.status);
      const float* cs = L.rope_cos + (int64_t)my_row * (D / 2);
      const float* sn = L.rope_sin + (int64_t)my_row * (D / 2);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4* pa = reinterpret_cast<uint4*>(sm + KR + chunk_off<BN>(tid, c));
        uint4* pb = reinterpret_cast<uint4*>(sm + KR + chunk_off<BN>(tid, c + 8));
        uint4 y1, y2;
        rotate8(*pa, *pb, cs + 8 * c, sn + 8 * c, y1, y2);
        *pa = y1;
        *pb = y2;
      }
    }
    const bool key_ok = (my_info & AI_KEY_ATTN) != 0;
    const bool key_abs = has_abs && (my_info & AI_KEY_ABS);
    ptx::fence_proxy_async_smem();
    __syncthreads();

    bool dkr_started = false;
    for (int q0 = qs; q0 < blk.e && !aborted; q0 += BQ) {
      const int q1 = min(q0 + BQ, blk.e);
      for (int g = 0; g < G; ++g) {
        const int h = hk * G + g;
        const uint32_t qdst = has_abs ? QA : QR;
        if (tid == 0) {
          ptx::fence_proxy_async_smem();
          ptx::mbar_arrive_expect_tx(bar_q, 4 * 8192);
          ptx::tma_load_4d(sbase + qdst, &tm_q, bar_q, 0, q0, h, b);
          ptx::tma_load_4d(sbase + qdst + 8192, &tm_q, bar_q, 64, q0, h, b);
          ptx::tma_load_4d(sbase + DO, &tm_do, bar_q, 0, q0, h, b);
          ptx::tma_load_4d(sbase + DO + 8192, &tm_do, bar_q, 64, q0, h, b);
        }
        if (tid < BQ) {
          const int r = q0 + tid;
          float l2 = CUDART_INF_F, dlt = 0.f;
          int qp = 0;
          if (r < q1) {
            const int64_t idx = ((int64_t)b * f.num_q_heads + h) * f.seq_len + r;
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
        {
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
            const int c = 32 * cc + x, r = q0 + c;
            const bool valid = key_ok && (j <= r) && (r < q1) && (j < kmax);
            const float p = valid ? exp2f(s[c] * sl2 - s_lse[c]) : 0.f;
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

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

bool strides_ok(const AiTensor4& t) {
  return ((uintptr_t)t.ptr % 16 == 0) && (t.stride_b % 8 == 0) && (t.stride_h % 8 == 0) && (t.stride_t % 8 == 0);
}

}  // namespace sm100bwd

bool sm100_bwd_supported(int dtype, int head_dim) { return dtype == AI_DTYPE_BF16 && head_dim == sm100bwd::D; }

int sm100_kv_tile_rows() { return sm100bwd::kv::BN; }

int sm100_bwd(const AiAttnBwdArgs& a, float* delta, cudaStream_t st, cudaError_t* cuda_err) {
  using namespace sm100bwd;
  const AiAttnFwdArgs& f = a.fwd;
  if (!strides_ok(f.q) || !strides_ok(f.k) || !strides_ok(f.v) || !strides_ok(a.dout) || !strides_ok(a.dq) ||
      !strides_ok(a.dk) || !strides_ok(a.dv))
    return AI_ERR_STRIDE;
  cudaError_t e = bwd_delta(a, delta, st);
  if (e == cudaSuccess && f.layout.n_fwd_items > 0) {
    CUtensorMap tk, tv;
    if (!sm100_make_map(&tk, f.k, f.batch, f.num_kv_heads, f.seq_len, dq::BN) ||
        !sm100_make_map(&tv, f.v, f.batch, f.num_kv_heads, f.seq_len, dq::BN))
      return AI_ERR_TMA;
    e = cudaFuncSetAttribute(dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dq::kSmem);
    if (e == cudaSuccess) {
      dq_kernel<<<dim3(f.layout.n_fwd_items, f.num_q_heads), kThreads, dq::kSmem, st>>>(a, delta, tk, tv);
      e = cudaGetLastError();
    }
  }
  if (e == cudaSuccess && f.layout.n_kv_items > 0) {
    CUtensorMap tk, tv, tq, tdo;
    if (!sm100_make_map(&tk, f.k, f.batch, f.num_kv_heads, f.seq_len, kv::BN) ||
        !sm100_make_map(&tv, f.v, f.batch, f.num_kv_heads, f.seq_len, kv::BN) ||
        !sm100_make_map(&tq, f.q, f.batch, f.num_q_heads, f.seq_len, kv::BQ) ||
        !sm100_make_map(&tdo, a.dout, f.batch, f.num_q_heads, f.seq_len, kv::BQ))
      return AI_ERR_TMA;
    e = cudaFuncSetAttribute(dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kv::kSmem);
    if (e == cudaSuccess) {
      dkdv_kernel<<<dim3(f.layout.n_kv_items, f.num_kv_heads), kThreads, kv::kSmem, st>>>(a, delta, tk, tv, tq, tdo);
      e = cudaGetLastError();
    }
  }
  if (e == cudaSuccess) e = bwd_fill(a, st);
  if (cuda_err) *cuda_err = e;
  return e == cudaSuccess ? AI_OK : AI_ERR_LAUNCH;
}

}  // namespace ai
