// Forward of the chain-of-edits attention on sm_100a tensor cores
// (tcgen05.mma with TMEM accumulators, TMA tile loads), bf16 in / fp32
// accumulate, head_dim 128.
//
// One CTA computes one work item (block b, query rows [q0, q1) with
// q1 - q0 <= 128) for one query head:
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

struct Smem {
  static constexpr uint32_t Q = 0;
  static constexpr uint32_t QA = Q + kTile;
  static constexpr uint32_t K = QA + kTile;
  static constexpr uint32_t V = K + kTile;
  static constexpr uint32_t P = V + kTile;
  static constexpr uint32_t INFO = P + kTile;
  static constexpr uint32_t BAR_TMA = INFO + 4 * BN;
  static constexpr uint32_t BAR_MMA = BAR_TMA + 8;
  static constexpr uint32_t TMEM_SLOT = BAR_MMA + 8;
  static constexpr uint32_t ABORT = TMEM_SLOT + 4;
  static constexpr uint32_t TOTAL = ABORT + 4;
};
constexpr size_t kSmemBytes = Smem::TOTAL + 1024;

using tile::pack8;
using tile::rotate8;

__device__ __forceinline__ uint32_t chunk_off(int r, int c) { return tile::chunk_off<BM>(r, c); }

__global__ void __launch_bounds__(kThreads, 1)
    fwd_kernel(const AiAttnFwdArgs a, const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = ptx::smem_u32(sm);
  const int tid = threadIdx.x, warp = tid / 32;
  uint32_t* s_info = reinterpret_cast<uint32_t*>(sm + Smem::INFO);
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + Smem::ABORT);
  const uint32_t bar_tma = sbase + Smem::BAR_TMA, bar_mma = sbase + Smem::BAR_MMA;

  const AiAttnLayout& L = a.layout;
  const int32_t* item = L.fwd_items + 4 * (int64_t)blockIdx.x;
  const Block blk = load_block(L.blocks, item[0]);
  const int q0 = item[1], q1 = item[2];
  const int h = blockIdx.y, G = a.num_q_heads / a.num_kv_heads, hk = h / G, b = blk.row;
  const bool has_abs = (blk.flags & AI_BLOCKF_ABS) != 0;
  const int kv_hi = min(blk.e, q1);

  if (tid == 0) {
    ptx::mbar_init(bar_tma, 1);
    ptx::mbar_init(bar_mma, 1);
    *s_abort = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tm_k);
    ptx::prefetch_tmap(&tm_v);
  }
  if (warp == 0) {
    ptx::tmem_alloc(sbase + Smem::TMEM_SLOT, kTmemCols);
    ptx::tmem_relinquish();
  }

  // Query row `tid`: rotated into Q, raw into QA (abs blocks only).
  {
    const int i = q0 + tid;
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
  const int i = q0 + tid;
  float m_use = -CUDART_INF_F, l = 0.f;
  uint32_t ph_tma = 0, ph_mma = 0;
  int n_tiles = 0;
  bool aborted = false;

  for (int k0 = blk.kv_lo; k0 < kv_hi; k0 += BN) {
    // 1. K and V tiles by TMA.
    if (tid == 0) {
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive_expect_tx(bar_tma, 2 * kTile);
      ptx::tma_load_4d(sbase + Smem::K, &tm_k, bar_tma, 0, k0, hk, b);
      ptx::tma_load_4d(sbase + Smem::K + kHalf, &tm_k, bar_tma, 64, k0, hk, b);
      ptx::tma_load_4d(sbase + Smem::V, &tm_v, bar_tma, 0, k0, hk, b);
      ptx::tma_load_4d(sbase + Smem::V + kHalf, &tm_v, bar_tma, 64, k0, hk, b);
    }
    if (!ptx::mbar_wait(bar_tma, ph_tma, kWaitCycles)) {
      report(a.status, AI_ERR_DEV_TIMEOUT);
      *s_abort = 1;
    }
    ph_tma ^= 1;
    __syncthreads();
    if (*s_abort) {
      aborted = true;
      break;
    }

    // 2. Rotate key row `tid` in place by its position in this block.
    {
      const int j = k0 + tid;
      uint32_t info = 0;
      if (j < kv_hi) {
        info = (uint32_t)L.key_info[blk.key_off + j];
        const int p = key_row(info, L.n_pos, a.status);
        const float* cs = L.rope_cos + (int64_t)p * (D / 2);
        const float* sn = L.rope_sin + (int64_t)p * (D / 2);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4* pa = reinterpret_cast<uint4*>(sm + Smem::K + chunk_off(tid, c));
          uint4* pb = reinterpret_cast<uint4*>(sm + Smem::K + chunk_off(tid, c + 8));
          uint4 y1, y2;
          rotate8(*pa, *pb, cs + 8 * c, sn + 8 * c, y1, y2);
          *pa = y1;
          *pb = y2;
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
                    ptx::sdesc_sw128(sbase + Smem::K + off, 16, 1024), idesc_qk, kk > 0);
      }
      if (has_abs) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(kk >> 2) * kHalf + (uint32_t)(kk & 3) * 32u;
          ptx::mma_ss(tmem + kColSabs, ptx::sdesc_sw128(sbase + Smem::QA + off, 16, 1024),
                      ptx::sdesc_sw128(sbase + Smem::K + off, 16, 1024), idesc_qk, kk > 0);
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
      if (has_abs) {
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
      if (n_tiles > 0 && l > 0.f) {
        alpha = exp2f(m_use - m_new);
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
        pv[x] = (v == -CUDART_INF_F) ? 0.f : exp2f(v - m_use);
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
                    ptx::sdesc_sw128(sbase + Smem::V + boff, kHalf, 1024), idesc_pv, (n_tiles > 0 || kk > 0) ? 1u : 0u);
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

  // Epilogue: O / l -> bf16 row, lse.
  if (!aborted) {
    __nv_bfloat16* Orow =
        static_cast<__nv_bfloat16*>(a.out.ptr) + b * a.out.stride_b + h * a.out.stride_h + (int64_t)i * a.out.stride_t;
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int cc = 0; cc < D / 32; ++cc) {
      uint32_t r[32];
      if (n_tiles > 0) {
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

int sm100_fwd(const AiAttnFwdArgs& a, cudaStream_t st, cudaError_t* cuda_err) {
  using namespace sm100;
  if (!strides_ok(a.q) || !strides_ok(a.k) || !strides_ok(a.v) || !strides_ok(a.out)) return AI_ERR_STRIDE;
  if (a.layout.n_fwd_items == 0) return AI_OK;
  CUtensorMap tm_k, tm_v;
  if (!sm100_make_map(&tm_k, a.k, a.batch, a.num_kv_heads, a.seq_len, BN)) return AI_ERR_TMA;
  if (!sm100_make_map(&tm_v, a.v, a.batch, a.num_kv_heads, a.seq_len, BN)) return AI_ERR_TMA;
  cudaError_t e = cudaFuncSetAttribute(fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (e == cudaSuccess) {
    fwd_kernel<<<dim3(a.layout.n_fwd_items, a.num_q_heads), kThreads, kSmemBytes, st>>>(a, tm_k, tm_v);
    e = cudaGetLastError();
  }
  if (cuda_err) *cuda_err = e;
  return e == cudaSuccess ? AI_OK : AI_ERR_LAUNCH;
}

}  // namespace ai
