// Once-rotated copies of Q and K for the tensor-core kernels.
//
// q_rot[b, h, i] = R(q_pos[b, i]) q[b, h, i] for every query row, and
// k_rot[b, g, j] = R(k_own[b, j]) k[b, g, j] with k_own the key's position in
// the block whose query rows hold it.  Every query row has one position, so
// q_rot is exact for all blocks; a block flagged AI_BLOCKF_OWNPOS attends every
// key at its k_own position (packed documents do), so k_rot serves it and the
// kernels skip the per-tile rotation; other blocks rotate K in shared memory.
//
// k_cls[c, g, r] (rotation classes of the layout, 64 keys each): key
// k0 + r of batch row b rotated by the position its class's defining block
// gives it, so that blocks without own positions read their keys rotated
// from HBM instead of rotating every K tile they see in shared memory.
//
// HBM-bound: each thread rotates one 8-wide chunk pair of one row (chunk c
// and its rotate-half partner c + 8); eight consecutive threads cover a row,
// so loads and stores are 128-byte coalesced.  Output is contiguous
// (B, H, T, 128) bf16, then (n_classes, Hkv, 64, 128) bf16.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ai_common.cuh"
#include "ai_kernels.h"
#include "sm100_tile.cuh"

namespace ai {
namespace {

constexpr int D = 128;

__global__ void __launch_bounds__(256) prerot_kernel(const AiAttnFwdArgs a, __nv_bfloat16* __restrict__ q_rot,
                                                     __nv_bfloat16* __restrict__ k_rot,
                                                     __nv_bfloat16* __restrict__ k_cls) {
  const AiAttnLayout& L = a.layout;
  const int64_t T = a.seq_len;
  const int64_t nq = (int64_t)a.batch * a.num_q_heads * T * 8;
  const int64_t nk = (int64_t)a.batch * a.num_kv_heads * T * 8;
  const int64_t nc = (int64_t)L.n_rot_classes * a.num_kv_heads * AI_ROT_CLASS_KEYS * 8;
  const uint4* cs16 = static_cast<const uint4*>(L.rope_cs16);
  for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < nq + nk + nc;
       w += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(w & 7);
    const __nv_bfloat16* x;
    __nv_bfloat16* y;
    int p;
    if (w < nq + nk) {
      const bool is_q = w < nq;
      const int64_t row = (is_q ? w : w - nq) >> 3;  // (b, h, t) flattened, t fastest
      const int H = is_q ? a.num_q_heads : a.num_kv_heads;
      const int64_t t = row % T;
      const int h = (int)((row / T) % H);
      const int b = (int)(row / (T * H));
      const AiTensor4& src = is_q ? a.q : a.k;
      x = static_cast<const __nv_bfloat16*>(src.ptr) + b * src.stride_b + h * src.stride_h + t * src.stride_t;
      p = clamp_row((is_q ? L.q_pos : L.k_own)[(int64_t)b * T + t], L.n_pos, a.status);
      y = (is_q ? q_rot : k_rot) + row * D;
    } else {
      // Class chunks: (class, KV head, key of the chunk), key fastest; the
      // keys rotated by the rows the class's defining block gives them, zero
      // rows at or past that block's end.
      const int64_t row = (w - nq - nk) >> 3;
      const int r = (int)(row % AI_ROT_CLASS_KEYS);
      const int hk = (int)((row / AI_ROT_CLASS_KEYS) % a.num_kv_heads);
      const int64_t cls = row / ((int64_t)AI_ROT_CLASS_KEYS * a.num_kv_heads);
      y = k_cls + row * D;
      const int bi = L.rot_classes[2 * cls];
      const int key = L.rot_classes[2 * cls + 1] + r;
      bool ok = bi >= 0 && bi < L.n_blocks;
      if (!ok) report(a.status, AI_ERR_DEV_BOUNDS);
      const Block blk = load_block(L.blocks, ok ? bi : 0);
      if (!ok || key < 0 || key >= blk.e || key >= T) {
        *reinterpret_cast<uint4*>(y + 8 * c) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(y + 64 + 8 * c) = make_uint4(0, 0, 0, 0);
        continue;
      }
      p = key_row((uint32_t)__ldg(L.key_info + blk.key_off + key), L.n_pos, a.status);
      x = static_cast<const __nv_bfloat16*>(a.k.ptr) + blk.row * a.k.stride_b + hk * a.k.stride_h + key * a.k.stride_t;
    }
    const uint4 t0 = __ldg(cs16 + (int64_t)p * (D / 8) + 2 * c), t1 = __ldg(cs16 + (int64_t)p * (D / 8) + 2 * c + 1);
    const uint4 xa = __ldg(reinterpret_cast<const uint4*>(x + 8 * c));
    const uint4 xb = __ldg(reinterpret_cast<const uint4*>(x + 64 + 8 * c));
    uint4 ya, yb;
    tile::rotate8h(xa, xb, t0, t1, ya, yb);
    *reinterpret_cast<uint4*>(y + 8 * c) = ya;
    *reinterpret_cast<uint4*>(y + 64 + 8 * c) = yb;
  }
}

}  // namespace

size_t prerot_bytes(const AiAttnFwdArgs& a, size_t* q_bytes, size_t* qk_bytes) {
  const size_t q = ((size_t)a.batch * a.num_q_heads * a.seq_len * D * 2 + 255) & ~size_t(255);
  const size_t k = ((size_t)a.batch * a.num_kv_heads * a.seq_len * D * 2 + 255) & ~size_t(255);
  const size_t n_cls = a.layout.n_rot_classes > 0 ? (size_t)a.layout.n_rot_classes : 0;
  const size_t c = (n_cls * a.num_kv_heads * AI_ROT_CLASS_KEYS * D * 2 + 255) & ~size_t(255);
  if (q_bytes) *q_bytes = q;
  if (qk_bytes) *qk_bytes = q + k;
  return q + k + c;
}

cudaError_t prerot(const AiAttnFwdArgs& a, void* buf, cudaStream_t st) {
  size_t qb = 0, qkb = 0;
  prerot_bytes(a, &qb, &qkb);
  __nv_bfloat16* q_rot = static_cast<__nv_bfloat16*>(buf);
  __nv_bfloat16* k_rot = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(buf) + qb);
  __nv_bfloat16* k_cls = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(buf) + qkb);
  const int64_t n_cls = a.layout.n_rot_classes > 0 ? a.layout.n_rot_classes : 0;
  const int64_t work = ((int64_t)a.batch * (a.num_q_heads + a.num_kv_heads) * a.seq_len +
                        n_cls * a.num_kv_heads * AI_ROT_CLASS_KEYS) * 8;
  int blocks = (int)((work + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  ProfScope ps(AI_PROF_PREROT, st);
  prerot_kernel<<<blocks, 256, 0, st>>>(a, q_rot, k_rot, k_cls);
  return cudaGetLastError();
}

}  // namespace ai
