// SIMT (FP32 FMA) kernels of the chain-of-edits attention: forward, backward
// dQ, backward dK/dV, the dO.O row-sum and the fills for rows no block owns.
//
// These carry the fp32 path (the reference's own tests run the attention in
// fp32 and compare at 1e-3; tensor cores cannot meet that in bf16/tf32) and
// every (dtype, head_dim) the tcgen05 kernels do not cover.  All arithmetic is
// fp32; inputs may be fp32, bf16 or fp16.
//
// Math restated from attention/reference.py:11-64 and :96-141 of the reference
// (per-block rotated keys, abs columns use the unrotated query, global causal
// mask, scale, softmax, P.V); the backward is the hand-derived gradient of that
// function (the reference differentiates it with autograd).
//
// Tiling: BM = 32 query rows x BN = 64 keys, 256 threads.  A thread owns the
// (row, key) pairs r = ty + 16 i, c = tx + 16 j of a score tile and the
// (row, dim) pairs r = ty + 16 i, d = tx + 16 j of an output tile, so the two
// halves d and d + D/2 of every rotate-half pair sit in the same thread.

#include <cuda_runtime.h>
#include <math_constants.h>

#include "ai_common.cuh"
#include "ai_kernels.h"

namespace ai {
namespace simt {

constexpr int kThreads = 256;
constexpr int BM = 32;
constexpr int BN = 64;

template <int D>
struct Cfg {
  static constexpr int H2 = D / 2;
  static constexpr int LD = D + 1;   // padded row pitch of [rows][D] tiles
  static constexpr int LS = BN + 1;  // padded row pitch of [BM][BN] tiles
  static constexpr int DJ = D / 16;  // output dims per thread
};

template <int D>
size_t fwd_smem_bytes() {
  using C = Cfg<D>;
  return sizeof(float) * (2 * BM * C::LD + BN * C::LD + BN * D + BM * C::LS + 3 * BM) + sizeof(uint32_t) * BN;
}

template <int D>
size_t dq_smem_bytes() {
  using C = Cfg<D>;
  return sizeof(float) * (3 * BM * C::LD + 2 * BN * C::LD + BM * C::LS + 2 * BM) + sizeof(uint32_t) * BN;
}

template <int D>
size_t dkdv_smem_bytes() {
  using C = Cfg<D>;
  return sizeof(float) * (3 * BM * C::LD + 3 * BN * C::LD + 2 * BM * C::LS + 2 * BM) + sizeof(uint32_t) * BN;
}

// Loads query rows [q0, q1) of one head into sQr (rotated by the row's query
// position) and, if sQ != nullptr, sQ (unrotated).  Rows past q1 are zero.
template <typename T, int D>
__device__ void load_query_rows(float* sQr, float* sQ, const T* Q, int64_t st, int q0, int q1,
                                const int32_t* qpos_row, const AiAttnLayout& L, int32_t* status) {
  using C = Cfg<D>;
  for (int idx = threadIdx.x; idx < BM * C::H2; idx += kThreads) {
    const int r = idx / C::H2, d = idx % C::H2, i = q0 + r;
    float x1 = 0.f, x2 = 0.f, y1 = 0.f, y2 = 0.f;
    if (i < q1) {
      x1 = to_f32(Q[i * st + d]);
      x2 = to_f32(Q[i * st + d + C::H2]);
      const int p = clamp_row(qpos_row[i], L.n_pos, status);
      const float c = L.rope_cos[(int64_t)p * C::H2 + d], s = L.rope_sin[(int64_t)p * C::H2 + d];
      y1 = x1 * c - x2 * s;
      y2 = x2 * c + x1 * s;
    }
    sQr[r * C::LD + d] = y1;
    sQr[r * C::LD + d + C::H2] = y2;
    if (sQ) {
      sQ[r * C::LD + d] = x1;
      sQ[r * C::LD + d + C::H2] = x2;
    }
  }
}

// Plain copy of rows [r0, r0 + n) (n <= rows) into a [rows][ld] fp32 tile.
template <typename T, int D>
__device__ void load_rows(float* dst, int ld, const T* X, int64_t st, int r0, int n, int rows) {
  for (int idx = threadIdx.x; idx < rows * D; idx += kThreads) {
    const int r = idx / D, d = idx % D;
    dst[r * ld + d] = r < n ? to_f32(X[(int64_t)(r0 + r) * st + d]) : 0.f;
  }
}

// Rotates keys [k0, k0 + nk) of block `blk` (positions from key_info) from a
// raw source into sK; writes each key's info word into sInfo (0 = masked for
// the slots past nk).  `raw` is either global memory (T*) or a smem tile.
template <int D, typename Src>
__device__ void rotate_keys(float* sK, uint32_t* sInfo, Src raw, int k0, int nk, const Block& blk,
                            const AiAttnLayout& L, int32_t* status) {
  using C = Cfg<D>;
  if (threadIdx.x < BN) {
    uint32_t info = 0;
    if ((int)threadIdx.x < nk) info = (uint32_t)L.key_info[blk.key_off + k0 + threadIdx.x];
    sInfo[threadIdx.x] = info;
  }
  for (int idx = threadIdx.x; idx < BN * C::H2; idx += kThreads) {
    const int c = idx / C::H2, d = idx % C::H2;
    float y1 = 0.f, y2 = 0.f;
    if (c < nk) {
      const uint32_t info = (uint32_t)L.key_info[blk.key_off + k0 + c];
      const int p = key_row(info, L.n_pos, status);
      const float x1 = raw(c, d), x2 = raw(c, d + C::H2);
      const float cs = L.rope_cos[(int64_t)p * C::H2 + d], sn = L.rope_sin[(int64_t)p * C::H2 + d];
      y1 = x1 * cs - x2 * sn;
      y2 = x2 * cs + x1 * sn;
    }
    sK[c * C::LD + d] = y1;
    sK[c * C::LD + d + C::H2] = y2;
  }
}

template <typename T>
struct GlobalRows {
  const T* base;
  int64_t st;
  int k0;
  __device__ float operator()(int c, int d) const { return to_f32(base[(int64_t)(k0 + c) * st + d]); }
};

template <int D>
struct SmemRows {
  const float* base;
  __device__ float operator()(int c, int d) const { return base[c * Cfg<D>::LD + d]; }
};

// Scores of the thread's 2x4 (row, key) pairs: rotated-query dot rotated-key,
// or unrotated-query dot rotated-key on abs columns; masked pairs get -inf.
// Result is in log2 units (multiplied by scale * log2(e)).
template <int D>
__device__ void tile_scores(float (&s)[2][4], const float* sQr, const float* sQ, const float* sK,
                            const uint32_t* sInfo, bool has_abs, int q0, int q1, int k0, float sl2) {
  using C = Cfg<D>;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float sr[2][4] = {}, sa[2][4] = {};
#pragma unroll 4
  for (int d = 0; d < D; ++d) {
    float kk[4], qr[2];
#pragma unroll
    for (int j = 0; j < 4; ++j) kk[j] = sK[(tx + 16 * j) * C::LD + d];
#pragma unroll
    for (int i = 0; i < 2; ++i) qr[i] = sQr[(ty + 16 * i) * C::LD + d];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sr[i][j] += qr[i] * kk[j];
    if (has_abs) {
      float qa[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) qa[i] = sQ[(ty + 16 * i) * C::LD + d];
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) sa[i][j] += qa[i] * kk[j];
    }
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = ty + 16 * i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = tx + 16 * j;
      const uint32_t info = sInfo[c];
      const bool valid = (info & AI_KEY_ATTN) && (k0 + c <= q0 + r) && (q0 + r < q1);
      const float v = (has_abs && (info & AI_KEY_ABS)) ? sa[i][j] : sr[i][j];
      s[i][j] = valid ? v * sl2 : -CUDART_INF_F;
    }
  }
}

// dP = dO . V for the thread's 2x4 (row, key) pairs.
template <int D>
__device__ void tile_dp(float (&dp)[2][4], const float* sdO, const float* sV) {
  using C = Cfg<D>;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) dp[i][j] = 0.f;
#pragma unroll 4
  for (int d = 0; d < D; ++d) {
    float vv[4], g[2];
#pragma unroll
    for (int j = 0; j < 4; ++j) vv[j] = sV[(tx + 16 * j) * C::LD + d];
#pragma unroll
    for (int i = 0; i < 2; ++i) g[i] = sdO[(ty + 16 * i) * C::LD + d];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) dp[i][j] += g[i] * vv[j];
  }
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) fwd_kernel(const AiAttnFwdArgs a) {
  using C = Cfg<D>;
  extern __shared__ float sm[];
  float* sQr = sm;
  float* sQ = sQr + BM * C::LD;
  float* sK = sQ + BM * C::LD;
  float* sV = sK + BN * C::LD;
  float* sS = sV + BN * D;
  float* sM = sS + BM * C::LS;
  float* sL = sM + BM;
  float* sAlpha = sL + BM;
  uint32_t* sInfo = reinterpret_cast<uint32_t*>(sAlpha + BM);

  const AiAttnLayout& L = a.layout;
  const int32_t* item = L.fwd_items + 4 * (int64_t)blockIdx.x;
  const Block blk = load_block(L.blocks, item[0]);
  const int h = blockIdx.y, G = a.num_q_heads / a.num_kv_heads, hk = h / G, b = blk.row;
  const bool has_abs = blk.flags & AI_BLOCKF_ABS;
  const int T_ = a.seq_len;
  const T* Q = static_cast<const T*>(a.q.ptr) + b * a.q.stride_b + h * a.q.stride_h;
  const T* K = static_cast<const T*>(a.k.ptr) + b * a.k.stride_b + hk * a.k.stride_h;
  const T* V = static_cast<const T*>(a.v.ptr) + b * a.v.stride_b + hk * a.v.stride_h;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;

  // A work item may span several BM-row sub-tiles (its tile size is chosen for
  // the fastest kernel of the dtype); each sub-tile is an independent pass.
  for (int q0 = item[1]; q0 < item[2]; q0 += BM) {
  const int q1 = min(q0 + BM, item[2]);
  __syncthreads();
  load_query_rows<T, D>(sQr, has_abs ? sQ : nullptr, Q, a.q.stride_t, q0, q1, L.q_pos + (int64_t)b * T_, L, a.status);
  if (threadIdx.x < BM) {
    sM[threadIdx.x] = -CUDART_INF_F;
    sL[threadIdx.x] = 0.f;
  }
  float acc[2][C::DJ];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < C::DJ; ++j) acc[i][j] = 0.f;

  const float sl2 = a.scale * kLog2e;
  const int kv_hi = min(blk.e, q1);
  for (int k0 = blk.kv_lo; k0 < kv_hi; k0 += BN) {
    const int nk = min(BN, kv_hi - k0);
    __syncthreads();
    rotate_keys<D>(sK, sInfo, GlobalRows<T>{K, a.k.stride_t, k0}, k0, nk, blk, L, a.status);
    load_rows<T, D>(sV, D, V, a.v.stride_t, k0, nk, BN);
    __syncthreads();
    float s[2][4];
    tile_scores<D>(s, sQr, sQ, sK, sInfo, has_abs, q0, q1, k0, sl2);
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sS[(ty + 16 * i) * C::LS + tx + 16 * j] = s[i][j];
    __syncthreads();
    if (threadIdx.x < BM) {
      const int r = threadIdx.x;
      const float m_old = sM[r];
      float mx = -CUDART_INF_F;
      for (int c = 0; c < BN; ++c) mx = fmaxf(mx, sS[r * C::LS + c]);
      const float m_new = fmaxf(m_old, mx);
      const float alpha = (m_new == -CUDART_INF_F) ? 1.f : exp2f(m_old - m_new);
      float sum = 0.f;
      for (int c = 0; c < BN; ++c) {
        const float v = sS[r * C::LS + c];
        const float p = (v == -CUDART_INF_F) ? 0.f : exp2f(v - m_new);
        sS[r * C::LS + c] = p;
        sum += p;
      }
      sL[r] = sL[r] * alpha + sum;
      sM[r] = m_new;
      sAlpha[r] = alpha;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int r = ty + 16 * i;
      const float alpha = sAlpha[r];
#pragma unroll
      for (int j = 0; j < C::DJ; ++j) acc[i][j] *= alpha;
      for (int c = 0; c < BN; ++c) {
        const float p = sS[r * C::LS + c];
#pragma unroll
        for (int j = 0; j < C::DJ; ++j) acc[i][j] += p * sV[c * D + tx + 16 * j];
      }
    }
  }
  __syncthreads();
  T* O = static_cast<T*>(a.out.ptr) + b * a.out.stride_b + h * a.out.stride_h;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = ty + 16 * i, row = q0 + r;
    if (row >= q1) continue;
    const float l = sL[r];
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int j = 0; j < C::DJ; ++j) O[(int64_t)row * a.out.stride_t + tx + 16 * j] = from_f32<T>(acc[i][j] * inv);
    if (tx == 0)
      a.lse[((int64_t)b * a.num_q_heads + h) * T_ + row] = l > 0.f ? (sM[r] + log2f(l)) * kLn2 : -CUDART_INF_F;
  }
  }
}

// Rows no block owns: the reference leaves a lone zero logit on the diagonal
// (reference.py:42-43), so out = v of the row and lse = 0.
template <typename T, int D>
__global__ void fwd_fill_kernel(const AiAttnFwdArgs a) {
  const int i = blockIdx.x, b = blockIdx.y;
  if (i < a.layout.row_cov[b]) return;
  const int G = a.num_q_heads / a.num_kv_heads;
  for (int idx = threadIdx.x; idx < a.num_q_heads * D; idx += blockDim.x) {
    const int h = idx / D, d = idx % D;
    const T* V = static_cast<const T*>(a.v.ptr) + b * a.v.stride_b + (h / G) * a.v.stride_h + (int64_t)i * a.v.stride_t;
    T* O = static_cast<T*>(a.out.ptr) + b * a.out.stride_b + h * a.out.stride_h + (int64_t)i * a.out.stride_t;
    O[d] = V[d];
  }
  for (int h = threadIdx.x; h < a.num_q_heads; h += blockDim.x)
    a.lse[((int64_t)b * a.num_q_heads + h) * a.seq_len + i] = 0.f;
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------

// delta[b, h, i] = sum_d dO[b, i, h, d] * O[b, i, h, d]; one warp per row.
template <typename T, int D>
__global__ void delta_kernel(const AiAttnBwdArgs a, float* delta) {
  const AiAttnFwdArgs& f = a.fwd;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  const int64_t total = (int64_t)f.batch * f.num_q_heads * f.seq_len;
  if (w >= total) return;
  const int i = (int)(w % f.seq_len);
  const int h = (int)((w / f.seq_len) % f.num_q_heads);
  const int b = (int)(w / ((int64_t)f.seq_len * f.num_q_heads));
  const T* O = static_cast<const T*>(f.out.ptr) + b * f.out.stride_b + h * f.out.stride_h + (int64_t)i * f.out.stride_t;
  const T* dO = static_cast<const T*>(a.dout.ptr) + b * a.dout.stride_b + h * a.dout.stride_h + (int64_t)i * a.dout.stride_t;
  float s = 0.f;
  for (int d = lane; d < D; d += 32) s += to_f32(O[d]) * to_f32(dO[d]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) delta[w] = s;
}

// Dot product of two 16-byte chunks (8 bf16 / 8 fp16 / 4 fp32 values).
template <typename T>
__device__ __forceinline__ float dot16(const uint4& x, const uint4& y);
template <>
__device__ __forceinline__ float dot16<__nv_bfloat16>(const uint4& x, const uint4& y) {
  const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(&x);
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&y);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 u = __bfloat1622float2(a[i]), v = __bfloat1622float2(b[i]);
    s = fmaf(u.x, v.x, fmaf(u.y, v.y, s));
  }
  return s;
}
template <>
__device__ __forceinline__ float dot16<__half>(const uint4& x, const uint4& y) {
  const __half2* a = reinterpret_cast<const __half2*>(&x);
  const __half2* b = reinterpret_cast<const __half2*>(&y);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 u = __half22float2(a[i]), v = __half22float2(b[i]);
    s = fmaf(u.x, v.x, fmaf(u.y, v.y, s));
  }
  return s;
}
template <>
__device__ __forceinline__ float dot16<float>(const uint4& x, const uint4& y) {
  return fmaf(__uint_as_float(x.x), __uint_as_float(y.x),
              fmaf(__uint_as_float(x.y), __uint_as_float(y.y),
                   fmaf(__uint_as_float(x.z), __uint_as_float(y.z), __uint_as_float(x.w) * __uint_as_float(y.w))));
}

// delta as above with 16-byte loads: kTpr = D * sizeof(T) / 16 consecutive
// lanes share a row (one chunk each) and reduce by shuffles.  Requires
// 16-byte aligned rows (checked on the host).
// Grid (query-row blocks, batch x head): kTpr lanes per row, no 64-bit
// index arithmetic.
template <typename T, int D>
__global__ void __launch_bounds__(256) delta_vec_kernel(const AiAttnBwdArgs a, float* delta) {
  // kR rows per lane group (kRpb rows apart), their loads issued before any
  // use: more bytes in flight per thread for this HBM-bound pass.
  constexpr int kTpr = D * (int)sizeof(T) / 16, kPer = 16 / (int)sizeof(T), kRpb = 256 / kTpr, kR = 2;
  static_assert(kTpr >= 1 && kTpr <= 32 && (32 % kTpr) == 0, "row chunking");
  const AiAttnFwdArgs& f = a.fwd;
  const int i0 = blockIdx.x * (kRpb * kR) + (int)threadIdx.x / kTpr, c = (int)threadIdx.x % kTpr;
  const int bh = blockIdx.y, b = bh / f.num_q_heads, h = bh - b * f.num_q_heads;
  const T* O0 = static_cast<const T*>(f.out.ptr) + b * f.out.stride_b + h * f.out.stride_h + kPer * c;
  const T* dO0 = static_cast<const T*>(a.dout.ptr) + b * a.dout.stride_b + h * a.dout.stride_h + kPer * c;
  uint4 xo[kR], xd[kR];
#pragma unroll
  for (int r = 0; r < kR; ++r) {
    const int i = i0 + r * kRpb;
    xo[r] = xd[r] = make_uint4(0, 0, 0, 0);
    if (i < f.seq_len) {
      xo[r] = __ldg(reinterpret_cast<const uint4*>(O0 + (int64_t)i * f.out.stride_t));
      xd[r] = __ldg(reinterpret_cast<const uint4*>(dO0 + (int64_t)i * a.dout.stride_t));
    }
  }
#pragma unroll
  for (int r = 0; r < kR; ++r) {
    const int i = i0 + r * kRpb;
    float s = dot16<T>(xo[r], xd[r]);
#pragma unroll
    for (int o = kTpr / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (i < f.seq_len && c == 0) delta[(int64_t)bh * f.seq_len + i] = s;
  }
}

template <typename T>
static bool rows16(const AiTensor4& t) {
  constexpr int64_t e = 16 / (int64_t)sizeof(T);
  return ((uintptr_t)t.ptr % 16 == 0) && t.stride_b % e == 0 && t.stride_h % e == 0 && t.stride_t % e == 0;
}

// P and dS (gradient of the unscaled logits) of the thread's 2x4 pairs.
template <int D>
__device__ void tile_p_ds(float (&p)[2][4], float (&ds)[2][4], const float* sQr, const float* sQ,
                          const float* sdO, const float* sK, const float* sV, const uint32_t* sInfo,
                          const float* sLse2, const float* sDelta, bool has_abs, int q0, int q1, int k0,
                          float scale) {
  const int ty = threadIdx.x / 16;
  float s[2][4], dp[2][4];
  tile_scores<D>(s, sQr, sQ, sK, sInfo, has_abs, q0, q1, k0, scale * kLog2e);
  tile_dp<D>(dp, sdO, sV);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = ty + 16 * i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      p[i][j] = (s[i][j] == -CUDART_INF_F) ? 0.f : exp2f(s[i][j] - sLse2[r]);
      ds[i][j] = p[i][j] * (dp[i][j] - sDelta[r]) * scale;
    }
  }
}

template <typename T, int D>
__device__ void load_row_stats(float* sLse2, float* sDelta, const AiAttnBwdArgs& a, const float* delta, int b,
                               int h, int q0, int q1) {
  if (threadIdx.x < BM) {
    const int i = q0 + threadIdx.x;
    float l2 = 0.f, dl = 0.f;
    if (i < q1) {
      const int64_t idx = ((int64_t)b * a.fwd.num_q_heads + h) * a.fwd.seq_len + i;
      const float lse = a.fwd.lse[idx];
      // A row with no visible key has lse = -inf; its P is 0 everywhere.
      l2 = lse == -CUDART_INF_F ? CUDART_INF_F : lse * kLog2e;
      dl = delta[idx];
    }
    sLse2[threadIdx.x] = l2;
    sDelta[threadIdx.x] = dl;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) dq_kernel(const AiAttnBwdArgs a, const float* delta) {
  using C = Cfg<D>;
  extern __shared__ float sm[];
  float* sQr = sm;
  float* sQ = sQr + BM * C::LD;
  float* sdO = sQ + BM * C::LD;
  float* sK = sdO + BM * C::LD;
  float* sV = sK + BN * C::LD;
  float* sdS = sV + BN * C::LD;
  float* sLse2 = sdS + BM * C::LS;
  float* sDelta = sLse2 + BM;
  uint32_t* sInfo = reinterpret_cast<uint32_t*>(sDelta + BM);

  const AiAttnFwdArgs& f = a.fwd;
  const AiAttnLayout& L = f.layout;
  const int32_t* item = L.fwd_items + 4 * (int64_t)blockIdx.x;
  const Block blk = load_block(L.blocks, item[0]);
  const int h = blockIdx.y, G = f.num_q_heads / f.num_kv_heads, hk = h / G, b = blk.row;
  const bool has_abs = blk.flags & AI_BLOCKF_ABS;
  const T* Q = static_cast<const T*>(f.q.ptr) + b * f.q.stride_b + h * f.q.stride_h;
  const T* K = static_cast<const T*>(f.k.ptr) + b * f.k.stride_b + hk * f.k.stride_h;
  const T* V = static_cast<const T*>(f.v.ptr) + b * f.v.stride_b + hk * f.v.stride_h;
  const T* dO = static_cast<const T*>(a.dout.ptr) + b * a.dout.stride_b + h * a.dout.stride_h;
  const int32_t* qpos_row = L.q_pos + (int64_t)b * f.seq_len;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;

  for (int q0 = item[1]; q0 < item[2]; q0 += BM) {
  const int q1 = min(q0 + BM, item[2]);
  __syncthreads();
  load_query_rows<T, D>(sQr, has_abs ? sQ : nullptr, Q, f.q.stride_t, q0, q1, qpos_row, L, f.status);
  load_rows<T, D>(sdO, C::LD, dO, a.dout.stride_t, q0, q1 - q0, BM);
  load_row_stats<T, D>(sLse2, sDelta, a, delta, b, h, q0, q1);

  float dqr[2][C::DJ], dqa[2][C::DJ];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < C::DJ; ++j) dqr[i][j] = dqa[i][j] = 0.f;

  const int kv_hi = min(blk.e, q1);
  for (int k0 = blk.kv_lo; k0 < kv_hi; k0 += BN) {
    const int nk = min(BN, kv_hi - k0);
    __syncthreads();
    rotate_keys<D>(sK, sInfo, GlobalRows<T>{K, f.k.stride_t, k0}, k0, nk, blk, L, f.status);
    load_rows<T, D>(sV, C::LD, V, f.v.stride_t, k0, nk, BN);
    __syncthreads();
    float p[2][4], ds[2][4];
    tile_p_ds<D>(p, ds, sQr, sQ, sdO, sK, sV, sInfo, sLse2, sDelta, has_abs, q0, q1, k0, f.scale);
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sdS[(ty + 16 * i) * C::LS + tx + 16 * j] = ds[i][j];
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int r = ty + 16 * i;
      for (int c = 0; c < BN; ++c) {
        const float g = sdS[r * C::LS + c];
        if (has_abs && (sInfo[c] & AI_KEY_ABS)) {
#pragma unroll
          for (int j = 0; j < C::DJ; ++j) dqa[i][j] += g * sK[c * C::LD + tx + 16 * j];
        } else {
#pragma unroll
          for (int j = 0; j < C::DJ; ++j) dqr[i][j] += g * sK[c * C::LD + tx + 16 * j];
        }
      }
    }
  }
  // dQ = R(qpos)^T dQ_rot + dQ_abs.
  T* dQ = static_cast<T*>(a.dq.ptr) + b * a.dq.stride_b + h * a.dq.stride_h;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = ty + 16 * i, row = q0 + r;
    if (row >= q1) continue;
    const int pr = clamp_row(qpos_row[row], L.n_pos, f.status);
#pragma unroll
    for (int j = 0; j < C::DJ / 2; ++j) {
      const int d = tx + 16 * j;
      const float cs = L.rope_cos[(int64_t)pr * C::H2 + d], sn = L.rope_sin[(int64_t)pr * C::H2 + d];
      const float g1 = dqr[i][j], g2 = dqr[i][j + C::DJ / 2];
      dQ[(int64_t)row * a.dq.stride_t + d] = from_f32<T>(g1 * cs + g2 * sn + dqa[i][j]);
      dQ[(int64_t)row * a.dq.stride_t + d + C::H2] = from_f32<T>(g2 * cs - g1 * sn + dqa[i][j + C::DJ / 2]);
    }
  }
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) dkdv_kernel(const AiAttnBwdArgs a, const float* delta) {
  using C = Cfg<D>;
  extern __shared__ float sm[];
  float* sQr = sm;
  float* sQ = sQr + BM * C::LD;
  float* sdO = sQ + BM * C::LD;
  float* sK = sdO + BM * C::LD;
  float* sKraw = sK + BN * C::LD;
  float* sV = sKraw + BN * C::LD;
  float* sP = sV + BN * C::LD;
  float* sdS = sP + BM * C::LS;
  float* sLse2 = sdS + BM * C::LS;
  float* sDelta = sLse2 + BM;
  uint32_t* sInfo = reinterpret_cast<uint32_t*>(sDelta + BM);

  const AiAttnFwdArgs& f = a.fwd;
  const AiAttnLayout& L = f.layout;
  const int32_t* item = L.kv_items + 4 * (int64_t)blockIdx.x;
  const int b = item[0], j0 = item[1], j1 = item[2];
  const int hk = blockIdx.y, G = f.num_q_heads / f.num_kv_heads;
  const T* K = static_cast<const T*>(f.k.ptr) + b * f.k.stride_b + hk * f.k.stride_h;
  const T* V = static_cast<const T*>(f.v.ptr) + b * f.v.stride_b + hk * f.v.stride_h;
  const int32_t* qpos_row = L.q_pos + (int64_t)b * f.seq_len;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  constexpr int CI = BN / 16;  // keys per thread in the accumulators

  load_rows<T, D>(sKraw, C::LD, K, f.k.stride_t, j0, j1 - j0, BN);
  load_rows<T, D>(sV, C::LD, V, f.v.stride_t, j0, j1 - j0, BN);

  float dv[CI][C::DJ], dk[CI][C::DJ], dkr[CI][C::DJ];
#pragma unroll
  for (int i = 0; i < CI; ++i)
#pragma unroll
    for (int j = 0; j < C::DJ; ++j) dv[i][j] = dk[i][j] = 0.f;

  for (int bi = L.row_blocks[b]; bi < L.row_blocks[b + 1]; ++bi) {
    const Block blk = load_block(L.blocks, bi);
    if (blk.e <= j0 || blk.kv_lo >= j1) continue;
    const int qs = max(blk.s, j0);
    if (qs >= blk.e) continue;
    const bool has_abs = blk.flags & AI_BLOCKF_ABS;
    const int nk = min(j1, blk.e) - j0;
    __syncthreads();
    rotate_keys<D>(sK, sInfo, SmemRows<D>{sKraw}, j0, nk, blk, L, f.status);
#pragma unroll
    for (int i = 0; i < CI; ++i)
#pragma unroll
      for (int j = 0; j < C::DJ; ++j) dkr[i][j] = 0.f;
    for (int q0 = qs; q0 < blk.e; q0 += BM) {
      const int q1 = min(q0 + BM, blk.e);
      for (int g = 0; g < G; ++g) {
        const int h = hk * G + g;
        const T* Q = static_cast<const T*>(f.q.ptr) + b * f.q.stride_b + h * f.q.stride_h;
        const T* dO = static_cast<const T*>(a.dout.ptr) + b * a.dout.stride_b + h * a.dout.stride_h;
        __syncthreads();
        load_query_rows<T, D>(sQr, has_abs ? sQ : nullptr, Q, f.q.stride_t, q0, q1, qpos_row, L, f.status);
        load_rows<T, D>(sdO, C::LD, dO, a.dout.stride_t, q0, q1 - q0, BM);
        load_row_stats<T, D>(sLse2, sDelta, a, delta, b, h, q0, q1);
        __syncthreads();
        float p[2][4], ds[2][4];
        tile_p_ds<D>(p, ds, sQr, sQ, sdO, sK, sV, sInfo, sLse2, sDelta, has_abs, q0, q1, j0, f.scale);
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            sP[(ty + 16 * i) * C::LS + tx + 16 * j] = p[i][j];
            sdS[(ty + 16 * i) * C::LS + tx + 16 * j] = ds[i][j];
          }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < CI; ++i) {
          const int c = ty + 16 * i;
          const bool col_abs = has_abs && (sInfo[c] & AI_KEY_ABS);
          const float* qsrc = col_abs ? sQ : sQr;
          for (int r = 0; r < BM; ++r) {
            const float pv = sP[r * C::LS + c], g = sdS[r * C::LS + c];
#pragma unroll
            for (int j = 0; j < C::DJ; ++j) {
              dv[i][j] += pv * sdO[r * C::LD + tx + 16 * j];
              dkr[i][j] += g * qsrc[r * C::LD + tx + 16 * j];
            }
          }
        }
      }
    }
    // dK += R(key position in this block)^T dK_rot.
#pragma unroll
    for (int i = 0; i < CI; ++i) {
      const int c = ty + 16 * i;
      if (c >= nk) continue;
      const int pr = key_row(sInfo[c], L.n_pos, f.status);
#pragma unroll
      for (int j = 0; j < C::DJ / 2; ++j) {
        const int d = tx + 16 * j;
        const float cs = L.rope_cos[(int64_t)pr * C::H2 + d], sn = L.rope_sin[(int64_t)pr * C::H2 + d];
        const float g1 = dkr[i][j], g2 = dkr[i][j + C::DJ / 2];
        dk[i][j] += g1 * cs + g2 * sn;
        dk[i][j + C::DJ / 2] += g2 * cs - g1 * sn;
      }
    }
  }
  T* dK = static_cast<T*>(a.dk.ptr) + b * a.dk.stride_b + hk * a.dk.stride_h;
  T* dV = static_cast<T*>(a.dv.ptr) + b * a.dv.stride_b + hk * a.dv.stride_h;
#pragma unroll
  for (int i = 0; i < CI; ++i) {
    const int c = ty + 16 * i, j = j0 + c;
    if (j >= j1) continue;
#pragma unroll
    for (int jj = 0; jj < C::DJ; ++jj) {
      dK[(int64_t)j * a.dk.stride_t + tx + 16 * jj] = from_f32<T>(dk[i][jj]);
      dV[(int64_t)j * a.dv.stride_t + tx + 16 * jj] = from_f32<T>(dv[i][jj]);
    }
  }
}

// Rows (and keys) no block owns: dV = sum over the group's heads of dO, dK = 0,
// dQ = 0 (the lone diagonal logit is a constant).
template <typename T, int D>
__global__ void bwd_fill_kernel(const AiAttnBwdArgs a) {
  const AiAttnFwdArgs& f = a.fwd;
  const int i = blockIdx.x, b = blockIdx.y;
  if (i < f.layout.row_cov[b]) return;
  const int G = f.num_q_heads / f.num_kv_heads;
  for (int idx = threadIdx.x; idx < f.num_kv_heads * D; idx += blockDim.x) {
    const int hk = idx / D, d = idx % D;
    float s = 0.f;
    for (int g = 0; g < G; ++g) {
      const int h = hk * G + g;
      s += to_f32(static_cast<const T*>(a.dout.ptr)[b * a.dout.stride_b + h * a.dout.stride_h + (int64_t)i * a.dout.stride_t + d]);
      static_cast<T*>(a.dq.ptr)[b * a.dq.stride_b + h * a.dq.stride_h + (int64_t)i * a.dq.stride_t + d] = from_f32<T>(0.f);
    }
    static_cast<T*>(a.dv.ptr)[b * a.dv.stride_b + hk * a.dv.stride_h + (int64_t)i * a.dv.stride_t + d] = from_f32<T>(s);
    static_cast<T*>(a.dk.ptr)[b * a.dk.stride_b + hk * a.dk.stride_h + (int64_t)i * a.dk.stride_t + d] = from_f32<T>(0.f);
  }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------

template <typename K>
static cudaError_t set_smem(K kernel, size_t bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

template <typename T, int D>
static cudaError_t fwd_fill_impl(const AiAttnFwdArgs& a, cudaStream_t st) {
  if (a.layout.all_rows_owned) return cudaSuccess;
  fwd_fill_kernel<T, D><<<dim3(a.seq_len, a.batch), 128, 0, st>>>(a);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t fwd_impl(const AiAttnFwdArgs& a, cudaStream_t st) {
  if (a.layout.n_fwd_items > 0) {
    const size_t smem = fwd_smem_bytes<D>();
    cudaError_t e = set_smem(fwd_kernel<T, D>, smem);
    if (e != cudaSuccess) return e;
    fwd_kernel<T, D><<<dim3(a.layout.n_fwd_items, a.num_q_heads), kThreads, smem, st>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (a.layout.all_rows_owned) return cudaSuccess;
  fwd_fill_kernel<T, D><<<dim3(a.seq_len, a.batch), 128, 0, st>>>(a);
  return cudaGetLastError();
}

// delta for every (b, h, i) row: 16-byte loads when both row layouts allow.
template <typename T, int D>
static cudaError_t launch_delta(const AiAttnBwdArgs& a, float* delta, cudaStream_t st) {
  const AiAttnFwdArgs& f = a.fwd;
  const int64_t rows = (int64_t)f.batch * f.num_q_heads * f.seq_len;
  if (rows16<T>(f.out) && rows16<T>(a.dout)) {
    constexpr int kTpr = D * (int)sizeof(T) / 16, kRpb = 256 / kTpr * 2;
    const dim3 grid((unsigned)((f.seq_len + kRpb - 1) / kRpb), (unsigned)(f.batch * f.num_q_heads));
    delta_vec_kernel<T, D><<<grid, 256, 0, st>>>(a, delta);
  } else {
    delta_kernel<T, D><<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>(a, delta);
  }
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t bwd_impl(const AiAttnBwdArgs& a, float* delta, cudaStream_t st) {
  const AiAttnFwdArgs& f = a.fwd;
  cudaError_t e = launch_delta<T, D>(a, delta, st);
  if (e != cudaSuccess) return e;
  if (f.layout.n_fwd_items > 0) {
    const size_t smem = dq_smem_bytes<D>();
    if ((e = set_smem(dq_kernel<T, D>, smem)) != cudaSuccess) return e;
    dq_kernel<T, D><<<dim3(f.layout.n_fwd_items, f.num_q_heads), kThreads, smem, st>>>(a, delta);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (f.layout.n_kv_items > 0) {
    const size_t smem = dkdv_smem_bytes<D>();
    if ((e = set_smem(dkdv_kernel<T, D>, smem)) != cudaSuccess) return e;
    dkdv_kernel<T, D><<<dim3(f.layout.n_kv_items, f.num_kv_heads), kThreads, smem, st>>>(a, delta);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (f.layout.all_rows_owned) return cudaSuccess;
  bwd_fill_kernel<T, D><<<dim3(f.seq_len, f.batch), 128, 0, st>>>(a);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t delta_impl(const AiAttnBwdArgs& a, float* delta, cudaStream_t st) {
  return launch_delta<T, D>(a, delta, st);
}

template <typename T, int D>
static cudaError_t bwd_fill_impl(const AiAttnBwdArgs& a, cudaStream_t st) {
  if (a.fwd.layout.all_rows_owned) return cudaSuccess;
  bwd_fill_kernel<T, D><<<dim3(a.fwd.seq_len, a.fwd.batch), 128, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace simt

#define AI_DISPATCH_SIMT_D(FN, T, ...)                                                   \
  return D == 32 ? simt::FN<T, 32>(__VA_ARGS__)                                        \
                 : (D == 64 ? simt::FN<T, 64>(__VA_ARGS__) : simt::FN<T, 128>(__VA_ARGS__));
#define AI_DISPATCH_SIMT(FN, ...)                      \
  switch (dtype) {                                     \
    case AI_DTYPE_F32:                                 \
      AI_DISPATCH_SIMT_D(FN, float, __VA_ARGS__)       \
    case AI_DTYPE_BF16:                                \
      AI_DISPATCH_SIMT_D(FN, __nv_bfloat16, __VA_ARGS__) \
    default:                                           \
      AI_DISPATCH_SIMT_D(FN, __half, __VA_ARGS__)      \
  }

cudaError_t simt_fwd(const AiAttnFwdArgs& a, cudaStream_t st) {
  const int dtype = a.dtype, D = a.head_dim;
  AI_DISPATCH_SIMT(fwd_impl, a, st)
}

cudaError_t fwd_fill(const AiAttnFwdArgs& a, cudaStream_t st) {
  const int dtype = a.dtype, D = a.head_dim;
  AI_DISPATCH_SIMT(fwd_fill_impl, a, st)
}

cudaError_t simt_bwd(const AiAttnBwdArgs& a, float* delta, cudaStream_t st) {
  const int dtype = a.fwd.dtype, D = a.fwd.head_dim;
  AI_DISPATCH_SIMT(bwd_impl, a, delta, st)
}

cudaError_t bwd_delta(const AiAttnBwdArgs& a, float* delta, cudaStream_t st) {
  const int dtype = a.fwd.dtype, D = a.fwd.head_dim;
  AI_DISPATCH_SIMT(delta_impl, a, delta, st)
}

cudaError_t bwd_fill(const AiAttnBwdArgs& a, cudaStream_t st) {
  const int dtype = a.fwd.dtype, D = a.fwd.head_dim;
  AI_DISPATCH_SIMT(bwd_fill_impl, a, st)
}

int simt_tile_rows() { return simt::BM; }
int simt_kv_tile_rows() { return simt::BN; }

}  // namespace ai
