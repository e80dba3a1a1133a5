// Decode step (one query token per batch row) against an unrotated K/V cache:
// the IterPositions branch of the reference's attention interface
// (attention/__init__.py:36-51 with attn_layers.py:15-27
// compute_attn_weights_iter).  Each key is rotated by its own position id as
// it is read (the reference rotates the whole cache every token), one CTA
// reads a key chunk of one KV head once for the whole query-head group (the
// reference expands K/V per query head), and a second launch combines the
// chunks' partial softmax results.
//
// HBM-bound: per key 2 x 256 B of K and V (bf16, D = 128) plus a 256 B rotary
// row that stays in L2.  The default split kernel streams K and V by TMA
// (decode_tma_kernel, below); without 16-byte aligned K / V it falls back to
// the register-streaming split kernel (256 threads), per 256-key sub-tile:
//   phase 1  thread t = key: rotated K row . q_g for each query head g
//            (q in shared memory, broadcast reads), logits to shared memory;
//   softmax  warp g = query head g: sub-tile max, running max / sum, the
//            probabilities back to shared memory, the rescale factor of O;
//   phase 2  warp w = keys 32 w .. 32 w + 31, lane = dims 4 l .. 4 l + 3 (V
//            rows read coalesced): o_g += p_g,j v_j in registers.
// At the end the eight warps' O partials are summed through shared memory and
// (m, l, o[128]) per query head go to the workspace; the combine kernel
// merges the chunks and writes bf16 out.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>

#include "../../include/ai_attn.h"
#include "ai_common.cuh"
#include "ai_kernels.h"
#include "sm100_ptx.cuh"
#include "sm100_tile.cuh"

namespace ai {
namespace dec {

constexpr int D = 128;
constexpr int kThreads = 256;  // one key per thread in phase 1
constexpr int kSub = kThreads;  // keys per sub-tile
constexpr int kMaxG = 8;       // query heads per KV head
constexpr float kLog2e = 1.4426950408889634f;

struct Smem {
  float q[kMaxG][D];           // the group's queries, fp32
  float p[kMaxG][kSub];        // logits, then probabilities, of the sub-tile
  float alpha[kMaxG];          // O rescale factor of the sub-tile
  float o[kThreads / 32][D];   // per-warp O partial of one head at the end
};

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// kG: query heads per KV head rounded up to 1, 2, 4 or 8 (the register
// arrays are sized by it; G, the actual count, guards the loops).
template <int kG>
__global__ void __launch_bounds__(kThreads, kG <= 4 ? 4 : 3)
    decode_split_kernel(const AiAttnDecodeArgs a, float* __restrict__ part, int n_split, int chunk) {
  __shared__ Smem sm;
  const int split = blockIdx.x, bh = blockIdx.y;
  const int b = bh / a.num_kv_heads, hk = bh % a.num_kv_heads;
  const int G = a.num_q_heads / a.num_kv_heads;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int c0 = split * chunk, c1 = min(a.kv_len, c0 + chunk);

  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    const __nv_bfloat16* qr = static_cast<const __nv_bfloat16*>(a.q.ptr) + b * a.q.stride_b +
                              (int64_t)(hk * G + g) * a.q.stride_h;
    sm.q[g][d] = __bfloat162float(qr[d]);
  }
  const __nv_bfloat16* kbase = static_cast<const __nv_bfloat16*>(a.k.ptr) + b * a.k.stride_b + hk * a.k.stride_h;
  const __nv_bfloat16* vbase = static_cast<const __nv_bfloat16*>(a.v.ptr) + b * a.v.stride_b + hk * a.v.stride_h;
  const int32_t* krow = a.key_rows + b * a.key_rows_stride_b;
  const uint8_t* kok = a.key_ok ? a.key_ok + b * a.key_ok_stride_b : nullptr;
  const uint4* cs = static_cast<const uint4*>(a.rope_cs16);  // 16 uint4 per table row
  const float sl2 = a.scale * kLog2e;

  float m_run = -CUDART_INF_F, l_run = 0.f;  // warp g < G: head g's running max (log2 units) and sum
  float o[kG][4];
#pragma unroll
  for (int g = 0; g < kG; ++g) o[g][0] = o[g][1] = o[g][2] = o[g][3] = 0.f;
  __syncthreads();

  for (int s0 = c0; s0 < c1; s0 += kSub) {
    // ---- phase 1: logits of key s0 + tid for every head of the group
    {
      const int j = s0 + tid;
      float acc[kG];
#pragma unroll
      for (int g = 0; g < kG; ++g) acc[g] = 0.f;
      // The key's table row and flag are requested together (neither waits
      // for the other).
      const bool inb = j < c1;
      int r = inb ? __ldg(krow + j) : 0;
      const bool ok = inb && (kok == nullptr || __ldg(kok + j) != 0);
      if (ok) {
        if (r < 0 || r >= a.n_pos) {
          report(a.status, AI_ERR_DEV_BOUNDS);
          r = 0;
        }
        const uint4* kr = reinterpret_cast<const uint4*>(kbase + (int64_t)j * a.k.stride_t);
        const uint4* tr = cs + (int64_t)r * (D / 8);
#pragma unroll 2
        for (int c = 0; c < 8; ++c) {
          // dims 8c .. 8c+7 and their rotate-half partners 64 + 8c .. 64 + 8c + 7
          float x1[8], x2[8];
          unpack8(__ldg(kr + c), x1);
          unpack8(__ldg(kr + 8 + c), x2);
          const uint4 t0 = __ldg(tr + 2 * c), t1 = __ldg(tr + 2 * c + 1);
          const __half2* h = reinterpret_cast<const __half2*>(&t0);
          const __half2* h1 = reinterpret_cast<const __half2*>(&t1);
          float y1[8], y2[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float2 csn = __half22float2(i < 4 ? h[i] : h1[i - 4]);
            y1[i] = x1[i] * csn.x - x2[i] * csn.y;
            y2[i] = x2[i] * csn.x + x1[i] * csn.y;
          }
#pragma unroll
          for (int g = 0; g < kG; ++g) {
            if (g < G) {
#pragma unroll
              for (int i = 0; i < 8; ++i) acc[g] = fmaf(y1[i], sm.q[g][8 * c + i], fmaf(y2[i], sm.q[g][64 + 8 * c + i], acc[g]));
            }
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kG; ++g)
        if (g < G) sm.p[g][tid] = ok ? acc[g] * sl2 : -CUDART_INF_F;
    }
    __syncthreads();
    // ---- softmax bookkeeping: warp g handles head g
    if (warp < G) {
      float v[kSub / 32];
      float mx = -CUDART_INF_F;
#pragma unroll
      for (int i = 0; i < kSub / 32; ++i) {
        v[i] = sm.p[warp][lane + 32 * i];
        mx = fmaxf(mx, v[i]);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m_run, mx);
      const float msub = m_new == -CUDART_INF_F ? 0.f : m_new;
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < kSub / 32; ++i) {
        const float pv = exp2f(v[i] - msub);
        sm.p[warp][lane + 32 * i] = pv;
        sum += pv;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      const float alpha = exp2f(m_run - msub);  // 0 while m_run is -inf
      l_run = l_run * alpha + sum;
      m_run = m_new;
      if (lane == 0) sm.alpha[warp] = alpha;
    }
    __syncthreads();
    // ---- phase 2: o_g += p_g,j v_j over this warp's 32 keys
    {
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        if (g < G) {
          const float al = sm.alpha[g];
          o[g][0] *= al;
          o[g][1] *= al;
          o[g][2] *= al;
          o[g][3] *= al;
        }
      }
      const int jb = 32 * warp;
#pragma unroll 4
      for (int jj = 0; jj < 32; ++jj) {
        const int j = s0 + jb + jj;
        if (j >= c1) break;
        const uint2 raw = __ldg(reinterpret_cast<const uint2*>(vbase + (int64_t)j * a.v.stride_t) + lane);
        const float2 v01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
        const float2 v23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
#pragma unroll
        for (int g = 0; g < kG; ++g) {
          if (g < G) {
            const float pv = sm.p[g][jb + jj];
            o[g][0] = fmaf(pv, v01.x, o[g][0]);
            o[g][1] = fmaf(pv, v01.y, o[g][1]);
            o[g][2] = fmaf(pv, v23.x, o[g][2]);
            o[g][3] = fmaf(pv, v23.y, o[g][3]);
          }
        }
      }
    }
    __syncthreads();
  }

  // ---- partials: per head, (m, l, o[128]) with o summed over the warps
  float* base = part + ((int64_t)(b * a.num_q_heads + hk * G) * n_split + split) * (2 + D);
#pragma unroll
  for (int g = 0; g < kG; ++g) {
    if (g >= G) break;  // (G is uniform: every thread leaves together)
    sm.o[warp][4 * lane] = o[g][0];
    sm.o[warp][4 * lane + 1] = o[g][1];
    sm.o[warp][4 * lane + 2] = o[g][2];
    sm.o[warp][4 * lane + 3] = o[g][3];
    __syncthreads();
    float* dst = base + (int64_t)g * n_split * (2 + D);
    if (tid < D) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < kThreads / 32; ++w) acc += sm.o[w][tid];
      dst[2 + tid] = acc;
    }
    if (warp == g && lane == 0) {
      dst[0] = m_run;
      dst[1] = l_run;
    }
    __syncthreads();
  }
}

// TMA-pipelined variant (the default when K and V allow tensor maps): the
// K and V rows of 64-key sub-tiles stream into shared memory by TMA through
// a 3-stage ring, so every CTA keeps up to three sub-tiles (96 KB) in
// flight and the cache is read at full line width; two CTAs per SM.
//   phase 1  eight threads per key (one rotation pair of 8 + 8 dims each,
//            the group's query dims of that pair in registers): the key's
//            dims rotated with the fp16 table row, dotted with the queries,
//            summed over the eight lanes;
//   softmax  warp g = query head g, as in the split kernel;
//   phase 2  warp w = keys 8 w .. 8 w + 7, lane = dims 4 l .. 4 l + 3 of the
//            V rows in shared memory: o_g += p_g,j v_j.
// A bounded wait that expires records AI_ERR_DEV_TIMEOUT, waits (bounded)
// for the loads still in flight and ends the CTA.
namespace tma {
constexpr int kKeys = 64;                   // keys per sub-tile (TMA box rows)
constexpr int kStages = 3;
constexpr uint32_t kHalf = kKeys * 128;     // one 64-dim column block of a sub-tile (128-byte rows)
constexpr uint32_t kTile = 2 * kHalf;       // 16 KB
constexpr uint32_t K0 = 0;                  // K ring
constexpr uint32_t V0 = K0 + kStages * kTile;
constexpr uint32_t Q = V0 + kStages * kTile;  // float [kMaxG][D]
constexpr uint32_t P = Q + kMaxG * D * 4;     // float [kMaxG][kKeys]
constexpr uint32_t ALPHA = P + kMaxG * kKeys * 4;
constexpr uint32_t OSUM = ALPHA + kMaxG * 4;  // float [8 warps][D]
constexpr uint32_t BARS = OSUM + (kThreads / 32) * D * 4;
constexpr uint32_t TOTAL = BARS + 8 * kStages;
constexpr size_t kSmem = TOTAL + 1024;
static_assert(2 * kSmem <= 227 * 1024, "two CTAs per SM");
constexpr long long kWait = 1000000000LL;
}  // namespace tma

template <int kG>
__global__ void __launch_bounds__(kThreads, 2)
    decode_tma_kernel(const AiAttnDecodeArgs a, const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, float* __restrict__ part, int n_split, int chunk) {
  using namespace tma;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = tile::align1024(smem_raw);
  const uint32_t sbase = ptx::smem_u32(sm);
  float* s_q = reinterpret_cast<float*>(sm + Q);
  float* s_p = reinterpret_cast<float*>(sm + P);
  float* s_alpha = reinterpret_cast<float*>(sm + ALPHA);
  float* s_o = reinterpret_cast<float*>(sm + OSUM);
  auto bar = [&](int i) { return sbase + BARS + 8u * (uint32_t)i; };

  const int split = blockIdx.x, bh = blockIdx.y;
  const int b = bh / a.num_kv_heads, hk = bh % a.num_kv_heads;
  const int G = a.num_q_heads / a.num_kv_heads;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int c0 = split * chunk, c1 = min(a.kv_len, c0 + chunk);
  const int n_tiles = c1 > c0 ? (c1 - c0 + kKeys - 1) / kKeys : 0;

  auto issue = [&](int i) {  // sub-tile i into stage i % kStages (thread 0)
    const int st = i % kStages, k0 = c0 + i * kKeys;
    ptx::mbar_arrive_expect_tx(bar(st), 2 * kTile);
    ptx::tma_load_4d(sbase + K0 + st * kTile, &tm_k, bar(st), 0, k0, hk, b);
    ptx::tma_load_4d(sbase + K0 + st * kTile + kHalf, &tm_k, bar(st), 64, k0, hk, b);
    ptx::tma_load_4d(sbase + V0 + st * kTile, &tm_v, bar(st), 0, k0, hk, b);
    ptx::tma_load_4d(sbase + V0 + st * kTile + kHalf, &tm_v, bar(st), 64, k0, hk, b);
  };
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) ptx::mbar_init(bar(i), 1);
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&tm_k);
    ptx::prefetch_tmap(&tm_v);
    for (int i = 0; i < kStages && i < n_tiles; ++i) issue(i);
  }
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    const __nv_bfloat16* qr = static_cast<const __nv_bfloat16*>(a.q.ptr) + b * a.q.stride_b +
                              (int64_t)(hk * G + g) * a.q.stride_h;
    s_q[g * D + d] = __bfloat162float(qr[d]);
  }
  __syncthreads();

  const int32_t* krow = a.key_rows + b * a.key_rows_stride_b;
  const uint8_t* kok = a.key_ok ? a.key_ok + b * a.key_ok_stride_b : nullptr;
  const uint4* cs = static_cast<const uint4*>(a.rope_cs16);  // 16 uint4 per table row
  const float sl2 = a.scale * kLog2e;
  float m_run = -CUDART_INF_F, l_run = 0.f;
  float2 o[kG][2];
#pragma unroll
  for (int g = 0; g < kG; ++g) o[g][0] = o[g][1] = make_float2(0.f, 0.f);

  // Thread t owns rotation pair c = t % 8 (dims 8c .. 8c+7 and 64+8c ..
  // 64+8c+7) of keys t / 8 and t / 8 + 32 of every sub-tile; with at most
  // four heads per group their query dims stay in registers (shared-memory
  // reads of the queries would bound the loop otherwise).
  const int c = tid % 8;
  constexpr bool kQReg = kG <= 4;
  // (pairs of dims in float2: the rotation, the dot products and the P.V
  // accumulation run as packed fp32 FMAs, two dims an instruction)
  float2 qa[kQReg ? kG : 1][4], qb[kQReg ? kG : 1][4];
  if (kQReg) {
#pragma unroll
    for (int g = 0; g < (kQReg ? kG : 1); ++g)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        qa[g][e] = g < G ? make_float2(s_q[g * D + 8 * c + 2 * e], s_q[g * D + 8 * c + 2 * e + 1])
                         : make_float2(0.f, 0.f);
        qb[g][e] = g < G ? make_float2(s_q[g * D + 64 + 8 * c + 2 * e], s_q[g * D + 64 + 8 * c + 2 * e + 1])
                         : make_float2(0.f, 0.f);
      }
  }

  int done = 0;  // sub-tiles consumed
  bool ok_all = true;
  for (int i = 0; i < n_tiles; ++i) {
    const int st = i % kStages;
    // The keys' table rows, flags and rotary values are fetched before the
    // wait for their tile (the table reads hide under it).
    bool okk[2];
    uint4 tt[2][2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int j = c0 + i * kKeys + tid / 8 + 32 * hh;
      const bool inb = j < c1;
      int r = inb ? __ldg(krow + j) : 0;
      okk[hh] = inb && (kok == nullptr || __ldg(kok + j) != 0);
      if (okk[hh] && (r < 0 || r >= a.n_pos)) {
        report(a.status, AI_ERR_DEV_BOUNDS);
        r = 0;
      }
      const uint4* tr = cs + (int64_t)r * (D / 8);
      tt[hh][0] = okk[hh] ? __ldg(tr + 2 * c) : make_uint4(0, 0, 0, 0);
      tt[hh][1] = okk[hh] ? __ldg(tr + 2 * c + 1) : make_uint4(0, 0, 0, 0);
    }
    if (!ptx::mbar_wait(bar(st), (uint32_t)(i / kStages) & 1u, kWait)) {
      report(a.status, AI_ERR_DEV_TIMEOUT);
      ok_all = false;
    }
    if (__syncthreads_or(!ok_all)) break;
    // ---- phase 1: keys tid / 8 and tid / 8 + 32, rotation pair c
    const uint8_t* kt = sm + K0 + st * kTile;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int kk = tid / 8 + 32 * hh;
      float acc[kG];
#pragma unroll
      for (int g = 0; g < kG; ++g) acc[g] = 0.f;
      if (okk[hh]) {
        const uint4 ra = *reinterpret_cast<const uint4*>(kt + tile::chunk_off<kKeys>(kk, c));
        const uint4 rb = *reinterpret_cast<const uint4*>(kt + tile::chunk_off<kKeys>(kk, c + 8));
        const __nv_bfloat162* ka = reinterpret_cast<const __nv_bfloat162*>(&ra);
        const __nv_bfloat162* kb = reinterpret_cast<const __nv_bfloat162*>(&rb);
        const __half2* h0 = reinterpret_cast<const __half2*>(&tt[hh][0]);
        const __half2* h1 = reinterpret_cast<const __half2*>(&tt[hh][1]);
        float2 y1[4], y2[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 x1 = __bfloat1622float2(ka[e]), x2 = __bfloat1622float2(kb[e]);
          const float2 cs0 = __half22float2(e < 2 ? h0[2 * e] : h1[2 * e - 4]);      // (cos, sin) of dim 2e
          const float2 cs1 = __half22float2(e < 2 ? h0[2 * e + 1] : h1[2 * e - 3]);  // of dim 2e + 1
          const float2 cv = make_float2(cs0.x, cs1.x), sv = make_float2(cs0.y, cs1.y);
          const float2 nsv = make_float2(-sv.x, -sv.y);
          y1[e] = __ffma2_rn(x1, cv, __fmul2_rn(x2, nsv));
          y2[e] = __ffma2_rn(x2, cv, __fmul2_rn(x1, sv));
        }
#pragma unroll
        for (int g = 0; g < kG; ++g) {
          if (g < G) {
            float2 a2 = make_float2(0.f, 0.f);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 q1 = kQReg ? qa[kQReg ? g : 0][e]
                                      : make_float2(s_q[g * D + 8 * c + 2 * e], s_q[g * D + 8 * c + 2 * e + 1]);
              const float2 q2 = kQReg ? qb[kQReg ? g : 0][e]
                                      : make_float2(s_q[g * D + 64 + 8 * c + 2 * e], s_q[g * D + 64 + 8 * c + 2 * e + 1]);
              a2 = __ffma2_rn(y1[e], q1, __ffma2_rn(y2[e], q2, a2));
            }
            acc[g] = a2.x + a2.y;
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 1);
        acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 2);
        acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 4);
        if (g < G && c == 0) s_p[g * kKeys + kk] = okk[hh] ? acc[g] * sl2 : -CUDART_INF_F;
      }
    }
    __syncthreads();
    // ---- softmax bookkeeping: warp g handles head g
    if (warp < G) {
      const float v0 = s_p[warp * kKeys + lane], v1 = s_p[warp * kKeys + 32 + lane];
      float mx = fmaxf(v0, v1);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m_run, mx);
      const float msub = m_new == -CUDART_INF_F ? 0.f : m_new;
      const float p0 = exp2f(v0 - msub), p1 = exp2f(v1 - msub);
      s_p[warp * kKeys + lane] = p0;
      s_p[warp * kKeys + 32 + lane] = p1;
      float sum = p0 + p1;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      const float alpha = exp2f(m_run - msub);  // 0 while m_run is -inf
      l_run = l_run * alpha + sum;
      m_run = m_new;
      if (lane == 0) s_alpha[warp] = alpha;
    }
    __syncthreads();
    // ---- phase 2: o_g += p_g,j v_j over this warp's 8 keys
    {
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        if (g < G) {
          const float2 al = make_float2(s_alpha[g], s_alpha[g]);
          o[g][0] = __fmul2_rn(o[g][0], al);
          o[g][1] = __fmul2_rn(o[g][1], al);
        }
      }
      const uint8_t* vt = sm + V0 + st * kTile;
      const int hf = lane / 16, cidx = (lane % 16) / 2, sub = (lane % 2) * 8;
#pragma unroll
      for (int x = 0; x < kKeys / (kThreads / 32); ++x) {
        const int key = warp * (kKeys / (kThreads / 32)) + x;
        const uint2 raw = *reinterpret_cast<const uint2*>(vt + tile::chunk_off<kKeys>(key, 8 * hf + cidx) + sub);
        const float2 v01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
        const float2 v23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
#pragma unroll
        for (int g = 0; g < kG; ++g) {
          if (g < G) {
            const float pv = s_p[g * kKeys + key];
            const float2 p2 = make_float2(pv, pv);
            o[g][0] = __ffma2_rn(p2, v01, o[g][0]);
            o[g][1] = __ffma2_rn(p2, v23, o[g][1]);
          }
        }
      }
    }
    __syncthreads();  // stage st and the probabilities are free again
    done = i + 1;
    if (tid == 0 && i + kStages < n_tiles) issue(i + kStages);
  }
  if (!ok_all) {
    // Loads still in flight land before the CTA ends (bounded).
    if (tid == 0)
      for (int i = done; i < n_tiles && i < done + kStages; ++i)
        ptx::mbar_wait(bar(i % kStages), (uint32_t)(i / kStages) & 1u, kWait);
    __syncthreads();
    return;
  }

  // ---- partials: per head, (m, l, o[128]) with o summed over the warps; lane
  // l holds dims 4 l .. 4 l + 3 of its warp's keys
  float* base = part + ((int64_t)(b * a.num_q_heads + hk * G) * n_split + split) * (2 + D);
#pragma unroll
  for (int g = 0; g < kG; ++g) {
    if (g >= G) break;  // (G is uniform: every thread leaves together)
    s_o[warp * D + 4 * lane] = o[g][0].x;
    s_o[warp * D + 4 * lane + 1] = o[g][0].y;
    s_o[warp * D + 4 * lane + 2] = o[g][1].x;
    s_o[warp * D + 4 * lane + 3] = o[g][1].y;
    __syncthreads();
    float* dst = base + (int64_t)g * n_split * (2 + D);
    if (tid < D) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < kThreads / 32; ++w) acc += s_o[w * D + tid];
      dst[2 + tid] = acc;
    }
    if (warp == g && lane == 0) {
      dst[0] = m_run;
      dst[1] = l_run;
    }
    __syncthreads();
  }
}

// One CTA per (row, query head), thread = dim: merges the chunks' partials.
__global__ void __launch_bounds__(D) decode_combine_kernel(const AiAttnDecodeArgs a, const float* __restrict__ part,
                                                           int n_split) {
  const int bh = blockIdx.x, b = bh / a.num_q_heads, h = bh % a.num_q_heads, d = threadIdx.x;
  const float* p = part + (int64_t)bh * n_split * (2 + D);
  float M = -CUDART_INF_F;
  for (int s = 0; s < n_split; ++s) M = fmaxf(M, p[s * (2 + D)]);
  float L = 0.f, acc = 0.f;
  if (M != -CUDART_INF_F) {
    for (int s = 0; s < n_split; ++s) {
      const float w = exp2f(p[s * (2 + D)] - M);
      L += w * p[s * (2 + D) + 1];
      acc += w * p[s * (2 + D) + 2 + d];
    }
  }
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(a.out.ptr) + b * a.out.stride_b + h * a.out.stride_h;
  o[d] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
}

}  // namespace dec

// Whether the TMA kernel can read K and V: 16-byte aligned bases and strides
// (what a tensor map needs).
static bool decode_tma_ok(const AiAttnDecodeArgs& a) {
  const uintptr_t m = reinterpret_cast<uintptr_t>(a.k.ptr) | reinterpret_cast<uintptr_t>(a.v.ptr);
  const int64_t st = a.k.stride_t | a.k.stride_h | a.k.stride_b | a.v.stride_t | a.v.stride_h | a.v.stride_b;
  return (m & 15) == 0 && (st & 7) == 0;
}

// Splits of each (row, KV head) pair's keys into chunks of whole 64-key
// sub-tiles: the count that minimises (waves of CTAs) x (sub-tiles per CTA
// + one for a CTA's first loads), at the kernel's CTAs per SM.
static void decode_plan(const AiAttnDecodeArgs& a, int* n_split, int* chunk) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int pairs = a.batch * a.num_kv_heads;
  constexpr int kUnit = dec::tma::kKeys;
  const int units = (a.kv_len + kUnit - 1) / kUnit;
  const int per_sm = decode_tma_ok(a) ? 2 : (a.num_q_heads / a.num_kv_heads <= 4 ? 4 : 3);
  const int64_t slots = (int64_t)per_sm * sms;
  int best = 1;
  int64_t best_cost = -1;
  for (int n = 1; n <= units && n <= 1024; ++n) {
    const int per = (units + n - 1) / n;
    const int used = (units + per - 1) / per;  // chunks actually needed
    if (used != n) continue;
    const int64_t waves = ((int64_t)pairs * n + slots - 1) / slots;
    const int64_t cost = waves * (per + 1);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = n;
    }
  }
  const int per = (units + best - 1) / best;
  *chunk = per * kUnit;
  *n_split = (a.kv_len + *chunk - 1) / *chunk;
  if (*n_split < 1) *n_split = 1;
}

int decode_check(const AiAttnDecodeArgs* a) {
  if (!a) return AI_ERR_NULL;
  if (a->batch <= 0 || a->kv_len <= 0 || a->num_q_heads <= 0 || a->num_kv_heads <= 0 ||
      a->num_q_heads % a->num_kv_heads != 0 || a->num_q_heads / a->num_kv_heads > dec::kMaxG)
    return AI_ERR_SHAPE;
  if (a->head_dim != dec::D) return AI_ERR_HEAD_DIM;
  if (a->dtype != AI_DTYPE_BF16) return AI_ERR_DTYPE;
  if (!a->q.ptr || !a->k.ptr || !a->v.ptr || !a->out.ptr || !a->key_rows || !a->rope_cs16) return AI_ERR_NULL;
  if (a->n_pos <= 0) return AI_ERR_SHAPE;
  // 16-byte K rows (uint4 loads), 8-byte V slices, 16-byte rotary rows
  if ((reinterpret_cast<uintptr_t>(a->k.ptr) & 15) || (a->k.stride_t & 7) || (a->k.stride_h & 7) ||
      (a->k.stride_b & 7))
    return AI_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(a->v.ptr) & 7) || (a->v.stride_t & 3) || (a->v.stride_h & 3) ||
      (a->v.stride_b & 3))
    return AI_ERR_ALIGN;
  if (reinterpret_cast<uintptr_t>(a->rope_cs16) & 15) return AI_ERR_ALIGN;
  if (a->key_rows_stride_b < 0 || a->key_ok_stride_b < 0) return AI_ERR_STRIDE;
  return AI_OK;
}

size_t decode_workspace_bytes(const AiAttnDecodeArgs& a) {
  int n_split = 1, chunk = dec::kSub;
  decode_plan(a, &n_split, &chunk);
  const size_t b = (size_t)a.batch * a.num_q_heads * n_split * (2 + dec::D) * sizeof(float);
  return (b + 255) / 256 * 256;
}

int decode_launch(const AiAttnDecodeArgs& a, cudaStream_t st) {
  int n_split = 1, chunk = dec::kSub;
  decode_plan(a, &n_split, &chunk);
  if (!a.workspace || a.workspace_bytes < decode_workspace_bytes(a)) return AI_ERR_WORKSPACE;
  float* part = static_cast<float*>(a.workspace);
  ProfScope ps(AI_PROF_DECODE, st);
  const dim3 grid(n_split, a.batch * a.num_kv_heads);
  const int G = a.num_q_heads / a.num_kv_heads;
  CUtensorMap tk, tv;
  AiTensor4 k4 = a.k, v4 = a.v;
  if (decode_tma_ok(a) && sm100_make_map(&tk, k4, a.batch, a.num_kv_heads, a.kv_len, dec::tma::kKeys) &&
      sm100_make_map(&tv, v4, a.batch, a.num_kv_heads, a.kv_len, dec::tma::kKeys)) {
    auto run = [&](auto kernel) -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dec::tma::kSmem);
      if (e == cudaSuccess) kernel<<<grid, dec::kThreads, dec::tma::kSmem, st>>>(a, tk, tv, part, n_split, chunk);
      return e;
    };
    cudaError_t e;
    if (G <= 1)
      e = run(dec::decode_tma_kernel<1>);
    else if (G <= 2)
      e = run(dec::decode_tma_kernel<2>);
    else if (G <= 4)
      e = run(dec::decode_tma_kernel<4>);
    else
      e = run(dec::decode_tma_kernel<8>);
    if (e != cudaSuccess) return AI_ERR_LAUNCH;
  } else if (G <= 1)
    dec::decode_split_kernel<1><<<grid, dec::kThreads, 0, st>>>(a, part, n_split, chunk);
  else if (G <= 2)
    dec::decode_split_kernel<2><<<grid, dec::kThreads, 0, st>>>(a, part, n_split, chunk);
  else if (G <= 4)
    dec::decode_split_kernel<4><<<grid, dec::kThreads, 0, st>>>(a, part, n_split, chunk);
  else
    dec::decode_split_kernel<8><<<grid, dec::kThreads, 0, st>>>(a, part, n_split, chunk);
  dec::decode_combine_kernel<<<a.batch * a.num_q_heads, dec::D, 0, st>>>(a, part, n_split);
  return cudaGetLastError() == cudaSuccess ? AI_OK : AI_ERR_LAUNCH;
}

}  // namespace ai

extern "C" int ai_attn_decode_workspace(const AiAttnDecodeArgs* args, size_t* bytes) {
  const int rc = ai::decode_check(args);
  if (rc != AI_OK) return rc;
  if (!bytes) return AI_ERR_NULL;
  *bytes = ai::decode_workspace_bytes(*args);
  return AI_OK;
}

extern "C" int ai_attn_decode(const AiAttnDecodeArgs* args, void* stream) {
  const int rc = ai::decode_check(args);
  if (rc != AI_OK) return rc;
  return ai::decode_launch(*args, static_cast<cudaStream_t>(stream));
}
