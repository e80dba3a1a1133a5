// Index-head cursor attention (the AutoIndexer edit-cursor losses), batched.
//
// Restates compute_index_losses (attn_layers.py:40-110, reference): for every
// edit (an EXTEND block) one "start" row (head 0, the query just before the
// edit marker) and one "end" row (head 1, the edit marker) attend over a key
// prefix with keys rotated by their position relative to the query
// (compute_attn_weights_iter, attn_layers.py:15-27: q . R(rel_j) k_j, masked
// keys -inf, times scale), and the loss of the row is -log_softmax at the
// cursor key.  The reference loops over the edits in Python with a dozen
// small torch ops each; here every row of every edit is one CTA of one
// launch (forward), and the backward is two launches with no atomics:
//
//   index_fwd_kernel    (row, batch):  logits, log-sum-exp, loss of the row
//   index_dq_kernel     (row, batch):  dq_row = scale sum_j g_j R(rel_j) k_j
//   index_dk_kernel     (key chunk, head, batch): dk_j = scale sum_rows g_rj R(rel_rj)^T q_r
//
// with g_j = dloss * (softmax_j - [j == target]).  Layout: a warp per key,
// lane l owning the rotation pairs (d, d + D/2) with d = l, l + 32, ... (the
// rotate-half pairing of attention/utils.py:5-6), so a key's dot product is
// one warp reduction and its rotation needs no exchange between lanes.

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math_constants.h>

#include "../../include/ai_attn.h"
#include "ai_common.cuh"

namespace ai {
namespace index {

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;

template <typename T>
__device__ __forceinline__ const T* row_ptr(const AiTensor4& t, int b, int h, int i) {
  return static_cast<const T*>(t.ptr) + (int64_t)b * t.stride_b + (int64_t)h * t.stride_h + (int64_t)i * t.stride_t;
}

// Lane l's pairs: d = l + 32 * p for p < P (P = max(1, D / 64); lanes with
// l >= D / 2 own nothing when D < 64).
template <int D>
struct Lane {
  static constexpr int H = D / 2;
  static constexpr int P = H >= 32 ? H / 32 : 1;
  __device__ static bool owns(int lane, int p) { return lane + 32 * p < H; }
};

template <int D, typename T>
__device__ __forceinline__ void load_pairs(const T* row, int lane, float (&x1)[Lane<D>::P], float (&x2)[Lane<D>::P]) {
#pragma unroll
  for (int p = 0; p < Lane<D>::P; ++p) {
    const int d = lane + 32 * p;
    x1[p] = Lane<D>::owns(lane, p) ? to_f32(row[d]) : 0.f;
    x2[p] = Lane<D>::owns(lane, p) ? to_f32(row[d + D / 2]) : 0.f;
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// q . R(rel) k for the lane's pairs (summed over the warp by the caller):
// R(rel) k = (k1 c - k2 s, k2 c + k1 s) on each pair (k1, k2) = (k_d, k_{d+D/2}).
template <int D>
__device__ __forceinline__ float pair_dot(const float (&q1)[Lane<D>::P], const float (&q2)[Lane<D>::P],
                                          const float (&k1)[Lane<D>::P], const float (&k2)[Lane<D>::P],
                                          const float* cs, const float* sn, int lane) {
  float acc = 0.f;
#pragma unroll
  for (int p = 0; p < Lane<D>::P; ++p) {
    if (!Lane<D>::owns(lane, p)) continue;
    const int d = lane + 32 * p;
    const float c = cs[d], s = sn[d];
    acc += q1[p] * (k1[p] * c - k2[p] * s) + q2[p] * (k2[p] * c + k1[p] * s);
  }
  return acc;
}

template <int D, typename T>
__global__ void __launch_bounds__(kThreads) index_fwd_kernel(const AiIndexArgs a) {
  const int r = blockIdx.x, b = blockIdx.y, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int32_t* row = a.rows + 4 * (int64_t)r;
  const int h = row[0], qi = row[1], n = row[2], off = row[3];
  float q1[Lane<D>::P], q2[Lane<D>::P];
  load_pairs<D>(row_ptr<T>(a.q, b, h, qi), lane, q1, q2);
  float* logits = a.logits + (int64_t)b * a.n_keys + off;
  float m = -CUDART_INF_F, l = 0.f;
  for (int j = warp; j < n; j += kWarps) {
    const bool ok = a.key_ok[off + j] != 0;
    float v = -CUDART_INF_F;
    if (ok) {
      float k1[Lane<D>::P], k2[Lane<D>::P];
      load_pairs<D>(row_ptr<T>(a.k, b, h, j), lane, k1, k2);
      const int tr = clamp_row(a.key_rows[off + j], a.n_pos, a.status);
      const float dot = warp_sum(pair_dot<D>(q1, q2, k1, k2, a.rope_cos + (int64_t)tr * (D / 2),
                                             a.rope_sin + (int64_t)tr * (D / 2), lane));
      v = dot * a.scale;
      const float mn = fmaxf(m, v);
      l = l * __expf(m - mn) + __expf(v - mn);
      m = mn;
    }
    if (lane == 0) logits[j] = v;
  }
  __shared__ float s_m[kWarps], s_l[kWarps];
  if (lane == 0) {
    s_m[warp] = m;
    s_l[warp] = l;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = -CUDART_INF_F, L = 0.f;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, s_m[w]);
    for (int w = 0; w < kWarps; ++w)
      if (s_l[w] > 0.f) L += s_l[w] * __expf(s_m[w] - M);
    const float lse = L > 0.f ? M + __logf(L) : -CUDART_INF_F;
    a.lse[(int64_t)b * a.n_rows + r] = lse;
    const int t = a.targets[r];
    float tv = -CUDART_INF_F;
    if (t >= 0 && t < n) {
      __threadfence_block();
      tv = logits[t];
    }
    a.loss[(int64_t)b * a.n_rows + r] = lse - tv;  // +inf when the cursor key is masked
  }
}

// Weight of key j in row r: dloss * (softmax_j - [j == target]).
__device__ __forceinline__ float key_grad(float logit, float lse, float dl, bool is_target) {
  const float p = logit == -CUDART_INF_F ? 0.f : __expf(logit - lse);
  return dl * (p - (is_target ? 1.f : 0.f));
}

template <int D, typename T>
__global__ void __launch_bounds__(kThreads) index_dq_kernel(const AiIndexBwdArgs a) {
  const AiIndexArgs& f = a.fwd;
  const int r = blockIdx.x, b = blockIdx.y, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int32_t* row = f.rows + 4 * (int64_t)r;
  const int h = row[0], qi = row[1], n = row[2], off = row[3], t = f.targets[r];
  const float lse = f.lse[(int64_t)b * f.n_rows + r], dl = a.dloss[(int64_t)b * f.n_rows + r];
  const float* logits = f.logits + (int64_t)b * f.n_keys + off;
  float g1[Lane<D>::P], g2[Lane<D>::P];
#pragma unroll
  for (int p = 0; p < Lane<D>::P; ++p) g1[p] = g2[p] = 0.f;
  for (int j = warp; j < n; j += kWarps) {
    const float gj = key_grad(logits[j], lse, dl, j == t);
    if (gj == 0.f) continue;
    float k1[Lane<D>::P], k2[Lane<D>::P];
    load_pairs<D>(row_ptr<T>(f.k, b, h, j), lane, k1, k2);
    const int tr = clamp_row(f.key_rows[off + j], f.n_pos, f.status);
    const float* cs = f.rope_cos + (int64_t)tr * (D / 2);
    const float* sn = f.rope_sin + (int64_t)tr * (D / 2);
#pragma unroll
    for (int p = 0; p < Lane<D>::P; ++p) {
      if (!Lane<D>::owns(lane, p)) continue;
      const int d = lane + 32 * p;
      const float c = cs[d], s = sn[d];
      g1[p] += gj * (k1[p] * c - k2[p] * s);
      g2[p] += gj * (k2[p] * c + k1[p] * s);
    }
  }
  __shared__ float s_g[kWarps][D];
#pragma unroll
  for (int p = 0; p < Lane<D>::P; ++p) {
    if (!Lane<D>::owns(lane, p)) continue;
    const int d = lane + 32 * p;
    s_g[warp][d] = g1[p];
    s_g[warp][d + D / 2] = g2[p];
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += kThreads) {
    float v = 0.f;
    for (int w = 0; w < kWarps; ++w) v += s_g[w][d];
    T* out = static_cast<T*>(a.dq.ptr) + (int64_t)b * a.dq.stride_b + (int64_t)h * a.dq.stride_h +
             (int64_t)qi * a.dq.stride_t;
    out[d] = from_f32<T>(v * f.scale);
  }
}

// dk of keys [j0, j0 + kWarps * kKeysPerWarp) of one head: a warp per key,
// every index row of the head that sees the key.
constexpr int kKeysPerWarp = 4;

template <int D, typename T>
__global__ void __launch_bounds__(kThreads) index_dk_kernel(const AiIndexBwdArgs a) {
  const AiIndexArgs& f = a.fwd;
  const int h = blockIdx.y, b = blockIdx.z, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int kk = 0; kk < kKeysPerWarp; ++kk) {
    const int j = (blockIdx.x * kKeysPerWarp + kk) * kWarps + warp;
    if (j >= f.seq_len) break;
    float g1[Lane<D>::P], g2[Lane<D>::P];
#pragma unroll
    for (int p = 0; p < Lane<D>::P; ++p) g1[p] = g2[p] = 0.f;
    for (int r = 0; r < f.n_rows; ++r) {
      const int32_t* row = f.rows + 4 * (int64_t)r;
      if (row[0] != h || j >= row[2]) continue;
      const int off = row[3];
      const float lse = f.lse[(int64_t)b * f.n_rows + r], dl = a.dloss[(int64_t)b * f.n_rows + r];
      const float gj = key_grad(f.logits[(int64_t)b * f.n_keys + off + j], lse, dl, j == f.targets[r]);
      if (gj == 0.f) continue;
      float q1[Lane<D>::P], q2[Lane<D>::P];
      load_pairs<D>(row_ptr<T>(f.q, b, h, row[1]), lane, q1, q2);
      const int tr = clamp_row(f.key_rows[off + j], f.n_pos, f.status);
      const float* cs = f.rope_cos + (int64_t)tr * (D / 2);
      const float* sn = f.rope_sin + (int64_t)tr * (D / 2);
      // R(rel)^T q = (q1 c + q2 s, q2 c - q1 s) on each pair.
#pragma unroll
      for (int p = 0; p < Lane<D>::P; ++p) {
        if (!Lane<D>::owns(lane, p)) continue;
        const int d = lane + 32 * p;
        const float c = cs[d], s = sn[d];
        g1[p] += gj * (q1[p] * c + q2[p] * s);
        g2[p] += gj * (q2[p] * c - q1[p] * s);
      }
    }
    T* out = static_cast<T*>(a.dk.ptr) + (int64_t)b * a.dk.stride_b + (int64_t)h * a.dk.stride_h +
             (int64_t)j * a.dk.stride_t;
#pragma unroll
    for (int p = 0; p < Lane<D>::P; ++p) {
      if (!Lane<D>::owns(lane, p)) continue;
      const int d = lane + 32 * p;
      out[d] = from_f32<T>(g1[p] * f.scale);
      out[d + D / 2] = from_f32<T>(g2[p] * f.scale);
    }
  }
}

int validate(const AiIndexArgs* a) {
  if (!a) return AI_ERR_NULL;
  if (a->batch <= 0 || a->seq_len <= 0 || a->n_rows < 0 || a->n_keys < 0 || a->n_pos <= 0) return AI_ERR_SHAPE;
  if (a->head_dim != 32 && a->head_dim != 64 && a->head_dim != 128) return AI_ERR_HEAD_DIM;
  if (a->dtype != AI_DTYPE_BF16 && a->dtype != AI_DTYPE_F32) return AI_ERR_DTYPE;
  if (!a->q.ptr || !a->k.ptr || !a->rope_cos || !a->rope_sin || !a->logits || !a->lse || !a->loss) return AI_ERR_NULL;
  if (a->n_rows > 0 && (!a->rows || !a->targets || !a->key_rows || !a->key_ok)) return AI_ERR_NULL;
  return AI_OK;
}

}  // namespace index
}  // namespace ai

// Launches KERNEL<D, T> for the args' head_dim and dtype.
#define AI_INDEX_DISPATCH(KERNEL, GRID, ARGS, D, DTYPE, ST)                                       \
  do {                                                                                            \
    if ((DTYPE) == AI_DTYPE_BF16) {                                                               \
      if ((D) == 32) KERNEL<32, __nv_bfloat16><<<(GRID), ai::index::kThreads, 0, (ST)>>>(ARGS);   \
      else if ((D) == 64) KERNEL<64, __nv_bfloat16><<<(GRID), ai::index::kThreads, 0, (ST)>>>(ARGS); \
      else KERNEL<128, __nv_bfloat16><<<(GRID), ai::index::kThreads, 0, (ST)>>>(ARGS);            \
    } else {                                                                                      \
      if ((D) == 32) KERNEL<32, float><<<(GRID), ai::index::kThreads, 0, (ST)>>>(ARGS);           \
      else if ((D) == 64) KERNEL<64, float><<<(GRID), ai::index::kThreads, 0, (ST)>>>(ARGS);      \
      else KERNEL<128, float><<<(GRID), ai::index::kThreads, 0, (ST)>>>(ARGS);                    \
    }                                                                                             \
  } while (0)

extern "C" {

int ai_index_fwd(const AiIndexArgs* a, void* stream) {
  using namespace ai::index;
  int rc = validate(a);
  if (rc != AI_OK) return rc;
  if (a->n_rows == 0) return AI_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  AI_INDEX_DISPATCH(index_fwd_kernel, dim3(a->n_rows, a->batch), *a, a->head_dim, a->dtype, st);
  return cudaGetLastError() == cudaSuccess ? AI_OK : AI_ERR_LAUNCH;
}

int ai_index_bwd(const AiIndexBwdArgs* a, void* stream) {
  using namespace ai::index;
  if (!a) return AI_ERR_NULL;
  int rc = validate(&a->fwd);
  if (rc != AI_OK) return rc;
  if (!a->dloss || !a->dq.ptr || !a->dk.ptr) return AI_ERR_NULL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const AiIndexArgs& f = a->fwd;
  if (f.n_rows > 0) {
    AI_INDEX_DISPATCH(index_dq_kernel, dim3(f.n_rows, f.batch), *a, f.head_dim, f.dtype, st);
    if (cudaGetLastError() != cudaSuccess) return AI_ERR_LAUNCH;
  }
  const int per = kWarps * kKeysPerWarp;
  AI_INDEX_DISPATCH(index_dk_kernel, dim3((f.seq_len + per - 1) / per, 2, f.batch), *a, f.head_dim, f.dtype, st);
  return cudaGetLastError() == cudaSuccess ? AI_OK : AI_ERR_LAUNCH;
}

}  // extern "C"
