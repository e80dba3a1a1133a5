// Shared-memory tile helpers of the sm_100a attention kernels.
//
// A bf16 tile of R rows x 128 columns (head_dim or keys) is stored as two
// column blocks of 64 elements; each block is R rows of 128 bytes with the
// 16-byte chunks XOR-swizzled by (row % 8): the layout TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B and tcgen05 descriptors read with layout type
// "128-byte swizzle".  Tiles start on 1024-byte boundaries.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace ai {
namespace tile {

// 1024-byte-aligned start inside the dynamic shared memory.  Derived by
// pointer arithmetic on the __shared__ array (not an integer round trip) so
// the compiler keeps it in the shared window: shared loads/stores, and no
// assumed aliasing with global loads.
__device__ __forceinline__ uint8_t* align1024(uint8_t* smem_raw) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw));
  return smem_raw + ((1024u - (a & 1023u)) & 1023u);
}

// Byte offset of 16-byte chunk c (0..15, 8 elements each) of row r in an
// R-row tile (c >> 3 selects the column block).
template <int R>
__device__ __forceinline__ uint32_t chunk_off(int r, int c) {
  return (uint32_t)(c >> 3) * (uint32_t)(R * 128) + (uint32_t)r * 128u + ((uint32_t)((c & 7) ^ (r & 7)) << 4);
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
}

// Rotate-half RoPE of one chunk pair: a = dims [8c, 8c + 8), b = the partner
// dims [64 + 8c, 64 + 8c + 8); cs / sn point at the table row's entry 8c.
__device__ __forceinline__ void rotate8(const uint4& a, const uint4& b, const float* cs, const float* sn, uint4& ya,
                                        uint4& yb) {
  float x1[8], x2[8], y1[8], y2[8], c[8], s[8];
  unpack8(a, x1);
  unpack8(b, x2);
  const float4* c4 = reinterpret_cast<const float4*>(cs);
  const float4* s4 = reinterpret_cast<const float4*>(sn);
  const float4 c0 = __ldg(c4), c1 = __ldg(c4 + 1), s0 = __ldg(s4), s1 = __ldg(s4 + 1);
  c[0] = c0.x; c[1] = c0.y; c[2] = c0.z; c[3] = c0.w; c[4] = c1.x; c[5] = c1.y; c[6] = c1.z; c[7] = c1.w;
  s[0] = s0.x; s[1] = s0.y; s[2] = s0.z; s[3] = s0.w; s[4] = s1.x; s[5] = s1.y; s[6] = s1.z; s[7] = s1.w;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    y1[i] = x1[i] * c[i] - x2[i] * s[i];
    y2[i] = x2[i] * c[i] + x1[i] * s[i];
  }
  ya = pack8(y1);
  yb = pack8(y2);
}

// Same rotation with the angles given as fp16 (cos, sin) pairs: t0 holds the
// pairs of dims 8c .. 8c+3, t1 those of 8c+4 .. 8c+7.
__device__ __forceinline__ void rotate8h(const uint4& a, const uint4& b, const uint4& t0, const uint4& t1, uint4& ya,
                                         uint4& yb) {
  float x1[8], x2[8], y1[8], y2[8];
  unpack8(a, x1);
  unpack8(b, x2);
  const __half2* h0 = reinterpret_cast<const __half2*>(&t0);
  const __half2* h1 = reinterpret_cast<const __half2*>(&t1);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 cs = __half22float2(i < 4 ? h0[i] : h1[i - 4]);
    y1[i] = x1[i] * cs.x - x2[i] * cs.y;
    y2[i] = x2[i] * cs.x + x1[i] * cs.y;
  }
  ya = pack8(y1);
  yb = pack8(y2);
}

}  // namespace tile
}  // namespace ai
