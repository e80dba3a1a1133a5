// Internal launch interface between the C ABI (ai_capi.cu) and the kernel
// translation units.  Not part of the public ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/ai_attn.h"

namespace ai {

// SIMT kernels: any supported dtype, head_dim 32, 64 or 128.
cudaError_t simt_fwd(const AiAttnFwdArgs& a, cudaStream_t st);
cudaError_t simt_bwd(const AiAttnBwdArgs& a, float* delta, cudaStream_t st);
// Rows no block owns: out = v of the row, lse = 0 (any dtype / head_dim).
cudaError_t fwd_fill(const AiAttnFwdArgs& a, cudaStream_t st);
int simt_tile_rows();
int simt_kv_tile_rows();

// Backward pieces shared by every backward path (any dtype / head_dim):
// delta[b, h, i] = sum_d dO * O, and the rows no block owns.
cudaError_t bwd_delta(const AiAttnBwdArgs& a, float* delta, cudaStream_t st);
cudaError_t bwd_fill(const AiAttnBwdArgs& a, cudaStream_t st);

// tcgen05 / TMEM / TMA kernels (sm_100a): bf16, head_dim 128.
bool sm100_fwd_supported(int dtype, int head_dim);
int sm100_fwd_tile_rows();
// Optional launch timing (ai_profile.cu): a scope around one kernel launch
// records CUDA events on the launch stream while profiling is enabled.
int prof_begin(int kind, cudaStream_t st);
void prof_end(int slot, cudaStream_t st);
struct ProfScope {
  int slot;
  cudaStream_t st;
  ProfScope(int kind, cudaStream_t s) : slot(prof_begin(kind, s)), st(s) {}
  ~ProfScope() { prof_end(slot, st); }
};

// Returns AI_OK or an AiStatus > 0; `cuda_err` receives the CUDA error of a failed launch.
int sm100_fwd(const AiAttnFwdArgs& a, cudaStream_t st, cudaError_t* cuda_err);
// Forward workspace after the rotated copies for the abs split: partial rows
// (fp32 O / l and log2-sum) of the abs-block items (0: no split possible).
size_t sm100_fwd_abs_part_bytes(const AiAttnFwdArgs& a);
bool sm100_bwd_supported(int dtype, int head_dim);
int sm100_kv_tile_rows();
// `rot`: scratch for the once-rotated Q/K copies (prerot_bytes), or nullptr to
// rotate every tile in shared memory; `rot_ready`: `rot` already holds them
// (written by the forward), so they are not rotated again.
// Bytes of fp32 partial sums the dK/dV pass wants for split key tiles (0:
// the layout splits none, or splitting would not pay on this device).
size_t sm100_kv_partial_bytes(const AiAttnFwdArgs& f);
// `dq_part`: scratch of sm100_dq_abs_part_bytes for the abs split of dQ, or
// nullptr (the one-head kernel then runs the abs-block items whole).
size_t sm100_dq_abs_part_bytes(const AiAttnFwdArgs& f);
// `parts`: AI_BWD_DQ and / or AI_BWD_DKDV (see AiAttnBwdArgs.parts).
int sm100_bwd(const AiAttnBwdArgs& a, float* delta, void* rot, bool rot_ready, float* partials, float* dq_part,
              int parts, cudaStream_t st, cudaError_t* cuda_err);
// TMA map over a (B, H, T, 128) bf16 tensor, box 64 x box_rows, 128-byte swizzle.
bool sm100_make_map(CUtensorMap* map, const AiTensor4& t, int B, int H, int T, int box_rows);

// Once-rotated Q and K copies (bf16, head_dim 128) for the tensor-core kernels:
// bytes of scratch they need (q_bytes: offset of the K copy), and the launch
// writing q_rot = R(q_pos) q at buf and k_rot = R(k_own) k at buf + q_bytes.
// The rotation-class chunks follow at buf + qk_bytes.
size_t prerot_bytes(const AiAttnFwdArgs& a, size_t* q_bytes, size_t* qk_bytes = nullptr);
cudaError_t prerot(const AiAttnFwdArgs& a, void* buf, cudaStream_t st);
// (B, H, T, 128) views of the two copies inside buf, and (n_rot_classes, Hkv,
// 64, 128) of the class chunks (false if buf is misaligned).
bool sm100_rotated_views(const AiAttnFwdArgs& a, void* buf, AiTensor4* qr, AiTensor4* kr, AiTensor4* kc = nullptr);

}  // namespace ai
