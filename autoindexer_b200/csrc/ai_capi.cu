// C ABI of the chain-of-edits attention (declared in include/ai_attn.h):
// host-side argument validation and kernel dispatch.  Nothing here allocates
// device memory; the backward's scratch comes from the caller.

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "../../include/ai_attn.h"
#include "ai_kernels.h"

namespace {

constexpr int kMaxDevices = 64;
int g_cc_major[kMaxDevices];  // 0 = not queried yet

bool device_is_sm100() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
  if (g_cc_major[dev] == 0) {
    int major = -1;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
    g_cc_major[dev] = major;
  }
  return g_cc_major[dev] == 10;
}

size_t elem_bytes(int dtype) { return dtype == AI_DTYPE_F32 ? 4 : 2; }

bool tensor_ok(const AiTensor4& t) {
  return t.ptr != nullptr && t.stride_b >= 0 && t.stride_h >= 0 && t.stride_t >= 0;
}

int validate_fwd(const AiAttnFwdArgs* a) {
  if (!a) return AI_ERR_NULL;
  if (a->batch <= 0 || a->seq_len <= 0 || a->num_q_heads <= 0 || a->num_kv_heads <= 0) return AI_ERR_SHAPE;
  if (a->num_q_heads % a->num_kv_heads != 0) return AI_ERR_SHAPE;
  if (a->dtype != AI_DTYPE_BF16 && a->dtype != AI_DTYPE_F16 && a->dtype != AI_DTYPE_F32) return AI_ERR_DTYPE;
  if (a->head_dim != 32 && a->head_dim != 64 && a->head_dim != 128) return AI_ERR_HEAD_DIM;
  if (!tensor_ok(a->q) || !tensor_ok(a->k) || !tensor_ok(a->v) || !tensor_ok(a->out)) return AI_ERR_NULL;
  if (!a->lse) return AI_ERR_NULL;
  const AiAttnLayout& L = a->layout;
  if (!L.blocks || !L.row_blocks || !L.row_cov || !L.key_info || !L.q_pos || !L.k_own || !L.rope_cos ||
      !L.rope_sin || !L.rope_cs16)
    return AI_ERR_NULL;
  if (a->workspace && ((uintptr_t)a->workspace % 256)) return AI_ERR_ALIGN;
  if (L.n_blocks < 0 || L.n_keys < 0 || L.n_pos <= 0 || L.n_fwd_items < 0 || L.n_kv_items < 0) return AI_ERR_LAYOUT;
  if (L.n_kv_chunks < 0 || L.n_kv_partials < 0 || L.n_kv_reduce < 0 || (L.n_kv_chunks > 0 && !L.kv_chunks) ||
      (L.n_kv_reduce > 0 && !L.kv_reduce) || (L.n_kv_chunks > 0 && L.n_kv_chunks < L.n_kv_items))
    return AI_ERR_LAYOUT;
  if (L.n_rot_classes < 0 || L.n_chunk_cls < 0 ||
      (L.n_rot_classes > 0 && (!L.blk_cls || !L.chunk_cls || !L.rot_classes || L.n_chunk_cls <= 0)))
    return AI_ERR_LAYOUT;
  if (L.n_fwd_abs_short_items < 0 || L.n_fwd_abs_short_items > L.n_fwd_abs_items) return AI_ERR_LAYOUT;
  if (L.n_fwd_abs_items < 0 || L.n_fwd_short_items < 0 ||
      (int64_t)L.n_fwd_abs_items + L.n_fwd_short_items > L.n_fwd_items || L.n_kv_abs_items < 0 ||
      L.n_kv_abs_items > L.n_kv_items)
    return AI_ERR_LAYOUT;
  if (L.n_fwd_items > 0 && !L.fwd_items) return AI_ERR_NULL;
  if (L.n_kv_items > 0 && !L.kv_items) return AI_ERR_NULL;
  if (L.fwd_tile != ai_attn_fwd_tile_rows(a->dtype, a->head_dim)) return AI_ERR_LAYOUT;
  if (L.kv_tile != ai_attn_kv_tile_rows(a->dtype, a->head_dim)) return AI_ERR_LAYOUT;
  const uintptr_t mis = (uintptr_t)a->q.ptr | (uintptr_t)a->k.ptr | (uintptr_t)a->v.ptr | (uintptr_t)a->out.ptr;
  if (mis % elem_bytes(a->dtype)) return AI_ERR_ALIGN;
  return AI_OK;
}

size_t delta_bytes(const AiAttnFwdArgs& f) {
  const size_t n = (size_t)f.batch * f.num_q_heads * f.seq_len * sizeof(float);
  return (n + 255) & ~size_t(255);
}

int launch_status(cudaError_t e) { return e == cudaSuccess ? AI_OK : AI_ERR_LAUNCH; }

// The caller vouches (fwd_rotated) that fwd.workspace still holds the
// forward's rotated copies; they are used when the workspace can hold them
// and is aligned (otherwise the backward rotates into its own workspace).
bool fwd_copies(const AiAttnBwdArgs& a) {
  return a.fwd_rotated == 1 && a.fwd.workspace && ((uintptr_t)a.fwd.workspace % 256) == 0 &&
         a.fwd.workspace_bytes >= ai::prerot_bytes(a.fwd, nullptr);
}

}  // namespace

extern "C" {

int ai_attn_abi_version(void) { return AI_ATTN_ABI_VERSION; }

int ai_attn_fwd_tile_rows(int dtype, int head_dim) {
  return ai::sm100_fwd_supported(dtype, head_dim) ? ai::sm100_fwd_tile_rows() : ai::simt_tile_rows();
}

int ai_attn_kv_tile_rows(int dtype, int head_dim) {
  return ai::sm100_bwd_supported(dtype, head_dim) ? ai::sm100_kv_tile_rows() : ai::simt_kv_tile_rows();
}

int ai_attn_fwd(const AiAttnFwdArgs* a, void* stream) {
  int rc = validate_fwd(a);
  if (rc != AI_OK) return rc;
  if (!device_is_sm100()) return AI_ERR_NO_DEVICE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (ai::sm100_fwd_supported(a->dtype, a->head_dim)) {
    cudaError_t ce = cudaSuccess;
    rc = ai::sm100_fwd(*a, st, &ce);
    if (rc != AI_OK) return rc;
    if (a->layout.all_rows_owned) return AI_OK;
    ai::ProfScope ps(AI_PROF_FWD_FILL, st);
    return launch_status(ai::fwd_fill(*a, st));
  }
  ai::ProfScope ps(AI_PROF_SIMT, st);
  return launch_status(ai::simt_fwd(*a, st));
}

int ai_attn_fwd_workspace(const AiAttnFwdArgs* a, size_t* bytes) {
  if (!a || !bytes) return AI_ERR_NULL;
  int rc = validate_fwd(a);
  if (rc != AI_OK) return rc;
  *bytes = ai::sm100_fwd_supported(a->dtype, a->head_dim)
               ? ai::prerot_bytes(*a, nullptr) + ai::sm100_fwd_abs_part_bytes(*a)
               : 0;
  return AI_OK;
}

int ai_attn_bwd_workspace(const AiAttnBwdArgs* a, size_t* bytes) {
  if (!a || !bytes) return AI_ERR_NULL;
  int rc = validate_fwd(&a->fwd);
  if (rc != AI_OK) return rc;
  *bytes = delta_bytes(a->fwd);
  if (ai::sm100_bwd_supported(a->fwd.dtype, a->fwd.head_dim)) {
    *bytes += ai::sm100_kv_partial_bytes(a->fwd) + ai::sm100_dq_abs_part_bytes(a->fwd);
    if (!fwd_copies(*a)) *bytes += ai::prerot_bytes(a->fwd, nullptr);
  }
  return AI_OK;
}

int ai_attn_bwd(const AiAttnBwdArgs* a, void* stream) {
  if (!a) return AI_ERR_NULL;
  int rc = validate_fwd(&a->fwd);
  if (rc != AI_OK) return rc;
  if (!tensor_ok(a->dout) || !tensor_ok(a->dq) || !tensor_ok(a->dk) || !tensor_ok(a->dv)) return AI_ERR_NULL;
  if (!a->workspace || a->workspace_bytes < delta_bytes(a->fwd)) return AI_ERR_WORKSPACE;
  if ((uintptr_t)a->workspace % 256) return AI_ERR_ALIGN;
  if (a->parts < 0 || a->parts > (AI_BWD_DQ | AI_BWD_DKDV)) return AI_ERR_LAYOUT;
  if (!device_is_sm100()) return AI_ERR_NO_DEVICE;
  const int parts = a->parts ? a->parts : (AI_BWD_DQ | AI_BWD_DKDV);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* delta = static_cast<float*>(a->workspace);
  if (ai::sm100_bwd_supported(a->fwd.dtype, a->fwd.head_dim)) {
    // Workspace: delta, then the dK/dV partial sums of split key tiles when
    // the layout splits some and they fit, then the dQ partials of the abs
    // split when they fit, then the rotated Q and K copies when the
    // forward's are not passed (fwd_rotated) and they fit (else every tile is
    // rotated in shared memory and the abs split is off).
    size_t used = delta_bytes(a->fwd);
    auto take = [&](size_t n) -> float* {
      if (n == 0 || a->workspace_bytes < used + n) return nullptr;
      float* p = reinterpret_cast<float*>(static_cast<char*>(a->workspace) + used);
      used += n;
      return p;
    };
    float* partials = take(ai::sm100_kv_partial_bytes(a->fwd));
    float* dq_part = take(ai::sm100_dq_abs_part_bytes(a->fwd));
    if (fwd_copies(*a))
      return ai::sm100_bwd(*a, delta, a->fwd.workspace, true, partials, dq_part, parts, st, nullptr);
    // (a dK/dV-only call finds the copies its dQ call rotated)
    void* rot = take(ai::prerot_bytes(a->fwd, nullptr));
    return ai::sm100_bwd(*a, delta, rot, !(parts & AI_BWD_DQ), partials, dq_part, parts, st, nullptr);
  }
  if (!(parts & AI_BWD_DQ)) return AI_OK;  // the fp32 / fp16 path did everything in the dQ call
  ai::ProfScope ps(AI_PROF_SIMT, st);
  return launch_status(ai::simt_bwd(*a, delta, st));
}

int ai_attn_read_status(int32_t* dev_status, void* stream, int32_t* host_out) {
  if (!dev_status || !host_out) return AI_ERR_NULL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(host_out, dev_status, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return AI_ERR_LAUNCH;
  if (cudaStreamSynchronize(st) != cudaSuccess) return AI_ERR_LAUNCH;
  if (cudaMemsetAsync(dev_status, 0, sizeof(int32_t), st) != cudaSuccess) return AI_ERR_LAUNCH;
  return AI_OK;
}

const char* ai_attn_strerror(int code) {
  switch (code) {
    case AI_OK: return "ok";
    case AI_ERR_NULL: return "a required pointer is NULL";
    case AI_ERR_SHAPE: return "inconsistent shape (sizes must be > 0 and num_q_heads % num_kv_heads == 0)";
    case AI_ERR_HEAD_DIM: return "head_dim must be 32, 64 or 128";
    case AI_ERR_DTYPE: return "dtype must be bf16, fp16 or fp32";
    case AI_ERR_STRIDE: return "a stride is negative or not a multiple of 16 bytes";
    case AI_ERR_ALIGN: return "a base pointer is misaligned";
    case AI_ERR_LAYOUT: return "layout tables inconsistent with the call (tile sizes or counts)";
    case AI_ERR_WORKSPACE: return "backward workspace missing or smaller than ai_attn_bwd_workspace";
    case AI_ERR_LAUNCH: return "a CUDA launch failed";
    case AI_ERR_NO_DEVICE: return "the current CUDA device is not an sm_100 (B200-class) GPU";
    case AI_ERR_TMA: return "TMA tensor-map encoding rejected a tensor";
    case AI_ERR_NOALLOC_LIMIT:
      return "batch * num_q_heads * seq_len exceeds the fixed scratch of ai_attn_bwd_noalloc (AI_ATTN_NOALLOC_MAX_ROWS)";
    case AI_ERR_DEV_TIMEOUT: return "device: a bounded wait expired";
    case AI_ERR_DEV_BOUNDS: return "device: an index fell outside its table";
    default: return "unknown status";
  }
}

}  // extern "C"
