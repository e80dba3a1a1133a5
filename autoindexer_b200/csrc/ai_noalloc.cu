// ai_attn_bwd_noalloc: the backward pass for callers that cannot allocate
// device memory.
//
// Some hosts of this library have no way to hand it a scratch buffer: a
// runtime whose memory pool is owned by another component and exposes only the
// tensors it manages, a plugin that may only touch the buffers it is given,
// or code running where cudaMalloc is forbidden after start-up.  ai_attn_bwd
// needs B * Hq * T floats of scratch (the per-row dO.O sums); this entry point
// takes them from a fixed array in the library's own device memory instead.
//
// The array below is a file-scope __device__ array of kNoAllocScratchFloats
// floats (16 MiB).  Every GPU that loads the library holds it until the
// process exits.  In host code its name is only a host-side stand-in: its
// device address is looked up with cudaGetSymbolAddress, once per device, by
// the first call made with that device current (so make that first call
// before any stream capture).  Every call shares the array and it keeps the
// last call's contents; the kernels overwrite every entry they read, so
// nothing needs clearing.  Calls that overlap on the GPU (different streams,
// or different host threads on one device) race on the array.
//
// What the array holds: the B * Hq * T row sums first; when the caller did
// not pass the forward's rotated Q/K copies (fwd_rotated = 0) and they fit in
// the rest of the array (B * Hq * T up to about 50,000 at head_dim 128 with
// four query heads per KV head), the once-rotated Q/K copies as well, exactly
// as ai_attn_bwd places them in a workspace of that size.  Above that the kernels rotate each tile in shared
// memory instead (same results to rounding, slower), so the speed of this
// entry point drops at a shape-dependent size and the race between
// overlapping calls covers the copies too when they are there.

#include <cuda_runtime.h>

#include <mutex>

#include "../../include/ai_attn.h"
#include "ai_kernels.h"

namespace {

constexpr size_t kNoAllocScratchFloats = AI_ATTN_NOALLOC_MAX_ROWS;  // 16 MiB of fp32

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices];
std::mutex g_scratch_mu;

// Device address of g_noalloc_scratch on the current device (looked up once).
int scratch_for_current_device(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return AI_ERR_NO_DEVICE;
  // The library holds sm_100a code only: on any other part the symbol does
  // not exist there, so say so before looking it up.
  int major = -1;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10) {
    cudaGetLastError();
    return AI_ERR_NO_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();  // leave no pending error for the next launch check of this thread
      return AI_ERR_NO_DEVICE;
    }
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return AI_OK;
}

}  // namespace

extern "C" int ai_attn_bwd_noalloc(const AiAttnBwdArgs* a, void* stream) {
  if (!a) return AI_ERR_NULL;
  const AiAttnFwdArgs& f = a->fwd;
  if (f.batch <= 0 || f.num_q_heads <= 0 || f.seq_len <= 0) return AI_ERR_SHAPE;
  const size_t rows = (size_t)f.batch * (size_t)f.num_q_heads * (size_t)f.seq_len;
  if (rows > kNoAllocScratchFloats) return AI_ERR_NOALLOC_LIMIT;
  float* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc != AI_OK) return rc;
  AiAttnBwdArgs b = *a;
  b.workspace = scratch;
  b.workspace_bytes = kNoAllocScratchFloats * sizeof(float);
  return ai_attn_bwd(&b, stream);
}
