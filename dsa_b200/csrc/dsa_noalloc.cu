// Allocation-free variant of the split-KV forward (dsa_sparse_mla_fwd_noalloc).
//
// Who needs it: callers that must not allocate device memory on the call
// path. A serving engine that reserves nearly all of HBM for its own pool
// at start-up leaves cudaMalloc nothing to hand out; cudaFree synchronises
// the whole device and would stall every other stream; and an FFI host
// (ctypes, cgo, JNI) that only owns the input and output buffers may have
// no device allocator at all. Such callers pass inputs and outputs only.
//
// How: the split-KV partials (FP32 numerators, maxima and sums) live in one
// file-scope __device__ array of DSA_NOALLOC_SCRATCH_BYTES instead of a
// caller-provided workspace. Every GPU that loads this library holds that
// array until the process exits. Host code cannot use the array's name as
// a device address (on the host it names a stand-in object), so the first
// call on each device, with that device current, resolves the address with
// cudaGetSymbolAddress and caches it; make that first call before any stream
// capture. Nothing here calls cudaMalloc, cudaFree or an allocating library.
//
// Sharing rules: every call uses the same array and leaves the last call's
// partials in it. The kernels write every partial element before the merge
// reads it, so nothing has to be cleared between calls; but two calls whose
// kernels overlap on the GPU (different streams, no ordering) race on the
// array and corrupt each other's results.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/dsa_b200.h"
#include "dsa_common.cuh"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[DSA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

constexpr uint64_t kAlignNa = 256;
inline uint64_t align_up_na(uint64_t x) { return (x + kAlignNa - 1) / kAlignNa * kAlignNa; }

// Device address of the scratch array on the current device (set-up on
// first use per device).
int scratch_for_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return DSA_STATUS_CUDA_ERROR;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr)
      return DSA_STATUS_CUDA_ERROR;
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return DSA_STATUS_OK;
}

bool aligned16_na(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int dsa_sparse_mla_fwd_noalloc(const dsa_fwd_args_t* a, void* stream) {
  if (a == nullptr) return DSA_STATUS_BAD_ARGUMENT;
  if (!a->q || !a->kv || !a->q_rope || !a->k_rope || !a->indices || !a->output ||
      !a->softmax_max || !a->softmax_sum)
    return DSA_STATUS_BAD_ARGUMENT;
  if (!aligned16_na(a->q) || !aligned16_na(a->kv) || !aligned16_na(a->q_rope) ||
      !aligned16_na(a->k_rope) || !aligned16_na(a->output))
    return DSA_STATUS_BAD_ARGUMENT;

  // This variant always runs the generic warp-MMA family; AUTO takes the
  // shape-only default entry and keeps its split.
  dsa_launch_t e = a->launch;
  if (e.family == DSA_FAMILY_AUTO) {
    int st = dsa_default_launch(a->batch, a->queries, a->heads, a->length, a->topk, &e);
    if (st != DSA_STATUS_OK) return st;
    if (e.family != DSA_FAMILY_WARP_MMA) {
      e.family = DSA_FAMILY_WARP_MMA;
      e.heads_per_cta = 16;
      e.keys_per_tile = 32;
      const int64_t tiles = (a->topk + 31) / 32;
      if (e.split > tiles) e.split = (int32_t)tiles;
    }
  }
  if (e.family != DSA_FAMILY_WARP_MMA) return DSA_STATUS_UNSUPPORTED;
  int st = dsa_check_launch(a->batch, a->queries, a->heads, a->length, a->topk, &e);
  if (st != DSA_STATUS_OK) return st;

  const int64_t tokens = a->batch * a->queries;
  char* scratch = nullptr;
  uint64_t num_off = 0, max_off = 0, sum_off = 0;
  if (e.split > 1) {
    const uint64_t rows = (uint64_t)tokens * (uint64_t)e.split * (uint64_t)a->heads;
    max_off = align_up_na(rows * dsa::kDimLatent * sizeof(float));
    sum_off = max_off + align_up_na(rows * sizeof(float));
    const uint64_t need = sum_off + align_up_na(rows * sizeof(float));
    if (need > (uint64_t)DSA_NOALLOC_SCRATCH_BYTES) return DSA_STATUS_WORKSPACE_TOO_SMALL;
    void* base = nullptr;
    st = scratch_for_current_device(&base);
    if (st != DSA_STATUS_OK) return st;
    scratch = static_cast<char*>(base);
  }

  dsa::FwdParams p;
  std::memset(&p, 0, sizeof(p));
  p.q = static_cast<const __nv_bfloat16*>(a->q);
  p.kv = static_cast<const __nv_bfloat16*>(a->kv);
  p.q_rope = static_cast<const __nv_bfloat16*>(a->q_rope);
  p.k_rope = static_cast<const __nv_bfloat16*>(a->k_rope);
  p.ids = a->indices;
  p.out = static_cast<__nv_bfloat16*>(a->output);
  p.out_max = a->softmax_max;
  p.out_sum = a->softmax_sum;
  if (e.split > 1) {
    p.part_num = reinterpret_cast<float*>(scratch + num_off);
    p.part_max = reinterpret_cast<float*>(scratch + max_off);
    p.part_sum = reinterpret_cast<float*>(scratch + sum_off);
  }
  p.status = a->status;
  p.batch = (int)a->batch;
  p.queries = (int)a->queries;
  p.heads = (int)a->heads;
  p.length = (int)a->length;
  p.topk = (int)a->topk;
  p.tokens = (int)tokens;
  p.split = e.split;
  p.keys_per_tile = e.keys_per_tile;
  p.heads_per_cta = e.heads_per_cta;
  if (!dsa::fill_scale(a->scale, p)) return DSA_STATUS_BAD_ARGUMENT;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dsa::launch_fwd_warp_mma(p, s) != cudaSuccess) return DSA_STATUS_LAUNCH_FAILED;
  if (e.split > 1 && dsa::launch_merge(p.part_num, p.part_max, p.part_sum, p.out, p.out_max,
                                       p.out_sum, p.tokens, p.heads, p.split, s) != cudaSuccess)
    return DSA_STATUS_LAUNCH_FAILED;
  return DSA_STATUS_OK;
}
