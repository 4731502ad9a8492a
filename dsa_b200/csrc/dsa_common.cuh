// Shared definitions for the sm_100a sparse-MLA forward kernels.
//
// Layout facts used everywhere (reference contract, dsa/api.py:18-38):
//   q      [T, H, 512]  bf16, T = B*SQ flattened tokens (batch-major)
//   q_rope [T, H, 64]   bf16
//   kv     [B, L, 512]  bf16 (the size-1 head axis is dropped)
//   k_rope [B, L, 64]   bf16
//   ids    [T, TOPK]    int32
//   out    [T, H, 512]  bf16; max/sum [T, H] fp32 (== [B,1,SQ,H] contiguous)
//   split-KV partials (dsa/api.py:111-113): numerator [T, S, H, 512] fp32,
//   partial max/sum [T, S, H] fp32.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dsa {

constexpr int kDimLatent = 512;
constexpr int kDimRope = 64;
constexpr int kDimQK = kDimLatent + kDimRope;  // 576
constexpr float kNegFltMax = -3.4028234663852886e38f;

// Device error bits OR-ed into the optional status word.
constexpr int kErrTimeout = 1;
constexpr int kErrBadLaunch = 2;
constexpr int kErrBounds = 4;  // a check of the bounds-checking build failed

// The bounds-checking build (-DDSA_BOUNDS_CHECK, libdsa_b200_checked.so)
// checks every gathered row index, batch row, shared-memory stage
// destination and tensor-memory column it uses; a failed check ORs
// kErrBounds into the status word and redirects the access to a safe
// address (row 0, the stage's first byte, column 0) instead of trapping.
// In the regular build the checks compile to nothing.
#ifdef DSA_BOUNDS_CHECK
constexpr bool kBoundsCheck = true;
#else
constexpr bool kBoundsCheck = false;
#endif

struct FwdParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* kv;
  const __nv_bfloat16* q_rope;
  const __nv_bfloat16* k_rope;
  const int32_t* ids;
  __nv_bfloat16* out;     // split == 1
  float* out_max;         // split == 1
  float* out_sum;         // split == 1
  float* part_num;        // split > 1: [T, S, H, 512]
  float* part_max;        // split > 1: [T, S, H]
  float* part_sum;        // split > 1: [T, S, H]
  // Union launch of the pair family (heads = 128 rows of 128 / H queries):
  // per block, `ulen` entries of key | (query membership << 24) at
  // uent[block * ucap ...]; row r of a block belongs to query r >> u_row_shift.
  const int32_t* uent;
  const int32_t* ulen;
  int ucap;
  int u_row_shift;
  int32_t* status;
  int batch, queries, heads, length, topk;
  int tokens;             // batch * queries
  int split;
  int keys_per_tile;
  int heads_per_cta;
  // Scores are divided by scale_div (= 1/scale; exactly 24 for the
  // reference's 1/sqrt(576)); the exp2-form families use
  // scale_log2 = log2(e) / scale_div.
  float scale_div;
  float scale_log2;
  // Bound of each device-side wait of the split-V family in ns (0: the
  // built-in 2 s); wait_test != 0 makes that family's first CTA wait on a
  // barrier nothing arrives at, so the bound runs out (failure-path test).
  unsigned long long wait_limit_ns;
  int wait_test;
};

// Host: fill scale_div / scale_log2 from the ABI's scale (0 = the
// reference's 1/sqrt(576), divisor exactly 24; otherwise (0, 0.5], which
// keeps -FLT_MAX * scale_log2 finite for the masked-key arithmetic).
// Returns false for a scale outside that range.
inline bool fill_scale(float scale, FwdParams& p) {
  if (scale == 0.f) {
    p.scale_div = 24.0f;
  } else {
    if (!(scale > 0.f && scale <= 0.5f)) return false;
    p.scale_div = (float)(1.0 / (double)scale);
  }
  p.scale_log2 = 1.4426950408889634f / p.scale_div;
  return true;
}

// Final statistics of one (token, head) row from the running max m (raw,
// unscaled scores) and the sum l: softmax_max = m / scale_div, or -inf for a
// row without a valid index (l == 0); the output row is 0 there.
__device__ __forceinline__ float final_max(float m_raw, float l, float scale_div) {
  return l > 0.f ? __fdiv_rn(m_raw, scale_div) : -INFINITY;
}

// Split bounds in whole tiles, uneven when the tile count does not divide
// (the tile-count split of dsa/ragged.py:141-143, generalised to a ragged
// last tile): split s covers keys [begin, end).
__host__ __device__ inline void split_bounds(int topk, int bn, int split, int s, int* begin,
                                             int* end) {
  int tiles = (topk + bn - 1) / bn;
  int t0 = (int)(((long long)s * tiles) / split);
  int t1 = (int)(((long long)(s + 1) * tiles) / split);
  *begin = min(t0 * bn, topk);
  *end = min(t1 * bn, topk);
}

// ---------------------------------------------------------------------------
// Small PTX wrappers (warp-level MMA path).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
// Every cp.async of this thread issued so far (committed or not) has completed.
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
// Arrive on the mbarrier once every cp.async this thread issued so far has
// completed; the arrival counts toward the barrier's expected count (noinc).
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void report_error(int32_t* status, int bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// Bounds-checking build: `v` inside [0, n), else kErrBounds and 0.
__device__ __forceinline__ int checked_index(int v, int n, int32_t* status) {
  if (kBoundsCheck && (v < 0 || v >= n)) {
    report_error(status, kErrBounds);
    return 0;
  }
  return v;
}
// Bounds-checking build: a shared-memory destination of `bytes` inside
// [lo, lo + size), else kErrBounds and lo.
__device__ __forceinline__ uint32_t checked_smem(uint32_t addr, uint32_t bytes, uint32_t lo, uint32_t size,
                                                 int32_t* status) {
  if (kBoundsCheck && (addr < lo || addr + bytes > lo + size)) {
    report_error(status, kErrBounds);
    return lo;
  }
  return addr;
}
// Bounds-checking build: `ncols` tensor-memory columns from `col` inside
// the allocation's `cols` columns (column = low 16 bits of the address),
// else kErrBounds and column 0 of the same lane.
__device__ __forceinline__ uint32_t checked_tmem(uint32_t taddr, uint32_t tbase, uint32_t ncols, uint32_t cols,
                                                 int32_t* status) {
  if (kBoundsCheck && ((taddr & 0xFFFFu) < (tbase & 0xFFFFu) || (taddr & 0xFFFFu) + ncols > (tbase & 0xFFFFu) + cols)) {
    report_error(status, kErrBounds);
    return (taddr & 0xFFFF0000u) | (tbase & 0xFFFFu);
  }
  return taddr;
}

// Launchers (each returns a cudaError_t from the launch).
cudaError_t launch_fwd_warp_mma(const FwdParams& p, cudaStream_t stream);
cudaError_t launch_fwd_umma(const FwdParams& p, cudaStream_t stream);
// CTAs of the umma family that fit on the current device at once (-1 on error).
int umma_max_ctas();
// Whether the umma family merges `split` > 1 partials inside one launch
// (clusters of `split` CTAs fit on the device; at most 16).
bool umma_cluster_merge(int split);
// Largest split <= `split` (and <= 16) whose clusters fit `clusters` at once
// on the device; `split` capped at 16 when none does.
int umma_cluster_split(long long clusters, int split);
cudaError_t launch_fwd_pair(const FwdParams& p, cudaStream_t stream);
// CTAs of the pair family (two per cluster) resident at once (-1 on error).
int pair_max_ctas();
cudaError_t launch_fwd_stream(const FwdParams& p, cudaStream_t stream);
cudaError_t launch_fwd_keys(const FwdParams& p, cudaStream_t stream);
cudaError_t launch_fwd_pair_union(const FwdParams& p, cudaStream_t stream);
cudaError_t launch_union_build(const int32_t* ids, int topk, int length, int qpb, int blocks, int32_t* uent,
                               int32_t* ulen, int ucap, cudaStream_t stream);
// CTAs of the stream family resident at once (-1 on error).
int stream_max_ctas();
bool stream_cluster_merge(int split);
int keys_max_ctas();
cudaError_t launch_paged_rows(const int32_t* ids, const int32_t* block_table, const int32_t* seq_lens, int32_t* rows,
                              long long n, int per_batch, int max_blocks, int block_size, int num_blocks,
                              cudaStream_t stream);
cudaError_t launch_fp8_gather(const uint8_t* cache, const int32_t* ids, __nv_bfloat16* kv_out, __nv_bfloat16* kr_out,
                              int32_t* ids_out, long long rows, int topk, int queries, int length,
                              cudaStream_t stream);
cudaError_t launch_indexer_logits(const __nv_bfloat16* q, const __nv_bfloat16* k, const float* w, const int32_t* lens,
                                  float* scores, int32_t* status, int batch, int queries, int heads, int length,
                                  cudaStream_t stream);
cudaError_t launch_topk(const float* scores, const int32_t* lens, int32_t* out, long long rows, int length, int topk,
                        cudaStream_t stream);
cudaError_t launch_merge(const float* num, const float* pmax, const float* psum,
                         __nv_bfloat16* out, float* omax, float* osum, int tokens, int heads,
                         int split, cudaStream_t stream);

}  // namespace dsa
