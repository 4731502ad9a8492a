// Per-block union of the selected keys, for running 16-, 32- or 64-head
// problems on the pair family at M = 128 (the "union" launch).
//
// A block is 128 / H consecutive queries of one batch row; their q rows,
// output rows and statistics are contiguous, so to the pair kernel a block
// is one 128-head query. It walks the union of the block's selected keys in
// ascending key order; each entry carries the key and one membership bit per
// query of the block. A key that a query selected c times appears in
// max-over-queries(c) entries, entry e holding the queries that selected it
// more than e times, so every selected slot is one (query, entry) pair and
// duplicate slots keep their repeated weight as in the reference
// (dsa/workspace.py:242-318). Invalid indices (< 0 or >= L) select nothing;
// a block with no valid index gets one entry that no query selects.
//
// One CTA per block: counts per (key, query) for a range of kKeysPerPass
// keys at a time in shared memory (16-bit, two queries per word), then a
// block-wide exclusive scan of the per-key entry counts gives each key's
// output position.
#include "dsa_common.cuh"

namespace dsa {
namespace {

constexpr int kUnionThreads = 1024;
constexpr int kKeysPerPass = 4096;
constexpr int kMaxQpb = 8;  // queries per block (H = 16)

__device__ __forceinline__ uint32_t count_of(const uint32_t* cnt, int key, int q, int qpb) {
  return (cnt[key * (qpb / 2) + (q >> 1)] >> (16 * (q & 1))) & 0xFFFFu;
}

__global__ void __launch_bounds__(kUnionThreads) union_build_kernel(const int32_t* __restrict__ ids, int topk,
                                                                     int length, int qpb, int32_t* __restrict__ uent,
                                                                     int32_t* __restrict__ ulen, int ucap) {
  extern __shared__ uint32_t cnt[];  // [kKeysPerPass][qpb / 2]
  __shared__ int warp_sums[kUnionThreads / 32];
  __shared__ int base_out;
  const int blk = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int32_t* bids = ids + (size_t)blk * qpb * topk;  // the block's qpb index rows
  int32_t* bent = uent + (size_t)blk * ucap;
  const int words = kKeysPerPass * (qpb / 2);
  if (tid == 0) base_out = 0;
  for (int k0 = 0; k0 < length; k0 += kKeysPerPass) {
    for (int i = tid; i < words; i += kUnionThreads) cnt[i] = 0u;
    __syncthreads();
    for (int i = tid; i < qpb * topk; i += kUnionThreads) {
      const int idx = __ldg(bids + i);
      if (idx >= k0 && idx < length && idx < k0 + kKeysPerPass) {
        const int q = i / topk;
        atomicAdd(&cnt[(idx - k0) * (qpb / 2) + (q >> 1)], 1u << (16 * (q & 1)));
      }
    }
    __syncthreads();
    // keys of this pass in ascending order, kUnionThreads at a time
    for (int kb = 0; kb < kKeysPerPass && k0 + kb < length; kb += kUnionThreads) {
      const int key = kb + tid;
      int m = 0;
      if (k0 + key < length) {
        for (int q = 0; q < qpb; ++q) m = max(m, (int)count_of(cnt, key, q, qpb));
      }
      // block-wide exclusive scan of m
      int incl = m;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (lane == 31) warp_sums[warp] = incl;
      __syncthreads();
      if (warp == 0) {
        int s = warp_sums[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, s, o);
          if (lane >= o) s += v;
        }
        warp_sums[lane] = s;  // inclusive prefix over warps
      }
      __syncthreads();
      const int pos = base_out + (warp > 0 ? warp_sums[warp - 1] : 0) + incl - m;
      for (int e = 0; e < m; ++e) {
        uint32_t bits = 0;
        for (int q = 0; q < qpb; ++q) bits |= (count_of(cnt, key, q, qpb) > (uint32_t)e ? 1u : 0u) << q;
        if (pos + e < ucap) bent[pos + e] = (int32_t)((uint32_t)(k0 + key) | (bits << 24));
      }
      __syncthreads();
      if (tid == 0) base_out += warp_sums[kUnionThreads / 32 - 1];
      __syncthreads();
    }
  }
  // a block whose queries have no valid index still gets one (fully masked)
  // entry, so that its item has a tile and writes zeros like any other row
  // without a valid index
  if (tid == 0) {
    if (base_out == 0) {
      bent[0] = 0;
      base_out = 1;
    }
    ulen[blk] = min(base_out, ucap);
  }
}

}  // namespace

uint64_t union_smem_bytes(int qpb) { return (uint64_t)kKeysPerPass * (uint64_t)(qpb / 2) * 4u; }

cudaError_t launch_union_build(const int32_t* ids, int topk, int length, int qpb, int blocks, int32_t* uent,
                               int32_t* ulen, int ucap, cudaStream_t stream) {
  if (qpb < 2 || qpb > kMaxQpb || (qpb & 1) || blocks <= 0 || length >= (1 << 24)) return cudaErrorInvalidValue;
  const int smem = (int)union_smem_bytes(qpb);
  if (cudaFuncSetAttribute(union_build_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return cudaErrorInvalidConfiguration;
  union_build_kernel<<<blocks, kUnionThreads, smem, stream>>>(ids, topk, length, qpb, uent, ulen, ucap);
  return cudaGetLastError();
}

}  // namespace dsa
