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

// Counts of one key for QPB queries: QPB / 2 words, 16 bits per query.
template <int QPB>
struct KeyCounts {
  uint32_t w[QPB / 2];
  __device__ __forceinline__ void load(const uint32_t* cnt, int key) {
    if constexpr (QPB == 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(cnt + key * 4);
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else if constexpr (QPB == 4) {
      const uint2 v = *reinterpret_cast<const uint2*>(cnt + key * 2);
      w[0] = v.x; w[1] = v.y;
    } else {
      w[0] = cnt[key];
    }
  }
  __device__ __forceinline__ uint32_t of(int q) const { return (w[q >> 1] >> (16 * (q & 1))) & 0xFFFFu; }
};

template <int QPB>
__global__ void __launch_bounds__(kUnionThreads, 2) union_build_kernel(const int32_t* __restrict__ ids, int topk,
                                                                     int length, int32_t* __restrict__ uent,
                                                                     int32_t* __restrict__ ulen, int ucap) {
  constexpr int kWords = QPB / 2;
  extern __shared__ __align__(16) uint32_t cnt[];  // [kKeysPerPass][kWords]
  __shared__ int warp_sums[2][kUnionThreads / 32];  // alternate chunks: two barriers per chunk
  const int blk = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int32_t* bids = ids + (size_t)blk * QPB * topk;  // the block's QPB index rows
  int32_t* bent = uent + (size_t)blk * ucap;
  const int n_ids = QPB * topk;
  int base_out = 0;  // entries written before this chunk (the same in every thread)
  int buf = 0;
  for (int k0 = 0; k0 < length; k0 += kKeysPerPass) {
    for (int i = tid; i < kKeysPerPass * kWords; i += kUnionThreads) cnt[i] = 0u;
    __syncthreads();
    const int k1 = min(length, k0 + kKeysPerPass);
#pragma unroll 4
    for (int i = tid; i < n_ids; i += kUnionThreads) {
      const int idx = __ldg(bids + i);
      if (idx >= k0 && idx < k1) {
        const int q = i / topk;
        atomicAdd(&cnt[(idx - k0) * kWords + (q >> 1)], 1u << (16 * (q & 1)));
      }
    }
    __syncthreads();
    // keys of this pass in ascending order, kUnionThreads at a time
    for (int kb = 0; kb < kKeysPerPass && k0 + kb < length; kb += kUnionThreads) {
      const int key = kb + tid;
      KeyCounts<QPB> c;
      int m = 0;
      if (k0 + key < length) {
        c.load(cnt, key);
#pragma unroll
        for (int q = 0; q < QPB; ++q) m = max(m, (int)c.of(q));
      }
      // block-wide exclusive scan of m
      int incl = m;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      // warp_sums[buf] was last read two chunks ago, before the barriers of
      // the previous chunk that every thread has passed
      int* ws = warp_sums[buf];
      if (lane == 31) ws[warp] = incl;
      __syncthreads();
      if (warp == 0) {
        int s = ws[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, s, o);
          if (lane >= o) s += v;
        }
        ws[lane] = s;  // inclusive prefix over warps
      }
      __syncthreads();
      const int pos = base_out + (warp > 0 ? ws[warp - 1] : 0) + incl - m;
      base_out += ws[kUnionThreads / 32 - 1];
      buf ^= 1;
      for (int e = 0; e < m; ++e) {
        uint32_t bits = 0;
#pragma unroll
        for (int q = 0; q < QPB; ++q) bits |= (c.of(q) > (uint32_t)e ? 1u : 0u) << q;
        if (pos + e < ucap) bent[pos + e] = (int32_t)((uint32_t)(k0 + key) | (bits << 24));
      }
    }
    __syncthreads();  // the next pass clears the counts
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

template <int QPB>
cudaError_t launch_union_qpb(const int32_t* ids, int topk, int length, int blocks, int32_t* uent, int32_t* ulen,
                             int ucap, cudaStream_t stream) {
  const int smem = kKeysPerPass * (QPB / 2) * 4;
  if (cudaFuncSetAttribute(union_build_kernel<QPB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return cudaErrorInvalidConfiguration;
  union_build_kernel<QPB><<<blocks, kUnionThreads, smem, stream>>>(ids, topk, length, uent, ulen, ucap);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_union_build(const int32_t* ids, int topk, int length, int qpb, int blocks, int32_t* uent,
                               int32_t* ulen, int ucap, cudaStream_t stream) {
  if (blocks <= 0 || length >= (1 << 24)) return cudaErrorInvalidValue;
  switch (qpb) {
    case 2: return launch_union_qpb<2>(ids, topk, length, blocks, uent, ulen, ucap, stream);
    case 4: return launch_union_qpb<4>(ids, topk, length, blocks, uent, ulen, ucap, stream);
    case 8: return launch_union_qpb<8>(ids, topk, length, blocks, uent, ulen, ucap, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace dsa
