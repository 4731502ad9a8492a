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
// keys at a time in shared memory (16-bit, two queries per word), then one
// block-wide exclusive scan per pass of the per-key entry counts (each thread
// owns four consecutive keys) gives each key's output position. The block's
// indices are read once into registers when they fit (16 per thread, two
// 16-bit keys per register, for L < 65535) and reused by every pass.
#include "dsa_common.cuh"

namespace dsa {
namespace {

constexpr int kUnionThreads = 1024;
constexpr int kKeysPerThread = 4;
constexpr int kKeysPerPass = kUnionThreads * kKeysPerThread;  // 4096
constexpr int kIdsCached = 16;                                // indices per thread kept in registers
constexpr uint32_t kNoKey = 0xFFFFu;                          // a cached index that selects nothing

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
  // max over the queries' 16-bit counts (per-halfword maxima, then the halves)
  __device__ __forceinline__ int max_count() const {
    uint32_t v = w[0];
#pragma unroll
    for (int k = 1; k < QPB / 2; ++k) v = __vmaxu2(v, w[k]);
    return (int)max(v & 0xFFFFu, v >> 16);
  }
  // membership bits of entry e: query q's bit is set when its count exceeds e
  __device__ __forceinline__ uint32_t bits_above(uint32_t e) const {
    const uint32_t ee = e | (e << 16);
    uint32_t bits = 0;
#pragma unroll
    for (int k = 0; k < QPB / 2; ++k) {
      const uint32_t gt = __vcmpgtu2(w[k], ee);  // 0xFFFF per halfword where count > e
      bits |= ((gt & 1u) | ((gt >> 15) & 2u)) << (2 * k);
    }
    return bits;
  }
};

// Count index slot j (query q = j / topk of the block) for key idx when it
// lies in this pass's keys [k0, k1).
template <int QPB>
__device__ __forceinline__ void count_slot(uint32_t* cnt, int idx, int q, int k0, int k1) {
  constexpr int kWords = QPB / 2;
  if (idx >= k0 && idx < k1) atomicAdd(&cnt[(idx - k0) * kWords + (q >> 1)], 1u << (16 * (q & 1)));
}

template <int QPB>
__global__ void __launch_bounds__(kUnionThreads, 2) union_build_kernel(const int32_t* __restrict__ ids, int topk,
                                                                     int length, int32_t* __restrict__ uent,
                                                                     int32_t* __restrict__ ulen, int ucap) {
  constexpr int kWords = QPB / 2;
  extern __shared__ __align__(16) uint32_t cnt[];  // [kKeysPerPass][kWords]
  __shared__ int warp_sums[kUnionThreads / 32];
  const int blk = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int32_t* bids = ids + (size_t)blk * QPB * topk;  // the block's QPB index rows
  int32_t* bent = uent + (size_t)blk * ucap;
  const int n_ids = QPB * topk;
  const bool cached = n_ids <= kIdsCached * kUnionThreads && length < (int)kNoKey;
  // cached path: thread tid holds slots tid % kPerQuery + i * kPerQuery of
  // query tid / kPerQuery, so a warp reads 32 consecutive indices of one row
  constexpr int kPerQuery = kUnionThreads / QPB;
  const int cq = tid / kPerQuery;
  uint32_t idr[kIdsCached / 2];  // two 16-bit keys per register
  if (cached) {
#pragma unroll
    for (int i = 0; i < kIdsCached; ++i) {
      const int j = tid % kPerQuery + i * kPerQuery;
      const int idx = j < topk ? __ldg(bids + (size_t)cq * topk + j) : -1;
      const uint32_t k = (idx >= 0 && idx < length) ? (uint32_t)idx : kNoKey;
      if (i & 1)
        idr[i >> 1] |= k << 16;
      else
        idr[i >> 1] = k;
    }
  }
  int base_out = 0;  // entries written before this pass (the same in every thread)
  for (int k0 = 0; k0 < length; k0 += kKeysPerPass) {
    uint4* const c4 = reinterpret_cast<uint4*>(cnt);
    for (int i = tid; i < kKeysPerPass * kWords / 4; i += kUnionThreads) c4[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
    const int k1 = min(length, k0 + kKeysPerPass);
    if (cached) {
#pragma unroll
      for (int i = 0; i < kIdsCached; ++i)
        count_slot<QPB>(cnt, (int)((idr[i >> 1] >> (16 * (i & 1))) & 0xFFFFu), cq, k0, k1);
    } else {
#pragma unroll 4
      for (int j = tid; j < n_ids; j += kUnionThreads) count_slot<QPB>(cnt, __ldg(bids + j), j / topk, k0, k1);
    }
    __syncthreads();
    // keys k0 + 4 tid .. 4 tid + 3 of this pass
    int tot = 0;
#pragma unroll
    for (int i = 0; i < kKeysPerThread; ++i) {
      const int key = kKeysPerThread * tid + i;
      if (k0 + key < length) {
        KeyCounts<QPB> c;
        c.load(cnt, key);
        tot += c.max_count();
      }
    }
    // block-wide exclusive scan of the threads' entry counts
    int incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int sw = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, sw, o);
        if (lane >= o) sw += v;
      }
      warp_sums[lane] = sw;  // inclusive prefix over warps
    }
    __syncthreads();
    int pos = base_out + (warp > 0 ? warp_sums[warp - 1] : 0) + incl - tot;
    base_out += warp_sums[kUnionThreads / 32 - 1];
#pragma unroll
    for (int i = 0; i < kKeysPerThread; ++i) {
      const int key = kKeysPerThread * tid + i;
      if (k0 + key >= length) break;
      KeyCounts<QPB> c;  // read again: fewer live registers across the scan
      c.load(cnt, key);
      const int mi = c.max_count();
      for (int e = 0; e < mi; ++e) {
        const uint32_t bits = c.bits_above((uint32_t)e);
        if (pos + e < ucap)
          bent[pos + e] = (int32_t)((uint32_t)(k0 + key) | (bits << 24));
      }
      pos += mi;
    }
    __syncthreads();  // the next pass clears the counts and reuses warp_sums
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
