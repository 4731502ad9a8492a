// Lightning indexer and top-k: the stage that produces the indices the
// sparse-MLA forward consumes (DeepSeek-V3.2's DSA indexer; the reference
// takes the indices as given and leaves the indexer and top-k out,
// README.md:19-20, DSA从原理到实现.md:625).
//
// For every query t (B*SQ flattened) and key j < L of its batch row:
//   score[t][j] = sum_h w[t][h] * relu(q[t][h] . k[b][j])      (d = 128)
// and the indices are the TOPK keys j < len[t] with the largest scores,
// ties to the smaller key, in ascending key order, padded with -1 when
// fewer than TOPK keys are valid.
//
// indexer_logits_kernel (tcgen05): one CTA per (batch row, group of G =
// 256 / HI consecutive queries, chunk of key tiles). The group's queries
// and heads are the N = 256 rows of the B operand (in shared memory for the
// whole CTA), a tile of 128 keys the A operand, so D = K . Q^T puts one key
// per TMEM lane: every epilogue thread owns one key and reduces its 256
// columns (G queries x HI heads) by itself, no cross-thread reduction.
//   warps 0-3  load Q and w, then the epilogue (TMEM lane quadrant = warp);
//   warp 4     loads key tiles (16-byte cp.async, two tiles in flight, three stages);
//   warp 5     issues the 8 MMAs (M=128, N=256, K=16) per tile into one of two
//              256-column D buffers.
// topk_kernel: one CTA per query row, radix select of the TOPK-th largest
// score over the order-preserving unsigned image of the FP32 scores (4
// passes of 8 bits), then a block-wide scan writes the selected keys in
// ascending key order. Every wait is bounded and reports through the
// status word.
#include "umma_ptx.cuh"

namespace dsa {
namespace {

using namespace umma;

constexpr int kIxD = 128;          // index head dim
constexpr int kIxN = 256;          // group rows: G queries x HI heads
constexpr int kIxKeys = 128;       // keys per tile (MMA M)
constexpr int kIxStages = 3;
constexpr int kIxThreads = 192;
constexpr int kIxEpiWarps = 4;
constexpr int kIxLoadWarp = 4;
constexpr int kIxMmaWarp = 5;
constexpr uint32_t kIxQBlk = (uint32_t)kIxN * 128u;      // 256 rows x 64 dims (SW128) = 32 KB
constexpr uint32_t kIxKBlk = (uint32_t)kIxKeys * 128u;   // 128 rows x 64 dims = 16 KB
constexpr uint32_t kIxOffQ = 0;
constexpr uint32_t kIxOffK = kIxOffQ + 2u * kIxQBlk;      // 64 KB
constexpr uint32_t kIxStage = 2u * kIxKBlk;              // 32 KB
constexpr uint32_t kIxOffW = kIxOffK + kIxStages * kIxStage;
constexpr uint32_t kIxOffBar = kIxOffW + kIxN * 4u;
enum IxBar { ixFull0 = 0, ixEmpty0 = ixFull0 + kIxStages, ixDFull0 = ixEmpty0 + kIxStages, ixDFree0 = ixDFull0 + 2,
             ixQFull = ixDFree0 + 2, ixDrain, ixBarCount };
constexpr uint32_t kIxOffTmem = kIxOffBar + ixBarCount * 8u;
constexpr uint32_t kIxOffAbort = kIxOffTmem + 8u;
constexpr uint32_t kIxSmem = kIxOffAbort + 8u + 1024u;
static_assert(kIxOffK % 1024 == 0 && kIxStage % 1024 == 0, "swizzle atoms");
static_assert(kIxSmem <= 232448, "shared memory budget");

struct IxParams {
  const __nv_bfloat16* q;   // [T, HI, 128]
  const __nv_bfloat16* k;   // [B, L, 128]
  const float* w;           // [T, HI]
  const int32_t* lens;      // [T] or null
  float* scores;            // [T, L]
  int32_t* status;
  int batch, queries, heads, length;
  int groups;               // query groups per batch row
  int chunk_tiles;          // key tiles per CTA
  int chunks;               // chunks per group
};

// Offset of 16-byte chunk jj (0..7) of row r in a 128-byte-swizzled K-major block.
__device__ __forceinline__ uint32_t sw128(int r, int jj) {
  return (uint32_t)(r >> 3) * 1024u + (uint32_t)(r & 7) * 128u + (uint32_t)((jj ^ (r & 7)) * 16);
}

__device__ __forceinline__ bool ix_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok) != 0;
}

__global__ void __launch_bounds__(kIxThreads, 1) indexer_logits_kernel(const IxParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const sbase = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sbase + kIxOffAbort);
  auto bar = [&](int i) -> uint32_t { return base + kIxOffBar + 8u * (uint32_t)i; };

  // the CTA's (batch row, query group, key chunk)
  const int item = blockIdx.x;
  const int kc = item % p.chunks;
  const int gi = (item / p.chunks) % p.groups;
  const int b = item / (p.chunks * p.groups);
  const int G = kIxN / p.heads;
  const int s0 = gi * G;
  const int ng = min(G, p.queries - s0);  // queries of this group
  const int t0 = b * p.queries + s0;      // first flattened query
  // keys any query of the group can select
  int kmax = p.length;
  if (p.lens != nullptr) {
    kmax = 0;
    for (int g = 0; g < ng; ++g) kmax = max(kmax, min(__ldg(p.lens + t0 + g), p.length));
  }
  const int ntiles = (kmax + kIxKeys - 1) / kIxKeys;
  const int tile0 = kc * p.chunk_tiles;
  const int tiles = max(0, min(ntiles - tile0, p.chunk_tiles));
  if (tiles == 0) return;  // uniform across the CTA: nothing to score

  if (threadIdx.x == 0) {
    for (int s = 0; s < kIxStages; ++s) {
      mbar_init(bar(ixFull0 + s), 1);
      mbar_init(bar(ixEmpty0 + s), 1);
    }
    for (int d = 0; d < 2; ++d) {
      mbar_init(bar(ixDFull0 + d), 1);
      mbar_init(bar(ixDFree0 + d), kIxEpiWarps);
    }
    mbar_init(bar(ixQFull), kIxEpiWarps);
    mbar_init(bar(ixDrain), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(base + kIxOffTmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sbase + kIxOffTmem);
  bool ok = true;

  if (warp < kIxEpiWarps) {
    // ---- the group's Q rows (row n = query g * HI + head h) and weights ----
    const uint32_t qs = base + kIxOffQ;
    for (int c = threadIdx.x; c < kIxN * 16; c += 128) {  // 16 chunks of 16 B per row
      const int n = c >> 4, j16 = c & 15;
      const int g = n / p.heads, h = n % p.heads;
      const int t = t0 + min(g, ng - 1);  // rows of absent queries repeat a real one (not written out)
      cp_async_16(qs + (uint32_t)(j16 >> 3) * kIxQBlk + sw128(n, j16 & 7),
                  p.q + ((size_t)t * p.heads + h) * kIxD + j16 * 8);
    }
    float* const ws = reinterpret_cast<float*>(sbase + kIxOffW);
    for (int n = threadIdx.x; n < kIxN; n += 128) {
      const int g = n / p.heads, h = n % p.heads;
      ws[n] = g < ng ? __ldg(p.w + (size_t)(t0 + g) * p.heads + h) : 0.f;
    }
    cp_async_commit();
    cp_async_wait<0>();
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(ixQFull));
    // every epilogue warp's weights are in shared memory once all four arrived
    ok = ix_wait(bar(ixQFull), 0u, abort_flag);
    // ---- epilogue: this thread's key, every query of the group ----
    const int row = warp * 32 + lane;
    const uint32_t t_lane = (uint32_t)(warp * 32) << 16;
    for (int j = 0; j < tiles && ok; ++j) {
      const uint32_t d = (uint32_t)j & 1u;
      if (!(ok = ix_wait(bar(ixDFull0 + d), (uint32_t)(j >> 1) & 1u, abort_flag))) break;
      tc_fence_after();
      const int key = (tile0 + j) * kIxKeys + row;
      const bool store = key < p.length;
      float cur = 0.f;  // running sum of the current query's heads
#pragma unroll 1
      for (int cb = 0; cb < kIxN; cb += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + t_lane + d * 256u + (uint32_t)cb, v);
        tmem_wait_ld();
        if (p.heads >= 32) {  // the 32 columns are heads of one query
          float part = 0.f;
#pragma unroll
          for (int k = 0; k < 32; ++k) part = fmaf(fmaxf(__uint_as_float(v[k]), 0.f), ws[cb + k], part);
          cur += part;
          if ((cb + 32) % p.heads == 0) {
            const int g = cb / p.heads;
            if (store && g < ng) p.scores[(size_t)(t0 + g) * p.length + key] = cur;
            cur = 0.f;
          }
        } else {  // 16 heads: the 32 columns are two queries
          float p0 = 0.f, p1 = 0.f;
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            p0 = fmaf(fmaxf(__uint_as_float(v[k]), 0.f), ws[cb + k], p0);
            p1 = fmaf(fmaxf(__uint_as_float(v[16 + k]), 0.f), ws[cb + 16 + k], p1);
          }
          const int g = cb / 16;
          if (store && g < ng) p.scores[(size_t)(t0 + g) * p.length + key] = p0;
          if (store && g + 1 < ng) p.scores[(size_t)(t0 + g + 1) * p.length + key] = p1;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(ixDFree0 + d));
    }
  } else if (warp == kIxLoadWarp) {
    // ---- key tiles: 128 rows x 256 B, two tiles in flight ----
    const __nv_bfloat16* kb = p.k + (size_t)b * p.length * kIxD;
    for (int j = 0; j < tiles && ok; ++j) {
      const int s = j % kIxStages;
      if (j >= kIxStages && !(ok = ix_wait(bar(ixEmpty0 + s), (uint32_t)((j / kIxStages) - 1) & 1u, abort_flag))) break;
      const uint32_t st = base + kIxOffK + (uint32_t)s * kIxStage;
      for (int c = lane; c < kIxKeys * 16; c += 32) {
        const int r = c >> 4, j16 = c & 15;
        const int key = min((tile0 + j) * kIxKeys + r, p.length - 1);
        cp_async_16(st + (uint32_t)(j16 >> 3) * kIxKBlk + sw128(r, j16 & 7), kb + (size_t)key * kIxD + j16 * 8);
      }
      cp_async_commit();
      if (j > 0) {  // the previous tile has landed
        cp_async_wait<1>();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(ixFull0 + (j - 1) % kIxStages));
      }
    }
    if (ok) {
      cp_async_wait<0>();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(ixFull0 + (tiles - 1) % kIxStages));
    } else {
      cp_async_wait<0>();
    }
  } else {
    // ---- MMA issuer: D[d] = K_tile (M=128) . Q_group^T (N=256), K = 128 dims ----
    const uint32_t idesc = idesc_bf16(128, kIxN, false, false);
    ok = ix_wait(bar(ixQFull), 0u, abort_flag);
    for (int j = 0; j < tiles && ok; ++j) {
      const int s = j % kIxStages;
      const uint32_t d = (uint32_t)j & 1u;
      if (!(ok = ix_wait(bar(ixFull0 + s), (uint32_t)(j / kIxStages) & 1u, abort_flag))) break;
      if (j >= 2 && !(ok = ix_wait(bar(ixDFree0 + d), (uint32_t)((j >> 1) - 1) & 1u, abort_flag))) break;
      tc_fence_after();
      const uint32_t st = base + kIxOffK + (uint32_t)s * kIxStage;
      if (elect_one()) {
#pragma unroll
        for (int ks = 0; ks < kIxD / 16; ++ks) {
          const uint64_t ad = smem_desc(st + (uint32_t)(ks >> 2) * kIxKBlk + (uint32_t)(ks & 3) * 32u, 16, 1024,
                                        kLayoutSw128);
          const uint64_t bd = smem_desc(base + kIxOffQ + (uint32_t)(ks >> 2) * kIxQBlk + (uint32_t)(ks & 3) * 32u,
                                        16, 1024, kLayoutSw128);
          mma_bf16_ss(tmem + d * 256u, ad, bd, idesc, ks > 0 ? 1u : 0u);
        }
        mma_commit(bar(ixEmpty0 + s));
        mma_commit(bar(ixDFull0 + d));
      }
      __syncwarp();
    }
  }
  if (!ok && lane == 0) report_error(p.status, kErrTimeout);
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (*abort_flag && warp == kIxMmaWarp) {
    // abort path: wait (bounded) for the MMAs already issued before TMEM is released
    tc_fence_after();
    if (elect_one()) mma_commit(bar(ixDrain));
    __syncwarp();
    (void)mbar_wait_drain(bar(ixDrain), 0u);
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// top-k
// ---------------------------------------------------------------------------
constexpr int kTkThreads = 1024;

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exclusive block-wide prefix count of a 0/1 flag (thread order); *total = sum.
__device__ __forceinline__ int block_scan_flag(bool flag, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t bits = __ballot_sync(0xffffffffu, flag);
  const int in_warp = __popc(bits & ((1u << lane) - 1u));
  if (lane == 0) warp_sums[warp] = __popc(bits);
  __syncthreads();
  if (warp == 0) {
    int v = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    warp_sums[32 + lane] = v;  // inclusive prefix over warps
  }
  __syncthreads();
  const int before = warp > 0 ? warp_sums[32 + warp - 1] : 0;
  *total = warp_sums[32 + 31];
  __syncthreads();
  return before + in_warp;
}

__global__ void __launch_bounds__(kTkThreads, 1) topk_kernel(const float* __restrict__ scores,
                                                             const int32_t* __restrict__ lens,
                                                             int32_t* __restrict__ out, int length, int topk) {
  __shared__ int hist[256];
  __shared__ int scan[64];
  __shared__ uint32_t sel[2];
  const long long t = blockIdx.x;
  const float* row = scores + t * (long long)length;
  int32_t* orow = out + t * (long long)topk;
  const int n = lens != nullptr ? max(0, min(__ldg(lens + t), length)) : length;
  if (n <= topk) {  // every valid key, then padding
    for (int i = threadIdx.x; i < topk; i += kTkThreads) orow[i] = i < n ? i : -1;
    return;
  }
  // radix select of the topk-th largest order key
  uint32_t prefix = 0, mask = 0;
  int need = topk;  // still to take among keys matching the prefix
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += kTkThreads) hist[i] = 0;
    __syncthreads();
    // rows of similar scores share their top bits: lanes adding to the same
    // bin are combined into one atomic (the lowest such lane adds the count)
    for (int c = 0; c < n; c += kTkThreads) {
      const int i = c + threadIdx.x;
      const uint32_t u = i < n ? order_key(__ldg(row + i)) : 0u;
      const bool in = i < n && (u & mask) == prefix;
      const uint32_t bin = in ? ((u >> shift) & 255u) : 256u;
      const uint32_t peers = __match_any_sync(0xffffffffu, bin);
      if (in && (threadIdx.x & 31) == (uint32_t)(__ffs(peers) - 1)) atomicAdd(&hist[bin], __popc(peers));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int above = 0, bin = 255;
      for (; bin > 0; --bin) {
        if (above + hist[bin] >= need) break;
        above += hist[bin];
      }
      sel[0] = (uint32_t)bin;
      sel[1] = (uint32_t)(need - above);
    }
    __syncthreads();
    prefix |= sel[0] << shift;
    mask |= 0xFFu << shift;
    need = (int)sel[1];
    __syncthreads();
  }
  // prefix is the threshold key; `need` keys equal to it are taken (the smallest indices)
  int base = 0, eq_seen = 0;
  for (int c = 0; c < n; c += kTkThreads) {
    const int i = c + threadIdx.x;
    const uint32_t u = i < n ? order_key(__ldg(row + i)) : 0u;
    const bool gt = i < n && u > prefix;
    const bool eq = i < n && u == prefix;
    int eq_total = 0, take_total = 0;
    const int eq_rank = block_scan_flag(eq, scan, &eq_total);
    const bool take = gt || (eq && eq_seen + eq_rank < need);
    const int pos = block_scan_flag(take, scan, &take_total);
    if (take) orow[base + pos] = i;
    base += take_total;
    eq_seen += eq_total;
  }
}

}  // namespace

int indexer_smem_bytes() { return (int)kIxSmem; }

cudaError_t launch_indexer_logits(const __nv_bfloat16* q, const __nv_bfloat16* k, const float* w, const int32_t* lens,
                                  float* scores, int32_t* status, int batch, int queries, int heads, int length,
                                  cudaStream_t stream) {
  if (heads <= 0 || kIxN % heads != 0 || heads < 16) return cudaErrorInvalidValue;
  IxParams p;
  p.q = q;
  p.k = k;
  p.w = w;
  p.lens = lens;
  p.scores = scores;
  p.status = status;
  p.batch = batch;
  p.queries = queries;
  p.heads = heads;
  p.length = length;
  const int G = kIxN / heads;
  p.groups = (queries + G - 1) / G;
  const int tiles = (length + kIxKeys - 1) / kIxKeys;
  p.chunk_tiles = 32;
  p.chunks = (tiles + p.chunk_tiles - 1) / p.chunk_tiles;
  const long long ctas = (long long)batch * p.groups * p.chunks;
  if (ctas > 0x7fffffffLL) return cudaErrorInvalidValue;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(indexer_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kIxSmem) !=
        cudaSuccess)
      return cudaErrorInvalidConfiguration;
    attr = true;
  }
  indexer_logits_kernel<<<(unsigned)ctas, kIxThreads, kIxSmem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_topk(const float* scores, const int32_t* lens, int32_t* out, long long rows, int length, int topk,
                        cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if (rows > 0x7fffffffLL) return cudaErrorInvalidValue;
  topk_kernel<<<(unsigned)rows, kTkThreads, 0, stream>>>(scores, lens, out, length, topk);
  return cudaGetLastError();
}

}  // namespace dsa
