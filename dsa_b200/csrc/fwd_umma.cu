// tcgen05/TMEM sparse-MLA forward for H = 128 heads (the "umma" family).
//
// Work item = (token, KV split, V half r). A persistent CTA (one per SM)
// loops over items; the two halves of a (token, split) are consecutive items,
// so they run at the same time on neighbouring SMs and the second gather of
// each row hits L2. Per item and per tile of 32 selected rows:
//
//   S    = Q . K^T                          (tcgen05, M=128 heads, N=32 keys, K=576)
//   P    = bf16(exp(S/24 - m))              (FP32 online softmax, thread = head row)
//   O_r += P . V[:, 256r .. 256r+256)       (tcgen05, M=128, N=256, K=32 keys)
//
// Both halves compute the full S (1.53x the minimum MMA work) so that no data
// crosses SMs: O for 128 heads x 512 dims needs all 512 TMEM columns of one
// SM, and exchanging partial scores between SMs every tile costs more than
// the duplicated QK.
//
// A tcgen05.mma costs its issuing warp ~120 cycles whatever its size, so the
// narrow (N = 32) QK MMAs are spread over three issuer warps, each with its
// own S accumulator (tile g -> issuer and S buffer g mod 3), and the PV MMAs
// have a fourth issuer. The A operand of 20 of the 36 QK steps (Q dims
// 0..319) is read from TMEM, so those steps cost no shared-memory bandwidth.
//
// TMEM (512 columns): O_r [0, 256), S buffers [256, 352), Q dims 0..319 as
// BF16 pairs [352, 512). Shared memory: Q dims 320..511 and the 64 rope dims
// (128-byte swizzle), the gathered rows (4 stages x 32 rows x 1152 B) and P.
//
// Warp roles (12 warps): 0-3 gather (warp w owns stage w: 16-byte cp.async of
// the indexed rows into swizzled K-major tiles plus a validity bitmask);
// 4-6 issue the QK MMAs; 7 issues the PV MMAs; 8-11 run the softmax, one head
// row per thread, and load Q per item. The epilogue of an item (O of the
// item's last PV -> output or FP32 partial) runs in eight warps: the softmax
// warp of each TMEM lane quadrant writes columns 0..127 of its 32 head rows
// and the issuer warp of the same quadrant (4-7, idle at the item boundary)
// columns 128..255. The online softmax
// keeps the reference's semantics (dsa/workspace.py:242-318): invalid index
// -> -inf, FP32 max/sum, BF16 P, FP32 O. O is only rescaled when the row max
// grows by more than 2^8 in exp2 units (lazy rescale); the reported max is
// the true max and the sum is rescaled to it at the end.
//
// No TMA and no clusters are used. Every wait is bounded and reports through
// the status word.
#include "umma_ptx.cuh"

namespace dsa {
namespace {

using namespace umma;

constexpr int kUmBN = 32;          // keys per tile
constexpr int kUmStages = 4;       // gather pipeline depth (one gather warp per stage)
constexpr int kGatherWarps = kUmStages;
constexpr int kQkIssuers = 3;      // QK issuer warps, one S buffer each
constexpr int kQkWarp0 = kGatherWarps;                  // 4
constexpr int kPvWarp = kQkWarp0 + kQkIssuers;          // 7
constexpr int kSoftWarp0 = kPvWarp + 1;                 // 8
constexpr int kSoftWarps = 4;
constexpr int kUmThreads = 32 * (kSoftWarp0 + kSoftWarps);  // 384
constexpr int kThreadsQ = kUmThreads - 64;                   // warps 2..11 load the first item's Q
constexpr int kUmHeads = 128;
constexpr int kQTmemDims = 320;    // Q dims kept in TMEM (A operand of TS steps)
constexpr int kQkSteps = kDimQK / 16;        // 36
constexpr int kUmMaxClusterSplit = 16;       // largest cluster of the cluster-merge launch
constexpr int kTsSteps = kQTmemDims / 16;    // 20

// Shared-memory layout (bytes from a 1024-aligned base).
constexpr uint32_t kQBlock = 128u * 128u;                    // 128 heads x 64 dims (SW128)
constexpr uint32_t kOffQ = 0;                                // Q dims 320..511 (3 blocks) + rope (1 block)
constexpr uint32_t kQBytes = 4u * kQBlock;                   // 65536
constexpr uint32_t kKBlock = (uint32_t)kUmBN * 128u;         // 4096: 32 keys x 64 dims (SW128)
constexpr uint32_t kKStage = 9u * kKBlock;                   // 8 latent blocks + 1 rope block
constexpr uint32_t kOffK = kOffQ + kQBytes;
constexpr uint32_t kOffP = kOffK + kUmStages * kKStage;      // P: 2 x (128 rows x 32 keys, SW64)
constexpr uint32_t kPBytes = 128u * (uint32_t)kUmBN * 2u;    // 8192 per buffer
constexpr uint32_t kOffMask = kOffP + 2u * kPBytes;          // validity bits per stage
constexpr uint32_t kOffStageTile = kOffMask + 16u;           // tile index each stage is being filled with
constexpr uint32_t kOffEpi = kOffMask + 64u;                  // (l, f) per head row for the epilogue
constexpr uint32_t kOffBar = kOffEpi + (uint32_t)kUmHeads * 8u;

enum Bar {
  kFull0 = 0,
  kEmpty0 = kFull0 + kUmStages,
  kQFull = kEmpty0 + kUmStages,  // this item's Q is loaded (softmax warps)
  kQSeen,                        // every QK issuer has seen this item's Q (issuers)
  kQHelp,                        // the issuer warps' part of the first item's Q is loaded
  kSFull0,
  kSFree0 = kSFull0 + kQkIssuers,
  kPFull0 = kSFree0 + kQkIssuers,  // P buffer b written (tiles g with g % 2 == b)
  kPvDone0 = kPFull0 + 2,          // PV of tiles g with g % 2 == b done (P buffer b free)
  kEpiGo = kPvDone0 + 2,           // the item's last PV is done and (l, f) are posted (softmax warps)
  kOFree,                          // the QK issuers have read their part of O (next item's PV may start)
  kStall,                          // failure-path test: nothing ever arrives here
  kDrain0,                         // abort path: MMA issuer k's issued MMAs have completed
  kBarCount = kDrain0 + kQkIssuers + 1
};
constexpr uint32_t kOffTmemSlot = kOffBar + kBarCount * 8u;
constexpr uint32_t kOffAbort = kOffTmemSlot + 8u;
constexpr uint32_t kSmemUsed = kOffAbort + 8u;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024u;  // slack for the 1024-byte alignment

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 0;
constexpr uint32_t kTmemS = 256;
constexpr uint32_t kTmemQ = kTmemS + kQkIssuers * kUmBN;    // 352

static_assert(kOffK % 1024 == 0 && kKStage % 1024 == 0 && kOffP % 1024 == 0, "swizzle atoms");
static_assert(kTmemQ + kQTmemDims / 2 == kTmemCols, "TMEM budget");
static_assert((uint32_t)kUmHeads * 1024u <= kUmStages * kKStage, "the merged epilogue stages O in the stage buffers");
// Largest slice the merged epilogue loads: ceil(128 / S) rows of 1 KB from each of S splits.
constexpr uint32_t max_slice_bytes(int s = 2) {
  return s > kUmMaxClusterSplit ? 0u
                                : ((uint32_t)((kUmHeads + s - 1) / s * s) * 1024u > max_slice_bytes(s + 1)
                                       ? (uint32_t)((kUmHeads + s - 1) / s * s) * 1024u
                                       : max_slice_bytes(s + 1));
}
static_assert(max_slice_bytes() <= kUmStages * kKStage, "the merged epilogue loads its slice into the stage buffers");
static_assert((uint32_t)(kUmHeads / 2 + 1) * 16u * 4u <= 2u * kPBytes, "the slice weights fit the P buffers");
static_assert((uint32_t)kUmHeads * 8u <= kOffBar - kOffEpi, "the pushed row statistics fit the epilogue slots");
static_assert(kQTmemDims % 64 == 0, "Q TMEM part is a whole number of 64-dim blocks");
static_assert(kSmemBytes <= 232448, "shared memory budget");
static_assert(kOffStageTile + 4u * kUmStages <= kOffEpi, "stage tile words");
static_assert(kQkIssuers + 1 == 4 && kQkWarp0 % 4 == 0, "one issuer warp per TMEM lane quadrant");

struct Item {
  int token, sp, half, batch, kbeg, kend, ntiles;
};

__device__ __forceinline__ Item make_item(const FwdParams& p, int item) {
  Item it;
  it.half = item & 1;
  const int ts = item >> 1;
  it.token = ts / p.split;
  it.sp = ts % p.split;
  it.batch = it.token / p.queries;
  split_bounds(p.topk, kUmBN, p.split, it.sp, &it.kbeg, &it.kend);
  it.ntiles = (it.kend - it.kbeg + kUmBN - 1) / kUmBN;
  return it;
}

// Position of one tile in this CTA's sequence of tiles (items first,
// first + gridDim.x, ...; tiles 0..ntiles-1 of each).
struct TileCursor {
  int item, t;
  Item w;
};

__device__ __forceinline__ void cursor_advance(const FwdParams& p, int n_items, TileCursor& c, int k) {
  c.t += k;
  while (c.item < n_items && c.t >= c.w.ntiles) {
    c.t -= c.w.ntiles;
    c.item += gridDim.x;
    if (c.item < n_items) c.w = make_item(p, c.item);
  }
}

__device__ __forceinline__ TileCursor cursor_start(const FwdParams& p, int n_items, int first, int k) {
  TileCursor c;
  c.item = first;
  c.t = 0;
  if (c.item < n_items) c.w = make_item(p, c.item);
  cursor_advance(p, n_items, c, k);
  return c;
}

// Index of key `lane` of the cursor's tile (-1 past the split's end or past the last item).
__device__ __forceinline__ int cursor_index(const FwdParams& p, const TileCursor& c, int lane) {
  if (c.item >= p.tokens * p.split * 2) return -1;
  const int j = c.w.kbeg + c.t * kUmBN + lane;
  return j < c.w.kend ? __ldg(p.ids + (size_t)c.w.token * p.topk + j) : -1;
}

__device__ __forceinline__ float u2f(uint32_t v) { return __uint_as_float(v); }
__device__ __forceinline__ uint32_t f2u(float v) { return __float_as_uint(v); }

// 2^x on the special-function unit (flushes results below 2^-126 to zero,
// far below what the FP32 row sums can resolve).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// First work item of this CTA. Persistent launch: items blockIdx.x,
// blockIdx.x + gridDim.x, ... Cluster-merge launch (one item per CTA): the
// `split` CTAs of a cluster take the splits of one (token, value half).
template <bool kCM>
__device__ __forceinline__ int first_item(const FwdParams& p) {
  if (!kCM) return (int)blockIdx.x;
  const int c = (int)blockIdx.x / p.split;  // (token, half) of the cluster
  const int sp = (int)blockIdx.x % p.split;
  return (((c >> 1) * p.split + sp) << 1) | (c & 1);
}

// Bounded wait (limit_ns) whose result is the same in every lane of the warp.
__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity, volatile int* abort,
                                          unsigned long long limit_ns) {
  const bool ok = mbar_wait(bar, parity, abort, false, limit_ns);
  return __all_sync(0xffffffffu, ok) != 0;
}

// Columns [cb0, cb1) (multiples of 32) of O for this thread's head row (TMEM
// lane `o_lane`) -> the output (O / l as BF16, split 1) or the FP32 partial
// (O * f); two 32-column chunks in flight so each load overlaps a store.
__device__ __forceinline__ void store_o_part(const FwdParams& p, const Item& w, uint32_t o_lane, int row, int cb0,
                                             int cb1, float l, float f) {
  uint32_t oa[32], ob[32];
  const int col0 = w.half * 256;
  if (kBoundsCheck && (cb0 < 0 || cb1 > 256 || ((o_lane & 0xFFFFu) + (uint32_t)cb1 > kTmemCols))) {
    report_error(p.status, kErrBounds);
    return;
  }
  if (p.split == 1) {
    // correctly rounded reciprocal (within an FP32 ulp of O / l); a row
    // without a valid index (l == 0) is written as 0
    const float rl = l > 0.f ? __frcp_rn(l) : 0.f;
    // the lane pair's two rows (row and row ^ 1; lane parity = row parity)
    __nv_bfloat16* dst = p.out + ((size_t)w.token * kUmHeads + (row & ~1)) * kDimLatent + col0;
    const bool wide = (reinterpret_cast<uintptr_t>(p.out) & 31u) == 0;  // rows are 1024 B apart
#pragma unroll 1
    for (int cb = cb0; cb < cb1; cb += 32) {
      tmem_ld32(o_lane + cb, oa);
      tmem_wait_ld();
      uint32_t a[8], b[8];
      pack_bf16_row32_paired(oa, rl, a, b);
      store_bf16_row32_paired(dst + cb, kDimLatent, a, b, wide);
    }
  } else {
    float* dst = p.part_num + (((size_t)w.token * p.split + w.sp) * kUmHeads + row) * kDimLatent + col0;
    const bool wide = (reinterpret_cast<uintptr_t>(p.part_num) & 31u) == 0;  // rows are 2048 B apart
    tmem_ld32(o_lane + cb0, oa);
#pragma unroll 1
    for (int cb = cb0; cb < cb1; cb += 64) {
      tmem_wait_ld_regs32(oa);
      const bool more = cb + 32 < cb1;
      if (more) tmem_ld32(o_lane + cb + 32, ob);
      store_f32_row32(dst + cb, oa, f, wide);
      if (!more) break;
      tmem_wait_ld_regs32(ob);
      if (cb + 64 < cb1) tmem_ld32(o_lane + cb + 64, oa);
      store_f32_row32(dst + cb + 32, ob, f, wide);
    }
  }
}

// Step 3 of the merged epilogue for S splits: rows [r0, r0 + nrows) x 256
// columns, one 16-byte chunk (row, 4 columns) per unit; each thread loads
// the S partial chunks of up to 24 / S units at once (plain L2 loads: every
// load of a batch is in flight together), then sums them in split order with
// the rows' weights and writes BF16. The chunks of split `own_split` (the
// CTA's own rows, when it kept them) are read from its staging buffer.
template <int S>
__device__ __forceinline__ void slice_sum(const FwdParams& p, const float4* part, const float4* own,
                                          const float* wts, int r0, int nrows, int own_split, int token, int half) {
  constexpr int kUB = 24 / S > 0 ? 24 / S : 1;  // units per thread per batch
  const int nunits = nrows * 64;
#pragma unroll 1
  for (int u0 = threadIdx.x; u0 < nunits; u0 += kUmThreads * kUB) {
    float4 v[kUB][S];
#pragma unroll
    for (int b = 0; b < kUB; ++b) {
      const int u = u0 + b * kUmThreads;
      if (u < nunits) {
        const int rr = r0 + (u >> 6);
        const int pos = (u & 63) ^ (rr & 7);
#pragma unroll
        for (int k = 0; k < S; ++k) {
          if (k == own_split)
            v[b][k] = own[rr * 64 + pos];
          else
            v[b][k] = __ldcg(part + ((size_t)k * kUmHeads + rr) * 64 + pos);
        }
      }
    }
#pragma unroll
    for (int b = 0; b < kUB; ++b) {
      const int u = u0 + b * kUmThreads;
      if (u < nunits) {
        const int lr = u >> 6, ch = u & 63;
        const float* const w = wts + lr * 16;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < S; ++k) {
          const float wk = w[k];
          acc.x = fmaf(wk, v[b][k].x, acc.x);
          acc.y = fmaf(wk, v[b][k].y, acc.y);
          acc.z = fmaf(wk, v[b][k].z, acc.z);
          acc.w = fmaf(wk, v[b][k].w, acc.w);
        }
        uint2 h;
        h.x = pack_bf16x2(acc.x, acc.y);
        h.y = pack_bf16x2(acc.z, acc.w);
        *reinterpret_cast<uint2*>(p.out + ((size_t)token * kUmHeads + r0 + lr) * kDimLatent + half * 256 + ch * 4) =
            h;
      }
    }
  }
}

// Epilogue of the cluster-merge launch, run by all 384 threads of every CTA
// of the cluster (the cluster barrier is always taken, also by a CTA that
// gave up on a wait; it then skips the work). The CTA of split sp holds O_sp
// (128 rows x 256 columns of its value half, relative to its running max
// m_used) in TMEM and, per row, (m_sp, l, f) in shared memory, with l
// relative to m_used and f = exp(m_used - m_sp). The merge of
// dsa/merge.py:13-91 then is: M = max_s m_s, w_s = exp(m_s - M),
// L = sum_s w_s l_s f_s, O = sum_s (w_s / L) (f_s O_s).
//   1. each CTA publishes its rows' (m_sp, l f) and f O_sp, without waiting
//      for the other splits: O is staged in the free stage buffers (rows of
//      1 KB, 16-byte chunks XOR-swizzled by row % 8 so a warp's stores hit
//      distinct banks) and written to the L2 by bulk copies; the statistics
//      go to the L2 too, or, when S divides 128 (every owner has 128 / S
//      rows), straight into the owner's shared memory (DSMEM stores), and
//      the rows this CTA owns stay where they are staged;
//   2. cluster barrier;
//   3. CTA rank r computes the weights w_s / L of its rows [128 r / S,
//      128 (r + 1) / S) from the statistics (the owner of a row in half 0
//      writes softmax_max / softmax_sum), loads the rows of every split
//      from the L2, sums them in split order and writes them as BF16.
// Partials: [token][half][split][128][256] FP32, chunk-swizzled as staged;
// statistics: [token][half][split][128] (m, l f), or [split][row - r0] in
// the owner's shared memory (the epilogue slots, unused by this launch).
__device__ __forceinline__ void merged_epilogue(const FwdParams& p, uint8_t* sbase, uint32_t base, uint32_t tmem,
                                                volatile int* abort_flag) {
  const bool live = *abort_flag == 0;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.split;
  const int sp = (int)blockIdx.x % S;  // == %cluster_ctarank
  const int cl = (int)blockIdx.x / S;
  const int token = cl >> 1, half = cl & 1;
  const float c = p.scale_log2;
  const int r0 = sp * kUmHeads / S, r1 = (sp + 1) * kUmHeads / S;
  const int nrows = r1 - r0;
  const bool even = (kUmHeads % S) == 0;  // S in {2, 4, 8, 16}: 128 / S rows per owner
  float2* const sstat = reinterpret_cast<float2*>(sbase + kOffEpi);
  float4* const part = reinterpret_cast<float4*>(p.part_num) + (size_t)cl * S * kUmHeads * 64;  // this (token, half)
  float2* const pstat = reinterpret_cast<float2*>(p.part_max) + (size_t)cl * S * kUmHeads;
  if (live && warp >= kQkWarp0) {
    tc_fence_after();
    const int row = (warp & 3) * 32 + lane;
    const float4 st = reinterpret_cast<const float4*>(sbase + kOffQ)[row];
    const bool lower = warp >= kSoftWarp0;  // columns 0..127 of the half, else 128..255
    if (lower) {
      const float2 v = make_float2(st.x, st.y * st.z);
      if (even) {
        cluster_wait();  // every CTA of the cluster runs (first barrier phase)
        const int owner = row / nrows;
        st_shared_cluster_f2(mapa_shared(base + kOffEpi + (uint32_t)(sp * nrows + row - owner * nrows) * 8u,
                                         (uint32_t)owner),
                             v);
      } else {
        pstat[(size_t)sp * kUmHeads + row] = v;
      }
    }
    const float f = st.z;
    const uint32_t o_lane = tmem + ((uint32_t)((warp & 3) * 32) << 16) + kTmemO + (lower ? 0u : 128u);
    float4* const srow = reinterpret_cast<float4*>(sbase + kOffK + (uint32_t)row * 1024u);
    const int ch0 = lower ? 0 : 32;  // first 16-byte chunk of this thread's columns
#pragma unroll 1
    for (int cb = 0; cb < 128; cb += 64) {
      uint32_t o[64];
      tmem_ld32(o_lane + cb, o);
      tmem_ld32(o_lane + cb + 32, o + 32);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int ch = ch0 + cb / 4 + j;
        srow[checked_index(ch ^ (row & 7), 64, p.status)] =
            make_float4(__uint_as_float(o[4 * j]) * f, __uint_as_float(o[4 * j + 1]) * f,
                        __uint_as_float(o[4 * j + 2]) * f, __uint_as_float(o[4 * j + 3]) * f);
      }
    }
  }
  // the threads that did not take the first barrier phase above wait for it
  // here, so every thread of the CTA waits on it exactly once
  if (!(live && even && warp >= kSoftWarp0)) cluster_wait();
  tc_fence_before();
  fence_proxy_async_smem();  // the staged rows -> visible to the bulk copies
  __syncthreads();
  // bulk copies are issued by lane 0 of different warps (copies issued by the
  // lanes of one warp go out one after another)
  if (live && warp >= kQkWarp0 && lane == 0) {
    const int w = warp - kQkWarp0;  // 0..7
    float4* const dst = part + (size_t)sp * kUmHeads * 64;
    const uint32_t src = base + kOffK;
    bool issued = false;
    if (even) {  // rows [0, r0) and [r1, 128): the owned rows stay staged
      if (w == 0 && r0 > 0) {
        bulk_store_global(dst, src, (uint32_t)r0 * 1024u);
        issued = true;
      }
      if (w == 1 && r1 < kUmHeads) {
        bulk_store_global(dst + (size_t)r1 * 64, src + (uint32_t)r1 * 1024u, (uint32_t)(kUmHeads - r1) * 1024u);
        issued = true;
      }
    } else {  // 16 head rows (16 KB) per copy
      bulk_store_global(dst + (size_t)w * 16 * 64, src + (uint32_t)w * 16384u, 16384u);
      issued = true;
    }
    if (issued) {
      bulk_commit_group();
      bulk_wait_group_all();
      fence_proxy_async_global();
    }
  }
  cluster_sync();  // every split's statistics and partial rows are published
  if (!live) return;
  // weights w_s / L of the owned rows -> the (free) P buffers [row - r0][16]
  float* const wts = reinterpret_cast<float*>(sbase + kOffP);
  if (even) {
    // one thread per (row, split) in groups of S lanes of a warp (S divides
    // 32): the max and the sum are shuffle reductions over the group
    const int t = (int)threadIdx.x;
    if (t < nrows * S) {  // nrows * S == 128: warps 0..3, every lane
      const int lr = t / S, k = t % S;
      const float2 ms = sstat[k * nrows + lr];
      float M = ms.x;
      for (int o = 1; o < S; o <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
      // an all-masked split (l = 0, O = 0) and a row without any valid index
      // (L = 0: output 0) contribute nothing
      const float e = ms.y > 0.f ? ex2((ms.x - M) * c) : 0.f;
      float L = ms.y * e;
      for (int o = 1; o < S; o <<= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
      wts[lr * 16 + k] = L > 0.f ? e * (1.f / L) : 0.f;
      if (k == 0 && half == 0) {
        const size_t orow = (size_t)token * kUmHeads + r0 + lr;
        p.out_max[orow] = final_max(M, L, p.scale_div);
        p.out_sum[orow] = L;
      }
    }
  } else if (threadIdx.x < (unsigned)nrows) {
    const int lr = (int)threadIdx.x;
    const int row = r0 + lr;
    float2 ms[16];
#pragma unroll
    for (int k = 0; k < 16; ++k)
      if (k < S) ms[k] = __ldcg(pstat + (size_t)k * kUmHeads + row);
    float M = kNegFltMax;
#pragma unroll
    for (int k = 0; k < 16; ++k)
      if (k < S) M = fmaxf(M, ms[k].x);
    // an all-masked split (l = 0, O = 0) and a row without any valid index
    // (L = 0: output 0) contribute nothing
    float e[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) e[k] = (k < S && ms[k].y > 0.f) ? ex2((ms[k].x - M) * c) : 0.f;
    float L = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k)
      if (k < S) L = fmaf(ms[k].y, e[k], L);
    const float rl = L > 0.f ? 1.f / L : 0.f;
    float4* const w4 = reinterpret_cast<float4*>(wts + lr * 16);
#pragma unroll
    for (int k = 0; k < 16; k += 4)
      if (k < S) w4[k / 4] = make_float4(e[k] * rl, e[k + 1] * rl, e[k + 2] * rl, e[k + 3] * rl);
    if (half == 0) {
      const size_t orow = (size_t)token * kUmHeads + row;
      p.out_max[orow] = final_max(M, L, p.scale_div);
      p.out_sum[orow] = L;
    }
  }
  __syncthreads();  // the weights are in shared memory
  const float4* const own = reinterpret_cast<const float4*>(sbase + kOffK);
  switch (S) {
#define DSA_SLICE_SUM(n) \
  case n:                \
    slice_sum<n>(p, part, own, wts, r0, nrows, even ? sp : -1, token, half); \
    break;
    DSA_SLICE_SUM(2) DSA_SLICE_SUM(3) DSA_SLICE_SUM(4) DSA_SLICE_SUM(5) DSA_SLICE_SUM(6) DSA_SLICE_SUM(7)
    DSA_SLICE_SUM(8) DSA_SLICE_SUM(9) DSA_SLICE_SUM(10) DSA_SLICE_SUM(11) DSA_SLICE_SUM(12) DSA_SLICE_SUM(13)
    DSA_SLICE_SUM(14) DSA_SLICE_SUM(15) DSA_SLICE_SUM(16)
#undef DSA_SLICE_SUM
    default:
      break;
  }
}

// kCM: the cluster-merge launch. The `split` CTAs of one (token, value half)
// form a thread-block cluster and merge their partials themselves (row
// statistics and partial O through the L2, two cluster barriers), so no
// separate merge kernel runs; one item per CTA. Otherwise persistent CTAs
// write FP32 partials for merge_kernel (split > 1) or the output (split 1).
template <bool kCM>
__global__ void __launch_bounds__(kUmThreads, 1) fwd_umma_kernel(const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const sbase = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sbase + kOffAbort);
  auto bar = [&](int i) -> uint32_t { return base + kOffBar + 8u * (uint32_t)i; };
  const unsigned long long lim = p.wait_limit_ns != 0 ? p.wait_limit_ns : kWaitLimitNs;
  const int item0 = first_item<kCM>(p);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kUmStages; ++s) {
      mbar_init(bar(kFull0 + s), 1);
      mbar_init(bar(kEmpty0 + s), 1);
    }
    mbar_init(bar(kQFull), kSoftWarps);
    mbar_init(bar(kQSeen), kQkIssuers);
    mbar_init(bar(kQHelp), 4);
    for (int s = 0; s < kUmStages; ++s) reinterpret_cast<volatile uint32_t*>(sbase + kOffStageTile)[s] = 0xffffffffu;
    for (int k = 0; k < kQkIssuers; ++k) {
      mbar_init(bar(kSFull0 + k), 1);
      mbar_init(bar(kSFree0 + k), kSoftWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(kPFull0 + b), kSoftWarps);
      mbar_init(bar(kPvDone0 + b), 1);
    }
    mbar_init(bar(kEpiGo), kSoftWarps);
    mbar_init(bar(kOFree), kQkIssuers);
    mbar_init(bar(kStall), 1);
    for (int k = 0; k <= kQkIssuers; ++k) mbar_init(bar(kDrain0 + k), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(base + kOffTmemSlot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // cluster-merge launch: the first phase of the cluster barrier completes
  // once every CTA of the cluster runs; the merged epilogue waits on it
  // before it writes into a peer's shared memory
  if constexpr (kCM) cluster_arrive_relaxed();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sbase + kOffTmemSlot);

  const int n_items = p.tokens * p.split * 2;
  const int L = p.length;
  float2* const epi = reinterpret_cast<float2*>(sbase + kOffEpi);
  // Columns 128..255 of O for the item's head rows in TMEM lane quadrant
  // warp % 4, by an issuer warp once the softmax warps post the item's (l, f).
  auto epilogue_upper_half = [&](const Item& w, uint32_t it) -> bool {
    if (!wait_warp(bar(kEpiGo), it & 1u, abort_flag, lim)) return false;
    tc_fence_after();
    const int row = (warp & 3) * 32 + lane;
    const float2 lf = epi[row];
    store_o_part(p, w, tmem + ((uint32_t)((warp & 3) * 32) << 16) + kTmemO, row, 128, 256, lf.x, lf.y);
    tc_fence_before();
    __syncwarp();
    return true;
  };

  // The first item's Q, loaded by warps 2..11 together with coalesced
  // 16-byte loads (a warp reads 512 contiguous bytes per instruction; one
  // head row per thread would touch 32 rows per instruction): latent dims
  // 320..511 and the rope dims go straight into their swizzled shared-memory
  // blocks, dims 0..319 into a row-major staging area over stage buffers
  // 2..3 and the P buffers (rows of 640 B, 16-byte chunks XOR-swizzled by
  // row % 8), from which warps 4..11 move them into TMEM (q_first_tmem).
  // Stages 0 and 1 are gathered meanwhile; stages 2..3 start once Q has left
  // the staging area (the first P is written after the first scores, which
  // need all of Q in TMEM).
  constexpr uint32_t kOffQStage = kOffK + 2u * kKStage;
  static_assert(kOffQStage + (uint32_t)kUmHeads * 640u <= kOffP + 2u * kPBytes, "Q staging area");
  auto q_first = [&](int item) {
    constexpr int kTm = kUmHeads * (kQTmemDims / 8);  // 16-byte chunks of dims 0..319 (40 per row)
    constexpr int kSm = kUmHeads * 32;                // chunks of dims 320..511 (24) and rope (8) per row
    constexpr int kPerTm = (kTm + kThreadsQ - 1) / kThreadsQ;
    const int t = (int)threadIdx.x - 64;
    const size_t qrow0 = (size_t)make_item(p, item).token * kUmHeads;
    const uint4* const qsrc = reinterpret_cast<const uint4*>(p.q + qrow0 * kDimLatent);
    const uint4* const rsrc = reinterpret_cast<const uint4*>(p.q_rope + qrow0 * kDimRope);
    // dims 320..511 and the rope dims: asynchronous copies into the swizzled blocks
#pragma unroll 4
    for (int j = t; j < kSm; j += kThreadsQ) {
      const int r = j >> 5, c = j & 31;
      const uint4* const src = c < 24 ? qsrc + r * 64 + 40 + c : rsrc + r * 8 + (c - 24);
      const uint32_t dst = kOffQ + (uint32_t)(c >> 3) * kQBlock + (uint32_t)(r >> 3) * 1024u +
                           (uint32_t)(r & 7) * 128u + (uint32_t)(((c & 7) ^ (r & 7)) * 16);
      cp_async_16(base + dst, src);
    }
    cp_async_commit();
    // dims 0..319: registers, all loads in flight, then the staging area
    uint4 v[kPerTm];
#pragma unroll
    for (int i = 0; i < kPerTm; ++i) {
      const int j = t + i * kThreadsQ;
      if (j < kTm) v[i] = __ldg(qsrc + (j / 40) * 64 + (j % 40));
    }
#pragma unroll
    for (int i = 0; i < kPerTm; ++i) {
      const int j = t + i * kThreadsQ;
      if (j < kTm) {
        const int r = j / 40, c = j % 40;
        *reinterpret_cast<uint4*>(sbase + kOffQStage + (uint32_t)r * 640u + (uint32_t)((c ^ (r & 7)) * 16)) = v[i];
      }
    }
    cp_async_wait<0>();
    fence_proxy_async_smem();  // the shared-memory Q blocks -> visible to the tensor core
    named_bar_sync(1, kThreadsQ);
  };
  // Warps 4..11: dims 0..319 of the head rows of TMEM lane quadrant warp % 4
  // from the staging area into TMEM; the issuer warp takes chunks 0..19,
  // the softmax warp chunks 20..39 (16-byte chunk u -> TMEM columns 4u..4u+3).
  auto q_first_tmem = [&]() {
    const int row = (warp & 3) * 32 + lane;
    const int c0 = warp >= kSoftWarp0 ? 20 : 0;
    uint32_t r[80];
#pragma unroll
    for (int i = 0; i < 20; ++i) {
      const uint4 x =
          *reinterpret_cast<const uint4*>(sbase + kOffQStage + (uint32_t)row * 640u + (uint32_t)(((c0 + i) ^ (row & 7)) * 16));
      r[4 * i] = x.x;
      r[4 * i + 1] = x.y;
      r[4 * i + 2] = x.z;
      r[4 * i + 3] = x.w;
    }
    const uint32_t t_lane = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t col = tmem + t_lane + kTmemQ + (uint32_t)(4 * c0);
    tmem_st32(col, r);
    tmem_st32(col + 32, r + 32);
    tmem_st16(col + 64, r + 64);
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
  };
  auto q_help = [&](int item) {
    q_first(item);
    q_first_tmem();
    if (lane == 0) mbar_arrive(bar(kQHelp));
  };

  if (warp < kGatherWarps) {
    // ---------------- gather: warp w fills stage w for tiles g = w, w+4, ... ----------------
    // The indices of the tile two rounds ahead are loaded one round early, so
    // a freed stage waits only for its rows.
    const uint32_t s = (uint32_t)warp;
    const uint32_t stage = base + kOffK + s * kKStage;
    uint32_t* const mask_s = reinterpret_cast<uint32_t*>(sbase + kOffMask) + s;
    // lane -> (key quarter kq, 16-byte chunk j8): 4 rows x 128 contiguous bytes per instruction
    const int j8 = lane & 7;
    const int kq = lane >> 3;
    TileCursor cur = cursor_start(p, n_items, item0, (int)s);
    TileCursor nx = cur;
    cursor_advance(p, n_items, nx, kUmStages);
    TileCursor nx2 = nx;
    cursor_advance(p, n_items, nx2, kUmStages);
    int idx_cur = cursor_index(p, cur, lane);
    int idx_nx = cursor_index(p, nx, lane);
    if (s > 1 && item0 < n_items) q_first(item0);
    uint32_t n = 0;  // tiles this warp filled
    bool ok = true;
    while (cur.item < n_items) {
      if (n > 0) {  // the stage's previous tile has been consumed by its PV
        if (lane == 0) ok = mbar_wait(bar(kEmpty0 + s), (n - 1) & 1u, abort_flag, false, lim);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      } else if (s > 1) {
        // stages 2..3 hold the first item's Q staging area until warps 4..11
        // have moved it into TMEM
        ok = wait_warp(bar(kQFull), 0u, abort_flag, lim);
        if (ok) ok = wait_warp(bar(kQHelp), 0u, abort_flag, lim);
        if (!ok) break;
      }
      const int row = checked_index(min(max(idx_cur, 0), L - 1), L, p.status);  // clamped address; masked below
      const uint32_t bits = __ballot_sync(0xffffffffu, (idx_cur >= 0) & (idx_cur < L));
      if (lane == 0) {
        *mask_s = bits;
        // the stage's previous tile (g - 4) is consumed, so its Full phase completed
        reinterpret_cast<volatile uint32_t*>(sbase + kOffStageTile)[s] = s + kUmStages * n;
      }
      const int gb = checked_index(cur.w.batch, p.batch, p.status);
      const __nv_bfloat16* const kv_b = p.kv + (size_t)gb * L * kDimLatent;
      const __nv_bfloat16* const kr_b = p.k_rope + (size_t)gb * L * kDimRope;
#pragma unroll 2
      for (int i = 0; i < kUmBN / 4; ++i) {
        const int k = kq + 4 * i;
        const int rk = __shfl_sync(0xffffffffu, row, k);
        const uint32_t dst = checked_smem(stage + (uint32_t)(k >> 3) * 1024u + (uint32_t)(k & 7) * 128u +
                                              (uint32_t)((j8 ^ (k & 7)) * 16),
                                          8u * kKBlock + 16u, stage, kKStage, p.status);
        const __nv_bfloat16* src = kv_b + (size_t)rk * kDimLatent + j8 * 8;
#pragma unroll
        for (int kb = 0; kb < 8; ++kb) cp_async_16(dst + kb * kKBlock, src + kb * 64);
        cp_async_16(dst + 8 * kKBlock, kr_b + (size_t)rk * kDimRope + j8 * 8);
      }
      cp_async_commit();
      const int idx_nx2 = cursor_index(p, nx2, lane);  // consumed one round later
      cp_async_wait<0>();
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kFull0 + s));
      ++n;
      cur = nx;
      nx = nx2;
      cursor_advance(p, n_items, nx2, kUmStages);
      idx_cur = idx_nx;
      idx_nx = idx_nx2;
    }
    if (!ok) report_error(p.status, kErrTimeout);
  } else if (warp < kPvWarp) {
    // ---------------- QK issuer i: tiles g with g % 3 == i, into S buffer i ----------------
    // The whole warp runs the loop and waits; one elected lane issues.
    const uint32_t i = (uint32_t)(warp - kQkWarp0);
    const uint32_t idesc_qk = idesc_bf16(128, kUmBN, false, false);
    const uint32_t d = tmem + kTmemS + i * kUmBN;
    uint32_t g = 0, it = 0, n = 0;  // n: tiles this issuer ran
    bool ok = true;
    if (item0 < n_items) q_help(item0);
    for (int item = item0; item < n_items && ok; item += gridDim.x, ++it) {
      const Item w = make_item(p, item);
      // Every issuer observes every item's Q (even without a tile in it) and
      // acknowledges, so no issuer can fall a barrier phase behind.
      ok = wait_warp(bar(kQFull), it & 1u, abort_flag, lim);
      if (ok && it == 0) ok = wait_warp(bar(kQHelp), 0u, abort_flag, lim);
      if (!ok) break;
      if (elect_one()) mbar_arrive(bar(kQSeen));
      __syncwarp();
      for (int t = 0; t < w.ntiles && ok; ++t, ++g) {
        if (g % kQkIssuers != i) continue;
        const uint32_t s = g % kUmStages;
        // Issuer g % 3 has not observed the Full phase of the stage's previous
        // tile (g - 4, another issuer's). Once the gather of tile g has
        // started, that phase has completed and the parity wait refers to
        // tile g's phase exactly.
        ok = wait_word_warp(reinterpret_cast<volatile uint32_t*>(sbase + kOffStageTile) + s, g, abort_flag, lim);
        if (ok) ok = wait_warp(bar(kFull0 + s), (g / kUmStages) & 1u, abort_flag, lim);
        if (ok && n > 0) ok = wait_warp(bar(kSFree0 + i), (n - 1) & 1u, abort_flag, lim);
        if (!ok) break;
        tc_fence_after();
        const uint32_t stage = base + kOffK + s * kKStage;
        if (elect_one()) {
#pragma unroll
          for (int ks = 0; ks < kTsSteps; ++ks) {  // dims 0..319: A = Q from TMEM
            const uint64_t bd =
                smem_desc(stage + (ks >> 2) * kKBlock + (uint32_t)(ks & 3) * 32u, 16, 1024, kLayoutSw128);
            mma_bf16_ts(d, tmem + kTmemQ + (uint32_t)ks * 8u, bd, idesc_qk, ks > 0 ? 1u : 0u);
          }
#pragma unroll
          for (int ks = kTsSteps; ks < kQkSteps; ++ks) {  // dims 320..575: A from shared memory
            const uint32_t qb = (uint32_t)(ks - kTsSteps) >> 2;
            const uint64_t ad = smem_desc(base + kOffQ + qb * kQBlock + (uint32_t)(ks & 3) * 32u, 16, 1024,
                                          kLayoutSw128);
            const uint64_t bd =
                smem_desc(stage + (ks >> 2) * kKBlock + (uint32_t)(ks & 3) * 32u, 16, 1024, kLayoutSw128);
            mma_bf16_ss(d, ad, bd, idesc_qk, 1u);
          }
          mma_commit(bar(kSFull0 + i));
        }
        __syncwarp();
        ++n;
      }
      if (!ok) break;
      if (kCM) continue;  // the merged epilogue after the roles writes O
      if (!(ok = epilogue_upper_half(w, it))) break;
      if (lane == 0) mbar_arrive(bar(kOFree));
    }
    if (!ok && lane == 0) report_error(p.status, kErrTimeout);
  } else if (warp == kPvWarp) {
    // ---------------- PV issuer: every tile in order (warp-converged, one elected lane issues) ----
    const uint32_t idesc_pv = idesc_bf16(128, 256, false, true);
    uint32_t g = 0, it = 0;
    bool ok = true;
    if (item0 < n_items) q_help(item0);
    for (int item = item0; item < n_items && ok; item += gridDim.x, ++it) {
      const Item w = make_item(p, item);
      const uint32_t vblk = (uint32_t)w.half * 4u * kKBlock;  // first latent block of this V half
      for (int t = 0; t < w.ntiles && ok; ++t, ++g) {
        ok = wait_warp(bar(kPFull0 + (g & 1u)), (g >> 1) & 1u, abort_flag, lim);
        // the first PV of an item overwrites O: the previous item's epilogue
        // (the QK issuers' part) must have read it
        if (ok && t == 0 && it > 0) ok = wait_warp(bar(kOFree), (it - 1) & 1u, abort_flag, lim);
        if (!ok) break;
        tc_fence_after();
        const uint32_t stage = base + kOffK + (g % kUmStages) * kKStage;
        if (elect_one()) {
#pragma unroll
          for (int j = 0; j < kUmBN / 16; ++j) {
            const uint64_t ad = smem_desc(base + kOffP + (g & 1u) * kPBytes + j * 32, 16, 512, kLayoutSw64);
            const uint64_t bd = smem_desc(stage + vblk + j * 2048, kKBlock, 1024, kLayoutSw128);
            mma_bf16_ss(tmem + kTmemO, ad, bd, idesc_pv, (t == 0 && j == 0) ? 0u : 1u);
          }
          mma_commit(bar(kPvDone0 + (g & 1u)));
          mma_commit(bar(kEmpty0 + g % kUmStages));
        }
        __syncwarp();
      }
      if (!ok) break;
      if (kCM) continue;
      if (!(ok = epilogue_upper_half(w, it))) break;
    }
    if (!ok && lane == 0) report_error(p.status, kErrTimeout);
  } else {
    // ---------------- softmax + epilogue (one head row per thread) ----------------
    const int quad = warp & 3;  // TMEM lane quadrant of this warp
    const int row = quad * 32 + lane;
    const uint32_t t_lane = (uint32_t)(quad * 32) << 16;
    const float c = p.scale_log2;  // log2(e) / scale_div
    uint8_t* const prow0 = sbase + kOffP + (uint32_t)(row >> 3) * 512u + (uint32_t)(row & 7) * 64u;
    const uint32_t* const mask_all = reinterpret_cast<const uint32_t*>(sbase + kOffMask);
    uint32_t g = 0, it = 0;
    bool ok = true;
    // the first item's Q: the shared load of warps 2..11 (before any bounded
    // wait, so every participant reaches its named barrier), then this
    // warp's half of dims 0..319 into TMEM
    if (item0 < n_items) {
      q_first(item0);
      q_first_tmem();
    }
    for (int item = item0; item < n_items && ok; item += gridDim.x, ++it) {
      const Item w = make_item(p, item);
      if (it == 0 && p.wait_test != 0 && blockIdx.x == 0) {
        // failure-path test: wait on a barrier that nothing arrives at, so the
        // bounded wait runs out and the whole CTA takes its abort path
        ok = wait_warp(bar(kStall), 0u, abort_flag, lim);
        if (!ok) break;
      }
      // Q of this head row: dims 0..319 -> TMEM, dims 320..511 and the rope
      // dims -> shared memory (128-byte swizzle). The previous item's MMAs
      // are complete (its epilogue waited for its last PV), and every QK
      // issuer has seen the previous item's Q.
      if (it > 0 && !(ok = wait_warp(bar(kQSeen), (it - 1) & 1u, abort_flag, lim))) break;
      if (it > 0) {
        // later items: this thread's head row, dims 320..511 and the rope
        // dims -> shared memory asynchronously, dims 0..319 -> TMEM in 64-dim
        // chunks with three chunks' loads in flight
        const size_t qrow = (size_t)w.token * kUmHeads + row;
        const uint4* src = reinterpret_cast<const uint4*>(p.q + qrow * kDimLatent);
        const uint32_t qdst = base + kOffQ + (uint32_t)(row >> 3) * 1024u + (uint32_t)(row & 7) * 128u;
#pragma unroll
        for (int k = 0; k < (kDimLatent - kQTmemDims) / 8; ++k)  // latent dims 320..511: 3 blocks
          cp_async_16(qdst + (k >> 3) * kQBlock + (((k & 7) ^ (row & 7)) * 16), src + kQTmemDims / 8 + k);
        const uint4* rsrc = reinterpret_cast<const uint4*>(p.q_rope + qrow * kDimRope);
#pragma unroll
        for (int k = 0; k < 8; ++k) cp_async_16(qdst + 3 * kQBlock + ((k ^ (row & 7)) * 16), rsrc + k);
        cp_async_commit();
        uint4 qa[24];
#pragma unroll
        for (int k = 0; k < 24; ++k) qa[k] = __ldg(src + k);
#pragma unroll
        for (int ch = 0; ch < kQTmemDims / 64; ++ch) {
          uint32_t r[32];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint4 v = qa[(ch % 3) * 8 + k];
            r[4 * k] = v.x;
            r[4 * k + 1] = v.y;
            r[4 * k + 2] = v.z;
            r[4 * k + 3] = v.w;
          }
          tmem_st32(tmem + t_lane + kTmemQ + ch * 32, r);
          if (ch + 3 < kQTmemDims / 64) {
#pragma unroll
            for (int k = 0; k < 8; ++k) qa[(ch % 3) * 8 + k] = __ldg(src + (ch + 3) * 8 + k);
          }
        }
        cp_async_wait<0>();
        fence_proxy_async_smem();
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
      }
      if (lane == 0) mbar_arrive(bar(kQFull));
      float m_true = kNegFltMax, m_used = kNegFltMax, l = 0.f;
      for (int t = 0; t < w.ntiles && ok; ++t, ++g) {
        const uint32_t s = g % kUmStages;
        const uint32_t i = g % kQkIssuers;
        const uint32_t n = g / kQkIssuers;  // uses of S buffer i so far
        ok = wait_warp(bar(kSFull0 + i), n & 1u, abort_flag, lim);
        if (!ok) break;
        tc_fence_after();
        float x[32];
        {
          uint32_t sv[32];
          tmem_ld32(checked_tmem(tmem + t_lane + kTmemS + i * kUmBN, tmem, 32u, kTmemCols, p.status), sv);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k) x[k] = u2f(sv[k]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kSFree0 + i));
        // validity bits of the tile's keys (written by the gather warp)
        ok = wait_warp(bar(kFull0 + s), (g / kUmStages) & 1u, abort_flag, lim);
        if (!ok) break;
        const uint32_t mbits = mask_all[s];
        float mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          x[k] = ((mbits >> k) & 1u) ? x[k] : -INFINITY;
          mx = fmaxf(mx, x[k]);
        }
        m_true = fmaxf(m_true, mx);
        float alpha = 1.f;
        bool resc = false;
        if ((mx - m_used) * c > 8.f) {
          alpha = ex2((m_used - mx) * c);
          m_used = mx;
          resc = true;
        }
        const float mc = m_used * c;
        float sum = 0.f;
        uint32_t packed[16];
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          const float p0 = ex2(fmaf(x[k], c, -mc));
          const float p1 = ex2(fmaf(x[k + 1], c, -mc));
          sum += p0 + p1;
          packed[k / 2] = pack_bf16x2(p0, p1);
        }
        l = l * alpha + sum;
        // P buffer g % 2 is free once PV(g - 2) finished reading it
        const uint32_t pb = g & 1u;
        if (g >= 2) ok = wait_warp(bar(kPvDone0 + pb), ((g >> 1) - 1) & 1u, abort_flag, lim);
        if (!ok) break;
        uint8_t* const prow = prow0 + pb * kPBytes;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(prow + ((q ^ ((row & 7) >> 1)) * 16)) =
              make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        fence_proxy_async_smem();
        if (__any_sync(0xffffffffu, resc) && t > 0) {
          // O is read and rescaled: PV(g - 1) must have finished writing it
          ok = wait_warp(bar(kPvDone0 + (pb ^ 1u)), ((g - 1) >> 1) & 1u, abort_flag, lim);
          if (!ok) break;
          tc_fence_after();
          uint32_t o[32];
#pragma unroll 1
          for (int cb = 0; cb < 256; cb += 32) {
            const uint32_t a = tmem + t_lane + kTmemO + cb;
            tmem_ld32(a, o);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; ++k) o[k] = f2u(u2f(o[k]) * alpha);
            tmem_st32(a, o);
          }
          tmem_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kPFull0 + pb));
      }
      if (!ok) break;
      // ---- epilogue: columns 0..127 of this CTA's 256 dims of the head row
      // (the issuer warp of this lane quadrant writes 128..255) ----
      ok = wait_warp(bar(kPvDone0 + ((g - 1) & 1u)), ((g - 1) >> 1) & 1u, abort_flag, lim);
      if (!ok) break;
      const float f = (m_true == kNegFltMax) ? 1.f : ex2((m_used - m_true) * c);
      if (kCM) {
        // every QK and PV of the item is complete: the Q rows in shared
        // memory are free and hold the row statistics for the merged epilogue
        reinterpret_cast<float4*>(sbase + kOffQ)[row] = make_float4(m_true, l, f, 0.f);
        tc_fence_before();
        continue;
      }
      epi[row] = make_float2(l, f);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kEpiGo));
      tc_fence_after();
      const size_t orow = (size_t)w.token * kUmHeads + row;
      if (w.half == 0) {
        if (p.split == 1) {
          p.out_max[orow] = final_max(m_true, l, p.scale_div);
          p.out_sum[orow] = l * f;
        } else {
          const size_t prow_idx = ((size_t)w.token * p.split + w.sp) * kUmHeads + row;
          p.part_max[prow_idx] = (m_true == kNegFltMax) ? kNegFltMax : __fdiv_rn(m_true, p.scale_div);
          p.part_sum[prow_idx] = l * f;
        }
      }
      store_o_part(p, w, tmem + t_lane + kTmemO, row, 0, 128, l, f);
      tc_fence_before();
    }
    if (!ok) report_error(p.status, kErrTimeout);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    // Abort path: a role gave up, so MMAs an issuer warp enqueued may still be
    // running (on the normal path the softmax and epilogue waits have seen
    // every one complete). Each issuer commits once more and waits, bounded,
    // until its MMAs have completed before the TMEM they write is released.
    // elect.sync elects the same lane of a converged warp as at issue time.
    if (warp >= kQkWarp0 && warp <= kPvWarp) {
      const uint32_t k = (uint32_t)(warp - kQkWarp0);
      tc_fence_after();
      if (elect_one()) mma_commit(bar(kDrain0 + k));
      __syncwarp();
      const bool drained = mbar_wait_drain(bar(kDrain0 + k), 0u);
      if (!drained && lane == 0) report_error(p.status, kErrTimeout);
    }
    tc_fence_before();
    __syncthreads();
  }
  if constexpr (kCM) {
    merged_epilogue(p, sbase, base, tmem, abort_flag);
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

int umma_max_ctas() {
  static int cached = -1;
  if (cached > 0) return cached;
  if (cudaFuncSetAttribute(fwd_umma_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kSmemBytes) != cudaSuccess)
    return -1;
  int per_sm = 0, dev = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fwd_umma_kernel<false>, kUmThreads, kSmemBytes) !=
          cudaSuccess ||
      per_sm <= 0)
    return -1;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return -1;
  cached = per_sm * sms;
  return cached;
}

namespace {

// Cluster-merge launch of `split` CTAs per cluster (non-portable above 8).
void cm_launch_config(cudaLaunchConfig_t* cfg, cudaLaunchAttribute* attr, int split, long long ctas,
                      cudaStream_t stream) {
  attr->id = cudaLaunchAttributeClusterDimension;
  attr->val.clusterDim.x = (unsigned)split;
  attr->val.clusterDim.y = 1;
  attr->val.clusterDim.z = 1;
  *cfg = cudaLaunchConfig_t{};
  cfg->gridDim = dim3((unsigned)ctas, 1, 1);
  cfg->blockDim = dim3(kUmThreads, 1, 1);
  cfg->dynamicSmemBytes = kSmemBytes;
  cfg->stream = stream;
  cfg->attrs = attr;
  cfg->numAttrs = 1;
}

// Clusters of `split` CTAs resident at once (0 if none fits), cached per size.
int cm_active_clusters(int split) {
  static int cached[kUmMaxClusterSplit + 1];
  static bool init = false;
  if (!init) {
    if (cudaFuncSetAttribute(fwd_umma_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) !=
            cudaSuccess ||
        cudaFuncSetAttribute(fwd_umma_kernel<true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
      return 0;
    for (int s = 0; s <= kUmMaxClusterSplit; ++s) cached[s] = -1;
    init = true;
  }
  if (split < 2 || split > kUmMaxClusterSplit) return 0;
  if (cached[split] < 0) {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr;
    cm_launch_config(&cfg, &attr, split, split, nullptr);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fwd_umma_kernel<true>, &cfg) != cudaSuccess) {
      cudaGetLastError();  // clear the error an unsupported cluster size leaves behind
      n = 0;
    }
    cached[split] = n;
  }
  return cached[split];
}

}  // namespace

bool umma_cluster_merge(int split) { return cm_active_clusters(split) > 0; }

int umma_cluster_split(long long clusters, int split) {
  if (split > kUmMaxClusterSplit) split = kUmMaxClusterSplit;
  for (int s = split; s >= 2; --s)
    if (cm_active_clusters(s) >= clusters) return s;
  return split;
}

cudaError_t launch_fwd_umma(const FwdParams& p, cudaStream_t stream) {
  if (p.heads != kUmHeads || p.keys_per_tile != kUmBN) return cudaErrorInvalidValue;
  const long long items = (long long)p.tokens * p.split * 2;
  if (p.split > 1 && umma_cluster_merge(p.split)) {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr;
    cm_launch_config(&cfg, &attr, p.split, items, stream);
    return cudaLaunchKernelEx(&cfg, fwd_umma_kernel<true>, p);
  }
  const int max_ctas = umma_max_ctas();
  if (max_ctas <= 0) return cudaErrorInvalidConfiguration;
  const int ctas = (int)(items < max_ctas ? items : max_ctas);
  fwd_umma_kernel<false><<<ctas, kUmThreads, kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace dsa
