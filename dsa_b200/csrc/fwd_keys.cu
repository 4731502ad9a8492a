// tcgen05/TMEM sparse-MLA forward for 16-head groups with the selected keys
// as the MMA's M dimension (the "keys" family; any H % 16 == 0).
//
// Sixteen heads per gathered row are too few for the MMA's M (64 or 128), so
// both products are computed transposed, per work item (token, 16-head
// group, KV split) and tile of 64 selected rows:
//
//   S^T  = K . Q^T                 (tcgen05, M = 64 keys, N = 16 heads, K = 576 dims)
//   P    = bf16(exp(S / d - m))    (FP32, one key per thread, 16 heads per thread)
//   O^T += V^T . P^T               (tcgen05, M = 128 latent dims (x4), N = 16 heads, K = 64 keys)
//
// A gathered tile (64 rows x 1152 B in 64-dim blocks, 128-byte swizzle) is
// the K-major A operand of the score MMAs (rows = keys) and, read as an
// MN-major operand (rows = keys = the reduction dimension, 64 latent dims per
// 128-byte row), the A operand of the value MMAs: no copy or transpose.
// Both products read their A operand from shared memory; per key a tile
// moves ~1152 B into shared memory and ~2176 B out of it to the tensor core,
// which is what bounds the kernel (the MMAs use a fraction of the tensor
// pipe at N = 16).
//
// Online softmax with the reference's semantics (dsa/workspace.py:242-318:
// invalid index -> -inf, FP32 max/sum from the unrounded exponentials, BF16
// P, FP32 O): every softmax thread keeps the same per-head reference max
// m_used in registers; it only changes when a score exceeds it by more than
// 2^8 in exp2 units (lazy rescale). A tile that needs no change (almost all)
// costs one named-barrier vote among the four softmax warps; a tile that
// does reduces the per-head tile max over the 64 keys and rescales the
// per-thread partial sums and O^T. The true max and the sums are reduced over
// the keys once per item; the statistics are reported against the true max.
//
// TMEM (128 columns): S^T double buffer at columns 0 and 16 (M = 64 layout:
// key 16q + i in lane 32q + i), O^T at columns 64..127 (latent block jb of
// 128 dims at 64 + 16 jb, dim = lane).
//
// Warp roles (9 warps): 0-3 softmax (warp q reads TMEM lane quadrant q),
// load Q per item and write the epilogue; 4-7 gather (two per stage, 32 keys
// each, 16-byte cp.async into the swizzled tile plus a validity bitmask);
// 8 issues the MMAs (one elected lane, polling: the value MMAs of a tile as
// soon as its P is written, the score MMAs of the next tile as soon as its stage
// is gathered). Every mbarrier wait is bounded and reports
// through the status word; after a failed wait the softmax warps run their
// remaining tiles without waiting (every later wait fails at once), so the
// four of them always take the same named barriers.
#include "umma_ptx.cuh"

namespace dsa {
namespace {

using namespace umma;

constexpr int kKyHeads = 16;
constexpr int kKyBN = 64;                       // keys per tile (M of the score MMAs)
constexpr int kKyStages = 2;
constexpr int kKySoftWarps = 4;                 // warps 0-3
constexpr int kKyGatherWarp0 = kKySoftWarps;    // warps 4-7: stage (w - 4) / 2, key half (w - 4) % 2
constexpr int kKyMmaWarp = kKyGatherWarp0 + 2 * kKyStages;  // 8
constexpr int kKyThreads = 32 * (kKyMmaWarp + 1);            // 288
constexpr int kKyQkSteps = kDimQK / 16;         // 36
constexpr int kKyQChunks = kDimQK / 8;          // 72 x 16 B per Q row

// Shared memory (bytes from a 1024-aligned base).
constexpr uint32_t kKyBlk = (uint32_t)kKyBN * 128u;        // 8192: 64 keys x 64 dims (SW128)
constexpr uint32_t kKyStage = 9u * kKyBlk;                 // 8 latent blocks + the rope block
constexpr uint32_t kKyQBlk = (uint32_t)kKyHeads * 128u;    // 2048: 16 heads x 64 dims (SW128)
constexpr uint32_t kKyPBytes = (uint32_t)kKyHeads * 128u;  // 2048: 16 heads x 64 keys BF16 (SW128)
constexpr uint32_t kKyOffK = 0;
constexpr uint32_t kKyOffQ = kKyOffK + kKyStages * kKyStage;
constexpr uint32_t kKyOffP = kKyOffQ + 9u * kKyQBlk;
constexpr uint32_t kKyOffMask = kKyOffP + 2u * kKyPBytes;  // validity bits: [stage][key half]
// per-warp per-head values: tile maxima (votes), item sums and item maxima
// (epilogue), each [4][16] floats
constexpr uint32_t kKyOffRed = kKyOffMask + 64u;
constexpr uint32_t kKyOffBar = kKyOffRed + 3u * 4u * 16u * 4u;

enum KyBar {
  kyFull0 = 0,                 // stage s gathered (both gather warps of the stage)
  kyEmpty0 = kyFull0 + kKyStages,   // stage s consumed (value MMAs of its tile done)
  kySFull0 = kyEmpty0 + kKyStages,  // S^T buffer b written
  kySFree0 = kySFull0 + 2,          // S^T buffer b read (softmax warps)
  kyPFull0 = kySFree0 + 2,          // P^T buffer b written (softmax warps)
  kyPvDone0 = kyPFull0 + 2,         // value MMAs of the tile in P^T buffer b done
  kyQFull = kyPvDone0 + 2,          // the item's Q is in shared memory (softmax warps)
  kyQFree,                          // the item's score MMAs are done
  kyBarCount
};
constexpr uint32_t kKyOffTmemSlot = kKyOffBar + kyBarCount * 8u;
constexpr uint32_t kKyOffAbort = kKyOffTmemSlot + 8u;
constexpr uint32_t kKySmemUsed = kKyOffAbort + 8u;
constexpr uint32_t kKySmemBytes = kKySmemUsed + 1024u;  // slack for the 1024-byte alignment

constexpr uint32_t kKyTmemCols = 128;
constexpr uint32_t kKyTmemS = 0;   // S^T buffer b at column 16 b
constexpr uint32_t kKyTmemO = 64;  // O^T latent block jb at column 64 + 16 jb

static_assert(kKyOffQ % 1024 == 0 && kKyOffP % 1024 == 0 && kKyStage % 1024 == 0, "swizzle atoms");
static_assert(kKySmemBytes <= 232448, "shared memory budget");

struct KyItem {
  int token, hg, sp, batch, kbeg, kend, ntiles;
};

__device__ __forceinline__ KyItem ky_item(const FwdParams& p, int item) {
  const int hgroups = p.heads / kKyHeads;
  KyItem it;
  it.sp = item % p.split;
  const int rest = item / p.split;
  it.hg = rest % hgroups;
  it.token = rest / hgroups;
  it.batch = it.token / p.queries;
  split_bounds(p.topk, kKyBN, p.split, it.sp, &it.kbeg, &it.kend);
  it.ntiles = (it.kend - it.kbeg + kKyBN - 1) / kKyBN;
  return it;
}

// Position of one tile in this CTA's sequence (items blockIdx.x, +gridDim.x, ...).
struct KyCursor {
  int item, t;
  KyItem w;
};

__device__ __forceinline__ void ky_advance(const FwdParams& p, int n_items, KyCursor& c, int k) {
  c.t += k;
  while (c.item < n_items && c.t >= c.w.ntiles) {
    c.t -= c.w.ntiles;
    c.item += gridDim.x;
    if (c.item < n_items) c.w = ky_item(p, c.item);
  }
}

__device__ __forceinline__ KyCursor ky_start(const FwdParams& p, int n_items, int k) {
  KyCursor c;
  c.item = blockIdx.x;
  c.t = 0;
  if (c.item < n_items) c.w = ky_item(p, c.item);
  ky_advance(p, n_items, c, k);
  return c;
}

// Index of key slot j (0..63) of the cursor's tile (-1 past the split's end or the last item).
__device__ __forceinline__ int ky_index(const FwdParams& p, const KyCursor& c, int n_items, int j) {
  if (c.item >= n_items) return -1;
  const int pos = c.w.kbeg + c.t * kKyBN + j;
  return pos < c.w.kend ? __ldg(p.ids + (size_t)c.w.token * p.topk + pos) : -1;
}

__device__ __forceinline__ float ky_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ bool ky_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok) != 0;
}

// Named barrier 1 among the four softmax warps; returns whether `v` held in
// any of their threads.
__device__ __forceinline__ bool soft_vote_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "barrier.red.or.pred p, 1, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void soft_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void st_shared_u16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

__global__ void __launch_bounds__(kKyThreads, 1) fwd_keys_kernel(const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const sbase = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sbase + kKyOffAbort);
  auto bar = [&](int i) -> uint32_t { return base + kKyOffBar + 8u * (uint32_t)i; };
  uint32_t* const mask = reinterpret_cast<uint32_t*>(sbase + kKyOffMask);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kKyStages; ++s) {
      mbar_init(bar(kyFull0 + s), 2);
      mbar_init(bar(kyEmpty0 + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(kySFull0 + b), 1);
      mbar_init(bar(kySFree0 + b), kKySoftWarps);
      mbar_init(bar(kyPFull0 + b), kKySoftWarps);
      mbar_init(bar(kyPvDone0 + b), 1);
    }
    mbar_init(bar(kyQFull), kKySoftWarps);
    mbar_init(bar(kyQFree), 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(base + kKyOffTmemSlot, kKyTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sbase + kKyOffTmemSlot);

  const int n_items = p.tokens * (p.heads / kKyHeads) * p.split;
  const int L = p.length;

  if (warp >= kKyGatherWarp0 && warp < kKyMmaWarp) {
    // ---------------- gather: stage s, keys 32 hf .. 32 hf + 31 of tiles s, s + 2, ... ----------------
    const int gw = warp - kKyGatherWarp0;
    const uint32_t s = (uint32_t)(gw >> 1);
    const int hf = gw & 1;
    const uint32_t stage = base + kKyOffK + s * kKyStage;
    const int j8 = lane & 7;   // 16-byte chunk of a 128-byte block row
    const int kq = lane >> 3;  // row within a group of 4
    KyCursor cur = ky_start(p, n_items, (int)s);
    KyCursor nx = cur;
    ky_advance(p, n_items, nx, kKyStages);
    KyCursor nx2 = nx;
    ky_advance(p, n_items, nx2, kKyStages);
    int idx_cur = ky_index(p, cur, n_items, 32 * hf + lane);
    int idx_nx = ky_index(p, nx, n_items, 32 * hf + lane);
    uint32_t n = 0;
    bool ok = true;
    while (cur.item < n_items) {
      if (n > 0 && !(ok = ky_wait(bar(kyEmpty0 + s), (n - 1) & 1u, abort_flag))) break;
      const int row = checked_index(min(max(idx_cur, 0), L - 1), L, p.status);  // clamped; masked by the softmax
      const uint32_t bits = __ballot_sync(0xffffffffu, (idx_cur >= 0) & (idx_cur < L));
      if (lane == 0) mask[2 * s + hf] = bits;
      const int gb = checked_index(cur.w.batch, p.batch, p.status);
      const __nv_bfloat16* const kv_b = p.kv + (size_t)gb * L * kDimLatent;
      const __nv_bfloat16* const kr_b = p.k_rope + (size_t)gb * L * kDimRope;
#pragma unroll 2
      for (int i = 0; i < 8; ++i) {
        const int k = kq + 4 * i;  // key within this warp's half
        const int rk = __shfl_sync(0xffffffffu, row, k);
        const int krow = 32 * hf + k;
        const uint32_t dst = checked_smem(stage + (uint32_t)krow * 128u + (uint32_t)((j8 ^ (krow & 7)) * 16),
                                          8u * kKyBlk + 16u, stage, kKyStage, p.status);
        const __nv_bfloat16* src = kv_b + (size_t)rk * kDimLatent + j8 * 8;
#pragma unroll
        for (int b = 0; b < 8; ++b) cp_async_16(dst + (uint32_t)b * kKyBlk, src + b * 64);
        cp_async_16(dst + 8u * kKyBlk, kr_b + (size_t)rk * kDimRope + j8 * 8);
      }
      cp_async_commit();
      const int idx_nx2 = ky_index(p, nx2, n_items, 32 * hf + lane);  // consumed one round later
      cp_async_wait<0>();
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kyFull0 + s));
      ++n;
      cur = nx;
      nx = nx2;
      ky_advance(p, n_items, nx2, kKyStages);
      idx_cur = idx_nx;
      idx_nx = idx_nx2;
    }
    if (!ok && lane == 0) report_error(p.status, kErrTimeout);
  } else if (warp == kKyMmaWarp) {
    // ---------------- MMA issuer ----------------
    // Issues whichever is ready, value MMAs first (they free a stage): the
    // value MMAs of the oldest tile whose P is written, or the score MMAs of
    // the next tile once its stage is gathered and its S^T buffer is free.
    // Polling keeps one tile's value MMAs from waiting behind the next
    // tile's gather.
    const uint32_t idesc_qk = idesc_bf16(64, kKyHeads, false, false);
    const uint32_t idesc_pv = idesc_bf16(128, kKyHeads, true, false);
    auto ready = [&](uint32_t b, uint32_t parity) -> bool {  // the same answer in every lane
      const bool r = lane == 0 ? mbar_test(bar((int)b), parity) : false;
      return __shfl_sync(0xffffffffu, r ? 1 : 0, 0) != 0;
    };
    KyCursor cq = ky_start(p, n_items, 0);  // tile of the next score MMAs
    KyCursor cv = cq;                       // tile of the next value MMAs
    uint32_t gq = 0, gv = 0, itq = 0;       // tile counters; items whose Q the issuer has used
    bool q_in = false;                      // the Q of cq's item is loaded
    bool ok = true;
    unsigned long long idle_since = 0;
    while (cv.item < n_items) {
      bool done_any = false;
      if (gv < gq && ready(kyPFull0 + (gv & 1u), (gv >> 1) & 1u)) {
        // O^T += V^T . P^T for tile gv (the item's first tile starts O^T)
        const uint32_t s = gv & 1u;
        const bool first = cv.t == 0;
        tc_fence_after();
        const uint32_t stage = base + kKyOffK + s * kKyStage;
        const uint32_t pbuf = base + kKyOffP + s * kKyPBytes;
        if (elect_one()) {
          // K-step outer, latent block inner: consecutive MMAs accumulate into
          // different O^T blocks
#pragma unroll
          for (int ks = 0; ks < kKyBN / 16; ++ks) {
#pragma unroll
            for (int jb = 0; jb < 4; ++jb) {
              // A = V^T: dims 128jb..128jb+127 (two 64-dim blocks, LBO apart) x
              // keys 16ks..16ks+15 (two 8-key groups, SBO apart), MN-major
              const uint64_t ad = smem_desc(stage + (uint32_t)(2 * jb) * kKyBlk + (uint32_t)ks * 2048u, kKyBlk,
                                            1024, kLayoutSw128);
              const uint64_t bd = smem_desc(pbuf + (uint32_t)ks * 32u, 16, 1024, kLayoutSw128);
              mma_bf16_ss(tmem + kKyTmemO + 16u * (uint32_t)jb, ad, bd, idesc_pv, (first && ks == 0) ? 0u : 1u);
            }
          }
          mma_commit(bar(kyPvDone0 + s));
          mma_commit(bar(kyEmpty0 + s));
        }
        __syncwarp();
        ky_advance(p, n_items, cv, 1);
        ++gv;
        done_any = true;
      } else if (cq.item < n_items) {
        const uint32_t s = gq & 1u;
        if (cq.t == 0 && !q_in) q_in = ready(kyQFull, itq & 1u);
        if ((cq.t > 0 || q_in) && ready(kyFull0 + s, (gq >> 1) & 1u) &&
            (gq < 2 || ready(kySFree0 + s, ((gq >> 1) - 1) & 1u))) {
          tc_fence_after();
          const uint32_t stage = base + kKyOffK + s * kKyStage;
          const bool last = cq.t == cq.w.ntiles - 1;
          if (elect_one()) {
#pragma unroll
            for (int ks = 0; ks < kKyQkSteps; ++ks) {
              const uint64_t ad =
                  smem_desc(stage + (uint32_t)(ks >> 2) * kKyBlk + (uint32_t)(ks & 3) * 32u, 16, 1024, kLayoutSw128);
              const uint64_t bd = smem_desc(base + kKyOffQ + (uint32_t)(ks >> 2) * kKyQBlk + (uint32_t)(ks & 3) * 32u,
                                            16, 1024, kLayoutSw128);
              mma_bf16_ss(tmem + kKyTmemS + 16u * s, ad, bd, idesc_qk, ks > 0 ? 1u : 0u);
            }
            mma_commit(bar(kySFull0 + s));
            if (last) mma_commit(bar(kyQFree));
          }
          __syncwarp();
          if (last) {
            q_in = false;
            ++itq;
          }
          ky_advance(p, n_items, cq, 1);
          ++gq;
          done_any = true;
        }
      }
      if (done_any) {
        idle_since = 0;
      } else {  // bounded: give up after kWaitLimitNs without progress
        if (*abort_flag) {
          ok = false;
          break;
        }
        const unsigned long long now = global_ns();
        if (idle_since == 0) {
          idle_since = now;
        } else if (now - idle_since > kWaitLimitNs) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        __nanosleep(32);  // leave issue slots to the softmax warp on this scheduler
      }
    }
    if (!ok && lane == 0) report_error(p.status, kErrTimeout);
  } else if (warp < kKySoftWarps) {
    // ---------------- softmax + epilogue: thread = key slot 16q + lane (lane < 16) ----------------
    const int q = warp;  // TMEM lane quadrant
    const uint32_t t_lane = (uint32_t)(q * 32) << 16;
    const bool slot = lane < 16;
    const int key = 16 * q + lane;
    const float c = p.scale_log2;
    float* const red_m = reinterpret_cast<float*>(sbase + kKyOffRed);  // tile maxima [4][16]
    float* const red_l = red_m + 64;                                   // item sums [4][16]
    float* const red_e = red_m + 128;                                  // item maxima [4][16]
    const int ctid = threadIdx.x;  // 0..127
    bool ok = true;
    uint32_t g = 0, it = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
      const KyItem w = ky_item(p, item);
      const int h0 = w.hg * kKyHeads;
      // Q of the item's 16 heads -> shared memory (B operand of the score
      // MMAs, 128-byte swizzle); the previous item's score MMAs are done.
      if (it > 0 && ok) ok = ky_wait(bar(kyQFree), (it - 1) & 1u, abort_flag);
      for (int cidx = ctid; cidx < kKyHeads * kKyQChunks; cidx += 32 * kKySoftWarps) {
        const int r = cidx / kKyQChunks, ch = cidx % kKyQChunks;
        const size_t qrow = (size_t)w.token * p.heads + h0 + r;
        const __nv_bfloat16* src = ch < kDimLatent / 8 ? p.q + qrow * kDimLatent + ch * 8
                                                       : p.q_rope + qrow * kDimRope + (ch - kDimLatent / 8) * 8;
        const uint32_t dst = base + kKyOffQ + (uint32_t)(ch >> 3) * kKyQBlk + (uint32_t)r * 128u +
                             (uint32_t)(((ch & 7) ^ (r & 7)) * 16);
        cp_async_16(dst, src);
      }
      cp_async_commit();
      cp_async_wait<0>();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kyQFull));

      float mu[kKyHeads], lp[kKyHeads], mt[kKyHeads];
#pragma unroll
      for (int h = 0; h < kKyHeads; ++h) {
        mu[h] = kNegFltMax;  // finite start, as dsa/workspace.py:68
        lp[h] = 0.f;
        mt[h] = kNegFltMax;
      }
      for (int t = 0; t < w.ntiles; ++t, ++g) {
        const uint32_t s = g & 1u;
        float x[kKyHeads];
        if (ok) ok = ky_wait(bar(kySFull0 + s), (g >> 1) & 1u, abort_flag);
        {
          uint32_t sv[kKyHeads];
          tc_fence_after();
          tmem_ld16(tmem + t_lane + kKyTmemS + 16u * s, sv);
          tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < kKyHeads; ++h) x[h] = __uint_as_float(sv[h]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kySFree0 + s));
        if (ok) ok = ky_wait(bar(kyFull0 + s), (g >> 1) & 1u, abort_flag);  // the tile's validity bits
        const bool valid = slot && ((mask[2 * s + (q >> 1)] >> (key & 31)) & 1u);
        bool need = false;
#pragma unroll
        for (int h = 0; h < kKyHeads; ++h) {
          x[h] = valid ? x[h] : -INFINITY;
          mt[h] = fmaxf(mt[h], x[h]);
          need |= (x[h] - mu[h]) * c > 8.f;
        }
        if (soft_vote_any(need)) {
          // a head's max grew past the lazy threshold: per-head max of the
          // tile over the 64 keys (lanes 16..31 hold -inf)
          float tm[kKyHeads];
#pragma unroll
          for (int h = 0; h < kKyHeads; ++h) {
            float v = x[h];
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
            tm[h] = v;
          }
#pragma unroll
          for (int h = 0; h < kKyHeads; ++h)
            if (lane == h) red_m[q * 16 + h] = tm[h];
          soft_sync();
          float alpha[kKyHeads];
          bool resc = false;
#pragma unroll
          for (int h = 0; h < kKyHeads; ++h) {
            const float mx = fmaxf(fmaxf(red_m[h], red_m[16 + h]), fmaxf(red_m[32 + h], red_m[48 + h]));
            const float m_new = (mx - mu[h]) * c > 8.f ? mx : mu[h];
            alpha[h] = m_new == mu[h] ? 1.f : ky_ex2((mu[h] - m_new) * c);
            resc |= m_new != mu[h];
            lp[h] *= alpha[h];
            mu[h] = m_new;
          }
          if (resc && t > 0) {  // the same in every softmax thread
            // O^T holds the value MMAs of tiles before g: rescale its column h by alpha[h]
            if (ok) ok = ky_wait(bar(kyPvDone0 + ((g - 1) & 1u)), ((g - 1) >> 1) & 1u, abort_flag);
            tc_fence_after();
#pragma unroll 1
            for (int jb = 0; jb < 4; ++jb) {
              uint32_t o[kKyHeads];
              const uint32_t a = tmem + t_lane + kKyTmemO + 16u * (uint32_t)jb;
              tmem_ld16(a, o);
              tmem_wait_ld();
#pragma unroll
              for (int h = 0; h < kKyHeads; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * alpha[h]);
              tmem_st16(a, o);
            }
            tmem_wait_st();
          }
        }
        // P of this key for the 16 heads -> P^T buffer s (K-major: one
        // 128-byte row of 64 keys per head, 128-byte swizzle)
        float pr[kKyHeads];
#pragma unroll
        for (int h = 0; h < kKyHeads; ++h) {
          pr[h] = ky_ex2(fmaf(x[h], c, -mu[h] * c));
          lp[h] += pr[h];
        }
        if (g >= 2 && ok) ok = ky_wait(bar(kyPvDone0 + s), ((g >> 1) - 1) & 1u, abort_flag);
        if (slot) {
          const uint32_t pbuf = base + kKyOffP + s * kKyPBytes;
#pragma unroll
          for (int h = 0; h < kKyHeads; ++h) {
            const uint32_t addr = pbuf + (uint32_t)h * 128u + (uint32_t)((((key >> 3) ^ (h & 7))) * 16) +
                                  (uint32_t)(key & 7) * 2u;
            const __nv_bfloat16 b = __float2bfloat16_rn(pr[h]);
            st_shared_u16(addr, *reinterpret_cast<const uint16_t*>(&b));
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kyPFull0 + s));
      }

      // ---- epilogue: sums and true maxima over the 64 key slots ----
#pragma unroll
      for (int h = 0; h < kKyHeads; ++h) {
        float lv = lp[h], mv = mt[h];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) {
          lv += __shfl_xor_sync(0xffffffffu, lv, o);
          mv = fmaxf(mv, __shfl_xor_sync(0xffffffffu, mv, o));
        }
        if (lane == h) {
          red_l[q * 16 + h] = lv;
          red_e[q * 16 + h] = mv;
        }
      }
      soft_sync();
      float l[kKyHeads], f[kKyHeads];
      float mtr[kKyHeads];
#pragma unroll
      for (int h = 0; h < kKyHeads; ++h) {
        l[h] = ((red_l[h] + red_l[16 + h]) + red_l[32 + h]) + red_l[48 + h];
        mtr[h] = fmaxf(fmaxf(red_e[h], red_e[16 + h]), fmaxf(red_e[32 + h], red_e[48 + h]));
        f[h] = mtr[h] == kNegFltMax ? 1.f : ky_ex2((mu[h] - mtr[h]) * c);
      }
      soft_sync();  // red_* are read before the next item's votes write them
      if (ok) ok = ky_wait(bar(kyPvDone0 + ((g - 1) & 1u)), ((g - 1) >> 1) & 1u, abort_flag);
      tc_fence_after();
#pragma unroll 1
      for (int jb = 0; jb < 4; ++jb) {
        uint32_t o[kKyHeads];
        tmem_ld16(tmem + t_lane + kKyTmemO + 16u * (uint32_t)jb, o);
        tmem_wait_ld();
        const int dim = 128 * jb + 32 * q + lane;
        if (p.split == 1) {
          __nv_bfloat16* dst = p.out + ((size_t)w.token * p.heads + h0) * kDimLatent + dim;
#pragma unroll
          for (int h = 0; h < kKyHeads; ++h) {
            // correctly rounded reciprocal; a row without a valid index (l == 0) is written as 0
            const float rl = l[h] > 0.f ? __frcp_rn(l[h]) : 0.f;
            dst[(size_t)h * kDimLatent] = __float2bfloat16_rn(__uint_as_float(o[h]) * rl);
          }
        } else {
          float* dst = p.part_num + (((size_t)w.token * p.split + w.sp) * p.heads + h0) * kDimLatent + dim;
#pragma unroll
          for (int h = 0; h < kKyHeads; ++h) dst[(size_t)h * kDimLatent] = __uint_as_float(o[h]) * f[h];
        }
      }
      if (q == 0) {
#pragma unroll
        for (int h = 0; h < kKyHeads; ++h) {
          if (lane != h) continue;
          if (p.split == 1) {
            const size_t orow = (size_t)w.token * p.heads + h0 + h;
            p.out_max[orow] = final_max(mtr[h], l[h], p.scale_div);
            p.out_sum[orow] = l[h] * f[h];
          } else {
            const size_t prow = ((size_t)w.token * p.split + w.sp) * p.heads + h0 + h;
            p.part_max[prow] = mtr[h] == kNegFltMax ? kNegFltMax : __fdiv_rn(mtr[h], p.scale_div);
            p.part_sum[prow] = l[h] * f[h];
          }
        }
      }
      tc_fence_before();
    }
    if (!ok && lane == 0) report_error(p.status, kErrTimeout);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kKyTmemCols);
  }
}

}  // namespace

int keys_max_ctas() {
  static int cached = -1;
  if (cached > 0) return cached;
  if (cudaFuncSetAttribute(fwd_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kKySmemBytes) !=
      cudaSuccess)
    return -1;
  int per_sm = 0, dev = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fwd_keys_kernel, kKyThreads, kKySmemBytes) !=
          cudaSuccess ||
      per_sm <= 0)
    return -1;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return -1;
  cached = per_sm * sms;
  return cached;
}

cudaError_t launch_fwd_keys(const FwdParams& p, cudaStream_t stream) {
  if (p.heads % kKyHeads != 0 || p.keys_per_tile != kKyBN) return cudaErrorInvalidValue;
  const int max_ctas = keys_max_ctas();
  if (max_ctas <= 0) return cudaErrorInvalidConfiguration;
  const long long items = (long long)p.tokens * (p.heads / kKyHeads) * p.split;
  if (items <= 0 || items > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  const int ctas = (int)(items < max_ctas ? items : max_ctas);
  fwd_keys_kernel<<<ctas, kKyThreads, kKySmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace dsa
