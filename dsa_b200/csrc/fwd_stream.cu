// Persistent warp-specialised sparse-MLA forward for 16-head groups (the
// "stream" family: any H % 16 == 0, BN = 32 selected rows per tile).
//
// Built for the shapes where few heads share each gathered row (H = 16 at
// TP8): the math per row is small, so the kernel is bound by how many
// gathered bytes are in flight (decode, rows from HBM) or by the L2 gather
// rate (prefill with an L2-resident KV). Each CTA loops over work items
// (token, 16-head group, KV split). Gathered rows land in a ring of 16-row
// units (a 32-key tile is two units): two gather warps, one per tile half,
// fill the units with 16-byte cp.async (validity taken from the original
// index, dsa/workspace.py:121-128) that complete on the unit's mbarrier, so
// a warp runs ahead of the compute warps as far as the ring allows; two CTAs
// share an SM. The ring has four units in the stage buffers plus, in the
// cluster-merge launch (one item per CTA), a fifth in the Q buffer once the
// compute warps hold Q in registers: up to 2.5 tiles of rows gathered ahead
// instead of two (the rows' latency sets the tile rate when they come from
// HBM).
//
// The four compute warps run the reference's per-tile dataflow
// (dsa/workspace.py:242-318) with warp-level m16n8k16 BF16 MMAs: S = Q.K^T
// (warp w owns dims 144w..144w+143 for all 32 keys and keeps its Q slice in
// registers for the whole item; the four partial scores are added in shared
// memory, so Q is read from shared memory once per item and every gathered
// element once per tile), masked FP32 online softmax (scale 1/24,
// invalid index -> -inf), P rounded to BF16, O += P.V (warp w owns latent
// columns 128w..128w+127, O stays in registers for the item), then the BF16
// output and stats (split == 1) or FP32 partials for the merge (split > 1,
// dsa/workspace.py:356-385).
//
// Synchronisation: stage full / empty mbarriers between the gather and the
// compute warps (every wait bounded, reporting through the status word), and
// a named barrier among the four compute warps only (two per tile); the
// compute warps take every named barrier in the same order and leave
// together, after the tile's last barrier, when a bounded wait gives up.
#include "umma_ptx.cuh"

namespace dsa {
namespace {

using namespace umma;

constexpr int kStHeads = 16;
constexpr int kStBN = 32;
constexpr int kStStages = 2;             // 32-row stage buffers (four 16-row units)
constexpr int kStUnitRows = 16;          // rows per ring unit (one half of a tile)
constexpr int kStGatherWarps = 2;        // gather warp w fills rows 16w..16w+15 of every tile
constexpr int kStMaxUnits = 2 * kStStages + 1;  // the fifth unit is the Q buffer (cluster-merge launch)
constexpr int kStComputeWarps = 4;
constexpr int kStThreads = 32 * (kStGatherWarps + kStComputeWarps);
constexpr int kStRow = kDimQK + 8;       // padded smem row (elements): 1168 B, odd multiple of 16 B
constexpr int kStPRow = kStBN + 8;
constexpr int kChunks = kDimQK / 8;      // 72 x 16 B per gathered row
constexpr int kLatChunks = kDimLatent / 8;

struct StSmem {
  __nv_bfloat16 q[kStHeads * kStRow];
  __nv_bfloat16 k[kStStages][kStBN * kStRow];
  __nv_bfloat16 p[kStHeads * kStPRow];
  float s[kStComputeWarps][kStHeads * kStBN];  // partial scores of each compute warp's dims
  int ids[kStMaxUnits][kStUnitRows];
  float m[kStHeads];
  float l[kStHeads];
  float alpha[kStHeads];
  unsigned long long full[kStMaxUnits];   // unit gathered (32 cp.async arrivals, one per gather lane)
  unsigned long long empty[kStMaxUnits];  // unit consumed (the four compute warps)
  int abort;
  int stop;  // a compute warp's bounded wait gave up: all compute warps leave
};

constexpr uint32_t kStUnitBytes = (uint32_t)(kStUnitRows * kStRow * 2);
static_assert(sizeof(StSmem::q) == kStUnitBytes, "the Q buffer doubles as one ring unit");
static_assert(sizeof(StSmem::k) == 2 * kStStages * kStUnitBytes, "the stage buffers hold four ring units");

// Ring units of a launch: the Q buffer is the fifth unit only when every CTA
// runs one item (its Q is loaded once, into registers).
template <bool kCM>
constexpr uint32_t st_units() {
  return kCM ? (uint32_t)kStMaxUnits : (uint32_t)(2 * kStStages);
}

__device__ __forceinline__ uint32_t st_unit_addr(const StSmem& sm, uint32_t u) {
  return u < (uint32_t)(2 * kStStages) ? smem_u32(sm.k) + u * kStUnitBytes : smem_u32(sm.q);
}

struct StItem {
  int token, hg, sp, batch, kbeg, kend, ntiles;
};

__device__ __forceinline__ StItem st_item(const FwdParams& p, int item) {
  const int hgroups = p.heads / kStHeads;
  StItem it;
  it.sp = item % p.split;
  int rest = item / p.split;
  it.hg = rest % hgroups;
  it.token = rest / hgroups;
  it.batch = it.token / p.queries;
  split_bounds(p.topk, kStBN, p.split, it.sp, &it.kbeg, &it.kend);
  it.ntiles = (it.kend - it.kbeg + kStBN - 1) / kStBN;
  return it;
}

// Position of one tile in this CTA's sequence (items blockIdx.x, +gridDim.x, ...).
struct StCursor {
  int item, t;
  StItem w;
};

__device__ __forceinline__ void st_advance(const FwdParams& p, int n_items, StCursor& c, int k) {
  c.t += k;
  while (c.item < n_items && c.t >= c.w.ntiles) {
    c.t -= c.w.ntiles;
    c.item += gridDim.x;
    if (c.item < n_items) c.w = st_item(p, c.item);
  }
}

__device__ __forceinline__ StCursor st_start(const FwdParams& p, int n_items, int k) {
  StCursor c;
  c.item = blockIdx.x;
  c.t = 0;
  if (c.item < n_items) c.w = st_item(p, c.item);
  st_advance(p, n_items, c, k);
  return c;
}

__device__ __forceinline__ int st_index(const FwdParams& p, const StCursor& c, int n_items, int lane) {
  if (c.item >= n_items) return -1;
  const int j = c.w.kbeg + c.t * kStBN + lane;
  return j < c.w.kend ? __ldg(p.ids + (size_t)c.w.token * p.topk + j) : -1;
}

// 2^x on the special-function unit (flushes results below 2^-126 to zero,
// far below what the FP32 row sums can resolve).
__device__ __forceinline__ float ex2f_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void compute_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kStComputeWarps) : "memory");
}

// Split merge inside the cluster-merge launch: the `split` CTAs of one
// (token, 16-head group) form a cluster, one item each, and after their
// partials (dsa/api.py:111-113 layout) are in the L2 and one cluster
// barrier, CTA rank r merges heads [16 r / S, 16 (r + 1) / S) of the group:
// the merge of dsa/merge.py:13-91 (as merge_kernel: M = max m_s,
// w_s = exp(m_s - M), L = sum w_s l_s, O = sum w_s u_s / L, splits in
// order), one warp per head row, lane i owning columns 4i + 128j. Every
// thread of every CTA takes the barrier, also after a failed wait (it then
// skips the work).
__device__ __forceinline__ void stream_cluster_merge(const FwdParams& p, bool live) {
  cluster_sync();  // every split's partials of the cluster are in the L2
  if (!live) return;
  const int S = p.split;
  const int item = (int)blockIdx.x;
  const int sp = item % S;
  const int rest = item / S;
  const int hgroups = p.heads / kStHeads;
  const int hg = rest % hgroups, token = rest / hgroups;
  const int r0 = sp * kStHeads / S, r1 = (sp + 1) * kStHeads / S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = r0 + warp; r < r1; r += kStThreads / 32) {
    const int h = hg * kStHeads + r;
    const size_t stat0 = (size_t)token * S * p.heads + h;  // + s * heads
    const float ms = lane < S ? __ldcg(p.part_max + stat0 + (size_t)lane * p.heads) : -INFINITY;
    const float ls = lane < S ? __ldcg(p.part_sum + stat0 + (size_t)lane * p.heads) : 0.f;
    float m = ms;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float ws = lane < S ? expf(ms - m) : 0.f;
    float l = ws * ls;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    float4 u[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) u[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < S; s0 += 4) {  // four splits' rows in flight
      float4 v[4][4];
#pragma unroll
      for (int b = 0; b < 4; ++b)
        if (s0 + b < S) {
          const float4* row =
              reinterpret_cast<const float4*>(p.part_num + (stat0 + (size_t)(s0 + b) * p.heads) * kDimLatent) + lane;
#pragma unroll
          for (int j = 0; j < 4; ++j) v[b][j] = __ldcg(row + 32 * j);
        }
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const float wb = __shfl_sync(0xffffffffu, ws, (s0 + b) & 31);
        if (s0 + b < S) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            u[j].x += wb * v[b][j].x;
            u[j].y += wb * v[b][j].y;
            u[j].z += wb * v[b][j].z;
            u[j].w += wb * v[b][j].w;
          }
        }
      }
    }
    const float ld = l > 0.f ? l : INFINITY;  // no valid index in any split: output 0
    __nv_bfloat16* const orow = p.out + ((size_t)token * p.heads + h) * kDimLatent;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint2 packed;
      packed.x = pack_bf16x2(__fdiv_rn(u[j].x, ld), __fdiv_rn(u[j].y, ld));
      packed.y = pack_bf16x2(__fdiv_rn(u[j].z, ld), __fdiv_rn(u[j].w, ld));
      *reinterpret_cast<uint2*>(orow + 4 * lane + 128 * j) = packed;
    }
    if (lane == 0) {
      p.out_max[(size_t)token * p.heads + h] = l > 0.f ? m : -INFINITY;
      p.out_sum[(size_t)token * p.heads + h] = l;
    }
  }
}

// kCM: the cluster-merge launch (one item per CTA, the split CTAs of a
// (token, head group) as one cluster, stream_cluster_merge at the end);
// otherwise persistent CTAs and merge_kernel for split > 1.
template <bool kCM>
__global__ void __launch_bounds__(kStThreads, 2) fwd_stream_kernel(const FwdParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  StSmem& sm = *reinterpret_cast<StSmem*>(smem_raw);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int n_items = p.tokens * (p.heads / kStHeads) * p.split;
  const int L = p.length;
  volatile int* abort_flag = &sm.abort;
  const uint32_t full0 = smem_u32(&sm.full[0]);
  const uint32_t empty0 = smem_u32(&sm.empty[0]);

  if (tid == 0) {
    for (int u = 0; u < kStMaxUnits; ++u) {
      mbar_init(full0 + 8u * u, 32);  // one cp.async arrival per gather lane
      mbar_init(empty0 + 8u * u, kStComputeWarps);
    }
    sm.abort = 0;
    sm.stop = 0;
    fence_barrier_init();
  }
  __syncthreads();

  constexpr uint32_t kUnits = st_units<kCM>();
  if (warp < kStGatherWarps) {
    // ---------------- gather: warp hw fills rows 16 hw..16 hw + 15 of every tile ----------------
    // Unit n = 2 gt + hw of the CTA's sequence goes to ring unit n % kUnits.
    // A unit is free once the compute warps consumed its previous contents
    // (the Q unit: once they hold Q in registers); the warp does not wait for
    // its own copies, which complete on the unit's full barrier.
    const int hw = warp;
    const int j8 = lane & 7;  // 16-byte chunk within a 128-byte run
    const int kq = lane >> 3;  // row within a group of 4
    StCursor cur = st_start(p, n_items, 0);
    StCursor nx = cur;
    st_advance(p, n_items, nx, 1);
    StCursor nx2 = nx;
    st_advance(p, n_items, nx2, 1);
    int idx_cur = st_index(p, cur, n_items, lane);
    int idx_nx = st_index(p, nx, n_items, lane);
    bool ok = true;
    for (uint32_t gt = 0; cur.item < n_items; ++gt) {
      const uint32_t n = 2u * gt + (uint32_t)hw;
      const uint32_t u = n % kUnits, use = n / kUnits;
      const bool q_unit = u == (uint32_t)(2 * kStStages);  // only in the cluster-merge launch
      if (use > 0 || q_unit) {
        if (lane == 0) ok = mbar_wait(empty0 + 8u * u, (q_unit ? use : use - 1u) & 1u, abort_flag);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
      if ((lane >> 4) == hw) sm.ids[u][lane & 15] = idx_cur;  // validity is judged from the original index
      const int row = checked_index(min(max(idx_cur, 0), L - 1), L, p.status);
      const int gb = checked_index(cur.w.batch, p.batch, p.status);
      const __nv_bfloat16* kv_b = p.kv + (size_t)gb * L * kDimLatent;
      const __nv_bfloat16* kr_b = p.k_rope + (size_t)gb * L * kDimRope;
      const uint32_t unit = st_unit_addr(sm, u);
#pragma unroll 2
      for (int i = 0; i < kStUnitRows / 4; ++i) {
        const int key = kq + 4 * i;  // row of the unit
        const int rk = __shfl_sync(0xffffffffu, row, 16 * hw + key);
        const uint32_t dst = checked_smem(unit + (uint32_t)(key * kStRow + j8 * 8) * 2u, 8u * 128u + 16u, unit,
                                          kStUnitBytes, p.status);
        const __nv_bfloat16* src = kv_b + (size_t)rk * kDimLatent + j8 * 8;
#pragma unroll
        for (int kb = 0; kb < 8; ++kb) cp_async_16(dst + kb * 128u, src + kb * 64);
        cp_async_16(dst + 8u * 128u, kr_b + (size_t)rk * kDimRope + j8 * 8);
      }
      cp_async_mbar_arrive_noinc(full0 + 8u * u);
      const int idx_nx2 = st_index(p, nx2, n_items, lane);  // consumed two tiles later
      cur = nx;
      nx = nx2;
      st_advance(p, n_items, nx2, 1);
      idx_cur = idx_nx;
      idx_nx = idx_nx2;
    }
    cp_async_wait_all();  // no copy into this CTA's shared memory outlives the warp
    if (!ok && lane == 0) report_error(p.status, kErrTimeout);
    if constexpr (kCM) stream_cluster_merge(p, !(*abort_flag) && !*reinterpret_cast<volatile int*>(&sm.stop));
    return;
  }

  // ---------------- compute warps ----------------
  const int ctid = tid - 32 * kStGatherWarps;  // 0..127
  const int cw = ctid >> 5;                    // compute warp 0..3
  const int g = lane >> 2;                     // mma group id (row within 8)
  const int tq = lane & 3;                     // thread in group
  uint32_t gt = 0;                             // tile counter of this CTA
  bool failed = false;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const StItem w = st_item(p, item);
    const int h0 = w.hg * kStHeads;
    // Q tile [16 heads x (512 | 64)] -> smem; the previous item's readers are done.
    compute_sync();
    for (int c = ctid; c < kStHeads * kChunks; c += 32 * kStComputeWarps) {
      const int r = c / kChunks, part = c % kChunks;
      const size_t qrow = (size_t)w.token * p.heads + h0 + r;
      const __nv_bfloat16* src = part < kLatChunks ? p.q + qrow * kDimLatent + part * 8
                                                   : p.q_rope + qrow * kDimRope + (part - kLatChunks) * 8;
      cp_async_16(smem_u32(&sm.q[r * kStRow + part * 8]), src);
    }
    cp_async_commit();
    if (ctid < kStHeads) {
      sm.m[ctid] = kNegFltMax;  // finite start, as dsa/workspace.py:68
      sm.l[ctid] = 0.f;
    }
    cp_async_wait<0>();
    compute_sync();
    // this warp's Q slice (dims 144cw..144cw+143) as m16n8k16 A fragments
    constexpr int kQkSteps = kDimQK / 16 / kStComputeWarps;  // 9
    uint32_t qf[kQkSteps][4];
    {
      const uint32_t qbase = smem_u32(sm.q) +
                             (((lane & 7) + ((lane >> 3) & 1) * 8) * kStRow + (lane >> 4) * 8 + cw * 16 * kQkSteps) * 2;
#pragma unroll
      for (int ks = 0; ks < kQkSteps; ++ks) ldmatrix_x4(qbase + ks * 32, qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
    }
    if constexpr (kCM) {  // the Q buffer becomes the ring's fifth unit (the CTA's only item)
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8u * (uint32_t)(2 * kStStages));
    }

    float acc[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

    for (int t = 0; t < w.ntiles; ++t, ++gt) {
      // the tile's two units (keys 0..15 in ua, 16..31 in ub)
      const uint32_t n0 = 2u * gt, n1 = n0 + 1u;
      const uint32_t ua = n0 % kUnits, ub = n1 % kUnits;
      const uint32_t unit_a = st_unit_addr(sm, ua), unit_b = st_unit_addr(sm, ub);
      // units full: every compute warp waits (bounded); a warp that gives up
      // flags it and still takes this tile's barriers, and all leave after
      // the last one
      if (!mbar_wait(full0 + 8u * ua, (n0 / kUnits) & 1u, abort_flag) ||
          !mbar_wait(full0 + 8u * ub, (n1 / kUnits) & 1u, abort_flag))
        sm.stop = 1;

      // ---- partial S = Q.K^T over this warp's dims, all 32 keys ----
      {
        float d[kStBN / 8][4];
#pragma unroll
        for (int nt = 0; nt < kStBN / 8; ++nt) d[nt][0] = d[nt][1] = d[nt][2] = d[nt][3] = 0.f;
        // ldmatrix_x4 over 8 keys x 32 dims: b0,b1 = k-step 2j, b2,b3 = k-step 2j+1
        const uint32_t koff = (uint32_t)((lane & 7) * kStRow + (lane >> 3) * 8 + cw * 16 * kQkSteps) * 2u;
#pragma unroll
        for (int nt = 0; nt < kStBN / 8; ++nt) {
          // keys 8 nt..8 nt + 7: rows 8 (nt % 2).. of unit a (nt < 2) or b
          const uint32_t kbase = (nt < 2 ? unit_a : unit_b) + koff + (uint32_t)((nt & 1) * 8 * kStRow) * 2u;
#pragma unroll
          for (int j = 0; j < kQkSteps / 2; ++j) {
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4(kbase + (j * 32) * 2, b0, b1, b2, b3);
            mma_bf16_16816(d[nt], qf[2 * j][0], qf[2 * j][1], qf[2 * j][2], qf[2 * j][3], b0, b1);
            mma_bf16_16816(d[nt], qf[2 * j + 1][0], qf[2 * j + 1][1], qf[2 * j + 1][2], qf[2 * j + 1][3], b2, b3);
          }
          // odd step count: the last 16 dims with an x2 load (8 keys x 16 dims)
          uint32_t b0, b1;
          ldmatrix_x2(kbase + ((kQkSteps - 1) * 16) * 2, b0, b1);
          mma_bf16_16816(d[nt], qf[kQkSteps - 1][0], qf[kQkSteps - 1][1], qf[kQkSteps - 1][2],
                         qf[kQkSteps - 1][3], b0, b1);
        }
        float* const sp = sm.s[cw];
#pragma unroll
        for (int nt = 0; nt < kStBN / 8; ++nt) {
          const int col = nt * 8 + tq * 2;
          *reinterpret_cast<float2*>(&sp[g * kStBN + col]) = make_float2(d[nt][0], d[nt][1]);
          *reinterpret_cast<float2*>(&sp[(g + 8) * kStBN + col]) = make_float2(d[nt][2], d[nt][3]);
        }
      }
      compute_sync();

      // ---- online softmax: 8 threads per head row ----
      {
        // raw (unscaled) scores; exp(s / d - m) = 2^(s * c - m * c) with
        // c = log2(e) / d, d = scale_div (24 for the reference's scale)
        const float c = p.scale_log2;
        constexpr int kCols = kStBN / 8;
        const int r = ctid >> 3;
        const int c0 = (ctid & 7) * kCols;
        const float m_old = sm.m[r];
        const float l_old = sm.l[r];
        __syncwarp();
        float x[kCols];
        float mx = -INFINITY;
        static_assert(kStUnitRows % kCols == 0, "a thread's columns lie in one unit");
        const int* const ids_c = c0 < kStUnitRows ? &sm.ids[ua][c0] : &sm.ids[ub][c0 - kStUnitRows];
#pragma unroll
        for (int i = 0; i < kCols; ++i) {
          const int col = c0 + i;
          const float sc = sm.s[0][r * kStBN + col] + sm.s[1][r * kStBN + col] + sm.s[2][r * kStBN + col] +
                           sm.s[3][r * kStBN + col];
          const int id = ids_c[i];
          x[i] = ((id >= 0) & (id < L)) ? sc : -INFINITY;
          mx = fmaxf(mx, x[i]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        const float m_new = fmaxf(m_old, mx);
        const float alpha = m_new == m_old ? 1.f : ex2f_approx((m_old - m_new) * c);
        const float mc = m_new * c;
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < kCols; i += 2) {
          const float p0 = ex2f_approx(fmaf(x[i], c, -mc));
          const float p1 = ex2f_approx(fmaf(x[i + 1], c, -mc));
          sum += p0 + p1;
          *reinterpret_cast<uint32_t*>(&sm.p[r * kStPRow + c0 + i]) = pack_bf16x2(p0, p1);
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        if ((ctid & 7) == 0) {
          sm.m[r] = m_new;
          sm.l[r] = alpha * l_old + sum;
          sm.alpha[r] = alpha;
        }
      }
      compute_sync();

      // ---- O = alpha*O + P.V over this warp's 128 latent columns ----
      {
        const float al0 = sm.alpha[g], al1 = sm.alpha[g + 8];
        if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {  // a row max grew
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            acc[j][0] *= al0;
            acc[j][1] *= al0;
            acc[j][2] *= al1;
            acc[j][3] *= al1;
          }
        }
        const uint32_t pbase =
            smem_u32(sm.p) + (((lane & 7) + ((lane >> 3) & 1) * 8) * kStPRow + (lane >> 4) * 8) * 2;
        const uint32_t voff =
            (uint32_t)((((lane & 7) + ((lane >> 3) & 1) * 8) * kStRow + cw * 128 + (lane >> 4) * 8) * 2);
#pragma unroll
        for (int kk = 0; kk < kStBN / 16; ++kk) {  // keys 16 kk..16 kk + 15: unit a, then b
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4(pbase + kk * 32, a0, a1, a2, a3);
          const uint32_t vbase = (kk == 0 ? unit_a : unit_b) + voff;
#pragma unroll
          for (int jp = 0; jp < 8; ++jp) {
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4_trans(vbase + (jp * 16) * 2, b0, b1, b2, b3);
            mma_bf16_16816(acc[2 * jp], a0, a1, a2, a3, b0, b1);
            mma_bf16_16816(acc[2 * jp + 1], a0, a1, a2, a3, b2, b3);
          }
        }
      }
      // this warp is done with the tile's units
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(empty0 + 8u * ua);
        mbar_arrive(empty0 + 8u * ub);
      }
      if (*reinterpret_cast<volatile int*>(&sm.stop)) {  // set before the softmax barrier
        failed = true;
        break;
      }
    }
    if (failed) break;

    // ---- epilogue (sm.m / sm.l final after the last softmax barrier) ----
    const float l0 = sm.l[g], l1 = sm.l[g + 8];
    if (p.split == 1) {
      // a row without a valid index (l == 0, O == 0) is written as 0 (O / inf)
      const float d0 = l0 > 0.f ? l0 : INFINITY, d1 = l1 > 0.f ? l1 : INFINITY;
      __nv_bfloat16* o0 = p.out + ((size_t)w.token * p.heads + h0 + g) * kDimLatent + cw * 128 + tq * 2;
      __nv_bfloat16* o1 = o0 + 8 * kDimLatent;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        *reinterpret_cast<uint32_t*>(o0 + j * 8) = pack_bf16x2(__fdiv_rn(acc[j][0], d0), __fdiv_rn(acc[j][1], d0));
        *reinterpret_cast<uint32_t*>(o1 + j * 8) = pack_bf16x2(__fdiv_rn(acc[j][2], d1), __fdiv_rn(acc[j][3], d1));
      }
      if (ctid < kStHeads) {
        const float mr = sm.m[ctid];
        p.out_max[(size_t)w.token * p.heads + h0 + ctid] = final_max(mr, sm.l[ctid], p.scale_div);
        p.out_sum[(size_t)w.token * p.heads + h0 + ctid] = sm.l[ctid];
      }
    } else {
      const size_t prow = ((size_t)w.token * p.split + w.sp) * p.heads + h0;
      float* n0 = p.part_num + (prow + g) * kDimLatent + cw * 128 + tq * 2;
      float* n1 = n0 + 8 * kDimLatent;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        *reinterpret_cast<float2*>(n0 + j * 8) = make_float2(acc[j][0], acc[j][1]);
        *reinterpret_cast<float2*>(n1 + j * 8) = make_float2(acc[j][2], acc[j][3]);
      }
      if (ctid < kStHeads) {
        const float mr = sm.m[ctid];
        p.part_max[prow + ctid] = mr == kNegFltMax ? mr : __fdiv_rn(mr, p.scale_div);
        p.part_sum[prow + ctid] = sm.l[ctid];
      }
    }
  }
  if (failed && ctid == 0) report_error(p.status, kErrTimeout);
  if constexpr (kCM) stream_cluster_merge(p, !(*abort_flag) && !*reinterpret_cast<volatile int*>(&sm.stop));
}

}  // namespace

int stream_max_ctas() {
  static int cached = -1;
  if (cached > 0) return cached;
  const int smem = (int)sizeof(StSmem);
  if (cudaFuncSetAttribute(fwd_stream_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return -1;
  int per_sm = 0, dev = 0, sms = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fwd_stream_kernel<false>, kStThreads, smem) !=
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

constexpr int kStMaxClusterSplit = 8;  // portable cluster sizes only

void st_cm_launch_config(cudaLaunchConfig_t* cfg, cudaLaunchAttribute* attr, int split, long long ctas,
                         cudaStream_t stream) {
  attr->id = cudaLaunchAttributeClusterDimension;
  attr->val.clusterDim.x = (unsigned)split;
  attr->val.clusterDim.y = 1;
  attr->val.clusterDim.z = 1;
  *cfg = cudaLaunchConfig_t{};
  cfg->gridDim = dim3((unsigned)ctas, 1, 1);
  cfg->blockDim = dim3(kStThreads, 1, 1);
  cfg->dynamicSmemBytes = sizeof(StSmem);
  cfg->stream = stream;
  cfg->attrs = attr;
  cfg->numAttrs = 1;
}

}  // namespace

// Whether the stream family merges `split` partials in its cluster launch:
// a portable cluster size whose clusters fit on the GPU (they may run in
// waves: clusters do not wait on one another).
bool stream_cluster_merge(int split) {
  static int cached[kStMaxClusterSplit + 1];
  static bool init = false;
  if (split < 2 || split > kStMaxClusterSplit) return false;
  if (!init) {
    if (cudaFuncSetAttribute(fwd_stream_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(StSmem)) != cudaSuccess)
      return false;
    for (int k = 0; k <= kStMaxClusterSplit; ++k) cached[k] = -1;
    init = true;
  }
  if (cached[split] < 0) {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr;
    st_cm_launch_config(&cfg, &attr, split, split, nullptr);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fwd_stream_kernel<true>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    cached[split] = n;
  }
  return cached[split] > 0;
}

cudaError_t launch_fwd_stream(const FwdParams& p, cudaStream_t stream) {
  if (p.heads % kStHeads != 0 || p.keys_per_tile != kStBN) return cudaErrorInvalidValue;
  const long long items = (long long)p.tokens * (p.heads / kStHeads) * p.split;
  if (items <= 0 || items > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  if (p.split > 1 && stream_cluster_merge(p.split)) {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr;
    st_cm_launch_config(&cfg, &attr, p.split, items, stream);
    return cudaLaunchKernelEx(&cfg, fwd_stream_kernel<true>, p);
  }
  const int max_ctas = stream_max_ctas();
  if (max_ctas <= 0) return cudaErrorInvalidConfiguration;
  const int ctas = (int)(items < max_ctas ? items : max_ctas);
  fwd_stream_kernel<false><<<ctas, kStThreads, sizeof(StSmem), stream>>>(p);
  return cudaGetLastError();
}

}  // namespace dsa
