// tcgen05/TMEM sparse-MLA forward for H = 128 heads on a pair of SMs (the
// "pair" family).
//
// A thread-block cluster of two CTAs owns one work item (token, KV split) at
// a time and walks its selected rows in tiles of 32. The two CTAs split the
// work by operation, so no MMA is computed twice:
//
//   score CTA (rank 0)  S = Q . K^T         tcgen05, M=128 heads, N=32 keys, K=576,
//                                           A = Q held in TMEM (all 576 dims)
//                       P = bf16(exp(S/24 - m)), FP32 online softmax (thread = head row)
//                       P, the per-row rescale factor and a per-warp rescale flag are
//                       staged in the score CTA's shared memory and copied into the
//                       value CTA's with one bulk copy per tile
//   value CTA (rank 1)  O += P . V          tcgen05, M=128, N=2x256, K=32 keys,
//                                           O (128 x 512 FP32) fills the whole TMEM
//
// O needs all 512 TMEM columns of an SM and Q.K^T needs 288 columns of Q plus
// the S accumulators, so neither fits beside the other on one SM; P is the
// smallest thing that has to cross (8 KB per tile). The value CTA returns a
// P slot to the score CTA with the commit of the PV that read it
// (tcgen05.commit multicast to both CTAs: the same barrier offset means
// "P slot free" in the score CTA and "value stage free" in the value CTA).
//
// Online softmax semantics follow dsa/workspace.py:242-318: invalid index ->
// -inf, FP32 max and sum, BF16 P, FP32 O. O is rescaled only when a row max
// grows by more than 2^8 in exp2 units (lazy rescale); the value CTA applies
// the factor before the PV of that tile, on request of its PV issuer, which
// reads the per-warp flags. The reported max is the true max; the sum and
// split partials are rescaled to it at the end.
//
// Roles (20 warps per CTA):
//   score CTA: 0-4 gather (warp w owns stage w: 16-byte cp.async of the full
//              rows into 128-byte-swizzled K-major tiles), 5 P sender (one
//              bulk shared-to-shared copy per tile from a local staging slot
//              to the value CTA's P slot, so the softmax warps only write
//              their own shared memory: cross-SM stores issued by the
//              softmax warps themselves held them ~0.3 us per tile), 6-13
//              softmax: two warps per TMEM lane quadrant (head rows
//              32q..32q+31), the warp of quadrant q among 6-9 / 10-13
//              takes the even / odd tiles. The running
//              max is the only dependence between consecutive tiles: a warp
//              posts the max it used for its tile (one bounded mbarrier phase
//              per tile) right after its row-max reduction, and the other warp
//              waits for it before deciding its own, so the exponentials and
//              the P transfer of consecutive tiles overlap. Key validity comes
//              from the gather warps (a tagged ring of per-tile bit masks), so
//              a stage is free as soon as its QK MMAs complete. 14-19 QK
//              issuers (tile g -> issuer g % 6: issuing a tcgen05.mma occupies
//              the issuing warp's scheduler, so the 36 MMAs of each tile are
//              spread over the schedulers) into S buffer g % 6 (a buffer
//              returns to the issuers only after its softmax read). The
//              issuers also load Q into TMEM: once every QK MMA of an item is
//              done, all nine chunks of the next item's Q (prefetched into L2
//              eight tiles ahead), while the softmax warps finish the item.
//   value CTA: 0-4 gather of the 512 latent dims (warp w owns stage w), 6 PV
//              issuer, 8-19 rescale and epilogue (three warps per lane
//              quadrant, O * (1/l) -> output with 32-byte stores).
// Every wait is bounded and reports through the status word; no TMA and no
// multicast loads are used.
#include "umma_ptx.cuh"

namespace dsa {
namespace {

using namespace umma;

constexpr int kPrBN = 32;       // keys per tile
constexpr int kPrHeads = 128;
// Tile g of the cluster's sequence uses S buffer and P slot g % 6, QK issuer
// g % 6, stage and gather warp g % 5, local staging slot g % 4 and softmax
// warp g % 2 of each lane quadrant: every mbarrier is waited on by one role
// whose consecutive waits on it are one phase apart, the condition for
// parity waits to be exact. The one exception, a QK issuer waiting for the
// stage g % 5 of its tile g % 6, first waits until the gather warp has
// started that tile (a per-stage tile word), which fixes the phase.
constexpr int kKStages = 5;     // score CTA: gathered full rows (gather warp w owns stage w)
constexpr int kLSlots = 4;      // score CTA: local P staging slots (even: slot g % 4 is always softmax warp g % 2's)
constexpr int kSendWarp = kKStages;  // score CTA: warp 5 sends the staged P
constexpr int kSBufs = 6;       // score CTA: S accumulators in TMEM
constexpr int kQkIssuers = 6;   // score CTA: QK issuer i takes tiles g = i mod 6
constexpr int kVStages = 5;     // value CTA: gathered value rows
constexpr int kPSlots = 6;      // value CTA: P slots
constexpr int kPrThreads = 640;
constexpr int kPvWarp = 6;      // value CTA: gather 0-4, PV issuer 6, rescale+epilogue 8-19
constexpr int kSoftWarp0 = 6;   // score CTA: gather 0-4, sender 5, softmax 6-13, QK issuers 14-19
constexpr int kSoftWarps = 8;
constexpr int kEpiWarp0 = 8;
constexpr int kEpiWarps = 12;   // value CTA: warps 8..19, three per TMEM lane quadrant
// first 32-column chunk of O owned by epilogue part 0, 1, 2 (chunks 0-5, 6-10, 11-15)
__host__ __device__ constexpr int epi_chunk0(int part) { return part == 0 ? 0 : 5 * part + 1; }
constexpr int kQkWarp0 = 14;    // score CTA: QK issuer i = warp 14 + i
constexpr int kQkSteps = kDimQK / 16;  // 36

// Shared memory (byte offsets from a 1024-aligned base; same layout in both
// CTAs for the barrier block so that multicast commits and mapa addresses
// line up).
constexpr uint32_t kBlk = (uint32_t)kPrBN * 128u;       // 32 rows x 64 dims, SW128
constexpr uint32_t kKStage = 9u * kBlk;                 // 8 latent + 1 rope block
constexpr uint32_t kVStage = 8u * kBlk;                 // 8 latent blocks
constexpr uint32_t kPBytes = 128u * (uint32_t)kPrBN * 2u;  // P: 128 rows x 32 keys (SW64)
constexpr uint32_t kAlphaOff = kPBytes;                 // 128 FP32 rescale factors
constexpr uint32_t kFlagOff = kPBytes + 512u;           // 4 per-warp rescale flags
constexpr uint32_t kMsgBytes = kPBytes + 512u + 16u;    // bytes the score CTA sends per tile
constexpr uint32_t kSlotBytes = kPBytes + 1024u;        // P slot stride (1024-aligned)
constexpr uint32_t kFinBytes = 128u * 8u;               // per item: (l, f) per row

enum Bar {
  // score CTA
  kFull0 = 0,
  kEmpty0 = kFull0 + kKStages,      // QK commit (the softmax takes validity from the indices)
  kQFull = kEmpty0 + kKStages,
  kQkDone,                          // every QK MMA of the item is done (one commit per issuer)
  kSFull0,
  kSFree0 = kSFull0 + kSBufs,
  kFinFree0 = kSFree0 + kSBufs,     // 2: value CTA has read the (l, f) buffer
  kXchg0 = kFinFree0 + 2,           // 4: per lane quadrant, both softmax warps posted their item totals
  kMReady0 = kXchg0 + 4,            // 4: per lane quadrant, the running max of the latest tile is posted
  kPSlotFree0 = kMReady0 + 4,       // P slot's PV done (commit multicast from the value CTA)
  kLFull0 = kPSlotFree0 + kPSlots,  // local staging slot written (the tile's 4 softmax warps)
  kLFree0 = kLFull0 + kLSlots,      // local staging slot read by its bulk copy (sender)
  // value CTA
  kVFull0 = kLFree0 + kLSlots,
  kVFree0 = kVFull0 + kVStages,     // value stage's PV done
  kPFull0 = kVFree0 + kVStages,     // P message landed (complete_tx)
  kReq = kPFull0 + kPSlots,         // a rescale or epilogue request is posted
  kReqDone,                         // rescale done (kEpiWarps warps)
  kOFree,                           // epilogue has read O (kEpiWarps warps)
  kFin0,                            // 2: (l, f) of an item landed (complete_tx)
  kBarCount = kFin0 + 2
};
constexpr uint32_t kOffBar = 0;
constexpr uint32_t kOffTmemSlot = kOffBar + kBarCount * 8u;
constexpr uint32_t kOffAbort = kOffTmemSlot + 8u;
constexpr uint32_t kOffReq = kOffAbort + 8u;
constexpr uint32_t kOffStageTile = kOffReq + 8u;        // score CTA: tile each stage is being filled with
// score CTA: validity bits of tile g's 32 keys at entry g % 16, tagged with
// g, written by the tile's gather warp. A gather warp can be at most 13
// tiles ahead of the softmax warp reading the entry (stage reuse waits for
// the QK of tile g - 5, which waits for the softmax of tile g - 11 to read
// its S, which that warp does after finishing tile g - 13 or after the
// running max of tile g - 14, posted after its entry was read).
constexpr int kMaskRing = 16;
constexpr uint32_t kOffMaskRing = kOffStageTile + 4u * kKStages + 4u;  // [16] {bits, tag}, 8-byte aligned
constexpr uint32_t kOffData = 1024u;
constexpr uint32_t kOffK = kOffData;                     // score CTA stages
constexpr uint32_t kOffV = kOffData;                     // value CTA stages
constexpr uint32_t kOffSlot = kOffV + kVStages * kVStage;  // value CTA P slots
constexpr uint32_t kOffFin = kOffSlot + kPSlots * kSlotBytes;
constexpr uint32_t kOffLocal = kOffK + kKStages * kKStage;  // score CTA: P staging slots
constexpr uint32_t kOffX = kOffLocal + kLSlots * kSlotBytes;  // score CTA: [2][4 quads][2 warps][3][32] floats
constexpr uint32_t kOffM = kOffX + 2u * 4u * 2u * 3u * 32u * 4u;  // score CTA: [2][4 quads][32] running maxima
// score CTA, union launch: per tile one validity mask per query of the block
// (8 words) and the tile tag (word 8), 48-byte entries, same ring indexing
constexpr uint32_t kOffURing = kOffM + 2u * 4u * 32u * 4u;
constexpr uint32_t kURingStride = 48u;
constexpr uint32_t kSmemScore = kOffURing + kMaskRing * kURingStride;
constexpr uint32_t kSmemValue = kOffFin + 2u * kFinBytes;
constexpr uint32_t kSmemUsed = kSmemScore > kSmemValue ? kSmemScore : kSmemValue;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024u;  // slack for the 1024-byte alignment

constexpr uint32_t kReqRescale = 1u << 31;

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemQ = 0;      // score CTA: Q, 288 columns (dims 0..575 as BF16 pairs)
constexpr uint32_t kTmemS = 288;    // score CTA: S buffers, 32 columns each
constexpr uint32_t kTmemO = 0;      // value CTA: O, 512 columns

static_assert(kOffMaskRing % 8 == 0 && kOffMaskRing + 8u * kMaskRing <= kOffData, "barrier block");
static_assert(kOffURing % 16 == 0, "union ring entries are 16-byte aligned");
static_assert(kLSlots % 2 == 0, "a staging slot must always belong to the same softmax warp");
static_assert(kOffLocal % 1024 == 0 && kMsgBytes % 16 == 0, "bulk copy alignment");
static_assert(kOffSlot % 1024 == 0 && kSlotBytes % 1024 == 0, "P slots are 1024-aligned");
static_assert(kSmemBytes <= 232448, "shared memory budget");
static_assert(kTmemS + kSBufs * kPrBN <= kTmemCols, "score TMEM budget");

struct PItem {
  int token, sp, batch, kbeg, kend, ntiles;
};

__device__ __forceinline__ PItem make_pitem(const FwdParams& p, int item) {
  PItem it;
  it.token = item / p.split;
  it.sp = item % p.split;
  it.batch = it.token / p.queries;
  if (p.uent != nullptr) {  // union launch: the block's union entries (split 1)
    it.kbeg = 0;
    it.kend = __ldg(p.ulen + it.token);
  } else {
    split_bounds(p.topk, kPrBN, p.split, it.sp, &it.kbeg, &it.kend);
  }
  it.ntiles = (it.kend - it.kbeg + kPrBN - 1) / kPrBN;
  return it;
}

// Position of one tile in the cluster's sequence of tiles (items cid,
// cid + nclusters, ...; tiles 0..ntiles-1 of each).
struct PCursor {
  int item, t;
  PItem w;
};

__device__ __forceinline__ void pcursor_advance(const FwdParams& p, int n_items, int stride, PCursor& c, int k) {
  c.t += k;
  while (c.item < n_items && c.t >= c.w.ntiles) {
    c.t -= c.w.ntiles;
    c.item += stride;
    if (c.item < n_items) c.w = make_pitem(p, c.item);
  }
}

__device__ __forceinline__ PCursor pcursor_start(const FwdParams& p, int n_items, int first, int stride, int k) {
  PCursor c;
  c.item = first;
  c.t = 0;
  if (c.item < n_items) c.w = make_pitem(p, c.item);
  pcursor_advance(p, n_items, stride, c, k);
  return c;
}

// Index of key `lane` of the cursor's tile (-1 past the split's end or past
// the last item); for the union launch the packed entry key | bits << 24.
__device__ __forceinline__ int pcursor_index(const FwdParams& p, const PCursor& c, int n_items, int lane) {
  if (c.item >= n_items) return -1;
  const int j = c.w.kbeg + c.t * kPrBN + lane;
  if (j >= c.w.kend) return -1;
  return p.uent != nullptr ? __ldg(p.uent + (size_t)c.w.token * p.ucap + j)
                           : __ldg(p.ids + (size_t)c.w.token * p.topk + j);
}
// Row address of an index or union entry: clamped to [0, L - 1]; masked by
// the softmax. A union entry is key | bits << 24 (negative when the block's
// eighth query selected it); -1 marks a slot past the block's entries (no
// key reaches 2^24 - 1).
__device__ __forceinline__ int pcursor_row(const FwdParams& p, int idx, int L) {
  if (p.uent != nullptr) return idx != -1 ? (idx & 0xFFFFFF) : 0;
  return min(max(idx, 0), L - 1);
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

// Bounded wait whose result is the same in every lane of the warp.
__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity, volatile int* abort,
                                          bool cluster_scope = false) {
  const bool ok = mbar_wait(bar, parity, abort, cluster_scope);
  return __all_sync(0xffffffffu, ok) != 0;
}

// 8-byte shared-memory store / load (both words together)
__device__ __forceinline__ void st_shared_v2(uint32_t addr, uint32_t a, uint32_t b) {
  asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ void ld_shared_v2(uint32_t addr, uint32_t& a, uint32_t& b) {
  asm volatile("ld.volatile.shared.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "r"(addr) : "memory");
}
__device__ __forceinline__ void st_async_b32x2(uint32_t remote_addr, uint32_t remote_bar, uint32_t a, uint32_t b) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.b32 [%0], {%1, %2}, [%3];" ::"r"(
                   remote_addr),
               "r"(a), "r"(b), "r"(remote_bar)
               : "memory");
}
// Arrive once on the barrier at `bar`'s offset in every CTA of `cta_mask`
// when all prior tcgen05.mma of this thread complete.
__device__ __forceinline__ void mma_commit_mc(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          bar),
      "h"(cta_mask)
      : "memory");
}

// 16-byte cp.async of 32 indexed rows into a swizzled K-major stage:
// `nblk` 64-dim blocks of the latent row (+ the rope block when `rope`).
__device__ __forceinline__ void gather_rows(uint32_t stage, const __nv_bfloat16* kv_b, const __nv_bfloat16* kr_b,
                                            int row, int lane, bool rope, int32_t* status) {
  const int j8 = lane & 7;
  const int kq = lane >> 3;
#pragma unroll 2
  for (int i = 0; i < kPrBN / 4; ++i) {
    const int k = kq + 4 * i;
    const int rk = __shfl_sync(0xffffffffu, row, k);
    const uint32_t dst = checked_smem(
        stage + (uint32_t)(k >> 3) * 1024u + (uint32_t)(k & 7) * 128u + (uint32_t)((j8 ^ (k & 7)) * 16),
        (rope ? 8u : 7u) * kBlk + 16u, stage, rope ? kKStage : kVStage, status);
    const __nv_bfloat16* src = kv_b + (size_t)rk * kDimLatent + j8 * 8;
#pragma unroll
    for (int kb = 0; kb < 8; ++kb) cp_async_16(dst + kb * kBlk, src + kb * 64);
    if (rope) cp_async_16(dst + 8 * kBlk, kr_b + (size_t)rk * kDimRope + j8 * 8);
  }
}

// Chunk `ch` (dims 64ch..64ch+63; ch == 8: the 64 rope dims) of one Q head
// row -> 32 TMEM columns of this thread's lane (BF16 pairs).
__device__ __forceinline__ void load_q_chunk(const FwdParams& p, size_t qrow, int ch, uint32_t taddr) {
  const uint4* s4 = ch < 8 ? reinterpret_cast<const uint4*>(p.q + qrow * kDimLatent) + ch * 8
                           : reinterpret_cast<const uint4*>(p.q_rope + qrow * kDimRope);
  uint32_t r[32];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint4 v = __ldg(s4 + k);
    r[4 * k] = v.x;
    r[4 * k + 1] = v.y;
    r[4 * k + 2] = v.z;
    r[4 * k + 3] = v.w;
  }
  tmem_st32(taddr, r);
}

// Chunks [c0, c1) of one Q head row, two chunks' loads in flight at a time
// (`tq` = this lane's TMEM address of chunk 0).
__device__ __forceinline__ void load_q_chunks(const FwdParams& p, size_t qrow, int c0, int c1, uint32_t tq) {
#pragma unroll 1
  for (int ch = c0; ch < c1; ch += 2) {
    if (ch + 1 == c1) {
      load_q_chunk(p, qrow, ch, tq + (uint32_t)ch * 32u);
      break;
    }
    uint32_t r[64];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int cc = ch + h;
      const uint4* s4 = cc < 8 ? reinterpret_cast<const uint4*>(p.q + qrow * kDimLatent) + cc * 8
                               : reinterpret_cast<const uint4*>(p.q_rope + qrow * kDimRope);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint4 v = __ldg(s4 + k);
        r[32 * h + 4 * k] = v.x;
        r[32 * h + 4 * k + 1] = v.y;
        r[32 * h + 4 * k + 2] = v.z;
        r[32 * h + 4 * k + 3] = v.w;
      }
    }
    tmem_st32(tq + (uint32_t)ch * 32u, r);
    tmem_st32(tq + (uint32_t)(ch + 1) * 32u, r + 32);
  }
}

// Q chunks that QK issuer i (warp kQkWarp0 + i, TMEM lane quadrant
// (kQkWarp0 + i) % 4) loads for each item: all nine chunks of its quadrant's
// head rows, split between the two issuers of quadrants 2 and 3.
__device__ __forceinline__ void issuer_q_chunks(int i, int* c0, int* c1) {
  const int quad = (kQkWarp0 + i) & 3;
  if (quad < 2) {  // the only issuer of its quadrant
    *c0 = 0;
    *c1 = 9;
  } else if (i < 4) {
    *c0 = 0;
    *c1 = 5;
  } else {
    *c0 = 5;
    *c1 = 9;
  }
}

// kUnion: the union launch (keys from per-block union entries, one
// validity mask per query of the block); otherwise one index row per item.
template <bool kUnion>
__global__ void __launch_bounds__(kPrThreads, 1) fwd_pair_kernel(const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const sbase = smem_raw + (base - raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cid = (int)(blockIdx.x >> 1);
  const int ncl = (int)(gridDim.x >> 1);
  const int n_items = p.tokens * p.split;
  const int L = p.length;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sbase + kOffAbort);
  auto bar = [&](int i) -> uint32_t { return base + kOffBar + 8u * (uint32_t)i; };

  if (threadIdx.x == 0) {
    if (rank == 0) {
      for (int s = 0; s < kKStages; ++s) {
        mbar_init(bar(kFull0 + s), 1);
        mbar_init(bar(kEmpty0 + s), 1);
      }
      mbar_init(bar(kQFull), kQkIssuers);  // Q chunks: the 6 QK issuers
      mbar_init(bar(kQkDone), kQkIssuers);
      for (int i = 0; i < kSBufs; ++i) {
        mbar_init(bar(kSFull0 + i), 1);
        mbar_init(bar(kSFree0 + i), 4);
      }
      mbar_init(bar(kFinFree0), kEpiWarps);
      mbar_init(bar(kFinFree0 + 1), kEpiWarps);
      for (int q = 0; q < 4; ++q) {
        mbar_init(bar(kXchg0 + q), 2);
        mbar_init(bar(kMReady0 + q), 1);
      }
      for (int s = 0; s < kPSlots; ++s) mbar_init(bar(kPSlotFree0 + s), 1);
      for (int s = 0; s < kLSlots; ++s) {
        mbar_init(bar(kLFull0 + s), 4);
        mbar_init(bar(kLFree0 + s), 1);
      }
      for (int s = 0; s < kKStages; ++s)
        reinterpret_cast<volatile uint32_t*>(sbase + kOffStageTile)[s] = 0xffffffffu;
      for (int k = 0; k < kMaskRing; ++k)
        reinterpret_cast<volatile uint32_t*>(sbase + kOffMaskRing)[2 * k + 1] = 0xffffffffu;
      if (kUnion)
        for (int k = 0; k < kMaskRing; ++k)
          reinterpret_cast<volatile uint32_t*>(sbase + kOffURing + k * kURingStride)[8] = 0xffffffffu;
    } else {
      for (int s = 0; s < kVStages; ++s) {
        mbar_init(bar(kVFull0 + s), 1);
        mbar_init(bar(kVFree0 + s), 1);
      }
      for (int s = 0; s < kPSlots; ++s) mbar_init(bar(kPFull0 + s), 1);
      mbar_init(bar(kReq), 1);
      mbar_init(bar(kReqDone), kEpiWarps);
      mbar_init(bar(kOFree), kEpiWarps);
      mbar_init(bar(kFin0), 1);
      mbar_init(bar(kFin0 + 1), 1);
    }
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
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sbase + kOffTmemSlot);
  // The value CTA arms its P slots and (l, f) buffers before the score CTA
  // can send anything (the cluster barrier below orders the two).
  if (rank == 1 && threadIdx.x == 0) {
    for (int s = 0; s < kPSlots; ++s) mbar_arrive_expect_tx(bar(kPFull0 + s), kMsgBytes);
    mbar_arrive_expect_tx(bar(kFin0), kFinBytes);
    mbar_arrive_expect_tx(bar(kFin0 + 1), kFinBytes);
  }
  cluster_sync();

  bool ok = true;
  if (rank == 0) {
    // =============================== score CTA ===============================
    if (warp < kKStages) {
      // ---- gather: warp w fills stage w for tiles g = w, w+5, ... ----
      const uint32_t s = (uint32_t)warp;
      const uint32_t stage = base + kOffK + s * kKStage;
      PCursor cur = pcursor_start(p, n_items, cid, ncl, (int)s);
      PCursor nx = cur;
      pcursor_advance(p, n_items, ncl, nx, kKStages);
      PCursor nx2 = nx;
      pcursor_advance(p, n_items, ncl, nx2, kKStages);
      int idx_cur = pcursor_index(p, cur, n_items, lane);
      int idx_nx = pcursor_index(p, nx, n_items, lane);
      uint32_t n = 0;
      while (cur.item < n_items) {
        if (n > 0 && !(ok = wait_warp(bar(kEmpty0 + s), (n - 1) & 1u, abort_flag))) break;
        // the stage's previous tile (g - 5) is consumed, so its Full phase completed
        const uint32_t gt = s + kKStages * n;  // the tile this warp fills
        if constexpr (kUnion) {
          // one mask per query of the block: entry lane selected by query j
          uint32_t um[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            um[j] = __ballot_sync(0xffffffffu, idx_cur != -1 && (((uint32_t)idx_cur >> (24 + j)) & 1u));
          if (lane == 0) {
            reinterpret_cast<volatile uint32_t*>(sbase + kOffStageTile)[s] = gt;
            volatile uint32_t* ue = reinterpret_cast<volatile uint32_t*>(sbase + kOffURing + (gt % kMaskRing) * kURingStride);
#pragma unroll
            for (int j = 0; j < 8; ++j) ue[j] = um[j];
            __threadfence_block();  // masks before the tag
            ue[8] = gt;
          }
        } else {
          const uint32_t vbits = __ballot_sync(0xffffffffu, (idx_cur >= 0) & (idx_cur < L));
          if (lane == 0) {
            reinterpret_cast<volatile uint32_t*>(sbase + kOffStageTile)[s] = gt;
            // validity bits of the tile for the softmax (one 8-byte store: bits and tag together)
            st_shared_v2(base + kOffMaskRing + 8u * (gt % kMaskRing), vbits, gt);
          }
        }
        const int row = checked_index(pcursor_row(p, idx_cur, L), L, p.status);  // clamped; masked by the softmax
        const int gb = checked_index(cur.w.batch, p.batch, p.status);
        gather_rows(stage, p.kv + (size_t)gb * L * kDimLatent, p.k_rope + (size_t)gb * L * kDimRope, row, lane, true,
                    p.status);
        cp_async_commit();
        const int idx_nx2 = pcursor_index(p, nx2, n_items, lane);  // consumed one round later
        cp_async_wait<0>();
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kFull0 + s));
        ++n;
        cur = nx;
        nx = nx2;
        pcursor_advance(p, n_items, ncl, nx2, kKStages);
        idx_cur = idx_nx;
        idx_nx = idx_nx2;
      }
    } else if (warp >= kQkWarp0 && warp < kQkWarp0 + kQkIssuers) {
      // ---- QK issuer i: S buffer g % 6 <- Q (TMEM) . K^T (stage g % 5) for tiles g = i mod 6 ----
      const uint32_t i = (uint32_t)(warp - kQkWarp0);
      const uint32_t idesc_qk = idesc_bf16(128, kPrBN, false, false);
      uint32_t g = 0, it = 0;
      const int quad = warp & 3;  // TMEM lane quadrant this warp can access
      const uint32_t t_lane = (uint32_t)(quad * 32) << 16;
      for (int item = cid; item < n_items && ok; item += ncl, ++it) {
        const PItem w = make_pitem(p, item);
        // This issuer's Q chunks of its lane quadrant's head rows: for the
        // first item here, for later items at the end of the previous one.
        int qc0, qc1;
        issuer_q_chunks((int)i, &qc0, &qc1);
        if (it == 0) {
          load_q_chunks(p, (size_t)w.token * kPrHeads + quad * 32 + lane, qc0, qc1, tmem + t_lane + kTmemQ);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kQFull));
        }
        // Every issuer waits for every item's Q (all chunks of all quadrants),
        // so none can fall a barrier phase behind.
        if (!(ok = wait_warp(bar(kQFull), it & 1u, abort_flag))) break;
        for (int t = 0; t < w.ntiles; ++t, ++g) {
          if (g % kQkIssuers != i) continue;
          const uint32_t s = g % kKStages, b = g % kSBufs;
          const uint32_t d = tmem + kTmemS + b * kPrBN;
          // this issuer has not observed the Full phase of the stage's previous
          // tile (g - 5, another issuer's); once the gather of tile g has
          // started, that phase has completed and the parity wait refers to
          // tile g's phase exactly
          if (!(ok = wait_word_warp(reinterpret_cast<volatile uint32_t*>(sbase + kOffStageTile) + s, g, abort_flag)))
            break;
          if (!(ok = wait_warp(bar(kFull0 + s), (g / kKStages) & 1u, abort_flag))) break;
          // S buffer b was last used by tile g - 6 (this issuer's): its softmax has read it
          if (g >= kSBufs && !(ok = wait_warp(bar(kSFree0 + b), ((g / kSBufs) - 1) & 1u, abort_flag))) break;
          tc_fence_after();
          const uint32_t stage = base + kOffK + s * kKStage;
          if (elect_one()) {
#pragma unroll
            for (int ks = 0; ks < kQkSteps; ++ks) {
              const uint64_t bd =
                  smem_desc(stage + (ks >> 2) * kBlk + (uint32_t)(ks & 3) * 32u, 16, 1024, kLayoutSw128);
              mma_bf16_ts(d, tmem + kTmemQ + (uint32_t)ks * 8u, bd, idesc_qk, ks > 0 ? 1u : 0u);
            }
            mma_commit(bar(kSFull0 + b));
            mma_commit(bar(kEmpty0 + s));
          }
          __syncwarp();
        }
        if (!ok) break;
        // Once every issuer's QK MMAs of this item are done, the Q columns are
        // free: load this issuer's chunks of the next item's Q while the
        // softmax warps finish this item.
        if (elect_one()) mma_commit(bar(kQkDone));
        __syncwarp();
        if (item + ncl < n_items) {
          if (!(ok = wait_warp(bar(kQkDone), it & 1u, abort_flag))) break;
          tc_fence_after();
          const PItem wn = make_pitem(p, item + ncl);
          load_q_chunks(p, (size_t)wn.token * kPrHeads + quad * 32 + lane, qc0, qc1, tmem + t_lane + kTmemQ);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kQFull));
        }
      }
    } else if (warp == kSendWarp) {
      // ---- P sender: staging slot g % 4 -> the value CTA's P slot g % 6, one bulk copy per tile ----
      const uint32_t r_slot0 = mapa_shared(base + kOffSlot, 1);
      const uint32_t r_pfull0 = mapa_shared(bar(kPFull0), 1);
      uint32_t g = 0;
      for (int item = cid; item < n_items && ok; item += ncl) {
        const PItem w = make_pitem(p, item);
        for (int t = 0; t < w.ntiles; ++t, ++g) {
          const uint32_t ls = g % kLSlots, ps = g % kPSlots;
          if (!(ok = wait_warp(bar(kLFull0 + ls), (g / kLSlots) & 1u, abort_flag))) break;
          // the value CTA's P slot ps is free once the PV of tile g - 6 is done
          if (g >= kPSlots && !(ok = wait_warp(bar(kPSlotFree0 + ps), ((g / kPSlots) - 1) & 1u, abort_flag)))
            break;
          if (lane == 0) {
            bulk_copy_to_peer(r_slot0 + ps * kSlotBytes, base + kOffLocal + ls * kSlotBytes, kMsgBytes,
                              r_pfull0 + 8u * ps);
            bulk_commit_group();
            bulk_wait_group_read<1>();  // the copy of tile g - 1 has read its staging slot
          }
          __syncwarp();
          if (g >= 1 && lane == 0) mbar_arrive(bar(kLFree0 + (g - 1) % kLSlots));
        }
      }
      if (lane == 0) bulk_wait_group_read<0>();
      __syncwarp();
      // the value CTA's last P-slot credits (its PVs have read every copy)
      for (uint32_t k = 0; ok && k < (uint32_t)kPSlots && k < g; ++k) {
        const uint32_t gl = g - 1 - k;
        ok = wait_warp(bar(kPSlotFree0 + gl % kPSlots), (gl / kPSlots) & 1u, abort_flag);
      }
    } else if (warp >= kSoftWarp0 && warp < kSoftWarp0 + kSoftWarps) {
      // ---- softmax: head row per thread; warp e = 0 / 1 of the quadrant takes tiles g % 2 == e ----
      const int quad = warp & 3;
      const uint32_t e = (uint32_t)(warp - kSoftWarp0) >> 2;
      const int row = quad * 32 + lane;
      const uint32_t t_lane = (uint32_t)(quad * 32) << 16;
      const float c = p.scale_log2;  // log2(e) / scale_div
      float* const xch = reinterpret_cast<float*>(sbase + kOffX);  // [parity][quad][warp][3][lane]
      float* const mpub = reinterpret_cast<float*>(sbase + kOffM);  // [tile parity][quad][lane]
      const uint32_t r_fin0 = mapa_shared(base + kOffFin, 1);
      const uint32_t r_finbar0 = mapa_shared(bar(kFin0), 1);
      // P row offset in a slot (SW64 K-major: 8-row groups of 512 B, 16-byte chunks swizzled)
      const uint32_t prow = (uint32_t)(row >> 3) * 512u + (uint32_t)(row & 7) * 64u;
      uint32_t xn = 0;  // item-end exchanges done with the other warp of this quadrant
      // This warp's tiles: e, e + 2, ... of the cluster's tile sequence.
      uint32_t g = 0, it = 0;
      for (int item = cid; item < n_items && ok; item += ncl, ++it) {
        const PItem w = make_pitem(p, item);
        // (Q of the item is loaded into TMEM by the QK issuers, during the
        // previous item's last tiles.)
        // this warp's running state for the item
        float m_w = kNegFltMax;     // max used for this warp's latest tile
        float m_true = kNegFltMax;  // true max over this warp's tiles
        float l = 0.f;              // sum over this warp's tiles, relative to m_w
        const uint32_t g_item = g;
        for (int t = (int)((e - g_item) & 1u); t < w.ntiles; t += 2) {
          g = g_item + (uint32_t)t;
          if (t == max(w.ntiles - 8, 0) && quad == 0 && item + ncl < n_items && lane < 9) {
            // the next item's Q rows -> L2 (128 KB latent + 16 KB rope), so
            // that its load at the item boundary hits L2
            const size_t qn = (size_t)((item + ncl) / p.split) * kPrHeads;
            if (lane < 8)
              prefetch_l2_bulk(p.q + qn * kDimLatent + (size_t)lane * 8192, 16384u);
            else
              prefetch_l2_bulk(p.q_rope + qn * kDimRope, 16384u);
          }
          const uint32_t i = g % kSBufs;
          // S complete (a non-blocking test first: it almost always is)
          if (!__all_sync(0xffffffffu, mbar_test(bar(kSFull0 + i), (g / kSBufs) & 1u)) &&
              !(ok = wait_warp(bar(kSFull0 + i), (g / kSBufs) & 1u, abort_flag)))
            break;
          // validity bits of the tile's keys, published by its gather warp
          // (written before the gather, so present once S is)
          uint32_t mbits, mtag;
          if constexpr (kUnion) {
            // the mask of this row's query (row >> u_row_shift) in the block
            const volatile uint32_t* ue =
                reinterpret_cast<const volatile uint32_t*>(sbase + kOffURing + (g % kMaskRing) * kURingStride);
            if (ue[8] != g && !(ok = wait_word_warp(const_cast<volatile uint32_t*>(ue + 8), g, abort_flag))) break;
            __threadfence_block();  // the tag was written after the masks
            mbits = ue[row >> p.u_row_shift];
          } else {
            const uint32_t ent = base + kOffMaskRing + 8u * (g % kMaskRing);
            ld_shared_v2(ent, mbits, mtag);
            if (mtag != g) {
              if (!(ok = wait_word_warp(reinterpret_cast<volatile uint32_t*>(sbase + kOffMaskRing + 8u * (g % kMaskRing) + 4u),
                                        g, abort_flag)))
                break;
              ld_shared_v2(ent, mbits, mtag);
            }
          }
          tc_fence_after();
          float x[32];
          {
            uint32_t sv[32];
            tmem_ld32(checked_tmem(tmem + t_lane + kTmemS + i * kPrBN, tmem, 32u, kTmemCols, p.status), sv);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; ++k) x[k] = u2f(sv[k]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kSFree0 + i));
          if (mbits != 0xFFFFFFFFu) {
#pragma unroll
            for (int k = 0; k < 32; ++k) x[k] = ((mbits >> k) & 1u) ? x[k] : -INFINITY;
          }
          float mx;
          {  // tree reduction: 5 dependent steps instead of 32
            float r[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) r[k] = fmaxf(x[k], x[k + 16]);
#pragma unroll
            for (int w2 = 8; w2 >= 1; w2 >>= 1)
#pragma unroll
              for (int k = 0; k < w2; ++k) r[k] = fmaxf(r[k], r[k + w2]);
            mx = r[0];
          }
          m_true = fmaxf(m_true, mx);
          // running max of the previous tile (posted by the other warp), then ours
          float m_prev = kNegFltMax;
          if (g > 0) {
            if (!(ok = wait_warp(bar(kMReady0 + quad), (g - 1) & 1u, abort_flag))) break;
            if (t > 0) m_prev = mpub[(((g - 1) & 1u) * 4 + quad) * 32 + lane];
          }
          const float m_t = ((mx - m_prev) * c > 8.f) ? mx : m_prev;  // lazy rescale threshold 2^8
          mpub[((g & 1u) * 4 + quad) * 32 + lane] = m_t;
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kMReady0 + quad));
          const bool resc = t > 0 && m_t != m_prev;  // the first PV of an item overwrites O
          const float alpha = resc ? ex2((m_prev - m_t) * c) : 1.f;
          const float mc = m_t * c;
          uint32_t packed[16];
          float psum[16];
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const float p0 = ex2(fmaf(x[k], c, -mc));
            const float p1 = ex2(fmaf(x[k + 1], c, -mc));
            psum[k / 2] = p0 + p1;
            packed[k / 2] = pack_bf16x2(p0, p1);
          }
#pragma unroll
          for (int w2 = 8; w2 >= 1; w2 >>= 1)
#pragma unroll
            for (int k = 0; k < w2; ++k) psum[k] += psum[k + w2];
          if (m_t != m_w) {  // bring this warp's sum to the new max
            l *= ex2((m_w - m_t) * c);
            m_w = m_t;
          }
          l += psum[0];
          const uint32_t flag = __any_sync(0xffffffffu, resc) ? 1u : 0u;
          // staging slot ls (this warp's) is free once the bulk copy of
          // tile g - 4 has read it
          const uint32_t ls = g % kLSlots;
          if (g >= kLSlots && !__all_sync(0xffffffffu, mbar_test(bar(kLFree0 + ls), ((g / kLSlots) - 1) & 1u)) &&
              !(ok = wait_warp(bar(kLFree0 + ls), ((g / kLSlots) - 1) & 1u, abort_flag)))
            break;
          uint8_t* const lslot = sbase + kOffLocal + ls * kSlotBytes;
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(lslot + prow + (uint32_t)((q ^ ((row & 7) >> 1)) * 16)) =
                make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
          *reinterpret_cast<uint32_t*>(lslot + kAlphaOff + (uint32_t)row * 4u) = f2u(alpha);
          if (lane == 0) *reinterpret_cast<uint32_t*>(lslot + kFlagOff + (uint32_t)quad * 4u) = flag;
          fence_proxy_async_smem();  // generic-proxy writes -> visible to the bulk copy
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kLFull0 + ls));
        }
        g = g_item + (uint32_t)w.ntiles;
        if (!ok) break;
        // ---- item end: combine the two warps' (max used, sum, true max) ----
        {
          const uint32_t par = xn & 1u;
          float* const mine = xch + ((par * 4 + quad) * 2 + e) * 96;
          const float* const other = xch + ((par * 4 + quad) * 2 + (e ^ 1u)) * 96;
          mine[lane] = m_w;
          mine[32 + lane] = l;
          mine[64 + lane] = m_true;
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kXchg0 + quad));
          if (!(ok = wait_warp(bar(kXchg0 + quad), par, abort_flag))) break;
          const float m_o = other[lane], l_o = other[32 + lane], mt_o = other[64 + lane];
          ++xn;
          const float m_fin = fmaxf(m_w, m_o);
          l = (m_w == m_fin ? l : l * ex2((m_w - m_fin) * c)) + (m_o == m_fin ? l_o : l_o * ex2((m_o - m_fin) * c));
          m_true = fmaxf(m_true, mt_o);
          m_w = m_fin;
        }
        if (e != 0) continue;
        const float f = (m_true == kNegFltMax) ? 1.f : ex2((m_w - m_true) * c);
        const size_t orow = (size_t)w.token * kPrHeads + row;
        if (p.split == 1) {
          p.out_max[orow] = final_max(m_true, l, p.scale_div);
          p.out_sum[orow] = l * f;
        } else {
          const size_t pr = ((size_t)w.token * p.split + w.sp) * kPrHeads + row;
          p.part_max[pr] = (m_true == kNegFltMax) ? kNegFltMax : __fdiv_rn(m_true, p.scale_div);
          p.part_sum[pr] = l * f;
        }
        const uint32_t fb = it & 1u;
        if (it >= 2 && !(ok = wait_warp(bar(kFinFree0 + fb), ((it >> 1) - 1) & 1u, abort_flag, true))) break;
        st_async_b32x2(r_fin0 + fb * kFinBytes + (uint32_t)row * 8u, r_finbar0 + 8u * fb, f2u(l), f2u(f));
      }
      // Drain: the value CTA's last (l, f) acknowledgements arrive here; wait
      // for them before the CTA can exit (the sender waits for the P-slot
      // credits).
      if (ok && e == 0) {
        for (uint32_t k = 0; ok && k < 2u && k < it; ++k) {
          const uint32_t il = it - 1 - k;
          ok = wait_warp(bar(kFinFree0 + (il & 1u)), (il >> 1) & 1u, abort_flag, true);
        }
      }
    }
  } else {
    // =============================== value CTA ===============================
    if (warp < kVStages) {
      // ---- gather of the 512 latent dims: warp w fills stage w for tiles g = w, w+5, ... ----
      const uint32_t s = (uint32_t)warp;
      const uint32_t stage = base + kOffV + s * kVStage;
      PCursor cur = pcursor_start(p, n_items, cid, ncl, (int)s);
      PCursor nx = cur;
      pcursor_advance(p, n_items, ncl, nx, kVStages);
      PCursor nx2 = nx;
      pcursor_advance(p, n_items, ncl, nx2, kVStages);
      int idx_cur = pcursor_index(p, cur, n_items, lane);
      int idx_nx = pcursor_index(p, nx, n_items, lane);
      uint32_t n = 0;
      while (cur.item < n_items) {
        if (n > 0 && !(ok = wait_warp(bar(kVFree0 + s), (n - 1) & 1u, abort_flag))) break;
        const int row = checked_index(pcursor_row(p, idx_cur, L), L, p.status);  // invalid rows get P = 0
        const int gb = checked_index(cur.w.batch, p.batch, p.status);
        gather_rows(stage, p.kv + (size_t)gb * L * kDimLatent, nullptr, row, lane, false, p.status);
        cp_async_commit();
        const int idx_nx2 = pcursor_index(p, nx2, n_items, lane);
        cp_async_wait<0>();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kVFull0 + s));
        ++n;
        cur = nx;
        nx = nx2;
        pcursor_advance(p, n_items, ncl, nx2, kVStages);
        idx_cur = idx_nx;
        idx_nx = idx_nx2;
      }
    } else if (warp == kPvWarp) {
      // ---- PV issuer: O[:, 0:256) and O[:, 256:512) += P . V ----
      const uint32_t idesc_pv = idesc_bf16(128, 256, false, true);
      volatile uint32_t* const req = reinterpret_cast<volatile uint32_t*>(sbase + kOffReq);
      uint32_t g = 0, it = 0, nresc = 0;
      for (int item = cid; item < n_items && ok; item += ncl, ++it) {
        const PItem w = make_pitem(p, item);
        for (int t = 0; t < w.ntiles; ++t, ++g) {
          const uint32_t vs = g % kVStages, s = g % kPSlots;
          if (!(ok = wait_warp(bar(kVFull0 + vs), (g / kVStages) & 1u, abort_flag))) break;
          if (!(ok = wait_warp(bar(kPFull0 + s), (g / kPSlots) & 1u, abort_flag))) break;
          const uint32_t slot = base + kOffSlot + s * kSlotBytes;
          // re-arm the slot for its next message (sent only after this PV's credit)
          if (elect_one()) mbar_arrive_expect_tx(bar(kPFull0 + s), kMsgBytes);
          __syncwarp();
          const volatile uint32_t* fl = reinterpret_cast<const volatile uint32_t*>(sbase + (slot - base) + kFlagOff);
          if ((fl[0] | fl[1] | fl[2] | fl[3]) != 0u) {
            if (elect_one()) {
              *req = kReqRescale | (g << 3) | s;
              mbar_arrive(bar(kReq));
            }
            __syncwarp();
            if (!(ok = wait_warp(bar(kReqDone), nresc & 1u, abort_flag))) break;
            ++nresc;
          }
          if (t == 0 && it > 0 && !(ok = wait_warp(bar(kOFree), (it - 1) & 1u, abort_flag))) break;
          const uint32_t vstage = base + kOffV + vs * kVStage;
          if (elect_one()) {
            tc_fence_after();
#pragma unroll
            for (int j = 0; j < kPrBN / 16; ++j) {
              const uint64_t ad = smem_desc(slot + j * 32, 16, 512, kLayoutSw64);
#pragma unroll
              for (int ch = 0; ch < 2; ++ch) {
                const uint64_t bd = smem_desc(vstage + (uint32_t)ch * 4u * kBlk + j * 2048, kBlk, 1024, kLayoutSw128);
                mma_bf16_ss(tmem + kTmemO + ch * 256, ad, bd, idesc_pv, (t == 0 && j == 0) ? 0u : 1u);
              }
            }
            mma_commit_mc(bar(kPSlotFree0 + s), (uint16_t)1);  // score CTA: P slot s is free
            mma_commit(bar(kVFree0 + vs));                      // value stage vs is free
          }
          __syncwarp();
        }
        if (!ok) break;
        // epilogue request for this item (the rescale warps read O once the last PV is done)
        if (elect_one()) {
          *req = it;
          mbar_arrive(bar(kReq));
        }
        __syncwarp();
      }
    } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kEpiWarps) {
      // ---- rescale requests and epilogue: one head row per thread, warp part
      // `part` of its lane quadrant owns O columns [cb0, cb1) ----
      const int quad = warp & 3;
      const int part = (warp - kEpiWarp0) >> 2;
      const int cb0 = 32 * epi_chunk0(part), cb1 = 32 * epi_chunk0(part + 1);
      if (kBoundsCheck && !(0 <= cb0 && cb0 < cb1 && cb1 <= (int)kTmemCols)) report_error(p.status, kErrBounds);
      const int row = quad * 32 + lane;
      const uint32_t t_lane = (uint32_t)(quad * 32) << 16;
      const volatile uint32_t* const req = reinterpret_cast<const volatile uint32_t*>(sbase + kOffReq);
      const uint32_t r_finfree0 = mapa_shared(bar(kFinFree0), 0);
      uint32_t nreq = 0, g_end = 0, it = 0;
      for (int item = cid; item < n_items && ok; item += ncl, ++it) {
        const PItem w = make_pitem(p, item);
        g_end += (uint32_t)w.ntiles;
        for (;;) {
          if (!(ok = wait_warp(bar(kReq), nreq & 1u, abort_flag))) break;
          ++nreq;
          const uint32_t r = *req;
          if (!(r & kReqRescale)) break;  // epilogue request of this item
          const uint32_t s = r & 7u;
          const uint32_t g = (r & ~kReqRescale) >> 3;
          const uint8_t* slot = sbase + kOffSlot + s * kSlotBytes;
          const uint32_t flag = *reinterpret_cast<const volatile uint32_t*>(slot + kFlagOff + quad * 4);
          if (flag != 0u) {
            const float alpha = *reinterpret_cast<const volatile float*>(slot + kAlphaOff + row * 4);
            // O is read and rescaled: the PV of tile g - 1 must be done
            const uint32_t gp = g - 1;
            if (!(ok = wait_warp(bar(kVFree0 + gp % kVStages), (gp / kVStages) & 1u, abort_flag))) break;
            tc_fence_after();
            uint32_t o[32];
#pragma unroll 1
            for (int cb = cb0; cb < cb1; cb += 32) {
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
          if (lane == 0) mbar_arrive(bar(kReqDone));
        }
        if (!ok) break;
        // ---- epilogue: (l, f) from the score CTA, O of the item's last PV ----
        const uint32_t fb = it & 1u;
        if (!(ok = wait_warp(bar(kFin0 + fb), (it >> 1) & 1u, abort_flag, true))) break;
        const volatile float* lfp = reinterpret_cast<const volatile float*>(sbase + kOffFin + fb * kFinBytes + row * 8);
        const float2 lf = make_float2(lfp[0], lfp[1]);
        __syncwarp();
        if (lane == 0) {
          if (quad == 0 && part == 0) mbar_arrive_expect_tx(bar(kFin0 + fb), kFinBytes);  // for item it + 2
          mbar_arrive_remote(r_finfree0 + 8u * fb);
        }
        const uint32_t gl = g_end - 1;
        if (!(ok = wait_warp(bar(kVFree0 + gl % kVStages), (gl / kVStages) & 1u, abort_flag))) break;
        tc_fence_after();
        const size_t orow = (size_t)w.token * kPrHeads + row;
        if (p.split == 1) {
          // O * (1/l) with the correctly rounded reciprocal (within an FP32 ulp of
          // O / l); a row without a valid index (l == 0) is written as 0
          const float rl = lf.x > 0.f ? __frcp_rn(lf.x) : 0.f;
          // the lane pair's two rows (orow and orow ^ 1: kPrHeads is even)
          __nv_bfloat16* dst = p.out + (orow & ~(size_t)1) * kDimLatent;
          const bool wide = (reinterpret_cast<uintptr_t>(p.out) & 31u) == 0;  // rows are 1024 B apart
          // one 32-column chunk at a time (with the next chunk's TMEM load in
          // flight during the stores the call measured ~1 % slower)
#pragma unroll 1
          for (int cb = cb0; cb < cb1; cb += 32) {
            uint32_t o[32];
            tmem_ld32(tmem + t_lane + kTmemO + cb, o);
            tmem_wait_ld();
            uint32_t a[8], b[8];
            pack_bf16_row32_paired(o, rl, a, b);
            store_bf16_row32_paired(dst + cb, kDimLatent, a, b, wide);
          }
        } else {
          const size_t pr = ((size_t)w.token * p.split + w.sp) * kPrHeads + row;
          float* dst = p.part_num + pr * kDimLatent;
#pragma unroll 1
          for (int cb = cb0; cb < cb1; cb += 32) {
            uint32_t o[32];
            tmem_ld32(tmem + t_lane + kTmemO + cb, o);
            tmem_wait_ld();
            float4* d4 = reinterpret_cast<float4*>(dst + cb);
#pragma unroll
            for (int k = 0; k < 8; ++k)
              d4[k] = make_float4(u2f(o[4 * k]) * lf.y, u2f(o[4 * k + 1]) * lf.y, u2f(o[4 * k + 2]) * lf.y,
                                  u2f(o[4 * k + 3]) * lf.y);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kOFree));
      }
    }
  }
  if (!ok && lane == 0) report_error(p.status, kErrTimeout);

  __syncwarp();
  tc_fence_before();
  cluster_sync();  // neither CTA leaves while the other may still address its shared memory
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

bool pair_launch_config(cudaLaunchConfig_t* cfg, cudaLaunchAttribute* attr, int ctas, cudaStream_t stream) {
  attr->id = cudaLaunchAttributeClusterDimension;
  attr->val.clusterDim.x = 2;
  attr->val.clusterDim.y = 1;
  attr->val.clusterDim.z = 1;
  *cfg = cudaLaunchConfig_t{};
  cfg->gridDim = dim3((unsigned)ctas, 1, 1);
  cfg->blockDim = dim3(kPrThreads, 1, 1);
  cfg->dynamicSmemBytes = kSmemBytes;
  cfg->stream = stream;
  cfg->attrs = attr;
  cfg->numAttrs = 1;
  return true;
}

}  // namespace

// Number of CTAs (two per cluster) that can be resident at once.
int pair_max_ctas() {
  static int cached = -1;
  if (cached > 0) return cached;
  if (cudaFuncSetAttribute(fwd_pair_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) !=
          cudaSuccess ||
      cudaFuncSetAttribute(fwd_pair_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) !=
          cudaSuccess)
    return -1;
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return -1;
  pair_launch_config(&cfg, &attr, sms & ~1, nullptr);
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, fwd_pair_kernel<false>, &cfg) != cudaSuccess || clusters <= 0)
    return -1;
  cached = 2 * clusters;
  return cached;
}

cudaError_t launch_fwd_pair(const FwdParams& p, cudaStream_t stream) {
  if (p.heads != kPrHeads || p.keys_per_tile != kPrBN || p.uent != nullptr) return cudaErrorInvalidValue;
  const int max_ctas = pair_max_ctas();
  if (max_ctas <= 0) return cudaErrorInvalidConfiguration;
  const long long items = (long long)p.tokens * p.split;
  const long long clusters = items < max_ctas / 2 ? items : max_ctas / 2;
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr;
  pair_launch_config(&cfg, &attr, (int)(2 * clusters), stream);
  return cudaLaunchKernelEx(&cfg, fwd_pair_kernel<false>, p);
}

// Union launch: p describes the blocks (tokens = blocks, heads = 128 rows,
// queries = blocks per batch row, split 1) and their union entries.
cudaError_t launch_fwd_pair_union(const FwdParams& p, cudaStream_t stream) {
  if (p.heads != kPrHeads || p.keys_per_tile != kPrBN || p.uent == nullptr || p.ulen == nullptr ||
      p.split != 1 || p.u_row_shift < 4 || p.u_row_shift > 6)
    return cudaErrorInvalidValue;
  const int max_ctas = pair_max_ctas();
  if (max_ctas <= 0) return cudaErrorInvalidConfiguration;
  const long long items = p.tokens;
  const long long clusters = items < max_ctas / 2 ? items : max_ctas / 2;
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr;
  pair_launch_config(&cfg, &attr, (int)(2 * clusters), stream);
  return cudaLaunchKernelEx(&cfg, fwd_pair_kernel<true>, p);
}

}  // namespace dsa
