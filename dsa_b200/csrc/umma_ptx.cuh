// Inline-PTX wrappers for the sm_100a tcgen05 / bulk-copy / cluster path.
//
// Every spin on an mbarrier is bounded (kWaitLimitNs of wall time read from
// %globaltimer unless the launch gives another limit); a wait that gives up
// returns false and the caller reports kErrTimeout through the status word
// instead of trapping.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "dsa_common.cuh"

namespace dsa {
namespace umma {

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
// Arrive on a barrier in another CTA of the cluster (address from mapa).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar)
               : "memory");
}
// try_wait suspends the waiting warp (instead of spinning) until the phase
// completes or kSuspendHintNs pass, so waiting warps leave the issue slots of
// their scheduler to the warps that share it.
constexpr uint32_t kSuspendHintNs = 20000;

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}
// Non-blocking: has the phase with this parity completed?
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; `abort` is a shared flag other roles set after a timeout.
// The wait gives up `limit_ns` after its 16th unsuccessful try.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                          bool cluster_scope = false,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  unsigned long long start = 0;
  for (uint32_t it = 0;; ++it) {
    if (cluster_scope ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 15u) {
      if (*abort) return false;
      const unsigned long long now = global_ns();
      if (start == 0) start = now;
      else if (now - start > limit_ns) {
        *abort = 1;
        return false;
      }
    }
  }
}

// Bounded wait (kWaitLimitNs) that ignores the abort flag: used on the abort
// path itself, for completions that always arrive (a tcgen05.commit of
// tensor-core work already issued).
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity) {
  unsigned long long start = 0;
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 15u) {
      const unsigned long long now = global_ns();
      if (start == 0) start = now;
      else if (now - start > kWaitLimitNs) return false;
    }
  }
}

// Bounded wait (lane 0 polls) until a shared word equals `value`; the same
// result in every lane of the warp.
__device__ __forceinline__ bool wait_word_warp(volatile uint32_t* word, uint32_t value, volatile int* abort,
                                               unsigned long long limit_ns = kWaitLimitNs) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0 && *word != value) {
    const unsigned long long start = global_ns();
    for (uint32_t k = 1; *word != value; ++k) {
      if ((k & 3u) == 0) {
        if (*abort) {
          ok = false;
          break;
        }
        if (global_ns() - start > limit_ns) {
          *abort = 1;
          ok = false;
          break;
        }
      }
      __nanosleep(32);
    }
  }
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// ---- cluster / DSMEM ------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// from this CTA's shared memory into a peer CTA's (shared::cluster address
// from mapa); complete_tx on the peer's mbarrier `remote_bar`. No multicast.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t remote_dst, uint32_t local_src, uint32_t bytes,
                                                  uint32_t remote_bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          remote_dst),
      "r"(local_src), "r"(bytes), "r"(remote_bar)
      : "memory");
}
// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// from this CTA's shared memory to global memory, tracked by bulk groups.
__device__ __forceinline__ void bulk_store_global(void* gdst, uint32_t local_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(gdst)),
               "r"(local_src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until this thread's bulk copy groups have completed (writes performed).
__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Wait until at most N of this thread's bulk copy groups still read their source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Named CTA barrier `id` (1..15; 0 is __syncthreads) over `threads` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// Split cluster barrier: arrive (no ordering) now, wait (acquire) later.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// 8 bytes into a cluster peer's shared memory (shared::cluster address from mapa).
__device__ __forceinline__ void st_shared_cluster_f2(uint32_t addr, float2 v) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(v.x), "f"(v.y) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// ---- fences -----------------------------------------------------------------------
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Async-proxy global writes (bulk copies) -> ordered before later generic operations.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// True in exactly one lane of a converged warp. tcgen05.mma / commit issued
// under this predicate keep the warp converged and issue at the tensor
// core's rate (a lane-0 branch measured ~60 cycles per MMA instead of ~17
// for M=128, N=32).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}


// ---- tcgen05 -------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (BF16 in, FP32 accumulate).
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}
// Same with the A operand read from tensor memory (M rows in TMEM lanes, two
// 16-bit K elements per 32-bit column).
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}
// Arrive once on a CTA-local mbarrier when all prior tcgen05.mma of this thread complete.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// tcgen05.wait::ld that also names the 32 destination registers of an
// earlier tcgen05.ld, so the compiler cannot move their uses above the wait
// (needed when a second load is in flight while the first is consumed).
__device__ __forceinline__ void tmem_wait_ld_regs32(uint32_t* r) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
        "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
        "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
        "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t gets row (lane base + t), columns c..c+31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// L2 prefetch of `bytes` (a multiple of 16) contiguous global bytes at a
// 16-byte-aligned address; a hint without completion tracking.
__device__ __forceinline__ void prefetch_l2_bulk(const void* gptr, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(gptr)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// ---- descriptors ------------------------------------------------------------------------
// Shared-memory matrix descriptor (sm_100 format): start>>4 [0,14), LBO>>4
// [16,30), SBO>>4 [32,46), version 1 at [46,48), layout type at [61,64)
// (2 = 128-byte swizzle, 4 = 64-byte swizzle).
constexpr uint32_t kLayoutSw128 = 2;
constexpr uint32_t kLayoutSw64 = 4;
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

// Instruction descriptor for kind::f16 with BF16 A/B and FP32 D.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// ---- row stores of the epilogues -------------------------------------------------------
__device__ __forceinline__ void st_global_v8(void* dst, const uint32_t* h) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(dst), "r"(h[0]), "r"(h[1]), "r"(h[2]),
               "r"(h[3]), "r"(h[4]), "r"(h[5]), "r"(h[6]), "r"(h[7])
               : "memory");
}

// 32 FP32 values (O columns of one head row) * rl -> 32 BF16 at dst (64 B).
// Each thread writes its own row, so a warp store touches 32 rows: 32-byte
// stores (whole L2 sectors, half the requests of 16-byte ones) when dst is
// 32-byte aligned (`wide`), 16-byte stores otherwise.
__device__ __forceinline__ void store_bf16_row32(__nv_bfloat16* dst, const uint32_t* o, float rl, bool wide) {
  uint32_t h[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) h[k] = pack_bf16x2(__uint_as_float(o[2 * k]) * rl, __uint_as_float(o[2 * k + 1]) * rl);
  if (wide) {
    st_global_v8(dst, h);
    st_global_v8(dst + 16, h + 8);
  } else {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int k = 0; k < 4; ++k) d4[k] = make_uint4(h[4 * k], h[4 * k + 1], h[4 * k + 2], h[4 * k + 3]);
  }
}

// store_bf16_row32 for a lane pair, in two steps. Pack: this lane's 32 FP32
// values (its row) * rl -> BF16, exchanged with the partner lane (lane ^ 1)
// so that a[] holds 32 bytes of the pair's even row and b[] 32 bytes of its
// odd row (bytes 0..31 in the even lane, 32..63 in the odd lane). Store:
// each store instruction then writes 64 contiguous bytes of one row per lane
// pair (16 rows x 64 B per warp instruction instead of 32 rows x 32 B:
// ~1.5x the per-SM store rate). All 32 lanes take part in the pack.
__device__ __forceinline__ void pack_bf16_row32_paired(const uint32_t* o, float rl, uint32_t* a, uint32_t* b) {
  const bool odd = (threadIdx.x & 1u) != 0u;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t lo = pack_bf16x2(__uint_as_float(o[2 * k]) * rl, __uint_as_float(o[2 * k + 1]) * rl);
    const uint32_t hi = pack_bf16x2(__uint_as_float(o[16 + 2 * k]) * rl, __uint_as_float(o[17 + 2 * k]) * rl);
    const uint32_t got = __shfl_xor_sync(0xffffffffu, odd ? lo : hi, 1);
    a[k] = odd ? got : lo;
    b[k] = odd ? hi : got;
  }
}
// `dst_even`: the chunk's first element in the pair's even row; the odd row
// starts `row_stride` elements later.
__device__ __forceinline__ void store_bf16_row32_paired(__nv_bfloat16* dst_even, size_t row_stride, const uint32_t* a,
                                                        const uint32_t* b, bool wide) {
  __nv_bfloat16* const de = dst_even + ((threadIdx.x & 1u) ? 16 : 0);
  __nv_bfloat16* const dod = de + row_stride;
  if (wide) {
    st_global_v8(de, a);
    st_global_v8(dod, b);
  } else {
    uint4* const e4 = reinterpret_cast<uint4*>(de);
    uint4* const o4 = reinterpret_cast<uint4*>(dod);
    e4[0] = make_uint4(a[0], a[1], a[2], a[3]);
    e4[1] = make_uint4(a[4], a[5], a[6], a[7]);
    o4[0] = make_uint4(b[0], b[1], b[2], b[3]);
    o4[1] = make_uint4(b[4], b[5], b[6], b[7]);
  }
}

// 32 FP32 values * f -> dst (128 B of an FP32 partial row); 32-byte stores
// when dst is 32-byte aligned (`wide`), 16-byte stores otherwise.
__device__ __forceinline__ void store_f32_row32(float* dst, const uint32_t* o, float f, bool wide) {
  uint32_t h[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) h[k] = __float_as_uint(__uint_as_float(o[k]) * f);
  if (wide) {
#pragma unroll
    for (int k = 0; k < 4; ++k) st_global_v8(dst + 8 * k, h + 8 * k);
  } else {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int k = 0; k < 8; ++k) d4[k] = make_uint4(h[4 * k], h[4 * k + 1], h[4 * k + 2], h[4 * k + 3]);
  }
}

}  // namespace umma
}  // namespace dsa
