// extern "C" boundary of libdsa_b200.so (declared in include/dsa_b200.h).
//
// Host-side orchestration of one forward call, the C++ counterpart of the
// reference's forward (dsa/api.py:76-132): pick or check the launch entry,
// carve the split partials out of the caller's workspace, launch the main
// kernel and, for split > 1, the FP32 merge. Input validation of shapes and
// dtypes happens in the Python mirror (dsa_b200/api.py); here only what the
// C ABI can see is checked (null pointers, sizes, alignment, launch entry).
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>

#include "../../include/dsa_b200.h"
#include "dsa_common.cuh"

namespace {

thread_local int g_last_launch_count = 0;

// Failure-path test settings of dsa_set_wait_test (process-wide).
std::atomic<unsigned long long> g_wait_limit_ns{0};
std::atomic<int> g_wait_test{0};

constexpr uint64_t kAlign = 256;
inline uint64_t align_up(uint64_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

bool shape_ok(int64_t b, int64_t sq, int64_t h, int64_t l, int64_t k) {
  if (b <= 0 || sq <= 0 || h <= 0 || l <= 0 || k <= 0) return false;
  if (b * sq > 0x7fffffffLL || l > 0x7fffffffLL || k > 0x7fffffffLL || h > 0x7fffffffLL) return false;
  if (b * l > 0x7fffffffLL) return false;
  return true;
}

struct Layout {
  uint64_t num_off, max_off, sum_off, total;
};

// Split partials (dsa/api.py:111-113): numerator [T, S, H, 512] FP32 and
// max / sum [T, S, H] FP32. The umma family's cluster merge keeps the
// numerator as [T, 2, S, H, 256] and, instead of max / sum, (max, sum)
// pairs per value half [T, 2, S, H] (each cluster merges one half on its own).
Layout partial_layout(int64_t tokens, int64_t heads, int64_t split, bool cluster_merge = false) {
  Layout lay{0, 0, 0, 0};
  if (split <= 1) return lay;
  const uint64_t rows = (uint64_t)tokens * (uint64_t)split * (uint64_t)heads;
  lay.num_off = 0;
  lay.max_off = align_up(rows * dsa::kDimLatent * sizeof(float));
  if (cluster_merge) {
    lay.sum_off = lay.max_off;
    lay.total = lay.max_off + align_up(rows * 2u * 2u * sizeof(float));
    return lay;
  }
  lay.sum_off = lay.max_off + align_up(rows * sizeof(float));
  lay.total = lay.sum_off + align_up(rows * sizeof(float));
  return lay;
}

// Whether a launch entry's partials take the split-V cluster merge's layout.
bool umma_layout_merge(const dsa_launch_t& e) {
  return e.family == DSA_FAMILY_UMMA && e.split > 1 && dsa::umma_cluster_merge(e.split);
}

// Whether a launch entry merges its split partials inside the main kernel
// (the split-V and stream families' cluster launches).
bool merges_in_kernel(const dsa_launch_t& e) {
  if (e.split <= 1) return false;
  if (e.family == DSA_FAMILY_UMMA) return dsa::umma_cluster_merge(e.split);
  if (e.family == DSA_FAMILY_STREAM) return dsa::stream_cluster_merge(e.split);
  return false;
}

// Union launch: per block of 128 / H queries, up to (128 / H) * topk union
// entries and their count.
struct UnionLayout {
  uint64_t ent_off, len_off, total;
  int64_t blocks, ucap;
};
UnionLayout union_layout(int64_t tokens, int64_t heads, int64_t topk) {
  UnionLayout u{0, 0, 0, 0, 0};
  const int64_t qpb = 128 / heads;
  u.blocks = tokens / qpb;
  u.ucap = qpb * topk;
  u.len_off = align_up((uint64_t)u.blocks * (uint64_t)u.ucap * sizeof(int32_t));
  u.total = u.len_off + align_up((uint64_t)u.blocks * sizeof(int32_t));
  return u;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Largest TOPK of the union launch: union_build_kernel keeps each query's
// count of a key in a 16-bit half-word, and (128 / H) * TOPK entries per
// block must fit an int.
constexpr int64_t kUnionMaxTopk = 65535;

}  // namespace

extern "C" {

int dsa_abi_version(void) { return DSA_B200_ABI_VERSION; }

const char* dsa_status_string(int status) {
  switch (status) {
    case DSA_STATUS_OK: return "ok";
    case DSA_STATUS_BAD_ARGUMENT: return "bad argument";
    case DSA_STATUS_UNSUPPORTED: return "launch entry not supported for this shape";
    case DSA_STATUS_WORKSPACE_TOO_SMALL: return "workspace too small";
    case DSA_STATUS_LAUNCH_FAILED: return "kernel launch failed";
    case DSA_STATUS_DEVICE_TIMEOUT: return "device-side wait timed out";
    case DSA_STATUS_CUDA_ERROR: return "CUDA runtime error";
    default: return "unknown status";
  }
}

int dsa_check_launch(int64_t batch, int64_t queries, int64_t heads, int64_t length, int64_t topk,
                     const dsa_launch_t* launch) {
  if (launch == nullptr || !shape_ok(batch, queries, heads, length, topk))
    return DSA_STATUS_BAD_ARGUMENT;
  const int bn = launch->keys_per_tile;
  if (launch->split < 1) return DSA_STATUS_UNSUPPORTED;
  switch (launch->family) {
    case DSA_FAMILY_WARP_MMA: {
      if (launch->heads_per_cta != 16 || heads % 16 != 0) return DSA_STATUS_UNSUPPORTED;
      if (bn != 32 && bn != 64) return DSA_STATUS_UNSUPPORTED;
      break;
    }
    case DSA_FAMILY_STREAM: {
      if (launch->heads_per_cta != 16 || heads % 16 != 0 || bn != 32) return DSA_STATUS_UNSUPPORTED;
      break;
    }
    case DSA_FAMILY_KEYS: {
      if (launch->heads_per_cta != 16 || heads % 16 != 0 || bn != 64) return DSA_STATUS_UNSUPPORTED;
      break;
    }
    case DSA_FAMILY_PAIR_UNION: {
      if (launch->heads_per_cta != 128 || bn != 32 || launch->split != 1) return DSA_STATUS_UNSUPPORTED;
      if (heads != 16 && heads != 32 && heads != 64) return DSA_STATUS_UNSUPPORTED;
      if (queries % (128 / heads) != 0 || length >= (1 << 24)) return DSA_STATUS_UNSUPPORTED;
      // the union build counts a key's repeats per query in 16 bits
      if (topk > kUnionMaxTopk) return DSA_STATUS_UNSUPPORTED;
      break;
    }
    case DSA_FAMILY_UMMA:
    case DSA_FAMILY_UMMA_PAIR: {
      if (launch->heads_per_cta != 128 || heads != 128 || bn != 32) return DSA_STATUS_UNSUPPORTED;
      break;
    }
    default:
      return DSA_STATUS_UNSUPPORTED;
  }
  const int64_t tiles = (topk + bn - 1) / bn;
  if (launch->split > tiles) return DSA_STATUS_UNSUPPORTED;
  return DSA_STATUS_OK;
}

int dsa_default_launch(int64_t batch, int64_t queries, int64_t heads, int64_t length, int64_t topk,
                       dsa_launch_t* out) {
  if (out == nullptr || !shape_ok(batch, queries, heads, length, topk))
    return DSA_STATUS_BAD_ARGUMENT;
  if (heads % 16 != 0) return DSA_STATUS_UNSUPPORTED;
  dsa_launch_t e;
  if (heads == 128) {
    e.heads_per_cta = 128;
    e.keys_per_tile = 32;
    int ctas = dsa::umma_max_ctas();
    if (ctas <= 0) ctas = sm_count();
    const int64_t halves = 2 * batch * queries;
    const int64_t tiles = (topk + 31) / 32;
    const int pair_ctas = dsa::pair_max_ctas();
    if (pair_ctas > 0 && ctas / halves < 2) {
      // pair family: one (score CTA, value CTA) cluster per query, once the
      // split-V family could no longer split the TOPK range (a pair's tile
      // costs ~0.6 us against ~1 us for a split-V CTA, which also computes
      // QK twice); measured on B200: 64 queries 65.5 us against 82.0 us,
      // 32 queries (split-V split 2) 53 us and no faster as pairs.
      e.family = DSA_FAMILY_UMMA_PAIR;
      e.split = 1;
      *out = e;
      return DSA_STATUS_OK;
    }
    // split-V family for few queries: persistent CTAs over (token, split,
    // V half) items; split the TOPK range only until every resident CTA has
    // an item.
    e.family = DSA_FAMILY_UMMA;
    int64_t split = ctas / halves;  // one wave: at most one item per resident CTA
    // at least two tiles per item: a one-tile item is all start-up (Q load,
    // first gather, epilogue) and doubles the partials the merge reads
    if (split > tiles / 2) split = tiles / 2;
    // the split CTAs of a (token, value half) merge their partials as one
    // cluster (at most 16 CTAs), all clusters resident at once if possible
    if (split > 1) split = dsa::umma_cluster_split(halves, (int)split);
    if (split < 1) split = 1;
    e.split = (int32_t)split;
    *out = e;
    return DSA_STATUS_OK;
  }
  // union launch of the pair family for 16, 32 or 64 heads: blocks of
  // 128 / H queries of one batch row over the union of their keys, when the
  // blocks fill the clusters and the keys are dense enough that the MMA work
  // (128 rows x the union) stays within ~4x the per-query work, which the
  // tcgen05 pair kernel still beats the mma.sync stream family at: L <= 4
  // TOPK (8 queries' union ~3.6 TOPK for H = 16, 4 queries' ~2.7 TOPK for
  // H = 32), any L for H = 64 (a 2-query union is at most 2 TOPK). Measured
  // on B200 (B=4, SQ=8192, L=8192, TOPK=2048): H = 64 18.8 ms against 46.6 ms,
  // H = 32 14.6 ms against 23.3 ms for the stream family.
  const bool dense = heads == 64 || length <= 4 * topk;
  if ((heads == 16 || heads == 32 || heads == 64) && queries % (128 / heads) == 0 && dense &&
      length < (1 << 24) && topk <= kUnionMaxTopk) {
    const int pair_ctas = dsa::pair_max_ctas();
    if (pair_ctas > 0 && batch * queries / (128 / heads) >= pair_ctas / 2) {
      e.family = DSA_FAMILY_PAIR_UNION;
      e.heads_per_cta = 128;
      e.keys_per_tile = 32;
      e.split = 1;
      *out = e;
      return DSA_STATUS_OK;
    }
  }
  // stream family: persistent CTAs over (token, 16-head group, split)
  // items; split the TOPK range only until every resident CTA has an item.
  e.family = DSA_FAMILY_STREAM;
  e.heads_per_cta = 16;
  e.keys_per_tile = 32;
  int ctas = dsa::stream_max_ctas();
  if (ctas <= 0) ctas = 2 * sm_count();
  const int64_t jobs = batch * queries * (heads / 16);
  const int64_t tiles = (topk + e.keys_per_tile - 1) / e.keys_per_tile;
  int64_t split = ctas / jobs;  // one wave of items
  if (split > tiles) split = tiles;
  // with four or more jobs, at most the eight splits that merge inside the
  // cluster launch (one kernel; measured faster than more splits and the
  // merge kernel for 4-8 jobs: 22.5-22.6 us against 23.6-25.6 us)
  if (jobs >= 4 && split > 8) split = 8;
  if (split < 1) split = 1;
  e.split = (int32_t)split;
  *out = e;
  return DSA_STATUS_OK;
}

uint64_t dsa_fwd_workspace_bytes(const dsa_fwd_args_t* a) {
  if (a == nullptr) return 0;
  dsa_launch_t e = a->launch;
  if (e.family == DSA_FAMILY_AUTO &&
      dsa_default_launch(a->batch, a->queries, a->heads, a->length, a->topk, &e) != DSA_STATUS_OK)
    return 0;
  if (dsa_check_launch(a->batch, a->queries, a->heads, a->length, a->topk, &e) != DSA_STATUS_OK)
    return 0;
  if (e.family == DSA_FAMILY_PAIR_UNION) return union_layout(a->batch * a->queries, a->heads, a->topk).total;
  return partial_layout(a->batch * a->queries, a->heads, e.split, umma_layout_merge(e)).total;
}

int dsa_sparse_mla_fwd(const dsa_fwd_args_t* a, void* stream) {
  g_last_launch_count = 0;
  if (a == nullptr) return DSA_STATUS_BAD_ARGUMENT;
  if (!a->q || !a->kv || !a->q_rope || !a->k_rope || !a->indices || !a->output ||
      !a->softmax_max || !a->softmax_sum)
    return DSA_STATUS_BAD_ARGUMENT;
  if (!aligned16(a->q) || !aligned16(a->kv) || !aligned16(a->q_rope) || !aligned16(a->k_rope) ||
      !aligned16(a->output))
    return DSA_STATUS_BAD_ARGUMENT;
  dsa_launch_t e = a->launch;
  if (e.family == DSA_FAMILY_AUTO) {
    int st = dsa_default_launch(a->batch, a->queries, a->heads, a->length, a->topk, &e);
    if (st != DSA_STATUS_OK) return st;
  }
  int st = dsa_check_launch(a->batch, a->queries, a->heads, a->length, a->topk, &e);
  if (st != DSA_STATUS_OK) return st;

  const int64_t tokens = a->batch * a->queries;
  const bool fused_merge = merges_in_kernel(e);
  const Layout lay = partial_layout(tokens, a->heads, e.split, umma_layout_merge(e));
  if (e.family == DSA_FAMILY_PAIR_UNION) {
    const UnionLayout ul = union_layout(tokens, a->heads, a->topk);
    if (a->workspace == nullptr || a->workspace_bytes < ul.total ||
        (reinterpret_cast<uintptr_t>(a->workspace) & (kAlign - 1)) != 0)
      return DSA_STATUS_WORKSPACE_TOO_SMALL;
  }
  if (lay.total > 0) {
    if (a->workspace == nullptr || a->workspace_bytes < lay.total ||
        (reinterpret_cast<uintptr_t>(a->workspace) & (kAlign - 1)) != 0)
      return DSA_STATUS_WORKSPACE_TOO_SMALL;
  }
  char* ws = static_cast<char*>(a->workspace);

  dsa::FwdParams p;
  std::memset(&p, 0, sizeof(p));
  p.q = static_cast<const __nv_bfloat16*>(a->q);
  p.kv = static_cast<const __nv_bfloat16*>(a->kv);
  p.q_rope = static_cast<const __nv_bfloat16*>(a->q_rope);
  p.k_rope = static_cast<const __nv_bfloat16*>(a->k_rope);
  p.ids = a->indices;
  p.out = static_cast<__nv_bfloat16*>(a->output);
  p.out_max = a->softmax_max;
  p.out_sum = a->softmax_sum;
  if (e.split > 1) {
    p.part_num = reinterpret_cast<float*>(ws + lay.num_off);
    p.part_max = reinterpret_cast<float*>(ws + lay.max_off);
    p.part_sum = reinterpret_cast<float*>(ws + lay.sum_off);
  }
  p.status = a->status;
  p.batch = (int)a->batch;
  p.queries = (int)a->queries;
  p.heads = (int)a->heads;
  p.length = (int)a->length;
  p.topk = (int)a->topk;
  p.tokens = (int)tokens;
  p.split = e.split;
  p.keys_per_tile = e.keys_per_tile;
  p.heads_per_cta = e.heads_per_cta;
  if (!dsa::fill_scale(a->scale, p)) return DSA_STATUS_BAD_ARGUMENT;
  p.wait_limit_ns = g_wait_limit_ns.load(std::memory_order_relaxed);
  p.wait_test = g_wait_test.load(std::memory_order_relaxed);

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err = cudaSuccess;
  switch (e.family) {
    case DSA_FAMILY_WARP_MMA: err = dsa::launch_fwd_warp_mma(p, s); break;
    case DSA_FAMILY_UMMA: err = dsa::launch_fwd_umma(p, s); break;
    case DSA_FAMILY_UMMA_PAIR: err = dsa::launch_fwd_pair(p, s); break;
    case DSA_FAMILY_STREAM: err = dsa::launch_fwd_stream(p, s); break;
    case DSA_FAMILY_KEYS: err = dsa::launch_fwd_keys(p, s); break;
    case DSA_FAMILY_PAIR_UNION: {
      // blocks of 128 / H queries become 128-row items over their union entries
      const UnionLayout ul = union_layout(tokens, a->heads, a->topk);
      const int qpb = 128 / (int)a->heads;
      int32_t* uent = reinterpret_cast<int32_t*>(ws + ul.ent_off);
      int32_t* ulen = reinterpret_cast<int32_t*>(ws + ul.len_off);
      err = dsa::launch_union_build(p.ids, p.topk, p.length, qpb, (int)ul.blocks, uent, ulen, (int)ul.ucap, s);
      if (err != cudaSuccess) break;
      dsa::FwdParams pu = p;
      pu.tokens = (int)ul.blocks;
      pu.queries = (int)(a->queries / qpb);
      pu.heads = 128;
      pu.heads_per_cta = 128;
      pu.uent = uent;
      pu.ulen = ulen;
      pu.ucap = (int)ul.ucap;
      pu.u_row_shift = a->heads == 16 ? 4 : a->heads == 32 ? 5 : 6;
      err = dsa::launch_fwd_pair_union(pu, s);
      break;
    }
    default: return DSA_STATUS_UNSUPPORTED;
  }
  if (err != cudaSuccess) return DSA_STATUS_LAUNCH_FAILED;
  int launches = e.family == DSA_FAMILY_PAIR_UNION ? 2 : 1;  // union build + pair kernel
  if (e.split > 1 && !fused_merge) {
    err = dsa::launch_merge(p.part_num, p.part_max, p.part_sum, p.out, p.out_max, p.out_sum,
                            p.tokens, p.heads, p.split, s);
    if (err != cudaSuccess) return DSA_STATUS_LAUNCH_FAILED;
    ++launches;
  }
  g_last_launch_count = launches;
  return DSA_STATUS_OK;
}

int dsa_merge_partials(const float* numerator, const float* partial_max, const float* partial_sum,
                       void* output, float* softmax_max, float* softmax_sum, int64_t tokens,
                       int64_t heads, int64_t split, void* stream) {
  if (!numerator || !partial_max || !partial_sum || !output || !softmax_max || !softmax_sum)
    return DSA_STATUS_BAD_ARGUMENT;
  if (tokens <= 0 || heads <= 0 || split <= 0 || tokens * heads > 0x7fffffffLL)
    return DSA_STATUS_BAD_ARGUMENT;
  if (!aligned16(numerator) || (reinterpret_cast<uintptr_t>(output) & 7u) != 0)
    return DSA_STATUS_BAD_ARGUMENT;
  cudaError_t err = dsa::launch_merge(numerator, partial_max, partial_sum,
                                      static_cast<__nv_bfloat16*>(output), softmax_max,
                                      softmax_sum, (int)tokens, (int)heads, (int)split,
                                      static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? DSA_STATUS_OK : DSA_STATUS_LAUNCH_FAILED;
}

int dsa_last_launch_count(void) { return g_last_launch_count; }

namespace {
// Inner (flat-pool) forward arguments of a paged call; false when invalid.
bool paged_inner(const dsa_fwd_args_t* a, const dsa_paged_kv_t* pg, dsa_fwd_args_t* inner, uint64_t* rows_bytes) {
  if (a == nullptr || pg == nullptr || pg->block_table == nullptr) return false;
  if (pg->max_blocks <= 0 || pg->block_size <= 0 || pg->num_blocks <= 0) return false;
  if (pg->num_blocks * pg->block_size > 0x7fffffffLL || pg->max_blocks * pg->block_size > 0x7fffffffLL) return false;
  if (!shape_ok(a->batch, a->queries, a->heads, 1, a->topk)) return false;
  *inner = *a;
  inner->batch = 1;
  inner->queries = a->batch * a->queries;
  inner->length = pg->num_blocks * pg->block_size;
  *rows_bytes = align_up((uint64_t)a->batch * (uint64_t)a->queries * (uint64_t)a->topk * sizeof(int32_t));
  return true;
}
}  // namespace

uint64_t dsa_fwd_paged_workspace_bytes(const dsa_fwd_args_t* a, const dsa_paged_kv_t* pg) {
  dsa_fwd_args_t inner;
  uint64_t rows_bytes = 0;
  if (!paged_inner(a, pg, &inner, &rows_bytes)) return 0;
  dsa_launch_t e = inner.launch;
  if (e.family == DSA_FAMILY_AUTO &&
      dsa_default_launch(inner.batch, inner.queries, inner.heads, inner.length, inner.topk, &e) != DSA_STATUS_OK)
    return 0;
  if (dsa_check_launch(inner.batch, inner.queries, inner.heads, inner.length, inner.topk, &e) != DSA_STATUS_OK)
    return 0;
  inner.launch = e;
  return rows_bytes + dsa_fwd_workspace_bytes(&inner);
}

int dsa_sparse_mla_fwd_paged(const dsa_fwd_args_t* a, const dsa_paged_kv_t* pg, void* stream) {
  g_last_launch_count = 0;
  dsa_fwd_args_t inner;
  uint64_t rows_bytes = 0;
  if (!paged_inner(a, pg, &inner, &rows_bytes) || a->indices == nullptr) return DSA_STATUS_BAD_ARGUMENT;
  if (a->workspace == nullptr || a->workspace_bytes < rows_bytes ||
      (reinterpret_cast<uintptr_t>(a->workspace) & (kAlign - 1)) != 0)
    return DSA_STATUS_WORKSPACE_TOO_SMALL;
  int32_t* rows = static_cast<int32_t*>(a->workspace);
  inner.indices = rows;
  inner.workspace = a->workspace_bytes > rows_bytes ? static_cast<char*>(a->workspace) + rows_bytes : nullptr;
  inner.workspace_bytes = a->workspace_bytes - rows_bytes;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dsa::launch_paged_rows(a->indices, pg->block_table, pg->seq_lens, rows, a->batch * a->queries * a->topk,
                             (int)(a->queries * a->topk), (int)pg->max_blocks, (int)pg->block_size,
                             (int)pg->num_blocks, s) != cudaSuccess)
    return DSA_STATUS_LAUNCH_FAILED;
  const int st = dsa_sparse_mla_fwd(&inner, stream);
  if (st != DSA_STATUS_OK) return st;
  g_last_launch_count += 1;
  return DSA_STATUS_OK;
}

namespace {
// Inner (dequantised, compact) forward of an FP8 call: B*SQ batch rows of
// one query each over its TOPK gathered rows.
struct Fp8Layout {
  uint64_t kv_off, kr_off, ids_off, fwd_off;
};
bool fp8_inner(const dsa_fwd_args_t* a, dsa_fwd_args_t* inner, Fp8Layout* lay) {
  if (a == nullptr || !shape_ok(a->batch, a->queries, a->heads, a->length, a->topk)) return false;
  const uint64_t rows = (uint64_t)a->batch * (uint64_t)a->queries * (uint64_t)a->topk;
  if (rows > 0x7fffffffULL) return false;
  *inner = *a;
  inner->batch = a->batch * a->queries;
  inner->queries = 1;
  inner->length = a->topk;
  lay->kv_off = 0;
  lay->kr_off = align_up(rows * dsa::kDimLatent * 2u);
  lay->ids_off = lay->kr_off + align_up(rows * dsa::kDimRope * 2u);
  lay->fwd_off = lay->ids_off + align_up(rows * 4u);
  return true;
}
}  // namespace

uint64_t dsa_fwd_fp8_workspace_bytes(const dsa_fwd_args_t* a) {
  dsa_fwd_args_t inner;
  Fp8Layout lay;
  if (!fp8_inner(a, &inner, &lay)) return 0;
  dsa_launch_t e = inner.launch;
  if (e.family == DSA_FAMILY_AUTO &&
      dsa_default_launch(inner.batch, inner.queries, inner.heads, inner.length, inner.topk, &e) != DSA_STATUS_OK)
    return 0;
  if (dsa_check_launch(inner.batch, inner.queries, inner.heads, inner.length, inner.topk, &e) != DSA_STATUS_OK)
    return 0;
  inner.launch = e;
  return lay.fwd_off + dsa_fwd_workspace_bytes(&inner);
}

int dsa_sparse_mla_fwd_fp8(const dsa_fwd_args_t* a, void* stream) {
  g_last_launch_count = 0;
  dsa_fwd_args_t inner;
  Fp8Layout lay;
  if (!fp8_inner(a, &inner, &lay) || a->kv == nullptr || a->indices == nullptr) return DSA_STATUS_BAD_ARGUMENT;
  if (!aligned16(a->kv)) return DSA_STATUS_BAD_ARGUMENT;
  if (a->workspace == nullptr || a->workspace_bytes < lay.fwd_off ||
      (reinterpret_cast<uintptr_t>(a->workspace) & (kAlign - 1)) != 0)
    return DSA_STATUS_WORKSPACE_TOO_SMALL;
  char* ws = static_cast<char*>(a->workspace);
  __nv_bfloat16* kv_c = reinterpret_cast<__nv_bfloat16*>(ws + lay.kv_off);
  __nv_bfloat16* kr_c = reinterpret_cast<__nv_bfloat16*>(ws + lay.kr_off);
  int32_t* ids_c = reinterpret_cast<int32_t*>(ws + lay.ids_off);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dsa::launch_fp8_gather(static_cast<const uint8_t*>(a->kv), a->indices, kv_c, kr_c, ids_c,
                             a->batch * a->queries * a->topk, (int)a->topk, (int)a->queries, (int)a->length,
                             s) != cudaSuccess)
    return DSA_STATUS_LAUNCH_FAILED;
  inner.kv = kv_c;
  inner.k_rope = kr_c;
  inner.indices = ids_c;
  inner.workspace = a->workspace_bytes > lay.fwd_off ? ws + lay.fwd_off : nullptr;
  inner.workspace_bytes = a->workspace_bytes - lay.fwd_off;
  const int st = dsa_sparse_mla_fwd(&inner, stream);
  if (st != DSA_STATUS_OK) return st;
  g_last_launch_count += 1;
  return DSA_STATUS_OK;
}

namespace {
bool indexer_ok(const dsa_indexer_args_t* a) {
  if (a == nullptr) return false;
  if (a->batch <= 0 || a->queries <= 0 || a->length <= 0 || a->topk <= 0) return false;
  if (a->heads != 16 && a->heads != 32 && a->heads != 64 && a->heads != 128) return false;
  if (a->batch * a->queries > 0x7fffffffLL || a->length > 0x7fffffffLL || a->topk > 0x7fffffffLL) return false;
  return true;
}
}  // namespace

uint64_t dsa_indexer_workspace_bytes(const dsa_indexer_args_t* a) {
  if (!indexer_ok(a) || a->scores != nullptr) return 0;
  return align_up((uint64_t)a->batch * (uint64_t)a->queries * (uint64_t)a->length * sizeof(float));
}

int dsa_indexer_topk(const dsa_indexer_args_t* a, void* stream) {
  if (!indexer_ok(a) || !a->q || !a->k || !a->weights || !a->indices) return DSA_STATUS_BAD_ARGUMENT;
  if (!aligned16(a->q) || !aligned16(a->k)) return DSA_STATUS_BAD_ARGUMENT;
  float* scores = a->scores;
  if (scores == nullptr) {
    if (a->workspace == nullptr || a->workspace_bytes < dsa_indexer_workspace_bytes(a))
      return DSA_STATUS_WORKSPACE_TOO_SMALL;
    scores = static_cast<float*>(a->workspace);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dsa::launch_indexer_logits(static_cast<const __nv_bfloat16*>(a->q), static_cast<const __nv_bfloat16*>(a->k),
                                 a->weights, a->lengths, scores, a->status, (int)a->batch, (int)a->queries,
                                 (int)a->heads, (int)a->length, s) != cudaSuccess)
    return DSA_STATUS_LAUNCH_FAILED;
  if (dsa::launch_topk(scores, a->lengths, a->indices, a->batch * a->queries, (int)a->length, (int)a->topk, s) !=
      cudaSuccess)
    return DSA_STATUS_LAUNCH_FAILED;
  return DSA_STATUS_OK;
}

int dsa_set_wait_test(uint64_t limit_ns, int stall) {
  g_wait_limit_ns.store((unsigned long long)limit_ns, std::memory_order_relaxed);
  g_wait_test.store(stall != 0 ? 1 : 0, std::memory_order_relaxed);
  return DSA_STATUS_OK;
}

}  // extern "C"
