/*
 * dsa_b200.h — C ABI of the B200 (sm_100a) sparse-MLA attention forward.
 *
 * This is the drop-in boundary for the one hot path of CHNJZ/dsa: the BF16
 * sparse MLA forward with caller-given top-k indices,
 *
 *     forward(q, kv, q_rope, k_rope, indices) -> (output, softmax_max, softmax_sum)
 *
 * (reference: dsa/api.py:76-132). Shapes, dtypes and semantics are the
 * reference's (dsa/api.py:18-38, dsa/api.py:77-86):
 *
 *   q        BF16  [B, SQ, H, 512]   contiguous
 *   kv       BF16  [B, L, 1, 512]    contiguous (shared key and value)
 *   q_rope   BF16  [B, SQ, H, 64]    contiguous
 *   k_rope   BF16  [B, L, 1, 64]     contiguous
 *   indices  INT32 [B, SQ, 1, TOPK]  contiguous; entries outside [0, L) are
 *                                    masked (their address is clamped), and
 *                                    duplicates keep their repeated weight
 *   output       BF16 [B, SQ, H, 512]
 *   softmax_max  FP32 [B, 1, SQ, H]  max_j s_j, with s_j = (q.kv_j + qr.kr_j) * scale
 *                                    (scale 1/sqrt(576) = 1/24 unless the caller sets one)
 *   softmax_sum  FP32 [B, 1, SQ, H]  sum_j exp(s_j - max)
 *
 * A (token, head) row whose indices are all outside [0, L) gets output 0,
 * softmax_max -inf and softmax_sum 0 (the reference requires at least one
 * valid index per query and leaves this case undefined, dsa/api.py:77-86).
 *
 * Every pointer is a device pointer on the current device. No function
 * allocates device memory: temporaries (split-KV partials) live in a
 * caller-provided workspace whose size dsa_fwd_workspace_bytes() reports.
 * Launches are asynchronous on the given stream (a cudaStream_t passed as
 * void*, NULL = legacy default stream); nothing synchronises the host.
 *
 * No torch types cross this boundary; the Python package binds it with
 * ctypes (dsa_b200/_native.py).
 */
#ifndef DSA_B200_H_
#define DSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSA_B200_ABI_VERSION 2

#if defined(__GNUC__)
#define DSA_B200_API __attribute__((visibility("default")))
#else
#define DSA_B200_API
#endif

/* Status codes. The Python wrapper maps BAD_ARGUMENT/UNSUPPORTED to
 * ValueError and the rest to RuntimeError, as the reference raises
 * ValueError for shape/config problems (dsa/api.py:22-37, 92). */
typedef enum dsa_status {
  DSA_STATUS_OK = 0,
  DSA_STATUS_BAD_ARGUMENT = 1,      /* null pointer, non-positive size, misaligned buffer */
  DSA_STATUS_UNSUPPORTED = 2,       /* launch entry not valid for this shape */
  DSA_STATUS_WORKSPACE_TOO_SMALL = 3,
  DSA_STATUS_LAUNCH_FAILED = 4,     /* cudaGetLastError() after a launch */
  DSA_STATUS_DEVICE_TIMEOUT = 5,    /* a bounded device-side wait gave up (status word) */
  DSA_STATUS_CUDA_ERROR = 6         /* other CUDA runtime error */
} dsa_status_t;

/* Kernel families of the sm_100a launch table (replaces the reference's
 * workspace/ragged kernel choice, dsa/api.py:115-123). */
typedef enum dsa_family {
  DSA_FAMILY_AUTO = 0,      /* pick by shape (dsa_default_launch) */
  DSA_FAMILY_WARP_MMA = 1,  /* generic: 16 heads per CTA, warp-level MMA, any H % 16 == 0 */
  DSA_FAMILY_UMMA = 2,      /* tcgen05/TMEM path, H == 128: one CTA per (query, half of the 512
                               value columns); each CTA computes the full scores */
  DSA_FAMILY_UMMA_PAIR = 3, /* tcgen05/TMEM path, H == 128: a 2-CTA cluster per query, one CTA
                               computes scores + softmax, the other P.V over all 512 columns */
  DSA_FAMILY_STREAM = 4,    /* persistent warp-level MMA, 16 heads per CTA item, gather warps keep
                               the selected rows in flight; any H % 16 == 0, keys_per_tile 32 */
  DSA_FAMILY_KEYS = 5,      /* persistent tcgen05/TMEM path for 16 heads per CTA item with the
                               selected keys as the MMA's M dimension (scores and P.V computed
                               transposed); any H % 16 == 0, keys_per_tile 64 */
  DSA_FAMILY_PAIR_UNION = 6 /* the pair family over blocks of 128 / H queries of one batch row
                               (H = 16, 32 or 64; SQ a multiple of 128 / H), each block walking
                               the union of its queries' selected keys with one membership mask
                               per query; heads_per_cta 128, keys_per_tile 32, split 1 */
} dsa_family_t;

/* One entry of the shape-keyed launch table (reference: Tuning,
 * dsa/config.py:10-19, and its constraints dsa/api.py:41-60). */
typedef struct dsa_launch {
  int32_t family;          /* dsa_family_t */
  int32_t heads_per_cta;   /* BM: heads sharing one gathered tile in one CTA */
  int32_t keys_per_tile;   /* BN: gathered kv rows per pipeline stage */
  int32_t split;           /* KV splits per (query, head tile); >1 writes FP32
                              partials into the workspace, then merges */
} dsa_launch_t;

/* Arguments of one forward call (reference: forward's tensors and the
 * kernel arguments of dsa/api.py:115-128). */
typedef struct dsa_fwd_args {
  const void* q;            /* BF16 [B,SQ,H,512] */
  const void* kv;           /* BF16 [B,L,1,512] */
  const void* q_rope;       /* BF16 [B,SQ,H,64] */
  const void* k_rope;       /* BF16 [B,L,1,64] */
  const int32_t* indices;   /* INT32 [B,SQ,1,TOPK] */
  void* output;             /* BF16 [B,SQ,H,512] */
  float* softmax_max;       /* FP32 [B,1,SQ,H] */
  float* softmax_sum;       /* FP32 [B,1,SQ,H] */
  int64_t batch, queries, heads, length, topk;
  dsa_launch_t launch;      /* family AUTO => dsa_default_launch() */
  void* workspace;          /* split-KV partials; may be NULL when the size is 0 */
  uint64_t workspace_bytes;
  int32_t* status;          /* optional device word; kernels only OR error bits
                               into it (never clear it). NULL disables reporting. */
  float scale;              /* softmax scale on q.kv + qr.kr, in (0, 0.5]; 0 selects the
                               reference's fixed 1/24 (README.md:81-84). The scale_value
                               of the vendor operator's interface. */
} dsa_fwd_args_t;

/* ABI version (DSA_B200_ABI_VERSION of the built library). No reference
 * counterpart (the reference is JIT-compiled Python). */
DSA_B200_API int dsa_abi_version(void);

/* Human-readable name of a dsa_status_t. */
DSA_B200_API const char* dsa_status_string(int status);

/* Shape-keyed default launch entry (replaces the import-time validated
 * table _DEFAULT_CONFIGS, dsa/api.py:63-73, and config.select,
 * dsa/config.py:64-69). Depends only on the shape and the SM count of the
 * current device, never on input values. Returns DSA_STATUS_OK. */
DSA_B200_API int dsa_default_launch(int64_t batch, int64_t queries, int64_t heads, int64_t length,
                       int64_t topk, dsa_launch_t* out);

/* Check a launch entry against a shape (replaces _check_tuning,
 * dsa/api.py:41-60). Returns OK or UNSUPPORTED. */
DSA_B200_API int dsa_check_launch(int64_t batch, int64_t queries, int64_t heads, int64_t length,
                     int64_t topk, const dsa_launch_t* launch);

/* Workspace bytes the call needs (replaces the per-call torch.empty of the
 * GM workspace and the split partials, dsa/api.py:102-113). Returns 0 for
 * split == 1 and for an invalid entry. */
DSA_B200_API uint64_t dsa_fwd_workspace_bytes(const dsa_fwd_args_t* args);

/* The forward: main kernel and, when split > 1, the FP32 merge, both
 * enqueued on `stream` (reference: forward, dsa/api.py:76-132).
 * Returns a dsa_status_t. */
DSA_B200_API int dsa_sparse_mla_fwd(const dsa_fwd_args_t* args, void* stream);

/* Standalone FP32 split-KV merge (reference: merge_partials,
 * dsa/merge.py:13-91): numerator FP32 [T,S,H,512] (unnormalised),
 * partial_max/partial_sum FP32 [T,S,H] -> output BF16 [T,H,512],
 * softmax_max/softmax_sum FP32 [T,H]. T = B*SQ tokens, S = splits. */
DSA_B200_API int dsa_merge_partials(const float* numerator, const float* partial_max,
                       const float* partial_sum, void* output, float* softmax_max,
                       float* softmax_sum, int64_t tokens, int64_t heads, int64_t split,
                       void* stream);

/* Paged KV cache of a forward call (no counterpart in the reference, which
 * reads a dense kv per batch row and lists paged caches as out of scope,
 * README.md:19-20). args->kv / args->k_rope then point at page pools
 * [num_blocks, block_size, 1, 512] / [num_blocks, block_size, 1, 64] BF16;
 * block_table[b * max_blocks + j] is the pool block holding tokens
 * [j * block_size, (j + 1) * block_size) of batch row b; args->indices are
 * logical token positions of each batch row. An index is masked when it is
 * negative, at or past seq_lens[b] (or max_blocks * block_size when
 * seq_lens is NULL), or when its block table entry is outside
 * [0, num_blocks). args->length is ignored. */
typedef struct dsa_paged_kv {
  const int32_t* block_table;  /* INT32 [B, max_blocks] */
  const int32_t* seq_lens;     /* INT32 [B], or NULL */
  int64_t max_blocks;
  int64_t block_size;
  int64_t num_blocks;
} dsa_paged_kv_t;

/* Workspace bytes of dsa_sparse_mla_fwd_paged: the translated row indices
 * plus the forward's own workspace. 0 for invalid arguments. */
DSA_B200_API uint64_t dsa_fwd_paged_workspace_bytes(const dsa_fwd_args_t* args, const dsa_paged_kv_t* paged);

/* Forward over a paged KV cache: one kernel maps every logical index to its
 * pool row, then the forward runs over the pool as one batch row of
 * num_blocks * block_size rows (same kernels, same arithmetic as the dense
 * call on the same logical data). Returns a dsa_status_t. */
DSA_B200_API int dsa_sparse_mla_fwd_paged(const dsa_fwd_args_t* args, const dsa_paged_kv_t* paged, void* stream);

/* Bytes per token of the FP8 KV cache of dsa_sparse_mla_fwd_fp8:
 * 512 float8 e4m3 latent values, 4 FP32 scales (one per 128 latent dims),
 * 64 BF16 rope dims (DeepSeek-V3.2's FP8 MLA cache layout). */
#define DSA_FP8_ROW_BYTES 656

/* Workspace bytes of dsa_sparse_mla_fwd_fp8 (the dequantised selected rows
 * of every query plus the forward's own workspace); 0 for invalid arguments. */
DSA_B200_API uint64_t dsa_fwd_fp8_workspace_bytes(const dsa_fwd_args_t* args);

/* Forward over an FP8 KV cache (no counterpart in the reference, whose kv
 * is BF16 and which lists quantised caches as out of scope,
 * DSA从原理到实现.md:626). args->kv points at the cache, uint8
 * [B, L, 1, DSA_FP8_ROW_BYTES]; args->k_rope is ignored. One kernel
 * gathers each query's selected rows and dequantises them
 * (latent = bf16(e4m3 * scale)) into the workspace; the BF16 forward then
 * runs on them as B*SQ batch rows of TOPK keys. Returns a dsa_status_t. */
DSA_B200_API int dsa_sparse_mla_fwd_fp8(const dsa_fwd_args_t* args, void* stream);

/* Lightning indexer + top-k: the stage that produces the indices of the
 * forward (no counterpart in the reference, which takes the indices as
 * given and leaves the indexer and top-k out, README.md:19-20). For every
 * query t of batch row b and key j < L:
 *   score[t][j] = sum_h weights[t][h] * relu(q[t][h] . k[b][j])
 * (FP32, tcgen05 BF16 products), and indices[t] = the TOPK keys
 * j < lengths[t] (or L) with the largest scores, ties to the smaller key,
 * in ascending key order, padded with -1 when fewer keys are valid. */
typedef struct dsa_indexer_args {
  const void* q;            /* BF16 [B, SQ, HI, 128], HI in {16, 32, 64, 128} */
  const void* k;            /* BF16 [B, L, 128] */
  const float* weights;     /* FP32 [B, SQ, HI] */
  const int32_t* lengths;   /* INT32 [B, SQ] valid keys per query, or NULL (all L) */
  int32_t* indices;         /* INT32 [B, SQ, 1, TOPK] (output) */
  float* scores;            /* FP32 [B, SQ, L] (output), or NULL: kept in the workspace */
  int64_t batch, queries, heads, length, topk;
  void* workspace;          /* scores when `scores` is NULL */
  uint64_t workspace_bytes;
  int32_t* status;          /* optional device word (bounded-wait timeouts) */
} dsa_indexer_args_t;

/* Workspace bytes of dsa_indexer_topk (B*SQ*L FP32 scores when the caller
 * does not take them; 0 otherwise or for invalid arguments). */
DSA_B200_API uint64_t dsa_indexer_workspace_bytes(const dsa_indexer_args_t* args);

/* Indexer scores then top-k, two kernels on `stream`. Returns a dsa_status_t. */
DSA_B200_API int dsa_indexer_topk(const dsa_indexer_args_t* args, void* stream);

/* Number of kernels the last successful dsa_sparse_mla_fwd on this host
 * thread enqueued (1 or 2), for launch accounting. Calls of
 * dsa_sparse_mla_fwd_noalloc do not update it. */
DSA_B200_API int dsa_last_launch_count(void);

/* Test hook of the device-side failure path (no counterpart in the
 * reference, which bounds a hung run with a host-side watchdog,
 * tools/review.py:298-299). Applies to later launches of the split-V family
 * (DSA_FAMILY_UMMA) from this process; every other family keeps its fixed
 * 2 s bound. limit_ns bounds each device-side wait (0 restores the built-in
 * 2 s). stall != 0 makes the first CTA of each launch wait on a barrier that
 * nothing arrives at: that wait runs out, the CTA ORs the timeout bit (1)
 * into the status word, waits for the tensor-core work it already issued,
 * releases its tensor memory and leaves, and the launch completes (the
 * outputs of that CTA's items are then undefined). Returns DSA_STATUS_OK. */
DSA_B200_API int dsa_set_wait_test(uint64_t limit_ns, int stall);

/* Size of the library's built-in scratch array used by
 * dsa_sparse_mla_fwd_noalloc (32 MiB, held on every GPU that loads the
 * library until the process exits). */
#define DSA_NOALLOC_SCRATCH_BYTES (32u << 20)

/* Forward that allocates nothing and takes no workspace: the same warp-MMA
 * split-KV kernels and FP32 merge as dsa_sparse_mla_fwd, with the split
 * partials kept in the library's own DSA_NOALLOC_SCRATCH_BYTES array.
 * It has no counterpart in the reference. It is for callers that cannot
 * call cudaMalloc on this path: engines whose memory pool already holds
 * the HBM, code that must not pay cudaFree's device-wide synchronisation,
 * and FFI hosts that own only the input and output buffers. args->workspace
 * is ignored; launch family must be AUTO or WARP_MMA. Returns
 * DSA_STATUS_WORKSPACE_TOO_SMALL when the partials (tokens * split * heads
 * * 2056 bytes, 256-byte aligned per region) exceed the array. The first
 * call on a device resolves the array's device address (make it before any
 * stream capture). All calls share the array: calls that overlap on the GPU
 * race with each other. */
DSA_B200_API int dsa_sparse_mla_fwd_noalloc(const dsa_fwd_args_t* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSA_B200_H_ */
