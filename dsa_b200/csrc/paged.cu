// Paged KV cache: logical top-k indices -> physical cache rows.
//
// A paged cache holds each sequence's tokens in fixed-size blocks of a
// shared page pool: kv_cache [num_blocks, block_size, 1, 512] and
// k_rope_cache [num_blocks, block_size, 1, 64], with block_table[b][j] the
// pool block that holds tokens [j * block_size, (j + 1) * block_size) of
// sequence b. The reference has no paged layout (its kv is dense per batch
// row and it lists paged caches as out of scope, README.md:19-20,
// DSA从原理到实现.md:625); this build maps a paged call onto the dense
// kernels: every logical index i of batch row b becomes the flat pool row
//   block_table[b][i / block_size] * block_size + i % block_size
// and the forward then runs as one batch row over the whole pool
// (kv = the pool viewed as [1, num_blocks * block_size, 1, 512]).
// An index is invalid (-1, masked like any index outside [0, L)) when it is
// negative, at or past the sequence length (seq_lens[b], or the table's
// max_blocks * block_size when no lengths are given), or when its block
// table entry is outside [0, num_blocks).
#include <cuda_runtime.h>

#include <cstdint>

#include "dsa_common.cuh"

namespace dsa {
namespace {

__global__ void __launch_bounds__(256) paged_rows_kernel(const int32_t* __restrict__ ids,
                                                         const int32_t* __restrict__ block_table,
                                                         const int32_t* __restrict__ seq_lens,
                                                         int32_t* __restrict__ rows, long long n, int per_batch,
                                                         int max_blocks, int block_size, int num_blocks) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int b = (int)(i / per_batch);
    const int idx = __ldg(ids + i);
    const long long limit = seq_lens != nullptr ? (long long)__ldg(seq_lens + b) : (long long)max_blocks * block_size;
    int row = -1;
    if (idx >= 0 && idx < limit) {
      const int j = idx / block_size;
      if (j < max_blocks) {
        const int blk = __ldg(block_table + (size_t)b * max_blocks + j);
        if (blk >= 0 && blk < num_blocks) row = blk * block_size + idx % block_size;
      }
    }
    rows[i] = row;
  }
}

}  // namespace

cudaError_t launch_paged_rows(const int32_t* ids, const int32_t* block_table, const int32_t* seq_lens, int32_t* rows,
                              long long n, int per_batch, int max_blocks, int block_size, int num_blocks,
                              cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  paged_rows_kernel<<<(int)blocks, 256, 0, stream>>>(ids, block_table, seq_lens, rows, n, per_batch, max_blocks,
                                                     block_size, num_blocks);
  return cudaGetLastError();
}

}  // namespace dsa
