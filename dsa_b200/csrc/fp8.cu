// FP8 KV cache: gather and dequantise the selected rows.
//
// Format (DeepSeek-V3.2's FP8 MLA cache layout; the reference has no
// quantised cache, DSA从原理到实现.md:626): one 656-byte row per token,
//   bytes [0, 512)    512 float8 e4m3 values of the latent (kv) part,
//   bytes [512, 528)  4 FP32 scales, scale k for latent dims [128k, 128k + 128),
//   bytes [528, 656)  64 BF16 rope dims (not quantised).
// A latent value is bf16(float(e4m3) * scale) (round to nearest even); the
// forward then runs unchanged on BF16 rows. This kernel writes, per
// flattened query t and selected slot j, the dequantised row into a compact
// workspace row t * TOPK + j and the compact index j (or -1 when the
// selected index is outside [0, L); the row is then zero, so a masked key
// contributes exactly 0 to P.V).
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "dsa_common.cuh"

namespace dsa {
namespace {

constexpr int kFp8RowBytes = 656;

// One warp per (query, slot): lane l converts latent dims 16l..16l+15 and
// lanes 0..7 copy the 128 rope bytes.
__global__ void __launch_bounds__(256) fp8_gather_kernel(const uint8_t* __restrict__ cache,
                                                         const int32_t* __restrict__ ids, __nv_bfloat16* kv_out,
                                                         __nv_bfloat16* kr_out, int32_t* ids_out, long long rows,
                                                         int topk, int queries, int length) {
  const int lane = threadIdx.x & 31;
  const long long stride = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += stride) {
    const long long t = r / topk;
    const int j = (int)(r % topk);
    const int idx = __ldg(ids + r);
    const bool valid = idx >= 0 && idx < length;
    uint4 lat0 = make_uint4(0, 0, 0, 0), lat1 = make_uint4(0, 0, 0, 0), rope = make_uint4(0, 0, 0, 0);
    if (valid) {
      const uint8_t* row = cache + ((size_t)(t / queries) * length + idx) * kFp8RowBytes;
      const uint4 f8 = __ldg(reinterpret_cast<const uint4*>(row) + lane);  // 16 e4m3 values
      const float sc = __ldg(reinterpret_cast<const float*>(row + 512) + (lane >> 3));
      const uint32_t w[4] = {f8.x, f8.y, f8.z, f8.w};
      uint32_t o[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const __nv_fp8x2_storage_t pair = (__nv_fp8x2_storage_t)((w[k] >> (16 * h)) & 0xFFFFu);
          const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3);
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
          o[2 * k + h] = pack_bf16x2(f.x * sc, f.y * sc);
        }
      }
      lat0 = make_uint4(o[0], o[1], o[2], o[3]);
      lat1 = make_uint4(o[4], o[5], o[6], o[7]);
      if (lane < 8) rope = __ldg(reinterpret_cast<const uint4*>(row + 528) + lane);
    }
    uint4* dkv = reinterpret_cast<uint4*>(kv_out + (size_t)r * kDimLatent) + 2 * lane;
    dkv[0] = lat0;
    dkv[1] = lat1;
    if (lane < 8) reinterpret_cast<uint4*>(kr_out + (size_t)r * kDimRope)[lane] = rope;
    if (lane == 0) ids_out[r] = valid ? j : -1;
  }
}

}  // namespace

cudaError_t launch_fp8_gather(const uint8_t* cache, const int32_t* ids, __nv_bfloat16* kv_out, __nv_bfloat16* kr_out,
                              int32_t* ids_out, long long rows, int topk, int queries, int length,
                              cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  long long blocks = (rows + 7) / 8;
  if (blocks > 148 * 32) blocks = 148 * 32;
  fp8_gather_kernel<<<(int)blocks, 256, 0, stream>>>(cache, ids, kv_out, kr_out, ids_out, rows, topk, queries, length);
  return cudaGetLastError();
}

}  // namespace dsa
