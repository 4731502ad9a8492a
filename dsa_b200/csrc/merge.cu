// FP32 split-KV merge (reference: merge_partials, dsa/merge.py:13-91).
//
// For one (token, head): m = max_s m_s, w_s = exp(m_s - m),
// l = sum_s w_s l_s, o = sum_s w_s u_s / l -> BF16, stats (m, l). A row
// whose splits are all masked (every partial max -FLT_MAX, l == 0) gets
// output 0, max -inf, sum 0.
// Many splits: one block per (token, head): kMergeGroups groups of 128 threads, each
// thread owning 4 consecutive latent columns, so every partial row is read
// once with 16-byte loads. The split statistics are reduced across lanes;
// group g sums the numerators of splits 8g..8g+7, 8g+32.. (kMergeUnroll rows
// in flight per thread) and the groups are added through shared memory.
#include "dsa_common.cuh"

namespace dsa {
namespace {

constexpr int kMergeGroups = 4;                  // thread groups per (token, head), each over 1/4 of the splits
constexpr int kMergeThreads = 128 * kMergeGroups; // a group's thread owns 4 consecutive columns
constexpr int kMergeUnroll = 8;                  // partial rows in flight per thread

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(kMergeThreads) merge_kernel(
    const float* __restrict__ num, const float* __restrict__ pmax,
    const float* __restrict__ psum, __nv_bfloat16* __restrict__ out,
    float* __restrict__ omax, float* __restrict__ osum, int tokens, int heads, int split) {
  __shared__ float4 acc[kMergeGroups - 1][128];
  const long long th = blockIdx.x;
  const int t = (int)(th / heads), h = (int)(th % heads);
  const int lane = threadIdx.x & 31;
  const int grp = threadIdx.x >> 7;
  const int c = (threadIdx.x & 127) * 4;
  const size_t stat0 = (size_t)t * split * heads + h;  // + s*heads

  // split statistics: lanes take splits lane, lane+32, ... (every warp computes them)
  float m = -INFINITY;
  for (int s = lane; s < split; s += 32) m = fmaxf(m, __ldg(pmax + stat0 + (size_t)s * heads));
  m = warp_max(m);
  float l = 0.f;
  for (int s = lane; s < split; s += 32)
    l += expf(__ldg(pmax + stat0 + (size_t)s * heads) - m) * __ldg(psum + stat0 + (size_t)s * heads);
  l = warp_sum(l);

  // numerator over this group's splits, kMergeUnroll 16-byte loads in flight per thread
  float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = grp * kMergeUnroll; s0 < split; s0 += kMergeGroups * kMergeUnroll) {
    float4 v[kMergeUnroll];
    float w[kMergeUnroll];
#pragma unroll
    for (int j = 0; j < kMergeUnroll; ++j) {
      const int s = s0 + j;
      if (s < split) {
        v[j] = __ldg(reinterpret_cast<const float4*>(num + (stat0 + (size_t)s * heads) * kDimLatent + c));
        w[j] = __ldg(pmax + stat0 + (size_t)s * heads);
      } else {
        v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        w[j] = -INFINITY;
      }
    }
#pragma unroll
    for (int j = 0; j < kMergeUnroll; ++j) {
      const float ww = expf(w[j] - m);
      u.x += ww * v[j].x;
      u.y += ww * v[j].y;
      u.z += ww * v[j].z;
      u.w += ww * v[j].w;
    }
  }
  if (grp > 0) acc[grp - 1][threadIdx.x & 127] = u;
  __syncthreads();
  if (grp != 0) return;
#pragma unroll
  for (int g = 0; g < kMergeGroups - 1; ++g) {
    const float4 o = acc[g][threadIdx.x];
    u.x += o.x;
    u.y += o.y;
    u.z += o.z;
    u.w += o.w;
  }
  const float ld = l > 0.f ? l : INFINITY;  // no valid index in any split: output 0
  uint2 packed;
  packed.x = pack_bf16x2(__fdiv_rn(u.x, ld), __fdiv_rn(u.y, ld));
  packed.y = pack_bf16x2(__fdiv_rn(u.z, ld), __fdiv_rn(u.w, ld));
  *reinterpret_cast<uint2*>(out + (size_t)th * kDimLatent + c) = packed;
  if (threadIdx.x == 0) {
    omax[th] = l > 0.f ? m : -INFINITY;
    osum[th] = l;
  }
}

// Few splits (split <= kWarpMergeMaxSplit): one warp per (token, head). Lane
// s holds split s's statistics (the same lane order and shuffle tree as the
// block kernel above, so m and l are bit-identical); lane i owns columns
// 4i + 128j (j = 0..3), and kWarpMergeBatch splits' rows (4 x 16 B per lane
// each) are loaded before they are accumulated, in split order.
constexpr int kWarpMergeMaxSplit = 16;
constexpr int kWarpMergeWarps = 8;   // rows per block
constexpr int kWarpMergeBatch = 4;   // splits in flight per lane

__global__ void __launch_bounds__(32 * kWarpMergeWarps) merge_warp_kernel(
    const float* __restrict__ num, const float* __restrict__ pmax,
    const float* __restrict__ psum, __nv_bfloat16* __restrict__ out,
    float* __restrict__ omax, float* __restrict__ osum, int rows, int heads, int split) {
  const int lane = threadIdx.x & 31;
  const long long th = (long long)blockIdx.x * kWarpMergeWarps + (threadIdx.x >> 5);
  if (th >= rows) return;
  const int t = (int)(th / heads), h = (int)(th % heads);
  const size_t stat0 = (size_t)t * split * heads + h;  // + s*heads

  const float ms = lane < split ? __ldg(pmax + stat0 + (size_t)lane * heads) : -INFINITY;
  const float m = warp_max(ms);
  const float ws = lane < split ? expf(ms - m) : 0.f;
  const float l = warp_sum(lane < split ? ws * __ldg(psum + stat0 + (size_t)lane * heads) : 0.f);

  float4 u[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) u[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = 0; s0 < split; s0 += kWarpMergeBatch) {
    float4 v[kWarpMergeBatch][4];
#pragma unroll
    for (int b = 0; b < kWarpMergeBatch; ++b) {
      const int s = min(s0 + b, split - 1);
      const float4* row = reinterpret_cast<const float4*>(num + (stat0 + (size_t)s * heads) * kDimLatent) + lane;
#pragma unroll
      for (int j = 0; j < 4; ++j) v[b][j] = __ldg(row + 32 * j);
    }
#pragma unroll
    for (int b = 0; b < kWarpMergeBatch; ++b) {
      const float w = __shfl_sync(0xffffffffu, ws, (s0 + b) & 31);
      if (s0 + b < split) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          u[j].x += w * v[b][j].x;
          u[j].y += w * v[b][j].y;
          u[j].z += w * v[b][j].z;
          u[j].w += w * v[b][j].w;
        }
      }
    }
  }
  const float ld = l > 0.f ? l : INFINITY;  // no valid index in any split: output 0
  uint2* dst = reinterpret_cast<uint2*>(out + (size_t)th * kDimLatent) + lane;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint2 packed;
    packed.x = pack_bf16x2(__fdiv_rn(u[j].x, ld), __fdiv_rn(u[j].y, ld));
    packed.y = pack_bf16x2(__fdiv_rn(u[j].z, ld), __fdiv_rn(u[j].w, ld));
    dst[32 * j] = packed;
  }
  if (lane == 0) {
    omax[th] = l > 0.f ? m : -INFINITY;
    osum[th] = l;
  }
}

}  // namespace

cudaError_t launch_merge(const float* num, const float* pmax, const float* psum,
                         __nv_bfloat16* out, float* omax, float* osum, int tokens, int heads,
                         int split, cudaStream_t stream) {
  const long long blocks = (long long)tokens * heads;
  if (blocks <= 0 || blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  if (split <= kWarpMergeMaxSplit) {
    const long long wblocks = (blocks + kWarpMergeWarps - 1) / kWarpMergeWarps;
    merge_warp_kernel<<<(unsigned)wblocks, 32 * kWarpMergeWarps, 0, stream>>>(
        num, pmax, psum, out, omax, osum, (int)blocks, heads, split);
    return cudaGetLastError();
  }
  merge_kernel<<<(unsigned)blocks, kMergeThreads, 0, stream>>>(num, pmax, psum, out, omax, osum,
                                                              tokens, heads, split);
  return cudaGetLastError();
}

}  // namespace dsa
