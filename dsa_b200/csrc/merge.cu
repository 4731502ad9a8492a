// FP32 split-KV merge (reference: merge_partials, dsa/merge.py:13-91).
//
// For one (token, head): m = max_s m_s, w_s = exp(m_s - m),
// l = sum_s w_s l_s, o = sum_s w_s u_s / l -> BF16, stats (m, l).
// One 128-thread group per (token, head), each thread owning 4 consecutive
// latent columns, so every partial row is read once with 16-byte loads.
#include "dsa_common.cuh"

namespace dsa {
namespace {

constexpr int kMergeHeadsPerBlock = 2;
constexpr int kMergeThreads = 128 * kMergeHeadsPerBlock;

__global__ void __launch_bounds__(kMergeThreads) merge_kernel(
    const float* __restrict__ num, const float* __restrict__ pmax,
    const float* __restrict__ psum, __nv_bfloat16* __restrict__ out,
    float* __restrict__ omax, float* __restrict__ osum, int tokens, int heads, int split) {
  const long long th = (long long)blockIdx.x * kMergeHeadsPerBlock + (threadIdx.x >> 7);
  if (th >= (long long)tokens * heads) return;
  const int t = (int)(th / heads), h = (int)(th % heads);
  const int c = (threadIdx.x & 127) * 4;
  const size_t stat0 = (size_t)t * split * heads + h;  // + s*heads

  float m = -INFINITY;
  for (int s = 0; s < split; ++s) m = fmaxf(m, __ldg(pmax + stat0 + (size_t)s * heads));
  float l = 0.f;
  float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < split; ++s) {
    const float w = expf(__ldg(pmax + stat0 + (size_t)s * heads) - m);
    l += w * __ldg(psum + stat0 + (size_t)s * heads);
    const float4 v = __ldg(reinterpret_cast<const float4*>(
        num + (stat0 + (size_t)s * heads) * kDimLatent + c));
    u.x += w * v.x;
    u.y += w * v.y;
    u.z += w * v.z;
    u.w += w * v.w;
  }
  uint2 packed;
  packed.x = pack_bf16x2(__fdiv_rn(u.x, l), __fdiv_rn(u.y, l));
  packed.y = pack_bf16x2(__fdiv_rn(u.z, l), __fdiv_rn(u.w, l));
  *reinterpret_cast<uint2*>(out + (size_t)th * kDimLatent + c) = packed;
  if (c == 0) {
    omax[th] = m;
    osum[th] = l;
  }
}

}  // namespace

cudaError_t launch_merge(const float* num, const float* pmax, const float* psum,
                         __nv_bfloat16* out, float* omax, float* osum, int tokens, int heads,
                         int split, cudaStream_t stream) {
  const long long pairs = (long long)tokens * heads;
  const long long blocks = (pairs + kMergeHeadsPerBlock - 1) / kMergeHeadsPerBlock;
  if (blocks <= 0 || blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  merge_kernel<<<(unsigned)blocks, kMergeThreads, 0, stream>>>(num, pmax, psum, out, omax, osum,
                                                              tokens, heads, split);
  return cudaGetLastError();
}

}  // namespace dsa
