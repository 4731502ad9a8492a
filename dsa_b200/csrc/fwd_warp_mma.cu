// Generic sparse-MLA forward: one CTA per (token, KV split, 16-head group).
//
// This is the shape-agnostic family of the launch table (any H % 16 == 0,
// any TOPK, any split). It follows the reference's per-job dataflow
// (dsa/workspace.py:25-390): gather the selected [kv(512) | k_rope(64)]
// rows, S = Q.K^T over 576 dims in FP32, masked online softmax in FP32
// (scale 1/24, invalid index -> -inf, dsa/workspace.py:252-269), P rounded
// to BF16, O += P.V over the 512-d latent in FP32, then either the
// normalised BF16 output and stats (split == 1) or FP32 partials (split > 1,
// dsa/workspace.py:356-385).
//
// B200 mapping: the gather is a 2-stage cp.async pipeline straight into
// padded (ldmatrix-conflict-free) shared memory rows — no global-memory
// workspace round trip as on the NPU (dsa/workspace.py:129-140). QK and PV
// use warp-level m16n8k16 BF16 MMAs: warp w owns keys [8w, 8w+8) of a tile
// for QK and latent columns [128w, 128w+128) for PV, so O stays in
// registers for the whole job.
#include "dsa_common.cuh"

namespace dsa {
namespace {

constexpr int kWmHeads = 16;
constexpr int kWmThreads = 128;
constexpr int kWmStages = 2;
constexpr int kWmRow = kDimQK + 8;  // padded smem row (elements): 1168 B, odd multiple of 16 B
constexpr int kChunksPerRow = kDimQK / 8;       // 72 x 16 B per gathered row
constexpr int kLatentChunks = kDimLatent / 8;   // 64

template <int BN>
struct WmSmem {
  static constexpr int kPRow = BN + 8;
  __nv_bfloat16 q[kWmHeads * kWmRow];
  __nv_bfloat16 k[kWmStages][BN * kWmRow];
  __nv_bfloat16 p[kWmHeads * kPRow];
  float s[kWmHeads * BN];
  int ids[kWmStages][BN];
  float m[kWmHeads];
  float l[kWmHeads];
  float alpha[kWmHeads];
};

template <int BN>
__global__ void __launch_bounds__(kWmThreads, 2) fwd_warp_mma_kernel(FwdParams p) {
  static_assert(BN % 32 == 0 && BN >= 32, "BN must be a multiple of 32");
  constexpr int kKeysPerWarp = BN / 4;          // QK keys per warp
  constexpr int kNT = kKeysPerWarp / 8;         // n8 tiles per warp in QK
  using Smem = WmSmem<BN>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int g = lane >> 2;   // mma group id (row within 8)
  const int tq = lane & 3;   // thread in group

  const int hgroups = p.heads / kWmHeads;
  long long bid = blockIdx.x;
  const int hg = (int)(bid % hgroups);
  bid /= hgroups;
  const int sp = (int)(bid % p.split);
  const int token = (int)(bid / p.split);
  const int batch = checked_index(token / p.queries, p.batch, p.status);
  const int h0 = hg * kWmHeads;

  int kbeg, kend;
  split_bounds(p.topk, BN, p.split, sp, &kbeg, &kend);
  const int ntiles = (kend - kbeg + BN - 1) / BN;

  const __nv_bfloat16* kv_b = p.kv + (size_t)batch * p.length * kDimLatent;
  const __nv_bfloat16* kr_b = p.k_rope + (size_t)batch * p.length * kDimRope;
  const int32_t* ids_t = p.ids + (size_t)token * p.topk;
  const int L = p.length;

  // Q tile [16 heads x (512 | 64)] -> smem (joins the first cp.async group).
  for (int c = tid; c < kWmHeads * kChunksPerRow; c += kWmThreads) {
    const int r = c / kChunksPerRow, part = c % kChunksPerRow;
    const size_t row = (size_t)token * p.heads + h0 + r;
    const __nv_bfloat16* src = part < kLatentChunks
                                   ? p.q + row * kDimLatent + part * 8
                                   : p.q_rope + row * kDimRope + (part - kLatentChunks) * 8;
    cp_async_16(smem_u32(&sm.q[r * kWmRow + part * 8]), src);
  }
  if (tid < kWmHeads) {
    sm.m[tid] = kNegFltMax;  // finite start, as dsa/workspace.py:68
    sm.l[tid] = 0.f;
  }

  // Gather one tile of BN selected rows. Addresses are clamped to [0, L-1];
  // validity is judged later from the original index (dsa/workspace.py:121-128,
  // 252-257). Keys past the split end gather row 0 and are masked.
  auto issue_tile = [&](int t, int stage) {
    const int k0 = kbeg + t * BN;
    for (int c = tid; c < BN * kChunksPerRow; c += kWmThreads) {
      const int key = c / kChunksPerRow, part = c % kChunksPerRow;
      const int j = k0 + key;
      const int idx = (j < kend) ? __ldg(ids_t + j) : 0;
      const int safe = checked_index(min(max(idx, 0), L - 1), L, p.status);
      const __nv_bfloat16* src = part < kLatentChunks
                                     ? kv_b + (size_t)safe * kDimLatent + part * 8
                                     : kr_b + (size_t)safe * kDimRope + (part - kLatentChunks) * 8;
      cp_async_16(checked_smem(smem_u32(&sm.k[stage][key * kWmRow + part * 8]), 16u, smem_u32(sm.k[stage]),
                               (uint32_t)(BN * kWmRow * 2), p.status),
                  src);
    }
    if (tid < BN) {
      const int j = k0 + tid;
      sm.ids[stage][tid] = (j < kend) ? __ldg(ids_t + j) : -1;
    }
  };

  float acc[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

  if (ntiles > 0) issue_tile(0, 0);
  cp_async_commit();

  const float inv_scale_div = p.scale_div;  // scores / scale_div (24 for the reference's scale)
  for (int t = 0; t < ntiles; ++t) {
    const int stage = t & 1;
    if (t + 1 < ntiles) issue_tile(t + 1, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    // ---- S = Q.K^T for this warp's keys ----------------------------------
    {
      const uint32_t qbase = smem_u32(sm.q) +
                             (((lane & 7) + ((lane >> 3) & 1) * 8) * kWmRow + (lane >> 4) * 8) * 2;
#pragma unroll
      for (int nt = 0; nt < kNT; ++nt) {
        const int key0 = warp * kKeysPerWarp + nt * 8;
        const uint32_t kbase =
            smem_u32(sm.k[stage]) + ((key0 + (lane & 7)) * kWmRow + (lane >> 3) * 8) * 2;
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 6
        for (int kp = 0; kp < kDimQK / 32; ++kp) {
          uint32_t a0, a1, a2, a3, a4, a5, a6, a7, b0, b1, b2, b3;
          ldmatrix_x4(qbase + kp * 64, a0, a1, a2, a3);
          ldmatrix_x4(qbase + kp * 64 + 32, a4, a5, a6, a7);
          ldmatrix_x4(kbase + kp * 64, b0, b1, b2, b3);
          mma_bf16_16816(d0, a0, a1, a2, a3, b0, b1);
          mma_bf16_16816(d1, a4, a5, a6, a7, b2, b3);
        }
        const int col = key0 + tq * 2;
        const int i0 = sm.ids[stage][col], i1 = sm.ids[stage][col + 1];
        const bool v0 = (i0 >= 0) & (i0 < L), v1 = (i1 >= 0) & (i1 < L);
        const float ninf = -INFINITY;
        sm.s[g * BN + col] = v0 ? __fdiv_rn(d0[0] + d1[0], inv_scale_div) : ninf;
        sm.s[g * BN + col + 1] = v1 ? __fdiv_rn(d0[1] + d1[1], inv_scale_div) : ninf;
        sm.s[(g + 8) * BN + col] = v0 ? __fdiv_rn(d0[2] + d1[2], inv_scale_div) : ninf;
        sm.s[(g + 8) * BN + col + 1] = v1 ? __fdiv_rn(d0[3] + d1[3], inv_scale_div) : ninf;
      }
    }
    __syncthreads();

    // ---- online softmax: 8 threads per head row ------------------------------
    {
      constexpr int kCols = BN / 8;  // columns per thread
      const int r = tid >> 3;
      const int c0 = (tid & 7) * kCols;
      const float m_old = sm.m[r];
      const float l_old = sm.l[r];
      __syncwarp();
      float x[kCols];
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < kCols; ++i) {
        x[i] = sm.s[r * BN + c0 + i];
        mx = fmaxf(mx, x[i]);
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      const float m_new = fmaxf(m_old, mx);
      const float alpha = expf(m_old - m_new);
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < kCols; i += 2) {
        const float p0 = expf(x[i] - m_new);
        const float p1 = expf(x[i + 1] - m_new);
        sum += p0 + p1;
        *reinterpret_cast<uint32_t*>(&sm.p[r * Smem::kPRow + c0 + i]) = pack_bf16x2(p0, p1);
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      if ((tid & 7) == 0) {
        sm.m[r] = m_new;
        sm.l[r] = alpha * l_old + sum;
        sm.alpha[r] = alpha;
      }
    }
    __syncthreads();

    // ---- O = alpha*O + P.V over this warp's 128 latent columns --------------
    {
      const float al0 = sm.alpha[g], al1 = sm.alpha[g + 8];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        acc[j][0] *= al0;
        acc[j][1] *= al0;
        acc[j][2] *= al1;
        acc[j][3] *= al1;
      }
      const uint32_t pbase =
          smem_u32(sm.p) +
          (((lane & 7) + ((lane >> 3) & 1) * 8) * Smem::kPRow + (lane >> 4) * 8) * 2;
      const uint32_t vbase =
          smem_u32(sm.k[stage]) +
          (((lane & 7) + ((lane >> 3) & 1) * 8) * kWmRow + warp * 128 + (lane >> 4) * 8) * 2;
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(pbase + kk * 32, a0, a1, a2, a3);
#pragma unroll
        for (int jp = 0; jp < 8; ++jp) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(vbase + (kk * 16 * kWmRow + jp * 16) * 2, b0, b1, b2, b3);
          mma_bf16_16816(acc[2 * jp], a0, a1, a2, a3, b0, b1);
          mma_bf16_16816(acc[2 * jp + 1], a0, a1, a2, a3, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- epilogue --------------------------------------------------------------
  const float l0 = sm.l[g], l1 = sm.l[g + 8];
  if (p.split == 1) {
    // a row without a valid index (l == 0, O == 0) is written as 0 (O / inf)
    const float d0 = l0 > 0.f ? l0 : INFINITY, d1 = l1 > 0.f ? l1 : INFINITY;
    __nv_bfloat16* o0 = p.out + ((size_t)token * p.heads + h0 + g) * kDimLatent + warp * 128 + tq * 2;
    __nv_bfloat16* o1 = o0 + 8 * kDimLatent;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      *reinterpret_cast<uint32_t*>(o0 + j * 8) =
          pack_bf16x2(__fdiv_rn(acc[j][0], d0), __fdiv_rn(acc[j][1], d0));
      *reinterpret_cast<uint32_t*>(o1 + j * 8) =
          pack_bf16x2(__fdiv_rn(acc[j][2], d1), __fdiv_rn(acc[j][3], d1));
    }
    if (tid < kWmHeads) {
      p.out_max[(size_t)token * p.heads + h0 + tid] = sm.l[tid] > 0.f ? sm.m[tid] : -INFINITY;
      p.out_sum[(size_t)token * p.heads + h0 + tid] = sm.l[tid];
    }
  } else {
    const size_t prow = ((size_t)token * p.split + sp) * p.heads + h0;
    float* n0 = p.part_num + (prow + g) * kDimLatent + warp * 128 + tq * 2;
    float* n1 = n0 + 8 * kDimLatent;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      *reinterpret_cast<float2*>(n0 + j * 8) = make_float2(acc[j][0], acc[j][1]);
      *reinterpret_cast<float2*>(n1 + j * 8) = make_float2(acc[j][2], acc[j][3]);
    }
    if (tid < kWmHeads) {
      p.part_max[prow + tid] = sm.m[tid];
      p.part_sum[prow + tid] = sm.l[tid];
    }
  }
}

template <int BN>
cudaError_t launch_bn(const FwdParams& p, cudaStream_t stream) {
  const size_t smem = sizeof(WmSmem<BN>);
  cudaError_t e = cudaFuncSetAttribute(fwd_warp_mma_kernel<BN>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long blocks = (long long)p.tokens * p.split * (p.heads / kWmHeads);
  if (blocks <= 0 || blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  fwd_warp_mma_kernel<BN><<<(unsigned)blocks, kWmThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fwd_warp_mma(const FwdParams& p, cudaStream_t stream) {
  switch (p.keys_per_tile) {
    case 32: return launch_bn<32>(p, stream);
    case 64: return launch_bn<64>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace dsa
