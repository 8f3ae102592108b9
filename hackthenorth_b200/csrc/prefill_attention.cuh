// prefill_attention.cuh — the row-wise helpers of the prefill layer chain
// (RMSNorm of the prompt rows with the layer-0 embedding gather, and the
// position helpers); the prefill attention itself is flash_prefill_tc_kernel
// in prefill_attention_tc.cuh.
#pragma once
#include "attention.cuh"

namespace qb {

// Embedding gather (optional) + RMSNorm of T rows, one CTA of 128 threads per
// row: xn[r] = bf16(bf16(x * inv) * gain) (dryft/engine/kernels/rmsnorm.py:70-81);
// with ids, x = embed[ids[r]] is also stored to x_out[r] (the residual stream).
struct NormRowsArgs {
  const bf16* x;          // [T][K] or NULL (gather)
  const bf16* embed;
  const int64_t* ids;
  int vocab;
  bf16* x_out;            // gather: [T][K]
  const bf16* gain;
  bf16* xn;               // [T][K]
  int K;
  float eps;
  int* err;
};

__global__ void __launch_bounds__(128) norm_rows_kernel(const NormRowsArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ float part[4];
  const int r = blockIdx.x;
  const bf16* src = a.x ? a.x + (size_t)r * a.K : nullptr;
  if (!src) {
    long long t = a.ids[r];
    if (t < 0 || t >= a.vocab) {
      if (threadIdx.x == 0) report_error(a.err, DEV_BAD_TOKEN);
      t = 0;
    }
    src = a.embed + (size_t)t * a.K;
  }
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < a.K; i += 128 * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + i);
    if (!a.x) *reinterpret_cast<uint4*>(a.x_out + (size_t)r * a.K + i) = v;
    ss = dot8(v, v, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float tot = part[0] + part[1] + part[2] + part[3];
  const float inv = 1.0f / sqrtf(tot / (float)a.K + a.eps);
  for (int i = threadIdx.x * 8; i < a.K; i += 128 * 8) {
    uint4 v = *reinterpret_cast<const uint4*>(src + i);
    const uint4 g = ldg128_nc(a.gain + i);
    uint32_t* pv = reinterpret_cast<uint32_t*>(&v);
    const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float n0 = round_bf16(bf_lo(pv[j]) * inv) * bf_lo(pg[j]);
      const float n1 = round_bf16(bf_hi(pv[j]) * inv) * bf_hi(pg[j]);
      pv[j] = pack_bf16(n0, n1);
    }
    *reinterpret_cast<uint4*>(a.xn + (size_t)r * a.K + i) = v;
  }
}

__global__ void set_i64_kernel(int64_t* p, long long v) {
  pdl_wait();
  pdl_trigger();
  *p = v;
}

}  // namespace qb
