// gemv.cuh — batch-one weight-streaming GEMV for sm_100a with fused prologue
// (embedding gather, RMSNorm) and epilogues (store, +residual, SwiGLU pair,
// bf16 logits + greedy argmax).
//
// Design (HBM-bound: every weight byte is read exactly once per decode step):
//  * grid = one CTA per SM; CTA b owns the contiguous row range
//    [b*U/G, (b+1)*U/G) of the row-major weight (U = output units), which
//    balances the work to within one row.
//  * rows are taken 8 at a time (one per consumer warp) and K in pieces of
//    1024 columns: a 16 KB stage holds the same 1024-column piece of 8 rows,
//    brought in by 8 one-dimensional bulk copies (cp.async.bulk + mbarrier
//    complete_tx, 2 KB each, evict-first in L2) issued by one producer lane
//    into a ring of 3-8 stages;
//  * consumer warp w owns row w of every 8-row block for the whole K, so it
//    accumulates in registers (fp32) across stages and reduces across its
//    lanes (5 shuffles) once per row; x sits in shared memory as fp32 after
//    the prologue. Each row's sum has one fixed order, so results are
//    deterministic;
//  * PDL: the producer fills the ring before griddepcontrol.wait (weights are
//    immutable), so a GEMV streams its first stages while the previous kernel
//    finishes.
#pragma once
#include "common.cuh"

namespace qb {

constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvThreads = (kGemvConsumerWarps + 1) * 32;
constexpr int kGemvKChunk = 1024;                                   // columns per row piece
constexpr int kGemvPieceBytes = kGemvKChunk * 2;                    // 2 KB
constexpr int kGemvStageBytes = kGemvConsumerWarps * kGemvPieceBytes;  // 16 KB
constexpr int kGemvBarrierId = 1;  // named barrier of the 256 consumer threads

enum GemvEpilogue : int { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

struct GemvArgs {
  const bf16* w;        // [rows][K]
  int K;                // multiple of 256
  int rows;             // weight rows (2F for SwiGLU)
  const bf16* x;        // [K] input row, or NULL with embed
  const bf16* embed;    // [vocab][K] embedding table (layer-0 gather) or NULL
  const int64_t* token; // device token id for the gather
  int vocab;            // rows of embed (bounds check)
  bf16* x_copy;         // gather: CTA 0 stores the gathered row here (residual stream)
  const bf16* gain;     // [K] RMSNorm gain, or NULL (no norm)
  float eps;
  const bf16* residual; // EPI_RESIDUAL
  bf16* out;            // EPI_STORE/RESIDUAL: [rows]; SWIGLU: [rows/2]
  bf16* logits;         // EPI_ARGMAX: optional [rows]
  float* part_val;      // EPI_ARGMAX: [gridDim] partial maxima
  int* part_idx;        // EPI_ARGMAX: [gridDim] partial argmax
  unsigned* counter;    // EPI_ARGMAX: arrival counter (restored to 0)
  int64_t* token_out;   // EPI_ARGMAX: greedy token
  int64_t* pos_inc;     // optional: *pos_inc += 1 once the result is written
  int* err;             // device error word
  int stages;           // ring stages
  int max_rows;         // max rows any CTA owns (size of rowsum)
};

__host__ __device__ inline int gemv_rows_per_unit(int epi) { return epi == EPI_SWIGLU ? 2 : 1; }

__host__ inline size_t gemv_smem_bytes(int K, int stages, int max_rows) {
  return (size_t)stages * kGemvStageBytes + (size_t)K * 4 + (((size_t)max_rows * 4 + 15) & ~size_t(15)) +
         (size_t)2 * stages * 8 + 64 * 4;
}

__device__ __forceinline__ float dot8_f32x(const uint4 w, const float* x, float acc) {
  const float4 x0 = *reinterpret_cast<const float4*>(x);
  const float4 x1 = *reinterpret_cast<const float4*>(x + 4);
  acc = fmaf(bf_lo(w.x), x0.x, acc);
  acc = fmaf(bf_hi(w.x), x0.y, acc);
  acc = fmaf(bf_lo(w.y), x0.z, acc);
  acc = fmaf(bf_hi(w.y), x0.w, acc);
  acc = fmaf(bf_lo(w.z), x1.x, acc);
  acc = fmaf(bf_hi(w.z), x1.y, acc);
  acc = fmaf(bf_lo(w.w), x1.z, acc);
  acc = fmaf(bf_hi(w.w), x1.w, acc);
  return acc;
}

template <int EPI>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = gridDim.x;
  const int b = blockIdx.x;
  const int K = a.K;
  const int stages = a.stages;

  constexpr int rpu = (EPI == EPI_SWIGLU) ? 2 : 1;
  const int units = a.rows / rpu;
  const int u0 = (int)(((long long)units * b) / G);
  const int u1 = (int)(((long long)units * (b + 1)) / G);
  const int r0 = u0 * rpu;
  const int nrows = (u1 - u0) * rpu;
  const int nkc = (K + kGemvKChunk - 1) / kGemvKChunk;
  const int nblk = (nrows + kGemvConsumerWarps - 1) / kGemvConsumerWarps;
  const int nstage = nblk * nkc;

  uint8_t* ring = smem;
  float* xs = reinterpret_cast<float*>(smem + (size_t)stages * kGemvStageBytes);
  float* rowsum = xs + K;
  uint64_t* full = reinterpret_cast<uint64_t*>(rowsum + ((a.max_rows + 3) & ~3));
  uint64_t* empty = full + stages;
  float* misc = reinterpret_cast<float*>(empty + stages);

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGemvConsumerWarps);
    }
    fence_mbar_init();
    reinterpret_cast<int*>(misc)[60] = 0;  // CTA-wide abort flag
  }
  __syncthreads();

  if (warp == kGemvConsumerWarps) {
    // ---------------- producer warp ----------------
    if (lane == 0) {
      const uint64_t policy = policy_evict_first();
      int issued = 0;
      bool ok = true;
      bool waited = false;
      for (int c = 0; c < nstage; ++c) {
        const int s = c % stages;
        if (c >= stages) {
          if (!waited) {
            pdl_wait();
            pdl_trigger();
            waited = true;
          }
          if (!mbar_wait(&empty[s], ((c / stages) - 1) & 1, a.err, DEV_TIMEOUT_GEMV_EMPTY)) {
            ok = false;
            break;
          }
        }
        const int blk = c / nkc, kc = c - blk * nkc;
        const int nr = min(kGemvConsumerWarps, nrows - blk * kGemvConsumerWarps);
        const int c0 = kc * kGemvKChunk;
        const uint32_t piece = (uint32_t)min(kGemvKChunk, K - c0) * 2;
        mbar_arrive_expect_tx(&full[s], piece * nr);
        const bf16* src = a.w + (size_t)(r0 + blk * kGemvConsumerWarps) * K + c0;
        uint8_t* dst = ring + (size_t)s * kGemvStageBytes;
        for (int r = 0; r < nr; ++r)
          bulk_g2s(dst + r * kGemvPieceBytes, src + (size_t)r * K, piece, &full[s], policy);
        issued = c + 1;
      }
      if (!waited) {
        pdl_wait();
        pdl_trigger();
      }
      if (!ok) {
        // Keep shared memory alive until the copies already in flight land.
        for (int c = (issued > stages ? issued - stages : 0); c < issued; ++c)
          mbar_wait(&full[c % stages], (c / stages) & 1, nullptr, 0);
      }
    } else {
      pdl_wait();
      pdl_trigger();
    }
    return;
  }

  // ---------------- consumer warps (256 threads) ----------------
  const int ctid = tid;  // 0..255
  pdl_wait();
  pdl_trigger();

  // 1. Input row (optionally the embedding gather) and its RMSNorm, to fp32 smem.
  const bf16* xsrc = a.x;
  if (a.embed != nullptr) {
    long long t = *a.token;
    if (t < 0 || t >= a.vocab) {
      if (ctid == 0 && b == 0) report_error(a.err, DEV_BAD_TOKEN);
      t = 0;
    }
    xsrc = a.embed + (size_t)t * K;
  }
  float ss = 0.f;
  for (int i = ctid * 8; i < K; i += 256 * 8) {
    const uint4 v = ldg128_nc(xsrc + i);
    if (a.x_copy != nullptr && b == 0) *reinterpret_cast<uint4*>(a.x_copy + i) = v;
    const float f[8] = {bf_lo(v.x), bf_hi(v.x), bf_lo(v.y), bf_hi(v.y),
                        bf_lo(v.z), bf_hi(v.z), bf_lo(v.w), bf_hi(v.w)};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      xs[i + j] = f[j];
      ss = fmaf(f[j], f[j], ss);
    }
  }
  if (a.gain != nullptr) {
    ss = warp_sum(ss);
    if (lane == 0) misc[warp] = ss;
    named_barrier(kGemvBarrierId, 256);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kGemvConsumerWarps; ++w) tot += misc[w];
    // rsqrt(mean(x^2) + eps) as 1/sqrt: correctly rounded sqrt and division.
    const float inv = 1.0f / sqrtf(tot / (float)K + a.eps);
    for (int i = ctid * 8; i < K; i += 256 * 8) {
      const uint4 g = ldg128_nc(a.gain + i);
      const float gf[8] = {bf_lo(g.x), bf_hi(g.x), bf_lo(g.y), bf_hi(g.y),
                           bf_lo(g.z), bf_hi(g.z), bf_lo(g.w), bf_hi(g.w)};
#pragma unroll
      for (int j = 0; j < 8; ++j) xs[i + j] = round_bf16(round_bf16(xs[i + j] * inv) * gf[j]);
    }
  }
  named_barrier(kGemvBarrierId, 256);

  // 2. Stream the weights: warp w owns row w of every 8-row block.
  float rowacc = 0.f;
  bool ok = true;
  for (int c = 0; c < nstage; ++c) {
    const int s = c % stages;
    if (!mbar_wait(&full[s], (c / stages) & 1, a.err, DEV_TIMEOUT_GEMV_FULL)) {
      ok = false;
      break;
    }
    const int blk = c / nkc, kc = c - blk * nkc;
    const int row = blk * kGemvConsumerWarps + warp;
    if (row < nrows) {
      const int c0 = kc * kGemvKChunk;
      const int nwc = min(kGemvKChunk, K - c0) >> 8;  // 256-column warp chunks: 1..4
      const uint8_t* piece = ring + (size_t)s * kGemvStageBytes + warp * kGemvPieceBytes + lane * 16;
      const float* xp = xs + c0 + lane * 8;
      float a0 = 0.f, a1 = 0.f;
      if (nwc == 4) {
        const uint4 w0 = lds128(piece);
        const uint4 w1 = lds128(piece + 512);
        const uint4 w2 = lds128(piece + 1024);
        const uint4 w3 = lds128(piece + 1536);
        a0 = dot8_f32x(w0, xp, a0);
        a1 = dot8_f32x(w1, xp + 256, a1);
        a0 = dot8_f32x(w2, xp + 512, a0);
        a1 = dot8_f32x(w3, xp + 768, a1);
      } else {
        for (int j = 0; j < nwc; ++j) {
          const uint4 wv = lds128(piece + j * 512);
          if (j & 1) a1 = dot8_f32x(wv, xp + j * 256, a1);
          else a0 = dot8_f32x(wv, xp + j * 256, a0);
        }
      }
      rowacc += a0 + a1;
      if (kc == nkc - 1) {
        const float t = warp_sum(rowacc);
        if (lane == 0) rowsum[row] = t;
        rowacc = 0.f;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (!ok && lane == 0) reinterpret_cast<volatile int*>(misc)[60] = 1;
  named_barrier(kGemvBarrierId, 256);
  if (reinterpret_cast<volatile int*>(misc)[60] != 0) return;  // uniform across the CTA

  // 3. Epilogue.
  if constexpr (EPI == EPI_STORE) {
    for (int r = ctid; r < nrows; r += 256) a.out[r0 + r] = __float2bfloat16_rn(rowsum[r]);
  } else if constexpr (EPI == EPI_RESIDUAL) {
    for (int r = ctid; r < nrows; r += 256) {
      const float p = round_bf16(rowsum[r]);
      a.out[r0 + r] = __float2bfloat16_rn(p + __bfloat162float(a.residual[r0 + r]));
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    for (int j = ctid; j < nrows / 2; j += 256) {
      const float g = round_bf16(rowsum[2 * j]);
      const float u = round_bf16(rowsum[2 * j + 1]);
      const float act = round_bf16(silu_f32(g));
      a.out[r0 / 2 + j] = __float2bfloat16_rn(act * u);
    }
  } else {  // EPI_ARGMAX
    float best = -INFINITY;
    int best_i = 0x7fffffff;
    for (int r = ctid; r < nrows; r += 256) {
      const bf16 lb = __float2bfloat16_rn(rowsum[r]);
      if (a.logits != nullptr) a.logits[r0 + r] = lb;
      const float v = __bfloat162float(lb);
      if (v > best) { best = v; best_i = r0 + r; }  // rows ascend: first max kept
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
    }
    int* misci = reinterpret_cast<int*>(misc);
    if (lane == 0) { misc[8 + warp] = best; misci[16 + warp] = best_i; }
    named_barrier(kGemvBarrierId, 256);
    if (ctid == 0) {
      for (int w = 0; w < kGemvConsumerWarps; ++w) {
        const float ov = misc[8 + w];
        const int oi = misci[16 + w];
        if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
      }
      a.part_val[b] = best;
      a.part_idx[b] = best_i;
      __threadfence();
      const unsigned ticket = atomicAdd(a.counter, 1u);
      misci[32] = (ticket == (unsigned)(G - 1)) ? 1 : 0;
    }
    named_barrier(kGemvBarrierId, 256);
    if (misci[32]) {
      __threadfence();
      best = -INFINITY;
      best_i = 0x7fffffff;
      for (int i = ctid; i < G; i += 256) {
        const float ov = __ldcg(a.part_val + i);
        const int oi = __ldcg(a.part_idx + i);
        if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
        if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
      }
      if (lane == 0) { misc[40 + warp] = best; misci[48 + warp] = best_i; }
      named_barrier(kGemvBarrierId, 256);
      if (ctid == 0) {
        for (int w = 0; w < kGemvConsumerWarps; ++w) {
          const float ov = misc[40 + w];
          const int oi = misci[48 + w];
          if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
        }
        *a.token_out = (best_i == 0x7fffffff) ? 0 : (int64_t)best_i;
        if (a.pos_inc != nullptr) *a.pos_inc += 1;
        *a.counter = 0u;
      }
    }
    return;
  }
  if (a.pos_inc != nullptr && b == 0 && ctid == 0) {
    // Only used when the step skips the head (prefill rows): all CTAs of this
    // grid are past pdl_wait, and the next reader runs after this grid ends.
    *a.pos_inc += 1;
  }
}

}  // namespace qb
