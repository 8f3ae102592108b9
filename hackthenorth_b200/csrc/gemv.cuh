// gemv.cuh — batch-one weight-streaming GEMV for sm_100a with fused prologue
// (embedding gather, RMSNorm) and epilogues (store, +residual, SwiGLU pair,
// bf16 logits + greedy argmax).
//
// Design (HBM-bound: every weight byte is read exactly once per decode step):
//  * grid = one CTA per SM; CTA b owns the contiguous row range
//    [b*U/G, (b+1)*U/G) of the row-major weight (U = output units), so its
//    bytes are one contiguous stream.
//  * one producer lane streams that range through a ring of 16 KB stages with
//    1D bulk copies (cp.async.bulk + mbarrier complete_tx), evict-first in L2;
//  * 8 consumer warps: warp w takes the 512-byte "warp chunks" w, w+8, ... of
//    the stream; lane l multiplies 8 weights by x[col .. col+8) held in shared
//    memory and accumulates in fp32. Because K is a multiple of 256, a warp
//    chunk never straddles rows; when a warp moves to a new row it reduces its
//    partial (shuffles) into red[row][warp]. The epilogue sums the 8 warp
//    partials in a fixed order, so results are deterministic.
//  * PDL: the producer fills the ring before griddepcontrol.wait (weights are
//    immutable), so a GEMV's first ~100 KB per SM load while the previous
//    kernel is still finishing.
#pragma once
#include "common.cuh"

namespace qb {

constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvThreads = (kGemvConsumerWarps + 1) * 32;
constexpr int kGemvStageBytes = 16384;
constexpr int kGemvWarpChunk = 512;  // bytes: 32 lanes x 16 B
constexpr int kGemvChunksPerStage = kGemvStageBytes / kGemvWarpChunk;  // 32
constexpr int kGemvBarrierId = 1;    // named barrier of the 256 consumer threads

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
  int max_rows;         // max rows any CTA owns (size of red)
};

__host__ __device__ inline int gemv_rows_per_unit(int epi) { return epi == EPI_SWIGLU ? 2 : 1; }

__host__ inline size_t gemv_smem_bytes(int K, int stages, int max_rows) {
  return (size_t)stages * kGemvStageBytes + (size_t)K * 2 + (size_t)max_rows * kGemvConsumerWarps * 4 +
         (size_t)2 * stages * 8 + 64 * 4;
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
  const long long bytes_total = (long long)nrows * K * 2;
  const int nchunks = (int)((bytes_total + kGemvStageBytes - 1) / kGemvStageBytes);

  uint8_t* ring = smem;
  bf16* xs = reinterpret_cast<bf16*>(smem + (size_t)stages * kGemvStageBytes);
  float* red = reinterpret_cast<float*>(xs + K);
  uint64_t* full = reinterpret_cast<uint64_t*>(red + (size_t)a.max_rows * kGemvConsumerWarps);
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
      const uint8_t* src = reinterpret_cast<const uint8_t*>(a.w + (size_t)r0 * K);
      const uint64_t policy = policy_evict_first();
      int issued = 0;
      bool ok = true;
      bool waited = false;
      for (int c = 0; c < nchunks; ++c) {
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
        const long long left = bytes_total - (long long)c * kGemvStageBytes;
        const uint32_t bytes = (uint32_t)(left < kGemvStageBytes ? left : kGemvStageBytes);
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_g2s(ring + (size_t)s * kGemvStageBytes, src + (size_t)c * kGemvStageBytes, bytes, &full[s], policy);
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

  // 1. Input row (optionally the embedding gather) and its RMSNorm.
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
    *reinterpret_cast<uint4*>(xs + i) = v;
    if (a.x_copy != nullptr && b == 0) *reinterpret_cast<uint4*>(a.x_copy + i) = v;
    ss = fmaf(bf_lo(v.x), bf_lo(v.x), ss);
    ss = fmaf(bf_hi(v.x), bf_hi(v.x), ss);
    ss = fmaf(bf_lo(v.y), bf_lo(v.y), ss);
    ss = fmaf(bf_hi(v.y), bf_hi(v.y), ss);
    ss = fmaf(bf_lo(v.z), bf_lo(v.z), ss);
    ss = fmaf(bf_hi(v.z), bf_hi(v.z), ss);
    ss = fmaf(bf_lo(v.w), bf_lo(v.w), ss);
    ss = fmaf(bf_hi(v.w), bf_hi(v.w), ss);
  }
  for (int i = ctid; i < a.max_rows * kGemvConsumerWarps; i += 256) red[i] = 0.f;
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
      uint4 v = *reinterpret_cast<const uint4*>(xs + i);
      const uint4 g = ldg128_nc(a.gain + i);
      uint32_t* pv = reinterpret_cast<uint32_t*>(&v);
      const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float n0 = round_bf16(bf_lo(pv[j]) * inv) * bf_lo(pg[j]);
        const float n1 = round_bf16(bf_hi(pv[j]) * inv) * bf_hi(pg[j]);
        pv[j] = pack_bf16(n0, n1);
      }
      *reinterpret_cast<uint4*>(xs + i) = v;
    }
  }
  named_barrier(kGemvBarrierId, 256);

  // 2. Stream the weights.
  const int wc_total = (int)(bytes_total / kGemvWarpChunk);
  int row = 0;
  int col = warp * 256;
  while (col >= K) { col -= K; ++row; }
  int cur_row = row;
  float acc = 0.f;
  bool touched = false;
  bool ok = true;
  for (int c = 0; c < nchunks && ok; ++c) {
    const int s = c % stages;
    if (!mbar_wait(&full[s], (c / stages) & 1, a.err, DEV_TIMEOUT_GEMV_FULL)) {
      ok = false;
      break;
    }
    const uint8_t* st = ring + (size_t)s * kGemvStageBytes;
    const int base_wc = c * kGemvChunksPerStage;
    const int nwc = min(kGemvChunksPerStage, wc_total - base_wc);
    float d[kGemvChunksPerStage / kGemvConsumerWarps];
    int rws[kGemvChunksPerStage / kGemvConsumerWarps];
#pragma unroll
    for (int j = 0; j < kGemvChunksPerStage / kGemvConsumerWarps; ++j) {
      const int wc = warp + kGemvConsumerWarps * j;
      d[j] = 0.f;
      rws[j] = row;
      if (wc < nwc) {
        const uint4 wv = lds128(st + wc * kGemvWarpChunk + lane * 16);
        const uint4 xv = lds128(xs + col + lane * 8);
        d[j] = dot8(wv, xv, 0.f);
        col += kGemvConsumerWarps * 256;
        while (col >= K) { col -= K; ++row; }
      }
    }
#pragma unroll
    for (int j = 0; j < kGemvChunksPerStage / kGemvConsumerWarps; ++j) {
      const int wc = warp + kGemvConsumerWarps * j;
      if (wc < nwc) {
        if (rws[j] != cur_row) {
          const float t = warp_sum(acc);
          if (lane == 0) red[cur_row * kGemvConsumerWarps + warp] = t;
          acc = 0.f;
          cur_row = rws[j];
        }
        acc += d[j];
        touched = true;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (touched) {
    const float t = warp_sum(acc);
    if (lane == 0) red[cur_row * kGemvConsumerWarps + warp] = t;
  }
  if (!ok && lane == 0) reinterpret_cast<volatile int*>(misc)[60] = 1;
  named_barrier(kGemvBarrierId, 256);
  if (reinterpret_cast<volatile int*>(misc)[60] != 0) return;  // uniform across the CTA

  // 3. Epilogue.
  auto row_sum = [&](int r) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kGemvConsumerWarps; ++w) s += red[r * kGemvConsumerWarps + w];
    return s;
  };
  if constexpr (EPI == EPI_STORE) {
    for (int r = ctid; r < nrows; r += 256) a.out[r0 + r] = __float2bfloat16_rn(row_sum(r));
  } else if constexpr (EPI == EPI_RESIDUAL) {
    for (int r = ctid; r < nrows; r += 256) {
      const float p = round_bf16(row_sum(r));
      a.out[r0 + r] = __float2bfloat16_rn(p + __bfloat162float(a.residual[r0 + r]));
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    for (int j = ctid; j < nrows / 2; j += 256) {
      const float g = round_bf16(row_sum(2 * j));
      const float u = round_bf16(row_sum(2 * j + 1));
      const float act = round_bf16(silu_f32(g));
      a.out[r0 / 2 + j] = __float2bfloat16_rn(act * u);
    }
  } else {  // EPI_ARGMAX
    float best = -INFINITY;
    int best_i = 0x7fffffff;
    for (int r = ctid; r < nrows; r += 256) {
      const bf16 lb = __float2bfloat16_rn(row_sum(r));
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
