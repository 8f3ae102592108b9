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

constexpr int kGemvConsumerWarps = 16;
constexpr int kGemvConsumers = kGemvConsumerWarps * 32;
constexpr int kGemvThreads = kGemvConsumers + 32;
// A stage holds the same kc-column piece (kc = 1024 or 2048) of 16 rows:
// 16 one-dimensional bulk copies of 2 or 4 KB, one per row, issued by 16
// producer lanes in parallel.
__host__ __device__ inline int gemv_stage_bytes(int kc) { return kGemvConsumerWarps * kc * 2; }
constexpr int kGemvBarrierId = 1;  // named barrier of the consumer threads
constexpr int kGemvL2Ahead = 2;    // stages of the next GEMV brought into L2 by each CTA

enum GemvEpilogue : int { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3, EPI_PARTIAL = 4 };

constexpr int kMaxTp = 8;
constexpr int kPeerFlagSlots = 256;  // producer CTAs per (parity, sender)

// Tensor-parallel reduction over NVLink peer memory, fused into the o-proj and
// down GEMVs (EPI_RESIDUAL with tp.size > 1): each CTA stores its fp32 partial
// rows into recv[parity][my_rank][row] of every rank as 64-bit words
// {token, value}, reads back the n words of its own rows (waiting, bounded,
// until their tokens match: one aligned store carries both halves, so no
// fences or flags are needed) and sums them in rank order, so every rank gets
// the same bf16 result. Tokens grow with a per-context epoch (one per decode
// row), so nothing is ever reset; the two parity halves keep a fast rank's
// next sublayer from overwriting words a slow rank has not read yet.
struct TpPeers {
  unsigned long long* recv[kMaxTp];     // each rank's receive words [2][n][H]
  const unsigned long long* epoch;      // this rank's decode-row counter
  int rank, size;
};

__device__ __forceinline__ uint32_t tp_token(const TpPeers& t, int sub_id) {
  return (uint32_t)((*t.epoch + 1ull) * 256ull + (unsigned long long)(sub_id + 1));
}

struct GemvArgs {
  const bf16* w;        // [rows][K]
  int K;                // multiple of 128
  int rows;             // weight rows (2F for SwiGLU)
  const bf16* x;        // [K] input row, or NULL with embed
  const bf16* embed;    // [vocab][K] embedding table (layer-0 gather) or NULL
  const int64_t* token; // device token id for the gather
  int vocab;            // rows of embed (bounds check)
  bf16* x_copy;         // gather: CTA 0 stores the gathered row here (residual stream)
  const float* x32;     // tensor parallel: all-reduced fp32 projection sums; the input row is
                        // then bf16(bf16(x32) + x_res) and CTA 0 stores it to x_copy
  const bf16* x_res;    // residual added to x32
  const bf16* gain;     // [K] RMSNorm gain, or NULL (no norm)
  float eps;
  const bf16* residual; // EPI_RESIDUAL
  int res_early;        // EPI_RESIDUAL: the residual was written at least two launches earlier
                        // (decode steps), so each thread reads its first row before the dependency wait
  bf16* out;            // EPI_STORE/RESIDUAL: [rows]; SWIGLU: [rows/2]
  float* out32;         // EPI_PARTIAL: [rows] fp32 sums (not rounded; reduced across ranks next)
  int row_base;         // EPI_ARGMAX: global index of weight row 0 (vocabulary shard offset)
  float* pair_out;      // EPI_ARGMAX under tensor parallelism: {max, index bits} instead of a token
  TpPeers tp;           // EPI_RESIDUAL across ranks (tp.size > 1): peer-memory reduction
  int tp_sub;           // sublayer id of the reduction (0..255)
  int tp_parity;        // receive buffer half (0: o-proj, 1: down)
  int hidden;           // H (length of the reduced vector)
  bf16* logits;         // EPI_ARGMAX: optional [rows]
  float* part_val;      // EPI_ARGMAX: [gridDim] partial maxima
  int* part_idx;        // EPI_ARGMAX: [gridDim] partial argmax
  unsigned* counter;    // EPI_ARGMAX: arrival counter (restored to 0)
  int64_t* token_out;   // EPI_ARGMAX: greedy token
  int64_t* pos_inc;     // optional: *pos_inc += 1 once the result is written
  int* err;             // device error word
  int stages;           // ring stages
  int max_rows;         // max rows any CTA owns (size of rowsum)
  int kc;               // columns per row piece: 1024 or 2048
  // The next GEMV of the chain (weights [nx_rows][nx_K], nx_rpu rows per unit,
  // pieces of nx_kc columns): once this CTA has issued its last stage it asks
  // L2 for the first stages of the rows the same CTA index streams next, so
  // they come from L2 across the kernel boundary. NULL: nothing to prefetch.
  const bf16* nx_w;
  int nx_K, nx_rows, nx_rpu, nx_kc, nx_grid;
  unsigned long long* trace;  // this launch's trace records (see common.cuh), or NULL
};

__host__ __device__ inline int gemv_rows_per_unit(int epi) { return epi == EPI_SWIGLU ? 2 : 1; }

__host__ inline size_t gemv_smem_bytes(int K, int stages, int max_rows, int kc) {
  return (size_t)stages * gemv_stage_bytes(kc) + (size_t)K * 2 + (((size_t)max_rows * 4 + 15) & ~size_t(15)) +
         (size_t)2 * stages * 8 + 128 * 4;
}

// acc += w.x for two packed bf16 pairs with sm_100's mixed-precision FMA
// (bf16 operands, fp32 addend and result, one rounding): the same value as
// converting both operands to fp32 and calling fmaf.
__device__ __forceinline__ float fma2_bf16(uint32_t w, uint32_t x, float acc) {
  asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\t"
      "mov.b32 {wl, wh}, %1;\n\t"
      "mov.b32 {xl, xh}, %2;\n\t"
      "fma.rn.f32.bf16 %0, wl, xl, %0;\n\t"
      "fma.rn.f32.bf16 %0, wh, xh, %0;\n\t}"
      : "+f"(acc)
      : "r"(w), "r"(x));
  return acc;
}
__device__ __forceinline__ float dot8_bf16(const uint4 w, const uint4 x, float acc) {
  acc = fma2_bf16(w.x, x.x, acc);
  acc = fma2_bf16(w.y, x.y, acc);
  acc = fma2_bf16(w.z, x.z, acc);
  acc = fma2_bf16(w.w, x.w, acc);
  return acc;
}

template <int EPI, bool TRACE = false>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvArgs a) {
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
  const int KC = a.kc;
  const int stage_bytes = gemv_stage_bytes(KC);
  const int nkc = (K + KC - 1) / KC;
  const int nblk = (nrows + kGemvConsumerWarps - 1) / kGemvConsumerWarps;
  const int nstage = nblk * nkc;

  uint8_t* ring = smem;
  bf16* xs = reinterpret_cast<bf16*>(smem + (size_t)stages * stage_bytes);
  float* rowsum = reinterpret_cast<float*>(xs + K);
  uint64_t* full = reinterpret_cast<uint64_t*>(rowsum + ((a.max_rows + 3) & ~3));
  uint64_t* empty = full + stages;
  float* misc = reinterpret_cast<float*>(empty + stages);
  if (TRACE && tid == 0) trace_stamp(trace_slot(a.trace), TRACE_ENTRY);

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGemvConsumerWarps);
    }
    fence_mbar_init();
    reinterpret_cast<int*>(misc)[100] = 0;  // CTA-wide abort flag
  }
  __syncthreads();

  if (warp == kGemvConsumerWarps) {
    // ---------------- producer warp ----------------
    // Lane r copies row r of each 16-row block; lane 0 also drives the ring.
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
        int good = 1;
        if (lane == 0) good = mbar_wait(&empty[s], ((c / stages) - 1) & 1, a.err, DEV_TIMEOUT_GEMV_EMPTY) ? 1 : 0;
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) {
          ok = false;
          break;
        }
      }
      const int blk = c / nkc, kc = c - blk * nkc;
      const int nr = min(kGemvConsumerWarps, nrows - blk * kGemvConsumerWarps);
      const int c0 = kc * KC;
      const uint32_t piece = (uint32_t)min(KC, K - c0) * 2;
      if (lane == 0) mbar_arrive_expect_tx(&full[s], piece * nr);
      __syncwarp();
      if (lane < nr)
        bulk_g2s(ring + (size_t)s * stage_bytes + lane * (KC * 2),
                 a.w + (size_t)(r0 + blk * kGemvConsumerWarps + lane) * K + c0, piece, &full[s], policy);
      issued = c + 1;
    }
    if (ok && a.nx_w != nullptr && b < a.nx_grid) {
      // first kGemvL2Ahead stages of the next GEMV's rows for CTA b (16 rows x
      // one piece per stage, one lane per row)
      const int nunits = a.nx_rows / a.nx_rpu;
      const int nu0 = (int)(((long long)nunits * b) / a.nx_grid);
      const int nu1 = (int)(((long long)nunits * (b + 1)) / a.nx_grid);
      const int nr0 = nu0 * a.nx_rpu, nrows_n = (nu1 - nu0) * a.nx_rpu;
      const int nkc_n = (a.nx_K + a.nx_kc - 1) / a.nx_kc;
      for (int c = 0; c < kGemvL2Ahead; ++c) {
        const int blk = c / nkc_n, kc = c - blk * nkc_n;
        const int row = blk * kGemvConsumerWarps + lane;
        if (lane < kGemvConsumerWarps && row < nrows_n) {
          const int c0 = kc * a.nx_kc;
          const uint32_t bytes = (uint32_t)min(a.nx_kc, a.nx_K - c0) * 2;
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.nx_w + (size_t)(nr0 + row) * a.nx_K + c0),
                       "r"(bytes)
                       : "memory");
        }
      }
    }
    if (!waited) {
      pdl_wait();
      pdl_trigger();
    }
    if (!ok && lane == 0) {
      // Keep shared memory alive until the copies already in flight land.
      for (int c = (issued > stages ? issued - stages : 0); c < issued; ++c)
        mbar_wait(&full[c % stages], (c / stages) & 1, nullptr, 0);
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int ctid = tid;  // 0..kGemvConsumers-1
  // Inputs that do not depend on the previous launch, read before the wait so
  // that no dependent global load sits between the input row and the loop or
  // the epilogue: this thread's RMSNorm gain chunks (weights) and, when the
  // caller marks the residual as written two launches earlier, its first
  // residual row.
  constexpr bool kPreGain = EPI == EPI_STORE || EPI == EPI_SWIGLU || EPI == EPI_ARGMAX;  // the normed projections
  uint4 gpre0 = make_uint4(0u, 0u, 0u, 0u), gpre1 = make_uint4(0u, 0u, 0u, 0u);
  if (kPreGain && a.gain != nullptr) {
    if (ctid * 8 < K) gpre0 = ldg128_nc(a.gain + ctid * 8);
    if (ctid * 8 + kGemvConsumers * 8 < K) gpre1 = ldg128_nc(a.gain + ctid * 8 + kGemvConsumers * 8);
  }
  float res_pre = 0.f;
  if constexpr (EPI == EPI_RESIDUAL)
    if (a.res_early && ctid < nrows) res_pre = __bfloat162float(a.residual[r0 + ctid]);
  pdl_wait();
  pdl_trigger();
  if (TRACE && ctid == 0) trace_stamp(trace_slot(a.trace), TRACE_WAIT);

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
  const float* x32 = a.x32;
  float ss = 0.f;
  for (int i = ctid * 8; i < K; i += kGemvConsumers * 8) {
    uint4 v;
    if (x32 != nullptr) {
      // Residual add after the cross-rank reduction: the projection is
      // rounded to bf16 once, then added to the residual and rounded again.
      const float4 p0 = __ldcg(reinterpret_cast<const float4*>(x32 + i));
      const float4 p1 = __ldcg(reinterpret_cast<const float4*>(x32 + i + 4));
      const uint4 rv = *reinterpret_cast<const uint4*>(a.x_res + i);
      v.x = pack_bf16(round_bf16(p0.x) + bf_lo(rv.x), round_bf16(p0.y) + bf_hi(rv.x));
      v.y = pack_bf16(round_bf16(p0.z) + bf_lo(rv.y), round_bf16(p0.w) + bf_hi(rv.y));
      v.z = pack_bf16(round_bf16(p1.x) + bf_lo(rv.z), round_bf16(p1.y) + bf_hi(rv.z));
      v.w = pack_bf16(round_bf16(p1.z) + bf_lo(rv.w), round_bf16(p1.w) + bf_hi(rv.w));
    } else {
      v = ldg128_nc(xsrc + i);
    }
    if (a.x_copy != nullptr && b == 0) *reinterpret_cast<uint4*>(a.x_copy + i) = v;
    *reinterpret_cast<uint4*>(xs + i) = v;
    ss = fmaf(bf_lo(v.x), bf_lo(v.x), ss);
    ss = fmaf(bf_hi(v.x), bf_hi(v.x), ss);
    ss = fmaf(bf_lo(v.y), bf_lo(v.y), ss);
    ss = fmaf(bf_hi(v.y), bf_hi(v.y), ss);
    ss = fmaf(bf_lo(v.z), bf_lo(v.z), ss);
    ss = fmaf(bf_hi(v.z), bf_hi(v.z), ss);
    ss = fmaf(bf_lo(v.w), bf_lo(v.w), ss);
    ss = fmaf(bf_hi(v.w), bf_hi(v.w), ss);
  }
  if (a.gain != nullptr) {
    ss = warp_sum(ss);
    if (lane == 0) misc[warp] = ss;
    named_barrier(kGemvBarrierId, kGemvConsumers);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kGemvConsumerWarps; ++w) tot += misc[w];
    // rsqrt(mean(x^2) + eps) as 1/sqrt: correctly rounded sqrt and division.
    const float inv = 1.0f / sqrtf(tot / (float)K + a.eps);
    for (int i = ctid * 8, it = 0; i < K; i += kGemvConsumers * 8, ++it) {
      uint4 v = *reinterpret_cast<const uint4*>(xs + i);
      const uint4 g = (kPreGain && it == 0) ? gpre0 : ((kPreGain && it == 1) ? gpre1 : ldg128_nc(a.gain + i));
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
  named_barrier(kGemvBarrierId, kGemvConsumers);

  // 2. Stream the weights: warp w owns row w of every 16-row block.
  float rowacc = 0.f;
  bool ok = true;
  int c = 0;
  for (int blk = 0; blk < nblk && ok; ++blk) {
    const int row = blk * kGemvConsumerWarps + warp;
    const bool active = row < nrows;
    for (int kc = 0; kc < nkc; ++kc, ++c) {
      const int s = c % stages;
      if (!mbar_wait(&full[s], (c / stages) & 1, a.err, DEV_TIMEOUT_GEMV_FULL)) {
        ok = false;
        break;
      }
      if (TRACE && c == 0 && ctid == 0) trace_stamp(trace_slot(a.trace), TRACE_FIRST);
      if (active) {
        const int c0 = kc * KC;
        const uint8_t* piece = ring + (size_t)s * stage_bytes + warp * (KC * 2) + lane * 16;
        const bf16* xp = xs + c0 + lane * 8;
        const int ncols = min(KC, K - c0);
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        int j = 0;
        for (; j + 1024 <= ncols; j += 1024) {
          const uint4 w0 = lds128(piece + j * 2);
          const uint4 w1 = lds128(piece + j * 2 + 512);
          const uint4 w2 = lds128(piece + j * 2 + 1024);
          const uint4 w3 = lds128(piece + j * 2 + 1536);
          const uint4 x0 = lds128(xp + j);
          const uint4 x1 = lds128(xp + j + 256);
          const uint4 x2 = lds128(xp + j + 512);
          const uint4 x3 = lds128(xp + j + 768);
          a0 = dot8_bf16(w0, x0, a0);
          a1 = dot8_bf16(w1, x1, a1);
          a2 = dot8_bf16(w2, x2, a2);
          a3 = dot8_bf16(w3, x3, a3);
        }
        for (; j < ncols; j += 256)  // K a multiple of 128: the last chunk may be half a warp wide
          if (j + lane * 8 < ncols) a0 = dot8_bf16(lds128(piece + j * 2), lds128(xp + j), a0);
        rowacc += (a0 + a1) + (a2 + a3);
        if (kc == nkc - 1) {
          const float t = warp_sum(rowacc);
          if (lane == 0) rowsum[row] = t;
          rowacc = 0.f;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  if (!ok && lane == 0) reinterpret_cast<volatile int*>(misc)[100] = 1;
  named_barrier(kGemvBarrierId, kGemvConsumers);
  if (reinterpret_cast<volatile int*>(misc)[100] != 0) return;  // uniform across the CTA
  if (TRACE && ctid == 0) trace_stamp(trace_slot(a.trace), TRACE_LOOP);

  // 3. Epilogue.
  if constexpr (EPI == EPI_STORE) {
    for (int r = ctid; r < nrows; r += kGemvConsumers) a.out[r0 + r] = __float2bfloat16_rn(rowsum[r]);
  } else if constexpr (EPI == EPI_PARTIAL) {
    for (int r = ctid; r < nrows; r += kGemvConsumers) a.out32[r0 + r] = rowsum[r];
  } else if constexpr (EPI == EPI_RESIDUAL) {
    if (a.tp.size > 1) {
      // Tensor parallel: every rank partitions the rows across CTAs the same
      // way, so CTA b exchanges only its own rows with CTA b of the other ranks.
      // Send {token, partial} words to every rank, then gather the n partials of
      // each row (one NVLink round trip), add them in rank order and finish the
      // row as on one GPU: bf16(bf16(sum) + residual).
      const size_t slot = (size_t)a.tp_parity * a.tp.size * a.hidden + r0;
      const uint32_t tok = tp_token(a.tp, a.tp_sub);
      const unsigned long long tag = (unsigned long long)tok << 32;
      for (int p = 0; p < a.tp.size; ++p)
        for (int r = ctid; r < nrows; r += kGemvConsumers)
          st_relaxed_sys_u64(a.tp.recv[p] + slot + (size_t)a.tp.rank * a.hidden + r, tag | __float_as_uint(rowsum[r]));
      const unsigned long long* mine = a.tp.recv[a.tp.rank] + slot;
      for (int r = ctid; r < nrows; r += kGemvConsumers) {
        unsigned long long w[kMaxTp];
#pragma unroll
        for (int p = 0; p < kMaxTp; ++p)
          if (p < a.tp.size) w[p] = ld_relaxed_sys_u64(mine + (size_t)p * a.hidden + r);
        float sum = 0.f;
#pragma unroll
        for (int p = 0; p < kMaxTp; ++p)
          if (p < a.tp.size)
            sum += ((uint32_t)(w[p] >> 32) == tok)
                       ? __uint_as_float((uint32_t)w[p])
                       : wait_tagged(mine + (size_t)p * a.hidden + r, tok, a.err, DEV_TIMEOUT_PEER_FLAG);
        const float res = (a.res_early && r == ctid) ? res_pre : __bfloat162float(a.residual[r0 + r]);
        a.out[r0 + r] = __float2bfloat16_rn(round_bf16(sum) + res);
      }
    } else {
      for (int r = ctid; r < nrows; r += kGemvConsumers) {
        const float p = round_bf16(rowsum[r]);
        const float res = (a.res_early && r == ctid) ? res_pre : __bfloat162float(a.residual[r0 + r]);
        a.out[r0 + r] = __float2bfloat16_rn(p + res);
      }
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    for (int j = ctid; j < nrows / 2; j += kGemvConsumers) {
      const float g = round_bf16(rowsum[2 * j]);
      const float u = round_bf16(rowsum[2 * j + 1]);
      const float act = round_bf16(silu_f32(g));
      a.out[r0 / 2 + j] = __float2bfloat16_rn(act * u);
    }
  } else {  // EPI_ARGMAX
    float best = -INFINITY;
    int best_i = 0x7fffffff;
    for (int r = ctid; r < nrows; r += kGemvConsumers) {
      const bf16 lb = __float2bfloat16_rn(rowsum[r]);
      if (a.logits != nullptr) a.logits[r0 + r] = lb;
      const float v = __bfloat162float(lb);
      if (v > best) { best = v; best_i = a.row_base + r0 + r; }  // rows ascend: first max kept
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
    }
    int* misci = reinterpret_cast<int*>(misc);
    if (lane == 0) { misc[16 + warp] = best; misci[32 + warp] = best_i; }
    named_barrier(kGemvBarrierId, kGemvConsumers);
    if (ctid == 0) {
      for (int w = 0; w < kGemvConsumerWarps; ++w) {
        const float ov = misc[16 + w];
        const int oi = misci[32 + w];
        if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
      }
      a.part_val[b] = best;
      a.part_idx[b] = best_i;
      __threadfence();
      const unsigned ticket = atomicAdd(a.counter, 1u);
      misci[48] = (ticket == (unsigned)(G - 1)) ? 1 : 0;
    }
    named_barrier(kGemvBarrierId, kGemvConsumers);
    if (misci[48]) {
      __threadfence();
      best = -INFINITY;
      best_i = 0x7fffffff;
      for (int i = ctid; i < G; i += kGemvConsumers) {
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
      if (lane == 0) { misc[64 + warp] = best; misci[80 + warp] = best_i; }
      named_barrier(kGemvBarrierId, kGemvConsumers);
      if (ctid == 0) {
        for (int w = 0; w < kGemvConsumerWarps; ++w) {
          const float ov = misc[64 + w];
          const int oi = misci[80 + w];
          if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
        }
        if (a.pair_out != nullptr) {
          a.pair_out[0] = best;
          a.pair_out[1] = __int_as_float(best_i);
        } else {
          *a.token_out = (best_i == 0x7fffffff) ? 0 : (int64_t)best_i;
          if (a.pos_inc != nullptr) *a.pos_inc += 1;
        }
        *a.counter = 0u;
      }
    }
    if (TRACE && ctid == 0) trace_stamp(trace_slot(a.trace), TRACE_EXIT);
    return;
  }
  if (a.pos_inc != nullptr && b == 0 && ctid == 0) {
    // Only used when the step skips the head (prefill rows): all CTAs of this
    // grid are past pdl_wait, and the next reader runs after this grid ends.
    *a.pos_inc += 1;
  }
  if (TRACE && ctid == 0) trace_stamp(trace_slot(a.trace), TRACE_EXIT);
}

}  // namespace qb

namespace qb {
// Tensor-parallel greedy pick: pairs[n] = {max logit, global index bits} from
// every rank's vocabulary shard; the largest value wins, the lowest index on
// ties (the single-device rule). Writes the token and advances the position.
// With wait_words set (prefill rows without the head), first waits until every
// rank's last down-projection words have arrived, so no rank starts the next
// row (and overwrites a peer's receive words) before all ranks have read them.
__global__ void tp_pick_kernel(const float* pairs, int n, int64_t* token_out, int64_t* pos_inc,
                               unsigned long long* epoch, const unsigned long long* wait_words,
                               unsigned long long wait_token_base, int wait_count, int* err) {
  pdl_wait();
  if (wait_words != nullptr) {
    const uint32_t tok = (uint32_t)((*epoch + 1ull) * 256ull + wait_token_base);
    for (int i = threadIdx.x; i < wait_count; i += blockDim.x) wait_tagged(wait_words + i, tok, err, DEV_TIMEOUT_PEER_FLAG);
    __syncthreads();
  }
  if (threadIdx.x != 0) return;
  if (epoch != nullptr) *epoch += 1;  // one decode row done on this rank
  float best = -INFINITY;
  int best_i = 0x7fffffff;
  for (int r = 0; r < n; ++r) {
    const float v = pairs[2 * r];
    const int i = __float_as_int(pairs[2 * r + 1]);
    if (v > best || (v == best && i < best_i)) { best = v; best_i = i; }
  }
  if (token_out != nullptr) *token_out = (best_i == 0x7fffffff) ? 0 : (int64_t)best_i;
  if (pos_inc != nullptr) *pos_inc += 1;
}
}  // namespace qb
