// gemv_rows.cuh — weight-streaming GEMV for Q <= 8 input rows (the verify
// pass of speculative decoding: the current token and k draft tokens) on
// tensor cores, streaming every weight byte once for all Q rows.
//
// Follows the reference's multi-row decode projections (dryft/engine/kernels/
// projection.py:13-83 and down.py:8-35 with several rows; verify_step in
// dryft/engine/decode.py:168-179): RMSNorm of each row (x * inv rounded to bf16,
// times the bf16 gain, rounded), fp32 accumulation, one bf16 rounding of each
// projection, then the same epilogues as the one-row path (store, + residual,
// SwiGLU pair, bf16 logits + greedy argmax with the lowest index on ties).
//
// Layout per CTA (one per SM, rows split as in gemv.cuh):
//  * a ring slot holds one 2048-column piece of 16 weight rows, each row
//    padded to 4112 bytes so that the 8 rows an ldmatrix reads fall in 8
//    different bank groups; the producer warp fills it with 1D bulk copies
//    issued before griddepcontrol.wait (weights are immutable);
//  * the Q input rows are resident in shared memory (loaded and RMS-normalised
//    once per CTA) when they fit (Q * K <= 8 * 4096); otherwise (the down
//    projection's long rows) each slot also carries the same 2048 columns of
//    the input rows, copied after griddepcontrol.wait (the slot's full barrier
//    then takes two arrivals) and normalised in the slot when a gain is given;
//  * resident rows of at most two pieces (K <= 4096) go one step further: each
//    warp loads the B fragments of its columns of every piece into registers
//    once (32 registers), and the shared memory that held the rows becomes a
//    third ring slot, so two 64 KB stages are in flight while one is consumed
//    (the producer fills that slot for the first time once all consumer warps
//    have arrived on a barrier after their fragment loads);
//  * consumer warp w takes columns [128w, 128w+128) of the piece: 8 k-steps of
//    mma.sync m16n8k16 with A = 16 weight rows (ldmatrix) and B = the Q input
//    rows transposed (ldmatrix of the row-major rows), accumulating a 16 x 8
//    fp32 tile over all pieces of a 16-row block;
//  * at the end of a block the 16 warps' tiles are summed in warp order through
//    shared memory and the block's epilogue runs at once (no per-CTA row
//    buffer: the LM head keeps a running argmax per input row).
#pragma once
#include "attention.cuh"
#include "gemv.cuh"

namespace qb {

constexpr int kRowsWarps = 16;
constexpr int kRowsThreads = kRowsWarps * 32 + 32;
constexpr int kRowsKC = 2048;
constexpr int kRowsPitch = kRowsKC * 2 + 16;  // padded row piece
constexpr int kRowsStageBytes = (16 + 8) * kRowsPitch;
constexpr int kRowsStages = 2;
constexpr int kRowsRegStages = 3;  // register-fragment mode: the resident rows' space is the third slot
constexpr int kRowsMaxQ = 8;
constexpr int kRowsBarrierId = 1;
constexpr int kRowsResidentBytes = kRowsMaxQ * (4096 + 8) * 2;  // resident input rows
// Ring bytes: the larger of the two slot layouts (2 x 24 rows, or 2 x 16 rows
// plus the resident input rows).
constexpr int kRowsRingBytes = kRowsStages * kRowsStageBytes > kRowsStages * 16 * kRowsPitch + kRowsResidentBytes
                                   ? kRowsStages * kRowsStageBytes
                                   : kRowsStages * 16 * kRowsPitch + kRowsResidentBytes;

static_assert(kRowsRegStages * 16 * kRowsPitch <= kRowsRingBytes, "three 16-row slots fit the ring");
static_assert(kRowsResidentBytes <= 16 * kRowsPitch, "the resident rows fit one 16-row slot");

// Input rows resident in shared memory (else carried by every slot).
__host__ __device__ inline bool rows_resident(int Q, int K) { return (size_t)Q * (K + 8) * 2 <= kRowsResidentBytes; }
// Resident rows whose B fragments stay in registers (at most two pieces).
__host__ __device__ inline bool rows_in_regs(int Q, int K) { return rows_resident(Q, K) && K <= 2 * kRowsKC; }

struct RowsArgs {
  const bf16* w;            // [rows][K]
  int K, rows, Q;
  const bf16* x;            // [Q][K] input rows, or NULL: embedding rows of tokens[q]
  const bf16* embed;
  const int64_t* tokens;    // [Q] device ids for the gather
  int vocab;
  bf16* x_copy;             // gather: CTA 0 stores the gathered rows here [Q][K]
  const bf16* gain;         // RMSNorm gain or NULL
  float eps;
  const bf16* residual;     // EPI_RESIDUAL: [Q][rows]
  bf16* out;                // STORE/RESIDUAL: [Q][rows]; SWIGLU: [Q][rows/2]
  bf16* logits;             // ARGMAX: optional [Q][rows]
  float* part_val;          // ARGMAX: [Q][grid]
  int* part_idx;
  unsigned* counter;        // ARGMAX: arrival counter (restored to 0)
  int64_t* tokens_out;      // ARGMAX: [Q] greedy tokens
  float* pair_out;          // ARGMAX, tensor parallel: [Q][2] (bf16 max logit, global index bits)
                            // instead of tokens_out, for the cross-rank pick
  int row_base;             // ARGMAX: global index of this shard's first row
  float* out32;             // EPI_PARTIAL: [Q][rows] fp32 sums (reduced across ranks next)
  TpPeers tp;               // EPI_RESIDUAL across ranks (tp.size > 1): peer-memory reduction
  int tp_sub;               // sublayer id of the reduction (0..255)
  int tp_parity;            // receive buffer half (0: o-proj, 1: down)
  int hidden;               // H (rows of the reduced projection)
  int* err;
};

// Receive words of the rows reduction: after the decode rows' [2][n][H], a
// region [2][n][kRowsMaxQ][H] (parity, sender rank, input row, output row).
__host__ __device__ inline size_t rows_tp_words(int tp, int hidden) {
  return (size_t)2 * tp * hidden + (size_t)2 * tp * kRowsMaxQ * hidden;
}
__device__ __forceinline__ size_t rows_tp_slot(const RowsArgs& a, int sender, int q) {
  return (size_t)2 * a.tp.size * a.hidden +
         (((size_t)a.tp_parity * a.tp.size + sender) * kRowsMaxQ + q) * a.hidden;
}

// ring, two reduction buffers, row factors, barriers (full, empty, the
// fragments-loaded barrier), scratch.
__host__ inline size_t rows_smem_bytes() {
  return 16 + (size_t)kRowsRingBytes + 2 * 16 * 16 * 8 * 4 + kRowsMaxQ * 4 + (2 * kRowsRegStages + 1) * 8 + 256 * 4;
}

// One 2048-column piece of a 16-row block for warp w's columns [128w, 128w+128):
// 8 k-steps, A = 16 weight rows from the slot, B = the input-row fragments.
__device__ __forceinline__ void rows_piece_mma(float (&acc)[4], const uint8_t* slot, int warp, int lane,
                                               const uint32_t (&bq)[4][4]) {
#pragma unroll
  for (int k2 = 0; k2 < 4; ++k2) {
    const int col = warp * 128 + k2 * 32;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t af[4];
      const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
      ldsm_x4(af, slot + row * kRowsPitch + (col + h * 16 + (lane >> 4) * 8) * 2);
      mma_bf16_16816(acc, af, bq[k2][2 * h], bq[k2][2 * h + 1]);
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(kRowsThreads, 1) gemv_rows_kernel(const RowsArgs a) {
  extern __shared__ __align__(16) uint8_t smem_rows[];
  const bool resident = rows_resident(a.Q, a.K);
  const bool regs = rows_in_regs(a.Q, a.K);  // B fragments in registers, three ring slots
  const int NS = regs ? kRowsRegStages : kRowsStages;
  const int stage_bytes = resident ? 16 * kRowsPitch : kRowsStageBytes;
  const int xpitch = (a.K + 8) * 2;  // resident row pitch (bytes)
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_rows) + 15) & ~uintptr_t(15));
  // resident rows [Q][K + 8] (resident mode); in register mode the third slot
  uint8_t* xres = ring + kRowsStages * 16 * kRowsPitch;
  float* red = reinterpret_cast<float*>(ring + kRowsRingBytes);
  // red: two buffers [16 warps][16 rows][8], alternating by block
  float* inv = red + 2 * 16 * 16 * 8;  // [8]
  uint64_t* full = reinterpret_cast<uint64_t*>(inv + kRowsMaxQ);
  uint64_t* empty = full + kRowsRegStages;
  uint64_t* xfree = empty + kRowsRegStages;  // register mode: every consumer warp holds its fragments
  float* misc = reinterpret_cast<float*>(xfree + 1);  // 256 floats
  volatile int* flags = reinterpret_cast<volatile int*>(misc + 240);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = gridDim.x;
  const int b = blockIdx.x;
  const int K = a.K;
  const int Q = a.Q;
  constexpr int rpu = (EPI == EPI_SWIGLU) ? 2 : 1;
  const int units = a.rows / rpu;
  const int u0 = (int)(((long long)units * b) / G);
  const int u1 = (int)(((long long)units * (b + 1)) / G);
  const int r0 = u0 * rpu;
  const int nrows = (u1 - u0) * rpu;
  const int nkc = (K + kRowsKC - 1) / kRowsKC;
  const int nblk = (nrows + 15) / 16;
  const int nstage = nblk * nkc;

  if (tid == 0) {
    for (int s = 0; s < kRowsRegStages; ++s) {
      mbar_init(&full[s], resident ? 1 : 2);  // weights (+ the slot's input rows)
      mbar_init(&empty[s], kRowsWarps);
    }
    mbar_init(xfree, kRowsWarps);
    fence_mbar_init();
    flags[0] = 0;
    flags[1] = 0;
  }
  __syncthreads();

  if (warp == kRowsWarps) {
    // ---------------- producer warp: lanes 0..15 weight rows, 16..16+Q-1 input rows
    const uint64_t policy = policy_evict_first();
    auto issue_w = [&](int c) {
      const int s = c % NS, blk = c / nkc, kc = c - blk * nkc;
      const int nr = min(16, nrows - blk * 16);
      const int c0 = kc * kRowsKC;
      const uint32_t piece = (uint32_t)min(kRowsKC, K - c0) * 2;
      if (lane == 0) mbar_arrive_expect_tx(&full[s], piece * nr);
      __syncwarp();
      if (lane < nr)
        bulk_g2s(ring + (size_t)s * stage_bytes + lane * kRowsPitch,
                 a.w + (size_t)(r0 + blk * 16 + lane) * K + c0, piece, &full[s], policy);
    };
    const bf16* xrow = nullptr;  // this lane's input row (lanes 16..16+Q-1)
    auto issue_x = [&](int c) {
      if (resident) return;
      const int s = c % NS, kc = c % nkc;
      const int c0 = kc * kRowsKC;
      const uint32_t piece = (uint32_t)min(kRowsKC, K - c0) * 2;
      if (lane == 0) mbar_arrive_expect_tx(&full[s], piece * Q);
      __syncwarp();
      if (lane >= 16 && lane < 16 + Q)
        bulk_g2s(ring + (size_t)s * kRowsStageBytes + lane * kRowsPitch, xrow + c0, piece, &full[s], policy);
    };
    // weights are immutable: the first two stages go before the wait (in
    // register mode the third slot still holds the input rows then)
    const int pre = min(nstage, kRowsStages);
    for (int c = 0; c < pre; ++c) issue_w(c);
    pdl_wait();
    pdl_trigger();
    if (lane >= 16 && lane < 16 + Q) {
      const int q = lane - 16;
      if (a.x != nullptr) {
        xrow = a.x + (size_t)q * K;
      } else {
        long long t = a.tokens[q];
        if (t < 0 || t >= a.vocab) {
          if (b == 0) report_error(a.err, DEV_BAD_TOKEN);
          t = 0;
        }
        xrow = a.embed + (size_t)t * K;
      }
    }
    for (int c = 0; c < pre; ++c) issue_x(c);
    int issued = pre;
    bool ok = true;
    for (int c = pre; c < nstage; ++c) {
      const int s = c % NS;
      int good = 1;
      if (lane == 0)
        good = (c < NS ? mbar_wait(xfree, 0, a.err, DEV_TIMEOUT_GEMV_EMPTY)  // first fill of the rows' slot
                       : mbar_wait(&empty[s], ((c / NS) - 1) & 1, a.err, DEV_TIMEOUT_GEMV_EMPTY))
                   ? 1
                   : 0;
      good = __shfl_sync(0xffffffffu, good, 0);
      if (!good) {
        ok = false;
        break;
      }
      issue_w(c);
      issue_x(c);
      issued = c + 1;
    }
    if (lane == 0) {
      // Keep shared memory alive until the copies in flight land.
      for (int c = (issued > NS ? issued - NS : 0); c < issued; ++c) mbar_wait(&full[c % NS], (c / NS) & 1, nullptr, 0);
    }
    (void)ok;
    return;
  }

  // ---------------- consumer warps
  const int ctid = tid;
  const int g4 = lane >> 2, t4 = lane & 3;
  pdl_wait();
  pdl_trigger();

  // 1. Per-row RMSNorm factors (and the gathered rows for the residual
  //    stream); resident mode also stores the normalised rows.
  if (resident || a.gain != nullptr || (a.x == nullptr && a.x_copy != nullptr && b == 0)) {
    for (int q = 0; q < Q; ++q) {
      const bf16* xr;
      if (a.x != nullptr) {
        xr = a.x + (size_t)q * K;
      } else {
        long long t = a.tokens[q];
        if (t < 0 || t >= a.vocab) t = 0;
        xr = a.embed + (size_t)t * K;
      }
      float ss = 0.f;
      for (int i = ctid * 8; i < K; i += kRowsWarps * 32 * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + i);
        if (a.x == nullptr && a.x_copy != nullptr && b == 0)
          *reinterpret_cast<uint4*>(a.x_copy + (size_t)q * K + i) = v;
        if (resident) *reinterpret_cast<uint4*>(xres + q * xpitch + i * 2) = v;
        ss = dot8(v, v, ss);
      }
      ss = warp_sum(ss);
      if (lane == 0) misc[q * 16 + warp] = ss;
    }
    named_barrier(kRowsBarrierId, kRowsWarps * 32);
    if (ctid < Q) {
      float tot = 0.f;
      for (int w = 0; w < kRowsWarps; ++w) tot += misc[ctid * 16 + w];
      inv[ctid] = 1.0f / sqrtf(tot / (float)K + a.eps);  // correctly rounded sqrt and division
    }
    named_barrier(kRowsBarrierId, kRowsWarps * 32);
    if (resident && a.gain != nullptr) {
      // bf16(bf16(x * inv) * gain), as the one-row prologue does
      for (int q = 0; q < Q; ++q) {
        const float iq = inv[q];
        for (int i = ctid * 8; i < K; i += kRowsWarps * 32 * 8) {
          uint4 v = *reinterpret_cast<const uint4*>(xres + q * xpitch + i * 2);
          const uint4 g = ldg128_nc(a.gain + i);
          uint32_t* pv = reinterpret_cast<uint32_t*>(&v);
          const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float n0 = round_bf16(bf_lo(pv[j]) * iq) * bf_lo(pg[j]);
            const float n1 = round_bf16(bf_hi(pv[j]) * iq) * bf_hi(pg[j]);
            pv[j] = pack_bf16(n0, n1);
          }
          *reinterpret_cast<uint4*>(xres + q * xpitch + i * 2) = v;
        }
      }
      named_barrier(kRowsBarrierId, kRowsWarps * 32);
    }
  }

  // Register mode: this warp's B fragments of every piece (rows >= Q repeat
  // row Q-1, as below), then the rows' slot is handed to the producer.
  uint32_t bqr[2][4][4];
  if (regs) {
    const int qrow = min(lane & 7, Q - 1);
#pragma unroll
    for (int kc = 0; kc < 2; ++kc)
#pragma unroll
      for (int k2 = 0; k2 < 4; ++k2) {
        const int col = kc * kRowsKC + warp * 128 + k2 * 32;
        if (kc < nkc && warp * 128 < min(kRowsKC, K - kc * kRowsKC))
          ldsm_x4(bqr[kc][k2], xres + qrow * xpitch + (col + (lane >> 3) * 8) * 2);
        else
          bqr[kc][k2][0] = bqr[kc][k2][1] = bqr[kc][k2][2] = bqr[kc][k2][3] = 0u;
      }
    __syncwarp();
    if (lane == 0) mbar_arrive(xfree);
  }

  // Running argmax per input row (thread t of the first 128 owns row t & 7).
  float best = -INFINITY;
  int best_i = 0x7fffffff;

  int c = 0;
  bool ok = true;
  for (int blk = 0; blk < nblk && ok; ++blk) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int kc = 0; kc < nkc; ++kc, ++c) {
      const int s = c % NS;
      if (!mbar_wait(&full[s], (c / NS) & 1, a.err, DEV_TIMEOUT_GEMV_FULL)) flags[0] = 1;
      uint8_t* slot = ring + (size_t)s * stage_bytes;
      const int c0 = kc * kRowsKC;
      // B operand rows: the resident rows at column c0, or the slot's copy
      const uint8_t* xs = resident ? xres + c0 * 2 : slot + 16 * kRowsPitch;
      const int xp = resident ? xpitch : kRowsPitch;
      const int ncols = min(kRowsKC, K - c0);
      if (!resident && a.gain != nullptr) {
        uint8_t* xw = slot + 16 * kRowsPitch;
        // Normalise the Q input rows of this piece in place:
        // bf16(bf16(x * inv) * gain), as the one-row prologue does.
        const int per_row = ncols / 8;
        for (int it = ctid; it < Q * per_row; it += kRowsWarps * 32) {
          const int q = it / per_row, c8 = it - q * per_row;
          uint4 v = *reinterpret_cast<const uint4*>(xw + q * kRowsPitch + c8 * 16);
          const uint4 g = ldg128_nc(a.gain + c0 + c8 * 8);
          const float iq = inv[q];
          uint32_t* pv = reinterpret_cast<uint32_t*>(&v);
          const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float n0 = round_bf16(bf_lo(pv[j]) * iq) * bf_lo(pg[j]);
            const float n1 = round_bf16(bf_hi(pv[j]) * iq) * bf_hi(pg[j]);
            pv[j] = pack_bf16(n0, n1);
          }
          *reinterpret_cast<uint4*>(xw + q * kRowsPitch + c8 * 16) = v;
        }
        named_barrier(kRowsBarrierId, kRowsWarps * 32);
      }
      if (regs && warp * 128 < ncols && flags[0] == 0) {
        if (kc == 0)
          rows_piece_mma(acc, slot, warp, lane, bqr[0]);
        else
          rows_piece_mma(acc, slot, warp, lane, bqr[1]);
      } else if (warp * 128 < ncols && flags[0] == 0) {
        // ldmatrix reads 8 input rows; rows >= Q repeat row Q-1 (their output
        // columns are never used), so no address leaves the Q stored rows.
        const int qrow = min(lane & 7, Q - 1);
#pragma unroll
        for (int k2 = 0; k2 < 4; ++k2) {
          const int col = warp * 128 + k2 * 32;
          uint32_t bq[4];  // B fragments of k-steps 2*k2 (bq[0..1]) and 2*k2+1 (bq[2..3])
          ldsm_x4(bq, xs + qrow * xp + (col + (lane >> 3) * 8) * 2);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t af[4];
            const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
            ldsm_x4(af, slot + row * kRowsPitch + (col + h * 16 + (lane >> 4) * 8) * 2);
            mma_bf16_16816(acc, af, bq[2 * h], bq[2 * h + 1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // 2. Sum the 16 warps' tiles (warp order) and finish the block's rows.
    //    Blocks alternate between two buffers, so one barrier per block
    //    suffices: a buffer is rewritten only after the next block's barrier.
    float* rb = red + (blk & 1) * 16 * 128;
    float* rw = rb + warp * 128;
    rw[g4 * 8 + 2 * t4] = acc[0];
    rw[g4 * 8 + 2 * t4 + 1] = acc[1];
    rw[(g4 + 8) * 8 + 2 * t4] = acc[2];
    rw[(g4 + 8) * 8 + 2 * t4 + 1] = acc[3];
    named_barrier(kRowsBarrierId, kRowsWarps * 32);
    if (flags[0] != 0) {
      ok = false;
      break;
    }
    if (ctid < 128) {
      const int row = ctid >> 3, q = ctid & 7;
      const int nr = min(16, nrows - blk * 16);
      const int R = r0 + blk * 16 + row;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kRowsWarps; ++w) v += rb[w * 128 + ctid];
      if constexpr (EPI == EPI_STORE) {
        if (q < Q && row < nr) a.out[(size_t)q * a.rows + R] = __float2bfloat16_rn(v);
      } else if constexpr (EPI == EPI_RESIDUAL) {
        if (q < Q && row < nr) {
          if (a.tp.size > 1) {
            // tensor parallel: {token, partial} into every rank's words for
            // (this rank, q, R); summed after the loop
            const unsigned long long word = ((unsigned long long)tp_token(a.tp, a.tp_sub) << 32) | __float_as_uint(v);
            for (int p = 0; p < a.tp.size; ++p) st_relaxed_sys_u64(a.tp.recv[p] + rows_tp_slot(a, a.tp.rank, q) + R, word);
          } else {
            a.out[(size_t)q * a.rows + R] =
                __float2bfloat16_rn(round_bf16(v) + __bfloat162float(a.residual[(size_t)q * a.rows + R]));
          }
        }
      } else if constexpr (EPI == EPI_PARTIAL) {
        if (q < Q && row < nr) a.out32[(size_t)q * a.rows + R] = v;
      } else if constexpr (EPI == EPI_SWIGLU) {
        // rows are interleaved (gate, up); the up sum sits 8 threads further
        const float u = __shfl_down_sync(0xffffffffu, v, 8);
        if (q < Q && row < nr && (row & 1) == 0) {
          const float act = round_bf16(silu_f32(round_bf16(v)));
          a.out[(size_t)q * (a.rows / 2) + R / 2] = __float2bfloat16_rn(act * round_bf16(u));
        }
      } else {  // EPI_ARGMAX
        if (q < Q && row < nr) {
          const bf16 lb = __float2bfloat16_rn(v);
          if (a.logits != nullptr) a.logits[(size_t)q * a.rows + R] = lb;
          const float lv = __bfloat162float(lb);
          if (lv > best || (lv == best && R < best_i)) { best = lv; best_i = R; }
        }
      }
    }
  }
  named_barrier(kRowsBarrierId, kRowsWarps * 32);
  if (!ok) return;

  if constexpr (EPI == EPI_RESIDUAL) {
    if (a.tp.size > 1) {
      // Every rank partitions the rows across CTAs the same way: gather the
      // n partials of this CTA's rows (bounded waits on their tokens), add
      // them in rank order and finish as on one GPU: bf16(bf16(sum) + residual).
      const uint32_t tok = tp_token(a.tp, a.tp_sub);
      const unsigned long long* mine = a.tp.recv[a.tp.rank];
      for (int i = ctid; i < nrows * Q; i += kRowsWarps * 32) {
        const int q = i / nrows, R = r0 + (i - q * nrows);
        unsigned long long w[kMaxTp];
#pragma unroll
        for (int p = 0; p < kMaxTp; ++p)
          if (p < a.tp.size) w[p] = ld_relaxed_sys_u64(mine + rows_tp_slot(a, p, q) + R);
        float sum = 0.f;
#pragma unroll
        for (int p = 0; p < kMaxTp; ++p)
          if (p < a.tp.size)
            sum += ((uint32_t)(w[p] >> 32) == tok)
                       ? __uint_as_float((uint32_t)w[p])
                       : wait_tagged(mine + rows_tp_slot(a, p, q) + R, tok, a.err, DEV_TIMEOUT_PEER_FLAG);
        a.out[(size_t)q * a.rows + R] =
            __float2bfloat16_rn(round_bf16(sum) + __bfloat162float(a.residual[(size_t)q * a.rows + R]));
      }
    }
  }

  if constexpr (EPI == EPI_ARGMAX) {
    // Per input row: the best of this CTA (threads t with t & 7 == q), then
    // across CTAs by the CTA that arrives last.
    if (ctid < 128) {
#pragma unroll
      for (int o = 8; o < 32; o <<= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
        if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
      }
      int* misci = reinterpret_cast<int*>(misc);
      if (lane < 8) { misc[warp * 8 + lane] = best; misci[64 + warp * 8 + lane] = best_i; }
    }
    named_barrier(kRowsBarrierId, kRowsWarps * 32);
    int* misci = reinterpret_cast<int*>(misc);
    if (ctid < Q) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int w = 0; w < 4; ++w) {
        const float ov = misc[w * 8 + ctid];
        const int oi = misci[64 + w * 8 + ctid];
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      a.part_val[(size_t)ctid * G + b] = bv;
      a.part_idx[(size_t)ctid * G + b] = bi;
    }
    named_barrier(kRowsBarrierId, kRowsWarps * 32);
    if (ctid == 0) {
      const unsigned ticket = atomic_add_acq_rel_gpu(a.counter, 1u);
      flags[1] = (ticket == (unsigned)(G - 1)) ? 1 : 0;
    }
    named_barrier(kRowsBarrierId, kRowsWarps * 32);
    if (flags[1]) {
      // one warp per input row
      for (int q = warp; q < Q; q += kRowsWarps) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = lane; i < G; i += 32) {
          const float ov = __ldcg(a.part_val + (size_t)q * G + i);
          const int oi = __ldcg(a.part_idx + (size_t)q * G + i);
          if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
          if (a.pair_out != nullptr) {
            a.pair_out[2 * q] = bv;
            a.pair_out[2 * q + 1] = __int_as_float(bi == 0x7fffffff ? bi : bi + a.row_base);
          } else {
            a.tokens_out[q] = (bi == 0x7fffffff) ? 0 : (int64_t)bi;
          }
        }
      }
      if (ctid == 0) *a.counter = 0u;
    }
  }
}

// Per-head q/k RMSNorm + RoPE for Q consecutive positions, K/V appended to the
// cache (dryft/engine/kernels/fused.py:9-30,47-82 with several rows). One warp
// per (row, head); also writes the rows' positions for the attention kernel
// (verify) when asked. Used for the verify rows and for prompt rows; batched,
// row q is the next token of sequence q (its own position and cache slice).
struct RopeRowsArgs {
  const bf16* qkv;        // [Q][Hq*D + 2*Hkv*D]
  const bf16* q_norm;
  const bf16* k_norm;
  const bf16* cos;
  const bf16* sin;
  float eps;
  const int64_t* pos;     // first position (device), or NULL: p0
  int p0;
  int64_t* positions;     // [Q] out, or NULL
  bf16* q_out;            // [Q][Hq][D]
  bf16* k_cache;          // this layer's [Hkv][cap][D] ([Q][Hkv][cap][D] when batched)
  bf16* v_cache;
  int* err;
  int Q, Hq, Hkv, cap;
  int batched;            // 1: row q is sequence q, at position pos[q], in cache slice q
};

__device__ __forceinline__ void norm_rope_global(const bf16* src, const bf16* gain, const bf16* cos_row,
                                                 const bf16* sin_row, float eps, int lane, bf16* dst) {
  const uint2 xv = *reinterpret_cast<const uint2*>(src + 4 * lane);
  const uint2 gv = *reinterpret_cast<const uint2*>(gain + 4 * lane);
  const uint2 cv = *reinterpret_cast<const uint2*>(cos_row + 4 * lane);
  const uint2 sv = *reinterpret_cast<const uint2*>(sin_row + 4 * lane);
  const float x[4] = {bf_lo(xv.x), bf_hi(xv.x), bf_lo(xv.y), bf_hi(xv.y)};
  const float g[4] = {bf_lo(gv.x), bf_hi(gv.x), bf_lo(gv.y), bf_hi(gv.y)};
  const float c[4] = {bf_lo(cv.x), bf_hi(cv.x), bf_lo(cv.y), bf_hi(cv.y)};
  const float s[4] = {bf_lo(sv.x), bf_hi(sv.x), bf_lo(sv.y), bf_hi(sv.y)};
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(x[i], x[i], ss);
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / (float)kAttnD + eps);
  float n[4], o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) n[i] = round_bf16(round_bf16(x[i] * inv) * g[i]);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float other = __shfl_xor_sync(0xffffffffu, n[i], 16);  // dim +-64
    const float r = (lane < 16) ? -other : other;
    o[i] = round_bf16(n[i] * c[i]) + round_bf16(r * s[i]);
  }
  uint2 ov;
  ov.x = pack_bf16(o[0], o[1]);
  ov.y = pack_bf16(o[2], o[3]);
  *reinterpret_cast<uint2*>(dst + 4 * lane) = ov;
}

__global__ void __launch_bounds__(128) rope_rows_kernel(const RopeRowsArgs a) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int heads = a.Hq + 2 * a.Hkv;
  if (gw >= a.Q * heads) return;
  const int q = gw / heads, h = gw - q * heads;
  long long pos;
  bf16* k_cache = a.k_cache;
  bf16* v_cache = a.v_cache;
  if (a.batched) {
    pos = a.pos[q];
    if (pos < 0 || pos >= a.cap) {
      if (h == 0 && lane == 0) report_error(a.err, DEV_BAD_POSITION);
      return;
    }
    const size_t slice = (size_t)q * a.Hkv * a.cap * kAttnD;
    k_cache += slice;
    v_cache += slice;
  } else {
    const long long p0 = a.pos ? *a.pos : (long long)a.p0;
    pos = p0 + q;
    if (p0 < 0 || p0 + a.Q > a.cap) {
      if (gw == 0 && lane == 0) report_error(a.err, DEV_BAD_POSITION);
      return;
    }
    if (a.positions != nullptr && gw == 0 && lane < a.Q) a.positions[lane] = p0 + lane;
  }
  const bf16* src = a.qkv + (size_t)q * heads * kAttnD + (size_t)h * kAttnD;
  const bf16* cos_row = a.cos + (size_t)pos * kAttnD;
  const bf16* sin_row = a.sin + (size_t)pos * kAttnD;
  if (h < a.Hq) {
    norm_rope_global(src, a.q_norm, cos_row, sin_row, a.eps, lane, a.q_out + ((size_t)q * a.Hq + h) * kAttnD);
  } else if (h < a.Hq + a.Hkv) {
    const int kvh = h - a.Hq;
    norm_rope_global(src, a.k_norm, cos_row, sin_row, a.eps, lane, k_cache + ((size_t)kvh * a.cap + pos) * kAttnD);
  } else {
    const int kvh = h - a.Hq - a.Hkv;
    *reinterpret_cast<uint2*>(v_cache + ((size_t)kvh * a.cap + pos) * kAttnD + 4 * lane) =
        *reinterpret_cast<const uint2*>(src + 4 * lane);
  }
}

// Tensor-parallel rows, after the fp32 all-reduce of a projection's partial
// sums: out = bf16(bf16(sum) + residual), the one rounding of the single-GPU
// epilogue (dryft/engine/kernels/projection.py:57-83, down.py:8-35). n is a
// multiple of 8; 8 values per thread.
__global__ void tp_finish_rows_kernel(const float* __restrict__ sum, const bf16* __restrict__ res,
                                      bf16* __restrict__ out, int n) {
  pdl_wait();
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i >= n) return;
  const float4 p0 = __ldcg(reinterpret_cast<const float4*>(sum + i));
  const float4 p1 = __ldcg(reinterpret_cast<const float4*>(sum + i + 4));
  const uint4 rv = *reinterpret_cast<const uint4*>(res + i);
  const bf16* r = reinterpret_cast<const bf16*>(&rv);
  const float s[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
  uint4 ov;
  bf16* o = reinterpret_cast<bf16*>(&ov);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = __float2bfloat16_rn(round_bf16(s[j]) + __bfloat162float(r[j]));
  *reinterpret_cast<uint4*>(out + i) = ov;
}

// Tensor-parallel LM head over Q rows: pairs [tp][Q][2] hold each rank's
// (bf16 max logit, global index bits) per row; the prediction is the largest
// value, lowest global index on exact ties (dryft/engine/kernels/greedy.py:27-31).
// epoch (peer-memory reductions): advanced once per verify pass, as after a
// decode row, so the next pass's tokens are new.
__global__ void tp_pick_rows_kernel(const float* __restrict__ pairs, int tp, int Q, int64_t* __restrict__ preds,
                                    unsigned long long* epoch) {
  pdl_wait();
  const int q = threadIdx.x;
  if (q == 0 && epoch != nullptr) *epoch += 1;
  if (q >= Q) return;
  float best = -INFINITY;
  int best_i = 0x7fffffff;
  for (int r = 0; r < tp; ++r) {
    const float v = pairs[((size_t)r * Q + q) * 2];
    const int i = __float_as_int(pairs[((size_t)r * Q + q) * 2 + 1]);
    if (v > best || (v == best && i < best_i)) { best = v; best_i = i; }
  }
  preds[q] = (best_i == 0x7fffffff) ? 0 : (int64_t)best_i;
}

// Batched decode: pos[b] += delta for the n sequences (after their pass).
__global__ void add_rows_i64_kernel(int64_t* pos, int n, long long delta) {
  pdl_wait();
  if ((int)threadIdx.x < n) pos[threadIdx.x] += delta;
}

// Batched prefill: out[b] = ids[b][col] for the n prompts of length len
// (ids row-major [n][len]), the token rows of one teacher-forced pass.
__global__ void gather_column_i64_kernel(const int64_t* ids, int len, int col, int n, int64_t* out) {
  pdl_wait();
  if ((int)threadIdx.x < n) out[threadIdx.x] = ids[(size_t)threadIdx.x * len + col];
}

}  // namespace qb
