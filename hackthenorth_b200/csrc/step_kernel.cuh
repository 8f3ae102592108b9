// step_kernel.cuh — one batch-one greedy decode step (every layer and the LM
// head) as ONE persistent kernel for sm_100a.
//
// Why: as separate launches, every GEMV CTA holds a whole SM (544 threads x 96
// registers, ~220 KB of shared memory), so the next kernel's CTAs cannot start
// streaming until the previous kernel's CTAs have left the SM, and HBM idles
// for 1-3 us at each of the 5 launches per layer. Here each CTA (one per SM,
// cooperative launch) keeps one weight/KV ring for the whole step:
//  * the producer warp walks the step's phase list and streams, phase after
//    phase, exactly the bytes this CTA consumes: its rows of each weight
//    matrix (16 row pieces of 4 KB per 64 KB slot, 1D bulk copies, evict-first)
//    and, for attention, its slice of the layer's K/V cache (2D TMA boxes,
//    128 keys per slot). Weights and the cache below the newest position do
//    not depend on the step's activations, so the producer never waits for
//    another CTA: it runs up to 3 slots ahead, across phase boundaries;
//  * activations travel between CTAs as tagged words: every value a phase
//    publishes (the QKV row, the attention output, the residual stream, the
//    SwiGLU activations) is stored as one 32-bit word {tag:16, bf16:16}, and
//    attention split partials as 64-bit words {tag:32, fp32:32}. The tag names
//    the step (a device counter that only grows) and the writing phase, so a
//    reader that loads a word knows whether it holds this step's value, and
//    waits (bounded) only for words that do not yet. One store carries both
//    halves, so no fence, counter or grid barrier sits between phases: the
//    load of a phase's input is its synchronisation.
// Buffer reuse is safe without a barrier: a CTA overwrites a vector only in a
// phase whose own input it has read in full, and that input was completed by
// every CTA after all reads of the vector's previous value (each vector is
// read at most three phases after it is written, and every phase but attention
// reads a vector that all CTAs write).
// Phases per layer (dryft/engine/model.py decode step, batch one):
//   qkv   : RMSNorm(x) . Wqkv^T                        (layer 0 gathers the embedding row)
//   attn  : q/k RMSNorm + RoPE, cache append, split-KV GQA attention, merge
//   o     : xb = xa + bf16(O . attn)
//   gu    : act = bf16(silu(bf16(g))) * bf16(u), [g;u] = RMSNorm(xb) . Wgu^T (interleaved rows)
//   down  : xa = xb + bf16(Down . act)
// then the LM head: bf16 logits of RMSNorm(xa), greedy argmax (lowest index on
// ties), token written and position advanced by the CTA that finishes last.
// Arithmetic and rounding points are those of gemv.cuh and
// decode_attention.cuh (reference citations there).
#pragma once
#include "decode_attention.cuh"
#include "gemv.cuh"

namespace qb {

constexpr int kStepWarps = 16;
constexpr int kStepConsumers = kStepWarps * 32;
constexpr int kStepThreads = kStepConsumers + 32;
constexpr int kStepKC = 2048;                              // columns per weight row piece
constexpr int kStepPiece = kStepKC * 2;                    // 4 KB
constexpr int kStepSlotBytes = kStepWarps * kStepPiece;    // 64 KB
constexpr int kStepSlots = 3;
constexpr int kStepKeys = 128;                             // keys per attention slot
constexpr int kStepSub = kStepKeys * 128;                  // [128 keys][64 dims] bf16 = 16 KB
static_assert(4 * kStepSub == kStepSlotBytes, "an attention slot holds K lo, K hi, V lo, V hi");
constexpr int kStepBarrierId = 1;
constexpr int kStepMaxSplits = 24;
constexpr int kStepCombineFloats = 640;                    // one warp state: o 512, m 64, l 64
constexpr int kStepCombineBytes = 8 * kStepCombineFloats * 4;

enum StepKind : int { PH_STORE = 0, PH_RESIDUAL = 1, PH_SWIGLU = 2, PH_ARGMAX = 3, PH_ATTN = 4 };

struct StepPhase {
  int kind;
  int K;                  // GEMV: columns
  int rows;               // GEMV: weight rows
  int x_from;             // phase that wrote x (its tag); -1: the embedding row of the step's token
  const bf16* w;          // GEMV: [rows][K]
  const uint32_t* x;      // GEMV input words [K]; attention: the QKV row words (written by phase p - 1)
  const bf16* gain;       // RMSNorm gain or NULL
  const uint32_t* residual;  // PH_RESIDUAL: residual words (written by phase res_from)
  int res_from;
  int pad;
  uint32_t* out;          // STORE/RESIDUAL: [rows] words; SWIGLU: [rows/2]; ATTN: [Hq*D]
  uint32_t* x_copy;       // phase 0: the embedding row, as words of phase 0, for the residual stream
  const bf16* q_norm;     // attention
  const bf16* k_norm;
  bf16* k_cache;          // this layer's [Hkv][cap][128]
  bf16* v_cache;
  const CUtensorMap* tmk; // 64-row boxes over the layer's caches (global memory, 64-byte aligned)
  const CUtensorMap* tmv;
};

struct StepArgs {
  const StepPhase* phases;
  int n_phases;
  int Hq, Hkv, cap, vocab, max_splits, xs_bytes, max_rows;
  float eps;
  const int64_t* token;   // input token
  int64_t* token_out;     // greedy token
  int64_t* pos;           // read at start, +1 by the last CTA
  unsigned* epoch;        // step counter (tags), +1 by the last CTA
  const bf16* embed;
  const bf16* cos;
  const bf16* sin;
  unsigned long long* part_o;    // [Hkv][kStepMaxSplits][8][128] {tag, normalised split output}
  unsigned long long* part_lse;  // [Hkv][kStepMaxSplits][8] {tag, log2-sum-exp}
  unsigned* head_ticket;         // restored to 0
  float* head_val;        // [grid] per-CTA maxima
  int* head_idx;
  bf16* logits;           // optional [vocab] bf16 logits of the head
  int* err;
};

// 16-bit tag of the words written by phase `p` in step `epoch` (never 0, so a
// zeroed workspace holds no valid word; consecutive writes of one word always
// carry different tags).
__device__ __forceinline__ uint32_t step_tag16(uint32_t epoch, int p, int n_phases) {
  return (uint32_t)(((unsigned long long)epoch * (unsigned)n_phases + (unsigned)p) % 65535ull) + 1u;
}
__device__ __forceinline__ uint32_t step_tag32(uint32_t epoch, int p, int n_phases) {
  return (uint32_t)((unsigned long long)epoch * (unsigned)n_phases + (unsigned)p) + 1u;
}
__device__ __forceinline__ uint32_t word_of(uint32_t tag16, float v) {
  return (tag16 << 16) | (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v));
}

__host__ inline size_t step_smem_bytes(int xs_bytes, int max_rows) {
  return 1024 + (size_t)kStepSlots * kStepSlotBytes + (size_t)xs_bytes + kDecRows * kAttnD * 2 + 2 * kAttnD * 2 +
         (((size_t)max_rows * 4 + 15) & ~size_t(15)) + 2 * kStepSlots * 8 + 128 * 4;
}

struct StepAttnItem {
  int kvh, split, Se, k0, k1, nst;
};

// The attention work of CTA b: KV head kvh, split `split` of Se splits of
// about kAttnMinSplitKeys keys (16-aligned), keys [k0, k1) in nst slots.
// Producer and consumers evaluate it identically.
__device__ __forceinline__ StepAttnItem step_attn_item(int b, int hkv, int max_splits, long long last) {
  StepAttnItem it;
  const int n = (int)last + 1;
  const int2 sl = attn_split_len(n, min(max_splits, (n + kAttnMinSplitKeys - 1) / kAttnMinSplitKeys));
  const int per = sl.x;
  it.Se = sl.y;  // every split below Se has keys
  if (b < hkv * it.Se && n > 0) {
    it.kvh = b / it.Se;
    it.split = b % it.Se;
    it.k0 = min(n, it.split * per);
    it.k1 = min(n, it.k0 + per);
  } else {
    it.kvh = 0;
    it.split = 0;
    it.k0 = it.k1 = 0;
  }
  it.nst = (it.k1 - it.k0 + kStepKeys - 1) / kStepKeys;
  return it;
}

struct StepRows {
  int r0, nrows, nkc, nblk;
};
__device__ __forceinline__ StepRows step_rows(const StepPhase& ph, int b, int G) {
  const int rpu = ph.kind == PH_SWIGLU ? 2 : 1;
  const int units = ph.rows / rpu;
  const int u0 = (int)(((long long)units * b) / G);
  const int u1 = (int)(((long long)units * (b + 1)) / G);
  StepRows r;
  r.r0 = u0 * rpu;
  r.nrows = (u1 - u0) * rpu;
  r.nkc = (ph.K + kStepKC - 1) / kStepKC;
  r.nblk = (r.nrows + kStepWarps - 1) / kStepWarps;
  return r;
}

// True once any CTA has recorded a failed wait (a bad token or position is
// recorded too, but the step then runs to completion on a clamped value).
__device__ __forceinline__ bool step_aborted(const int* err) {
  const int v = *reinterpret_cast<const volatile int*>(err);
  return v != 0 && v != DEV_BAD_TOKEN && v != DEV_BAD_POSITION;
}

// Producer-side wait for a free slot: bounded, and gives up early once any CTA
// has recorded a failed wait.
__device__ __forceinline__ bool step_wait_empty(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (step_aborted(err)) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      report_error(err, DEV_TIMEOUT_GEMV_EMPTY);
      return false;
    }
  }
}

// Consumer-side wait for a filled slot: bounded, and gives up early once any
// CTA has recorded a failed wait (so a failed step ends in one wait limit, not one
// per remaining slot).
__device__ __forceinline__ bool step_wait_full(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (step_aborted(err)) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      report_error(err, code);
      return false;
    }
  }
}

// Four tagged words at p (16-byte aligned), waiting (bounded, abandoned once
// any CTA has recorded a failed wait) until all four carry `tag`. Returns
// false on timeout; the words are then whatever was read.
__device__ __forceinline__ bool step_load_words4(const uint32_t* p, uint32_t tag, uint4& v, int* err) {
  v = __ldcg(reinterpret_cast<const uint4*>(p));
  auto good = [&]() {
    return (v.x >> 16) == tag && (v.y >> 16) == tag && (v.z >> 16) == tag && (v.w >> 16) == tag;
  };
  if (good()) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 16; ++i) {
      __nanosleep(64);  // late words only: keep the polling request rate low
      v = __ldcg(reinterpret_cast<const uint4*>(p));
      if (good()) return true;
    }
    if (step_aborted(err)) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      report_error(err, DEV_TIMEOUT_PEER_FLAG);
      return false;
    }
  }
}
__device__ __forceinline__ bool step_load_word(const uint32_t* p, uint32_t tag, uint32_t& v, int* err) {
  v = __ldcg(p);
  if ((v >> 16) == tag) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 16; ++i) {
      __nanosleep(64);
      v = __ldcg(p);
      if ((v >> 16) == tag) return true;
    }
    if (step_aborted(err)) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      report_error(err, DEV_TIMEOUT_PEER_FLAG);
      return false;
    }
  }
}
__device__ __forceinline__ bool step_load_word64(const unsigned long long* p, uint32_t tag, float& v, int* err) {
  unsigned long long w = __ldcg(p);
  if ((uint32_t)(w >> 32) == tag) {
    v = __uint_as_float((uint32_t)w);
    return true;
  }
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 16; ++i) {
      __nanosleep(64);
      w = __ldcg(p);
      if ((uint32_t)(w >> 32) == tag) {
        v = __uint_as_float((uint32_t)w);
        return true;
      }
    }
    if (step_aborted(err)) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      report_error(err, DEV_TIMEOUT_PEER_FLAG);
      return false;
    }
  }
}
__device__ __forceinline__ float word_val(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ bool tags4(const uint4& v, uint32_t tag) {
  return ((v.x >> 16) == tag) & ((v.y >> 16) == tag) & ((v.z >> 16) == tag) & ((v.w >> 16) == tag);
}
__device__ __forceinline__ uint32_t pack_words(uint32_t lo, uint32_t hi) { return (lo & 0xffffu) | (hi << 16); }

// Per-head RMSNorm + rotate-half RoPE (as norm_rope_head) of one 128-dim head
// read from tagged words; lane owns dims [4*lane, 4*lane+4). Returns false if
// the words did not arrive (error recorded).
__device__ __forceinline__ bool step_norm_rope(const uint32_t* src, uint32_t tag, const bf16* gain, const bf16* cos_row,
                                               const bf16* sin_row, float eps, int lane, bf16* dst_smem,
                                               bf16* dst_global, int* err) {
  uint4 w;
  const bool ok = step_load_words4(src + 4 * lane, tag, w, err);
  const uint2 gv = *reinterpret_cast<const uint2*>(gain + 4 * lane);
  const uint2 cv = *reinterpret_cast<const uint2*>(cos_row + 4 * lane);
  const uint2 sv = *reinterpret_cast<const uint2*>(sin_row + 4 * lane);
  float x[4] = {word_val(w.x), word_val(w.y), word_val(w.z), word_val(w.w)};
  const float g[4] = {bf_lo(gv.x), bf_hi(gv.x), bf_lo(gv.y), bf_hi(gv.y)};
  const float c[4] = {bf_lo(cv.x), bf_hi(cv.x), bf_lo(cv.y), bf_hi(cv.y)};
  const float s[4] = {bf_lo(sv.x), bf_hi(sv.x), bf_lo(sv.y), bf_hi(sv.y)};
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(x[i], x[i], ss);
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / (float)kAttnD + eps);
  float n[4], r[4], o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) n[i] = round_bf16(round_bf16(x[i] * inv) * g[i]);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float other = __shfl_xor_sync(0xffffffffu, n[i], 16);  // dim +-64
    r[i] = (lane < 16) ? -other : other;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = round_bf16(n[i] * c[i]) + round_bf16(r[i] * s[i]);
  uint2 ov;
  ov.x = pack_bf16(o[0], o[1]);
  ov.y = pack_bf16(o[2], o[3]);
  *reinterpret_cast<uint2*>(dst_smem + 4 * lane) = ov;
  if (dst_global != nullptr) *reinterpret_cast<uint2*>(dst_global + 4 * lane) = ov;
  return ok;
}

// Position in the producer's stage sequence: stage j of phase p (phases
// without work for this CTA are skipped).
struct StepCursor {
  int p, j, nst;
  StepAttnItem it;
  StepRows R;
};
__device__ __forceinline__ void step_cursor_enter(StepCursor& u, const StepArgs& a, int b, int G, long long last) {
  while (u.p < a.n_phases) {
    const StepPhase& ph = a.phases[u.p];
    if (ph.kind == PH_ATTN) {
      u.it = step_attn_item(b, a.Hkv, a.max_splits, last);
      u.nst = u.it.nst;
    } else {
      u.R = step_rows(ph, b, G);
      u.nst = u.R.nblk * u.R.nkc;
    }
    if (u.nst > 0) return;
    ++u.p;
  }
}
__device__ __forceinline__ void step_cursor_next(StepCursor& u, const StepArgs& a, int b, int G, long long last) {
  if (++u.j < u.nst) return;
  u.j = 0;
  ++u.p;
  step_cursor_enter(u, a, b, G, last);
}
// Online-softmax state of one warp: rows 2*t4 + e, dims dt*16 + g4 + 8*(i>>1).
struct StepAttnState {
  float m[2], l[2], o[4][4];
};
__device__ __forceinline__ void step_state_store(float* slot, const StepAttnState& s, int lane) {
#pragma unroll
  for (int dt = 0; dt < 4; ++dt)
#pragma unroll
    for (int i = 0; i < 4; ++i) slot[(dt * 4 + i) * 32 + lane] = s.o[dt][i];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    slot[512 + e * 32 + lane] = s.m[e];
    slot[576 + e * 32 + lane] = s.l[e];
  }
}
__device__ __forceinline__ void step_state_merge(StepAttnState& s, const float* slot, int lane) {
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float m2 = slot[512 + e * 32 + lane];
    const float l2 = slot[576 + e * 32 + lane];
    const float M = fmaxf(s.m[e], m2);
    const float f1 = (s.m[e] == -INFINITY) ? 0.f : exp2f(s.m[e] - M);
    const float f2 = (m2 == -INFINITY) ? 0.f : exp2f(m2 - M);
    s.l[e] = s.l[e] * f1 + l2 * f2;
    s.m[e] = M;
#pragma unroll
    for (int dt = 0; dt < 4; ++dt) {
      s.o[dt][e] = s.o[dt][e] * f1 + slot[(dt * 4 + e) * 32 + lane] * f2;
      s.o[dt][2 + e] = s.o[dt][2 + e] * f1 + slot[(dt * 4 + 2 + e) * 32 + lane] * f2;
    }
  }
}

// 17 warps share four 16K-register sub-partitions (5 warps on one of them), so
// launch_bounds(544, 1) caps a thread at 96 registers.
__global__ void __launch_bounds__(kStepThreads, 1) step_kernel(const StepArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  bf16* xs = reinterpret_cast<bf16*>(ring + kStepSlots * kStepSlotBytes);
  bf16* qs = reinterpret_cast<bf16*>(reinterpret_cast<uint8_t*>(xs) + a.xs_bytes);
  bf16* kvnew = qs + kDecRows * kAttnD;
  float* rowsum = reinterpret_cast<float*>(kvnew + 2 * kAttnD);
  uint64_t* full = reinterpret_cast<uint64_t*>(rowsum + ((a.max_rows + 3) & ~3));
  uint64_t* empty = full + kStepSlots;
  float* misc = reinterpret_cast<float*>(empty + kStepSlots);
  volatile int* flags = reinterpret_cast<volatile int*>(misc + 100);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = gridDim.x;
  const int b = blockIdx.x;
  const int Gq = a.Hq / a.Hkv;  // query rows per KV head (<= 8)

  if (tid == 0) {
    for (int s = 0; s < kStepSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kStepWarps);
    }
    fence_mbar_init();
    flags[0] = 0;
    flags[1] = 0;
  }
  __syncthreads();

  long long last = *a.pos;  // written by the previous step's kernel
  if (last < 0 || last >= a.cap) {
    if (tid == 0 && b == 0) report_error(a.err, DEV_BAD_POSITION);
    last = -1;
  }

  if (warp == kStepWarps) {
    // ================================================================ producer
    // The cursor walks this CTA's stages phase after phase; the producer
    // waits only for free ring slots, never for another CTA.
    const uint64_t policy = policy_evict_first();
    int issued = 0;
    bool ok = true;
    StepCursor cu;
    cu.p = 0;
    cu.j = 0;
    step_cursor_enter(cu, a, b, G, last);
    for (int c = 0; cu.p < a.n_phases; ++c) {
      const StepPhase& ph = a.phases[cu.p];
      const int s = c % kStepSlots;
      if (c >= kStepSlots) {
        int good = 1;
        if (lane == 0) good = step_wait_empty(&empty[s], ((c / kStepSlots) - 1) & 1, a.err) ? 1 : 0;
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) {
          ok = false;
          break;
        }
      }
      uint8_t* slot = ring + (size_t)s * kStepSlotBytes;
      if (ph.kind == PH_ATTN) {
        if (lane == 0) mbar_arrive_expect_tx(&full[s], kStepSlotBytes);
        __syncwarp();
        if (lane < 8) {
          const int sub = lane >> 1, half = lane & 1;
          const int y = cu.it.kvh * a.cap + cu.it.k0 + cu.j * kStepKeys + half * 64;
          tma_load_2d(slot + sub * kStepSub + half * (kStepSub / 2), sub < 2 ? ph.tmk : ph.tmv, (sub & 1) * 64, y,
                      &full[s]);
        }
      } else {
        const int blk = cu.j / cu.R.nkc, kc = cu.j - blk * cu.R.nkc;
        const int nr = min(kStepWarps, cu.R.nrows - blk * kStepWarps);
        const int c0 = kc * kStepKC;
        const uint32_t piece = (uint32_t)min(kStepKC, ph.K - c0) * 2;
        if (lane == 0) mbar_arrive_expect_tx(&full[s], piece * nr);
        __syncwarp();
        if (lane < nr)
          bulk_g2s(slot + lane * kStepPiece, ph.w + (size_t)(cu.R.r0 + blk * kStepWarps + lane) * ph.K + c0, piece,
                   &full[s], policy);
      }
      issued = c + 1;
      step_cursor_next(cu, a, b, G, last);
    }
    if (lane == 0) {
      // Keep shared memory alive until every issued copy has landed (normally
      // long consumed; after an error the consumers may already have left).
      for (int cc = (issued > kStepSlots ? issued - kStepSlots : 0); cc < issued; ++cc)
        mbar_wait(&full[cc % kStepSlots], (cc / kStepSlots) & 1, nullptr, 0);
    }
    return;
  }

  // ================================================================= consumers
  const int ctid = tid;
  const int g4 = lane >> 2, t4 = lane & 3;
  const uint32_t epoch = *a.epoch;  // advanced by the previous step's last CTA
  int c = 0;

  for (int p = 0; p < a.n_phases; ++p) {
    const StepPhase ph = a.phases[p];
    const uint32_t tag_out = step_tag16(epoch, p, a.n_phases);

    if (ph.kind == PH_ATTN) {
      // ================================================================ attention
      const StepAttnItem it = step_attn_item(b, a.Hkv, a.max_splits, last);
      if (it.nst > 0) {
        const int kvh = it.kvh;
        const int kg = warp & 7, hh = warp >> 3;
        const uint32_t tag_in = step_tag16(epoch, p - 1, a.n_phases);
        if (ctid < kDecRows * kAttnD / 8) reinterpret_cast<uint4*>(qs)[ctid] = make_uint4(0, 0, 0, 0);
        named_barrier(kStepBarrierId, kStepConsumers);
        const bool owns_new = (it.k0 <= last) && (last < it.k1);
        const bf16* cos_row = a.cos + (size_t)last * kAttnD;
        const bf16* sin_row = a.sin + (size_t)last * kAttnD;
        bool okw = true;
        if (warp < Gq)
          okw = step_norm_rope(ph.x + (size_t)(kvh * Gq + warp) * kAttnD, tag_in, ph.q_norm, cos_row, sin_row, a.eps,
                               lane, qs + warp * kAttnD, nullptr, a.err);
        if (owns_new) {
          const size_t cslot = ((size_t)kvh * a.cap + last) * kAttnD;
          if (warp == kStepWarps - 1) {
            okw = step_norm_rope(ph.x + (size_t)a.Hq * kAttnD + kvh * kAttnD, tag_in, ph.k_norm, cos_row, sin_row,
                                 a.eps, lane, kvnew, ph.k_cache + cslot, a.err);
          } else if (warp == kStepWarps - 2) {
            uint4 w;
            okw = step_load_words4(ph.x + (size_t)(a.Hq + a.Hkv) * kAttnD + kvh * kAttnD + 4 * lane, tag_in, w, a.err);
            uint2 v;
            v.x = pack_words(w.x, w.y);
            v.y = pack_words(w.z, w.w);
            *reinterpret_cast<uint2*>(kvnew + kAttnD + 4 * lane) = v;
            *reinterpret_cast<uint2*>(ph.v_cache + cslot + 4 * lane) = v;
          }
        }
        if (!okw) flags[1] = 1;
        named_barrier(kStepBarrierId, kStepConsumers);
        uint32_t qb[8][2];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t r[4];
          ldsm_x4(r, qs + (lane & 7) * kAttnD + j * 32 + (lane >> 3) * 8);
          qb[2 * j][0] = r[0];
          qb[2 * j][1] = r[1];
          qb[2 * j + 1][0] = r[2];
          qb[2 * j + 1][1] = r[3];
        }
        StepAttnState S;
#pragma unroll
        for (int dt = 0; dt < 4; ++dt) S.o[dt][0] = S.o[dt][1] = S.o[dt][2] = S.o[dt][3] = 0.f;
        S.m[0] = S.m[1] = -INFINITY;
        S.l[0] = S.l[1] = 0.f;
        const float scale = 0.12751743082459868f;  // log2(e) / sqrt(128)
        for (int j = 0; j < it.nst; ++j, ++c) {
          const int s = c % kStepSlots;
          uint8_t* slot = ring + (size_t)s * kStepSlotBytes;
          if (!__all_sync(0xffffffffu, step_wait_full(&full[s], (c / kStepSlots) & 1, a.err, DEV_TIMEOUT_ATTN_FULL)))
            flags[1] = 1;
          const int kstage = it.k0 + j * kStepKeys;
          if (owns_new && kstage <= last && last < kstage + kStepKeys) {  // CTA-uniform
            named_barrier(kStepBarrierId, kStepConsumers);
            if (warp == 0 && flags[1] == 0) {
              const int kr = (int)last - kstage;
              const int which = lane >> 3, ch = lane & 7;
              *reinterpret_cast<uint4*>(slot + which * kStepSub + swz(kr, ch)) =
                  *reinterpret_cast<const uint4*>(kvnew + (which >> 1) * kAttnD + (which & 1) * 64 + ch * 8);
            }
            named_barrier(kStepBarrierId, kStepConsumers);
          }
          const int kb = kstage + kg * 16;  // this warp's 16 keys
          if (flags[1] == 0 && kb < it.k1) {
            const int svalid = it.k1 - kb;
            if (svalid < 16) {
              // Rows past the live range may hold anything (even NaN); P is 0
              // there, but 0 * NaN is NaN, so clear this warp's V rows.
              for (int i = lane; i < 16 * 8; i += 32) {
                const int row = i >> 3, ch = i & 7;
                if (row >= svalid)
                  *reinterpret_cast<uint4*>(slot + (2 + hh) * kStepSub + swz(kg * 16 + row, ch)) =
                      make_uint4(0, 0, 0, 0);
              }
              __syncwarp();
            }
            float sc[2][4];
#pragma unroll
            for (int h = 0; h < 2; ++h) sc[h][0] = sc[h][1] = sc[h][2] = sc[h][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              const int key = kg * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
              const int ch = ((ks & 3) << 1) + (lane >> 4);
              uint32_t ka[4];
              ldsm_x4(ka, slot + (ks >> 2) * kStepSub + swz(key, ch));
              mma_bf16_16816(sc[ks & 1], ka, qb[ks][0], qb[ks][1]);
            }
            float pr[2][2];  // [h][e]
            float corr[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              float x[2];
              float rmax = -INFINITY;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int key = kb + h * 8 + g4;
                const float v = (sc[0][h * 2 + e] + sc[1][h * 2 + e]) * scale;
                x[h] = (key < it.k1) ? v : -INFINITY;
                rmax = fmaxf(rmax, x[h]);
              }
              rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 4));
              rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 8));
              rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 16));
              const float mnew = fmaxf(S.m[e], rmax);
              corr[e] = (S.m[e] == -INFINITY) ? 0.f : exp2f(S.m[e] - mnew);
              float rs = 0.f;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                pr[h][e] = (x[h] == -INFINITY) ? 0.f : exp2f(x[h] - mnew);
                rs += pr[h][e];
              }
              S.l[e] = S.l[e] * corr[e] + rs;  // per-lane partial, summed over the key lanes at the end
              S.m[e] = mnew;
            }
#pragma unroll
            for (int dt = 0; dt < 4; ++dt) {
              S.o[dt][0] *= corr[0];
              S.o[dt][1] *= corr[1];
              S.o[dt][2] *= corr[0];
              S.o[dt][3] *= corr[1];
            }
            const uint32_t pb0 = movmatrix_trans(pack_bf16(pr[0][0], pr[0][1]));
            const uint32_t pb1 = movmatrix_trans(pack_bf16(pr[1][0], pr[1][1]));
#pragma unroll
            for (int dt = 0; dt < 4; ++dt) {
              const int mi = lane >> 3;
              const int key = kg * 16 + (lane & 7) + (mi >> 1) * 8;
              const int ch = ((dt & 3) << 1) + (mi & 1);
              uint32_t va[4];
              ldsm_x4_t(va, slot + (2 + hh) * kStepSub + swz(key, ch));
              mma_bf16_16816(S.o[dt], va, pb0, pb1);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          S.l[e] += __shfl_xor_sync(0xffffffffu, S.l[e], 4);
          S.l[e] += __shfl_xor_sync(0xffffffffu, S.l[e], 8);
          S.l[e] += __shfl_xor_sync(0xffffffffu, S.l[e], 16);
        }
        // Combine the 8 key groups of each dim half (fixed order) through xs:
        // groups 4..7 into 0..3, then 1..3 into 0.
        float* comb = reinterpret_cast<float*>(xs);
        if (kg >= 4) step_state_store(comb + (hh * 4 + (kg - 4)) * kStepCombineFloats, S, lane);
        named_barrier(kStepBarrierId, kStepConsumers);
        if (kg < 4) step_state_merge(S, comb + (hh * 4 + kg) * kStepCombineFloats, lane);
        named_barrier(kStepBarrierId, kStepConsumers);
        if (kg >= 1 && kg < 4) step_state_store(comb + (hh * 4 + (kg - 1)) * kStepCombineFloats, S, lane);
        named_barrier(kStepBarrierId, kStepConsumers);
        const uint32_t tag_part = step_tag32(epoch, p, a.n_phases);
        if (kg == 0) {
#pragma unroll
          for (int q = 0; q < 3; ++q) step_state_merge(S, comb + (hh * 4 + q) * kStepCombineFloats, lane);
          // Split result for rows 2*t4 + e, dims hh*64 + dt*16 + g4 (+8).
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int row = 2 * t4 + e;
            if (row < Gq) {
              const float L = S.l[e];
              const float lse = L > 0.f ? S.m[e] + log2f(L) : -INFINITY;
#pragma unroll
              for (int dt = 0; dt < 4; ++dt)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const int d = hh * 64 + dt * 16 + g4 + 8 * h;
                  const float v = L > 0.f ? S.o[dt][2 * h + e] / L : 0.f;
                  if (it.Se == 1)
                    ph.out[(size_t)(kvh * Gq + row) * kAttnD + d] = word_of(tag_out, v);
                  else
                    a.part_o[(((size_t)kvh * kStepMaxSplits + it.split) * kDecRows + row) * kAttnD + d] =
                        ((unsigned long long)tag_part << 32) | __float_as_uint(v);
                }
              if (hh == 0 && g4 == 0 && it.Se > 1)
                a.part_lse[((size_t)kvh * kStepMaxSplits + it.split) * kDecRows + row] =
                    ((unsigned long long)tag_part << 32) | __float_as_uint(lse);
            }
          }
        }
        if (it.Se > 1 && it.split == 0) {
          // Split 0 merges its head once every split's words carry this
          // step's tag (weights exp2(lse_s - max) / sum, in split order; lane s
          // of a warp fetches split s's log-sum-exp of the warp's row).
          static_assert(kStepMaxSplits <= 32, "one split per lane");
          bool okm = true;
          for (int idx = ctid; idx < Gq * kAttnD; idx += kStepConsumers) {
            const int r = idx >> 7, d = idx & 127;  // r is uniform across the warp
            const unsigned long long* lp = a.part_lse + (size_t)kvh * kStepMaxSplits * kDecRows + r;
            const unsigned long long* op = a.part_o + ((size_t)kvh * kStepMaxSplits * kDecRows + r) * kAttnD + d;
            // All loads issued at once; a stale word (its split still
            // writing) is then re-read with waits.
            unsigned long long lw = lane < it.Se ? __ldcg(lp + lane * kDecRows) : 0ull;
            unsigned long long ow[kStepMaxSplits];
#pragma unroll
            for (int sp = 0; sp < kStepMaxSplits; ++sp)
              ow[sp] = sp < it.Se ? __ldcg(op + (size_t)sp * kDecRows * kAttnD) : 0ull;
            // Re-read every stale word together until all are this step's.
            unsigned long long t0 = 0;
            while (true) {
              bool stale = lane < it.Se && (uint32_t)(lw >> 32) != tag_part;
#pragma unroll
              for (int sp = 0; sp < kStepMaxSplits; ++sp) stale |= sp < it.Se && (uint32_t)(ow[sp] >> 32) != tag_part;
              if (!stale) break;
              if (t0 == 0) t0 = global_timer_ns();
              if (step_aborted(a.err) || global_timer_ns() - t0 > kWaitLimitNs) {
                report_error(a.err, DEV_TIMEOUT_PEER_FLAG);
                okm = false;
                break;
              }
              __nanosleep(64);
              if (lane < it.Se && (uint32_t)(lw >> 32) != tag_part) lw = __ldcg(lp + lane * kDecRows);
#pragma unroll
              for (int sp = 0; sp < kStepMaxSplits; ++sp)
                if (sp < it.Se && (uint32_t)(ow[sp] >> 32) != tag_part) ow[sp] = __ldcg(op + (size_t)sp * kDecRows * kAttnD);
            }
            const float lse_l = lane < it.Se ? __uint_as_float((uint32_t)lw) : -INFINITY;
            float ov[kStepMaxSplits];
#pragma unroll
            for (int sp = 0; sp < kStepMaxSplits; ++sp) ov[sp] = sp < it.Se ? __uint_as_float((uint32_t)ow[sp]) : 0.f;
            const float mx = warp_max(lse_l);
            const float w_l = lane < it.Se ? exp2f(lse_l - mx) : 0.f;
            float den = 0.f, acc = 0.f;
#pragma unroll
            for (int sp = 0; sp < kStepMaxSplits; ++sp) {
              const float w = __shfl_sync(0xffffffffu, w_l, sp);
              if (sp < it.Se) {
                den += w;
                acc = fmaf(ov[sp], w, acc);
              }
            }
            ph.out[(size_t)(kvh * Gq + r) * kAttnD + d] = word_of(tag_out, acc / den);
          }
          if (!okm) flags[1] = 1;
        }
        named_barrier(kStepBarrierId, kStepConsumers);
        if (flags[1] != 0) return;
      }
    } else {
      // ===================================================================== GEMV
      const StepRows R = step_rows(ph, b, G);
      const int K = ph.K;
      // 1. Input row (the embedding row of the token, or the words of phase
      //    x_from) and its RMSNorm, into xs as bf16.
      float ss = 0.f;
      bool okw = true;
      if (ph.x_from < 0) {
        long long t = *a.token;
        if (t < 0 || t >= a.vocab) {
          if (ctid == 0 && b == 0) report_error(a.err, DEV_BAD_TOKEN);
          t = 0;
        }
        const bf16* xsrc = a.embed + (size_t)t * K;
        for (int i = ctid * 8; i < K; i += kStepConsumers * 8) {
          const uint4 v = ldg128_nc(xsrc + i);
          if (ph.x_copy != nullptr && b == 0) {
            const uint32_t* pv = reinterpret_cast<const uint32_t*>(&v);
            uint4 w0, w1;
            w0.x = (tag_out << 16) | (pv[0] & 0xffffu);
            w0.y = (tag_out << 16) | (pv[0] >> 16);
            w0.z = (tag_out << 16) | (pv[1] & 0xffffu);
            w0.w = (tag_out << 16) | (pv[1] >> 16);
            w1.x = (tag_out << 16) | (pv[2] & 0xffffu);
            w1.y = (tag_out << 16) | (pv[2] >> 16);
            w1.z = (tag_out << 16) | (pv[3] & 0xffffu);
            w1.w = (tag_out << 16) | (pv[3] >> 16);
            *reinterpret_cast<uint4*>(ph.x_copy + i) = w0;
            *reinterpret_cast<uint4*>(ph.x_copy + i + 4) = w1;
          }
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
      } else {
        // Optimistic: every load is issued without waiting on the previous
        // one; only a thread that saw a stale word re-reads (with waits).
        const uint32_t tag_in = step_tag16(epoch, ph.x_from, a.n_phases);
        bool fresh = true;
        for (int i = ctid * 8; i < K; i += kStepConsumers * 8) {
          const uint4 w0 = __ldcg(reinterpret_cast<const uint4*>(ph.x + i));
          const uint4 w1 = __ldcg(reinterpret_cast<const uint4*>(ph.x + i + 4));
          fresh &= tags4(w0, tag_in) & tags4(w1, tag_in);
          uint4 v;
          v.x = pack_words(w0.x, w0.y);
          v.y = pack_words(w0.z, w0.w);
          v.z = pack_words(w1.x, w1.y);
          v.w = pack_words(w1.z, w1.w);
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
        unsigned long long t0 = 0;
        while (!fresh) {  // re-read this thread's chunks together until all are fresh
          if (t0 == 0) t0 = global_timer_ns();
          if (step_aborted(a.err) || global_timer_ns() - t0 > kWaitLimitNs) {
            report_error(a.err, DEV_TIMEOUT_PEER_FLAG);
            okw = false;
            break;
          }
          __nanosleep(64);
          fresh = true;
          ss = 0.f;
          for (int i = ctid * 8; i < K; i += kStepConsumers * 8) {
          const uint4 w0 = __ldcg(reinterpret_cast<const uint4*>(ph.x + i));
          const uint4 w1 = __ldcg(reinterpret_cast<const uint4*>(ph.x + i + 4));
          fresh &= tags4(w0, tag_in) & tags4(w1, tag_in);
          uint4 v;
          v.x = pack_words(w0.x, w0.y);
          v.y = pack_words(w0.z, w0.w);
          v.z = pack_words(w1.x, w1.y);
          v.w = pack_words(w1.z, w1.w);
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
        }
      }
      if (!okw) flags[1] = 1;
      if (ph.gain != nullptr) {
        ss = warp_sum(ss);
        if (lane == 0) misc[warp] = ss;
        named_barrier(kStepBarrierId, kStepConsumers);
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kStepWarps; ++w) tot += misc[w];
        const float inv = 1.0f / sqrtf(tot / (float)K + a.eps);
        for (int i = ctid * 8; i < K; i += kStepConsumers * 8) {
          uint4 v = *reinterpret_cast<const uint4*>(xs + i);
          const uint4 g = ldg128_nc(ph.gain + i);
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
      // The residual rows (final since phase res_from, whose words this CTA
      // has already seen complete) are fetched now, off the critical path.
      float resv = 0.f;
      if (ph.kind == PH_RESIDUAL && ctid < R.nrows) {
        uint32_t w;
        if (!step_load_word(ph.residual + R.r0 + ctid, step_tag16(epoch, ph.res_from, a.n_phases), w, a.err))
          flags[1] = 1;
        resv = word_val(w);
      }
      named_barrier(kStepBarrierId, kStepConsumers);

      // 2. Stream this CTA's rows: warp w owns row w of every 16-row block.
      float rowacc = 0.f;
      for (int blk = 0; blk < R.nblk; ++blk) {
        const int row = blk * kStepWarps + warp;
        const bool active = row < R.nrows;
        for (int kc = 0; kc < R.nkc; ++kc, ++c) {
          const int s = c % kStepSlots;
          if (!step_wait_full(&full[s], (c / kStepSlots) & 1, a.err, DEV_TIMEOUT_GEMV_FULL)) flags[1] = 1;
          if (active && flags[1] == 0) {
            const int c0 = kc * kStepKC;
            const uint8_t* piece = ring + (size_t)s * kStepSlotBytes + warp * kStepPiece + lane * 16;
            const bf16* xp = xs + c0 + lane * 8;
            const int ncols = min(kStepKC, K - c0);
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
            for (; j < ncols; j += 256) a0 = dot8_bf16(lds128(piece + j * 2), lds128(xp + j), a0);
            rowacc += (a0 + a1) + (a2 + a3);
            if (kc == R.nkc - 1) {
              const float t = warp_sum(rowacc);
              if (lane == 0) rowsum[row] = t;
              rowacc = 0.f;
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        }
      }
      named_barrier(kStepBarrierId, kStepConsumers);
      if (flags[1] != 0) return;

      // 3. Epilogue: this phase's words (no fence: each word carries its tag).
      const int r0 = R.r0, nrows = R.nrows;
      if (ph.kind == PH_STORE) {
        for (int r = ctid; r < nrows; r += kStepConsumers) ph.out[r0 + r] = word_of(tag_out, rowsum[r]);
      } else if (ph.kind == PH_RESIDUAL) {
        if (ctid < nrows) ph.out[r0 + ctid] = word_of(tag_out, round_bf16(rowsum[ctid]) + resv);
      } else if (ph.kind == PH_SWIGLU) {
        for (int j = ctid; j < nrows / 2; j += kStepConsumers) {
          const float g = round_bf16(rowsum[2 * j]);
          const float u = round_bf16(rowsum[2 * j + 1]);
          const float act = round_bf16(silu_f32(g));
          ph.out[r0 / 2 + j] = word_of(tag_out, act * u);
        }
      } else {  // PH_ARGMAX: the last phase
        float best = -INFINITY;
        int best_i = 0x7fffffff;
        for (int r = ctid; r < nrows; r += kStepConsumers) {
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
        if (lane == 0) { misc[16 + warp] = best; misci[32 + warp] = best_i; }
        named_barrier(kStepBarrierId, kStepConsumers);
        if (ctid == 0) {
          for (int w = 0; w < kStepWarps; ++w) {
            const float ov = misc[16 + w];
            const int oi = misci[32 + w];
            if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
          }
          a.head_val[b] = best;
          a.head_idx[b] = best_i;
          const unsigned ticket = atomic_add_acq_rel_gpu(a.head_ticket, 1u);
          flags[2] = (ticket == (unsigned)(G - 1)) ? 1 : 0;
        }
        named_barrier(kStepBarrierId, kStepConsumers);
        if (flags[2]) {
          best = -INFINITY;
          best_i = 0x7fffffff;
          for (int i = ctid; i < G; i += kStepConsumers) {
            const float ov = __ldcg(a.head_val + i);
            const int oi = __ldcg(a.head_idx + i);
            if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
          }
          if (lane == 0) { misc[64 + warp] = best; misci[80 + warp] = best_i; }
          named_barrier(kStepBarrierId, kStepConsumers);
          if (ctid == 0) {
            for (int w = 0; w < kStepWarps; ++w) {
              const float ov = misc[64 + w];
              const int oi = misci[80 + w];
              if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
            }
            *a.token_out = (best_i == 0x7fffffff) ? 0 : (int64_t)best_i;
            *a.pos += 1;
            // Every CTA has drawn its head ticket, so all are past their last
            // tagged read of this step: the next step may use a new tag.
            *a.epoch = epoch + 1u;
            *a.head_ticket = 0u;
          }
        }
        return;
      }
    }
  }
}

}  // namespace qb
