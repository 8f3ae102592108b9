// prefill_attention.cuh — causal GQA attention for a block of prompt rows
// (prefill), plus the row-wise helpers of the prefill layer chain.
//
// The reference runs prompt attention through SDPA's flash kernel with a
// causal mask (dryft/engine/attention.py:92-98); this is the same math with
// the decode path's numerics (base-2 online softmax, P rounded to bf16 before
// P.V, fp32 accumulation; dryft/engine/kernels/attention.py:49-57).
//
// flash_prefill_kernel: CTA = (block of 64 prompt rows, query head h); warp w
// takes rows 16w..16w+15 (query positions p0 + r). A producer warp streams K and
// V of KV head h / G in 64-key stages (TMA, [64 keys][64 dims] boxes, 128-byte
// swizzle) up to the block's last position into a 3-stage ring shared by the 4
// consumer warps. Per stage a warp computes S = Q.K^T (16 x 64, mma.sync
// m16n8k16 with the query rows on M), masks keys > its rows' positions, updates
// the online softmax, and accumulates O += P.V with P's accumulators reused as
// the A operand. The K/V of the block's own rows were appended by the previous
// kernel, so every key the block needs is in the cache.
#pragma once
#include "attention.cuh"

namespace qb {

constexpr int kFpRows = 64;        // prompt rows per CTA
constexpr int kFpKeys = 64;        // keys per stage
constexpr int kFpStages = 3;
constexpr int kFpWarps = 4;
constexpr int kFpThreads = (kFpWarps + 1) * 32;
constexpr int kFpBarrierId = 5;

struct FpArgs {
  const bf16* q;    // [T][Hq][128] (RoPE applied)
  bf16* out;        // [T][Hq][128]
  int T, p0, Hq, Hkv, cap;
  int* err;
};

__host__ inline size_t fp_smem_bytes() { return 1024 + (size_t)kFpStages * kAttnStageBytes + 2 * kFpStages * 8 + 64; }

__global__ void __launch_bounds__(kFpThreads, 2)
    flash_prefill_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                         const FpArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kFpStages * kAttnStageBytes);
  uint64_t* empty = full + kFpStages;
  volatile int* flags = reinterpret_cast<volatile int*>(empty + kFpStages);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int h = blockIdx.y;
  const int G = a.Hq / a.Hkv;
  const int kvh = h / G;
  const int r0 = blockIdx.x * kFpRows;
  const int rlast = min(r0 + kFpRows, a.T) - 1;    // last prompt row of the block
  const int pmax = a.p0 + rlast;                   // largest position the block attends from
  const int nkb = pmax / kFpKeys + 1;              // key blocks 0 .. pmax

  if (tid == 0) {
    for (int s = 0; s < kFpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kFpWarps);
    }
    fence_mbar_init();
    flags[0] = 0;
  }
  __syncthreads();
  pdl_wait();  // q and the appended K/V come from the previous kernel
  pdl_trigger();

  if (warp == kFpWarps) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensormap(&tmk);
      prefetch_tensormap(&tmv);
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kFpStages;
        if (kb >= kFpStages && !mbar_wait(&empty[s], ((kb / kFpStages) - 1) & 1, a.err, DEV_TIMEOUT_ATTN_EMPTY)) break;
        uint8_t* st = ring + s * kAttnStageBytes;
        const int y = kvh * a.cap + kb * kFpKeys;
        mbar_arrive_expect_tx(&full[s], kAttnStageBytes);
        tma_load_2d(st, &tmk, 0, y, &full[s]);
        tma_load_2d(st + kAttnSubTile, &tmk, 64, y, &full[s]);
        tma_load_2d(st + 2 * kAttnSubTile, &tmv, 0, y, &full[s]);
        tma_load_2d(st + 3 * kAttnSubTile, &tmv, 64, y, &full[s]);
        issued = kb + 1;
      }
      for (int kb = (issued > kFpStages ? issued - kFpStages : 0); kb < issued; ++kb)
        mbar_wait(&full[kb % kFpStages], (kb / kFpStages) & 1, nullptr, 0);
    }
    __syncwarp();
    return;
  }

  // ----------------------------------------------------------------- consumers
  const int g4 = lane >> 2, t4 = lane & 3;
  const int wr0 = r0 + 16 * warp;                 // this warp's first row
  const int wlast = min(wr0 + 15, a.T - 1);       // its last valid row
  const int wkb = wr0 <= rlast ? (a.p0 + wlast) / kFpKeys + 1 : 0;  // key blocks this warp needs
  // Query fragments (A operand): rows wr0 + g4 (+8), dims ks*16 + 2*t4 (+1) and +8.
  uint32_t qa[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = wr0 + g4 + (i & 1) * 8;
      const int d = ks * 16 + 2 * t4 + (i >> 1) * 8;
      qa[ks][i] = r < a.T ? *reinterpret_cast<const uint32_t*>(a.q + ((size_t)r * a.Hq + h) * kAttnD + d) : 0u;
    }
  const int prow[2] = {a.p0 + wr0 + g4, a.p0 + wr0 + g4 + 8};  // positions of the thread's two rows
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  const float scale = 0.12751743082459868f;  // log2(e) / sqrt(128)
  bool ok = true;

  for (int kb = 0; kb < nkb; ++kb) {
    const int s = kb % kFpStages;
    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (kb / kFpStages) & 1, a.err, DEV_TIMEOUT_ATTN_FULL))) ok = false;
    uint8_t* stage = ring + s * kAttnStageBytes;
    if (kb == nkb - 1 && pmax < kb * kFpKeys + kFpKeys - 1) {
      // Keys past the block's last position may hold anything (even NaN):
      // their P is 0, but 0 * NaN is NaN, so clear those V rows once.
      if (warp == 0 && ok) {
        const int valid = pmax - kb * kFpKeys + 1;
        for (int i = lane; i < (kFpKeys - valid) * 16; i += 32) {
          const int row = valid + (i >> 4);
          const int sub = (i >> 3) & 1, ch = i & 7;
          *reinterpret_cast<uint4*>(stage + (2 + sub) * kAttnSubTile + swz(row, ch)) = make_uint4(0, 0, 0, 0);
        }
      }
      named_barrier(kFpBarrierId, kFpWarps * 32);
    }
    if (ok && kb < wkb) {
      // S = Q . K^T for 64 keys: sc[nt] holds keys kb*64 + 8nt + 2*t4 (+1), rows g4 / g4+8.
      float sc[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int sb = 0; sb < 4; ++sb) {
        const uint8_t* st = stage + sb * kAttnSub * 128;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int mi = lane >> 3;
          const int key = (lane & 7) + (mi >> 1) * 8;
          const int ch = ((ks & 3) << 1) + (mi & 1);
          uint32_t b[4];
          ldsm_x4(b, st + (ks >> 2) * kAttnSubTile + swz(key, ch));
          mma_bf16_16816(sc[2 * sb], qa[ks], b[0], b[1]);
          mma_bf16_16816(sc[2 * sb + 1], qa[ks], b[2], b[3]);
        }
      }
      float corr[2];
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        float rmax = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = kb * kFpKeys + nt * 8 + 2 * t4 + e;
            const float v = sc[nt][hr * 2 + e] * scale;
            sc[nt][hr * 2 + e] = key <= prow[hr] ? v : -INFINITY;
            rmax = fmaxf(rmax, sc[nt][hr * 2 + e]);
          }
        rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 1));
        rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 2));
        const float mnew = fmaxf(m[hr], rmax);
        corr[hr] = (m[hr] == -INFINITY) ? 0.f : exp2f(m[hr] - mnew);
        float rs = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float x = sc[nt][hr * 2 + e];
            const float p = (x == -INFINITY) ? 0.f : exp2f(x - mnew);
            sc[nt][hr * 2 + e] = p;
            rs += p;
          }
        l[hr] = l[hr] * corr[hr] + rs;  // per-lane partial; summed over the 4 lanes of a row at the end
        m[hr] = mnew;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= corr[0];
        o[j][1] *= corr[0];
        o[j][2] *= corr[1];
        o[j][3] *= corr[1];
      }
      // O += P . V, 16 keys per k-step: P's C fragments are the A fragments.
#pragma unroll
      for (int sb = 0; sb < 4; ++sb) {
        uint32_t pa[4];
        pa[0] = pack_bf16(sc[2 * sb][0], sc[2 * sb][1]);          // row g4, keys 2t4..
        pa[1] = pack_bf16(sc[2 * sb][2], sc[2 * sb][3]);          // row g4+8
        pa[2] = pack_bf16(sc[2 * sb + 1][0], sc[2 * sb + 1][1]);  // row g4, keys 8+2t4..
        pa[3] = pack_bf16(sc[2 * sb + 1][2], sc[2 * sb + 1][3]);  // row g4+8, keys 8+2t4..
        const uint8_t* st = stage + sb * kAttnSub * 128;
#pragma unroll
        for (int dp = 0; dp < 8; ++dp) {
          const int mi = lane >> 3;
          const int key = (lane & 7) + (mi & 1) * 8;
          const int dch = dp * 2 + (mi >> 1);
          uint32_t b[4];
          ldsm_x4_t(b, st + (2 + (dch >> 3)) * kAttnSubTile + swz(key, dch & 7));
          mma_bf16_16816(o[2 * dp], pa, b[0], b[1]);
          mma_bf16_16816(o[2 * dp + 1], pa, b[2], b[3]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (!ok) return;
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    l[hr] += __shfl_xor_sync(0xffffffffu, l[hr], 1);
    l[hr] += __shfl_xor_sync(0xffffffffu, l[hr], 2);
  }
  // o[j]: dims 8j + 2*t4 (+1) of rows g4 (c0, c1) and g4+8 (c2, c3).
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int r = wr0 + g4 + hr * 8;
    if (r >= a.T) continue;
    const float inv = l[hr] > 0.f ? 1.0f / l[hr] : 0.f;
    bf16* dst = a.out + ((size_t)r * a.Hq + h) * kAttnD;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      *reinterpret_cast<uint32_t*>(dst + 8 * j + 2 * t4) = pack_bf16(o[j][2 * hr] * inv, o[j][2 * hr + 1] * inv);
  }
}

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
