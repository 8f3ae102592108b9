// attention.cuh — split-KV grouped-query decode attention for sm_100a.
//
// Grid = Hkv x S CTAs; CTA (h, s) owns KV head h and the s-th of S equal,
// 16-aligned slices of the live key range [0, last_position]. Split sizes are
// computed on the device from the live position, so one captured launch stays
// balanced as the context grows.
//
// Per CTA: one producer lane streams 16-key stages of K and V with 2D TMA tensor
// loads ([16 keys][64 dims] boxes, 128-byte swizzle, no multicast) into an
// 8-stage ring; 4 consumer warps take stages round-robin and run
// S = Q.K^T and O += P.V on mma.sync m16n8k16 (bf16 in, fp32 accumulate) with a
// base-2 online softmax; P is rounded to bf16 before the P.V product and the
// softmax denominator sums the unrounded fp32 P, as the reference kernel does
// (dryft/engine/kernels/attention.py:49-57). Rows are (head-in-group, query)
// pairs of one KV head, head-major, padded to 16 or 32. The 4 warps' states are
// combined in a fixed order; splits are merged by log-sum-exp in the CTA that
// arrives last for its KV head (dryft/engine/kernels/attention.py:200-210).
//
// PRO (decode prologue) variant: the CTA computes its query rows from the
// packed QKV row (per-head RMSNorm, bf16 x gain, rotate-half RoPE with the
// reference's bf16 roundings: dryft/engine/kernels/fused.py:9-30), and the CTA
// whose slice holds the newest position computes K/V for it, stores them in the
// cache and patches them into its staged tile. Because the cache up to the
// previous position is final before this launch's predecessor started, the
// producer streams it before griddepcontrol.wait.
#pragma once
#include "common.cuh"

namespace qb {

constexpr int kAttnD = 128;
constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = (kAttnWarps + 1) * 32;
constexpr int kAttnKeys = 16;
constexpr int kAttnSubTile = kAttnKeys * 128;        // [16 keys][64 dims] bf16 = 2 KB
constexpr int kAttnStageBytes = 4 * kAttnSubTile;    // K lo, K hi, V lo, V hi
constexpr int kAttnStages = 8;
constexpr int kAttnBarrierId = 2;
constexpr float kLog2e = 1.4426950408889634f;

struct AttnArgs {
  const bf16* qkv;       // PRO: packed row [Hq*D + 2*Hkv*D]
  const bf16* q;         // plain: [Q][Hq][D]
  const bf16* q_norm;
  const bf16* k_norm;
  const bf16* cos;       // [cap][D]
  const bf16* sin;
  float eps;
  const int64_t* pos;    // PRO: &position; plain: positions[Q]
  bf16* k_cache;         // [Hkv][cap][D] of this layer
  bf16* v_cache;
  bf16* out;             // [Q][Hq][D]
  float* part_o;         // [Hkv][S][ROWS][D]
  float* part_lse;       // [Hkv][S][ROWS]
  unsigned* counters;    // [Hkv]
  int* err;
  int Hq, Hkv, Q, cap, splits;
};

__host__ inline size_t attn_smem_bytes(int mt) {
  const int rows = 16 * mt;
  return 1024 + (size_t)kAttnStages * kAttnStageBytes + (size_t)rows * kAttnD * 2 + 2 * kAttnD * 2 +
         2 * kAttnStages * 8 + (size_t)kAttnWarps * rows * 2 * 4 + 64;
}

__device__ __forceinline__ void ldsm_x4(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_bf16_16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of (row, 16-byte chunk) inside a 128-byte-swizzled [rows][64 bf16] tile.
__device__ __forceinline__ int swz(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

// Per-head RMSNorm + rotate-half RoPE of one 128-dim head, one warp; lane owns
// dims [4*lane, 4*lane+4). Roundings follow dryft/engine/kernels/fused.py:9-30.
__device__ __forceinline__ void norm_rope_head(const bf16* src, const bf16* gain, const bf16* cos_row,
                                               const bf16* sin_row, float eps, int lane, bf16* dst_smem,
                                               bf16* dst_global) {
  const uint2 xv = *reinterpret_cast<const uint2*>(src + 4 * lane);
  const uint2 gv = *reinterpret_cast<const uint2*>(gain + 4 * lane);
  const uint2 cv = *reinterpret_cast<const uint2*>(cos_row + 4 * lane);
  const uint2 sv = *reinterpret_cast<const uint2*>(sin_row + 4 * lane);
  float x[4] = {bf_lo(xv.x), bf_hi(xv.x), bf_lo(xv.y), bf_hi(xv.y)};
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
}

template <int MT, bool PRO>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, const AttnArgs a) {
  constexpr int ROWS = 16 * MT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  bf16* qs = reinterpret_cast<bf16*>(ring + kAttnStages * kAttnStageBytes);  // [ROWS][128]
  bf16* kvnew = qs + ROWS * kAttnD;                                          // k_new[128], v_new[128]
  uint64_t* full = reinterpret_cast<uint64_t*>(kvnew + 2 * kAttnD);
  uint64_t* empty = full + kAttnStages;
  float* ml = reinterpret_cast<float*>(empty + kAttnStages);  // [warps][ROWS][2]
  volatile int* flags = reinterpret_cast<volatile int*>(ml + kAttnWarps * ROWS * 2);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int S = a.splits;
  const int kvh = blockIdx.x / S;
  const int split = blockIdx.x % S;
  const int G = a.Hq / a.Hkv;
  const int nrows = G * a.Q;

  if (tid == 0) {
    for (int s = 0; s < kAttnStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
    flags[0] = 0;
    flags[1] = 0;
  }
  __syncthreads();

  // Live key range. PRO reads the position before griddepcontrol.wait: it was
  // written by the previous step, two or more launches earlier.
  if (!PRO) {
    pdl_wait();
    pdl_trigger();
  }
  long long last = PRO ? a.pos[0] : a.pos[a.Q - 1];
  if (last < 0 || last >= a.cap) {
    if (tid == 0 && blockIdx.x == 0) report_error(a.err, DEV_BAD_POSITION);
    last = -1;
  }
  const int n = (int)last + 1;
  int per = (n + S - 1) / S;
  per = (per + kAttnKeys - 1) & ~(kAttnKeys - 1);
  const int k0 = min(n, split * per);
  const int k1 = min(n, k0 + per);
  const int nst = (k1 - k0 + kAttnKeys - 1) / kAttnKeys;

  if (warp == kAttnWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&tmk);
      prefetch_tensormap(&tmv);
      bool waited = !PRO;
      bool ok = true;
      int issued = 0;
      for (int c = 0; c < nst; ++c) {
        const int s = c % kAttnStages;
        if (c >= kAttnStages) {
          if (!waited) {
            pdl_wait();
            pdl_trigger();
            waited = true;
          }
          if (!mbar_wait(&empty[s], ((c / kAttnStages) - 1) & 1, a.err, DEV_TIMEOUT_ATTN_EMPTY)) {
            ok = false;
            break;
          }
        }
        uint8_t* st = ring + s * kAttnStageBytes;
        const int y = kvh * a.cap + k0 + c * kAttnKeys;
        mbar_arrive_expect_tx(&full[s], kAttnStageBytes);
        tma_load_2d(st, &tmk, 0, y, &full[s]);
        tma_load_2d(st + kAttnSubTile, &tmk, 64, y, &full[s]);
        tma_load_2d(st + 2 * kAttnSubTile, &tmv, 0, y, &full[s]);
        tma_load_2d(st + 3 * kAttnSubTile, &tmv, 64, y, &full[s]);
        issued = c + 1;
      }
      if (!waited) {
        pdl_wait();
        pdl_trigger();
      }
      if (!ok) {
        for (int c = (issued > kAttnStages ? issued - kAttnStages : 0); c < issued; ++c)
          mbar_wait(&full[c % kAttnStages], (c / kAttnStages) & 1, nullptr, 0);
      }
    } else if (PRO) {
      pdl_wait();
      pdl_trigger();
    }
    return;
  }

  // ---------------- consumers (128 threads) ----------------
  const int ctid = tid;
  if (PRO) {
    pdl_wait();
    pdl_trigger();
  }
  for (int i = ctid; i < ROWS * kAttnD / 8; i += kAttnWarps * 32)
    reinterpret_cast<uint4*>(qs)[i] = make_uint4(0, 0, 0, 0);
  named_barrier(kAttnBarrierId, kAttnWarps * 32);
  const bool owns_new = PRO && (k0 <= last) && (last < k1);
  if (PRO) {
    if (n > 0) {
      const bf16* cos_row = a.cos + (size_t)last * kAttnD;
      const bf16* sin_row = a.sin + (size_t)last * kAttnD;
      for (int g = warp; g < G; g += kAttnWarps)
        norm_rope_head(a.qkv + (size_t)(kvh * G + g) * kAttnD, a.q_norm, cos_row, sin_row, a.eps, lane,
                       qs + g * kAttnD, nullptr);
      if (owns_new) {
        const size_t slot = ((size_t)kvh * a.cap + last) * kAttnD;
        if (warp == kAttnWarps - 1) {
          norm_rope_head(a.qkv + (size_t)a.Hq * kAttnD + kvh * kAttnD, a.k_norm, cos_row, sin_row, a.eps, lane,
                         kvnew, a.k_cache + slot);
        } else if (warp == kAttnWarps - 2) {
          const uint2 v =
              *reinterpret_cast<const uint2*>(a.qkv + (size_t)(a.Hq + a.Hkv) * kAttnD + kvh * kAttnD + 4 * lane);
          *reinterpret_cast<uint2*>(kvnew + kAttnD + 4 * lane) = v;
          *reinterpret_cast<uint2*>(a.v_cache + slot + 4 * lane) = v;
        }
      }
    }
  } else {
    for (int r = warp; r < nrows; r += kAttnWarps) {
      const int g = r / a.Q, qi = r % a.Q;
      const uint2 v = *reinterpret_cast<const uint2*>(a.q + ((size_t)qi * a.Hq + kvh * G + g) * kAttnD + 4 * lane);
      *reinterpret_cast<uint2*>(qs + r * kAttnD + 4 * lane) = v;
    }
  }
  named_barrier(kAttnBarrierId, kAttnWarps * 32);

  // Query fragments (A operand, row-major [ROWS][128]).
  uint32_t qa[MT][8][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int row = mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int col = ks * 16 + (lane >> 4) * 8;
      ldsm_x4(qa[mt][ks], qs + row * kAttnD + col);
    }

  const int g4 = lane >> 2;  // fragment row within an 8-row half
  const int t4 = lane & 3;
  int lim[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + g4 + h * 8;
      if (r >= nrows) lim[mt][h] = -1;
      else if (PRO) lim[mt][h] = (int)last;
      else lim[mt][h] = (int)a.pos[r % a.Q];
    }

  float o[MT][16][4];
  float m[MT][2], l[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int j = 0; j < 16; ++j) o[mt][j][0] = o[mt][j][1] = o[mt][j][2] = o[mt][j][3] = 0.f;
    m[mt][0] = m[mt][1] = -INFINITY;
    l[mt][0] = l[mt][1] = 0.f;
  }
  // log2(e) / sqrt(128), folded in double precision as the reference does.
  const float scale = 0.12751743082459868f;

  bool ok = true;
  for (int c = warp; c < nst; c += kAttnWarps) {
    const int s = c % kAttnStages;
    if (!mbar_wait(&full[s], (c / kAttnStages) & 1, a.err, DEV_TIMEOUT_ATTN_FULL)) {
      ok = false;
      break;
    }
    uint8_t* st = ring + s * kAttnStageBytes;
    const int kb = k0 + c * kAttnKeys;
    if (owns_new && kb <= last && last < kb + kAttnKeys) {
      const int kr = (int)last - kb;
      const int which = lane >> 3, ch = lane & 7;
      *reinterpret_cast<uint4*>(st + which * kAttnSubTile + swz(kr, ch)) =
          *reinterpret_cast<const uint4*>(kvnew + (which >> 1) * kAttnD + (which & 1) * 64 + ch * 8);
    }
    const int valid = k1 - kb;
    if (valid < kAttnKeys) {
      // Slots past the live range may hold anything (even NaN); P is 0 there,
      // but 0 * NaN is NaN, so clear those V rows.
      for (int i = lane; i < (kAttnKeys - valid) * 16; i += 32) {
        const int row = valid + (i >> 4);
        const int sub = (i >> 3) & 1, ch = i & 7;
        *reinterpret_cast<uint4*>(st + (2 + sub) * kAttnSubTile + swz(row, ch)) = make_uint4(0, 0, 0, 0);
      }
    }
    __syncwarp();

    float sc[MT][2][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) sc[mt][nt][0] = sc[mt][nt][1] = sc[mt][nt][2] = sc[mt][nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int mi = lane >> 3;
      const int key = (lane & 7) + (mi >> 1) * 8;
      const int ch = ((ks & 3) << 1) + (mi & 1);
      uint32_t b[4];
      ldsm_x4(b, st + (ks >> 2) * kAttnSubTile + swz(key, ch));
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        mma_bf16_16816(sc[mt][0], qa[mt][ks], b[0], b[1]);
        mma_bf16_16816(sc[mt][1], qa[mt][ks], b[2], b[3]);
      }
    }

    uint32_t pa[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v[4];
        bool vis[4];
        float rmax = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = kb + nt * 8 + 2 * t4 + e;
            const bool vv = (key <= lim[mt][h]) && (key < k1);
            const float x = sc[mt][nt][h * 2 + e] * scale;
            vis[nt * 2 + e] = vv;
            v[nt * 2 + e] = vv ? x : -INFINITY;
            rmax = fmaxf(rmax, v[nt * 2 + e]);
          }
        rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 1));
        rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 2));
        const float mnew = fmaxf(m[mt][h], rmax);
        const float corr = (m[mt][h] == -INFINITY) ? 0.f : exp2f(m[mt][h] - mnew);
        float p[4], rsum = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          p[i] = vis[i] ? exp2f(v[i] - mnew) : 0.f;
          rsum += p[i];
        }
        rsum += __shfl_xor_sync(0xffffffffu, rsum, 1);
        rsum += __shfl_xor_sync(0xffffffffu, rsum, 2);
        l[mt][h] = l[mt][h] * corr + rsum;
        m[mt][h] = mnew;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          o[mt][j][h * 2] *= corr;
          o[mt][j][h * 2 + 1] *= corr;
        }
        // A fragment of P: reg h -> (row g4 + 8h, keys 2t..2t+1), reg 2+h -> keys 8+2t..
        pa[mt][h] = pack_bf16(p[0], p[1]);
        pa[mt][2 + h] = pack_bf16(p[2], p[3]);
      }
    }

#pragma unroll
    for (int dp = 0; dp < 8; ++dp) {
      const int mi = lane >> 3;
      const int key = (lane & 7) + (mi & 1) * 8;
      const int dch = dp * 2 + (mi >> 1);
      uint32_t b[4];
      ldsm_x4_t(b, st + (2 + (dch >> 3)) * kAttnSubTile + swz(key, dch & 7));
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        mma_bf16_16816(o[mt][2 * dp], pa[mt], b[0], b[1]);
        mma_bf16_16816(o[mt][2 * dp + 1], pa[mt], b[2], b[3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (!ok && lane == 0) flags[0] = 1;
  named_barrier(kAttnBarrierId, kAttnWarps * 32);
  if (flags[0] != 0) return;

  // Combine the four warps (fixed order) through the drained ring.
  float* ob = reinterpret_cast<float*>(ring);  // [warps][ROWS][128]
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + g4 + h * 8;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float2 v = make_float2(o[mt][j][h * 2], o[mt][j][h * 2 + 1]);
        *reinterpret_cast<float2*>(ob + ((size_t)warp * ROWS + r) * kAttnD + j * 8 + 2 * t4) = v;
      }
      if (t4 == 0) {
        ml[(warp * ROWS + r) * 2] = m[mt][h];
        ml[(warp * ROWS + r) * 2 + 1] = l[mt][h];
      }
    }
  named_barrier(kAttnBarrierId, kAttnWarps * 32);
  const int d = ctid;  // one head dim per thread
  for (int r = 0; r < nrows; ++r) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, ml[(w * ROWS + r) * 2]);
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float mw = ml[(w * ROWS + r) * 2];
      const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      L += ml[(w * ROWS + r) * 2 + 1] * f;
      acc += ob[((size_t)w * ROWS + r) * kAttnD + d] * f;
    }
    const float val = L > 0.f ? acc / L : 0.f;
    const float lse = L > 0.f ? M + log2f(L) : -INFINITY;
    const int g = r / a.Q, qi = r % a.Q;
    if (S == 1) {
      a.out[((size_t)qi * a.Hq + kvh * G + g) * kAttnD + d] = __float2bfloat16_rn(val);
    } else {
      const size_t idx = ((size_t)kvh * S + split) * ROWS + r;
      a.part_o[idx * kAttnD + d] = val;
      if (d == 0) a.part_lse[idx] = lse;
    }
  }
  if (S == 1) return;

  // The CTA that completes its KV head merges the S slices.
  __threadfence();
  named_barrier(kAttnBarrierId, kAttnWarps * 32);
  if (ctid == 0) {
    const unsigned ticket = atomicAdd(&a.counters[kvh], 1u);
    flags[1] = (ticket == (unsigned)(S - 1)) ? 1 : 0;
  }
  named_barrier(kAttnBarrierId, kAttnWarps * 32);
  if (flags[1] == 0) return;
  __threadfence();
  // Merge weights exp2(lse_s - max) / sum, as dryft/engine/kernels/attention.py:204-206.
  // All LSEs are loaded at once (independent loads), each row's weights are
  // computed once, then every (row, dim) output sums its S partials in split order.
  float* wts = reinterpret_cast<float*>(ring);  // [nrows][S]; the ring is free now
  for (int i = ctid; i < nrows * S; i += kAttnWarps * 32) {
    const int r = i / S, sp = i - r * S;
    wts[i] = __ldcg(a.part_lse + ((size_t)kvh * S + sp) * ROWS + r);
  }
  named_barrier(kAttnBarrierId, kAttnWarps * 32);
  if (ctid < nrows) {
    float* wr = wts + ctid * S;
    float mx = -INFINITY;
    for (int sp = 0; sp < S; ++sp) mx = fmaxf(mx, wr[sp]);
    float wsum = 0.f;
    for (int sp = 0; sp < S; ++sp) wsum += exp2f(wr[sp] - mx);
    for (int sp = 0; sp < S; ++sp) wr[sp] = exp2f(wr[sp] - mx) / wsum;
  }
  named_barrier(kAttnBarrierId, kAttnWarps * 32);
  for (int r = 0; r < nrows; ++r) {
    const float* wr = wts + r * S;
    const float* po = a.part_o + ((size_t)kvh * S * ROWS + r) * kAttnD + d;
    float acc = 0.f;
    int sp = 0;
    for (; sp + 4 <= S; sp += 4) {
      const float p0 = __ldcg(po + (size_t)(sp + 0) * ROWS * kAttnD);
      const float p1 = __ldcg(po + (size_t)(sp + 1) * ROWS * kAttnD);
      const float p2 = __ldcg(po + (size_t)(sp + 2) * ROWS * kAttnD);
      const float p3 = __ldcg(po + (size_t)(sp + 3) * ROWS * kAttnD);
      acc += p0 * wr[sp];
      acc += p1 * wr[sp + 1];
      acc += p2 * wr[sp + 2];
      acc += p3 * wr[sp + 3];
    }
    for (; sp < S; ++sp) acc += __ldcg(po + (size_t)sp * ROWS * kAttnD) * wr[sp];
    const int g = r / a.Q, qi = r % a.Q;
    a.out[((size_t)qi * a.Hq + kvh * G + g) * kAttnD + d] = __float2bfloat16_rn(acc);
  }
  if (ctid == 0) a.counters[kvh] = 0u;
}

}  // namespace qb
