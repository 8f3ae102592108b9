// attention.cuh — split-KV grouped-query decode attention for sm_100a.
//
// Grid = Hkv x S CTAs; CTA (h, s) owns KV head h and the s-th of S equal,
// 16-aligned slices of the live key range [0, last_position]. Split sizes are
// computed on the device from the live position, so one captured launch stays
// balanced as the context grows.
//
// Per CTA: one producer lane streams 64-key stages of K and V with 2D TMA tensor
// loads ([64 keys][64 dims] boxes of 8 KB, 128-byte swizzle, no multicast) into
// a 4-stage ring; 4 consumer warps take stages round-robin and, 16 keys at a
// time, run
// S = Q.K^T and O += P.V on mma.sync m16n8k16 (bf16 in, fp32 accumulate) with a
// base-2 online softmax; P is rounded to bf16 before the P.V product and the
// softmax denominator sums the unrounded fp32 P, as the reference kernel does
// (dryft/engine/kernels/attention.py:49-57). Rows are (head-in-group, query)
// pairs of one KV head, head-major, padded to 16 or 32. The 4 warps' states are
// combined in a fixed order; splits are merged by log-sum-exp
// (dryft/engine/kernels/attention.py:200-210) through global memory in the CTA
// that arrives last for its KV head (attn_kernel). Batch-one decode has its own
// cluster kernel (decode_attention.cuh), which reuses the helpers below.
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
constexpr int kAttnKeys = 64;                        // keys per stage (one TMA box row count)
constexpr int kAttnSub = 16;                         // keys per mma sub-block
constexpr int kAttnSubTile = kAttnKeys * 128;        // [64 keys][64 dims] bf16 = 8 KB
constexpr int kAttnStageBytes = 4 * kAttnSubTile;    // K lo, K hi, V lo, V hi = 32 KB
constexpr int kAttnStages = 4;
// Warp w consumes stages w, w+4, ...; a ring slot must always be consumed by
// the same warp, so that warp observes every phase of the slot's mbarrier
// (a parity wait on a phase two steps ahead would pass immediately).
static_assert(kAttnStages % kAttnWarps == 0, "each ring slot must map to one consumer warp");
constexpr int kAttnBarrierId = 2;
constexpr int kAttnMinSplitKeys = 256;
constexpr float kLog2e = 1.4426950408889634f;

// Split length for n live keys over at most `want` splits (16-aligned), and
// the number of splits that receive keys: rounding the length up can leave the
// last of `want` splits empty, and those are dropped, so every split below the
// returned count has k0 = split * per < n (merges never see an empty split).
__device__ __forceinline__ int2 attn_split_len(int n, int want) {
  int per = (n + max(1, want) - 1) / max(1, want);
  per = (per + kAttnSub - 1) & ~(kAttnSub - 1);
  return make_int2(per, per > 0 ? max(1, (n + per - 1) / per) : 1);
}

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
  int clusters;          // decode cluster kernel: clusters per KV head (<= 1: one)
  int part_splits;       // decode cluster kernel: second extent of part_o / part_lse
  unsigned* tickets;     // decode cluster kernel: [Hkv][splits] cross-cluster merge tickets
  int batch_hkv;         // rows kernel, batched decode: KV heads per sequence (KV head h of the
                         // launch belongs to sequence h / batch_hkv, whose position is pos[h / batch_hkv]);
                         // 0: one sequence, pos[i] is query i's position
  unsigned long long* trace;  // decode cluster kernel: this launch's trace records (common.cuh), or NULL
  int multi_keys;             // decode cluster kernel: live keys from which a KV head uses all its
                              // clusters (0: kDecMultiClusterKeys)
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

// Cluster helpers (thread-block clusters, distributed shared memory).
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Full-cluster barrier; every thread of every CTA in the cluster must execute it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_shared_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

struct AttnSmem {
  uint8_t* ring;
  bf16* qs;
  bf16* kvnew;
  uint64_t* full;
  uint64_t* empty;
  float* ml;
  volatile int* flags;
};

template <int MT>
__device__ __forceinline__ AttnSmem attn_carve(uint8_t* smem_raw) {
  constexpr int ROWS = 16 * MT;
  AttnSmem m;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  m.ring = smem;
  m.qs = reinterpret_cast<bf16*>(m.ring + kAttnStages * kAttnStageBytes);  // [ROWS][128]
  m.kvnew = m.qs + ROWS * kAttnD;                                          // k_new[128], v_new[128]
  m.full = reinterpret_cast<uint64_t*>(m.kvnew + 2 * kAttnD);
  m.empty = m.full + kAttnStages;
  m.ml = reinterpret_cast<float*>(m.empty + kAttnStages);  // [warps][ROWS][2]
  m.flags = reinterpret_cast<volatile int*>(m.ml + kAttnWarps * ROWS * 2);
  return m;
}

// Producer lane: stream stages [0, nst) of keys [k0, k1) of KV head kvh.
template <bool PRO>
__device__ __forceinline__ void attn_produce(const CUtensorMap* tmk, const CUtensorMap* tmv, const AttnArgs& a,
                                             const AttnSmem& sm, int kvh, int k0, int nst) {
  prefetch_tensormap(tmk);
  prefetch_tensormap(tmv);
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
      if (!mbar_wait(&sm.empty[s], ((c / kAttnStages) - 1) & 1, a.err, DEV_TIMEOUT_ATTN_EMPTY)) {
        ok = false;
        break;
      }
    }
    uint8_t* st = sm.ring + s * kAttnStageBytes;
    const int y = kvh * a.cap + k0 + c * kAttnKeys;
    mbar_arrive_expect_tx(&sm.full[s], kAttnStageBytes);
    tma_load_2d(st, tmk, 0, y, &sm.full[s]);
    tma_load_2d(st + kAttnSubTile, tmk, 64, y, &sm.full[s]);
    tma_load_2d(st + 2 * kAttnSubTile, tmv, 0, y, &sm.full[s]);
    tma_load_2d(st + 3 * kAttnSubTile, tmv, 64, y, &sm.full[s]);
    issued = c + 1;
  }
  if (!waited) {
    pdl_wait();
    pdl_trigger();
  }
  if (!ok) {
    // Keep shared memory alive until the copies already in flight land.
    for (int c = (issued > kAttnStages ? issued - kAttnStages : 0); c < issued; ++c)
      mbar_wait(&sm.full[c % kAttnStages], (c / kAttnStages) & 1, nullptr, 0);
  }
}

// Consumers: build the query rows (PRO: norm + RoPE + KV append), stream the
// stages, and combine the 4 warps. On return thread d (< 128) holds, for every
// row r < nrows, the split's normalised output val[r] and its log-sum-exp
// lse[r]. Returns false if a bounded wait gave up (CTA-uniform).
template <int MT, bool PRO>
__device__ __forceinline__ bool attn_consume(const AttnArgs& a, const AttnSmem& sm, int kvh, long long last, int n,
                                             int k0, int k1, int nst, float (&val)[16 * MT],
                                             float (&lsev)[16 * MT]) {
  constexpr int ROWS = 16 * MT;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int ctid = tid;
  const int G = a.Hq / a.Hkv;
  const int nrows = G * a.Q;
  uint8_t* ring = sm.ring;
  bf16* qs = sm.qs;
  bf16* kvnew = sm.kvnew;
  float* ml = sm.ml;

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
    if (!mbar_wait(&sm.full[s], (c / kAttnStages) & 1, a.err, DEV_TIMEOUT_ATTN_FULL)) {
      ok = false;
      break;
    }
    uint8_t* stage = ring + s * kAttnStageBytes;
    const int kstage = k0 + c * kAttnKeys;
    if (owns_new && kstage <= last && last < kstage + kAttnKeys) {
      const int kr = (int)last - kstage;
      const int which = lane >> 3, ch = lane & 7;
      *reinterpret_cast<uint4*>(stage + which * kAttnSubTile + swz(kr, ch)) =
          *reinterpret_cast<const uint4*>(kvnew + (which >> 1) * kAttnD + (which & 1) * 64 + ch * 8);
    }
    const int svalid = k1 - kstage;
    if (svalid < kAttnKeys) {
      // Slots past the live range may hold anything (even NaN); P is 0 there,
      // but 0 * NaN is NaN, so clear those V rows.
      for (int i = lane; i < (kAttnKeys - svalid) * 16; i += 32) {
        const int row = svalid + (i >> 4);
        const int sub = (i >> 3) & 1, ch = i & 7;
        *reinterpret_cast<uint4*>(stage + (2 + sub) * kAttnSubTile + swz(row, ch)) = make_uint4(0, 0, 0, 0);
      }
    }
    __syncwarp();
    for (int sb = 0; sb < kAttnKeys / kAttnSub && kstage + sb * kAttnSub < k1; ++sb) {
    uint8_t* st = stage + sb * kAttnSub * 128;  // 16-row block inside each sub-tile
    const int kb = kstage + sb * kAttnSub;
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
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[s]);
  }
  if (!ok && lane == 0) sm.flags[0] = 1;
  named_barrier(kAttnBarrierId, kAttnWarps * 32);
  if (sm.flags[0] != 0) return false;

  // Combine the four warps (fixed order) through the drained ring.
  constexpr int kObStride = kAttnD + 4;  // padded row: no bank conflicts on the fragment stores
  float* ob = reinterpret_cast<float*>(ring);  // [warps][ROWS][kObStride]
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + g4 + h * 8;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float2 v = make_float2(o[mt][j][h * 2], o[mt][j][h * 2 + 1]);
        *reinterpret_cast<float2*>(ob + ((size_t)warp * ROWS + r) * kObStride + j * 8 + 2 * t4) = v;
      }
      if (t4 == 0) {
        ml[(warp * ROWS + r) * 2] = m[mt][h];
        ml[(warp * ROWS + r) * 2 + 1] = l[mt][h];
      }
    }
  named_barrier(kAttnBarrierId, kAttnWarps * 32);
  const int d = ctid;  // one head dim per thread
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    val[r] = 0.f;
    lsev[r] = -INFINITY;
    if (r < nrows) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, ml[(w * ROWS + r) * 2]);
      float L = 0.f, acc = 0.f;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float mw = ml[(w * ROWS + r) * 2];
        const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
        L += ml[(w * ROWS + r) * 2 + 1] * f;
        acc += ob[((size_t)w * ROWS + r) * kObStride + d] * f;
      }
      val[r] = L > 0.f ? acc / L : 0.f;
      lsev[r] = L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
  return true;
}

// Setup shared by both kernels: barriers, the live key range and this CTA's slice.
struct AttnRange {
  long long last;
  int n, Se, k0, k1, nst;
};

template <int MT>
__device__ __forceinline__ AttnRange attn_setup(const AttnArgs& a, const AttnSmem& sm, int split, bool pro) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < kAttnStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    fence_mbar_init();
    sm.flags[0] = 0;
    sm.flags[1] = 0;
  }
  __syncthreads();
  // Live key range. The decode prologue variant reads the position before
  // griddepcontrol.wait: it was written by the previous step, two or more
  // launches earlier.
  if (!pro) {
    pdl_wait();
    pdl_trigger();
  }
  AttnRange R;
  long long last = pro ? a.pos[0] : a.pos[a.Q - 1];
  if (last < 0 || last >= a.cap) {
    if (tid == 0 && blockIdx.x == 0) report_error(a.err, DEV_BAD_POSITION);
    last = -1;
  }
  R.last = last;
  R.n = (int)last + 1;
  // Splits actually used: about kAttnMinSplitKeys keys each, at most the
  // grid's split count. Short contexts then need no merge at all.
  const int2 sl = attn_split_len(R.n, min(a.splits, (R.n + kAttnMinSplitKeys - 1) / kAttnMinSplitKeys));
  const int per = sl.x;
  R.Se = sl.y;
  R.k0 = min(R.n, split * per);
  R.k1 = min(R.n, R.k0 + per);
  R.nst = (R.k1 - R.k0 + kAttnKeys - 1) / kAttnKeys;
  return R;
}

__device__ __forceinline__ void attn_store_out(const AttnArgs& a, int kvh, int r, int d, float v) {
  const int G = a.Hq / a.Hkv;
  const int g = r / a.Q, qi = r % a.Q;
  a.out[((size_t)qi * a.Hq + kvh * G + g) * kAttnD + d] = __float2bfloat16_rn(v);
}

// Split-KV attention with the splits merged through global memory by the CTA
// that arrives last for its KV head (any query count, either prologue mode).
template <int MT, bool PRO>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, const AttnArgs a) {
  constexpr int ROWS = 16 * MT;
  extern __shared__ uint8_t smem_raw[];
  const AttnSmem sm = attn_carve<MT>(smem_raw);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int S = a.splits;
  const int kvh = blockIdx.x / S;
  const int split = blockIdx.x % S;
  const int nrows = (a.Hq / a.Hkv) * a.Q;
  const AttnRange R = attn_setup<MT>(a, sm, split, PRO);
  const int Se = R.Se;
  if (split >= Se) return;  // surplus CTA: no loads, no partials, not counted

  if (warp == kAttnWarps) {
    if ((tid & 31) == 0) attn_produce<PRO>(&tmk, &tmv, a, sm, kvh, R.k0, R.nst);
    else if (PRO) {
      pdl_wait();
      pdl_trigger();
    }
    return;
  }
  float val[ROWS], lsev[ROWS];
  if (!attn_consume<MT, PRO>(a, sm, kvh, R.last, R.n, R.k0, R.k1, R.nst, val, lsev)) return;
  const int ctid = tid, d = tid;
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    if (r < nrows) {
      if (Se == 1) {
        attn_store_out(a, kvh, r, d, val[r]);
      } else {
        const size_t idx = ((size_t)kvh * S + split) * ROWS + r;
        a.part_o[idx * kAttnD + d] = val[r];
        if (d == 0) a.part_lse[idx] = lsev[r];
      }
    }
  }
  if (Se == 1) return;

  // The CTA that completes its KV head merges the Se slices.
  named_barrier(kAttnBarrierId, kAttnWarps * 32);
  if (ctid == 0) {
    const unsigned ticket = atomic_add_acq_rel_gpu(&a.counters[kvh], 1u);
    sm.flags[1] = (ticket == (unsigned)(Se - 1)) ? 1 : 0;
  }
  named_barrier(kAttnBarrierId, kAttnWarps * 32);
  if (sm.flags[1] == 0) return;
  // Merge by log-sum-exp: weight_s = exp2(lse_s - max) / sum_s exp2(lse_s - max)
  // as dryft/engine/kernels/attention.py:204-206, with the division applied
  // once after the weighted sum. Each thread owns one head dim; per batch of up
  // to 8 splits x 4 rows the log-sum-exps and partials are loaded in a single
  // round (indices clamped into the written range, extra terms dropped), and
  // batches combine with a running max.
  for (int r0 = 0; r0 < nrows; r0 += 4) {
    float acc[4], den[4], mx[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) { acc[j] = 0.f; den[j] = 0.f; mx[j] = -INFINITY; }
    for (int sp0 = 0; sp0 < Se; sp0 += 8) {
      float v[8][4], lv[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const size_t idx = ((size_t)kvh * S + min(sp0 + i, Se - 1)) * ROWS + min(r0 + j, nrows - 1);
          lv[i][j] = __ldcg(a.part_lse + idx);
          v[i][j] = __ldcg(a.part_o + idx * kAttnD + d);
        }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float bm = mx[j];
#pragma unroll
        for (int i = 0; i < 8; ++i) bm = (sp0 + i < Se) ? fmaxf(bm, lv[i][j]) : bm;
        const float corr = (mx[j] == -INFINITY) ? 0.f : exp2f(mx[j] - bm);
        acc[j] *= corr;
        den[j] *= corr;
        mx[j] = bm;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float w = (sp0 + i < Se) ? exp2f(lv[i][j] - bm) : 0.f;
          den[j] += w;
          acc[j] = fmaf(v[i][j], w, acc[j]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (r0 + j < nrows) attn_store_out(a, kvh, r0 + j, d, acc[j] / den[j]);
  }
  if (ctid == 0) a.counters[kvh] = 0u;
}

}  // namespace qb
