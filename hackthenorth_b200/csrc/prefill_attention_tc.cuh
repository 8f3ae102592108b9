// prefill_attention_tc.cuh — causal GQA flash attention for a block of prompt
// rows on sm_100a's tcgen05 tensor cores (the prefill attention).
//
// The reference runs prompt attention through SDPA's flash kernel with a
// causal mask (dryft/engine/attention.py:92-98); this kernel keeps the decode
// path's numerics (dryft/engine/kernels/attention.py:49-57): scores
// scaled by 1/sqrt(128) in base 2, masked to keys <= the row's position, fp32
// softmax statistics, P rounded to bf16 before P.V, fp32 accumulation, one
// bf16 rounding of O / l. The running maximum is kept lazily: O and l are
// rescaled only when a row's maximum grows by more than 8 (P then stays below
// 2^8), which changes P's rounding point but not its relative precision.
//
// CTA = (256 / G prompt rows, KV head g) (1D grid, the longest causal row
// blocks first): its 256 query rows (each prompt row
// with the G query heads of g, in two M = 128 tiles) share one stream of g's
// keys and values, so every K/V byte is fetched once per 256 query rows.
//  * warp 0, one lane: TMA. Q tiles [prompt rows][G heads][64 dims] x 2 halves
//    through a 3D map (128-byte swizzle); then 64-key stages of K lo/hi and V
//    lo/hi ([64 keys][64 dims] boxes) into a 3-slot ring.
//  * warp 1: owns 512 TMEM columns; one lane issues, per key tile j and M tile
//    t, S_t = Q_t . K_j^T (M 128, N 64, K-major operands) into TMEM columns
//    64t.., and once the softmax warps have written P_t, O_t += P_t . V_j
//    (M 128, N 128; V read as an MN-major operand straight from the cache
//    tile) into columns 128 + 128t.. The two tiles alternate, so one tile's
//    softmax runs under the other tile's MMAs.
//  * warps 2-5 (tile 0) and 6-9 (tile 1): thread = one query row. Reads its 64
//    scores from TMEM (tcgen05.ld), masks, updates max/sum, writes P (bf16) to
//    shared memory in the MMA's swizzled layout, rescales O in TMEM when
//    needed, and finally writes O / l.
// Every wait is bounded; on failure the kernel records an error, stops issuing
// and releases TMEM after its MMAs have completed.
#pragma once
#include "prefill_gemm.cuh"
#include "verify_attention.cuh"

namespace qb {

constexpr int kFtRowsQ = 256;                  // query rows per CTA (two M = 128 tiles)
constexpr int kFtKeys = 64;                    // keys per stage
constexpr int kFtStages = 3;
constexpr int kFtThreads = 10 * 32;
constexpr int kFtQTile = 128 * 128 * 2;        // one M tile of Q: [128 rows][128 dims], 32 KB
constexpr int kFtKvStage = 4 * 64 * 128;       // K lo, K hi, V lo, V hi: 32 KB
constexpr int kFtPTile = 128 * 64 * 2;         // P of one M tile: [128 rows][64 keys], 16 KB

struct FtArgs {
  bf16* out;        // [T][Hq][128]
  int T, p0, Hq, Hkv, cap;
  int* err;
};

__host__ __device__ inline size_t ft_smem_bytes() {
  return 1024 + 2 * (size_t)kFtQTile + (size_t)kFtStages * kFtKvStage + 2 * (size_t)kFtPTile + 512;
}

// Shared-memory descriptor with explicit leading and stride byte offsets
// (128-byte swizzle; K-major: sbo = stride between 8-row groups; MN-major:
// lbo = stride between 64-element column blocks, sbo = stride between 8-row
// groups along K).
__device__ __forceinline__ uint64_t ft_desc(const void* smem_tile, uint32_t lbo, uint32_t sbo) {
  const uint64_t addr = smem_u32(smem_tile);
  return ((addr >> 4) & 0x3FFFull) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) | ((uint64_t)(sbo >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

// 2^x with the MUFU's approximate base-2 exponential (relative error about
// 2^-22; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// 64 consecutive fp32 columns of this warp's 32 TMEM lanes, one load and one wait.
__device__ __forceinline__ void tc_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, "
      "%38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, "
      "%60, %61, %62, %63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]),
        "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]),
        "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]),
        "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]),
        "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tc_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kFtThreads, 1)
    flash_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                            const __grid_constant__ CUtensorMap tmv, const FtArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* qs = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = qs + 2 * kFtQTile;               // [3] stages: K lo, K hi, V lo, V hi
  uint8_t* ps = ring + kFtStages * kFtKvStage;     // [2] P tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(ps + 2 * kFtPTile);
  uint64_t* kv_full = bars;        // [3]
  uint64_t* kv_empty = bars + 3;   // [3]
  uint64_t* q_full = bars + 6;
  uint64_t* s_full = bars + 7;     // [2] S_t computed
  uint64_t* p_full = bars + 11;    // [2] P_t written by the tile's 4 softmax warps
  uint64_t* o_done = bars + 13;    // [2] O_t += P_t . V complete
  uint64_t* done = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = a.Hq / a.Hkv;
  const int RH = (kFtRowsQ / G) / 2;  // prompt rows per M tile
  // Grid = row blocks x KV heads, row blocks in descending order (KV head
  // fastest): the causal blocks with the most keys start first and the short
  // ones fill the last wave.
  const int g = blockIdx.x % a.Hkv;
  const int nrb = gridDim.x / a.Hkv;
  const int r0 = (nrb - 1 - (int)(blockIdx.x / a.Hkv)) * 2 * RH;
  int nkb[2], pm[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int first = r0 + t * RH;
    if (first < a.T) {
      pm[t] = a.p0 + min(first + RH, a.T) - 1;  // largest position of the tile's rows
      nkb[t] = pm[t] / kFtKeys + 1;
    } else {
      pm[t] = -1;
      nkb[t] = 0;
    }
  }
  const int nk = max(nkb[0], nkb[1]);
  const int pmax = max(pm[0], pm[1]);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFtStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(q_full, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_done[t], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
    flags[0] = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // q and the prompt rows' K/V come from the previous kernel
  pdl_trigger();

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensormap(&tmq);
      prefetch_tensormap(&tmk);
      prefetch_tensormap(&tmv);
      const int nq = nkb[1] > 0 ? 2 : 1;
      mbar_arrive_expect_tx(q_full, (uint32_t)nq * kFtQTile);
      for (int t = 0; t < nq; ++t)
        for (int h = 0; h < 2; ++h)
          tma_load_3d(qs + t * kFtQTile + h * (kFtQTile / 2), &tmq, 64 * h, g * G, r0 + t * RH, q_full);
      int issued = 0;
      for (int j = 0; j < nk; ++j) {
        const int s = j % kFtStages;
        if (j >= kFtStages && !mbar_wait(&kv_empty[s], ((j / kFtStages) - 1) & 1, a.err, DEV_TIMEOUT_ATTN_EMPTY)) {
          flags[0] = 1;
          break;
        }
        uint8_t* st = ring + s * kFtKvStage;
        const int y = g * a.cap + j * kFtKeys;
        mbar_arrive_expect_tx(&kv_full[s], kFtKvStage);
        tma_load_2d(st, &tmk, 0, y, &kv_full[s]);
        tma_load_2d(st + kFtKvStage / 4, &tmk, 64, y, &kv_full[s]);
        tma_load_2d(st + kFtKvStage / 2, &tmv, 0, y, &kv_full[s]);
        tma_load_2d(st + 3 * (kFtKvStage / 4), &tmv, 64, y, &kv_full[s]);
        issued = j + 1;
      }
      // keep shared memory alive until every issued copy has landed
      mbar_wait(q_full, 0, nullptr, 0);
      for (int j = (issued > kFtStages ? issued - kFtStages : 0); j < issued; ++j)
        mbar_wait(&kv_full[j % kFtStages], (j / kFtStages) & 1, nullptr, 0);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    // Order: S_0(0) S_1(0) | PV_0(0) S_0(1) PV_1(0) S_1(1) | PV_0(1) S_0(2) ...:
    // S_t(j+1) is issued right after PV_t(j) (the tile's softmax has read S_t(j)
    // before it wrote P_t(j)), so each tile's softmax runs under the other
    // tile's MMAs.
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, a.err, DEV_TIMEOUT_ATTN_FULL) &&
                mbar_wait(&kv_full[0], 0, a.err, DEV_TIMEOUT_ATTN_FULL);
      const uint32_t idesc_s = pg_idesc(128, kFtKeys);
      const uint32_t idesc_o = pg_idesc(128, 128) | (1u << 16);  // B (V) MN-major
      auto issue_s = [&](int t, const uint8_t* st) {  // S_t = Q_t . K^T: 8 K steps of 16 dims
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint64_t ad = ft_desc(qs + t * kFtQTile + (k >> 2) * (kFtQTile / 2), 16, 1024) + (uint64_t)((k & 3) * 2);
          const uint64_t bd = ft_desc(st + (k >> 2) * (kFtKvStage / 4), 16, 1024) + (uint64_t)((k & 3) * 2);
          tc_mma(tmem + (uint32_t)(t * kFtKeys), ad, bd, idesc_s, k > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[t]);
      };
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < 2; ++t)
          if (nkb[t] > 0) issue_s(t, ring);
      }
      for (int j = 0; j < nk && ok; ++j) {
        const int s = j % kFtStages, s1 = (j + 1) % kFtStages;
        const uint8_t* st = ring + s * kFtKvStage;
        bool next_ready = false;
        for (int t = 0; t < 2 && ok; ++t) {
          if (j >= nkb[t]) continue;
          // O_t += P_t . V_j: 4 K steps of 16 keys
          if (!mbar_wait(&p_full[t], j & 1, a.err, DEV_TIMEOUT_ATTN_FULL) || flags[0] != 0) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = ft_desc(ps + t * kFtPTile, 16, 1024) + (uint64_t)(k * 2);
            const uint64_t bd = ft_desc(st + kFtKvStage / 2 + k * 2048, kFtKvStage / 4, 1024);
            tc_mma(tmem + (uint32_t)(128 + 128 * t), ad, bd, idesc_o, (j > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&o_done[t]);
          if (j + 1 < nkb[t]) {
            if (!next_ready) {
              if (!mbar_wait(&kv_full[s1], ((j + 1) / kFtStages) & 1, a.err, DEV_TIMEOUT_ATTN_FULL)) {
                ok = false;
                break;
              }
              tc_fence_after();
              next_ready = true;
            }
            issue_s(t, ring + s1 * kFtKvStage);
          }
        }
        if (!ok) break;
        tc_commit(&kv_empty[s]);  // every MMA reading stage s has been issued
      }
      if (!ok) flags[0] = 1;
      tc_commit(done);  // TMEM is released below only after every MMA issued here has completed
      mbar_wait(done, 0, nullptr, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------- softmax / output
    const int t = (warp - 2) >> 2;  // M tile of this warp
    const int quarter = warp & 3;   // TMEM lanes 32 quarter .. +31
    const int qrow = quarter * 32 + lane;
    const int qi = qrow / G, hj = qrow - qi * G;
    const int pr = r0 + t * RH + qi;  // prompt row of this thread's query row
    const bool valid = pr < a.T;
    const long long pos = valid ? (long long)a.p0 + pr : -1;
    const uint32_t lanebase = (uint32_t)(quarter * 32) << 16;
    const uint32_t o_col = 128 + 128 * t;
    const float scale = 0.12751743082459868f;  // log2(e) / sqrt(128)
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    const int my_nkb = nkb[t];
    uint8_t* pt = ps + t * kFtPTile;
    for (int j = 0; j < my_nkb; ++j) {
      const int s = j % kFtStages;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, a.err, DEV_TIMEOUT_ATTN_FULL) && flags[0] == 0);
      if (!ok) break;
      tc_fence_after();
      float sv[64];
      tc_ld64(tmem + lanebase + (uint32_t)(t * kFtKeys), sv);
      // Keys beyond the row's position: only on the tiles that reach past it.
      if (!__all_sync(0xffffffffu, (long long)j * kFtKeys + kFtKeys - 1 <= pos)) {
        const long long lim = pos - (long long)j * kFtKeys + 1;  // keys [0, lim) of the tile are visible
#pragma unroll
        for (int c = 0; c < 64; ++c) sv[c] = c < lim ? sv[c] : -INFINITY;  // also clears NaN of keys past the prompt
      }
      // row maximum with 8 independent chains
      float mx[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx[e] = sv[e];
#pragma unroll
      for (int c = 8; c < 64; ++c) mx[c & 7] = fmaxf(mx[c & 7], sv[c]);
      const float rmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * scale;
      const float m_new = fmaxf(m_ref, rmax);
      if (j > 0) {
        // O_t and the P_t buffer are free once the previous P.V has completed
        ok = __all_sync(0xffffffffu, mbar_wait(&o_done[t], (j - 1) & 1, a.err, DEV_TIMEOUT_ATTN_FULL));
        if (!ok) break;
        tc_fence_after();
        const bool need = (m_new > m_ref + 8.f) || (m_ref == -INFINITY && m_new != -INFINITY);
        if (__any_sync(0xffffffffu, need)) {
          const float corr = (m_ref == -INFINITY) ? 0.f : exp2f(m_ref - m_new);
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float ov[32];
            tc_ld32(tmem + lanebase + o_col + 32 * c, ov);
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] *= corr;
            tc_st32(tmem + lanebase + o_col + 32 * c, ov);
          }
          l *= corr;
          m_ref = m_new;
        }
      } else {
        m_ref = m_new;
      }
      // P (bf16) in the swizzled [128 rows][64 keys] layout of the MMA's A operand:
      // p = 2^(s * scale - m), one FMA and one ex2 per score (masked scores are
      // -inf and give 0; a row with nothing visible yet uses m = 0).
      const float mu = m_ref == -INFINITY ? 0.f : m_ref;
      float rsum[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) rsum[e] = 0.f;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = ex2_approx(fmaf(sv[8 * ch + 2 * e], scale, -mu));
          const float p1 = ex2_approx(fmaf(sv[8 * ch + 2 * e + 1], scale, -mu));
          rsum[2 * e] += p0;
          rsum[2 * e + 1] += p1;
          w[e] = pack_bf16(p0, p1);
        }
        *reinterpret_cast<uint4*>(pt + qrow * 128 + ((ch ^ (qrow & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l += ((rsum[0] + rsum[1]) + (rsum[2] + rsum[3])) + ((rsum[4] + rsum[5]) + (rsum[6] + rsum[7]));
      if (j == nk - 1 && (long long)(j + 1) * kFtKeys - 1 > pmax) {
        // Keys past the CTA's last position may hold anything (even NaN):
        // their P is 0, but 0 * NaN is NaN, so clear those V rows first.
        const int keep = pmax - j * kFtKeys + 1;
        uint8_t* vt = ring + s * kFtKvStage + kFtKvStage / 2;
        const int gt = (warp - 2 - 4 * t) * 32 + lane;  // 0..127 within the tile's warps
        for (int idx = gt; idx < (kFtKeys - keep) * 16; idx += 128) {
          const int row = keep + (idx >> 4), sub = (idx >> 3) & 1, ch = idx & 7;
          *reinterpret_cast<uint4*>(vt + sub * (kFtKvStage / 4) + swz(row, ch)) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();  // the generic-proxy writes, before the tensor cores read them
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    if (ok && my_nkb > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(&o_done[t], (my_nkb - 1) & 1, a.err, DEV_TIMEOUT_ATTN_FULL));
      if (ok) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        bf16* dst = a.out + ((size_t)pr * a.Hq + (size_t)g * G + hj) * kAttnD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float ov[32];
          tc_ld32(tmem + lanebase + o_col + 32 * c, ov);
          if (valid) {
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8) {
              uint4 o;
              o.x = pack_bf16(ov[8 * q8 + 0] * inv, ov[8 * q8 + 1] * inv);
              o.y = pack_bf16(ov[8 * q8 + 2] * inv, ov[8 * q8 + 3] * inv);
              o.z = pack_bf16(ov[8 * q8 + 4] * inv, ov[8 * q8 + 5] * inv);
              o.w = pack_bf16(ov[8 * q8 + 6] * inv, ov[8 * q8 + 7] * inv);
              *reinterpret_cast<uint4*>(dst + 32 * c + 8 * q8) = o;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

}  // namespace qb
