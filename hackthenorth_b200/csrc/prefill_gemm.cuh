// prefill_gemm.cuh — dense bf16 GEMM for prompt prefill on sm_100a's 5th-gen
// tensor cores: D[T][N] = X[T][K] . W[N][K]^T with fp32 accumulation in tensor
// memory (TMEM) and one bf16 rounding, plus the projection epilogues of the
// decode path (store, + residual, SwiGLU over gate/up-interleaved rows, the
// QKV heads' norm + RoPE + cache append); a tensor-parallel rank computes a
// block of output columns over the whole input (unshard_cols_kernel lays the
// all-gathered blocks out as whole rows).
//
// This is the prefill counterpart of the reference's dense projections
// (dryft/engine/attention.py:92-98 uses torch linear for prompt rows; the
// roundings are those of kernels/projection.py:13-83 and down.py:8-35).
//
// Output tiles of 128 x 256 (128 prompt rows x 256 weight rows); one
// persistent CTA per SM walks tiles b, b + G, ...:
//  * warp 0, one lane: TMA producer. X tile [128 rows][64 cols] and W tile
//    [256 rows][64 cols] per K block (128-byte swizzle, no multicast) into a
//    4-stage ring of 48 KB, continuously across the CTA's tiles;
//  * warp 1: allocates 512 TMEM columns (two 128-lane x 256-column fp32
//    accumulators); one lane issues 4 tcgen05.mma.cta_group::1.kind::f16
//    (M 128, N 256, K 16) per K block with shared-memory descriptors of both
//    operands (K-major, 128-byte swizzle); tcgen05.commit frees each stage once
//    its MMAs have read it and signals a tile's accumulator complete; tile i
//    uses accumulator i & 1 once the epilogue has drained tile i - 2;
//  * warps 2-5: each reads its 32 TMEM lanes (32 prompt rows) with
//    tcgen05.ld.32x32b and runs the epilogue on 8 columns at a time, under
//    the MMAs of the next tile.
// Every wait is bounded (the kernel records an error and returns), and TMEM is
// released by warp 1 after its MMAs have completed and all readers are done,
// on every path.
#pragma once
#include "common.cuh"

namespace qb {

constexpr int kPgBM = 128;                       // prompt rows per tile (MMA M)
constexpr int kPgBN = 256;                       // weight rows per tile (MMA N)
constexpr int kPgBK = 64;                        // K per stage (one 128-byte swizzle row)
constexpr int kPgStages = 4;
constexpr int kPgABytes = kPgBM * kPgBK * 2;     // 16 KB
constexpr int kPgBBytes = kPgBN * kPgBK * 2;     // 32 KB
constexpr int kPgStageBytes = kPgABytes + kPgBBytes;
constexpr int kPgThreads = 6 * 32;
constexpr int kPgTmemCols = 256;

enum PrefillEpi : int { PG_STORE = 0, PG_RESIDUAL = 1, PG_SWIGLU = 2, PG_QKV_ROPE = 3 };

struct PgArgs {
  int T, N, K;              // rows of X, rows of W, shared K
  bf16* out;                // STORE/RESIDUAL: [T][N]; SWIGLU: [T][N/2]
  const bf16* residual;     // RESIDUAL: [T][res_stride] (res_stride 0: N)
  int res_stride;
  int* err;
  // PG_QKV_ROPE: the QKV projection of prompt rows at positions p0 + row,
  // finished per head as the decode path does (q/k RMSNorm + RoPE, K/V to the
  // cache): q_out [T][Hq][128], caches [Hkv][cap][128] of this layer.
  const bf16* q_norm;
  const bf16* k_norm;
  const bf16* cos;          // [cap][128]
  const bf16* sin;
  float eps;
  bf16* q_out;
  bf16* k_cache;
  bf16* v_cache;
  int Hq, Hkv, cap, p0;
};

__host__ inline size_t pg_smem_bytes() { return 1024 + (size_t)kPgStages * kPgStageBytes + 256; }  // + barriers, TMEM slot

// Shared-memory matrix descriptor, K-major operand with 128-byte swizzle:
// start address >> 4 at [0,14), leading byte offset (unused for swizzled
// K-major, 1) at [16,30), stride byte offset between 8-row groups (1024 B) >> 4
// at [32,46), descriptor version 1 at [46,48), layout type 2 (128-byte
// swizzle) at [61,64).
__device__ __forceinline__ uint64_t pg_desc(const void* smem_tile) {
  const uint64_t addr = smem_u32(smem_tile);
  return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulator, bf16 A and B, both
// K-major, N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t pg_idesc(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// PG_QKV_ROPE epilogue for one 128-column head of one prompt row: the
// projection rounded to bf16; q and k heads then RMSNorm'd over the head
// (bf16(bf16(x * inv) * gain)) and rotated (rotate-half RoPE with the cos/sin
// row of the position, each product rounded, the sum rounded), exactly the
// rope_rows_kernel arithmetic (dryft/engine/kernels/fused.py:9-30); q goes to
// q_out, k and v to the cache at the row's position.
// The TMEM loads are warp-collective: every lane of the warp calls this for the
// same head; lanes whose row is past T (valid false) only take part in them.
__device__ __forceinline__ void pg_qkv_rope_head(const PgArgs& a, int row, bool valid, int head, uint32_t taddr) {
  float x[128];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float v[32];
    tc_ld32(taddr + (uint32_t)(32 * c), v);
#pragma unroll
    for (int i = 0; i < 32; ++i) x[32 * c + i] = round_bf16(v[i]);
  }
  if (!valid) return;
  const int pos = a.p0 + row;
  if (pos < 0 || pos >= a.cap) {
    report_error(a.err, DEV_BAD_POSITION);
    return;
  }
  bf16* dst;
  const bf16* gain = nullptr;
  if (head < a.Hq) {
    dst = a.q_out + ((size_t)row * a.Hq + head) * 128;
    gain = a.q_norm;
  } else if (head < a.Hq + a.Hkv) {
    dst = a.k_cache + ((size_t)(head - a.Hq) * a.cap + pos) * 128;
    gain = a.k_norm;
  } else {
    dst = a.v_cache + ((size_t)(head - a.Hq - a.Hkv) * a.cap + pos) * 128;
  }
  if (gain != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 128; ++i) ss = fmaf(x[i], x[i], ss);
    const float inv = 1.0f / sqrtf(ss / 128.0f + a.eps);  // correctly rounded sqrt and division
#pragma unroll
    for (int c8 = 0; c8 < 16; ++c8) {
      const uint4 gv = ldg128_nc(gain + 8 * c8);
      const uint32_t* pg = reinterpret_cast<const uint32_t*>(&gv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x[8 * c8 + 2 * j] = round_bf16(round_bf16(x[8 * c8 + 2 * j] * inv) * bf_lo(pg[j]));
        x[8 * c8 + 2 * j + 1] = round_bf16(round_bf16(x[8 * c8 + 2 * j + 1] * inv) * bf_hi(pg[j]));
      }
    }
    const bf16* crow = a.cos + (size_t)pos * 128;
    const bf16* srow = a.sin + (size_t)pos * 128;
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8) {  // dims d in [8 c8, 8 c8 + 8) and their partners d + 64
      const uint4 clo = ldg128_nc(crow + 8 * c8), chi = ldg128_nc(crow + 64 + 8 * c8);
      const uint4 slo = ldg128_nc(srow + 8 * c8), shi = ldg128_nc(srow + 64 + 8 * c8);
      const uint32_t* pcl = reinterpret_cast<const uint32_t*>(&clo);
      const uint32_t* pch = reinterpret_cast<const uint32_t*>(&chi);
      const uint32_t* psl = reinterpret_cast<const uint32_t*>(&slo);
      const uint32_t* psh = reinterpret_cast<const uint32_t*>(&shi);
      uint32_t olo[4], ohi[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int d0 = 8 * c8 + 2 * j;
        const float a0 = x[d0], a1 = x[d0 + 1], b0 = x[d0 + 64], b1 = x[d0 + 65];
        olo[j] = pack_bf16(round_bf16(a0 * bf_lo(pcl[j])) + round_bf16(-b0 * bf_lo(psl[j])),
                           round_bf16(a1 * bf_hi(pcl[j])) + round_bf16(-b1 * bf_hi(psl[j])));
        ohi[j] = pack_bf16(round_bf16(b0 * bf_lo(pch[j])) + round_bf16(a0 * bf_lo(psh[j])),
                           round_bf16(b1 * bf_hi(pch[j])) + round_bf16(a1 * bf_hi(psh[j])));
      }
      *reinterpret_cast<uint4*>(dst + 8 * c8) = make_uint4(olo[0], olo[1], olo[2], olo[3]);
      *reinterpret_cast<uint4*>(dst + 64 + 8 * c8) = make_uint4(ohi[0], ohi[1], ohi[2], ohi[3]);
    }
  } else {
#pragma unroll
    for (int c8 = 0; c8 < 16; ++c8) {
      uint4 o;
      o.x = pack_bf16(x[8 * c8 + 0], x[8 * c8 + 1]);
      o.y = pack_bf16(x[8 * c8 + 2], x[8 * c8 + 3]);
      o.z = pack_bf16(x[8 * c8 + 4], x[8 * c8 + 5]);
      o.w = pack_bf16(x[8 * c8 + 6], x[8 * c8 + 7]);
      *reinterpret_cast<uint4*>(dst + 8 * c8) = o;
    }
  }
}

template <int EPI>
__device__ __forceinline__ void pg_epilogue_store(const PgArgs& a, int row, int n, const float (&v)[8]) {
  if constexpr (EPI == PG_STORE) {
    uint4 o;
    o.x = pack_bf16(v[0], v[1]);
    o.y = pack_bf16(v[2], v[3]);
    o.z = pack_bf16(v[4], v[5]);
    o.w = pack_bf16(v[6], v[7]);
    *reinterpret_cast<uint4*>(a.out + (size_t)row * a.N + n) = o;
  } else if constexpr (EPI == PG_RESIDUAL) {
    const uint4 r = *reinterpret_cast<const uint4*>(a.residual + (size_t)row * (a.res_stride ? a.res_stride : a.N) + n);
    const uint32_t* pr = reinterpret_cast<const uint32_t*>(&r);
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      po[j] = pack_bf16(round_bf16(v[2 * j]) + bf_lo(pr[j]), round_bf16(v[2 * j + 1]) + bf_hi(pr[j]));
    *reinterpret_cast<uint4*>(a.out + (size_t)row * a.N + n) = o;
  } else {  // PG_SWIGLU: columns (2j, 2j+1) = (gate j, up j)
    float h[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float act = round_bf16(silu_f32(round_bf16(v[2 * j])));
      h[j] = act * round_bf16(v[2 * j + 1]);
    }
    uint2 o;
    o.x = pack_bf16(h[0], h[1]);
    o.y = pack_bf16(h[2], h[3]);
    *reinterpret_cast<uint2*>(a.out + (size_t)row * (a.N / 2) + n / 2) = o;
  }
}

// Persistent: CTA b takes tiles b, b + G, b + 2G, ... (m tile fastest, so
// consecutive CTAs share a weight tile in L2). The producer and the MMA lane
// run through the k blocks of all their tiles without stopping; the MMA lane
// alternates between two 256-column accumulators in TMEM, so the epilogue of
// tile i (acc_full -> read -> acc_empty) overlaps the MMAs of tile i + 1.
template <int EPI>
__global__ void __launch_bounds__(kPgThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                        const PgArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kPgStages * kPgStageBytes);
  uint64_t* empty = full + kPgStages;
  uint64_t* acc_full = empty + kPgStages;  // [2] MMAs of the buffer's tile complete
  uint64_t* acc_empty = acc_full + 2;      // [2] the 4 epilogue warps have read the buffer
  uint64_t* done = acc_empty + 2;          // every MMA this CTA issued has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nkb = (a.K + kPgBK - 1) / kPgBK;
  const int mt = (a.T + kPgBM - 1) / kPgBM;
  const int tiles = mt * ((a.N + kPgBN - 1) / kPgBN);
  const int my_tiles = blockIdx.x < tiles ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPgStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(done, 1);
    fence_mbar_init();
    flags[0] = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * kPgTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_wait();  // X is written by the previous kernel
  pdl_trigger();

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tensormap(&tmx);
      prefetch_tensormap(&tmw);
      int g = 0;  // k blocks issued over all tiles
      for (int i = 0; i < my_tiles && flags[0] == 0; ++i) {
        const int t = blockIdx.x + i * gridDim.x;
        const int m0 = (t % mt) * kPgBM, n0 = (t / mt) * kPgBN;
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % kPgStages;
          if (g >= kPgStages && !mbar_wait(&empty[s], ((g / kPgStages) - 1) & 1, a.err, DEV_TIMEOUT_GEMV_EMPTY)) {
            flags[0] = 1;
            break;
          }
          uint8_t* st = ring + s * kPgStageBytes;
          mbar_arrive_expect_tx(&full[s], kPgStageBytes);
          tma_load_2d(st, &tmx, kb * kPgBK, m0, &full[s]);
          tma_load_2d(st + kPgABytes, &tmw, kb * kPgBK, n0, &full[s]);
        }
      }
      // keep shared memory alive until every issued copy has landed
      for (int c = (g > kPgStages ? g - kPgStages : 0); c < g; ++c)
        mbar_wait(&full[c % kPgStages], (c / kPgStages) & 1, nullptr, 0);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = pg_idesc(kPgBM, kPgBN);
      int g = 0;  // k blocks consumed over all tiles
      for (int i = 0; i < my_tiles; ++i) {
        const int ab = i & 1;
        const uint32_t acc = tmem + (uint32_t)(ab * kPgTmemCols);
        // the epilogue of tile i - 2 has read this buffer
        bool ok = flags[0] == 0;
        if (ok && i >= 2 && !mbar_wait(&acc_empty[ab], ((i >> 1) - 1) & 1, a.err, DEV_TIMEOUT_ATTN_FULL)) ok = false;
        if (ok) tc_fence_after();
        for (int kb = 0; kb < nkb && ok; ++kb, ++g) {
          const int s = g % kPgStages;
          if (!mbar_wait(&full[s], (g / kPgStages) & 1, a.err, DEV_TIMEOUT_GEMV_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* st = ring + s * kPgStageBytes;
          const uint64_t ad = pg_desc(st), bd = pg_desc(st + kPgABytes);
#pragma unroll
          for (int k = 0; k < kPgBK / 16; ++k)  // K 16 per MMA = 32 bytes along the swizzled row
            tc_mma(acc, ad + (uint64_t)(k * 2), bd + (uint64_t)(k * 2), idesc, (kb | k) != 0 ? 1u : 0u);
          tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        if (!ok) flags[0] = 1;
        tc_commit(&acc_full[ab]);  // this tile's MMAs complete (also after a stop: wakes the epilogue)
        if (!ok) break;
      }
      // TMEM is released below only after every MMA issued here has completed
      // (on the normal path the epilogue has already seen them all)
      tc_commit(done);
      mbar_wait(done, 0, nullptr, 0);
    }
    __syncwarp();
  } else {
    // --------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lanes 32q .. 32q+31
    for (int i = 0; i < my_tiles; ++i) {
      const int ab = i & 1;
      const int t = blockIdx.x + i * gridDim.x;
      const int m0 = (t % mt) * kPgBM, n0 = (t / mt) * kPgBN;
      const int row = m0 + 32 * q + lane;
      const bool ok = mbar_wait(&acc_full[ab], (i >> 1) & 1, a.err, DEV_TIMEOUT_ATTN_FULL) && flags[0] == 0;
      tc_fence_after();
      if (!ok) break;
      const uint32_t base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(ab * kPgTmemCols);
      if constexpr (EPI == PG_QKV_ROPE) {
        // the tile's 256 columns are two whole heads (N is a multiple of 128)
        for (int hh = 0; hh < kPgBN / 128 && n0 + 128 * hh < a.N; ++hh)
          pg_qkv_rope_head(a, row, row < a.T, n0 / 128 + hh, base + (uint32_t)(128 * hh));
      } else {
        for (int c = 0; c < kPgBN; c += 8) {
          float v[8];
          tc_ld8(base + (uint32_t)c, v);
          const int n = n0 + c;
          if (row < a.T && n < a.N) pg_epilogue_store<EPI>(a, row, n, v);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kPgTmemCols)
                 : "memory");
  }
}

// dst[t][r*C + c] = src[r][t][c]: the rank-major result of an NCCL all-gather
// of every tensor-parallel rank's column block [T][C], laid out as whole rows
// [T][n*C]. C is a multiple of 8 (one 16-byte vector per thread).
__global__ void unshard_cols_kernel(const bf16* __restrict__ src, bf16* __restrict__ dst, int T, int C, int n) {
  pdl_wait();
  const long long W = (long long)C * n;
  const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i >= (long long)T * W) return;
  const long long t = i / W, col = i - t * W;
  const long long r = col / C, c = col - r * C;
  *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(src + (r * T + t) * C + c);
}

}  // namespace qb
