// Batch-one decode attention (one query token, GQA group G <= 8) as C
// thread-block clusters of S CTAs per KV head (S = the cluster size, 16, 8 or
// 4; C = 1 at short capacities, more when the GPU has room for them).
//
// Follows the split-KV decode of dryft/engine/kernels/attention.py (per-split
// online softmax in base 2 with P rounded to bf16 for the P.V product, splits
// merged with weights exp2(lse_s - max) / sum, :204-206) and the fused
// q/k RMSNorm + RoPE + cache append prologue of dryft/engine/kernels/fused.py:9-30.
//
// Layout of the work:
//  * CTA `split` of the cluster for KV head h takes keys [k0, k1) of h; a
//    producer lane streams them as 32-key stages (K lo/hi, V lo/hi boxes of
//    [32 keys][64 dims], 128-byte swizzle) into an 8-slot ring. The cache up to
//    the previous position is final before this launch's predecessor started,
//    so the first 8 stages are issued before griddepcontrol.wait.
//  * 8 consumer warps; warp w owns ring slot w (stages w, w+8, ...), so every
//    slot's mbarrier phases are observed by one warp.
//  * Scores are computed transposed, S^T = K . Q^T, as m16n8k16 tiles with the
//    keys on M and the (at most 8) query rows on N, and the output as
//    O^T = V^T . P^T: half the tensor-core work of putting the query rows on M.
//    P^T's B fragments come from the S^T accumulators through movmatrix.trans.
//  * The 8 warps are merged in the CTA (fixed warp order), then each CTA sends
//    row r, dims [t*W, (t+1)*W) (W = 128 / S) of its normalised split output,
//    and its lse, into the shared memory of cluster CTA t. After one cluster
//    barrier every CTA merges its own dim slice over the splits in split order.
//    The first cluster barrier phase is arrived at kernel start and waited just
//    before the first remote store (all CTAs of the cluster are then running);
//    the receive buffers lie outside the ring, so no CTA has to wait for the
//    others to finish streaming before the exchange.
//  * With C > 1 clusters per head, cluster c takes splits [c*S, c*S+S) of the
//    head's C*S; each CTA writes its merged dim slice and the cluster's lse to
//    global partial rows, and the CTA of the same slice index that takes the
//    last merge ticket merges the C clusters in cluster order and resets the
//    ticket.
#pragma once
#include "attention.cuh"

namespace qb {

constexpr int kDecWarps = 8;                         // consumer warps; warp w owns ring slot w
constexpr int kDecThreads = (kDecWarps + 1) * 32;
constexpr int kDecKeys = 32;                         // keys per stage
constexpr int kDecSubTile = kDecKeys * 128;          // [32 keys][64 dims] bf16 = 4 KB
constexpr int kDecStageBytes = 4 * kDecSubTile;      // K lo, K hi, V lo, V hi = 16 KB
constexpr int kDecStages = kDecWarps;
constexpr int kDecMergeThreads = 256;                // the in-CTA merge: dim tid & 127, rows (tid >> 7) + 2i
constexpr int kDecRows = 8;                          // query rows per KV head (N of the mma)
constexpr int kDecMaxCluster = 16;
constexpr int kDecObStride = kAttnD + 4;             // padded fp32 row of the in-CTA merge
constexpr int kDecBarrierId = 3;
constexpr int kDecMultiClusterKeys = 8192;  // live keys from which a KV head may use all its clusters
constexpr int kDecShortSplits = 8;          // splits per KV head below that (clusters of 4: two clusters)
constexpr int kDecMaxClusters = 8;          // clusters per KV head

__host__ __device__ inline size_t dec_smem_bytes(int nw = kDecStages) {
  return 1024 + (size_t)nw * kDecStageBytes             // ring
         + kDecRows * kAttnD * 2                        // query rows
         + 2 * kAttnD * 2                               // new k, v
         + 2 * nw * 8                                   // full, empty
         + nw * kDecRows * 2 * 4                        // per-warp m, l
         + kDecRows * kAttnD * 4                        // receive slices [split][row][128 / S]
         + kDecMaxCluster * kDecRows * 4                // receive lse
         + 64;
}
static_assert(kDecWarps * kDecRows * kDecObStride * 4 <= kDecStages * kDecStageBytes, "merge buffer fits the ring");

struct DecSmem {
  uint8_t* ring;
  bf16* qs;
  bf16* kvnew;
  uint64_t* full;
  uint64_t* empty;
  float* ml;     // [warp][row][2]
  float* rbuf;   // [split][row][W]
  float* rlse;   // [split][row]
  volatile int* flags;
};

__device__ __forceinline__ DecSmem dec_carve(uint8_t* smem_raw, int nw) {
  DecSmem m;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  m.ring = smem;
  m.qs = reinterpret_cast<bf16*>(m.ring + nw * kDecStageBytes);
  m.kvnew = m.qs + kDecRows * kAttnD;
  m.full = reinterpret_cast<uint64_t*>(m.kvnew + 2 * kAttnD);
  m.empty = m.full + nw;
  m.ml = reinterpret_cast<float*>(m.empty + nw);
  m.rbuf = m.ml + nw * kDecRows * 2;
  m.rlse = m.rbuf + kDecRows * kAttnD;
  m.flags = reinterpret_cast<volatile int*>(m.rlse + kDecMaxCluster * kDecRows);
  return m;
}

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t v) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(v));
  return r;
}

template <bool TRACE = false>
__global__ void __launch_bounds__(kDecThreads, 1)
    attn_decode_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                       const AttnArgs a) {
  constexpr int NW = kDecWarps;  // consumer warps = ring slots
  extern __shared__ uint8_t smem_raw[];
  const DecSmem sm = dec_carve(smem_raw, NW);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int S = a.splits;  // cluster size
  const int C = max(1, a.clusters);  // clusters per KV head
  const int kvh = blockIdx.x / (C * S);
  const int cl = (blockIdx.x / S) % C;
  const int split = blockIdx.x % S;  // == cluster rank
  const int G = a.Hq / a.Hkv;        // query rows, <= kDecRows
  if (TRACE && tid == 0) trace_stamp(trace_slot(a.trace), TRACE_ENTRY);

  // First cluster phase: arrived now, waited before the first remote store.
  cluster_arrive_relaxed();
  if (tid == 0) {
    for (int s = 0; s < NW; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    fence_mbar_init();
    sm.flags[0] = 0;
  }
  __syncthreads();

  // Live key range (the position was written by the previous step, two or
  // more launches earlier, so it is read before griddepcontrol.wait).
  long long last = a.pos[0];
  if (last < 0 || last >= a.cap) {
    if (tid == 0 && blockIdx.x == 0) report_error(a.err, DEV_BAD_POSITION);
    last = -1;
  }
  const int n = (int)last + 1;
  // Splits over the whole head: about kAttnMinSplitKeys keys each, at most
  // kDecShortSplits (at least one cluster's worth) below kDecMultiClusterKeys
  // live keys, up to C clusters' worth above. Cluster cl takes global splits [cl*S, cl*S+S).
  const int mk = a.multi_keys > 0 ? a.multi_keys : kDecMultiClusterKeys;
  const int cmax = n >= mk ? C : min(C, max(1, kDecShortSplits / S));
  const int2 sl = attn_split_len(n, min(cmax * S, (n + kAttnMinSplitKeys - 1) / kAttnMinSplitKeys));
  const int per = sl.x, SeT = sl.y;            // every split below SeT has keys
  const int Cact = (SeT + S - 1) / S;           // clusters with work (uniform over the grid)
  const int Se = max(0, min(S, SeT - cl * S));  // active splits of this cluster
  const int k0 = min(n, (cl * S + split) * per);
  const int k1 = min(n, k0 + per);
  const int nst = (k1 - k0 + kDecKeys - 1) / kDecKeys;
  const bool active = split < Se && nst > 0;

  float val[4], lsev[4];  // this thread's rows (tid >> 7) + 2i, dim tid & 127
  bool ok = true;
  if (Se == 0) {  // a cluster without work leaves at once (it reads nothing of the previous kernel)
    cluster_wait();
    return;
  }

  if (warp == NW) {
    // ---------------------------------------------------------------- producer
    if (active && lane == 0) {
      prefetch_tensormap(&tmk);
      prefetch_tensormap(&tmv);
      bool waited = false;
      int issued = 0;
      for (int c = 0; c < nst; ++c) {
        const int s = c % NW;
        if (c >= NW) {
          if (!waited) {
            pdl_wait();
            pdl_trigger();
            waited = true;
          }
          if (!mbar_wait(&sm.empty[s], ((c / NW) - 1) & 1, a.err, DEV_TIMEOUT_ATTN_EMPTY)) {
            ok = false;
            break;
          }
        }
        uint8_t* st = sm.ring + s * kDecStageBytes;
        const int y = kvh * a.cap + k0 + c * kDecKeys;
        mbar_arrive_expect_tx(&sm.full[s], kDecStageBytes);
        tma_load_2d(st, &tmk, 0, y, &sm.full[s]);
        tma_load_2d(st + kDecSubTile, &tmk, 64, y, &sm.full[s]);
        tma_load_2d(st + 2 * kDecSubTile, &tmv, 0, y, &sm.full[s]);
        tma_load_2d(st + 3 * kDecSubTile, &tmv, 64, y, &sm.full[s]);
        issued = c + 1;
      }
      if (!waited) {
        pdl_wait();
        pdl_trigger();
      }
      if (!ok) {
        // Keep shared memory alive until the copies already in flight land.
        for (int c = (issued > NW ? issued - NW : 0); c < issued; ++c)
          mbar_wait(&sm.full[c % NW], (c / NW) & 1, nullptr, 0);
      }
    } else {
      pdl_wait();
      pdl_trigger();
    }
    __syncwarp();
  } else {
    // --------------------------------------------------------------- consumers
    pdl_wait();
    pdl_trigger();
    if (TRACE && tid == 0) trace_stamp(trace_slot(a.trace), TRACE_WAIT);
    if (active) {
      if (tid < kDecRows * kAttnD / 8) reinterpret_cast<uint4*>(sm.qs)[tid] = make_uint4(0, 0, 0, 0);
      named_barrier(kDecBarrierId, NW * 32);
      const bool owns_new = (k0 <= last) && (last < k1);
      const bf16* cos_row = a.cos + (size_t)last * kAttnD;
      const bf16* sin_row = a.sin + (size_t)last * kAttnD;
      if (warp < G)
        norm_rope_head(a.qkv + (size_t)(kvh * G + warp) * kAttnD, a.q_norm, cos_row, sin_row, a.eps, lane,
                       sm.qs + warp * kAttnD, nullptr);
      if (owns_new) {
        const size_t slot = ((size_t)kvh * a.cap + last) * kAttnD;
        if (warp == NW - 1) {
          norm_rope_head(a.qkv + (size_t)a.Hq * kAttnD + kvh * kAttnD, a.k_norm, cos_row, sin_row, a.eps, lane,
                         sm.kvnew, a.k_cache + slot);
        } else if (warp == NW - 2) {
          const uint2 v =
              *reinterpret_cast<const uint2*>(a.qkv + (size_t)(a.Hq + a.Hkv) * kAttnD + kvh * kAttnD + 4 * lane);
          *reinterpret_cast<uint2*>(sm.kvnew + kAttnD + 4 * lane) = v;
          *reinterpret_cast<uint2*>(a.v_cache + slot + 4 * lane) = v;
        }
      }
      named_barrier(kDecBarrierId, NW * 32);

      // Q^T as the B operand of every k-step: qb[ks] = dims [16ks, 16ks+16) of rows 0..7.
      uint32_t qb[8][2];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t r[4];
        ldsm_x4(r, sm.qs + (lane & 7) * kAttnD + j * 32 + (lane >> 3) * 8);
        qb[2 * j][0] = r[0];
        qb[2 * j][1] = r[1];
        qb[2 * j + 1][0] = r[2];
        qb[2 * j + 1][1] = r[3];
      }
      const int g4 = lane >> 2;
      const int t4 = lane & 3;
      float o[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
      float m[2] = {-INFINITY, -INFINITY};
      float l[2] = {0.f, 0.f};
      // log2(e) / sqrt(128), folded in double precision as the reference does.
      const float scale = 0.12751743082459868f;
      const int s = warp;
      uint8_t* stage = sm.ring + s * kDecStageBytes;

      for (int c = warp; c < nst; c += NW) {
        // Every lane waits; the verdict is made warp-uniform before the shuffles below.
        if (!__all_sync(0xffffffffu, mbar_wait(&sm.full[s], (c / NW) & 1, a.err, DEV_TIMEOUT_ATTN_FULL))) {
          ok = false;
          break;
        }
        if (TRACE && c == 0 && lane == 0) trace_stamp(trace_slot(a.trace), TRACE_FIRST);
        const int kstage = k0 + c * kDecKeys;
        if (owns_new && kstage <= last && last < kstage + kDecKeys) {
          const int kr = (int)last - kstage;
          const int which = lane >> 3, ch = lane & 7;
          *reinterpret_cast<uint4*>(stage + which * kDecSubTile + swz(kr, ch)) =
              *reinterpret_cast<const uint4*>(sm.kvnew + (which >> 1) * kAttnD + (which & 1) * 64 + ch * 8);
        }
        const int svalid = k1 - kstage;
        if (svalid < kDecKeys) {
          // Slots past the live range may hold anything (even NaN); P is 0
          // there, but 0 * NaN is NaN, so clear those V rows.
          for (int i = lane; i < (kDecKeys - svalid) * 16; i += 32) {
            const int row = svalid + (i >> 4);
            const int sub = (i >> 3) & 1, ch = i & 7;
            *reinterpret_cast<uint4*>(stage + (2 + sub) * kDecSubTile + swz(row, ch)) = make_uint4(0, 0, 0, 0);
          }
        }
        __syncwarp();

        // S^T: two 16-key m-tiles; two accumulators each (even / odd k-steps).
        float sc[2][2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int h = 0; h < 2; ++h) sc[mt][h][0] = sc[mt][h][1] = sc[mt][h][2] = sc[mt][h][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int ch = ((ks & 3) << 1) + (lane >> 4);
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            const int key = mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
            uint32_t ka[4];
            ldsm_x4(ka, stage + (ks >> 2) * kDecSubTile + swz(key, ch));
            mma_bf16_16816(sc[mt][ks & 1], ka, qb[ks][0], qb[ks][1]);
          }
        }
        // Thread holds keys {mt*16 + g4 + 8h} for query rows 2*t4 + e.
        float p[2][2][2];  // [mt][h][e]
        float corr[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float x[2][2];
          float rmax = -INFINITY;
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int key = kstage + mt * 16 + h * 8 + g4;
              const float v = (sc[mt][0][h * 2 + e] + sc[mt][1][h * 2 + e]) * scale;
              x[mt][h] = (key < k1) ? v : -INFINITY;
              rmax = fmaxf(rmax, x[mt][h]);
            }
          rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 4));
          rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 8));
          rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 16));
          const float mnew = fmaxf(m[e], rmax);
          corr[e] = (m[e] == -INFINITY) ? 0.f : exp2f(m[e] - mnew);
          float rs = 0.f;
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              p[mt][h][e] = (x[mt][h] == -INFINITY) ? 0.f : exp2f(x[mt][h] - mnew);
              rs += p[mt][h][e];
            }
          l[e] = l[e] * corr[e] + rs;  // per-lane partial; summed over the key lanes at the end
          m[e] = mnew;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j][0] *= corr[0];
          o[j][1] *= corr[1];
          o[j][2] *= corr[0];
          o[j][3] *= corr[1];
        }
        // P^T B fragments: transpose the bf16 [keys][rows] 8x8 blocks.
        uint32_t pb[2][2];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int h = 0; h < 2; ++h) pb[mt][h] = movmatrix_trans(pack_bf16(p[mt][h][0], p[mt][h][1]));
        // O^T += V^T . P^T over the two key m-tiles.
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int dt = 0; dt < 8; ++dt) {
            const int mi = lane >> 3;
            const int key = mt * 16 + (lane & 7) + (mi >> 1) * 8;
            const int ch = ((dt & 3) << 1) + (mi & 1);
            uint32_t va[4];
            ldsm_x4_t(va, stage + (2 + (dt >> 2)) * kDecSubTile + swz(key, ch));
            mma_bf16_16816(o[dt], va, pb[mt][0], pb[mt][1]);
          }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[s]);
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        l[e] += __shfl_xor_sync(0xffffffffu, l[e], 4);
        l[e] += __shfl_xor_sync(0xffffffffu, l[e], 8);
        l[e] += __shfl_xor_sync(0xffffffffu, l[e], 16);
      }
      if (!ok && lane == 0) sm.flags[0] = 1;
      named_barrier(kDecBarrierId, NW * 32);
      if (TRACE && tid == 0) trace_stamp(trace_slot(a.trace), TRACE_LOOP);
      ok = sm.flags[0] == 0;
      if (ok) {
        // Merge the 8 warps (fixed order) through the drained ring.
        float* ob = reinterpret_cast<float*>(sm.ring);  // [warp][row][kDecObStride]
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) {
          const int d = dt * 16 + g4;
          float* r0 = ob + ((size_t)warp * kDecRows + 2 * t4) * kDecObStride;
          float* r1 = r0 + kDecObStride;
          r0[d] = o[dt][0];
          r1[d] = o[dt][1];
          r0[d + 8] = o[dt][2];
          r1[d + 8] = o[dt][3];
        }
        if (g4 == 0) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            sm.ml[(warp * kDecRows + 2 * t4 + e) * 2] = m[e];
            sm.ml[(warp * kDecRows + 2 * t4 + e) * 2 + 1] = l[e];
          }
        }
        named_barrier(kDecBarrierId, NW * 32);
        const int d = tid & 127;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = (tid >> 7) + 2 * i;
          val[i] = 0.f;
          lsev[i] = -INFINITY;
          if (r < G && tid < kDecMergeThreads) {
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < NW; ++w) M = fmaxf(M, sm.ml[(w * kDecRows + r) * 2]);
            float L = 0.f, acc = 0.f;
#pragma unroll
            for (int w = 0; w < NW; ++w) {
              const float mw = sm.ml[(w * kDecRows + r) * 2];
              const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
              L += sm.ml[(w * kDecRows + r) * 2 + 1] * f;
              acc += ob[((size_t)w * kDecRows + r) * kDecObStride + d] * f;
            }
            val[i] = L > 0.f ? acc / L : 0.f;
            lsev[i] = L > 0.f ? M + log2f(L) : -INFINITY;
          }
        }
      }
    }
  }
  if (TRACE && tid == 0) trace_stamp(trace_slot(a.trace), TRACE_MERGED);

  // ------------------------------------------------------------ cluster merge
  cluster_wait();  // every CTA of the cluster is running
  if (TRACE && tid == 0) trace_stamp(trace_slot(a.trace), TRACE_CWAIT);
  if (Se == 1 && Cact == 1) {  // uniform: the single split is the answer
    if (tid < kDecMergeThreads && split == 0 && active && ok) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = (tid >> 7) + 2 * i;
        if (r < G) attn_store_out(a, kvh, r, tid & 127, val[i]);
      }
    }
    if (TRACE && tid == 0) trace_stamp(trace_slot(a.trace), TRACE_EXIT);
    return;
  }
  const int W = kAttnD / S;
  if (tid < kDecMergeThreads && active && ok) {
    const int d = tid & 127;
    const int owner = d / W;
    const uint32_t rb = map_shared_rank(sm.rbuf, owner);
    const uint32_t rl = map_shared_rank(sm.rlse, owner);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = (tid >> 7) + 2 * i;
      if (r < G) {
        st_cluster_f32(rb + (uint32_t)(((split * kDecRows + r) * W + (d - owner * W)) * 4), val[i]);
        if (d == owner * W) st_cluster_f32(rl + (uint32_t)((split * kDecRows + r) * 4), lsev[i]);
      }
    }
  }
  cluster_sync_all();
  if (TRACE && tid == 0) trace_stamp(trace_slot(a.trace), TRACE_CSYNC);
  // Merge dims [split*W, split*W + W) of every row over the cluster's Se
  // splits, in split order (dryft/engine/kernels/attention.py:204-206).
  float cval = 0.f, clse = -INFINITY;
  if (tid < G * W) {
    const int r = tid / W, off = tid % W;
    float mx = -INFINITY;
    for (int sp = 0; sp < Se; ++sp) mx = fmaxf(mx, sm.rlse[sp * kDecRows + r]);
    float den = 0.f, acc = 0.f;
    for (int sp = 0; sp < Se; ++sp) {
      const float w = exp2f(sm.rlse[sp * kDecRows + r] - mx);
      den += w;
      acc = fmaf(sm.rbuf[(sp * kDecRows + r) * W + off], w, acc);
    }
    cval = acc / den;
    clse = mx + log2f(den);
    if (Cact == 1) attn_store_out(a, kvh, r, split * W + off, cval);
  }
  if (TRACE && tid == 0 && Cact == 1) trace_stamp(trace_slot(a.trace), TRACE_EXIT);
  if (Cact == 1) return;
  // Several clusters per head: each CTA publishes its slice of the cluster's
  // result (normalised rows + log-sum-exp) and the CTA of the same slice
  // index that arrives last merges the clusters in cluster order.
  float* po = a.part_o + (size_t)kvh * a.part_splits * kDecRows * kAttnD;
  float* pl = a.part_lse + (size_t)kvh * a.part_splits * kDecRows;
  if (tid < G * W) {
    const int r = tid / W, off = tid % W;
    po[((size_t)cl * kDecRows + r) * kAttnD + split * W + off] = cval;
    if (off == 0) pl[cl * kDecRows + r] = clse;
  }
  __syncthreads();
  if (tid == 0) {
    const unsigned t = atomic_add_acq_rel_gpu(a.tickets + kvh * S + split, 1u);
    sm.flags[1] = (t == (unsigned)(Cact - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (TRACE && tid == 0) trace_stamp(trace_slot(a.trace), TRACE_EXIT);  // the merging CTA overwrites it below
  if (sm.flags[1] == 0) return;
  if (tid < G * W) {
    const int r = tid / W, off = tid % W;
    float mx = -INFINITY;
    for (int c = 0; c < Cact; ++c) mx = fmaxf(mx, __ldcg(pl + c * kDecRows + r));
    float den = 0.f, acc = 0.f;
    for (int c = 0; c < Cact; ++c) {
      const float w = exp2f(__ldcg(pl + c * kDecRows + r) - mx);
      den += w;
      acc = fmaf(__ldcg(po + ((size_t)c * kDecRows + r) * kAttnD + split * W + off), w, acc);
    }
    attn_store_out(a, kvh, r, split * W + off, acc / den);
  }
  if (tid == 0) a.tickets[kvh * S + split] = 0u;
  if (TRACE && tid == 0) trace_stamp(trace_slot(a.trace), TRACE_EXIT);
}

}  // namespace qb
