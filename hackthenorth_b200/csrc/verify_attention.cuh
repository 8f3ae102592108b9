// Multi-query decode attention for the verify pass: Q consecutive query
// positions of one sequence (the current token and the draft tokens), GQA
// group G, R = G * Q <= 24 query rows per KV head, as C thread-block clusters
// of S CTAs per KV head (C > 1 from kDecMultiClusterKeys live keys when the
// launch provides merge tickets; the clusters then merge through global
// partial rows as in the decode kernel).
//
// Same arithmetic as the decode kernel (decode_attention.cuh) and the
// reference's partial attention + LSE merge (dryft/engine/kernels/
// attention.py:14-63,200-237): base-2 online softmax, P rounded to bf16 for the
// P.V product, row r (head g = r / Q, query i = r % Q) sees keys <= positions[i]
// (causal by absolute position).
//
// Differences from the decode kernel, for the larger row count:
//  * the rows form NT = ceil(R / 8) n-tiles of the transposed products
//    (S^T = K . Q^T, O^T = V^T . P^T); each 32-key stage is processed one
//    n-tile at a time, so only the O^T accumulators grow with NT;
//  * no producer warp: consumer warp w owns ring slot w, issues its first
//    stage once the positions are known (they come from the previous kernel,
//    so after griddepcontrol.wait; the new rows' K/V are then already in the
//    cache) and, after consuming stage c, refills the slot with stage c + 8
//    itself. Eight warps then have 255 registers each;
//  * the in-CTA merge and the cluster exchange carry R rows.
#pragma once
#include "decode_attention.cuh"

namespace qb {

constexpr int kVaWarps = 8;
constexpr int kVaThreads = kVaWarps * 32;
constexpr int kVaMaxRows = 24;
constexpr int kVaStages = 8;  // ring slots: warp w owns slot w
constexpr int kVaBarrierId = 4;

__host__ inline size_t va_smem_bytes() {
  return 1024 + (size_t)kVaStages * kDecStageBytes          // ring (also the in-CTA merge buffer)
         + kVaMaxRows * kAttnD * 2                           // query rows
         + kVaStages * 8                                    // full barriers
         + kVaWarps * kVaMaxRows * 2 * 4                     // per-warp m, l
         + kVaMaxRows * kAttnD * 4                           // receive slices [split][row][128 / S]
         + kDecMaxCluster * kVaMaxRows * 4                   // receive lse
         + 64;
}
static_assert(kVaWarps * kVaMaxRows * kDecObStride * 4 <= kVaStages * kDecStageBytes, "merge buffer fits the ring");

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int NT>
__global__ void __launch_bounds__(kVaThreads, 1)
    attn_rows_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                     const AttnArgs a) {
  constexpr int ROWS = NT * 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  bf16* qs = reinterpret_cast<bf16*>(ring + kVaStages * kDecStageBytes);  // [ROWS][128]
  uint64_t* full = reinterpret_cast<uint64_t*>(qs + kVaMaxRows * kAttnD);
  float* ml = reinterpret_cast<float*>(full + kVaStages);  // [warp][row][2]
  float* rbuf = ml + kVaWarps * kVaMaxRows * 2;             // [split][row][W]
  float* rlse = rbuf + kVaMaxRows * kAttnD;                 // [split][row]
  volatile int* flags = reinterpret_cast<volatile int*>(rlse + kDecMaxCluster * kVaMaxRows);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int S = a.splits;            // cluster size
  const int C = max(1, a.clusters);  // clusters per KV head
  const int kvh = blockIdx.x / (C * S);
  const int cl = (blockIdx.x / S) % C;
  const int split = blockIdx.x % S;  // == cluster rank
  const int G = a.Hq / a.Hkv;
  const int Qn = a.Q;
  const int R = G * Qn;  // <= ROWS

  cluster_arrive_relaxed();  // first cluster phase, waited before the first remote store
  if (tid == 0) {
    for (int s = 0; s < kVaStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    flags[0] = 0;
  }
  __syncthreads();

  // The newest position bounds the live range (positions ascend). The
  // positions are written by the previous kernel: read after the wait.
  pdl_wait();
  pdl_trigger();
  // batched decode: this KV head's sequence has its own position
  const int64_t* posv = a.batch_hkv > 0 ? a.pos + kvh / a.batch_hkv : a.pos;
  long long last = posv[Qn - 1];
  if (last < 0 || last >= a.cap) {
    if (tid == 0 && blockIdx.x == 0) report_error(a.err, DEV_BAD_POSITION);
    last = -1;
  }
  const int n = (int)last + 1;
  // Splits over the whole head as in the decode kernel: up to C clusters'
  // worth from kDecMultiClusterKeys live keys; cluster cl takes splits
  // [cl*S, cl*S+S) of SeT, every one of which has keys.
  const int cmax = n >= kDecMultiClusterKeys ? C : min(C, max(1, kDecShortSplits / S));
  const int2 sl = attn_split_len(n, min(cmax * S, (n + kAttnMinSplitKeys - 1) / kAttnMinSplitKeys));
  const int per = sl.x, SeT = sl.y;
  const int Cact = (SeT + S - 1) / S;           // clusters with work (uniform over the grid)
  const int Se = max(0, min(S, SeT - cl * S));  // splits of this cluster
  if (Se == 0) {  // a cluster without work leaves at once
    cluster_wait();
    return;
  }
  const int k0 = min(n, (cl * S + split) * per);
  const int k1 = min(n, k0 + per);
  const int nst = (k1 - k0 + kDecKeys - 1) / kDecKeys;
  const bool active = split < Se && nst > 0;

  auto issue = [&](int c) {  // lane 0 of warp c % 8: stage c into slot c % 8
    const int s = c % kVaStages;
    uint8_t* st = ring + s * kDecStageBytes;
    const int y = kvh * a.cap + k0 + c * kDecKeys;
    mbar_arrive_expect_tx(&full[s], kDecStageBytes);
    tma_load_2d(st, &tmk, 0, y, &full[s]);
    tma_load_2d(st + kDecSubTile, &tmk, 64, y, &full[s]);
    tma_load_2d(st + 2 * kDecSubTile, &tmv, 0, y, &full[s]);
    tma_load_2d(st + 3 * kDecSubTile, &tmv, 64, y, &full[s]);
  };
  if (active && lane == 0 && warp < nst) {
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
    issue(warp);
  }

  // Query rows r = g * Q + i into shared memory (zero padded to ROWS).
  for (int i = tid; i < ROWS * kAttnD / 8; i += kVaThreads) {
    const int r = i / (kAttnD / 8), c8 = i % (kAttnD / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < R) {
      const int g = r / Qn, qi = r % Qn;
      v = *reinterpret_cast<const uint4*>(a.q + ((size_t)qi * a.Hq + kvh * G + g) * kAttnD + c8 * 8);
    }
    reinterpret_cast<uint4*>(qs)[i] = v;
  }
  __syncthreads();

  const int g4 = lane >> 2, t4 = lane & 3;
  float val[(ROWS + 1) / 2], lsev[(ROWS + 1) / 2];  // thread's rows (tid >> 7) + 2j, dim tid & 127
  bool ok = true;

  if (active) {
    // Per-row key limits of this thread's C-fragment rows: row nt*8 + 2*t4 + e.
    int lim[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = nt * 8 + 2 * t4 + e;
        lim[nt][e] = r < R ? (int)posv[r % Qn] : -1;
      }
    float o[8][NT][4];
    float m[NT][2], l[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j][nt][0] = o[j][nt][1] = o[j][nt][2] = o[j][nt][3] = 0.f;
      m[nt][0] = m[nt][1] = -INFINITY;
      l[nt][0] = l[nt][1] = 0.f;
    }
    const float scale = 0.12751743082459868f;  // log2(e) / sqrt(128)
    // Query fragments: up to two n-tiles stay in registers for the whole key
    // loop; three are read from shared memory per stage (the registers hold
    // the 96 output accumulators then).
    constexpr int NQH = NT <= 2 ? NT : 1;
    uint32_t qh[NQH][8][2];
    if constexpr (NT <= 2) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t r4[4];
          ldsm_x4(r4, qs + (nt * 8 + (lane & 7)) * kAttnD + j * 32 + (lane >> 3) * 8);
          qh[nt][2 * j][0] = r4[0];
          qh[nt][2 * j][1] = r4[1];
          qh[nt][2 * j + 1][0] = r4[2];
          qh[nt][2 * j + 1][1] = r4[3];
        }
    }
    const int s = warp;
    uint8_t* stage = ring + s * kDecStageBytes;
    for (int c = warp; c < nst; c += kVaWarps) {
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (c / kVaStages) & 1, a.err, DEV_TIMEOUT_ATTN_FULL))) {
        ok = false;
        break;
      }
      const int kstage = k0 + c * kDecKeys;
      const int svalid = k1 - kstage;
      if (svalid < kDecKeys) {
        // Rows past the live range may hold anything (even NaN): clear V there.
        for (int i = lane; i < (kDecKeys - svalid) * 16; i += 32) {
          const int row = svalid + (i >> 4);
          const int sub = (i >> 3) & 1, ch = i & 7;
          *reinterpret_cast<uint4*>(stage + (2 + sub) * kDecSubTile + swz(row, ch)) = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      // Scores and softmax of every n-tile first (P^T fragments kept), then
      // P.V with each V fragment read once for all n-tiles; every output
      // accumulator still adds the two key m-tiles in the same order.
      uint32_t pb[NT][2][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        uint32_t qb[8][2];
        if constexpr (NT <= 2) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            qb[j][0] = qh[nt][j][0];
            qb[j][1] = qh[nt][j][1];
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t r4[4];
            ldsm_x4(r4, qs + (nt * 8 + (lane & 7)) * kAttnD + j * 32 + (lane >> 3) * 8);
            qb[2 * j][0] = r4[0];
            qb[2 * j][1] = r4[1];
            qb[2 * j + 1][0] = r4[2];
            qb[2 * j + 1][1] = r4[3];
          }
        }
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
              x[mt][h] = (key < k1 && key <= lim[nt][e]) ? v : -INFINITY;
              rmax = fmaxf(rmax, x[mt][h]);
            }
          rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 4));
          rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 8));
          rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, 16));
          const float mnew = fmaxf(m[nt][e], rmax);
          // (a row may see no key of a stage: then rmax, and possibly mnew, is -inf)
          corr[e] = (m[nt][e] == -INFINITY) ? 0.f : exp2f(m[nt][e] - mnew);
          float rs = 0.f;
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              p[mt][h][e] = (x[mt][h] == -INFINITY) ? 0.f : exp2f(x[mt][h] - mnew);
              rs += p[mt][h][e];
            }
          l[nt][e] = l[nt][e] * corr[e] + rs;
          m[nt][e] = mnew;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j][nt][0] *= corr[0];
          o[j][nt][1] *= corr[1];
          o[j][nt][2] *= corr[0];
          o[j][nt][3] *= corr[1];
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int h = 0; h < 2; ++h) pb[nt][mt][h] = movmatrix_trans(pack_bf16(p[mt][h][0], p[mt][h][1]));
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) {
          const int mi = lane >> 3;
          const int key = mt * 16 + (lane & 7) + (mi >> 1) * 8;
          const int ch = ((dt & 3) << 1) + (mi & 1);
          uint32_t va[4];
          ldsm_x4_t(va, stage + (2 + (dt >> 2)) * kDecSubTile + swz(key, ch));
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_bf16_16816(o[dt][nt], va, pb[nt][mt][0], pb[nt][mt][1]);
        }
      __syncwarp();
      if (lane == 0 && c + kVaStages < nst) {
        fence_proxy_async_smem();  // this warp's reads of the slot precede the refill
        issue(c + kVaStages);
      }
    }
    if (!ok) {
      // Let the copies this warp issued land before shared memory goes away.
      if (lane == 0)
        for (int c = warp; c < nst; c += kVaWarps) mbar_wait(&full[s], (c / kVaStages) & 1, nullptr, 0);
      flags[0] = 1;
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        l[nt][e] += __shfl_xor_sync(0xffffffffu, l[nt][e], 4);
        l[nt][e] += __shfl_xor_sync(0xffffffffu, l[nt][e], 8);
        l[nt][e] += __shfl_xor_sync(0xffffffffu, l[nt][e], 16);
      }
    named_barrier(kVaBarrierId, kVaThreads);
    ok = flags[0] == 0;
    if (ok) {
      // Merge the 8 warps (fixed order) through the drained ring.
      float* ob = reinterpret_cast<float*>(ring);  // [warp][ROWS][kDecObStride]
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float* r0p = ob + ((size_t)warp * ROWS + nt * 8 + 2 * t4) * kDecObStride;
        float* r1p = r0p + kDecObStride;
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) {
          const int d = dt * 16 + g4;
          r0p[d] = o[dt][nt][0];
          r1p[d] = o[dt][nt][1];
          r0p[d + 8] = o[dt][nt][2];
          r1p[d + 8] = o[dt][nt][3];
        }
        if (g4 == 0) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            ml[(warp * kVaMaxRows + nt * 8 + 2 * t4 + e) * 2] = m[nt][e];
            ml[(warp * kVaMaxRows + nt * 8 + 2 * t4 + e) * 2 + 1] = l[nt][e];
          }
        }
      }
      named_barrier(kVaBarrierId, kVaThreads);
      const int d = tid & 127;
#pragma unroll
      for (int j = 0; j < (ROWS + 1) / 2; ++j) {
        const int r = (tid >> 7) + 2 * j;
        val[j] = 0.f;
        lsev[j] = -INFINITY;
        if (r < R) {
          float M = -INFINITY;
#pragma unroll
          for (int w = 0; w < kVaWarps; ++w) M = fmaxf(M, ml[(w * kVaMaxRows + r) * 2]);
          float L = 0.f, acc = 0.f;
#pragma unroll
          for (int w = 0; w < kVaWarps; ++w) {
            const float mw = ml[(w * kVaMaxRows + r) * 2];
            const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
            L += ml[(w * kVaMaxRows + r) * 2 + 1] * f;
            acc += ob[((size_t)w * ROWS + r) * kDecObStride + d] * f;
          }
          val[j] = L > 0.f ? acc / L : 0.f;
          lsev[j] = L > 0.f ? M + log2f(L) : -INFINITY;
        }
      }
    }
  }

  // ------------------------------------------------------------ cluster merge
  cluster_wait();
  if (Se == 1 && Cact == 1) {  // uniform across the grid
    if (split == 0 && active && ok) {
#pragma unroll
      for (int j = 0; j < (ROWS + 1) / 2; ++j) {
        const int r = (tid >> 7) + 2 * j;
        if (r < R) attn_store_out(a, kvh, r, tid & 127, val[j]);
      }
    }
    return;
  }
  const int W = kAttnD / S;
  if (active && ok) {
    const int d = tid & 127;
    const int owner = d / W;
    const uint32_t rb = map_shared_rank(rbuf, owner);
    const uint32_t rl = map_shared_rank(rlse, owner);
#pragma unroll
    for (int j = 0; j < (ROWS + 1) / 2; ++j) {
      const int r = (tid >> 7) + 2 * j;
      if (r < R) {
        st_cluster_f32(rb + (uint32_t)(((split * R + r) * W + (d - owner * W)) * 4), val[j]);
        if (d == owner * W) st_cluster_f32(rl + (uint32_t)((split * R + r) * 4), lsev[j]);
      }
    }
  }
  cluster_sync_all();
  // Several clusters per head: each CTA publishes its dim slice of the
  // cluster's result (normalised rows + log-sum-exp) to global partial rows;
  // the CTA of the same slice index that draws the last ticket merges the
  // clusters in cluster order. A row may see no key of a later cluster
  // (causal limits): that cluster contributes 0 with weight 0.
  float* po = a.part_o + (size_t)kvh * a.part_splits * kVaMaxRows * kAttnD;
  float* pl = a.part_lse + (size_t)kvh * a.part_splits * kVaMaxRows;
  for (int idx = tid; idx < R * W; idx += kVaThreads) {
    const int r = idx / W, off = idx % W;
    float mx = -INFINITY;
    for (int sp = 0; sp < Se; ++sp) mx = fmaxf(mx, rlse[sp * R + r]);
    float den = 0.f, acc = 0.f;
    if (mx != -INFINITY) {
      for (int sp = 0; sp < Se; ++sp) {
        const float w = exp2f(rlse[sp * R + r] - mx);
        den += w;
        acc = fmaf(rbuf[(sp * R + r) * W + off], w, acc);
      }
    }
    const float cval = den > 0.f ? acc / den : 0.f;
    if (Cact == 1) {
      attn_store_out(a, kvh, r, split * W + off, cval);
    } else {
      po[((size_t)cl * R + r) * kAttnD + split * W + off] = cval;
      if (off == 0) pl[cl * R + r] = den > 0.f ? mx + log2f(den) : -INFINITY;
    }
  }
  if (Cact == 1) return;
  __syncthreads();
  if (tid == 0) {
    const unsigned t = atomic_add_acq_rel_gpu(a.tickets + kvh * S + split, 1u);
    flags[1] = (t == (unsigned)(Cact - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (flags[1] == 0) return;
  for (int idx = tid; idx < R * W; idx += kVaThreads) {
    const int r = idx / W, off = idx % W;
    float mx = -INFINITY;
    for (int c = 0; c < Cact; ++c) mx = fmaxf(mx, __ldcg(pl + c * R + r));
    float den = 0.f, acc = 0.f;
    for (int c = 0; c < Cact; ++c) {
      const float l = __ldcg(pl + c * R + r);
      const float w = l == -INFINITY ? 0.f : exp2f(l - mx);
      den += w;
      acc = fmaf(__ldcg(po + ((size_t)c * R + r) * kAttnD + split * W + off), w, acc);
    }
    attn_store_out(a, kvh, r, split * W + off, den > 0.f ? acc / den : 0.f);
  }
  if (tid == 0) a.tickets[kvh * S + split] = 0u;
}

}  // namespace qb
