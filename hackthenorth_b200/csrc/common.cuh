// common.cuh — sm_100a building blocks shared by the decode kernels:
// mbarrier pipelines, bulk (TMA) copies, programmatic dependent launch, bounded
// waits with an error word, bf16 packing and warp reductions.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qb {

typedef __nv_bfloat16 bf16;

// Device error word values (written once: the first failure wins).
enum DeviceError : int {
  DEV_OK = 0,
  DEV_TIMEOUT_GEMV_FULL = 0x101,
  DEV_TIMEOUT_GEMV_EMPTY = 0x102,
  DEV_TIMEOUT_ATTN_FULL = 0x201,
  DEV_TIMEOUT_ATTN_EMPTY = 0x202,
  DEV_TIMEOUT_PEER_FLAG = 0x401,
  DEV_BAD_TOKEN = 0x301,
  DEV_BAD_POSITION = 0x302,
};

// A wait gives up after this many nanoseconds of polling (about 2 s: far
// beyond any legitimate wait of a decode kernel, short enough that a broken
// pipeline returns control with an error instead of hanging the GPU).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ---- tracing -------------------------------------------------------------------
// Optional %globaltimer stamps (ns) of each CTA of a traced launch, written
// only when the launch carries a trace pointer (qb_set_trace): record
// trace[(launch * kTraceMaxCtas + cta) * kTraceStamps + k] with k =
// TRACE_ENTRY (CTA start), TRACE_WAIT (griddepcontrol.wait returned),
// TRACE_FIRST (first input stage landed), TRACE_LOOP (main loop done,
// epilogue / merge starts), TRACE_EXIT (CTA done). CTAs beyond kTraceMaxCtas
// are not recorded.
constexpr int kTraceMaxCtas = 256;
constexpr int kTraceStamps = 8;
enum TraceStamp : int { TRACE_ENTRY = 0, TRACE_WAIT = 1, TRACE_FIRST = 2, TRACE_LOOP = 3, TRACE_EXIT = 4,
                        // decode attention's merge: in-CTA merge done, cluster wait passed, cluster sync passed
                        TRACE_MERGED = 5, TRACE_CWAIT = 6, TRACE_CSYNC = 7 };
__device__ __forceinline__ unsigned long long* trace_slot(unsigned long long* launch_base) {
  return (launch_base != nullptr && blockIdx.x < kTraceMaxCtas) ? launch_base + (size_t)blockIdx.x * kTraceStamps
                                                                 : nullptr;
}
__device__ __forceinline__ void trace_stamp(unsigned long long* slot, int k) {
  if (slot != nullptr) slot[k] = global_timer_ns();
}

// ---- programmatic dependent launch --------------------------------------------
// Rule used by every kernel here: touch only immutable data (weights) or data
// written at least two launches earlier before pdl_wait(); call
// pdl_trigger() only after pdl_wait(). The dependent grid then overlaps only
// this grid's post-wait part, so its pre-wait reads never race a producer.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- mbarrier ------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity. Returns false (and records
// `code`) if the phase has not completed within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      report_error(err, code);
      return false;
    }
  }
}

// ---- bulk copies (TMA engine) -----------------------------------------------
// 1D bulk copy global -> shared, completion signalled on `bar` as tx bytes.
// src and dst 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// 2D tiled tensor copy global -> shared (coordinates: x innermost). No multicast.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- named barriers (subsets of the CTA) --------------------------------------
__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- bf16 helpers -------------------------------------------------------------
__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ float round_bf16(float f) { return __bfloat162float(__float2bfloat16_rn(f)); }
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float dot8(const uint4 w, const uint4 x, float acc) {
  acc = fmaf(bf_lo(w.x), bf_lo(x.x), acc);
  acc = fmaf(bf_hi(w.x), bf_hi(x.x), acc);
  acc = fmaf(bf_lo(w.y), bf_lo(x.y), acc);
  acc = fmaf(bf_hi(w.y), bf_hi(x.y), acc);
  acc = fmaf(bf_lo(w.z), bf_lo(x.z), acc);
  acc = fmaf(bf_hi(w.z), bf_hi(x.z), acc);
  acc = fmaf(bf_lo(w.w), bf_lo(x.w), acc);
  acc = fmaf(bf_hi(w.w), bf_hi(x.w), acc);
  return acc;
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}
__device__ __forceinline__ uint4 ldg128_nc(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// Ticket counter: one atomic with acquire-release semantics at GPU scope. The
// caller first synchronises its CTA (bar.sync), so every thread's earlier
// writes are released, and the CTA that draws the last ticket acquires all
// other CTAs' writes.
__device__ __forceinline__ unsigned atomic_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
// System-scope flag handshake for peer-to-peer reductions over NVLink.
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait for a 64-bit word whose high half equals `token`; returns its
// low half (fp32 bits). One aligned 64-bit store carries both halves, so a
// matching token means the value beside it is the one that was sent.
__device__ __forceinline__ float wait_tagged(const unsigned long long* p, uint32_t token, int* err, int code) {
  unsigned long long w = ld_relaxed_sys_u64(p);
  if ((uint32_t)(w >> 32) == token) return __uint_as_float((uint32_t)w);
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 32; ++i) {
      w = ld_relaxed_sys_u64(p);
      if ((uint32_t)(w >> 32) == token) return __uint_as_float((uint32_t)w);
    }
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      report_error(err, code);
      return 0.f;
    }
  }
}
// Bounded wait until *p >= v (another GPU's release store); false on timeout.
__device__ __forceinline__ bool wait_flag_geq(const unsigned long long* p, unsigned long long v, int* err, int code) {
  if (ld_acquire_sys_u64(p) >= v) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (ld_acquire_sys_u64(p) >= v) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      report_error(err, code);
      return false;
    }
  }
}
// Coherent (L1-bypassing) load for data written by other CTAs of this grid.
__device__ __forceinline__ float ldcg_f32(const float* p) { return __ldcg(p); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// SiLU in fp32: x * sigmoid(x), computed as x / (1 + exp(-x)) with CUDA's expf.
__device__ __forceinline__ float silu_f32(float x) { return x / (1.0f + expf(-x)); }

}  // namespace qb
