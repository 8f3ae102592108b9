// qb.cu — C ABI of the B200 batch-one Qwen3 decode engine (see include/qb.h).
//
// One decode step is 5 launches per layer plus the head:
//   gemv<STORE>     RMSNorm + QKV           (layer 0 also gathers the embedding)
//   attn<PRO>       q/k norm + RoPE + KV append + split-KV attention + merge
//   gemv<RESIDUAL>  o-proj + residual
//   gemv<SWIGLU>    RMSNorm + gate/up + SiLU * up
//   gemv<RESIDUAL>  down + residual
//   gemv<ARGMAX>    final RMSNorm + LM head + greedy argmax, position += 1
// every launch carries the programmatic-stream-serialization attribute, so in
// a stream or a captured graph each kernel starts streaming its weights while
// its predecessor drains.
#include "../../include/qb.h"

#include <nccl.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "attention.cuh"
#include "decode_attention.cuh"
#include "gemv_rows.cuh"
#include "verify_attention.cuh"
#include "prefill_gemm.cuh"
#include "prefill_attention.cuh"
#include "prefill_attention_tc.cuh"
#include "common.cuh"
#include "gemv.cuh"

using namespace qb;

namespace {

thread_local std::string g_last_error = "";

// Per-CTA shared-memory budget of the GEMV: two CTAs of consecutive kernels
// fit on one SM (228 KB), which is what lets PDL overlap them.
// QB_GEMV_SMEM_KB overrides the budget (tuning: a deeper ring keeps more bytes
// in flight per SM but stops the next kernel's CTAs from co-residing).
constexpr size_t kGemvSmemBudgetDefault = 220 * 1024;
constexpr int kMaxGemvStages = 12;
constexpr size_t kOpScratchBytes = 16u << 20;

// Op-level scratch layout (bytes).
constexpr int kOpRowsMaxCap = 16384;     // op attention: cluster rows kernel below this capacity
constexpr size_t kScrErr = 0;
constexpr size_t kScrCounters = 256;       // unsigned[192]
constexpr size_t kScrHeadVal = 1024;       // float[1024]
constexpr size_t kScrHeadIdx = 5120;       // int[1024]
constexpr size_t kScrAttnLse = 9216;       // float[16384]
constexpr size_t kScrAttnO = 9216 + 65536; // float[...] up to the tickets
constexpr size_t kScrTickets = kOpScratchBytes - 4096;  // unsigned[64 heads x 16]: rows-kernel cluster merges
constexpr int kMaxAttnCtas = 512;

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int set_err(std::string* dst, int code, const std::string& msg) {
  if (dst) *dst = msg;
  g_last_error = msg;
  return code;
}

int cuda_fail(std::string* dst, cudaError_t e, const char* what) {
  return set_err(dst, QB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int sm_count_of(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
  return n;
}

int current_sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  return sm_count_of(dev);
}

// Function attributes (cudaFuncSetAttribute) and occupancy results belong to
// one device, so everything this file caches about them is kept per device and
// looked up with the caller's device current. A device index beyond the table
// gets a fresh entry on every call (attributes set again, occupancy queried
// again): correct, only slower.
constexpr int kMaxDevices = 64;
struct DeviceCache {
  bool gemv_attr[5] = {};
  bool pg_attr[4] = {};
  bool attn_attr[2][2] = {};  // [MT - 1][PRO]
  bool rows_attr[5] = {};
  bool ft_attr = false;
  // attn_decode_kernel: cluster size for (hkv, rows) and clusters of 16/8/4 CTAs held at once
  int dec_hkv = -1, dec_rows = -1, dec_cs = 0;
  int dec_active[3] = {0, 0, 0};
  // attn_rows_kernel: cluster size for hkv and clusters of 16/8/4 CTAs held at once
  int rows_hkv = -1, rows_cs = 0;
  int rows_active[3] = {0, 0, 0};
  int batch_attrs = -1;
};
DeviceCache g_dev_cache[kMaxDevices];
std::mutex g_dev_cache_mu;  // guards the occupancy entries while they are computed

DeviceCache& dev_cache() {
  int d = 0;
  if (cudaGetDevice(&d) == cudaSuccess && d >= 0 && d < kMaxDevices) return g_dev_cache[d];
  static thread_local DeviceCache overflow;
  overflow = DeviceCache();
  return overflow;
}

bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("QB_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                      Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------- GEMV launch
struct GemvPlan {
  int grid, stages, max_rows, kc;
  size_t smem;
};

int gemv_kc_pref() {
  static int v = 0;
  if (v == 0) {
    const char* e = std::getenv("QB_GEMV_KC");
    v = (e && std::strtol(e, nullptr, 10) == 1024) ? 1024 : 2048;
  }
  return v;
}

size_t gemv_smem_budget() {
  static size_t v = 0;
  if (v == 0) {
    const char* e = std::getenv("QB_GEMV_SMEM_KB");
    long kb = e ? std::strtol(e, nullptr, 10) : 0;
    v = (kb >= 48 && kb <= 227) ? (size_t)kb * 1024 : kGemvSmemBudgetDefault;
  }
  return v;
}

bool plan_gemv(int epi, int K, int rows, int sm_count, GemvPlan* p) {
  const size_t kGemvSmemBudget = gemv_smem_budget();
  const int rpu = gemv_rows_per_unit(epi);
  const int units = rows / rpu;
  if (units <= 0) return false;
  p->grid = units < sm_count ? units : sm_count;
  p->max_rows = ((units + p->grid - 1) / p->grid) * rpu;
  const size_t fixed = gemv_smem_bytes(K, 0, p->max_rows, 1024);
  // Wider pieces when K allows and the ring still holds >= 3 of them.
  int kc = (K >= 2048 && gemv_kc_pref() == 2048) ? 2048 : 1024;
  if (kc == 2048 && (fixed + 3 * (size_t)(gemv_stage_bytes(2048) + 16) > kGemvSmemBudget)) kc = 1024;
  int stages = 0;
  if (fixed < kGemvSmemBudget) stages = (int)((kGemvSmemBudget - fixed) / (gemv_stage_bytes(kc) + 16));
  if (stages > kMaxGemvStages) stages = kMaxGemvStages;
  if (stages < 2) stages = 2;
  p->kc = kc;
  p->stages = stages;
  p->smem = gemv_smem_bytes(K, stages, p->max_rows, kc);
  return p->smem <= 227 * 1024;
}

template <int EPI>
cudaError_t launch_gemv(GemvArgs a, int sm_count, cudaStream_t st) {
  bool& attr_done = dev_cache().gemv_attr[EPI];
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<EPI, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemv_kernel<EPI, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  GemvPlan p;
  if (!plan_gemv(EPI, a.K, a.rows, sm_count, &p)) return cudaErrorInvalidValue;
  a.stages = p.stages;
  a.max_rows = p.max_rows;
  a.kc = p.kc;
  // the traced instantiation only when this launch records timestamps
  if (a.trace != nullptr) return launch_ex(gemv_kernel<EPI, true>, dim3(p.grid), dim3(kGemvThreads), p.smem, st, a);
  return launch_ex(gemv_kernel<EPI, false>, dim3(p.grid), dim3(kGemvThreads), p.smem, st, a);
}

// The GEMV launched after `a` in the step (its weights, shape and epilogue):
// `a`'s CTAs bring its first stages into L2 (gemv.cuh).
void set_next_gemv(GemvArgs& a, int epi, const void* w, int K, int rows, int sm_count) {
  GemvPlan p;
  if (std::getenv("QB_GEMV_L2_NEXT") && std::getenv("QB_GEMV_L2_NEXT")[0] == '0') return;
  if (!plan_gemv(epi, K, rows, sm_count, &p)) return;
  a.nx_w = static_cast<const bf16*>(w);
  a.nx_K = K;
  a.nx_rows = rows;
  a.nx_rpu = gemv_rows_per_unit(epi);
  a.nx_kc = p.kc;
  a.nx_grid = p.grid;
}

GemvArgs gemv_args(const void* w, int K, int rows, const void* x, void* out, int* err) {
  GemvArgs a;
  std::memset(&a, 0, sizeof(a));
  a.w = static_cast<const bf16*>(w);
  a.K = K;
  a.rows = rows;
  a.x = static_cast<const bf16*>(x);
  a.out = static_cast<bf16*>(out);
  a.err = err;
  return a;
}

// ----------------------------------------------------------- attention launch
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Tensor map over one layer's cache viewed as [Hkv*cap rows][128 dims] bf16,
// box [rows][64 dims] (64 rows for attn_kernel, 32 for attn_decode_kernel),
// 128-byte swizzle; out-of-range rows read as zero.
bool make_kv_map(CUtensorMap* m, const void* base, int hkv, int cap, int rows = kAttnKeys) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  cuuint64_t dims[2] = {(cuuint64_t)kAttnD, (cuuint64_t)hkv * (cuuint64_t)cap};
  cuuint64_t strides[1] = {(cuuint64_t)kAttnD * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor map over a row-major [rows][cols] bf16 matrix, box [box_rows][64
// cols], 128-byte swizzle (the K-major operand tiles of the prefill GEMM).
bool make_rows_map(CUtensorMap* m, const void* base, long long rows, long long cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (cols * 2) % 16 != 0) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// D[T][N] = X[T][K] . W[N][K]^T on tcgen05 (prefill_gemm_kernel).
// 3D map over the prompt rows' queries q[T][Hq][128] (dims innermost): boxes of
// [rows][G heads][64 dims] (128-byte swizzle) for flash_prefill_tc_kernel.
bool make_q3_map(CUtensorMap* m, const void* q, int T, int Hq, int G, int rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(q) & 15) != 0) return false;
  cuuint64_t dims[3] = {(cuuint64_t)kAttnD, (cuuint64_t)Hq, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)kAttnD * 2, (cuuint64_t)Hq * kAttnD * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)G, (cuuint32_t)rows};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// extra: the fields of the QKV_ROPE epilogue and the residual stride (the rest are set here).
cudaError_t launch_prefill_gemm(int epi, const bf16* x, const bf16* w, bf16* out, const bf16* residual, int T, int N,
                                int K, int* err, cudaStream_t st, const PgArgs* extra = nullptr) {
  CUtensorMap tx, tw;
  if (!make_rows_map(&tx, x, T, K, kPgBM) || !make_rows_map(&tw, w, N, K, kPgBN)) return cudaErrorInvalidValue;
  PgArgs a;
  if (extra != nullptr) a = *extra;
  else std::memset(&a, 0, sizeof(a));
  a.T = T;
  a.N = N;
  a.K = K;
  a.out = out;
  a.residual = residual;
  a.err = err;
  const size_t smem = pg_smem_bytes();
  bool* attr = dev_cache().pg_attr;
  void (*k)(const CUtensorMap, const CUtensorMap, const PgArgs) =
      epi == PG_STORE      ? prefill_gemm_kernel<PG_STORE>
      : epi == PG_RESIDUAL ? prefill_gemm_kernel<PG_RESIDUAL>
      : epi == PG_SWIGLU   ? prefill_gemm_kernel<PG_SWIGLU>
                           : prefill_gemm_kernel<PG_QKV_ROPE>;
  if (!attr[epi]) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr[epi] = true;
  }
  // persistent: one CTA per SM (at most one per tile)
  const long long tiles = (long long)((T + kPgBM - 1) / kPgBM) * ((N + kPgBN - 1) / kPgBN);
  const int grid = (int)std::min<long long>(tiles, current_sm_count());
  return launch_ex(k, dim3(grid), dim3(kPgThreads), smem, st, tx, tw, a);
}

int attn_splits_for(int hkv, int sm_count) {
  int s = sm_count / hkv;
  if (s < 1) s = 1;
  return s;
}

template <int MT, bool PRO>
cudaError_t launch_attn_t(const CUtensorMap& tk, const CUtensorMap& tv, const AttnArgs& a, cudaStream_t st) {
  bool& attr_done = dev_cache().attn_attr[MT - 1][PRO ? 1 : 0];
  const size_t smem = attn_smem_bytes(MT);
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(attn_kernel<MT, PRO>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  return launch_ex(attn_kernel<MT, PRO>, dim3(a.Hkv * a.splits), dim3(kAttnThreads), smem, st, tk, tv, a);
}

// Batch-one decode attention as thread-block clusters per KV head
// (attn_decode_kernel). Returns the cluster size for `hkv` heads of `rows`
// query rows (16 when 16-CTA clusters of this kernel fit `hkv` at once, else
// 8), or 0 when the kernel does not apply (then attn_kernel is used).
// QB_ATTN_CLUSTER=0 disables it. Also records how many clusters of 16, 8 and 4
// CTAs the GPU holds at once (DeviceCache::dec_active), for launch_attn_decode's
// long-context choice.
constexpr int kDecSizes[3] = {16, 8, 4};

typedef void (*DecKernelFn)(const CUtensorMap, const CUtensorMap, const AttnArgs);
// The traced instantiation records timestamps (qb_set_trace); the other has no trace code.
DecKernelFn dec_kernel(bool trace = false) { return trace ? attn_decode_kernel<true> : attn_decode_kernel<false>; }

int decode_cluster_size(int hkv, int rows) {
  DeviceCache& dc = dev_cache();
  std::lock_guard<std::mutex> lock(g_dev_cache_mu);
  if (hkv == dc.dec_hkv && rows == dc.dec_rows) return dc.dec_cs;
  dc.dec_hkv = hkv;
  dc.dec_rows = rows;
  dc.dec_cs = 0;
  const char* e = std::getenv("QB_ATTN_CLUSTER");
  if (e && e[0] == '0') return 0;
  if (rows > kDecRows) return 0;
  const size_t smem = dec_smem_bytes();
  for (int t = 0; t < 2; ++t) {
    if (cudaFuncSetAttribute(dec_kernel(t), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return 0;
    cudaFuncSetAttribute(dec_kernel(t), cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  }
  for (int i = 0; i < 3; ++i) {
    const int cs = kDecSizes[i];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(hkv * cs);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, dec_kernel(), &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    dc.dec_active[i] = n;
    if (dc.dec_cs == 0 && cs >= 8 && n >= hkv) dc.dec_cs = cs;
  }
  return dc.dec_cs;
}

// Decode-step SM partition around attention (bit 0: o-proj, bit 1: QKV).
// Default (-1): both, when the attention launch holds at most 1/8 of the SMs
// (one KV head per GPU: tensor parallel 8); QB_PART=0..3 forces the bits.
// Measured (one B200): with 16 attention CTAs (Qwen3-8B shapes of one of 8
// tensor-parallel ranks) 956 -> 986 tok/s; with 64 (8 KV heads) slower, 348 ->
// 325 tok/s at 8B and 1461 -> 1402 at 0.6B: one SM pulls at most ~60 GB/s, so
// GEMVs on 84 SMs lose bandwidth.
int gemv_partition() {
  static int v = -2;
  if (v == -2) {
    const char* e = std::getenv("QB_PART");
    v = e ? (int)(std::strtol(e, nullptr, 10) & 3) : -1;
  }
  return v;
}

// Capacity (and live keys) from which decode attention runs several clusters
// per KV head: kDecMultiClusterKeys, or QB_ATTN_MULTI_KEYS.
int dec_multi_keys() {
  static int v = 0;
  if (v == 0) {
    const char* e = std::getenv("QB_ATTN_MULTI_KEYS");
    const long x = e ? std::strtol(e, nullptr, 10) : 0;
    v = (x >= 256 && x <= (1 << 24)) ? (int)x : kDecMultiClusterKeys;
  }
  return v;
}

// The launch shape of decode attention (attn_decode_kernel) for `a`: cluster
// size (a.splits) and clusters per KV head (a.clusters).
void dec_shape(AttnArgs& a, int cs) {
  a.splits = cs;
  a.clusters = 1;
  a.multi_keys = dec_multi_keys();
  // Long contexts: the cluster size and clusters per KV head that put the
  // most CTAs to work at once (several clusters merge through tickets and
  // partial rows in global memory), e.g. 8 heads x 4 clusters x 4 CTAs.
  if (a.tickets != nullptr && a.part_splits >= 2 && a.cap >= a.multi_keys) {
    int best = a.Hkv * cs;
    for (int i = 0; i < 3; ++i) {
      const int s = kDecSizes[i];
      const int c = std::min({kDecMaxClusters, a.part_splits, dev_cache().dec_active[i] / a.Hkv,
                              current_sm_count() / (a.Hkv * s)});
      if (c >= 1 && a.Hkv * c * s > best) {
        best = a.Hkv * c * s;
        a.splits = s;
        a.clusters = c;
      }
    }
  }
}

// CTAs of the decode attention launch for `a` (launch_attn with the prologue,
// one query row), or 0 when attn_decode_kernel does not apply.
int dec_ctas(const AttnArgs& a) {
  if (a.Q != 1) return 0;
  const int cs = decode_cluster_size(a.Hkv, a.Hq / a.Hkv);
  if (cs <= 0) return 0;
  AttnArgs t = a;
  dec_shape(t, cs);
  return t.Hkv * t.clusters * t.splits;
}

cudaError_t launch_attn_decode(const CUtensorMap& tk, const CUtensorMap& tv, AttnArgs a, int cs, cudaStream_t st) {
  dec_shape(a, cs);
  static bool reported = false;
  if (!reported && std::getenv("QB_VERBOSE")) {
    reported = true;
    std::fprintf(stderr, "qb: decode attention: %d KV heads x %d clusters x %d CTAs (GPU holds %d/%d/%d clusters of 16/8/4)\n",
                 a.Hkv, a.clusters, a.splits, dev_cache().dec_active[0], dev_cache().dec_active[1],
                 dev_cache().dec_active[2]);
  }
  cs = a.splits;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.Hkv * a.clusters * cs);
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = dec_smem_bytes();
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, dec_kernel(a.trace != nullptr), tk, tv, a);
}

// Verify-pass attention (attn_rows_kernel, R = G * Q <= 24 rows) as one
// cluster per KV head: the cluster size (16 or 8) or 0 when it does not fit.
// Also records how many clusters of 16, 8 and 4 CTAs the GPU holds at once
// (DeviceCache::rows_active), for rows_attn_shape.
int rows_cluster_size(int hkv) {
  DeviceCache& dc = dev_cache();
  std::lock_guard<std::mutex> lock(g_dev_cache_mu);
  if (hkv == dc.rows_hkv) return dc.rows_cs;
  dc.rows_hkv = hkv;
  dc.rows_cs = 0;
  const char* e = std::getenv("QB_ATTN_CLUSTER");
  if (e && e[0] == '0') return 0;
  const size_t smem = va_smem_bytes();
  void (*kernels[3])(const CUtensorMap, const CUtensorMap, const AttnArgs) = {
      attn_rows_kernel<1>, attn_rows_kernel<2>, attn_rows_kernel<3>};
  for (auto k : kernels) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
        cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
  }
  for (int i = 0; i < 3; ++i) {
    const int cs = kDecSizes[i];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(hkv * cs);
    cfg.blockDim = dim3(kVaThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, attn_rows_kernel<3>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    dc.rows_active[i] = n;
    if (dc.rows_cs == 0 && cs >= 8 && n >= hkv) dc.rows_cs = cs;
  }
  return dc.rows_cs;
}

// Cluster size and clusters per KV head for the rows attention of a verify
// pass: one cluster of rows_cluster_size(hkv) CTAs below kDecMultiClusterKeys
// of capacity; above it the size and count that put the most CTAs to work at
// once (the clusters merge through tickets and partial rows).
void rows_attn_shape(AttnArgs& a, int cs) {
  a.splits = cs;
  a.clusters = 1;
  if (a.tickets == nullptr || a.cap < kDecMultiClusterKeys) return;
  // The kernel keeps part_splits * kVaMaxRows partial rows per KV head and
  // cluster cl writes rows cl * R + r (R <= kVaMaxRows), so at most
  // part_splits clusters stay inside their head's rows.
  const int cmax = std::min(kDecMaxClusters, a.part_splits);
  int best = a.Hkv * cs;
  for (int i = 0; i < 3; ++i) {
    const int s = kDecSizes[i];
    const int c = std::min({cmax, dev_cache().rows_active[i] / a.Hkv, current_sm_count() / (a.Hkv * s)});
    if (c >= 2 && a.Hkv * c * s > best) {
      best = a.Hkv * c * s;
      a.splits = s;
      a.clusters = c;
    }
  }
}

// Cluster size for the rows attention kernel over `vheads` KV heads of several
// sequences (batched decode): the largest power of two <= 16 with every
// cluster resident at once when possible (vheads * cs <= SMs); clusters do not
// wait on each other, so more than fit at once is still correct. 0 when the
// kernel's attributes cannot be set.
int batch_attn_cluster(int vheads, int sm_count) {
  int& attrs = dev_cache().batch_attrs;
  if (attrs < 0) {
    attrs = 1;
    void (*kernels[3])(const CUtensorMap, const CUtensorMap, const AttnArgs) = {
        attn_rows_kernel<1>, attn_rows_kernel<2>, attn_rows_kernel<3>};
    for (auto k : kernels)
      if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)va_smem_bytes()) != cudaSuccess ||
          cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        cudaGetLastError();
        attrs = 0;
      }
  }
  if (!attrs) return 0;
  int cs = 16;
  while (cs > 1 && vheads * cs > sm_count) cs >>= 1;
  return cs;
}

cudaError_t launch_attn_rows(const CUtensorMap& tk, const CUtensorMap& tv, AttnArgs a, int cs, cudaStream_t st) {
  if (a.clusters <= 1) {  // one cluster of cs CTAs per KV head
    a.splits = cs;
    a.clusters = 1;
  }
  const int rows = (a.Hq / a.Hkv) * a.Q;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.Hkv * a.clusters * a.splits);
  cfg.blockDim = dim3(kVaThreads);
  cfg.dynamicSmemBytes = va_smem_bytes();
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  if (rows <= 8) return cudaLaunchKernelEx(&cfg, attn_rows_kernel<1>, tk, tv, a);
  if (rows <= 16) return cudaLaunchKernelEx(&cfg, attn_rows_kernel<2>, tk, tv, a);
  return cudaLaunchKernelEx(&cfg, attn_rows_kernel<3>, tk, tv, a);
}

// tk/tv: 64-row-box maps (attn_kernel); dk/dv: 32-row-box maps of the same
// caches (attn_decode_kernel), or null.
cudaError_t launch_attn(const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap* dk, const CUtensorMap* dv,
                        const AttnArgs& a, bool pro, cudaStream_t st) {
  if (pro && a.Q == 1 && dk != nullptr && dv != nullptr) {
    const int cs = decode_cluster_size(a.Hkv, a.Hq / a.Hkv);
    if (cs > 0) return launch_attn_decode(*dk, *dv, a, cs, st);
  }
  const int rows = (a.Hq / a.Hkv) * a.Q;
  if (pro) return launch_attn_t<1, true>(tk, tv, a, st);
  if (rows <= 16) return launch_attn_t<1, false>(tk, tv, a, st);
  return launch_attn_t<2, false>(tk, tv, a, st);
}

bool ptr_ok(const void* p) { return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

// =================================================================== context
struct qb_ctx {
  qb_config cfg;  // the whole model
  qb_config lc;   // this rank's shard: Hq/n, Hkv/n, F/n, V/n (equal to cfg without tensor parallelism)
  int device = 0;
  int tp_rank = 0, tp_size = 1;
  int batch = 1;                    // sequences decoded together (qb_set_batch; cache [L][B][Hkv][cap][D])
  ncclComm_t comm = nullptr;
  bool p2p = false;                 // peer-memory reduction (else NCCL all-reduce)
  void* tp_base = nullptr;          // this rank's [tagged receive words | epoch] allocation
  TpPeers peers = {};               // every rank's receive words (peers IPC-mapped)
  unsigned long long* tp_epoch() { return const_cast<unsigned long long*>(peers.epoch); }
  float* y32 = nullptr;    // [H] fp32 partial sums, all-reduced across ranks
  float* pairs = nullptr;  // [2] this rank's {max, index}; then [2 * tp_size] gathered
  int sm_count = 148;
  std::vector<qb_layer_weights> layers;
  // tensor-parallel block prefill: rows [r*H/n, (r+1)*H/n) of o and down
  std::vector<const bf16*> o_rows, down_rows;
  const bf16* embed = nullptr;
  const bf16* final_norm = nullptr;
  const bf16* lm_head = nullptr;
  bool weights_bound = false;
  bool state_bound = false;
  bf16* kc = nullptr;
  bf16* vc = nullptr;
  int cap = 0;
  const bf16* cos = nullptr;
  const bf16* sin = nullptr;
  uint8_t* ws = nullptr;
  size_t ws_bytes = 0;
  int* err = nullptr;
  unsigned* counters = nullptr;
  float* head_val = nullptr;
  int* head_idx = nullptr;
  bf16 *xa = nullptr, *xb = nullptr, *qkv = nullptr, *attn = nullptr, *act = nullptr;
  float* part_o = nullptr;
  float* part_lse = nullptr;
  int splits = 1;
  std::vector<CUtensorMap> tmk, tmv;  // 64-row boxes
  std::vector<CUtensorMap> dmk, dmv;  // 32-row boxes (decode kernel)
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  // verify pass (k+1 rows)
  bf16 *r_xa = nullptr, *r_xb = nullptr, *r_qkv = nullptr, *r_q = nullptr, *r_attn = nullptr, *r_act = nullptr;
  int64_t* r_pos = nullptr;
  float* r_val = nullptr;
  int* r_idx = nullptr;
  float* r_y32 = nullptr;    // tensor parallel verify: [rows][H] fp32 partial sums
  float* r_pairs = nullptr;  // tensor parallel verify: [rows][2] + [tp][rows][2]
  cudaGraph_t vgraph = nullptr;
  cudaGraphExec_t vexec = nullptr;
  // tracing (qb_set_trace): launch i of the decode step records its CTAs'
  // stamps at trace + i * kTraceMaxCtas * kTraceStamps
  unsigned long long* trace = nullptr;
  size_t trace_launches = 0;  // capacity of the buffer in launches
  int trace_next = 0;         // next launch index while a step is built
  std::string trace_labels;   // one label per traced launch, '\n'-terminated
  std::string msg;
};

namespace {

struct WsLayout {
  size_t err, counters, head_val, head_idx, xa, xb, qkv, attn, act, part_lse, part_o, y32, pairs;
  // verify pass: up to kRowsMaxQ rows
  size_t r_xa, r_xb, r_qkv, r_q, r_attn, r_act, r_pos, r_val, r_idx, r_y32, r_pairs, total;
};

WsLayout ws_layout(const qb_ctx* c) {
  const qb_config& g = c->lc;
  WsLayout L;
  size_t o = 0;
  L.err = o; o += 256;
  L.counters = o; o += 4096;  // [0,64) attention, 64/66 heads, [512,..) decode clusters
  L.head_val = o; o = align_up(o + 4 * 1024, 256);
  L.head_idx = o; o = align_up(o + 4 * 1024, 256);
  L.xa = o; o = align_up(o + (size_t)g.hidden * 2, 256);
  L.xb = o; o = align_up(o + (size_t)g.hidden * 2, 256);
  L.qkv = o; o = align_up(o + (size_t)(g.n_heads + 2 * g.n_kv_heads) * g.head_dim * 2, 256);
  L.attn = o; o = align_up(o + (size_t)g.n_heads * g.head_dim * 2, 256);
  L.act = o; o = align_up(o + (size_t)g.ffn * 2, 256);
  const size_t parts = (size_t)g.n_kv_heads * c->splits * 32;
  L.part_lse = o; o = align_up(o + parts * 4, 256);
  L.part_o = o; o = align_up(o + parts * kAttnD * 4, 256);
  L.y32 = o; o = align_up(o + (size_t)g.hidden * 4, 256);
  L.pairs = o; o = align_up(o + (size_t)(2 + 2 * c->tp_size) * 4, 256);
  const int nqkv = (g.n_heads + 2 * g.n_kv_heads) * g.head_dim;
  const size_t R = kRowsMaxQ;
  L.r_xa = o; o = align_up(o + R * g.hidden * 2, 256);
  L.r_xb = o; o = align_up(o + R * g.hidden * 2, 256);
  L.r_qkv = o; o = align_up(o + R * nqkv * 2, 256);
  L.r_q = o; o = align_up(o + R * g.n_heads * g.head_dim * 2, 256);
  L.r_attn = o; o = align_up(o + R * g.n_heads * g.head_dim * 2, 256);
  L.r_act = o; o = align_up(o + R * g.ffn * 2, 256);
  L.r_pos = o; o = align_up(o + R * 8, 256);
  L.r_val = o; o = align_up(o + R * 1024 * 4, 256);
  L.r_idx = o; o = align_up(o + R * 1024 * 4, 256);
  L.r_y32 = o; o = align_up(o + (c->tp_size > 1 ? R * g.hidden * 4 : 0), 256);
  L.r_pairs = o; o = align_up(o + R * 2 * (1 + (size_t)c->tp_size) * 4, 256);
  L.total = o;
  return L;
}

int validate_config(const qb_config* g, std::string* msg) {
  if (!g) return set_err(msg, QB_ERR_ARG, "config is NULL");
  if (g->head_dim != 128) return set_err(msg, QB_ERR_UNSUPPORTED, "kernels implement head_dim == 128 only");
  if (g->n_kv_heads <= 0 || g->n_heads <= 0 || g->n_heads % g->n_kv_heads != 0)
    return set_err(msg, QB_ERR_ARG, "n_heads must be a positive multiple of n_kv_heads");
  if (g->n_heads / g->n_kv_heads > 16) return set_err(msg, QB_ERR_UNSUPPORTED, "GQA group above 16");
  if (g->n_kv_heads > 64) return set_err(msg, QB_ERR_UNSUPPORTED, "more than 64 KV heads");
  const int ks[3] = {g->hidden, g->n_heads * g->head_dim, g->ffn};
  for (int k : ks)
    if (k <= 0 || k % 256 != 0) return set_err(msg, QB_ERR_UNSUPPORTED, "hidden, Hq*D and ffn must be multiples of 256");
  if (g->n_layers <= 0 || g->vocab <= 0) return set_err(msg, QB_ERR_ARG, "n_layers and vocab must be positive");
  if (g->hidden > 16384 || g->ffn > 65536) return set_err(msg, QB_ERR_UNSUPPORTED, "hidden/ffn too large for one CTA's x row");
  return QB_OK;
}


// The trace records of the next launch of the step being built (NULL when
// tracing is off or the buffer is full), and its label.
unsigned long long* next_trace(qb_ctx* c, const char* label, int layer) {
  if (c->trace == nullptr || (size_t)c->trace_next >= c->trace_launches) return nullptr;
  char buf[64];
  std::snprintf(buf, sizeof(buf), "%s %d\n", label, layer);
  c->trace_labels += buf;
  return c->trace + (size_t)(c->trace_next++) * kTraceMaxCtas * kTraceStamps;
}

// One decode row through every layer. tok_in: device id; pos: device position
// (read, then incremented by the last kernel). head=false skips the LM head
// and lets the last down-projection increment the position (prefill rows).
// Under tensor parallelism (tp_size > 1) the o-proj and down GEMVs write fp32
// partial sums, one NCCL all-reduce per sublayer combines them, and the next
// GEMV's prologue rounds the sum, adds the residual and stores the new
// residual stream; the LM head picks the greedy token across vocabulary
// shards with an 8-byte all-gather.
int run_rows_decode(qb_ctx* c, const int64_t* tok_in, int64_t* tok_out, int64_t* pos, void* logits, bool head,
                    cudaStream_t st) {
  const qb_config& g = c->lc;
  const int H = g.hidden, D = g.head_dim;
  const int nqkv = (g.n_heads + 2 * g.n_kv_heads) * D;
  const bool tp = c->tp_size > 1;
  const bool p2p = tp && c->p2p;
  cudaError_t e;
  ncclResult_t nr;
  if (head) {  // a decode step: its launches are traced from index 0
    c->trace_next = 0;
    c->trace_labels.clear();
  }
  // NCCL fallback: the next GEMV finishes the all-reduced sum (round + residual).
  auto peer_reduce = [&](GemvArgs& a, int sub, int parity) {
    a.tp = c->peers;
    a.tp_sub = sub;
    a.tp_parity = parity;
    a.hidden = H;
  };
  auto consume = [&](GemvArgs& a, const bf16* res, bf16* copy) {
    a.x = nullptr;
    a.x_res = res;
    a.x_copy = copy;
    a.x32 = c->y32;
  };
  const int part = gemv_partition();
  for (int l = 0; l < g.n_layers; ++l) {
    const qb_layer_weights& w = c->layers[l];
    // attention of this layer (launched after the QKV GEMV)
    AttnArgs at;
    std::memset(&at, 0, sizeof(at));
    at.qkv = c->qkv;
    at.q_norm = static_cast<const bf16*>(w.q_norm);
    at.k_norm = static_cast<const bf16*>(w.k_norm);
    at.cos = c->cos;
    at.sin = c->sin;
    at.eps = g.rms_eps;
    at.pos = pos;
    const size_t layer_off = (size_t)l * g.n_kv_heads * c->cap * D;
    at.k_cache = c->kc + layer_off;
    at.v_cache = c->vc + layer_off;
    at.out = c->attn;
    at.part_o = c->part_o;
    at.part_lse = c->part_lse;
    at.counters = c->counters;
    at.err = c->err;
    at.Hq = g.n_heads;
    at.Hkv = g.n_kv_heads;
    at.Q = 1;
    at.cap = c->cap;
    at.splits = c->splits;
    at.part_splits = c->splits;
    at.tickets = c->counters + 512;
    // SM partition around attention (gemv_partition): the QKV and o-proj
    // GEMVs on the SMs attention does not hold (grid = SMs - attention CTAs),
    // so attention's CTAs find free SMs while the QKV GEMV streams and every
    // o-proj CTA starts (and prefetches its weights) during attention.
    const int attn_n = part != 0 ? dec_ctas(at) : 0;
    const int bits = part >= 0 ? part : (attn_n > 0 && 8 * attn_n <= c->sm_count ? 3 : 0);
    const int free_sms = (attn_n > 0 && 2 * attn_n <= c->sm_count) ? c->sm_count - attn_n : c->sm_count;
    const int qkv_sms = (bits & 2) ? free_sms : c->sm_count;
    const int o_sms = (bits & 1) ? free_sms : c->sm_count;
    // 1. RMSNorm + QKV (layer 0 gathers the embedding row into xa; under TP
    //    later layers finish the previous down's reduction: xa = xb + sum)
    GemvArgs a = gemv_args(w.qkv, H, nqkv, l == 0 ? nullptr : c->xa, c->qkv, c->err);
    a.gain = static_cast<const bf16*>(w.input_norm);
    a.eps = g.rms_eps;
    if (l == 0) {
      a.embed = c->embed;
      a.token = tok_in;
      a.vocab = c->cfg.vocab;
      a.x_copy = c->xa;
    } else if (tp && !p2p) {
      consume(a, c->xb, c->xa);
    }
    set_next_gemv(a, EPI_RESIDUAL, w.o, g.n_heads * D, H, o_sms);  // across the attention launch
    if (head) a.trace = next_trace(c, "qkv", l);
    if ((e = launch_gemv<EPI_STORE>(a, qkv_sms, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "qkv launch");
    // 2. attention with the norm/rope/append prologue
    if (head) at.trace = next_trace(c, "attn", l);
    if ((e = launch_attn(c->tmk[l], c->tmv[l], &c->dmk[l], &c->dmv[l], at, true, st)) != cudaSuccess)
      return cuda_fail(&c->msg, e, "attention launch");
    // 3. o-proj (+ residual): xb = xa + O . attn
    if (tp && !p2p) {
      a = gemv_args(w.o, g.n_heads * D, H, c->attn, nullptr, c->err);
      a.out32 = c->y32;
      set_next_gemv(a, EPI_SWIGLU, w.gate_up, H, 2 * g.ffn, c->sm_count);
      if (head) a.trace = next_trace(c, "o", l);
      if ((e = launch_gemv<EPI_PARTIAL>(a, o_sms, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "o launch");
      if ((nr = ncclAllReduce(c->y32, c->y32, H, ncclFloat32, ncclSum, c->comm, st)) != ncclSuccess)
        return set_err(&c->msg, QB_ERR_CUDA, std::string("ncclAllReduce: ") + ncclGetErrorString(nr));
    } else {
      a = gemv_args(w.o, g.n_heads * D, H, c->attn, c->xb, c->err);
      a.residual = c->xa;
      a.res_early = 1;  // xa: written by the previous down (or this layer's QKV gather), 2+ launches back
      if (p2p) peer_reduce(a, 2 * l, 0);
      set_next_gemv(a, EPI_SWIGLU, w.gate_up, H, 2 * g.ffn, c->sm_count);
      if (head) a.trace = next_trace(c, "o", l);
      if ((e = launch_gemv<EPI_RESIDUAL>(a, o_sms, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "o launch");
    }
    // 4. RMSNorm + gate/up + SwiGLU
    a = gemv_args(w.gate_up, H, 2 * g.ffn, c->xb, c->act, c->err);
    a.gain = static_cast<const bf16*>(w.post_norm);
    a.eps = g.rms_eps;
    if (tp && !p2p) consume(a, c->xa, c->xb);
    set_next_gemv(a, EPI_RESIDUAL, w.down, g.ffn, H, c->sm_count);
    if (head) a.trace = next_trace(c, "gateup", l);
    if ((e = launch_gemv<EPI_SWIGLU>(a, c->sm_count, st)) != cudaSuccess)
      return cuda_fail(&c->msg, e, "gate/up launch");
    // 5. down (+ residual): xa = xb + Down . act
    auto next_of_down = [&](GemvArgs& d) {
      if (l + 1 < g.n_layers) set_next_gemv(d, EPI_STORE, c->layers[l + 1].qkv, H, nqkv, qkv_sms);
      else if (head) set_next_gemv(d, EPI_ARGMAX, c->lm_head, H, g.vocab, c->sm_count);
    };
    if (tp && !p2p) {
      a = gemv_args(w.down, g.ffn, H, c->act, nullptr, c->err);
      a.out32 = c->y32;
      next_of_down(a);
      if (head) a.trace = next_trace(c, "down", l);
      if ((e = launch_gemv<EPI_PARTIAL>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "down launch");
      if ((nr = ncclAllReduce(c->y32, c->y32, H, ncclFloat32, ncclSum, c->comm, st)) != ncclSuccess)
        return set_err(&c->msg, QB_ERR_CUDA, std::string("ncclAllReduce: ") + ncclGetErrorString(nr));
    } else {
      a = gemv_args(w.down, g.ffn, H, c->act, c->xa, c->err);
      a.residual = c->xb;
      a.res_early = 1;  // xb: written by this layer's o-proj, two launches back
      if (p2p) peer_reduce(a, 2 * l + 1, 1);
      else if (!head && l == g.n_layers - 1) a.pos_inc = pos;
      next_of_down(a);
      if (head) a.trace = next_trace(c, "down", l);
      if ((e = launch_gemv<EPI_RESIDUAL>(a, c->sm_count, st)) != cudaSuccess)
        return cuda_fail(&c->msg, e, "down launch");
    }
  }
  if (tp) {
    if (head) {
      GemvArgs a = gemv_args(c->lm_head, H, g.vocab, c->xa, nullptr, c->err);
      if (!p2p) consume(a, c->xb, c->xa);
      a.gain = c->final_norm;
      a.eps = g.rms_eps;
      a.logits = static_cast<bf16*>(logits);
      a.part_val = c->head_val;
      a.part_idx = c->head_idx;
      a.counter = c->counters + 64;
      a.row_base = c->tp_rank * g.vocab;
      a.pair_out = c->pairs;
      a.trace = next_trace(c, "head", g.n_layers);
      if ((e = launch_gemv<EPI_ARGMAX>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "head launch");
      if ((nr = ncclAllGather(c->pairs, c->pairs + 2, 2, ncclFloat32, c->comm, st)) != ncclSuccess)
        return set_err(&c->msg, QB_ERR_CUDA, std::string("ncclAllGather: ") + ncclGetErrorString(nr));
      tp_pick_kernel<<<1, 32, 0, st>>>(c->pairs + 2, c->tp_size, tok_out, pos, p2p ? c->tp_epoch() : nullptr,
                                       nullptr, 0, 0, c->err);
    } else {
      // prefill row: advance the position (and the peer-reduction epoch)
      tp_pick_kernel<<<1, 32, 0, st>>>(nullptr, 0, nullptr, pos, p2p ? c->tp_epoch() : nullptr, nullptr, 0, 0,
                                       c->err);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(&c->msg, e, "pick launch");
    // The next step's layer 0 reads xa from the embedding; the final residual
    // is only needed by the head, which stored it.
    return QB_OK;
  }
  if (head) {
    GemvArgs a = gemv_args(c->lm_head, H, g.vocab, c->xa, nullptr, c->err);
    a.gain = c->final_norm;
    a.eps = g.rms_eps;
    a.logits = static_cast<bf16*>(logits);
    a.part_val = c->head_val;
    a.part_idx = c->head_idx;
    a.counter = c->counters + 64;
    a.token_out = tok_out;
    a.pos_inc = pos;
    a.trace = next_trace(c, "head", g.n_layers);
    if ((e = launch_gemv<EPI_ARGMAX>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "head launch");
  }
  return QB_OK;
}


template <int EPI>
cudaError_t launch_rows(const RowsArgs& a, int sm_count, cudaStream_t st) {
  bool& attr_done = dev_cache().rows_attr[EPI];
  const size_t smem = rows_smem_bytes();
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(gemv_rows_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  return launch_ex(gemv_rows_kernel<EPI>, dim3(sm_count), dim3(kRowsThreads), smem, st, a);
}

RowsArgs rows_args(const void* w, int K, int rows, int Q, const bf16* x, bf16* out, int* err) {
  RowsArgs a;
  std::memset(&a, 0, sizeof(a));
  a.w = static_cast<const bf16*>(w);
  a.K = K;
  a.rows = rows;
  a.Q = Q;
  a.x = x;
  a.out = out;
  a.err = err;
  return a;
}

// The verify pass (DecodeState.verify_step, dryft/engine/decode.py:168-179):
// rows ids[0..n) at positions *pos .. *pos+n-1 through every layer, their K/V
// appended, every row through the LM head; predictions[i] = greedy token after
// row i. The position itself is left to the caller (logical rollback).
// Tensor parallel: this rank's heads, FFN columns and vocabulary rows; the
// o-proj and down sums are exchanged as fp32 partial rows through peer memory
// inside the rows GEMV (NCCL all-reduce + tp_finish_rows_kernel without peer
// mappings) and rounded once with the residual added; the head's per-row
// (max, global index) pairs are all-gathered and picked per row.
int run_verify(qb_ctx* c, const int64_t* ids, int n, const int64_t* pos, int64_t* preds, void* logits,
               cudaStream_t st) {
  const qb_config& g = c->lc;
  const int H = g.hidden, D = g.head_dim;
  const int nqkv = (g.n_heads + 2 * g.n_kv_heads) * D;
  const bool tp = c->tp_size > 1;
  const bool p2p = tp && c->p2p;
  cudaError_t e;
  ncclResult_t nr;
  // NCCL fallback: fp32 partial rows -> all-reduce -> out = bf16(bf16(sum) + res)
  auto reduce_rows = [&](const bf16* res, bf16* out, const char* what) -> int {
    if ((nr = ncclAllReduce(c->r_y32, c->r_y32, (size_t)n * H, ncclFloat32, ncclSum, c->comm, st)) != ncclSuccess)
      return set_err(&c->msg, QB_ERR_CUDA, std::string("ncclAllReduce: ") + ncclGetErrorString(nr));
    const int threads = n * H / 8;
    if ((e = launch_ex(tp_finish_rows_kernel, dim3((threads + 255) / 256), dim3(256), 0, st, (const float*)c->r_y32,
                       res, out, n * H)) != cudaSuccess)
      return cuda_fail(&c->msg, e, what);
    return QB_OK;
  };
  int rc;
  for (int l = 0; l < g.n_layers; ++l) {
    const qb_layer_weights& w = c->layers[l];
    RowsArgs a = rows_args(w.qkv, H, nqkv, n, l == 0 ? nullptr : c->r_xa, c->r_qkv, c->err);
    a.gain = static_cast<const bf16*>(w.input_norm);
    a.eps = g.rms_eps;
    if (l == 0) {
      a.embed = c->embed;
      a.tokens = ids;
      a.vocab = c->cfg.vocab;
      a.x_copy = c->r_xa;
    }
    if ((e = launch_rows<EPI_STORE>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "verify qkv");
    RopeRowsArgs ra;
    std::memset(&ra, 0, sizeof(ra));
    ra.qkv = c->r_qkv;
    ra.q_norm = static_cast<const bf16*>(w.q_norm);
    ra.k_norm = static_cast<const bf16*>(w.k_norm);
    ra.cos = c->cos;
    ra.sin = c->sin;
    ra.eps = g.rms_eps;
    ra.pos = pos;
    ra.positions = c->r_pos;
    ra.q_out = c->r_q;
    const size_t layer_off = (size_t)l * g.n_kv_heads * c->cap * D;
    ra.k_cache = c->kc + layer_off;
    ra.v_cache = c->vc + layer_off;
    ra.err = c->err;
    ra.Q = n;
    ra.Hq = g.n_heads;
    ra.Hkv = g.n_kv_heads;
    ra.cap = c->cap;
    const int warps = n * (g.n_heads + 2 * g.n_kv_heads);
    if ((e = launch_ex(rope_rows_kernel, dim3((warps + 3) / 4), dim3(128), 0, st, ra)) != cudaSuccess)
      return cuda_fail(&c->msg, e, "verify rope");
    AttnArgs at;
    std::memset(&at, 0, sizeof(at));
    at.q = c->r_q;
    at.pos = c->r_pos;
    at.k_cache = ra.k_cache;
    at.v_cache = ra.v_cache;
    at.out = c->r_attn;
    at.part_o = c->part_o;
    at.part_lse = c->part_lse;
    at.counters = c->counters;
    at.err = c->err;
    at.Hq = g.n_heads;
    at.Hkv = g.n_kv_heads;
    at.Q = n;
    at.cap = c->cap;
    at.splits = c->splits;
    const int vcs = (g.n_heads / g.n_kv_heads) * n <= kVaMaxRows ? rows_cluster_size(g.n_kv_heads) : 0;
    if (vcs > 0) {
      at.part_splits = c->splits;
      at.tickets = c->counters + 512;
      rows_attn_shape(at, vcs);
    }
    e = vcs > 0 ? launch_attn_rows(c->dmk[l], c->dmv[l], at, vcs, st)
                : launch_attn(c->tmk[l], c->tmv[l], nullptr, nullptr, at, false, st);
    if (e != cudaSuccess) return cuda_fail(&c->msg, e, "verify attention");
    a = rows_args(w.o, g.n_heads * D, H, n, c->r_attn, c->r_xb, c->err);
    if (p2p) {
      a.residual = c->r_xa;
      a.tp = c->peers;
      a.tp_sub = 2 * l;
      a.tp_parity = 0;
      a.hidden = H;
      if ((e = launch_rows<EPI_RESIDUAL>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "verify o");
    } else if (tp) {
      a.out = nullptr;
      a.out32 = c->r_y32;
      if ((e = launch_rows<EPI_PARTIAL>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "verify o");
      if ((rc = reduce_rows(c->r_xa, c->r_xb, "verify o finish")) != QB_OK) return rc;
    } else {
      a.residual = c->r_xa;
      if ((e = launch_rows<EPI_RESIDUAL>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "verify o");
    }
    a = rows_args(w.gate_up, H, 2 * g.ffn, n, c->r_xb, c->r_act, c->err);
    a.gain = static_cast<const bf16*>(w.post_norm);
    a.eps = g.rms_eps;
    if ((e = launch_rows<EPI_SWIGLU>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "verify gu");
    a = rows_args(w.down, g.ffn, H, n, c->r_act, c->r_xa, c->err);
    if (p2p) {
      a.residual = c->r_xb;
      a.tp = c->peers;
      a.tp_sub = 2 * l + 1;
      a.tp_parity = 1;
      a.hidden = H;
      if ((e = launch_rows<EPI_RESIDUAL>(a, c->sm_count, st)) != cudaSuccess)
        return cuda_fail(&c->msg, e, "verify down");
    } else if (tp) {
      a.out = nullptr;
      a.out32 = c->r_y32;
      if ((e = launch_rows<EPI_PARTIAL>(a, c->sm_count, st)) != cudaSuccess)
        return cuda_fail(&c->msg, e, "verify down");
      if ((rc = reduce_rows(c->r_xb, c->r_xa, "verify down finish")) != QB_OK) return rc;
    } else {
      a.residual = c->r_xb;
      if ((e = launch_rows<EPI_RESIDUAL>(a, c->sm_count, st)) != cudaSuccess)
        return cuda_fail(&c->msg, e, "verify down");
    }
  }
  RowsArgs a = rows_args(c->lm_head, H, g.vocab, n, c->r_xa, nullptr, c->err);
  a.gain = c->final_norm;
  a.eps = g.rms_eps;
  a.logits = static_cast<bf16*>(logits);
  a.part_val = c->r_val;
  a.part_idx = c->r_idx;
  a.counter = c->counters + 66;
  a.tokens_out = preds;
  if (tp) {
    a.tokens_out = nullptr;
    a.pair_out = c->r_pairs;
    a.row_base = c->tp_rank * g.vocab;
  }
  if ((e = launch_rows<EPI_ARGMAX>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "verify head");
  if (tp) {
    if ((nr = ncclAllGather(c->r_pairs, c->r_pairs + 2 * n, 2 * n, ncclFloat32, c->comm, st)) != ncclSuccess)
      return set_err(&c->msg, QB_ERR_CUDA, std::string("ncclAllGather: ") + ncclGetErrorString(nr));
    if ((e = launch_ex(tp_pick_rows_kernel, dim3(1), dim3(32), 0, st, (const float*)(c->r_pairs + 2 * n),
                       c->tp_size, n, preds, p2p ? c->tp_epoch() : nullptr)) != cudaSuccess)
      return cuda_fail(&c->msg, e, "verify pick");
  }
  return QB_OK;
}

// Batched decode (the B = c->batch sequences of a batched context, one row
// each; dryft's DecodeState at B > 1, dryft/engine/decode.py:102-138):
// ids[b] at position pos[b] (device), sequence b's K/V in slice b of every
// layer's [B][Hkv][cap][D]. The rows kernels stream every weight once for the
// B rows; the rows attention runs B * Hkv KV heads, each reading its
// sequence's position. head: the greedy next token of each sequence to
// tok_out[b] (logits [B][V] optional); pos[b] += 1 either way.
int run_batch_pass(qb_ctx* c, const int64_t* ids, int64_t* pos, int64_t* tok_out, void* logits, bool head,
                   cudaStream_t st) {
  const qb_config& g = c->lc;
  const int B = c->batch, H = g.hidden, D = g.head_dim;
  const int nqkv = (g.n_heads + 2 * g.n_kv_heads) * D;
  const int vheads = B * g.n_kv_heads;
  const int acs = batch_attn_cluster(vheads, c->sm_count);
  if (acs <= 0) return set_err(&c->msg, QB_ERR_UNSUPPORTED, "rows attention kernel unavailable");
  cudaError_t e;
  for (int l = 0; l < g.n_layers; ++l) {
    const qb_layer_weights& w = c->layers[l];
    RowsArgs a = rows_args(w.qkv, H, nqkv, B, l == 0 ? nullptr : c->r_xa, c->r_qkv, c->err);
    a.gain = static_cast<const bf16*>(w.input_norm);
    a.eps = g.rms_eps;
    if (l == 0) {
      a.embed = c->embed;
      a.tokens = ids;
      a.vocab = c->cfg.vocab;
      a.x_copy = c->r_xa;
    }
    if ((e = launch_rows<EPI_STORE>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "batch qkv");
    const size_t layer_off = (size_t)l * vheads * c->cap * D;
    RopeRowsArgs ra;
    std::memset(&ra, 0, sizeof(ra));
    ra.qkv = c->r_qkv;
    ra.q_norm = static_cast<const bf16*>(w.q_norm);
    ra.k_norm = static_cast<const bf16*>(w.k_norm);
    ra.cos = c->cos;
    ra.sin = c->sin;
    ra.eps = g.rms_eps;
    ra.pos = pos;
    ra.q_out = c->r_q;
    ra.k_cache = c->kc + layer_off;
    ra.v_cache = c->vc + layer_off;
    ra.err = c->err;
    ra.Q = B;
    ra.Hq = g.n_heads;
    ra.Hkv = g.n_kv_heads;
    ra.cap = c->cap;
    ra.batched = 1;
    const int warps = B * (g.n_heads + 2 * g.n_kv_heads);
    if ((e = launch_ex(rope_rows_kernel, dim3((warps + 3) / 4), dim3(128), 0, st, ra)) != cudaSuccess)
      return cuda_fail(&c->msg, e, "batch rope");
    AttnArgs at;
    std::memset(&at, 0, sizeof(at));
    at.q = c->r_q;
    at.pos = pos;
    at.k_cache = ra.k_cache;
    at.v_cache = ra.v_cache;
    at.out = c->r_attn;
    at.counters = c->counters;
    at.err = c->err;
    at.Hq = B * g.n_heads;
    at.Hkv = vheads;
    at.Q = 1;
    at.cap = c->cap;
    at.batch_hkv = g.n_kv_heads;
    if ((e = launch_attn_rows(c->dmk[l], c->dmv[l], at, acs, st)) != cudaSuccess)
      return cuda_fail(&c->msg, e, "batch attention");
    a = rows_args(w.o, g.n_heads * D, H, B, c->r_attn, c->r_xb, c->err);
    a.residual = c->r_xa;
    if ((e = launch_rows<EPI_RESIDUAL>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "batch o");
    a = rows_args(w.gate_up, H, 2 * g.ffn, B, c->r_xb, c->r_act, c->err);
    a.gain = static_cast<const bf16*>(w.post_norm);
    a.eps = g.rms_eps;
    if ((e = launch_rows<EPI_SWIGLU>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "batch gu");
    a = rows_args(w.down, g.ffn, H, B, c->r_act, c->r_xa, c->err);
    a.residual = c->r_xb;
    if ((e = launch_rows<EPI_RESIDUAL>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "batch down");
  }
  if (head) {
    RowsArgs a = rows_args(c->lm_head, H, g.vocab, B, c->r_xa, nullptr, c->err);
    a.gain = c->final_norm;
    a.eps = g.rms_eps;
    a.logits = static_cast<bf16*>(logits);
    a.part_val = c->r_val;
    a.part_idx = c->r_idx;
    a.counter = c->counters + 66;
    a.tokens_out = tok_out;
    if ((e = launch_rows<EPI_ARGMAX>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "batch head");
  }
  if ((e = launch_ex(add_rows_i64_kernel, dim3(1), dim3(32), 0, st, pos, B, 1ll)) != cudaSuccess)
    return cuda_fail(&c->msg, e, "batch positions");
  return QB_OK;
}

// Batched prefill scratch: per prompt row xa, xb, xn [H]; qkv; q, attn [Hq*D];
// act [F] (bf16).
struct PrefillLayout {
  // tensor parallel only: gath (all-gather results, rank-major), full (rows
  // made whole), outl (this rank's [T][H/n] output columns)
  size_t xa, xb, xn, q, attn, act, gath, full, outl, total;
};
PrefillLayout prefill_layout(const qb_ctx* c, int n) {
  const qb_config& g = c->lc;
  const size_t T = (size_t)n;
  PrefillLayout L;
  size_t o = 0;
  L.xa = o; o = align_up(o + T * g.hidden * 2, 256);
  L.xb = o; o = align_up(o + T * g.hidden * 2, 256);
  L.xn = o; o = align_up(o + T * g.hidden * 2, 256);
  L.q = o; o = align_up(o + T * g.n_heads * g.head_dim * 2, 256);
  L.attn = o; o = align_up(o + T * g.n_heads * g.head_dim * 2, 256);
  L.act = o; o = align_up(o + T * g.ffn * 2, 256);
  const bool tp = c->tp_size > 1;
  const size_t wide = std::max<size_t>((size_t)c->cfg.n_heads * g.head_dim, std::max<size_t>(c->cfg.ffn, g.hidden));
  L.gath = o; o = align_up(o + (tp ? T * wide * 2 : 0), 256);
  L.full = o; o = align_up(o + (tp ? T * wide * 2 : 0), 256);
  L.outl = o; o = align_up(o + (tp ? T * (g.hidden / c->tp_size) * 2 : 0), 256);
  L.total = o;
  return L;
}

// Prompt rows ids[0..n) at positions 0..n-1 through every layer as dense
// blocks (tcgen05 GEMMs, causal flash attention), K/V appended; the last row
// through the LM head; *position = n (DecodeState.prefill,
// dryft/engine/decode.py:157-166, dryft/engine/prefill.py:6-26).
// Tensor parallel: each rank runs its heads and FFN slice (QKV + RoPE, flash
// attention, gate/up + SwiGLU); the o-proj and down projections run
// column-parallel: the attention output and the SwiGLU activations of every
// rank are all-gathered (NCCL) into whole rows, each rank computes output
// columns [r*H/n, (r+1)*H/n) over the whole input with the same GEMM and
// residual epilogue, and those blocks are all-gathered into the next
// residual. Every value is then computed as on one GPU, so the K/V rows and
// the first token equal the single-GPU prefill's; the last row's head is the
// vocabulary-sharded argmax of the decode step.
int run_prefill_batched(qb_ctx* c, const int64_t* ids, int n, uint8_t* scratch, int64_t* tok_out, int64_t* pos,
                        void* logits, cudaStream_t st) {
  const qb_config& g = c->lc;
  const int H = g.hidden, D = g.head_dim;
  const int nqkv = (g.n_heads + 2 * g.n_kv_heads) * D;
  const int tp = c->tp_size;
  const int Hr = H / tp;  // output columns of this rank under tensor parallelism
  const PrefillLayout P = prefill_layout(c, n);
  bf16* xa = reinterpret_cast<bf16*>(scratch + P.xa);
  bf16* xb = reinterpret_cast<bf16*>(scratch + P.xb);
  bf16* xn = reinterpret_cast<bf16*>(scratch + P.xn);
  bf16* q = reinterpret_cast<bf16*>(scratch + P.q);
  bf16* attn = reinterpret_cast<bf16*>(scratch + P.attn);
  bf16* act = reinterpret_cast<bf16*>(scratch + P.act);
  bf16* gath = reinterpret_cast<bf16*>(scratch + P.gath);
  bf16* full = reinterpret_cast<bf16*>(scratch + P.full);
  bf16* outl = reinterpret_cast<bf16*>(scratch + P.outl);
  cudaError_t e;
  ncclResult_t nr;
  // every rank's column block src [n][C] -> dst [n][tp * C]
  auto gather_cols = [&](const bf16* src, int C, bf16* dst, const char* what) -> int {
    if ((nr = ncclAllGather(src, gath, (size_t)n * C, ncclBfloat16, c->comm, st)) != ncclSuccess)
      return set_err(&c->msg, QB_ERR_CUDA, std::string("ncclAllGather: ") + ncclGetErrorString(nr));
    const long long vecs = (long long)n * C * tp / 8;
    if ((e = launch_ex(unshard_cols_kernel, dim3((unsigned)((vecs + 255) / 256)), dim3(256), 0, st,
                       (const bf16*)gath, dst, n, C, tp)) != cudaSuccess)
      return cuda_fail(&c->msg, e, what);
    return QB_OK;
  };
  // out[n][H] = x . W^T + res: on one GPU x [n][K] and W whole; tensor
  // parallel x is this rank's [n][K/tp] slice, w_rows this rank's output rows
  auto project_residual = [&](const bf16* x, const void* w, const bf16* w_rows, int K, const bf16* res, bf16* out,
                              const char* what) -> int {
    if (tp == 1) {
      if ((e = launch_prefill_gemm(PG_RESIDUAL, x, static_cast<const bf16*>(w), out, res, n, H, K, c->err, st)) !=
          cudaSuccess)
        return cuda_fail(&c->msg, e, what);
      return QB_OK;
    }
    int rc2;
    if ((rc2 = gather_cols(x, K / tp, full, what)) != QB_OK) return rc2;
    PgArgs ra;
    std::memset(&ra, 0, sizeof(ra));
    ra.res_stride = H;
    if ((e = launch_prefill_gemm(PG_RESIDUAL, full, w_rows, outl, res + (size_t)c->tp_rank * Hr, n, Hr, K, c->err,
                                 st, &ra)) != cudaSuccess)
      return cuda_fail(&c->msg, e, what);
    return gather_cols(outl, Hr, out, what);
  };
  int rc;
  auto norm = [&](const bf16* x, const bf16* gain, bool gather) {
    NormRowsArgs na;
    std::memset(&na, 0, sizeof(na));
    na.x = gather ? nullptr : x;
    na.embed = c->embed;
    na.ids = ids;
    na.vocab = c->cfg.vocab;
    na.x_out = xa;
    na.gain = gain;
    na.xn = xn;
    na.K = H;
    na.eps = g.rms_eps;
    na.err = c->err;
    return launch_ex(norm_rows_kernel, dim3(n), dim3(128), 0, st, na);
  };
  for (int l = 0; l < g.n_layers; ++l) {
    const qb_layer_weights& w = c->layers[l];
    if ((e = norm(xa, static_cast<const bf16*>(w.input_norm), l == 0)) != cudaSuccess)
      return cuda_fail(&c->msg, e, "prefill norm");
    // QKV GEMM with the q/k norm + RoPE + K/V append in its epilogue
    PgArgs qr;
    std::memset(&qr, 0, sizeof(qr));
    qr.q_norm = static_cast<const bf16*>(w.q_norm);
    qr.k_norm = static_cast<const bf16*>(w.k_norm);
    qr.cos = c->cos;
    qr.sin = c->sin;
    qr.eps = g.rms_eps;
    qr.q_out = q;
    const size_t layer_off = (size_t)l * g.n_kv_heads * c->cap * D;
    qr.k_cache = c->kc + layer_off;
    qr.v_cache = c->vc + layer_off;
    qr.Hq = g.n_heads;
    qr.Hkv = g.n_kv_heads;
    qr.cap = c->cap;
    qr.p0 = 0;
    if ((e = launch_prefill_gemm(PG_QKV_ROPE, xn, static_cast<const bf16*>(w.qkv), nullptr, nullptr, n, nqkv, H,
                                 c->err, st, &qr)) != cudaSuccess)
      return cuda_fail(&c->msg, e, "prefill qkv");
    const int G = g.n_heads / g.n_kv_heads;
    CUtensorMap tq;
    if (kFtRowsQ % (2 * G) != 0 || !make_q3_map(&tq, q, n, g.n_heads, G, kFtRowsQ / G / 2))
      return set_err(&c->msg, QB_ERR_UNSUPPORTED, "prefill attention: query map");
    {
      // 256 query rows (256 / G prompt rows x G heads) per CTA on tcgen05
      bool& ft_attr = dev_cache().ft_attr;
      if (!ft_attr) {
        if ((e = cudaFuncSetAttribute(flash_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)ft_smem_bytes())) != cudaSuccess)
          return cuda_fail(&c->msg, e, "prefill attention attribute");
        ft_attr = true;
      }
      FtArgs ft;
      ft.out = attn;
      ft.T = n;
      ft.p0 = 0;
      ft.Hq = g.n_heads;
      ft.Hkv = g.n_kv_heads;
      ft.cap = c->cap;
      ft.err = c->err;
      const int rows = kFtRowsQ / G;
      if ((e = launch_ex(flash_prefill_tc_kernel, dim3(((n + rows - 1) / rows) * g.n_kv_heads), dim3(kFtThreads),
                         ft_smem_bytes(), st, tq, c->tmk[l], c->tmv[l], ft)) != cudaSuccess)
        return cuda_fail(&c->msg, e, "prefill attention");
    }
    if ((rc = project_residual(attn, w.o, tp > 1 ? c->o_rows[l] : nullptr, c->cfg.n_heads * D, xa, xb,
                               "prefill o")) != QB_OK)
      return rc;
    if ((e = norm(xb, static_cast<const bf16*>(w.post_norm), false)) != cudaSuccess)
      return cuda_fail(&c->msg, e, "prefill norm");
    if ((e = launch_prefill_gemm(PG_SWIGLU, xn, static_cast<const bf16*>(w.gate_up), act, nullptr, n, 2 * g.ffn, H,
                                 c->err, st)) != cudaSuccess)
      return cuda_fail(&c->msg, e, "prefill gate/up");
    if ((rc = project_residual(act, w.down, tp > 1 ? c->down_rows[l] : nullptr, c->cfg.ffn, xb, xa,
                               "prefill down")) != QB_OK)
      return rc;
  }
  // The last row through the final norm, the LM head and the argmax (under
  // tensor parallelism: this rank's vocabulary rows, then the (max, index)
  // pairs of every rank and the lowest index among the largest values).
  GemvArgs a = gemv_args(c->lm_head, H, g.vocab, xa + (size_t)(n - 1) * H, nullptr, c->err);
  a.gain = c->final_norm;
  a.eps = g.rms_eps;
  a.logits = static_cast<bf16*>(logits);
  a.part_val = c->head_val;
  a.part_idx = c->head_idx;
  a.counter = c->counters + 64;
  a.token_out = tok_out;
  if (tp > 1) {
    a.token_out = nullptr;
    a.row_base = c->tp_rank * g.vocab;
    a.pair_out = c->pairs;
  }
  if ((e = launch_gemv<EPI_ARGMAX>(a, c->sm_count, st)) != cudaSuccess) return cuda_fail(&c->msg, e, "prefill head");
  if (tp > 1) {
    if ((nr = ncclAllGather(c->pairs, c->pairs + 2, 2, ncclFloat32, c->comm, st)) != ncclSuccess)
      return set_err(&c->msg, QB_ERR_CUDA, std::string("ncclAllGather: ") + ncclGetErrorString(nr));
    // no peer-reduction words were written, so the epoch stays as it is
    tp_pick_kernel<<<1, 32, 0, st>>>(c->pairs + 2, c->tp_size, tok_out, nullptr, nullptr, nullptr, 0, 0, c->err);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(&c->msg, e, "prefill pick");
  }
  if ((e = launch_ex(set_i64_kernel, dim3(1), dim3(1), 0, st, pos, (long long)n)) != cudaSuccess)
    return cuda_fail(&c->msg, e, "prefill position");
  return QB_OK;
}

int check_verify_args(qb_ctx* c, const int64_t* ids, int n, const int64_t* pos, const int64_t* preds) {
  if (!ids || !pos || !preds) return set_err(&c->msg, QB_ERR_ARG, "ids/position/predictions are NULL");
  if (n < 1 || n > kRowsMaxQ) return set_err(&c->msg, QB_ERR_UNSUPPORTED, "verify takes 1..8 rows");
  if ((c->lc.n_heads / c->lc.n_kv_heads) * n > 32)
    return set_err(&c->msg, QB_ERR_UNSUPPORTED, "GQA group x verify rows above 32");
  if (c->tp_size != 1 && c->comm == nullptr) return set_err(&c->msg, QB_ERR_STATE, "tensor parallel communicator not initialised");
  if (c->batch != 1) return set_err(&c->msg, QB_ERR_UNSUPPORTED, "verify takes one sequence");
  if (c->sm_count > 1024) return set_err(&c->msg, QB_ERR_UNSUPPORTED, "more than 1024 SMs");
  return QB_OK;
}

// Captured graphs hold the bound state's pointers: drop them whenever the
// state (or its layout) changes.
void drop_graphs(qb_ctx* c) {
  if (c->exec) {
    cudaGraphExecDestroy(c->exec);
    c->exec = nullptr;
  }
  if (c->graph) {
    cudaGraphDestroy(c->graph);
    c->graph = nullptr;
  }
  if (c->vexec) {
    cudaGraphExecDestroy(c->vexec);
    c->vexec = nullptr;
  }
  if (c->vgraph) {
    cudaGraphDestroy(c->vgraph);
    c->vgraph = nullptr;
  }
}

int require_ready(qb_ctx* c) {
  if (!c) return set_err(nullptr, QB_ERR_ARG, "ctx is NULL");
  if (!c->weights_bound) return set_err(&c->msg, QB_ERR_STATE, "weights not bound");
  if (!c->state_bound) return set_err(&c->msg, QB_ERR_STATE, "state not bound");
  if (c->tp_size > 1 && !c->comm) return set_err(&c->msg, QB_ERR_STATE, "tensor-parallel context without qb_tp_init");
  return QB_OK;
}

}  // namespace

// ====================================================================== C ABI
extern "C" {

const char* qb_version(void) { return "qb 0.1 sm_100a"; }

const char* qb_last_error(const qb_ctx* ctx) {
  if (ctx) return ctx->msg.c_str();
  return g_last_error.c_str();
}

int qb_create(const qb_config* cfg, int device, int tp_rank, int tp_size, qb_ctx** out) {
  if (!out) return set_err(nullptr, QB_ERR_ARG, "out is NULL");
  *out = nullptr;
  std::string msg;
  int rc = validate_config(cfg, &msg);
  if (rc) return rc;
  if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size)
    return set_err(nullptr, QB_ERR_ARG, "tp_rank must lie in [0, tp_size)");
  // Shard: KV heads (with their query heads), FFN columns and vocabulary rows.
  qb_config lc = *cfg;
  if (cfg->n_kv_heads % tp_size || cfg->ffn % tp_size || cfg->vocab % tp_size)
    return set_err(nullptr, QB_ERR_UNSUPPORTED, "n_kv_heads, ffn and vocab must divide by tp_size");
  lc.n_heads = cfg->n_heads / tp_size;
  lc.n_kv_heads = cfg->n_kv_heads / tp_size;
  lc.ffn = cfg->ffn / tp_size;
  lc.vocab = cfg->vocab / tp_size;
  if ((lc.n_heads * lc.head_dim) % 128 || lc.ffn % 128)
    return set_err(nullptr, QB_ERR_UNSUPPORTED, "per-rank Hq*D and ffn must be multiples of 128");
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaSetDevice");
  qb_ctx* c = new qb_ctx();
  c->cfg = *cfg;
  c->lc = lc;
  c->device = device;
  c->tp_rank = tp_rank;
  c->tp_size = tp_size;
  c->sm_count = sm_count_of(device);
  c->splits = attn_splits_for(lc.n_kv_heads, c->sm_count);
  *out = c;
  return QB_OK;
}

int qb_destroy(qb_ctx* c) {
  if (!c) return QB_OK;
  if (c->exec) cudaGraphExecDestroy(c->exec);
  if (c->graph) cudaGraphDestroy(c->graph);
  if (c->vexec) cudaGraphExecDestroy(c->vexec);
  if (c->vgraph) cudaGraphDestroy(c->vgraph);
  if (c->p2p) {
    cudaSetDevice(c->device);
    for (int r = 0; r < c->tp_size; ++r)
      if (r != c->tp_rank && c->peers.recv[r]) cudaIpcCloseMemHandle(c->peers.recv[r]);
  }
  if (c->tp_base) cudaFree(c->tp_base);
  if (c->comm) ncclCommDestroy(c->comm);
  delete c;
  return QB_OK;
}

int qb_bind_weights(qb_ctx* c, const qb_layer_weights* layers, int n_layers, const void* embed,
                    const void* final_norm, const void* lm_head) {
  if (!c) return set_err(nullptr, QB_ERR_ARG, "ctx is NULL");
  if (!layers || n_layers != c->cfg.n_layers) return set_err(&c->msg, QB_ERR_ARG, "layer table does not match n_layers");
  if (!ptr_ok(embed) || !ptr_ok(final_norm) || !ptr_ok(lm_head))
    return set_err(&c->msg, QB_ERR_ARG, "embed/final_norm/lm_head must be 16-byte aligned device pointers");
  for (int l = 0; l < n_layers; ++l) {
    const qb_layer_weights& w = layers[l];
    const void* ps[8] = {w.input_norm, w.qkv, w.q_norm, w.k_norm, w.o, w.post_norm, w.gate_up, w.down};
    for (const void* p : ps)
      if (!ptr_ok(p)) return set_err(&c->msg, QB_ERR_ARG, "layer weight pointers must be 16-byte aligned and non-NULL");
  }
  c->layers.assign(layers, layers + n_layers);
  c->embed = static_cast<const bf16*>(embed);
  c->final_norm = static_cast<const bf16*>(final_norm);
  c->lm_head = static_cast<const bf16*>(lm_head);
  c->weights_bound = true;
  return QB_OK;
}

int qb_bind_prefill_weights(qb_ctx* c, const void* const* o_rows, const void* const* down_rows, int n_layers) {
  if (!c) return set_err(nullptr, QB_ERR_ARG, "ctx is NULL");
  if (!o_rows || !down_rows || n_layers != c->cfg.n_layers)
    return set_err(&c->msg, QB_ERR_ARG, "o_rows/down_rows tables do not match n_layers");
  for (int l = 0; l < n_layers; ++l)
    if (!ptr_ok(o_rows[l]) || !ptr_ok(down_rows[l]))
      return set_err(&c->msg, QB_ERR_ARG, "prefill weight pointers must be 16-byte aligned and non-NULL");
  c->o_rows.resize(n_layers);
  c->down_rows.resize(n_layers);
  for (int l = 0; l < n_layers; ++l) {
    c->o_rows[l] = static_cast<const bf16*>(o_rows[l]);
    c->down_rows[l] = static_cast<const bf16*>(down_rows[l]);
  }
  return QB_OK;
}

int qb_workspace_bytes(const qb_ctx* c, size_t* bytes) {
  if (!c || !bytes) return set_err(nullptr, QB_ERR_ARG, "NULL argument");
  *bytes = ws_layout(c).total;
  return QB_OK;
}

int qb_bind_state(qb_ctx* c, void* k_cache, void* v_cache, int capacity, const void* rope_cos,
                  const void* rope_sin, void* workspace, size_t workspace_bytes) {
  if (!c) return set_err(nullptr, QB_ERR_ARG, "ctx is NULL");
  if (capacity <= 0) return set_err(&c->msg, QB_ERR_ARG, "capacity must be positive");
  if (!ptr_ok(k_cache) || !ptr_ok(v_cache) || !ptr_ok(rope_cos) || !ptr_ok(rope_sin) || !ptr_ok(workspace))
    return set_err(&c->msg, QB_ERR_ARG, "state pointers must be 16-byte aligned and non-NULL");
  const WsLayout L = ws_layout(c);
  if (workspace_bytes < L.total) return set_err(&c->msg, QB_ERR_ARG, "workspace smaller than qb_workspace_bytes()");
  cudaError_t e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return cuda_fail(&c->msg, e, "cudaSetDevice");
  c->kc = static_cast<bf16*>(k_cache);
  c->vc = static_cast<bf16*>(v_cache);
  c->cap = capacity;
  c->cos = static_cast<const bf16*>(rope_cos);
  c->sin = static_cast<const bf16*>(rope_sin);
  c->ws = static_cast<uint8_t*>(workspace);
  c->ws_bytes = workspace_bytes;
  c->err = reinterpret_cast<int*>(c->ws + L.err);
  c->counters = reinterpret_cast<unsigned*>(c->ws + L.counters);
  c->head_val = reinterpret_cast<float*>(c->ws + L.head_val);
  c->head_idx = reinterpret_cast<int*>(c->ws + L.head_idx);
  c->xa = reinterpret_cast<bf16*>(c->ws + L.xa);
  c->xb = reinterpret_cast<bf16*>(c->ws + L.xb);
  c->qkv = reinterpret_cast<bf16*>(c->ws + L.qkv);
  c->attn = reinterpret_cast<bf16*>(c->ws + L.attn);
  c->act = reinterpret_cast<bf16*>(c->ws + L.act);
  c->part_lse = reinterpret_cast<float*>(c->ws + L.part_lse);
  c->part_o = reinterpret_cast<float*>(c->ws + L.part_o);
  c->y32 = reinterpret_cast<float*>(c->ws + L.y32);
  c->pairs = reinterpret_cast<float*>(c->ws + L.pairs);
  c->r_xa = reinterpret_cast<bf16*>(c->ws + L.r_xa);
  c->r_xb = reinterpret_cast<bf16*>(c->ws + L.r_xb);
  c->r_qkv = reinterpret_cast<bf16*>(c->ws + L.r_qkv);
  c->r_q = reinterpret_cast<bf16*>(c->ws + L.r_q);
  c->r_attn = reinterpret_cast<bf16*>(c->ws + L.r_attn);
  c->r_act = reinterpret_cast<bf16*>(c->ws + L.r_act);
  c->r_pos = reinterpret_cast<int64_t*>(c->ws + L.r_pos);
  c->r_val = reinterpret_cast<float*>(c->ws + L.r_val);
  c->r_idx = reinterpret_cast<int*>(c->ws + L.r_idx);
  c->r_y32 = reinterpret_cast<float*>(c->ws + L.r_y32);
  c->r_pairs = reinterpret_cast<float*>(c->ws + L.r_pairs);
  if ((e = cudaMemset(workspace, 0, L.total)) != cudaSuccess) return cuda_fail(&c->msg, e, "workspace memset");
  const qb_config& g = c->lc;
  c->tmk.assign(g.n_layers, CUtensorMap());
  c->tmv.assign(g.n_layers, CUtensorMap());
  c->dmk.assign(g.n_layers, CUtensorMap());
  c->dmv.assign(g.n_layers, CUtensorMap());
  // batched: layer l holds the B sequences' [Hkv][cap][D] slices one after
  // another, so one map per layer covers B * Hkv heads
  const int mh = g.n_kv_heads * c->batch;
  for (int l = 0; l < g.n_layers; ++l) {
    const size_t off = (size_t)l * mh * capacity * g.head_dim;
    if (!make_kv_map(&c->tmk[l], c->kc + off, mh, capacity) ||
        !make_kv_map(&c->tmv[l], c->vc + off, mh, capacity) ||
        !make_kv_map(&c->dmk[l], c->kc + off, mh, capacity, kDecKeys) ||
        !make_kv_map(&c->dmv[l], c->vc + off, mh, capacity, kDecKeys))
      return set_err(&c->msg, QB_ERR_CUDA, "cuTensorMapEncodeTiled failed for the KV cache");
  }
  drop_graphs(c);
  c->state_bound = true;
  return QB_OK;
}

int qb_nccl_unique_id(void* out, size_t bytes) {
  if (!out || bytes < sizeof(ncclUniqueId)) return set_err(nullptr, QB_ERR_ARG, "unique id buffer smaller than 128 bytes");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return set_err(nullptr, QB_ERR_CUDA, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
  std::memcpy(out, &id, sizeof(id));
  return QB_OK;
}

int qb_tp_init(qb_ctx* c, const void* unique_id) {
  if (!c || !unique_id) return set_err(nullptr, QB_ERR_ARG, "NULL argument");
  if (c->tp_size == 1) return QB_OK;
  if (c->comm) return set_err(&c->msg, QB_ERR_STATE, "communicator already initialised");
  cudaError_t e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return cuda_fail(&c->msg, e, "cudaSetDevice");
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  ncclResult_t r = ncclCommInitRank(&c->comm, c->tp_size, id, c->tp_rank);
  if (r != ncclSuccess) {
    c->comm = nullptr;
    return set_err(&c->msg, QB_ERR_CUDA, std::string("ncclCommInitRank: ") + ncclGetErrorString(r));
  }
  if (c->tp_size > kMaxTp) return QB_OK;  // NCCL path only
  const char* env = std::getenv("QB_TP_NCCL");
  if (env && env[0] == '1') return QB_OK;
  // Peer-memory reduction buffers: tagged words [2][n][H] (decode rows) and
  // [2][n][kRowsMaxQ][H] (verify rows) u64 | epoch.
  const size_t recv_bytes = align_up(rows_tp_words(c->tp_size, c->cfg.hidden) * 8, 256);
  const size_t flag_bytes = 0;
  const size_t total = recv_bytes + flag_bytes + 256;
  if ((e = cudaMalloc(&c->tp_base, total)) != cudaSuccess) return cuda_fail(&c->msg, e, "peer buffer cudaMalloc");
  if ((e = cudaMemset(c->tp_base, 0, total)) != cudaSuccess) return cuda_fail(&c->msg, e, "peer buffer memset");
  cudaIpcMemHandle_t mine;
  if ((e = cudaIpcGetMemHandle(&mine, c->tp_base)) != cudaSuccess) return cuda_fail(&c->msg, e, "cudaIpcGetMemHandle");
  void* dev_handles = nullptr;
  if ((e = cudaMalloc(&dev_handles, sizeof(mine) * (c->tp_size + 1))) != cudaSuccess)
    return cuda_fail(&c->msg, e, "handle buffer");
  cudaMemcpy(dev_handles, &mine, sizeof(mine), cudaMemcpyHostToDevice);
  r = ncclAllGather(dev_handles, static_cast<char*>(dev_handles) + sizeof(mine), sizeof(mine), ncclChar, c->comm,
                    nullptr);
  std::vector<cudaIpcMemHandle_t> all(c->tp_size);
  cudaStreamSynchronize(nullptr);
  cudaMemcpy(all.data(), static_cast<char*>(dev_handles) + sizeof(mine), sizeof(mine) * c->tp_size,
             cudaMemcpyDeviceToHost);
  cudaFree(dev_handles);
  if (r != ncclSuccess) return set_err(&c->msg, QB_ERR_CUDA, std::string("ncclAllGather: ") + ncclGetErrorString(r));
  for (int k = 0; k < c->tp_size; ++k) {
    void* base = c->tp_base;
    if (k != c->tp_rank) {
      if ((e = cudaIpcOpenMemHandle(&base, all[k], cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess) {
        cudaGetLastError();
        for (int j = 0; j < k; ++j)
          if (j != c->tp_rank && c->peers.recv[j]) cudaIpcCloseMemHandle(c->peers.recv[j]);
        std::memset(&c->peers, 0, sizeof(c->peers));
        return QB_OK;  // no peer mapping: stay on the NCCL all-reduce path
      }
    }
    c->peers.recv[k] = static_cast<unsigned long long*>(base);
  }
  c->peers.epoch = reinterpret_cast<unsigned long long*>(static_cast<char*>(c->tp_base) + recv_bytes + flag_bytes);
  c->peers.rank = c->tp_rank;
  c->peers.size = c->tp_size;
  c->p2p = true;
  return QB_OK;
}

int qb_decode_step(qb_ctx* c, int64_t* token, int64_t* position, void* logits_out, void* stream) {
  int rc = require_ready(c);
  if (rc) return rc;
  if (!token || !position) return set_err(&c->msg, QB_ERR_ARG, "token/position are NULL");
  if (c->batch > 1)
    return run_batch_pass(c, token, position, token, logits_out, true, static_cast<cudaStream_t>(stream));
  return run_rows_decode(c, token, token, position, logits_out, true, static_cast<cudaStream_t>(stream));
}

int qb_set_batch(qb_ctx* c, int batch) {
  if (!c) return set_err(nullptr, QB_ERR_ARG, "ctx is NULL");
  if (batch < 1 || batch > kRowsMaxQ) return set_err(&c->msg, QB_ERR_UNSUPPORTED, "batch must lie in 1..8");
  if (batch > 1 && c->tp_size != 1) return set_err(&c->msg, QB_ERR_UNSUPPORTED, "batched decode runs on one GPU");
  if (batch != c->batch) {
    c->batch = batch;
    c->state_bound = false;  // the cache layout changed: bind the state again
    drop_graphs(c);
  }
  return QB_OK;
}

int qb_prefill(qb_ctx* c, const int64_t* ids, int n, int64_t* token, int64_t* position, void* logits_out,
               void* stream) {
  int rc = require_ready(c);
  if (rc) return rc;
  if (!ids || !token || !position || n <= 0) return set_err(&c->msg, QB_ERR_ARG, "bad prefill arguments");
  if (n > c->cap) return set_err(&c->msg, QB_ERR_CAPACITY, "prompt longer than the KV capacity");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(position, 0, sizeof(int64_t) * c->batch, st);
  if (e != cudaSuccess) return cuda_fail(&c->msg, e, "position reset");
  if (c->batch > 1) {
    // ids [B][n]: one batched pass per prompt column (teacher forced), the
    // column's ids gathered into the rows' token buffer
    for (int i = 0; i < n; ++i) {
      const bool last = (i == n - 1);
      if ((e = launch_ex(gather_column_i64_kernel, dim3(1), dim3(32), 0, st, ids, n, i, c->batch, c->r_pos)) !=
          cudaSuccess)
        return cuda_fail(&c->msg, e, "prompt column");
      rc = run_batch_pass(c, c->r_pos, position, token, last ? logits_out : nullptr, last, st);
      if (rc) return rc;
    }
    return QB_OK;
  }
  for (int i = 0; i < n; ++i) {
    const bool last = (i == n - 1);
    rc = run_rows_decode(c, ids + i, token, position, last ? logits_out : nullptr, last, st);
    if (rc) return rc;
  }
  return QB_OK;
}

int qb_prefill_scratch_bytes(const qb_ctx* c, int n, size_t* bytes) {
  if (!c || !bytes) return set_err(nullptr, QB_ERR_ARG, "NULL argument");
  if (n <= 0) return set_err(nullptr, QB_ERR_ARG, "n must be positive");
  *bytes = prefill_layout(c, n).total;
  return QB_OK;
}

int qb_prefill_batched(qb_ctx* c, const int64_t* ids, int n, void* scratch, size_t scratch_bytes, int64_t* token,
                       int64_t* position, void* logits_out, void* stream) {
  int rc = require_ready(c);
  if (rc) return rc;
  if (!ids || !token || !position || n <= 0) return set_err(&c->msg, QB_ERR_ARG, "bad prefill arguments");
  if (n > c->cap) return set_err(&c->msg, QB_ERR_CAPACITY, "prompt longer than the KV capacity");
  if (c->batch != 1) return set_err(&c->msg, QB_ERR_UNSUPPORTED, "block prefill takes one sequence (qb_prefill: batched contexts)");
  if (c->tp_size > 1) {
    if ((int)c->o_rows.size() != c->cfg.n_layers)
      return set_err(&c->msg, QB_ERR_ARG, "tensor-parallel block prefill needs qb_bind_prefill_weights");
    if (c->cfg.hidden % c->tp_size || (c->cfg.hidden / c->tp_size) % 8)
      return set_err(&c->msg, QB_ERR_UNSUPPORTED, "tensor-parallel block prefill needs hidden / tp_size a multiple of 8");
  }
  if (!ptr_ok(scratch) || scratch_bytes < prefill_layout(c, n).total)
    return set_err(&c->msg, QB_ERR_ARG, "scratch smaller than qb_prefill_scratch_bytes(n) or unaligned");
  return run_prefill_batched(c, ids, n, static_cast<uint8_t*>(scratch), token, position, logits_out,
                             static_cast<cudaStream_t>(stream));
}

int qb_capture_decode(qb_ctx* c, int64_t* token, int64_t* position, void* logits_out, void* stream) {
  int rc = require_ready(c);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (c->exec) {
    cudaGraphExecDestroy(c->exec);
    c->exec = nullptr;
  }
  if (c->graph) {
    cudaGraphDestroy(c->graph);
    c->graph = nullptr;
  }
  cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return cuda_fail(&c->msg, e, "begin capture");
  rc = c->batch > 1 ? run_batch_pass(c, token, position, token, logits_out, true, st)
                    : run_rows_decode(c, token, token, position, logits_out, true, st);
  cudaGraph_t graph = nullptr;
  e = cudaStreamEndCapture(st, &graph);
  if (rc == QB_OK && e == cudaSuccess) {
    e = cudaGraphInstantiate(&c->exec, graph, 0);
    if (e == cudaSuccess) {
      c->graph = graph;
      return QB_OK;
    }
  }
  if (graph) cudaGraphDestroy(graph);
  cudaGetLastError();
  if (rc) return rc;
  return cuda_fail(&c->msg, e, "decode graph capture");
}

int qb_replay_decode(qb_ctx* c, void* stream) {
  if (!c) return set_err(nullptr, QB_ERR_ARG, "ctx is NULL");
  if (!c->exec || !c->state_bound) return set_err(&c->msg, QB_ERR_STATE, "no captured decode graph");
  cudaError_t e = cudaGraphLaunch(c->exec, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(&c->msg, e, "graph launch");
  return QB_OK;
}

int qb_verify(qb_ctx* c, const int64_t* ids, int n, const int64_t* position, int64_t* predictions,
              void* logits_out, void* stream) {
  int rc = require_ready(c);
  if (rc) return rc;
  if ((rc = check_verify_args(c, ids, n, position, predictions))) return rc;
  return run_verify(c, ids, n, position, predictions, logits_out, static_cast<cudaStream_t>(stream));
}

int qb_capture_verify(qb_ctx* c, const int64_t* ids, int n, const int64_t* position, int64_t* predictions,
                      void* logits_out, void* stream) {
  int rc = require_ready(c);
  if (rc) return rc;
  if ((rc = check_verify_args(c, ids, n, position, predictions))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (c->vexec) {
    cudaGraphExecDestroy(c->vexec);
    c->vexec = nullptr;
  }
  if (c->vgraph) {
    cudaGraphDestroy(c->vgraph);
    c->vgraph = nullptr;
  }
  cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return cuda_fail(&c->msg, e, "begin capture");
  rc = run_verify(c, ids, n, position, predictions, logits_out, st);
  cudaGraph_t graph = nullptr;
  e = cudaStreamEndCapture(st, &graph);
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return cuda_fail(&c->msg, e, "end capture");
  if ((e = cudaGraphInstantiate(&c->vexec, graph, 0)) != cudaSuccess) {
    cudaGraphDestroy(graph);
    return cuda_fail(&c->msg, e, "graph instantiate");
  }
  c->vgraph = graph;
  return QB_OK;
}

int qb_replay_verify(qb_ctx* c, void* stream) {
  if (!c) return set_err(nullptr, QB_ERR_ARG, "ctx is NULL");
  if (!c->vexec || !c->state_bound) return set_err(&c->msg, QB_ERR_STATE, "no captured verify graph");
  cudaError_t e = cudaGraphLaunch(c->vexec, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(&c->msg, e, "graph launch");
  return QB_OK;
}

static int read_device_error(int* err_word, cudaStream_t st, std::string* msg) {
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(msg, e, "stream synchronize");
  int v = 0;
  e = cudaMemcpy(&v, err_word, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(msg, e, "error word read");
  if (v == 0) return QB_OK;
  cudaMemset(err_word, 0, sizeof(int));
  char buf[128];
  if (v == DEV_BAD_TOKEN) return set_err(msg, QB_ERR_ARG, "token id outside the vocabulary");
  if (v == DEV_BAD_POSITION) return set_err(msg, QB_ERR_CAPACITY, "position outside the KV capacity");
  std::snprintf(buf, sizeof(buf), "device wait timed out (site 0x%x); kernel returned early", v);
  return set_err(msg, QB_ERR_TIMEOUT, buf);
}

int qb_check(qb_ctx* c, void* stream) {
  int rc = require_ready(c);
  if (rc) return rc;
  rc = read_device_error(c->err, static_cast<cudaStream_t>(stream), &c->msg);
  if (rc == QB_ERR_TIMEOUT) {
    // A kernel that gave up left its merge tickets and arrival counters
    // mid-count: restore them so the next step starts clean.
    cudaError_t e = cudaMemset(c->counters, 0, 4096);
    if (e != cudaSuccess) return cuda_fail(&c->msg, e, "counter reset");
  }
  return rc;
}

int qb_gemm_bf16(const void* x, const void* w, void* out, const void* residual, int T, int N, int K, int epilogue,
                 void* scratch, void* stream) {
  if (!ptr_ok(x) || !ptr_ok(w) || !ptr_ok(out) || !ptr_ok(scratch))
    return set_err(nullptr, QB_ERR_ARG, "x, w, out and scratch must be 16-byte aligned device pointers");
  if (T <= 0 || N <= 0 || K <= 0 || K % 64 != 0 || N % 16 != 0)
    return set_err(nullptr, QB_ERR_UNSUPPORTED, "K must be a multiple of 64 and N of 16");
  if (epilogue < 0 || epilogue > 2) return set_err(nullptr, QB_ERR_ARG, "epilogue must be 0, 1 or 2");
  if (epilogue == 1 && !ptr_ok(residual)) return set_err(nullptr, QB_ERR_ARG, "residual must be an aligned pointer");
  int* err = reinterpret_cast<int*>(static_cast<uint8_t*>(scratch) + kScrErr);
  cudaError_t e = launch_prefill_gemm(epilogue, static_cast<const bf16*>(x), static_cast<const bf16*>(w),
                                      static_cast<bf16*>(out), static_cast<const bf16*>(residual), T, N, K, err,
                                      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "gemm launch");
  return QB_OK;
}

int qb_set_trace(qb_ctx* c, void* buffer, size_t bytes) {
  if (!c) return set_err(nullptr, QB_ERR_ARG, "ctx is NULL");
  if (buffer != nullptr && (reinterpret_cast<uintptr_t>(buffer) & 7) != 0)
    return set_err(&c->msg, QB_ERR_ARG, "trace buffer must be 8-byte aligned");
  const size_t per_launch = (size_t)kTraceMaxCtas * kTraceStamps * sizeof(unsigned long long);
  c->trace = static_cast<unsigned long long*>(buffer);
  c->trace_launches = buffer ? bytes / per_launch : 0;
  c->trace_next = 0;
  c->trace_labels.clear();
  // A captured step keeps the trace pointers it was built with: drop it.
  if (c->exec) { cudaGraphExecDestroy(c->exec); c->exec = nullptr; }
  if (c->graph) { cudaGraphDestroy(c->graph); c->graph = nullptr; }
  return QB_OK;
}

const char* qb_trace_labels(const qb_ctx* c) { return c ? c->trace_labels.c_str() : ""; }

// --------------------------------------------------------------- op level
size_t qb_op_scratch_bytes(void) { return kOpScratchBytes; }

int qb_op_check(void* scratch, void* stream) {
  if (!ptr_ok(scratch)) return set_err(nullptr, QB_ERR_ARG, "scratch is NULL or misaligned");
  return read_device_error(reinterpret_cast<int*>(static_cast<uint8_t*>(scratch) + kScrErr),
                           static_cast<cudaStream_t>(stream), nullptr);
}

int qb_norm_projection(const void* x, const void* gain, const void* w, void* out, int K, int rows, float eps,
                       int swiglu, void* stream) {
  if (!ptr_ok(x) || !ptr_ok(w) || !ptr_ok(out) || (gain && !ptr_ok(gain)))
    return set_err(nullptr, QB_ERR_ARG, "x, w, out (and gain) must be 16-byte aligned device pointers");
  if (K <= 0 || K % 128 != 0) return set_err(nullptr, QB_ERR_UNSUPPORTED, "K must be a positive multiple of 128");
  if (rows <= 0 || (swiglu && rows % 2 != 0)) return set_err(nullptr, QB_ERR_ARG, "packed gate/up width must be even");
  GemvArgs a = gemv_args(w, K, rows, x, out, nullptr);
  a.gain = static_cast<const bf16*>(gain);
  a.eps = eps;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int sms = current_sm_count();
  cudaError_t e = swiglu ? launch_gemv<EPI_SWIGLU>(a, sms, st) : launch_gemv<EPI_STORE>(a, sms, st);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "norm_projection launch");
  return QB_OK;
}

int qb_projection_residual(const void* x, const void* w, const void* residual, void* out, int K, int N,
                           void* stream) {
  if (!ptr_ok(x) || !ptr_ok(w) || !ptr_ok(out) || !residual)
    return set_err(nullptr, QB_ERR_ARG, "x, w, residual, out must be device pointers (16-byte aligned)");
  if (K <= 0 || K % 128 != 0) return set_err(nullptr, QB_ERR_UNSUPPORTED, "K must be a positive multiple of 128");
  if (N <= 0) return set_err(nullptr, QB_ERR_ARG, "N must be positive");
  GemvArgs a = gemv_args(w, K, N, x, out, nullptr);
  a.residual = static_cast<const bf16*>(residual);
  cudaError_t e = launch_gemv<EPI_RESIDUAL>(a, current_sm_count(), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "projection_residual launch");
  return QB_OK;
}

int qb_projection_residual_peer(const void* x, const void* w, const void* residual, void* out, int K, int N,
                                void* const* recv_words, int rank, int size, int sublayer, int parity,
                                const uint64_t* epoch, void* scratch, void* stream) {
  if (!ptr_ok(x) || !ptr_ok(w) || !ptr_ok(out) || !residual || !ptr_ok(scratch) || !epoch)
    return set_err(nullptr, QB_ERR_ARG, "x, w, residual, out, scratch, epoch must be device pointers (16-byte aligned)");
  if (K <= 0 || K % 128 != 0) return set_err(nullptr, QB_ERR_UNSUPPORTED, "K must be a positive multiple of 128");
  if (N <= 0) return set_err(nullptr, QB_ERR_ARG, "N must be positive");
  if (size < 1 || size > kMaxTp) return set_err(nullptr, QB_ERR_UNSUPPORTED, "size must be 1..8 ranks");
  if (rank < 0 || rank >= size) return set_err(nullptr, QB_ERR_ARG, "rank must lie in 0..size-1");
  if (sublayer < 0 || sublayer > 254 || (parity != 0 && parity != 1))
    return set_err(nullptr, QB_ERR_ARG, "sublayer must be 0..254 and parity 0 or 1");
  if (size > 1 && !recv_words) return set_err(nullptr, QB_ERR_ARG, "recv_words is NULL");
  GemvArgs a = gemv_args(w, K, N, x, out, reinterpret_cast<int*>(static_cast<uint8_t*>(scratch) + kScrErr));
  a.residual = static_cast<const bf16*>(residual);
  if (size > 1) {
    for (int p = 0; p < size; ++p) {
      if (!recv_words[p] || (reinterpret_cast<uintptr_t>(recv_words[p]) & 7) != 0)
        return set_err(nullptr, QB_ERR_ARG, "every receive buffer must be an 8-byte aligned device pointer");
      a.tp.recv[p] = static_cast<unsigned long long*>(recv_words[p]);
    }
    a.tp.epoch = reinterpret_cast<const unsigned long long*>(epoch);
    a.tp.rank = rank;
    a.tp.size = size;
    a.tp_sub = sublayer;
    a.tp_parity = parity;
    a.hidden = N;
  }
  cudaError_t e = launch_gemv<EPI_RESIDUAL>(a, current_sm_count(), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "projection_residual_peer launch");
  return QB_OK;
}

int qb_norm_greedy_head(const void* x, const void* gain, const void* w, int K, int V, float eps, void* logits_out,
                        int64_t* token_out, void* scratch, size_t scratch_bytes, void* stream) {
  if (!ptr_ok(x) || !ptr_ok(w) || !token_out || (gain && !ptr_ok(gain)) || !ptr_ok(scratch))
    return set_err(nullptr, QB_ERR_ARG, "x, w, gain, scratch must be 16-byte aligned device pointers");
  if (scratch_bytes < kOpScratchBytes) return set_err(nullptr, QB_ERR_ARG, "scratch smaller than qb_op_scratch_bytes()");
  if (K <= 0 || K % 128 != 0) return set_err(nullptr, QB_ERR_UNSUPPORTED, "K must be a positive multiple of 128");
  if (V <= 0) return set_err(nullptr, QB_ERR_ARG, "V must be positive");
  uint8_t* s = static_cast<uint8_t*>(scratch);
  GemvArgs a = gemv_args(w, K, V, x, nullptr, reinterpret_cast<int*>(s + kScrErr));
  a.gain = static_cast<const bf16*>(gain);
  a.eps = eps;
  a.logits = static_cast<bf16*>(logits_out);
  a.part_val = reinterpret_cast<float*>(s + kScrHeadVal);
  a.part_idx = reinterpret_cast<int*>(s + kScrHeadIdx);
  a.counter = reinterpret_cast<unsigned*>(s + kScrCounters) + 128;
  a.token_out = token_out;
  cudaError_t e = launch_gemv<EPI_ARGMAX>(a, current_sm_count(), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "greedy head launch");
  return QB_OK;
}

static int op_attention(const void* qkv, const void* q, const void* q_norm, const void* k_norm, const void* cos,
                        const void* sin, float eps, void* k_cache, void* v_cache, int hq, int hkv, int cap,
                        int queries, const int64_t* positions, void* out, void* scratch, size_t scratch_bytes,
                        bool pro, void* stream) {
  if (!ptr_ok(k_cache) || !ptr_ok(v_cache) || !ptr_ok(out) || !positions || !ptr_ok(scratch))
    return set_err(nullptr, QB_ERR_ARG, "caches, out, positions, scratch must be aligned device pointers");
  if (scratch_bytes < kOpScratchBytes) return set_err(nullptr, QB_ERR_ARG, "scratch smaller than qb_op_scratch_bytes()");
  if (hkv <= 0 || hq <= 0 || hq % hkv != 0) return set_err(nullptr, QB_ERR_ARG, "n_heads must be a multiple of n_kv_heads");
  if (hkv > 64) return set_err(nullptr, QB_ERR_UNSUPPORTED, "more than 64 KV heads");
  if (cap <= 0) return set_err(nullptr, QB_ERR_ARG, "capacity must be positive");
  if (queries < 1 || queries > 8) return set_err(nullptr, QB_ERR_UNSUPPORTED, "queries must be 1..8");
  const int rows = (hq / hkv) * queries;
  if (rows > 32 || (pro && rows > 16)) return set_err(nullptr, QB_ERR_UNSUPPORTED, "group x queries above 32 rows");
  const int sms = current_sm_count();
  int splits = attn_splits_for(hkv, sms);
  if (hkv * splits > kMaxAttnCtas) splits = kMaxAttnCtas / hkv > 0 ? kMaxAttnCtas / hkv : 1;
  if ((size_t)hkv * splits * 32 * 4 > 65536) return set_err(nullptr, QB_ERR_UNSUPPORTED, "too many KV heads for the op scratch");
  CUtensorMap tk, tv, dk, dv;
  if (!make_kv_map(&tk, k_cache, hkv, cap) || !make_kv_map(&tv, v_cache, hkv, cap) ||
      !make_kv_map(&dk, k_cache, hkv, cap, kDecKeys) || !make_kv_map(&dv, v_cache, hkv, cap, kDecKeys))
    return set_err(nullptr, QB_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  uint8_t* s = static_cast<uint8_t*>(scratch);
  AttnArgs a;
  std::memset(&a, 0, sizeof(a));
  a.qkv = static_cast<const bf16*>(qkv);
  a.q = static_cast<const bf16*>(q);
  a.q_norm = static_cast<const bf16*>(q_norm);
  a.k_norm = static_cast<const bf16*>(k_norm);
  a.cos = static_cast<const bf16*>(cos);
  a.sin = static_cast<const bf16*>(sin);
  a.eps = eps;
  a.pos = positions;
  a.k_cache = static_cast<bf16*>(k_cache);
  a.v_cache = static_cast<bf16*>(v_cache);
  a.out = static_cast<bf16*>(out);
  a.part_lse = reinterpret_cast<float*>(s + kScrAttnLse);
  a.part_o = reinterpret_cast<float*>(s + kScrAttnO);
  a.counters = reinterpret_cast<unsigned*>(s + kScrCounters);
  a.err = reinterpret_cast<int*>(s + kScrErr);
  a.Hq = hq;
  a.Hkv = hkv;
  a.Q = queries;
  a.cap = cap;
  a.splits = splits;
  cudaError_t e;
  // Without the prologue the cluster kernel of the verify pass runs short
  // caches (one cluster per KV head, DSMEM merge, no global round trip) and,
  // above 16 rows per KV head, long caches too, as several clusters per KV
  // head that merge through the partial rows and the tickets at the end of
  // the scratch (the split kernel's 17..32-row variant streams at a fraction
  // of the copy rate). Long caches of at most 16 rows keep the split kernel,
  // whose grid covers every SM.
  const int rcs = (!pro && rows <= kVaMaxRows && (cap < kOpRowsMaxCap || rows > 16)) ? rows_cluster_size(hkv) : 0;
  AttnArgs ra = a;  // the rows kernel's shape (the split kernel keeps `splits`)
  if (rcs > 0 && cap >= kOpRowsMaxCap) {
    ra.part_splits = splits;  // partial rows per KV head: splits x kVaMaxRows
    ra.tickets = reinterpret_cast<unsigned*>(s + kScrTickets);
    rows_attn_shape(ra, rcs);
  }
  if (rcs > 0 && (cap < kOpRowsMaxCap || ra.clusters > 1))
    e = launch_attn_rows(dk, dv, ra, rcs, static_cast<cudaStream_t>(stream));
  else
    e = launch_attn(tk, tv, &dk, &dv, a, pro, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "attention launch");
  return QB_OK;
}

int qb_grouped_attention(const void* q, const void* k_cache, const void* v_cache, int n_heads, int n_kv_heads,
                         int capacity, int queries, const int64_t* positions, void* out, void* scratch,
                         size_t scratch_bytes, void* stream) {
  if (!ptr_ok(q)) return set_err(nullptr, QB_ERR_ARG, "q must be an aligned device pointer");
  return op_attention(nullptr, q, nullptr, nullptr, nullptr, nullptr, 0.f, const_cast<void*>(k_cache),
                      const_cast<void*>(v_cache), n_heads, n_kv_heads, capacity, queries, positions, out, scratch,
                      scratch_bytes, false, stream);
}

int qb_rope_attention(const void* qkv, const void* q_norm, const void* k_norm, const void* rope_cos,
                      const void* rope_sin, float eps, void* k_cache, void* v_cache, int n_heads, int n_kv_heads,
                      int capacity, const int64_t* position, void* out, void* scratch, size_t scratch_bytes,
                      void* stream) {
  if (!ptr_ok(qkv) || !ptr_ok(q_norm) || !ptr_ok(k_norm) || !ptr_ok(rope_cos) || !ptr_ok(rope_sin))
    return set_err(nullptr, QB_ERR_ARG, "qkv, norms and rope tables must be aligned device pointers");
  return op_attention(qkv, nullptr, q_norm, k_norm, rope_cos, rope_sin, eps, k_cache, v_cache, n_heads, n_kv_heads,
                      capacity, 1, position, out, scratch, scratch_bytes, true, stream);
}

}  // extern "C"

// =========================================== allocation-free grouped attention
// Some hosts cannot let this library allocate device memory: servers and
// plugin hosts that hand out GPU memory only from their own pools sized at
// start-up (a stray cudaMalloc can stall the device and breaks their memory
// budget), or callers with a hard memory limit fixed before the first request.
// For them qb_grouped_attention_noalloc keeps the split-KV partials in the
// array below instead of a caller-provided scratch buffer. The array exists on
// every GPU that loads this library, for the life of the process.
namespace {

constexpr size_t kStaticHeaderBytes = 4096;          // error word at 0, counters at 256 (64 x u32)
constexpr size_t kStaticPartialBytes = 2u << 20;     // split partial outputs + log-sum-exps
constexpr size_t kStaticScratchBytes = kStaticHeaderBytes + kStaticPartialBytes;
constexpr int kStaticMaxDevices = 64;

static __device__ __align__(256) uint8_t g_attn_static_scratch[kStaticScratchBytes];

// Device address of g_attn_static_scratch per device. In host code the array's
// name is only a host-side stand-in, so the address must come from
// cudaGetSymbolAddress, called with the device current.
uint8_t* g_static_scratch_ptr[kStaticMaxDevices] = {};
std::mutex g_static_scratch_mu;

int static_scratch_for_current_device(uint8_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDevice");
  if (dev < 0 || dev >= kStaticMaxDevices) return set_err(nullptr, QB_ERR_UNSUPPORTED, "device index above 63");
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  if (g_static_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_static_scratch);
    if (e != cudaSuccess || p == nullptr) return cuda_fail(nullptr, e, "cudaGetSymbolAddress(static attention scratch)");
    g_static_scratch_ptr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_static_scratch_ptr[dev];
  return QB_OK;
}

}  // namespace

extern "C" int qb_grouped_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, int n_heads,
                                            int n_kv_heads, int capacity, int queries, const int64_t* positions,
                                            void* out, int* device_status, void* stream) {
  if (!ptr_ok(q) || !ptr_ok(k_cache) || !ptr_ok(v_cache) || !ptr_ok(out) || !positions)
    return set_err(nullptr, QB_ERR_ARG, "q, caches, out and positions must be aligned device pointers");
  if (n_kv_heads <= 0 || n_heads <= 0 || n_heads % n_kv_heads != 0)
    return set_err(nullptr, QB_ERR_ARG, "n_heads must be a multiple of n_kv_heads");
  if (n_kv_heads > 64) return set_err(nullptr, QB_ERR_UNSUPPORTED, "more than 64 KV heads");
  if (capacity <= 0) return set_err(nullptr, QB_ERR_ARG, "capacity must be positive");
  if (queries < 1 || queries > 8) return set_err(nullptr, QB_ERR_UNSUPPORTED, "queries must be 1..8");
  const int rows = (n_heads / n_kv_heads) * queries;
  if (rows > 32) return set_err(nullptr, QB_ERR_UNSUPPORTED, "group x queries above 32 rows");
  // One split of one KV head needs padded_rows x (128 + 1) floats.
  const int padded = rows <= 16 ? 16 : 32;
  const size_t per_split = (size_t)n_kv_heads * padded * (kAttnD + 1) * sizeof(float);
  const int fit = (int)((kStaticPartialBytes - 256) / per_split);  // 256: LSE block alignment
  if (fit < 1)
    return set_err(nullptr, QB_ERR_UNSUPPORTED,
                   "n_kv_heads x padded query rows exceeds the 2 MiB static attention scratch");
  int splits = attn_splits_for(n_kv_heads, current_sm_count());
  if (splits > fit) splits = fit;

  uint8_t* s = nullptr;
  int rc = static_scratch_for_current_device(&s);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents: clear the error word and the
  // merge counters (they must start at zero) on this call's stream.
  cudaError_t e = cudaMemsetAsync(s, 0, 512, st);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "clear static scratch header");
  if (device_status != nullptr && (e = cudaMemsetAsync(device_status, 0, sizeof(int), st)) != cudaSuccess)
    return cuda_fail(nullptr, e, "clear device status");

  CUtensorMap tk, tv;
  if (!make_kv_map(&tk, k_cache, n_kv_heads, capacity) || !make_kv_map(&tv, v_cache, n_kv_heads, capacity))
    return set_err(nullptr, QB_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  AttnArgs a;
  std::memset(&a, 0, sizeof(a));
  a.q = static_cast<const bf16*>(q);
  a.pos = positions;
  a.k_cache = static_cast<bf16*>(const_cast<void*>(k_cache));
  a.v_cache = static_cast<bf16*>(const_cast<void*>(v_cache));
  a.out = static_cast<bf16*>(out);
  const size_t lse_bytes = align_up((size_t)n_kv_heads * splits * padded * sizeof(float), 256);
  a.part_lse = reinterpret_cast<float*>(s + kStaticHeaderBytes);
  a.part_o = reinterpret_cast<float*>(s + kStaticHeaderBytes + lse_bytes);
  a.counters = reinterpret_cast<unsigned*>(s + 256);
  a.err = device_status != nullptr ? device_status : reinterpret_cast<int*>(s);
  a.Hq = n_heads;
  a.Hkv = n_kv_heads;
  a.Q = queries;
  a.cap = capacity;
  a.splits = splits;
  if (lse_bytes + (size_t)n_kv_heads * splits * padded * kAttnD * sizeof(float) > kStaticPartialBytes)
    return set_err(nullptr, QB_ERR_UNSUPPORTED, "static attention scratch too small for this call");
  e = launch_attn(tk, tv, nullptr, nullptr, a, false, st);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "attention launch");
  return QB_OK;
}
