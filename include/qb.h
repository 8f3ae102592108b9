/*
 * qb.h — C ABI of the B200 (sm_100a) Qwen3 batch-one decode engine.
 *
 * Plain pointers and sizes only. All tensors are device memory owned by the
 * caller (PyTorch in this repository), bf16 unless stated, row-major and
 * contiguous. Every function returns a status code (QB_OK == 0); the message
 * of the last failure is available from qb_last_error(). Nothing throws across
 * this boundary. Kernels are launched on the caller's stream and never
 * synchronise it, except qb_check().
 *
 * Each entry point names the reference interface it replaces
 * (rickytang666/hackthenorth, paths relative to the project root).
 */
#ifndef QB_H_
#define QB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define QB_OK 0
#define QB_ERR_ARG 1         /* shape/pointer/layout contract violated (reference: ValueError) */
#define QB_ERR_CAPACITY 2    /* position + rows beyond the KV capacity */
#define QB_ERR_CUDA 3        /* a CUDA runtime or driver call failed */
#define QB_ERR_TIMEOUT 4     /* a bounded device wait gave up; the kernel returned early */
#define QB_ERR_STATE 5       /* weights/state not bound, or graph not captured */
#define QB_ERR_UNSUPPORTED 6 /* shape outside what the kernels implement */

/* ---- model description --------------------------------------------------- */
typedef struct qb_config {
  int hidden;      /* H */
  int n_heads;     /* Hq (query heads) */
  int n_kv_heads;  /* Hkv */
  int head_dim;    /* D; the kernels implement D == 128 */
  int ffn;         /* F */
  int n_layers;    /* L */
  int vocab;       /* V */
  float rms_eps;   /* RMSNorm epsilon (hidden, q and k norms) */
} qb_config;

/* Per-layer device weights in the engine layout (bf16):
 *   input_norm [H]; qkv [Hq*D + 2*Hkv*D, H] (q rows, k rows, v rows);
 *   q_norm, k_norm [D]; o [H, Hq*D]; post_norm [H];
 *   gate_up [2F, H] with gate row j at 2j and up row j at 2j+1; down [H, F]. */
typedef struct qb_layer_weights {
  const void* input_norm;
  const void* qkv;
  const void* q_norm;
  const void* k_norm;
  const void* o;
  const void* post_norm;
  const void* gate_up;
  const void* down;
} qb_layer_weights;

typedef struct qb_ctx qb_ctx;

const char* qb_version(void);

/* Message of the last failure on `ctx`, or of the last context-free call on
 * this thread when ctx is NULL. Never returns NULL. */
const char* qb_last_error(const qb_ctx* ctx);

/* ---- engine lifecycle ---------------------------------------------------- */

/* Replaces Engine.__init__'s model preparation (dryft/engine/engine.py:176-200).
 * cfg describes the whole model. tp_rank/tp_size: tensor-parallel slot (0/1
 * for one GPU). With tp_size > 1 this rank owns KV heads
 * [r*Hkv/n, (r+1)*Hkv/n) with their query heads, FFN columns [r*F/n, (r+1)*F/n)
 * and vocabulary rows [r*V/n, (r+1)*V/n); the weights bound later are that
 * shard (see qb_bind_weights) and qb_tp_init must be called before a step.
 * The reference has no multi-GPU path; this follows its single-GPU arithmetic
 * with fp32 partial sums reduced across ranks before the one bf16 rounding. */
int qb_create(const qb_config* cfg, int device, int tp_rank, int tp_size, qb_ctx** out);

/* NCCL unique id for a tensor-parallel group (rank 0 creates it and shares the
 * bytes with the other ranks); `bytes` >= 128. */
int qb_nccl_unique_id(void* out, size_t bytes);

/* Join the tensor-parallel group: one NCCL communicator per context, used for
 * an fp32 all-reduce of [H] after every o-proj and down projection (when the
 * peer-memory reduction is off), the all-gathers of the block prefill and an
 * 8-byte all-gather of each rank's greedy candidate. No-op when tp_size == 1. */
int qb_tp_init(qb_ctx* ctx, const void* unique_id);
int qb_destroy(qb_ctx* ctx);

/* Borrow device weights (no copy). lm_head may equal embed (tied).
 * Replaces the module surgery of dryft/engine/engine.py:190-199.
 * Under tensor parallelism each table holds this rank's shard: qkv rows of its
 * q heads, k heads and v heads; o [H, Hq*D/n] (its input columns); gate_up
 * [2F/n, H]; down [H, F/n]; lm_head [V/n, H]; embed and norms whole. */
int qb_bind_weights(qb_ctx* ctx, const qb_layer_weights* layers, int n_layers,
                    const void* embed, const void* final_norm, const void* lm_head);

/* Bytes of workspace qb_bind_state needs (activations, split-KV partials,
 * counters, error word). */
int qb_workspace_bytes(const qb_ctx* ctx, size_t* bytes);

/* Borrow the decode state: K and V caches [L, Hkv/n, capacity, D] (bf16,
 * zero-filled by the caller, as KVCache does: dryft/engine/decode.py:25-46),
 * the RoPE tables [capacity, D] (bf16 cos and sin rows for positions
 * 0..capacity-1: dryft/engine/decode.py:49-67), and the workspace. The
 * workspace is zeroed here (synchronously). */
int qb_bind_state(qb_ctx* ctx, void* k_cache, void* v_cache, int capacity,
                  const void* rope_cos, const void* rope_sin,
                  void* workspace, size_t workspace_bytes);

/* Batched decode: decode `batch` (1..8) sequences together on one GPU
 * (DecodeState at B > 1, dryft/engine/decode.py:102-138). Call before
 * qb_bind_state (a change of batch unbinds the state): the caches bound next
 * are [L][batch][Hkv][capacity][D] (sequence b of layer l in slice b), and
 * qb_decode_step / qb_capture_decode / qb_prefill then take token[batch] and
 * position[batch] (one entry per sequence, positions may differ), logits
 * [batch][V], and qb_prefill takes ids [batch][n]. Every weight is streamed
 * once per step for all sequences (the rows kernels of the verify pass).
 * qb_verify and qb_prefill_batched take one sequence. QB_ERR_UNSUPPORTED for
 * batch > 1 under tensor parallelism. */
int qb_set_batch(qb_ctx* ctx, int batch);

/* One batch-one decode step: DecodeState.step (dryft/engine/decode.py:126-138).
 * Reads *token (int64, device) at *position (int64, device), appends its K/V,
 * writes the greedy next token to *token and increments *position.
 * logits_out (device bf16 [V], this rank's [V/tp_size] shard under tensor
 * parallelism) may be NULL. Graph-capturable: no host sync, no allocation.
 * Fails with QB_ERR_CAPACITY only when detectable on the host. */
int qb_decode_step(qb_ctx* ctx, int64_t* token, int64_t* position, void* logits_out,
                   void* stream);

/* Prefill: DecodeState.prefill / prefill.prefill (dryft/engine/decode.py:157-166,
 * dryft/engine/prefill.py:6-26). ids: device int64 [n]. Writes K/V for
 * positions 0..n-1, the first generated token to *token and sets
 * *position = n. Each prompt row runs through the decode kernels. */
int qb_prefill(qb_ctx* ctx, const int64_t* ids, int n, int64_t* token, int64_t* position,
               void* logits_out, void* stream);

/* Batched prefill: the prompt rows as dense blocks (tcgen05 projection GEMMs,
 * causal flash attention), the path the reference takes for prompt rows
 * (dryft/engine/attention.py:92-98, dryft/engine/prefill.py:6-26). Same
 * contract as qb_prefill (K/V for positions 0..n-1, first token to *token,
 * *position = n); scratch: a device buffer of qb_prefill_scratch_bytes(n)
 * bytes (prompt-row activations, plus the all-gather buffers under tensor
 * parallelism). Under tensor parallelism every rank calls it with the same
 * ids on its own stream, after qb_bind_prefill_weights: each rank runs its
 * heads and FFN slice; the o-proj and down projections run column-parallel
 * (the attention output and SwiGLU activations all-gathered into whole rows,
 * each rank's [n][hidden/tp_size] output columns all-gathered into the next
 * residual: four NCCL all-gathers per layer, then one 8-byte all-gather for
 * the head), so the K/V rows and the first token equal the single-GPU
 * prefill's; logits_out is this rank's [V/tp_size] shard. One sequence
 * (batch 1). hidden / tp_size must be a multiple of 8. */
int qb_prefill_scratch_bytes(const qb_ctx* ctx, int n, size_t* bytes);
/* The row shards of the tensor-parallel block prefill's column-parallel
 * projections, per layer: o_rows[l] = rows [r*H/n, (r+1)*H/n) of o
 * ([H/n][Hq*D], every input column) and down_rows[l] = the same rows of down
 * ([H/n][F]). Borrowed (no copy); required before qb_prefill_batched when
 * tp_size > 1, unused otherwise. */
int qb_bind_prefill_weights(qb_ctx* ctx, const void* const* o_rows, const void* const* down_rows, int n_layers);
int qb_prefill_batched(qb_ctx* ctx, const int64_t* ids, int n, void* scratch, size_t scratch_bytes,
                       int64_t* token, int64_t* position, void* logits_out, void* stream);

/* Capture qb_decode_step(token, position, logits_out) into a CUDA graph owned
 * by ctx (dryft/engine/decode.py:140-155), and replay it. */
int qb_capture_decode(qb_ctx* ctx, int64_t* token, int64_t* position, void* logits_out,
                      void* stream);
int qb_replay_decode(qb_ctx* ctx, void* stream);

/* The verify pass of speculative decoding: DecodeState.verify_step /
 * capture_verifier (dryft/engine/decode.py:168-192). ids: device int64 [n]
 * (the current token, then n-1 draft tokens), n in 1..8, run at positions
 * *position .. *position+n-1 (device int64, not modified: the caller applies
 * the accepted count, dryft/engine/decode.py:194-206); their K/V are written
 * to the cache. predictions (device int64 [n]): the greedy token after each
 * row; logits_out (device bf16 [n][V], [n][V/tp_size] of this rank's
 * vocabulary shard under tensor parallelism) may be NULL. Every weight is
 * streamed once for all n rows. Tensor parallel: every rank calls it in the
 * same order (peer-memory reduction of the o-proj and down rows, or NCCL with
 * QB_TP_NCCL=1); predictions are identical on all ranks. */
int qb_verify(qb_ctx* ctx, const int64_t* ids, int n, const int64_t* position, int64_t* predictions,
              void* logits_out, void* stream);
int qb_capture_verify(qb_ctx* ctx, const int64_t* ids, int n, const int64_t* position,
                      int64_t* predictions, void* logits_out, void* stream);
int qb_replay_verify(qb_ctx* ctx, void* stream);

/* Synchronise `stream` and report device-side errors (bounded waits that gave
 * up, out-of-range token ids). Clears the device error word. */
int qb_check(qb_ctx* ctx, void* stream);

/* Tracing (diagnostics; the reference's profiling is external, e.g. the timing
 * harness of dryft/experiments): give the context a device buffer (8-byte
 * aligned, zero-filled by the caller) and every launch of the decode steps
 * built afterwards records, per CTA, %globaltimer stamps in ns at its start,
 * after griddepcontrol.wait, when its first input stage landed, when its main
 * loop ended and at its exit: launch i, CTA b, stamp k at
 * buffer[(i * 256 + b) * 8 + k] (uint64; CTAs past 256 are not recorded,
 * stamps a kernel does not take stay 0). Launches beyond the buffer are not
 * traced. A captured decode graph keeps the buffer it was built with, so this
 * call drops the context's decode graph (capture again). NULL turns tracing
 * off. Replays overwrite the same records: the buffer holds the latest step. */
int qb_set_trace(qb_ctx* ctx, void* buffer, size_t bytes);
/* One label per traced launch of the last decode step built ("qkv 0", "attn 0",
 * "o 0", "gateup 0", "down 0", ..., "head 36"), each ended by '\n'. */
const char* qb_trace_labels(const qb_ctx* ctx);

/* ---- op-level entry points (the reference's kernel wrappers) ------------- */

/* Prefill projection on tcgen05 tensor cores: out = epilogue(x . w^T) for
 * x [T][K], w [N][K] bf16 row-major, fp32 accumulation, one bf16 rounding
 * (the dense prompt-row projections of dryft/engine/attention.py:92-98 with the
 * roundings of kernels/projection.py:13-83). epilogue 0: out [T][N] = bf16(y);
 * 1: out = bf16(bf16(y) + residual) (residual [T][N]); 2: out [T][N/2] =
 * bf16(bf16(silu(bf16 y[2j])) * bf16 y[2j+1]) over gate/up-interleaved rows.
 * K multiple of 64, N multiple of 16. scratch: qb_op_scratch_bytes() bytes
 * (device error word). */
int qb_gemm_bf16(const void* x, const void* w, void* out, const void* residual, int T, int N, int K,
                 int epilogue, void* scratch, void* stream);

/* RMSNorm(x; gain, eps) fused with y = W . x, fp32 accumulation, one bf16
 * rounding. gain == NULL skips the norm. swiglu != 0: W is [2N, K] with gate
 * and up rows interleaved and y[j] = bf16(bf16(silu(gate_j)) * up_j).
 * Replaces norm_projection (dryft/engine/kernels/projection.py:36-53).
 * x [K], W [rows, K], out [N]; K a multiple of 128. */
int qb_norm_projection(const void* x, const void* gain, const void* w, void* out,
                       int K, int rows, float eps, int swiglu, void* stream);

/* out = bf16(bf16(W . x) + residual). Replaces output_projection_residual
 * (dryft/engine/kernels/projection.py:70-83) and down_residual
 * (dryft/engine/kernels/down.py:288-296). x [K], W [N, K], residual/out [N];
 * K a multiple of 128. */
int qb_projection_residual(const void* x, const void* w, const void* residual, void* out,
                           int K, int N, void* stream);

/* One rank's share of a tensor-parallel output or down projection with the
 * cross-rank reduction fused into the epilogue: the op-level form of the
 * o-proj / down sublayer under tensor parallelism. The reference has one GPU
 * only; this keeps the single rounding of output_projection_residual
 * (dryft/engine/kernels/projection.py:70-83): out = bf16(bf16(sum over ranks
 * of W_r . x_r) + residual), the partials added in rank order.
 * x [K] (this rank's input columns), W [N, K] (this rank's column shard),
 * residual/out [N]. recv_words: host array of `size` device pointers, entry p
 * = rank p's receive words [2][size][N] (uint64; peers' buffers reachable by
 * this GPU, e.g. IPC-mapped). Every rank's grid writes {token, fp32 partial}
 * words of its rows into recv_words[p][parity][rank][row] of every rank p,
 * then waits (bounded, 2 s) until its own buffer holds the words of every
 * rank for the same token, token = (*epoch + 1) * 256 + sublayer + 1 (epoch:
 * device uint64 the caller advances between uses of the same sublayer id).
 * All ranks must use the same GPU model (same row partition). A wait that
 * gives up records a timeout in the scratch error word (qb_op_check returns
 * QB_ERR_TIMEOUT) and the kernel returns; the output of that call is not
 * defined. size 1 is qb_projection_residual. scratch: qb_op_scratch_bytes(). */
int qb_projection_residual_peer(const void* x, const void* w, const void* residual, void* out, int K, int N,
                                void* const* recv_words, int rank, int size, int sublayer, int parity,
                                const uint64_t* epoch, void* scratch, void* stream);

/* Scratch bytes the op-level head and attention calls need (a multiple of
 * 256). The scratch must be zero-filled before its first use; the kernels
 * leave their counters at zero again. */
size_t qb_op_scratch_bytes(void);

/* Final RMSNorm + LM-head GEMV + greedy argmax with the lowest index on exact
 * ties, logits rounded to bf16 before the comparison. Replaces the final norm
 * (dryft/engine/decode.py:95) and greedy_token (dryft/engine/kernels/greedy.py:45-60).
 * x [K], gain [K] or NULL, W [V, K]; logits_out bf16 [V] or NULL;
 * token_out device int64. */
int qb_norm_greedy_head(const void* x, const void* gain, const void* w, int K, int V,
                        float eps, void* logits_out, int64_t* token_out,
                        void* scratch, size_t scratch_bytes, void* stream);

/* Split-KV grouped-query attention over a fixed-capacity cache for `queries`
 * rows at absolute device positions (int64 [queries], ascending, consecutive
 * for queries > 1); query row j sees cache slot c iff c <= positions[j]; slots
 * past the last position are never read. q [queries, Hq, D] (already
 * normalised and rotated), k_cache/v_cache [Hkv, capacity, D],
 * out [queries, Hq, D]. Replaces grouped_attention
 * (dryft/engine/kernels/attention.py:213-237). queries in 1..8. */
int qb_grouped_attention(const void* q, const void* k_cache, const void* v_cache,
                         int n_heads, int n_kv_heads, int capacity, int queries,
                         const int64_t* positions, void* out,
                         void* scratch, size_t scratch_bytes, void* stream);

/* Decode attention with its prologue fused: per-head q/k RMSNorm + RoPE from
 * the packed QKV row, K/V appended at *position, then attention of the one
 * query row over slots 0..*position. Replaces norm_rope_cache +
 * grouped_attention on the batch-one path (dryft/engine/fused_layer.py:123-130,
 * dryft/engine/kernels/fused.py:153-165) and prologue_attention
 * (dryft/engine/kernels/attention.py:162-196). qkv [Hq*D + 2*Hkv*D];
 * q_norm/k_norm [D]; rope_cos/rope_sin [capacity, D]; out [Hq, D]. */
int qb_rope_attention(const void* qkv, const void* q_norm, const void* k_norm,
                      const void* rope_cos, const void* rope_sin, float eps,
                      void* k_cache, void* v_cache, int n_heads, int n_kv_heads,
                      int capacity, const int64_t* position, void* out,
                      void* scratch, size_t scratch_bytes, void* stream);

/* qb_grouped_attention without a scratch argument, for callers that cannot
 * let this library allocate device memory (hosts that hand out GPU memory only
 * from their own pools sized at start-up, or that run under a memory limit
 * fixed before the first request). No counterpart in the reference.
 * Allocates nothing: the split-KV partials live in a 2 MiB + 4 KiB static
 * device array built into libqb.so, present on every GPU that loads the
 * library until the process exits. The first call on a device looks up that
 * array's device address (cudaGetSymbolAddress, with the device current);
 * make that first call before any stream capture. Limits: those of
 * qb_grouped_attention (head_dim 128, <= 64 KV heads, queries 1..8, group x
 * queries <= 32 rows); the split count is reduced so the partials fit in
 * 2 MiB, and a call whose single split would not fit returns
 * QB_ERR_UNSUPPORTED. Every call shares the one array and clears its counters
 * first, so calls that overlap on the GPU (different streams, or different
 * host threads) race and must be serialised by the caller. device_status:
 * optional device int, zeroed by the call and set non-zero by a device-side
 * error (same codes as the error word qb_op_check reads); with NULL such
 * errors are not reported. */
int qb_grouped_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                 int n_heads, int n_kv_heads, int capacity, int queries,
                                 const int64_t* positions, void* out, int* device_status,
                                 void* stream);

/* Read the device error word of an op-level scratch (synchronises stream). */
int qb_op_check(void* scratch, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* QB_H_ */
