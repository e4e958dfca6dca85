/*
 * b2d.h — C ABI of the B200 decode engine (libb2d.so).
 *
 * The engine runs the fused 24-layer decode step of the 306M decoder
 * (embedding -> N x [RMSNorm, QKV, RoPE, GQA attention over the KV cache,
 * O-proj, RMSNorm, SwiGLU] -> final norm -> tied-embedding logits -> argmax)
 * as one persistent sm_100a kernel spanning every SM.
 *
 * Every entry point takes plain pointers and sizes: device pointers for the
 * tensors (the caller owns and allocates them, e.g. through PyTorch) and a
 * CUDA stream passed as `void*` (a `cudaStream_t`, NULL = legacy default
 * stream).  Calls are stream-ordered and asynchronous unless stated.  Every
 * call returns a b2d_status; no call aborts the process or traps the GPU.
 *
 * Reference interfaces replaced (paths inside zahlmann/transformer):
 *   b2d_decode_step      <- kernels/multi_sm_decode.py:369-432
 *                           multi_sm_decode_nlayer(w, config, token_id, pos,
 *                           kv_packed, kv_splits=1) -> (next_token, logits, kv_out)
 *                           and the jax_triton.triton_call at :402-430
 *   b2d_weights_layout   <- kernels/fused_decode_nlayer.py:250-270 pack_weights and
 *                           :299-321 prepare_decode_weights_nlayer (packed format)
 *   b2d_kv_layout        <- kernels/fused_decode_nlayer.py:273-296 pack_kv_caches /
 *                           unpack_kv_caches (KV format; kept identical)
 *   b2d_sample           <- generate.py:28-65 sample_token (host numpy sampler)
 *   b2d_model_create / b2d_workspace_create
 *                        <- the per-call `jnp.zeros(workspace)` at
 *                           kernels/multi_sm_decode.py:390-400 (allocated once here)
 */
#ifndef B2D_H_
#define B2D_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B2D_API __attribute__((visibility("default")))
#else
#define B2D_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  B2D_OK = 0,
  B2D_ERR_INVALID_ARG = 1,    /* rejected on the host before any launch */
  B2D_ERR_UNSUPPORTED = 2,    /* model shape not compiled into this library */
  B2D_ERR_CUDA = 3,           /* a CUDA runtime call failed (see b2d_cuda_error) */
  B2D_ERR_NO_MEMORY = 4,
  B2D_ERR_LAUNCH = 5,         /* cooperative launch refused (grid not co-resident) */
  B2D_ERR_DEVICE_TIMEOUT = 6, /* a bounded in-kernel wait ran out (status word) */
  B2D_ERR_DEVICE_INPUT = 7,   /* kernel saw a token/pos out of range (status word) */
  B2D_ERR_DEVICE_HALTED = 8,  /* workspace holds an earlier device error; reset it */
  B2D_ERR_SCRATCH_LIMIT = 9   /* needs more than b2d_decode_step_static's fixed scratch */
} b2d_status;

/* Model shape.  Same keys as the reference config dict (model.py:37-47). */
typedef struct {
  int32_t vocab_size;
  int32_t d_model;
  int32_t n_heads;
  int32_t n_kv_heads;
  int32_t n_layers;
  int32_t d_head;
  int32_t d_ff;
  int32_t context_len;
  float rms_eps;   /* 1e-5, model.py:94 */
  float rope_base; /* 10000, model.py:101 */
} b2d_config;

/*
 * Packed weight buffer layout (bytes from the buffer base; every section is
 * 256-byte aligned).  All matrices are bf16, stored "output-row major": row r
 * holds the weights that produce output r, contiguous along the reduction dim,
 * so a GEMV streams whole rows.  Per layer l, at l * layer_stride:
 *   qkv  [(H + 2*KVH) * dh][d]   rows: q (head-major), then k, then v
 *   o    [d][d]
 *   gu   [d_ff][2][d]            gate row j, then up row j
 *   down [d][d_ff]
 * then emb [vocab][d] bf16 (token_emb, read in place as the tied output
 * projection), then f32 vectors ln1 [L][d], ln2 [L][d], lnf [d], and the RoPE
 * tables cos/sin [context_len][dh/2] (model.py:101-107, f32).
 */
typedef struct {
  uint64_t layer_stride;
  uint64_t off_qkv, off_o, off_gu, off_down; /* within a layer */
  uint64_t off_emb, off_ln1, off_ln2, off_lnf, off_cos, off_sin;
  uint64_t total_bytes;
} b2d_weights_layout_t;

/* KV cache layout of one sequence, bf16 elements, identical to the reference
 * pack_kv_caches: [layer][K|V][kv_head][context_len][d_head], K post-RoPE. */
typedef struct {
  uint64_t elems_per_seq;
  uint64_t layer_elems; /* 2 * kv_heads * context_len * d_head */
  uint64_t kv_half_elems; /* kv_heads * context_len * d_head */
} b2d_kv_layout_t;

typedef struct b2d_model b2d_model;
typedef struct b2d_ws b2d_ws;

/* Sampling parameters, same meaning as generate.py:28-65. */
typedef struct {
  double temperature; /* 0 = greedy argmax; applied as float32 (numpy weak scalar) */
  double top_p;       /* 1 = off; compared in float64 like np.searchsorted */
  double rep_penalty; /* 1 = off; applied as float32 */
} b2d_sampling;

B2D_API const char* b2d_status_str(b2d_status s);
/* Last CUDA error string seen by this thread's failing call ("" if none). */
B2D_API const char* b2d_cuda_error(void);
/* 1 if this library was compiled with kernels for `cfg`'s shape. */
B2D_API int b2d_config_supported(const b2d_config* cfg);

B2D_API b2d_status b2d_weights_layout(const b2d_config* cfg, b2d_weights_layout_t* out);
B2D_API b2d_status b2d_kv_layout(const b2d_config* cfg, b2d_kv_layout_t* out);

/* Binds a packed weight buffer (device memory on `device`, caller-owned,
 * must outlive the model).  Nothing is copied. */
B2D_API b2d_status b2d_model_create(const b2d_config* cfg, const void* weights_dev,
                            uint64_t weights_bytes, int device, b2d_model** out);
B2D_API b2d_status b2d_model_destroy(b2d_model* m);
/* Number of CTAs the B=1 decode kernel launches: whole clusters of 4 CTAs
 * that fit co-resident (the cluster kernel), or one per SM (the flat kernel,
 * used where the cluster grid does not fit). */
B2D_API int b2d_model_grid(const b2d_model* m);

/* Workspace: inter-CTA exchange words, control words.  Allocated once here;
 * nothing is allocated per step.  One workspace per stream; not re-entrant. */
B2D_API b2d_status b2d_workspace_create(b2d_model* m, int max_batch, b2d_ws** out);
B2D_API b2d_status b2d_workspace_destroy(b2d_ws* ws);
/* Clears the exchange words and the device status (after a device error). */
B2D_API b2d_status b2d_workspace_reset(b2d_ws* ws, void* stream);
/* Synchronises `stream`, reads the device status word.  Returns B2D_OK or
 * the device error (B2D_ERR_DEVICE_*); *detail gets the raw status word. */
B2D_API b2d_status b2d_last_error(b2d_ws* ws, void* stream, uint32_t* detail);

/*
 * One decode step for `batch` sequences.
 *   tok_dev      int32[batch]  token fed at this step
 *   pos_dev      int32[batch]  its position (0-based); K/V written there
 *   kv_dev       bf16 KV caches, b2d_kv_layout per sequence, batch-major
 *   logits_dev   f32[batch][vocab] or NULL (then only the argmax is produced)
 *   next_tok_dev int32[batch]  argmax token (first index on ties)
 * batch == 1 runs the persistent megakernel.
 */
B2D_API b2d_status b2d_decode_step(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev,
                           const int32_t* pos_dev, int batch, void* kv_dev,
                           float* logits_dev, int32_t* next_tok_dev, void* stream);

/*
 * One greedy B=1 decode step with host values (no reference counterpart; the
 * reference's generate.py:112 loop reads the token back each step): tok / pos
 * (host ints, range-checked here) travel in the launch's arguments, the step
 * of b2d_decode_step runs, and the kernel writes the argmax into a mapped
 * pinned word of the workspace (allocated on first use); the call
 * synchronises `stream` and *next_tok (host) receives it.  Device-side
 * failures (the status word) are read with b2d_last_error, as for
 * b2d_decode_step.  Not capturable (it synchronises).
 */
B2D_API b2d_status b2d_decode_token(b2d_model* m, b2d_ws* ws, int32_t tok, int32_t pos, void* kv_dev,
                                    float* logits_dev, int32_t* next_tok, void* stream);

/*
 * Several greedy decode steps of one sequence (batch 1) in ONE launch: step s
 * consumes the token produced by step s-1 (the first consumes *tok_dev) at
 * position *pos_dev + s, appends its K/V to kv_dev and writes its argmax to
 * tokens_dev[s] (int32[n_steps]); logits_dev (or NULL) receives the last
 * step's logits.  The weights stream through the SMs without a break between
 * steps.  Same math and results as n_steps calls of b2d_decode_step feeding
 * next_tok back; *pos_dev + n_steps <= context_len (else the status word
 * reports a bad position).  No counterpart in the reference's kernels (one
 * launch per token, generate.py:112).
 */
B2D_API b2d_status b2d_decode_steps(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev, const int32_t* pos_dev,
                                    int n_steps, void* kv_dev, int32_t* tokens_dev, float* logits_dev,
                                    void* stream);

/*
 * Batched decode step over a paged KV pool (no
 * reference counterpart: the reference's batched kernels were deleted).
 *   tok_dev / pos_dev int32[batch]; pos < 0 marks a sequence inactive for this
 *                     step (no cache write; its outputs are not meaningful)
 *   kv_pool_dev       bf16 [n_layers][num_blocks][K|V][kv_heads][16][d_head]
 *   block_table_dev   int32[batch][blocks_per_seq]: physical block of
 *                     positions 16i..16i+15 of each sequence
 *   logits_dev        f32[batch][vocab] or NULL (workspace buffer used)
 *   next_tok_dev      int32[batch] argmax
 * Needs a workspace created with max_batch >= 2.  Projections run on the
 * tensor cores (tcgen05); out-of-range tokens / table entries set the status
 * word read by b2d_last_error.  From the second call with the same pointers,
 * batch and pool shape, the step's kernel sequence is replayed from a CUDA
 * graph cached in the workspace (16 argument sets, least recently used
 * replaced): keep the argument buffers alive and reuse them between steps
 * (their contents may change).  Free a pointer that a cached graph holds
 * only after the step that used it has completed.
 */
B2D_API b2d_status b2d_decode_step_paged(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev,
                                         const int32_t* pos_dev, int batch, void* kv_pool_dev,
                                         const int32_t* block_table_dev, int blocks_per_seq,
                                         int num_blocks, float* logits_dev, int32_t* next_tok_dev,
                                         void* stream);

/*
 * Device prefill (replaces the JAX prefill of generate.py:68-89 /
 * model.py:194-231 for the decode cache): feeds n_tokens prompt tokens
 * (tok_dev, int32) at positions start_pos.. of ONE sequence through the
 * batched tensor-core step, up to 512 positions per chunk, writing their K/V into
 * kv_dev (one sequence's cache in the reference layout, b2d_kv_layout).
 * Outputs the logits of the last position (f32 [vocab], or NULL) and its
 * argmax (or NULL).  Each position's math is the decode step's at that
 * position.  start_pos + n_tokens <= context_len.
 */
B2D_API b2d_status b2d_prefill(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev, int n_tokens, int start_pos,
                               void* kv_dev, float* logits_dev, int32_t* next_tok_dev, void* stream);

/*
 * b2d_prefill into a paged KV pool (the layout of b2d_decode_step_paged):
 * the sequence's positions are addressed through its block-table row
 * table_row_dev (int32 [blocks_per_seq]; every entry that covers positions
 * start_pos .. start_pos + n_tokens - 1 must name a block < num_blocks).
 * Same math and outputs as b2d_prefill; admits a request into a running
 * batch (the reference's serve.py / paged_kv.py, deleted upstream and
 * described in knowledge/program.md:213-216, 257).
 * start_pos + n_tokens <= min(context_len, 16 * blocks_per_seq).
 */
B2D_API b2d_status b2d_prefill_paged(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev, int n_tokens,
                                     int start_pos, void* kv_pool_dev, const int32_t* table_row_dev,
                                     int blocks_per_seq, int num_blocks, float* logits_dev,
                                     int32_t* next_tok_dev, void* stream);

/*
 * Prefill of several sequences in one pass over the weights (chunked prefill
 * for a continuous batch; the reference's prefill, model.py:194-231, takes
 * one padded prompt at a time).  Row i feeds token tok_dev[i] at position
 * pos_dev[i] of the sequence whose block-table row is table_dev[i][0..
 * blocks_per_seq) (rows of one sequence carry the same table row).  Every
 * row's K/V is written into the paged pool before any row attends, so a row
 * sees the positions <= its own of its sequence that are in the pool or among
 * this call's rows; a sequence longer than one call goes in several calls,
 * earlier positions first.  Rows with pos < 0 are idle.  The last n_out rows
 * (0 <= n_out <= n_rows; put each sequence's last prompt row there) get
 * logits (f32 [n_out][vocab] in logits_dev, or NULL) and their argmax (int32
 * [n_out] in next_tok_dev, or NULL); n_out = 0 writes the cache only.
 * 1 <= n_rows <= b2d_prefill_rows_max() (512).
 */
B2D_API b2d_status b2d_prefill_rows(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev, const int32_t* pos_dev,
                                    int n_rows, void* kv_pool_dev, const int32_t* table_dev, int blocks_per_seq,
                                    int num_blocks, int n_out, float* logits_dev, int32_t* next_tok_dev,
                                    void* stream);
B2D_API int b2d_prefill_rows_max(void);

/* Kernels launched by the last b2d_decode_step_paged (or prefill chunk). */
B2D_API int b2d_batched_launches(const b2d_ws* ws);

/*
 * Device sampler, one sequence per CTA (generate.py:28-65 semantics).
 *   logits_dev   f32[batch][vocab]     (read only)
 *   history_dev  int32[batch][hist_cap] tokens generated so far (prompt excluded)
 *   hist_len_dev int32[batch]          valid entries in history
 *   uniforms_dev f64[batch]            one uniform in [0,1) per sequence (the
 *                                      value np.random.choice would draw)
 *   out_tok_dev  int32[batch]
 */
B2D_API b2d_status b2d_sample(b2d_ws* ws, const float* logits_dev, int batch, int vocab,
                      const int32_t* history_dev, int hist_cap,
                      const int32_t* hist_len_dev, const double* uniforms_dev,
                      const b2d_sampling* params, int32_t* out_tok_dev, void* stream);

/*
 * b2d_decode_step_static: one decode step (batch 1) that allocates nothing.
 * No counterpart in the reference (its wrapper allocates a fresh workspace
 * with every call).  It exists for callers that cannot allocate device
 * memory themselves or through this library: hosts that own every device
 * buffer (a serving process with its own memory pool, a plugin host) or code
 * running where cudaMalloc is not permitted.  Instead of a workspace it uses
 * one fixed 4 MiB array of device memory inside the library (held by every
 * GPU that loads it, until exit); a model whose exchange area does not fit
 * gets B2D_ERR_SCRATCH_LIMIT.  The caller passes the packed weights, the
 * inputs and the outputs exactly as for b2d_decode_step on the current
 * device (every pointer is checked to be device memory of the current device).
 * The first call on a device looks up the array's device address,
 * so make it before any stream capture.  Each call clears the array on
 * `stream` before launching; calls that overlap on the GPU race on it.  No
 * model or workspace handle, no cudaMalloc/cudaFree, no host heap use.
 */
B2D_API b2d_status b2d_decode_step_static(const b2d_config* cfg, const void* weights_dev,
                                          uint64_t weights_bytes, const int32_t* tok_dev,
                                          const int32_t* pos_dev, void* kv_dev, float* logits_dev,
                                          int32_t* next_tok_dev, void* stream);
/*
 * Device status of the most recent b2d_decode_step_static call on the current
 * device, without a workspace: synchronises `stream`, then reads the status
 * word of the fixed array's control block.  Returns B2D_OK, or
 * B2D_ERR_DEVICE_TIMEOUT / B2D_ERR_DEVICE_INPUT (a token or position out of
 * range, read on the device) with the raw word in *detail.  Each static call
 * clears that word before it launches, so a later call replaces an earlier
 * call's error: check after every call whose inputs the host has not
 * validated.  Allocates nothing.  No counterpart in the reference (it has no
 * device status at all).
 */
B2D_API b2d_status b2d_static_last_error(void* stream, uint32_t* detail);

/*
 * Test hook, not part of the reference surface: bound every in-kernel wait by
 * `wait_ns` and split the work over `extra_ctas` more CTAs than are launched,
 * so the words those phantom CTAs own are never written.  A fault-detection
 * test uses it to make a wait run out and read B2D_ERR_DEVICE_TIMEOUT back
 * from b2d_last_error without hanging or faulting the GPU.
 */
B2D_API b2d_status b2d_debug_set(b2d_ws* ws, uint64_t wait_ns, int extra_ctas);

/*
 * Diagnostics (no reference counterpart; the reference only times whole
 * steps, profile_kernels.py:44-64).  b2d_debug_trace: every CTA records
 * global-timer stamps (ns) at its phase boundaries into buf_dev
 * [grid][stamps_per_cta] (slot 0 = start, 13 per layer, 3 final; NULL/0 turns
 * it off).  b2d_debug_tune: knob 1 = sleep (ns) between failed polls of the
 * exchange words (0 = spin); knob 2 = weight-stream copies in flight per CTA
 * (1..12, default 4); knob 3 = batched step with (1, default) or without (0)
 * programmatic dependent launch; knob 4 = batched step K split forced to
 * 1..8 (0 = automatic); knob 5 = batched attention units (warps) per
 * (sequence, kv head) forced to 1..32, used as 1, 2 or 4 (rounded down,
 * capped at 4; 0 = automatic); knob 6 = device address of a uint64
 * buffer [257 launches][256 CTAs][8] that the batched step's projections fill
 * with global-timer stamps (0 = off); knob 7 = device address of a uint64
 * buffer [grid][3][stride] for the B=1 step's weight stages (copy issued /
 * stage seen full / consumed by warp 0), knob 8 = that stride (0 = off);
 * knob 9 = device address of a uint64 buffer [n_layers][8192 units][8] that
 * the batched step's attention fills with global-timer stamps (0 = off);
 * knob 10 = device address of a uint64 buffer [batch][8] of b2d_sample phase
 * stamps (0 = off); knob 11 = b2d_decode_step_paged replays a cached CUDA
 * graph for repeated argument sets (1, default) or launches directly (0);
 * knob 12 = the B=1 step on the flat kernel (1) or on the cluster kernel
 * where it fits (0, default); knob 13 = b2d_sample's top-p draws on a
 * cluster of 16 CTAs per sequence where the batch fits one wave of such
 * clusters, else of 8 where that fits, else one CTA per sequence (0,
 * default); on one CTA per sequence (1); or on clusters of 8 where they fit
 * one wave (2); knob 14 = the B=1 cluster grid
 * launched without the cooperative attribute (1; for profilers, which cannot
 * replay a cooperative launch) or with it (0, default).
 * Every b2d_debug_tune call drops the cached graphs' validity.
 */
B2D_API b2d_status b2d_debug_trace(b2d_ws* ws, uint64_t* buf_dev, int stamps_per_cta);
B2D_API b2d_status b2d_debug_tune(b2d_ws* ws, int knob, int64_t value);

/*
 * Test hook (no reference counterpart): one tensor-core projection
 * Y[n][m] = sum_k X[n][k] W[m][k] (bf16 inputs, f32 accumulation) with the
 * batched path's epilogue `epi`: 0 = store f32 to y, 1 = y = resid + result,
 * 2 = SwiGLU of row pairs (2j gate, 2j+1 up) stored as bf16 column j of ybf.
 * Bits 8.. of `epi` force the K split (1..8 cluster CTAs; 0 = the split the
 * decode step would pick).  M % 128 == 0, K % 64 == 0.  Synchronises `stream`.
 */
B2D_API b2d_status b2d_test_gemm(const void* w_dev, int M, int K, const void* x_dev, int N, int epi,
                                 float* y_dev, const float* resid_dev, void* ybf_dev, int ldy, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* B2D_H_ */
