/* dz_attn.h -- C ABI of the B200-native hybrid-attention core (libdzattn.so).
 *
 * This is the drop-in boundary for Daiza's per-layer attention / Gated DeltaNet
 * core: everything after the Q/K/V (or qkv/alpha/beta/z) projection GEMV and
 * before the output projection.  Citations are paths inside guang384/Daiza.
 *
 * Conventions
 *  - Every function returns dz_status; DZ_OK == 0.  dz_last_error(ctx) gives a
 *    human-readable message for the last failure on that context.
 *  - Compute entry points take DEVICE pointers for tensors and a cudaStream_t
 *    passed as void*; they are stream-ordered and never synchronise.  Sequence
 *    ids are HOST int32 arrays: cache lengths and conv-ring heads are kept on
 *    the host (as KvCache::len and SsmState::conv_head are host fields in the
 *    reference), so the library sizes every launch without a device round
 *    trip.  The *_host variants take HOST tensors, stage them through the
 *    context and block until the output is back.
 *  - A context is used by one host thread at a time (the reference's model is
 *    a single owner thread calling forward; model/block.rs:53-81).
 *  - Shapes are the Bonsai-27B ones (Daiza-engine/src/model/config.rs:47-74):
 *    24 q heads / 4 kv heads / head_dim 256 / rope_dim 64 for full attention;
 *    16 k heads / 48 v heads / d 128 / conv 4 for Gated DeltaNet.  A context
 *    may own a contiguous slice of the heads (head sharding across GPUs).
 */
#ifndef DZ_ATTN_H
#define DZ_ATTN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    DZ_OK = 0,
    DZ_EINVAL = 1,    /* bad argument / shape / layer kind */
    DZ_ENOMEM = 2,    /* device or host allocation failed */
    DZ_ECUDA = 3,     /* a CUDA runtime call failed */
    DZ_ENCCL = 4,     /* reserved for collective failures */
    DZ_ETIMEOUT = 5,  /* a bounded wait ran out */
    DZ_ESTATE = 6,    /* call order violated (e.g. no cache yet, cache full) */
    DZ_EIO = 7        /* session file could not be written, read or parsed */
} dz_status;

typedef struct dz_ctx dz_ctx;

/* Model constants; mirrors Config (Daiza-engine/src/model/config.rs:5-45,47-74)
 * plus the head slice this context owns. */
typedef struct dz_config {
    int32_t n_layers;                 /* block_count */
    int32_t full_attention_interval;  /* layer i is GQA iff i % interval == interval-1 (config.rs:161-166) */
    int32_t head_count;               /* 24 */
    int32_t head_count_kv;            /* 4 */
    int32_t head_dim;                 /* 256 */
    int32_t rope_dim;                 /* 64 */
    float   rope_freq_base;           /* 1e7 */
    float   rms_eps;                  /* 1e-6 */
    int32_t ssm_conv_kernel;          /* 4 */
    int32_t ssm_state_size;           /* 128 */
    int32_t ssm_group_count;          /* 16 k heads */
    int32_t ssm_time_step_rank;       /* 48 v heads */
    int32_t ssm_inner_size;           /* 6144 */
    /* head slice owned by this context (head sharding); defaults: everything */
    int32_t kv_head_begin, kv_head_count;   /* GQA kv heads [begin, begin+count) */
    int32_t v_head_begin, v_head_count;     /* GDN v heads  [begin, begin+count) */
    /* GQA prefill computes only the 128-token query tiles t with
     * t % qtile_split_count == qtile_split_index (default 0 of 1 = all); the
     * rows of other tiles are left untouched.  Lets two contexts share one kv
     * head (8-way head sharding of 4 kv heads). */
    int32_t qtile_split_index, qtile_split_count;
} dz_config;

/* Fills the Bonsai-27B defaults (Config::default, config.rs:47-74). */
dz_status dz_config_default(dz_config* cfg);

/* Context on one CUDA device.  Replaces the ModelState owner
 * (Daiza-engine/src/model/forward.rs:32-77) for the attention/SSM caches. */
dz_status dz_ctx_create(int device, const dz_config* cfg, dz_ctx** out);
dz_status dz_ctx_destroy(dz_ctx* ctx);
const char* dz_last_error(const dz_ctx* ctx);
/* 1 if layer is full attention, 0 if Gated DeltaNet (config.rs:161-166). */
int dz_layer_is_attention(const dz_ctx* ctx, int layer);

/* ---- layer parameters (host f32 pointers, copied to HBM once) ----------- */
/* attn_q_norm, attn_k_norm [256]  (FullAttentionBlockWeights, weights.rs:1248-1259) */
dz_status dz_layer_set_attn_params(dz_ctx* ctx, int layer, const float* q_norm, const float* k_norm);
/* ssm_conv1d transposed [4][10240] (weights.rs:1339-1356), ssm_a [48] (= -exp(A_log)),
 * ssm_dt_bias [48], ssm_norm [128]  (SsmBlockWeights, weights.rs:1229-1246) */
dz_status dz_layer_set_ssm_params(dz_ctx* ctx, int layer, const float* conv1d_t, const float* ssm_a,
                                  const float* dt_bias, const float* ssm_norm);

/* ---- caches ------------------------------------------------------------- */
/* Allocates, for n_seqs sequence slots, a KV cache per full-attention layer
 * with capacity max_len[s] tokens (KvCache::new, cache/kv_cache.rs:34-40) and
 * an SsmState per Gated DeltaNet layer, zero state, zero conv history, head 0
 * (SsmState::new, cache/ssm_state.rs:24-32).  Also uploads the RoPE table for
 * positions [0, max(max_len)) computed with the reference formula
 * (math/rope.rs:27-38,82-101).  Replaces any previous cache set. */
dz_status dz_cache_create(dz_ctx* ctx, int n_seqs, const int64_t* max_len);
/* KvCache::len (kv_cache.rs:23) */
dz_status dz_kv_len(const dz_ctx* ctx, int layer, int seq, int64_t* out_len);
/* KvCache::truncate (kv_cache.rs:119-129): no-op if new_len >= len. */
dz_status dz_kv_truncate(dz_ctx* ctx, int layer, int seq, int64_t new_len);
/* KvCache::reset + SsmState::reset for every layer of one sequence
 * (kv_cache.rs:109-115, ssm_state.rs:34-39). */
dz_status dz_cache_reset(dz_ctx* ctx, int seq);
/* Export K and V as flat host [len][kv_head_count][256] f32, the DZSS session
 * layout (Daiza-runtime/src/session_persist.rs:106-118).  Bit-exact placement. */
dz_status dz_kv_export(dz_ctx* ctx, int layer, int seq, float* k_flat, float* v_flat);
/* KvCache::from_raw (kv_cache.rs:46-67): flat [len][kv_head_count][256].
 * Export/import buffers may be host or device pointers (unified addressing). */
dz_status dz_kv_import(dz_ctx* ctx, int layer, int seq, const float* k_flat, const float* v_flat, int64_t len);
/* SsmState fields (ssm_state.rs:9-21): state [v_head_count][128][128],
 * conv_history [4][10240] (only the channels this context uses are kept on
 * device; the others export as 0), conv_head. Host pointers. */
dz_status dz_ssm_export(dz_ctx* ctx, int layer, int seq, float* state, float* conv_history, int32_t* conv_head);
dz_status dz_ssm_import(dz_ctx* ctx, int layer, int seq, const float* state, const float* conv_history,
                        int32_t conv_head);
/* Synthetic-workload helper (benchmarks, tests): sets the first len rows of K
 * and V of one (layer, sequence) to a repeated byte pattern and sets the
 * cache length to len, without a host round trip. */
dz_status dz_kv_fill_pattern(dz_ctx* ctx, int layer, int seq, int64_t len, int byte_value);
/* The device RoPE table rows [pos0, pos0+n): cos[64] | sin[64] per row (host out). */
dz_status dz_rope_table(dz_ctx* ctx, int64_t pos0, int64_t n, float* out);

/* ---- compute: decode (one new token per sequence) ----------------------- */
/* Gated GQA core of attention_forward_into (model/attention.rs:90-203):
 * deinterleave [Q_h|gate_h], QK-RMSNorm, partial RoPE at pos = len, q *= 1/16,
 * KV append at slot len, online-softmax attention over len+1 positions,
 * * sigmoid(gate).  B sequences; seq_ids (host int32 [B], distinct) name the slots.
 *   q_gate [B][6*kvc][512]  (the [Q_h|gate_h] rows of this context's q heads)
 *   k, v   [B][kvc][256]     out [B][6*kvc][256]      (kvc = kv_head_count)  */
dz_status dz_gqa_decode(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* q_gate,
                        const float* k, const float* v, float* out, void* stream);
/* dz_gqa_decode with explicit RoPE positions: pos (host int32 [B]) is the position
 * of each sequence's new token, as ModelState::pos feeds rope_cos_sin_mrope_text_into
 * in the reference (model/forward.rs:230-238); the KV slot is still the cache
 * length.  pos[b] must lie inside the RoPE table (dz_cache_create's largest
 * capacity).  dz_gqa_decode is this call with pos = the cache lengths. */
dz_status dz_gqa_decode_at(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const int32_t* pos,
                           const float* q_gate, const float* k, const float* v, float* out, void* stream);
/* Gated DeltaNet core of ssm_forward_into (model/ssm.rs:466-611): ring conv1d
 * + SiLU, L2-norm q/k, q *= 1/sqrt(128), gates, gated delta rule on the
 * [v][k] state, gated RMSNorm output.
 *   qkv [B][10240] (full row; the context reads the channels it needs),
 *   alpha, beta [B][48], z [B][48*128], y [B][v_head_count*128]          */
dz_status dz_gdn_decode(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* qkv,
                        const float* alpha, const float* beta, const float* z, float* y, void* stream);

/* ---- compute: prefill (T tokens of one sequence) ------------------------ */
/* Parallel GQA prefill (model/forward.rs:599-721), positions len..len+T-1.
 * q_gate/k/v are bf16 (uint16 bit patterns) rows as above; out f32 [T][6*kvc][256].
 * Attention products run on the tensor cores in bf16 with f32 accumulation. */
dz_status dz_gqa_prefill_bf16(dz_ctx* ctx, int layer, int seq, int64_t T, const uint16_t* q_gate,
                              const uint16_t* k, const uint16_t* v, float* out, void* stream);
/* Same with f32 inputs (converted on device). */
dz_status dz_gqa_prefill(dz_ctx* ctx, int layer, int seq, int64_t T, const float* q_gate, const float* k,
                         const float* v, float* out, void* stream);
/* The two prefills with an explicit RoPE start: token t is rotated at position
 * start_pos + t (model/forward.rs:550-557, pos = start_pos + t) while its KV slot
 * is len + t.  The plain entry points use start_pos = the cache length. */
dz_status dz_gqa_prefill_bf16_at(dz_ctx* ctx, int layer, int seq, int64_t start_pos, int64_t T,
                                 const uint16_t* q_gate, const uint16_t* k, const uint16_t* v, float* out,
                                 void* stream);
dz_status dz_gqa_prefill_at(dz_ctx* ctx, int layer, int seq, int64_t start_pos, int64_t T, const float* q_gate,
                            const float* k, const float* v, float* out, void* stream);
/* Chunked (C=64) Gated DeltaNet prefill equal to the token-recurrent reference
 * (model/forward.rs:897-1059).  qkv [T][10240], alpha/beta [T][48], z [T][6144],
 * y [T][v_head_count*128]. */
dz_status dz_gdn_prefill(dz_ctx* ctx, int layer, int seq, int64_t T, const float* qkv, const float* alpha,
                         const float* beta, const float* z, float* y, void* stream);

/* ---- Q1_0 projection GEMV ------------------------------------------------- */
/* The projections that feed the cores: Q1_0Matrix::matvec_multi_into_slice
 * (Daiza-engine/src/model/weights.rs:831; row kernel tensor/quant.rs:267-328),
 * for T <= 8 tokens (the multi-token verify path) and up to 8 matrices that
 * share the input, e.g. attn_q / attn_k / attn_v (model/attention.rs:80-87) or
 * attn_qkv / ssm_alpha / ssm_beta / attn_gate (model/ssm.rs:451-463).
 *   w[m]    device pointer to matrix m in the reference's Q1_0 bytes: rows[m]
 *           rows of cols/128 blocks of 18 bytes (binary16 scale, little endian,
 *           then 16 sign bytes; bit b of byte j is weight 8j+b, 1 -> +scale,
 *           0 -> -scale); 16-byte aligned
 *   x       device [T][cols] f32, 16-byte aligned
 *   y[m]    device [T][rows[m]] f32
 * cols must be a multiple of 1024 (every projection of the model is) and small
 * enough for one CTA's shared memory: 64 rows of weights plus ~3*T*cols bytes of
 * prepared input (cols 5120 or 6144: any T <= 8; cols 17408: T = 1).  The input
 * is quantised to 23-bit fixed point per 128-input group (context-owned
 * scratch, grown on first use) and the integer dots are exact: outputs agree
 * with f32 arithmetic to ~1e-6 of the output scale. */
dz_status dz_q1_gemv(dz_ctx* ctx, int n_mats, const void* const* w, const int32_t* rows, int cols, int T,
                     const float* x, float* const* y, void* stream);

/* ---- sequence snapshots (speculative rollback) --------------------------- */
/* A snapshot holds one sequence's recurrent state across every layer: for each
 * Gated DeltaNet layer the state [v heads][128][128], the conv ring [4][10240]
 * and its head; for each full-attention layer the KV length (the KV rows
 * themselves stay in the cache: restoring is KvCache::truncate back to that
 * length, kv_cache.rs:119-129).  This is the SSM state snapshot/restore that
 * lets a drafter's k tokens be verified as one batched prefill and rolled back
 * on rejection -- the step the reference leaves out and verifies token by
 * token instead (Daiza-runtime/src/engine.rs:1295-1305).
 *
 * dz_snapshot_reserve allocates n_slots slots of device memory (each holds
 * Gated-DeltaNet-layers x (v heads x 16384 + 40960) floats) and drops earlier
 * slots.  dz_snapshot_save copies the sequence's state into a slot;
 * dz_snapshot_restore copies it back and sets every KV length to the saved
 * one; a slot can be restored any number of times.  Both copies are
 * stream-ordered device-to-device copies on `stream`.  Restore fails with
 * DZ_ESTATE if the slot holds no snapshot of this sequence, or if some KV
 * length went below the saved one since the save (cache reset, truncate,
 * import or fill: the rows under the saved length may have been rewritten).
 * dz_cache_create empties every slot. */
dz_status dz_snapshot_reserve(dz_ctx* ctx, int n_slots);
dz_status dz_snapshot_save(dz_ctx* ctx, int seq, int slot, void* stream);
dz_status dz_snapshot_restore(dz_ctx* ctx, int seq, int slot, void* stream);

/* Q1_0Matrix::matvec_add_into_slice (model/weights.rs:334-...): the same GEMV
 * with y[m][t][r] += instead of =, as the output projections accumulate into
 * the residual stream (attention.rs:207 attn_output, ssm.rs:615 ssm_out). */
dz_status dz_q1_gemv_add(dz_ctx* ctx, int n_mats, const void* const* w, const int32_t* rows, int cols, int T,
                         const float* x, float* const* y, void* stream);

/* ---- block entry norm ------------------------------------------------------- */
/* math::rmsnorm_into (math/rmsnorm.rs:85-140, 180-202) per row: out[t] =
 * (x[t] * inv_rms) * w with inv_rms = 1 / sqrt(sum x[t]^2 / n + eps) -- the
 * attn_norm in front of a block's input projections (attention.rs:72,
 * ssm.rs:443) and the post_attention_norm (block.rs:101).  x, out: device
 * [T][n] f32, w: device [n] f32, all 16-byte aligned; n a multiple of 4;
 * eps = the context's rms_eps. */
dz_status dz_rmsnorm_rows(dz_ctx* ctx, int T, int n, const float* x, const float* w, float* out, void* stream);

/* ---- block tail: post-norm + SwiGLU MLP ------------------------------------ */
/* The rest of a block after the attention / Gated DeltaNet output projection
 * (model/block.rs:93-124 with mlp.rs:28-51), for T <= 8 tokens:
 *   normed = rmsnorm(h, post_norm_w, eps)                (rmsnorm_into)
 *   gate, up = W_gate normed, W_up normed                (one two-matrix GEMV)
 *   h += W_down (silu(gate) * up)                        (matvec_add_into_slice)
 * h: device [T][hidden] f32, updated in place (16-byte aligned); post_norm_w:
 * device [hidden] f32; W_gate, W_up: Q1_0 [d_ff][hidden]; W_down: Q1_0
 * [hidden][d_ff] (device, 16-byte aligned; Bonsai-27B: hidden 5120, d_ff
 * 17408).  Intermediate rows live in context-owned scratch (grown on first
 * use).  With the output projection done by dz_q1_gemv_add, a whole block runs
 * on the device between the input projections and the next block. */
dz_status dz_block_mlp(dz_ctx* ctx, int T, int hidden, int d_ff, float* h, const float* post_norm_w,
                       const void* w_gate, const void* w_up, const void* w_down, void* stream);

/* ---- DZSS session files -------------------------------------------------- */
/* Save / restore one sequence's caches in the reference's session format v1
 * (Daiza-runtime/src/session_persist.rs:1-36, save_to_disk :76-140,
 * load_from_disk :186-290): a 128-byte header ("DZSS", version 1, cfg_hash,
 * pos, n_history, n_blocks, think flag, system-prompt flag), the history
 * tokens, then per layer either the KV cache (kind 0: per_token, len, K and V
 * as f32 [len][kv head][256]) or the DeltaNet state (kind 1: state, conv
 * history, conv_head), then the optional system prompt.  The files are byte
 * compatible with the reference's, provided the model matches: cfg_hash is
 * Rust's DefaultHasher (SipHash-1-3, zero key) over the reference's ten
 * config fields, with hidden = 5120 and context_length = 262144 (Bonsai-27B).
 * Only contexts that own whole layers (no head slice) read or write sessions.
 *
 * dz_session_save writes the file; pos, the history tokens, think_enabled and
 * system_prompt (NUL-terminated, or NULL) are the session fields the library
 * does not hold.  dz_session_load checks magic, version, cfg_hash, block count,
 * layer kinds and sizes, reads every block, then imports them into `seq`
 * (KV lengths must fit the caches' capacities: DZ_ESTATE otherwise).
 * *n_history gets the file's token count (DZ_EINVAL if it exceeds
 * history_cap); *prompt_len the prompt's byte count or -1 when there is none
 * (the buffer needs prompt_len + 1 bytes).  Format and I/O errors: DZ_EIO. */
dz_status dz_session_save(dz_ctx* ctx, int seq, const char* path, int64_t pos, const uint32_t* history,
                          int64_t n_history, int think_enabled, const char* system_prompt);
dz_status dz_session_load(dz_ctx* ctx, int seq, const char* path, int64_t* pos, uint32_t* history,
                          int64_t history_cap, int64_t* n_history, int* think_enabled, char* system_prompt,
                          int64_t prompt_cap, int64_t* prompt_len);

/* ---- host-buffer convenience (end-to-end path) -------------------------- */
/* Same as dz_gqa_decode / dz_gdn_decode with HOST input/output pointers and
 * HOST seq_ids; copies in, computes, copies out on `stream`, then waits. */
dz_status dz_gqa_decode_host(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* q_gate,
                             const float* k, const float* v, float* out, void* stream);
dz_status dz_gdn_decode_host(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* qkv,
                             const float* alpha, const float* beta, const float* z, float* y, void* stream);

/* The same two calls without the final synchronisation, for overlapping one
 * call's input upload with the previous call's work: the inputs go up on a
 * context-owned copy stream into a staging buffer per entry point (the upload
 * waits until the previous call of the same entry point has finished with
 * it), `stream` waits for them, runs the layer and queues the output download.
 * The caller synchronises `stream` before reading `out`/`y` or reusing the
 * input buffers; host buffers should be pinned for the copies to overlap. */
dz_status dz_gqa_decode_host_async(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* q_gate,
                                   const float* k, const float* v, float* out, void* stream);
dz_status dz_gdn_decode_host_async(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* qkv,
                                   const float* alpha, const float* beta, const float* z, float* y, void* stream);

/* dz_gqa_decode without any device allocation, for callers that cannot call
 * cudaMalloc: engines whose device memory is owned end to end by their own
 * allocator, and decode loops that must not risk the implicit device
 * synchronisation of cudaMalloc/cudaFree.  Same arguments, semantics and cache
 * updates as dz_gqa_decode; its split-K scratch lives in one fixed device array
 * inside the library (about 13.6 MiB per GPU that loads the library, held until
 * exit).  Limits: at most 64 sequences per call (DZ_EINVAL beyond that); the
 * split-K chunk is dz_gqa_decode's, doubled until a call needs at most 2048 work
 * items -- identical results when no doubling is needed, equal to f32 rounding
 * otherwise.  All calls on a device share the array: calls that overlap on the
 * GPU race, so order them.  The first call on each device looks up the array's
 * device address (again after the device's context changes); make that first
 * call before any stream capture begins.
 * No counterpart in the reference (the reference runs on the CPU and never
 * allocates device memory). */
dz_status dz_gqa_decode_noalloc(dz_ctx* ctx, int layer, int B, const int32_t* seq_ids, const float* q_gate,
                                const float* k, const float* v, float* out, void* stream);

/* Number of kernels launched by the last compute call on this context. */
int dz_last_launch_count(const dz_ctx* ctx);
/* Synchronises the context's device and reads (then clears) the device error
 * word that kernels set when a bounded wait runs out; *code = 0 if none. */
dz_status dz_device_error(dz_ctx* ctx, int32_t* code);

#ifdef __cplusplus
}
#endif
#endif /* DZ_ATTN_H */
