/* nitro_engine.h — C ABI of the B200 inference engine for NitroRAG's Q8_0 decoder.
 *
 * The engine replaces the reference's CPU engine surface (nvivek17/NitroRAG):
 * the model loader, the per-iteration forward step, the 16-token paged KV block
 * allocator with its block tables, and the FNV-1a prefix cache.  Each entry point
 * names the reference routine it stands in for (file:line within that project).
 *
 * Conventions
 *   - Every call returns an int status: NR_OK (0) or a negative NR_ERR_* code.  No
 *     call exits the process (the reference calls exit(1) on pool exhaustion,
 *     src/pagedMemory.hpp:117,212, and on a missing model file, src/model_q8.cpp:735).
 *   - Pointers are host pointers unless a parameter says "device".
 *   - One engine per GPU, driven from one host thread at a time.  All GPU work of an
 *     engine runs on the engine's own CUDA stream (nr_engine_stream); calls return
 *     after that work has finished unless stated otherwise.
 *   - Logits buffers are owned by the caller (the reference returned a borrowed
 *     pointer into RunState, src/model_q8.cpp:556,693).
 */
#ifndef NITRO_ENGINE_H
#define NITRO_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status codes */
#define NR_OK                 0
#define NR_ERR_INVALID       -1   /* bad argument (null pointer, size out of range)        */
#define NR_ERR_IO            -2   /* model file missing / unreadable                        */
#define NR_ERR_FORMAT        -3   /* model file shorter than its header implies, bad dims   */
#define NR_ERR_CUDA          -4   /* a CUDA call failed                                      */
#define NR_ERR_NO_BLOCKS     -5   /* KV pool exhausted after eviction (reference: exit(1))  */
#define NR_ERR_NO_DEVICE     -6   /* GPU work requested from a host-only engine            */
#define NR_ERR_UNKNOWN_SEQ   -7   /* sequence / request handle not found                    */
#define NR_ERR_CAPACITY      -8   /* batch or chunk larger than the engine was sized for    */
#define NR_ERR_TIMEOUT       -9   /* a bounded device-side wait gave up                     */

/* Q8 projection arithmetic.  The reference's batched Q8 matmul (src/model_q8.cpp:382-420)
 * overwrites its output per 32-wide K-block (:416) and so returns the LAST block's dot
 * product only; its single-token matmul (:92-125) sums every block. */
#define NR_Q8_FIXED     0   /* sum all blocks (the reference's matmul definition, default) */
#define NR_Q8_FAITHFUL  1   /* last block only, as the shipped batched path computes     */

/* Element type of the K/V pages.  The reference keeps them fp32 (src/pagedMemory.hpp:90-94,
 * src/model_q8.cpp:616-623), which NR_KV_F32 reproduces.  NR_KV_BF16 stores each K/V value
 * rounded to bf16 (half the page bytes, so half the bytes decode attention reads); the
 * attention still computes in fp32.  It changes the arithmetic (values carry 8 significant
 * bits), so it is never the default and never used for parity with the reference. */
#define NR_KV_F32   0
#define NR_KV_BF16  1

#define NR_SCHED_REFERENCE   0  /* Continuous_Scheduler::step, src/pagedMemory.hpp:317-398 */
/* Same release and decode rules; admission goes on past the FIFO head while token budget
 * is left (a request whose prompt completes makes room for the next), each request only if
 * every page it can take until it finishes (its prompt and max_new_tokens - 1 generated
 * tokens, at most seq_len tokens) fits in the free and reclaimable (cached, unreferenced)
 * pages left after what the running and earlier admitted requests can still take (or
 * nothing else runs), so a packed run does not exhaust the pool while decoding.  All
 * chunks of a step run in one forward pass.  No reference counterpart: the reference
 * admits one chunk per step. */
#define NR_SCHED_PACKED      1

typedef struct nr_config {
    int32_t total_blocks;          /* KV pool pages (reference TOTAL_BLOCKS, Server_Inference.cpp:85) */
    int32_t max_tokens_per_batch;  /* scheduler token budget, default 256 (pagedMemory.hpp:307)   */
    int32_t max_new_tokens;        /* finish after this many generated tokens, default 20 (:393)  */
    int32_t block_size;            /* must be 16 (pagedMemory.hpp:9)                               */
    int32_t sched_mode;            /* NR_SCHED_*                                                  */
    int32_t q8_mode;               /* NR_Q8_*                                                     */
    int32_t max_batch;             /* decode rows per forward call (scratch sizing), default 256, <= 1024 */
    int32_t max_prefill_tokens;    /* tokens per prefill call (scratch sizing), default 1024     */
    int32_t device;                /* CUDA device ordinal; -1 = host-only (metadata, no GPU)      */
    int32_t kv_dtype;              /* NR_KV_*: element type of the K/V pages, default fp32        */
    int32_t reserved[6];
} nr_config;

typedef struct nr_engine nr_engine;

/* Fill *cfg with the reference defaults. */
void nr_config_default(nr_config* cfg);

/* ------------------------------------------------------------------ lifecycle */
/* Load a model in the reference file format (7 x int32 header dim, hidden_dim, n_layers,
 * n_heads, n_kv_heads, vocab_size, seq_len; then fp32 embedding, fp32 rms_att, Q8_0 wq wk
 * wv wo, fp32 rms_ffn, Q8_0 w1 w2 w3, fp32 rms_final, fp32 freq_cis_real/imag), upload it
 * and create the KV pool.  Replaces the mmap loader of src/Server_Inference.cpp:41-69 and
 * the pool construction at :85-87 (KVBlock_Manager, PrefixCacheManager).
 * For a host-only engine (cfg->device == -1) only the header is used. */
int nr_engine_create(const nr_config* cfg, const char* weight_path, nr_engine** out);
/* Same, from a model image already in host memory (size bytes). */
int nr_engine_create_from_memory(const nr_config* cfg, const void* bytes, size_t size, nr_engine** out);
/* Host-only engine from a model shape alone (allocator / scheduler without a GPU). */
int nr_engine_create_host_only(const nr_config* cfg, const int32_t shape7[7], nr_engine** out);
int nr_engine_destroy(nr_engine* e);

/* shape7 = dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len */
int nr_model_shape(const nr_engine* e, int32_t shape7[7]);
/* The engine's cudaStream_t (as void*), or NULL for a host-only engine. */
void* nr_engine_stream(const nr_engine* e);
/* Last error message of this engine (static storage until the next call). */
const char* nr_last_error(const nr_engine* e);

/* ------------------------------------------------------------------ request level
 * Continuous_Scheduler::{add_request, has_active_requests, step},
 * src/pagedMemory.hpp:310-398. */
int nr_add_request(nr_engine* e, int32_t req_id, const int32_t* prompt, int32_t n);
/* 1 while any request is waiting or running, else 0 (negative on error). */
int nr_has_active(nr_engine* e);

typedef struct nr_step_out {
    /* filled by the engine */
    int32_t n_released;        /* finished requests released at the start of the step      */
    int32_t prefill_req_id;    /* request whose prompt chunk ran this step, -1 if none     */
    int32_t prefill_tokens;    /* tokens in that chunk                                     */
    int32_t prefill_hits;      /* prefix-cache pages mapped for that request this step     */
    int32_t n_decode;          /* rows in this step's decode batch                          */
    int32_t n_emitted;         /* (req_id, token) pairs written below                       */
    /* set by the caller */
    int32_t emitted_cap;       /* capacity of the arrays below                              */
    int32_t* emitted_req_ids;  /* [emitted_cap] request id per emitted token (prefill first, then decode rows) */
    int32_t* emitted_tokens;   /* [emitted_cap] greedy token ids (argmax, src/model_q8.cpp:559) */
    float*   emitted_logits;   /* [emitted_cap * vocab] or NULL: logits row per emitted token */
    /* filled by the engine */
    int32_t n_prefill;         /* prompt chunks run this step (reference mode: 0 or 1); prefill_req_id
                                  is the first one's request, prefill_tokens and prefill_hits the totals */
} nr_step_out;

/* One scheduler iteration: release finished requests, gather the decode batch, admit at
 * most one waiting request (prefix-cache scan then one prompt chunk within the token
 * budget; NR_SCHED_PACKED: several), run the prefill chunk(s) and the decode batch on the
 * GPU, sample greedily. */
int nr_step(nr_engine* e, nr_step_out* out);

/* The same iteration split in two for a host-only engine or an external executor:
 * nr_step_plan does everything up to the forward passes (including every block
 * allocation the forwards would make, in the reference's order); nr_step_commit records
 * the sampled tokens (one per chunk that completes its prompt, in chunk order, then one
 * per decode row). */
typedef struct nr_plan {
    int32_t n_released;
    int32_t prefill_req_id;    /* -1 if none */
    int32_t prefill_start;     /* position of the first chunk token */
    int32_t prefill_tokens;
    int32_t prefill_done;      /* 1 if the chunk completes the prompt (a token is sampled) */
    int32_t prefill_hits;
    int32_t n_decode;
    int32_t decode_cap;        /* caller: capacity of decode_req_ids */
    int32_t* decode_req_ids;   /* caller-owned [decode_cap] */
    /* every prompt chunk of the step (the prefill_* fields above describe the first): */
    int32_t n_prefill;
    int32_t prefill_cap;       /* caller: capacity of the four arrays below (each may be NULL) */
    int32_t* prefill_req_ids;
    int32_t* prefill_starts;
    int32_t* prefill_lens;
    int32_t* prefill_dones;
} nr_plan;
int nr_step_plan(nr_engine* e, nr_plan* plan);
int nr_step_commit(nr_engine* e, const nr_plan* plan, const int32_t* tokens, int32_t n_tokens);

/* Generated tokens of a request so far (n written to *n, at most cap into out). */
int nr_request_tokens(nr_engine* e, int32_t req_id, int32_t* out, int32_t cap, int32_t* n);
/* flags4 = prefill_idx, is_prefill_done, is_finished, next_token_to_process */
int nr_request_state(nr_engine* e, int32_t req_id, int32_t flags4[4]);
/* Block table of a request's sequence. */
int nr_request_block_table(nr_engine* e, int32_t req_id, int32_t* out, int32_t cap, int32_t* n);
/* Request ids of the running batch in order (the decode-row order). */
int nr_running_batch(nr_engine* e, int32_t* out, int32_t cap, int32_t* n);

/* ------------------------------------------------------------------ sequence level
 * Sequence (src/pagedMemory.hpp:233-285) handles for callers that drive the forward
 * passes themselves, like the reference's bench main (src/model_q8.cpp:790-939). */
int nr_seq_create(nr_engine* e, int32_t seq_id, int32_t* handle);
/* Sequence::allocate_next_token without a forward pass (src/pagedMemory.hpp:245-264). */
int nr_seq_append(nr_engine* e, int32_t handle, int32_t token);
int nr_seq_flush_cache(nr_engine* e, int32_t handle);     /* :265-273 */
int nr_seq_release(nr_engine* e, int32_t handle);         /* :274-283 */
int nr_seq_destroy(nr_engine* e, int32_t handle);         /* drop the handle (call release first) */
int nr_seq_block_table(nr_engine* e, int32_t handle, int32_t* out, int32_t cap, int32_t* n);
/* info3 = logical_token_count, token_buffer size, block_table size */
int nr_seq_info(nr_engine* e, int32_t handle, int32_t info3[3], uint64_t* current_hash);

/* forward_prefill_chunk (src/model_q8.cpp:424-557): allocates the T tokens into the
 * sequence, runs the model over them and writes the last token's logits (vocab floats)
 * to logits_out if it is not NULL; *argmax_out (if not NULL) receives argmax(logits). */
int nr_forward_prefill(nr_engine* e, int32_t handle, const int32_t* tokens, int32_t T,
                       int32_t start_pos, float* logits_out, int32_t* argmax_out);
/* forward_decode_batch (src/model_q8.cpp:571-694): allocates one token per row (in row
 * order), runs the model and writes B x vocab logits and/or B argmax ids. */
int nr_forward_decode(nr_engine* e, int32_t B, const int32_t* tokens, const int32_t* positions,
                      const int32_t* handles, float* logits_out, int32_t* argmax_out);
/* forward_paged (src/model_q8.cpp:244-368): single-token decode that always sums every
 * Q8 block (the reference's correct matmul), whatever q8_mode says. */
int nr_forward_paged(nr_engine* e, int32_t handle, int32_t token, int32_t pos,
                     float* logits_out, int32_t* argmax_out);
/* ingest_prompt (src/model_q8.cpp:695-724): prefix-cache scan over full 16-token chunks,
 * then one prefill over the rest.  *n_tokens = logical token count afterwards;
 * *computed = tokens that ran through the model (0 on a full hit, logits untouched). */
int nr_ingest_prompt(nr_engine* e, int32_t handle, const int32_t* prompt, int32_t n,
                     int32_t enable_prefix_caching, float* logits_out, int32_t* n_tokens,
                     int32_t* computed);

/* ------------------------------------------------------------------ pool introspection */
int nr_pool_free_count(nr_engine* e);                                      /* KVBlock_Manager::get_free_count, pagedMemory.hpp:134 */
int nr_pool_free_list(nr_engine* e, int32_t* out, int32_t cap, int32_t* n); /* free_list order, bottom to top */
/* state4 = num_tokens, ref_count, parent_id, child_count (KVBlock, pagedMemory.hpp:28-37) */
int nr_pool_block_state(nr_engine* e, int32_t block, int32_t state4[4]);
int nr_cache_lookup(nr_engine* e, uint64_t hash, int32_t* block);          /* check_cache, pagedMemory.hpp:187; -1 if absent */
int nr_cache_size(nr_engine* e);                                           /* entries in the hash -> block map */
int nr_cache_is_cached(nr_engine* e, int32_t block);                       /* is_cached, pagedMemory.hpp:168 */
int nr_cache_lru(nr_engine* e, int32_t* out, int32_t cap, int32_t* n);     /* evictable leaves, front to back */
int nr_cache_entries(nr_engine* e, uint64_t* hashes, int32_t* blocks, int32_t cap, int32_t* n);
/* Copy one page of the device K/V pools to host, converted to the reference's page
 * layout [layer][16][kv_dim] (src/pagedMemory.hpp:90) and to fp32. */
int nr_pool_read_page(nr_engine* e, int32_t block, float* k_out, float* v_out);

/* hash_block_state, src/pagedMemory.hpp:14-24 (FNV-1a 64 over 4 LE bytes per token). */
uint64_t nr_hash_block_state(uint64_t parent_hash, const int32_t* tokens, int32_t n);
/* argmax with the reference's semantics (src/model_q8.cpp:559-569). */
int32_t nr_argmax(const float* x, int32_t n);

/* Per-kernel-class profiling: when enabled, every launch is bracketed by CUDA events on the
 * engine stream and the elapsed times are accumulated per class.  Classes, in order:
 * 0 embed, 1 qkv, 2 attention, 3 wo, 4 w13, 5 w2, 6 logits, 7 argmax, 8 the merge of
 * split decode attention.  Enabling resets the accumulators; nr_engine_kernel_times
 * synchronises and reports ms and launch counts. */
#define NR_KERNEL_CLASSES 9
int nr_engine_set_profiling(nr_engine* e, int32_t enable);
int nr_engine_kernel_times(nr_engine* e, double ms[NR_KERNEL_CLASSES], int64_t launches[NR_KERNEL_CLASSES]);

/* Enqueue the kernels of the engine's last decode step n more times on its stream, from
 * the step descriptor still resident in HBM (same tokens, positions and pages; the K/V
 * append rewrites the same rows; logits written if that step wrote them), without host
 * copies or synchronisation.  For timing the device-resident decode step. */
int nr_replay_decode(nr_engine* e, int32_t n);
/* Enqueue only the paged decode attention launches of the engine's last decode step n more
 * times (every layer in order; with_merge != 0 adds the merge of split contexts after each),
 * back to back on its stream, without host copies or synchronisation.  The attention output
 * buffer is rewritten with the values the step computed.  For timing the attention kernel
 * at the step's shapes without the projections and per-launch events between launches. */
int nr_replay_decode_attention(nr_engine* e, int32_t n, int32_t with_merge);
/* Outputs of the most recent decode step or replay: *B_out rows; argmax_out (if not NULL,
 * [B]) the greedy ids, logits_out (if not NULL, [B x vocab]) the logits, which only a step
 * that computed them has (NR_ERR_INVALID otherwise).  Synchronises the engine stream. */
int nr_decode_last_outputs(nr_engine* e, int32_t* argmax_out, float* logits_out, int32_t* B_out);

typedef struct nr_stats {
    int64_t steps, prefill_tokens, decode_tokens, cache_hit_pages, evictions, kernel_launches;
} nr_stats;
int nr_engine_stats(nr_engine* e, nr_stats* out);

/* ------------------------------------------------------------------ kernel-level entry points
 * Device pointers, enqueued on `stream` (a cudaStream_t; NULL = legacy default stream),
 * asynchronous: the call returns after the launch.  Page layout of the device pools is
 * [page][layer][kv_head][16][head_dim] fp32.  B <= 1024. */

/* Decode paged attention for one layer (the per-(b,h) loop of src/model_q8.cpp:625-662 with
 * softmax :142-159).  q, out: [B][n_heads*head_dim]; kpool/vpool as above with n_layers
 * layers per page; block_tables: [B][max_pages] int32; ctx_lens[B] = pos+1 tokens to read,
 * each in [1, max_pages * 16] (the tokens the block table row can address).  A length
 * outside that range sets *error_flag to 2 and is clamped into [0, max_pages * 16] (a row
 * left with no tokens gets a zero output); a bounded wait that gives up sets it to 1.
 * workspace: device scratch of nr_paged_attention_workspace_size() bytes whose counter
 * region must be zero before the first call (each call leaves it zero again). */
size_t nr_paged_attention_workspace_size(int32_t B, int32_t n_heads, int32_t head_dim, int32_t max_pages);
int nr_paged_attention_decode(const float* q, const float* kpool, const float* vpool,
                              const int32_t* block_tables, int32_t max_pages, const int32_t* ctx_lens,
                              int32_t B, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                              int32_t n_layers, int32_t layer, float* out, void* workspace,
                              int32_t* error_flag, void* stream);

/* nr_paged_attention_decode without a workspace argument, for callers that may not
 * allocate device memory while stepping (their pool already holds all of HBM, or
 * cudaMalloc's device-wide synchronisation would stall their other streams).  No
 * counterpart in the reference.  The scratch is one fixed array of
 * NR_ATTN_STATIC_SCRATCH_BYTES in the library's device image, shared by every call on a
 * device: calls needing nr_paged_attention_workspace_size() above that return
 * NR_ERR_CAPACITY; the call clears the counters it needs, and two calls that overlap on
 * the device race on the array.  Every call resolves the array's address; the first call
 * on each device also sets kernel attributes, so make it before any stream capture, and
 * do not use the library across a cudaDeviceReset (those attributes are set once per
 * device for the life of the process).  Context lengths and error_flag as above. */
#define NR_ATTN_STATIC_SCRATCH_BYTES ((size_t)8 << 20)
int nr_paged_attention_decode_static(const float* q, const float* kpool, const float* vpool,
                                     const int32_t* block_tables, int32_t max_pages, const int32_t* ctx_lens,
                                     int32_t B, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                     int32_t n_layers, int32_t layer, float* out, int32_t* error_flag,
                                     void* stream);

/* Q8_0 matrix product out[m][n] = sum_k x[m][k] * q[n][k] * scale[n][k/32] (src/model_q8.cpp
 * :92-125 / :382-420).  q: device int8 [N][K]; scales: device fp32 [N][K/32]; x: [M][K];
 * out: [M][N].  q8_mode as NR_Q8_*.  M <= 8 runs on CUDA cores; wider M on the tensor
 * cores (K a multiple of 64), splitting K over the CTAs of a thread-block cluster when
 * the weight tiles alone cannot fill the GPU.  N must be even. */
int nr_q8_matmul(const float* x, const int8_t* q, const float* scales, float* out,
                 int32_t M, int32_t N, int32_t K, int32_t q8_mode, void* stream);

/* ------------------------------------------------------------------ Q8_0 quantizer
 * scripts/quantize.py (quantize_q8, :7-23) byte for byte: per 32 consecutive weights (the
 * last block of a tensor may be shorter) scale = max|w| / 127 in fp32 (1e-9 for an
 * all-zero block), q = round-half-to-even(w / scale) clamped to [-128, 127]; each block
 * is written as its scale (4 bytes, little-endian fp32) followed by its q bytes.  Weights
 * must be finite (the script raises on NaN). */
size_t nr_q8_quantized_size(int64_t n);
/* Device buffers: w and out 16-byte aligned, out of nr_q8_quantized_size(n) bytes;
 * enqueued on `stream` (a cudaStream_t; NULL = legacy default stream). */
int nr_quantize_q8_device(const float* w, int64_t n, uint8_t* out, void* stream);
/* Host buffers, on GPU `device`: streamed in 16 M-weight pieces through two pinned and
 * two device slots (made on the first call on a device, ~164 MB each side, and kept), the
 * copies of one piece overlapping the kernel of the other; returns when done. */
int nr_quantize_q8(const float* w, int64_t n, uint8_t* out, int32_t device);
/* The script's driver (quantize.py:27-60): read a llama2.c-format fp32 checkpoint, write
 * the Q8_0 model file (header and fp32 tensors copied, wq wk wv wo w1 w2 w3 quantized,
 * each as one flat array), on GPU `device`. */
int nr_quantize_model_file(const char* in_path, const char* out_path, int32_t device);

#ifdef __cplusplus
}
#endif
#endif /* NITRO_ENGINE_H */
