// Host-side launchers of the engine's sm_100a kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "common.cuh"

namespace nitro {

// What a projection does with its result tile.
enum EpiKind : int {
    kEpiStore = 0,     // out[m][n] = acc
    kEpiResidual = 1,  // out[m][n] += acc                          (src/model_q8.cpp:524-528, :546-551)
    kEpiQKV = 2,       // RoPE on q,k; q -> q_out, k,v -> KV pages  (:451-484, :594-624)
    kEpiSwiGLU = 3,    // rows interleaved (w1 i, w3 i): out[m][i] = silu(acc[2i]) * acc[2i+1]  (:535-545)
    kEpiLogits = 4,    // optional store + greedy argmax keys      (:553-556, :688-693, :559-569)
};

struct Epilogue {
    int kind = kEpiStore;
    float* out = nullptr;   // STORE / RESIDUAL / SWIGLU / LOGITS (may be null for LOGITS)
    int ldo = 0;
    // QKV
    float* q_out = nullptr;  // [M][dim]
    float* kpool = nullptr;
    float* vpool = nullptr;
    PoolGeom geom{};
    int layer = 0;
    const int* tok_page = nullptr;  // [M] physical page of each row's token
    const int* tok_pos = nullptr;   // [M] position of each row's token
    const float* freq_re = nullptr; // [seq_len][head_dim/2]
    const float* freq_im = nullptr;
    int dim = 0, kv_dim = 0, head_dim = 0;
    // LOGITS
    unsigned long long* argmax_keys = nullptr;  // [M]
    // RESIDUAL (tensor-core path): per 128-feature tile, sum of squares of the updated rows,
    // ss_out[tile * ss_ld + m], consumed by the next RMSNorm (GemmArgs::ss_in)
    float* ss_out = nullptr;
    int ss_ld = 0;
};

// out = x . W^T for M token rows: x [M][K] fp32 (row stride ldx), W either Q8_0 (int8
// [N][K] + fp32 scales [N][K/32]) or fp32 [N][K].  If norm_gain is set, each x row is
// RMS-normalised with that gain first (src/model_q8.cpp:128-140).  kbegin = K-32 limits
// the contraction to the last 32-wide block (the reference's batched Q8 arithmetic).
struct GemmArgs {
    const float* x = nullptr;
    int ldx = 0;
    const float* norm_gain = nullptr;
    const int8_t* wq = nullptr;
    const float* ws = nullptr;
    const float* wf = nullptr;
    int M = 0, N = 0, K = 0;
    int kbegin = 0;
    // RMSNorm from precomputed partial sums of squares of x: ss_in[p * ss_ld + m] for
    // p < ss_parts (tensor-core path only; otherwise the rows are re-read)
    const float* ss_in = nullptr;
    int ss_parts = 0, ss_ld = 0;
    int* err = nullptr;   // device error flag for bounded waits
    // Optional: the same weights pre-split into bf16 hi/lo halves in the tensor-core
    // kernel's shared-memory tile layout (tc_tile_weights); the kernel then fetches each
    // 128-row x 64-column tile with one bulk copy instead of converting q * scale itself.
    const uint8_t* wt = nullptr;
    // Optional, for Q8 matrices without hi/lo tiles (large ones, HBM-bound): the int8 rows
    // and scales regrouped per 128-row x 64-column tile (9 KB, tc_tile_q8_raw) so the
    // kernel can stream them with bulk copies through a deep shared-memory ring.
    const uint8_t* wr = nullptr;
    // Optional scratch for the stream-K kernel (batches of 3-64 rows over hi/lo or raw
    // tiles), laid out by tc_streamk_bind: one partial tile per CTA, the launch's
    // activations as hi/lo tiles (K up to sk_max_k), and one flag per CTA, zero when no
    // launch is in flight (each launch leaves them so).
    // Optional scratch for the activations pre-split into bf16 hi/lo tiles, taken by the
    // tensor-core GEMM's 128/256-token tiles over hi/lo weight tiles: xs_cap_rows x
    // xs_cap_k x 4 bytes.
    uint8_t* xs_tiles = nullptr;
    int xs_rows = 0;  // rows of the launch's tiles (set by the launcher)
    int xs_cap_rows = 0, xs_cap_k = 0;
    float* sk_partial = nullptr;
    uint8_t* sk_xs = nullptr;
    int* sk_flags = nullptr;
    int sk_capacity = 0;
    int sk_max_k = 0;
};

// Bytes of stream-K scratch for `ctas` CTAs and K up to max_k, and the binding of one
// such (zeroed) buffer to a GemmArgs.
size_t tc_streamk_scratch_bytes(int ctas, int max_k);
void tc_streamk_bind(GemmArgs& g, void* scratch, int ctas, int max_k);
// Whether the stream-K kernel may take raw-tile launches (NITRO_STREAMK=0 turns it off).
bool tc_streamk_enabled();

// M <= 8: CUDA-core matvec; M > 8 with K % 64 == 0: tcgen05 GEMM (gemm_tc.cu); otherwise
// the CUDA-core tiled kernel.
void launch_gemm(const GemmArgs& a, const Epilogue& e, cudaStream_t s);
bool tc_gemm_supported(const GemmArgs& a);
// Whether launch_gemm takes the tensor-core path for this shape.
bool gemm_uses_tc(int M, int N, int K);
void launch_tc_gemm(const GemmArgs& a, const Epilogue& e, cudaStream_t s);
// Bytes of the tiled hi/lo copy of an [N][K] weight matrix (K % 64 == 0; rows padded to
// a multiple of 128 with zeros), and the kernel that writes it from Q8_0 (q, scales) or
// fp32 (wf) weights.
size_t tc_tiled_weight_bytes(int N, int K);
void tc_tile_weights(const int8_t* q, const float* scales, const float* wf, int N, int K, uint8_t* out, cudaStream_t s);
size_t tc_raw_q8_bytes(int N, int K);
void tc_tile_q8_raw(const int8_t* q, const float* scales, int N, int K, uint8_t* out, cudaStream_t s);

// Decode attention over paged KV for one layer (see attention.cu).
struct DecodeAttnArgs {
    const float* q = nullptr;     // [B][n_heads*head_dim]
    const float* kpool = nullptr;
    const float* vpool = nullptr;
    PoolGeom geom{};
    int layer = 0;
    const int* block_tables = nullptr;  // [B][max_pages]
    int max_pages = 0;
    const int* ctx_lens = nullptr;      // [B] tokens to attend (pos + 1)
    int B = 0, n_heads = 0;
    float* out = nullptr;               // [B][n_heads*head_dim]
    float* part_o = nullptr;            // split partials [B][n_heads][max_splits][head_dim]
    float* part_ml = nullptr;           // [B][n_heads][max_splits][2]
    int* counters = nullptr;            // [B][n_heads], zero between calls
    int* work = nullptr;                // [2] work-item and finished-warp counters, zero between calls
    int max_splits = 0;
    int chunk_pages = 0;
    int* err = nullptr;
};
int decode_attn_chunk_pages(int head_dim);
size_t decode_attn_workspace_bytes(int B, int n_heads, int head_dim, int max_pages);
// Carve part_o/part_ml/counters out of a workspace of decode_attn_workspace_bytes().
void decode_attn_bind_workspace(DecodeAttnArgs& a, void* ws, int max_pages_capacity);
void launch_decode_attention(const DecodeAttnArgs& a, int max_ctx, cudaStream_t s);
// The same in parts: the launch plan (chunk length from the longest context), the attention
// kernel, and the merge kernel that combines its splits (nothing for small batches).
DecodeAttnArgs plan_decode_attention(const DecodeAttnArgs& a, int max_ctx);
bool decode_attn_splits(const DecodeAttnArgs& a);
void launch_decode_attention_main(const DecodeAttnArgs& a, cudaStream_t s);
void launch_decode_merge(const DecodeAttnArgs& a, cudaStream_t s);

// Causal prefill attention for T consecutive tokens of one sequence, or (seg != null) for
// chunks of several sequences whose rows are concatenated in q/out (see attention.cu).
struct PrefillAttnArgs {
    const float* q = nullptr;  // [T][n_heads*head_dim]
    const float* kpool = nullptr;
    const float* vpool = nullptr;
    PoolGeom geom{};
    int layer = 0;
    const int* block_table = nullptr;  // pages of the sequence (seg: all block tables, concatenated)
    int T = 0, start_pos = 0, n_heads = 0;
    float* out = nullptr;  // [T][n_heads*head_dim]
    int* err = nullptr;
    // several sequences: seg[4*i..] = first row, rows, position of the first row, offset of
    // the sequence's block table in block_table; tiles[2*j..] = (segment, query tile),
    // ordered by decreasing work; T, start_pos unused
    const int* seg = nullptr;
    const int* tiles = nullptr;
    int n_tiles = 0;
};
void launch_prefill_attention(const PrefillAttnArgs& a, cudaStream_t s);
// Queries per prefill attention CTA (the unit of the tile table).
int prefill_attn_query_tile(int head_dim);
// The tcgen05 causal prefill attention (attention_tc.cu): head_dim 64, 128 queries per
// CTA; launch_prefill_attention takes it when enabled (NITRO_DISABLE_TC_ATTN=1 turns it off).
bool prefill_attn_tc_enabled(int head_dim);
void launch_prefill_attention_tc(const PrefillAttnArgs& a, cudaStream_t s);

// Q8_0 quantizer of scripts/quantize.py:7-23 (quantize.cu): bytes of n weights' blocks,
// the device pass (w and out 16-byte aligned), the host-buffer pass through
// pinned slots, and the script's whole-file conversion (NR_* status codes).
size_t q8_quantized_bytes(int64_t n);
void launch_quantize_q8(const float* w, int64_t n, uint8_t* out, cudaStream_t s);
int quantize_q8_host(const float* w, int64_t n, uint8_t* out);
int quantize_model_file(const char* in_path, const char* out_path);

// x[m] = emb[tokens[m]] and argmax keys reset (src/model_q8.cpp:431-435, :578-582); with
// ss != null also the per-128-feature sums of squares of each row (ss[p * ss_ld + m]).
void launch_embed(const float* emb, const int* tokens, int M, int dim, float* x,
                  unsigned long long* keys, float* ss, int ss_ld, cudaStream_t s);
// Finalise argmax keys into token ids.
void launch_argmax_finish(const unsigned long long* keys, int M, int* out, cudaStream_t s);

// Kernel launches made so far by this process (host-side count of <<<>>> calls).
int64_t kernel_launch_count();
void count_launch();

}  // namespace nitro
