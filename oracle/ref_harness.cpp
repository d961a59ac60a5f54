// Test infrastructure only (the checker, never the product): a C harness around the
// reference's own inference code, compiled from src/model_q8.cpp and src/pagedMemory.hpp
// where they lie.  The reference has no library API of its own; its bench main()
// (src/model_q8.cpp:726-946) is renamed away and the engine surface it calls is
// exposed here through extern "C" functions so that Python tests can drive it:
//
//   forward_prefill_chunk  src/model_q8.cpp:424      forward_decode_batch  :571
//   forward_paged          src/model_q8.cpp:244      argmax                :559
//   ingest_prompt          src/model_q8.cpp:695      matmul_bulk           :370, :382
//   hash_block_state       src/pagedMemory.hpp:14    KVBlock_Manager       :42-160
//   PrefixCacheManager     src/pagedMemory.hpp:64-229  Sequence            :233-285
//   Request                src/pagedMemory.hpp:287   Continuous_Scheduler  :303-398
//
// `private` is widened to `public` only so the harness can read allocator state
// (free list, cache maps, LRU order) for bit-exact comparisons; no reference logic
// is changed by it.  The weight-file walk in ref_open() restates the loader in
// src/Server_Inference.cpp:41-69 (identical to src/model_q8.cpp:734-768).
#include <iostream>
#include <vector>
#include <list>
#include <queue>
#include <unordered_map>
#include <cstdint>
#include <cstring>
#include <cmath>
#include <chrono>
#include <iomanip>
#include <memory>
#include <omp.h>
#include <fcntl.h>
#include <unistd.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <immintrin.h>

#define private public
#define main nitro_reference_bench_main
#include "model_q8.cpp"
#undef main
#undef private

namespace {

struct Harness {
    // model
    void* map = nullptr;
    size_t map_size = 0;
    std::vector<uint8_t> owned;  // used when the model comes from memory
    Config_Transformer c{};
    Transformer_Weights w{};
    RunState s{};
    int max_tokens = 0;
    bool has_model = false;
    // pool
    std::unique_ptr<KVBlock_Manager> mem;
    std::unique_ptr<PrefixCacheManager> cache;
    int total_blocks = 0;
    int n_layers = 0;
    int kv_dim = 0;
    // requests (each owns a Sequence)
    std::vector<Request*> reqs;
    // scheduler
    std::unique_ptr<Continuous_Scheduler> sched;
    std::vector<Request*> sched_reqs;
    int last_decode_B = 0;
};

Harness* H = nullptr;

void free_runstate(RunState& s) {
    free(s.x); free(s.xb); free(s.xb2); free(s.hb); free(s.hb2);
    free(s.q); free(s.k); free(s.v); free(s.logits); free(s.attn);
    s = RunState{};
}

void drop_requests() {
    for (Request* r : H->reqs) delete r;
    H->reqs.clear();
    H->sched_reqs.clear();
    H->sched.reset();
}

int setup_weights(const uint8_t* base, size_t size) {
    const int* header = (const int*)base;
    Config_Transformer& c = H->c;
    c.dim = header[0]; c.hidden_dim = header[1]; c.n_layers = header[2];
    c.n_heads = header[3]; c.n_kv_heads = header[4]; c.vocab_size = header[5]; c.seq_len = header[6];
    int head_size = c.dim / c.n_heads;
    int kv_dim = c.n_kv_heads * head_size;
    const size_t QB = 32;
    uint8_t* p = (uint8_t*)base + 28;
    Transformer_Weights& w = H->w;
    auto take = [&](size_t bytes) { uint8_t* r = p; p += bytes; return r; };
    w.token_embedding_table = (float*)take((size_t)c.vocab_size * c.dim * 4);
    w.rms_attn_weights = (float*)take((size_t)c.n_layers * c.dim * 4);
    w.wq = (BlockQ8*)take((size_t)c.n_layers * c.dim * c.dim / QB * sizeof(BlockQ8));
    w.wk = (BlockQ8*)take((size_t)c.n_layers * c.dim * kv_dim / QB * sizeof(BlockQ8));
    w.wv = (BlockQ8*)take((size_t)c.n_layers * c.dim * kv_dim / QB * sizeof(BlockQ8));
    w.wo = (BlockQ8*)take((size_t)c.n_layers * c.dim * c.dim / QB * sizeof(BlockQ8));
    w.rms_ffn_weight = (float*)take((size_t)c.n_layers * c.dim * 4);
    w.w1 = (BlockQ8*)take((size_t)c.n_layers * c.hidden_dim * c.dim / QB * sizeof(BlockQ8));
    w.w2 = (BlockQ8*)take((size_t)c.n_layers * c.dim * c.hidden_dim / QB * sizeof(BlockQ8));
    w.w3 = (BlockQ8*)take((size_t)c.n_layers * c.hidden_dim * c.dim / QB * sizeof(BlockQ8));
    w.rms_final_weight = (float*)take((size_t)c.dim * 4);
    w.freq_cis_real = (float*)take((size_t)c.seq_len * head_size / 2 * 4);
    w.freq_cis_imag = (float*)take((size_t)c.seq_len * head_size / 2 * 4);
    w.wcls = w.token_embedding_table;
    if ((size_t)(p - base) > size) return -2;
    return 0;
}

void alloc_runstate(int max_tokens) {
    Config_Transformer& c = H->c;
    int head_size = c.dim / c.n_heads;
    int kv_dim = c.n_kv_heads * head_size;
    size_t M = (size_t)max_tokens;
    RunState& s = H->s;
    s.x = (float*)calloc(M * c.dim, 4);
    s.xb = (float*)calloc(M * c.dim, 4);
    s.xb2 = (float*)calloc(M * c.dim, 4);
    s.hb = (float*)calloc(M * c.hidden_dim, 4);
    s.hb2 = (float*)calloc(M * c.hidden_dim, 4);
    s.q = (float*)calloc(M * c.dim, 4);
    s.k = (float*)calloc(M * kv_dim, 4);
    s.v = (float*)calloc(M * kv_dim, 4);
    s.logits = (float*)calloc(M * c.vocab_size, 4);
    s.attn = (float*)calloc(M * c.n_heads * c.seq_len, 4);
    H->max_tokens = max_tokens;
}

Request* req_at(int h) {
    if (!H || h < 0 || h >= (int)H->reqs.size()) return nullptr;
    return H->reqs[h];
}

}  // namespace

extern "C" {

int ref_is_fixed() {
#ifdef NITRO_REF_FIXED
    return 1;
#else
    return 0;
#endif
}

void ref_set_threads(int n) { omp_set_num_threads(n > 0 ? n : omp_get_num_procs()); }
int ref_num_procs() { return omp_get_num_procs(); }

void ref_close() {
    if (!H) return;
    drop_requests();
    H->cache.reset();
    H->mem.reset();
    free_runstate(H->s);
    if (H->map) munmap(H->map, H->map_size);
    delete H;
    H = nullptr;
}

// Create a pool without a model (allocator / prefix-cache tests).
int ref_pool_only(int total_blocks, int n_layers, int kv_dim) {
    ref_close();
    H = new Harness();
    H->total_blocks = total_blocks;
    H->n_layers = n_layers;
    H->kv_dim = kv_dim;
    H->mem.reset(new KVBlock_Manager(total_blocks, n_layers, kv_dim));
    H->cache.reset(new PrefixCacheManager(*H->mem, total_blocks));
    H->sched.reset(new Continuous_Scheduler());
    return 0;
}

// Load a model file in the reference format; allocate a RunState for `max_tokens`
// rows (the reference's MAX_BATCH) and a pool of `total_blocks` pages.
int ref_open(const char* path, int max_tokens, int total_blocks) {
    ref_close();
    H = new Harness();
    int fd = open(path, O_RDONLY);
    if (fd < 0) { delete H; H = nullptr; return -1; }
    struct stat st;
    fstat(fd, &st);
    void* data = mmap(NULL, st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (data == MAP_FAILED) { delete H; H = nullptr; return -1; }
    H->map = data;
    H->map_size = st.st_size;
    int rc = setup_weights((const uint8_t*)data, st.st_size);
    if (rc) { ref_close(); return rc; }
    H->has_model = true;
    alloc_runstate(max_tokens);
    int head_size = H->c.dim / H->c.n_heads;
    int kv_dim = H->c.n_kv_heads * head_size;
    H->total_blocks = total_blocks;
    H->n_layers = H->c.n_layers;
    H->kv_dim = kv_dim;
    H->mem.reset(new KVBlock_Manager(total_blocks, H->c.n_layers, kv_dim));
    H->cache.reset(new PrefixCacheManager(*H->mem, total_blocks));
    H->sched.reset(new Continuous_Scheduler());
    // The reference pool comes from aligned_alloc and is never zeroed; zero it so
    // unused rows read as 0 in comparisons.
    size_t floats = (size_t)total_blocks * H->c.n_layers * BLOCK_SIZE * kv_dim;
    memset(H->mem->global_k_pool, 0, floats * 4);
    memset(H->mem->global_v_pool, 0, floats * 4);
    return 0;
}

int ref_config(int* out7) {
    if (!H || !H->has_model) return -1;
    const Config_Transformer& c = H->c;
    out7[0] = c.dim; out7[1] = c.hidden_dim; out7[2] = c.n_layers; out7[3] = c.n_heads;
    out7[4] = c.n_kv_heads; out7[5] = c.vocab_size; out7[6] = c.seq_len;
    return 0;
}

// ---------------------------------------------------------------- requests / sequences
int ref_req_new(int id, const int* prompt, int n) {
    if (!H) return -1;
    std::vector<int> p(prompt, prompt + n);
    H->reqs.push_back(new Request(id, p));
    return (int)H->reqs.size() - 1;
}

int ref_seq_alloc_token(int h, int token) {
    Request* r = req_at(h);
    if (!r) return -1;
    r->seq.allocate_next_token(token, *H->mem, *H->cache);
    return 0;
}

int ref_seq_flush(int h) {
    Request* r = req_at(h);
    if (!r) return -1;
    r->seq.flush_cache(*H->cache);
    return 0;
}

int ref_seq_release(int h) {
    Request* r = req_at(h);
    if (!r) return -1;
    r->seq.release(*H->mem, *H->cache);
    return 0;
}

// out: [logical_token_count, token_buffer.size(), block_table.size()], *hash = current_hash
int ref_seq_info(int h, int* out3, uint64_t* hash) {
    Request* r = req_at(h);
    if (!r) return -1;
    out3[0] = r->seq.logical_token_count;
    out3[1] = (int)r->seq.token_buffer.size();
    out3[2] = (int)r->seq.block_table.size();
    *hash = r->seq.current_hash;
    return 0;
}

int ref_seq_block_table(int h, int* out, int cap) {
    Request* r = req_at(h);
    if (!r) return -1;
    int n = (int)r->seq.block_table.size();
    for (int i = 0; i < n && i < cap; i++) out[i] = r->seq.block_table[i];
    return n;
}

// ---------------------------------------------------------------- pool / cache state
int ref_free_count() { return H ? H->mem->get_free_count() : -1; }

int ref_free_list(int* out, int cap) {
    if (!H) return -1;
    int n = (int)H->mem->free_list.size();
    for (int i = 0; i < n && i < cap; i++) out[i] = H->mem->free_list[i];
    return n;
}

// out: [num_tokens, ref_count, parent_id, child_count]
int ref_block_state(int id, int* out4) {
    if (!H || id < 0 || id >= H->total_blocks) return -1;
    const KVBlock& b = H->mem->blocks[id];
    out4[0] = b.num_tokens; out4[1] = b.ref_count; out4[2] = b.parent_id; out4[3] = b.child_count;
    return 0;
}

int ref_cache_lookup(uint64_t hash) { return H ? H->cache->check_cache(hash) : -1; }
int ref_cache_size() { return H ? (int)H->cache->cache_map.size() : -1; }
int ref_is_cached(int id) { return H ? (int)H->cache->is_cached(id) : -1; }

// cache_map entries (hash, block) in unspecified order
int ref_cache_entries(uint64_t* hashes, int* blocks, int cap) {
    if (!H) return -1;
    int i = 0;
    for (auto& kv : H->cache->cache_map) {
        if (i < cap) { hashes[i] = kv.first; blocks[i] = kv.second; }
        i++;
    }
    return i;
}

// reverse_map entries (block, hash)
int ref_reverse_entries(int* blocks, uint64_t* hashes, int cap) {
    if (!H) return -1;
    int i = 0;
    for (auto& kv : H->cache->reverse_map) {
        if (i < cap) { blocks[i] = kv.first; hashes[i] = kv.second; }
        i++;
    }
    return i;
}

// LRU list of evictable leaves, front to back
int ref_lru(int* out, int cap) {
    if (!H) return -1;
    int i = 0;
    for (int id : H->cache->evictable_leaves) {
        if (i < cap) out[i] = id;
        i++;
    }
    return i;
}

int ref_inc_ref(int id) {
    if (!H) return -1;
    H->mem->inc_ref_count(id, *H->cache);
    return 0;
}

int ref_free_block(int id) {
    if (!H) return -1;
    H->mem->free_block(id, *H->cache);
    return 0;
}

int ref_allocate_block() {
    if (!H) return -1;
    return H->mem->allocate_block(*H->cache);
}

// Copy page `id` (layout [layer][16][kv_dim], src/pagedMemory.hpp:90) of the K and V pools.
int ref_kv_page(int id, float* k_out, float* v_out) {
    if (!H || id < 0 || id >= H->total_blocks) return -1;
    size_t floats = (size_t)H->n_layers * BLOCK_SIZE * H->kv_dim;
    KVBlock& b = H->mem->get_block(id);
    if (k_out) memcpy(k_out, b.k_ptr, floats * 4);
    if (v_out) memcpy(v_out, b.v_ptr, floats * 4);
    return 0;
}

// Fill every page of the pool with a deterministic pattern (timing runs that skip prefill).
int ref_kv_fill(float scale) {
    if (!H) return -1;
    size_t floats = (size_t)H->total_blocks * H->n_layers * BLOCK_SIZE * H->kv_dim;
    float* k = H->mem->global_k_pool;
    float* v = H->mem->global_v_pool;
    #pragma omp parallel for
    for (size_t i = 0; i < floats; i++) {
        uint32_t x = (uint32_t)(i * 2654435761u);
        k[i] = scale * ((float)(x >> 8) / 16777216.0f - 0.5f);
        v[i] = scale * ((float)((x * 747796405u) >> 8) / 16777216.0f - 0.5f);
    }
    return 0;
}

uint64_t ref_hash_block_state(uint64_t parent, const int* tokens, int n) {
    std::vector<int> t(tokens, tokens + n);
    return hash_block_state(parent, t);
}

int ref_argmax(float* x, int n) { return argmax(x, n); }

// ---------------------------------------------------------------- kernels
void ref_matmul_bulk_q8(float* out, float* x, const void* w_aos, int batch, int n, int d) {
    matmul_bulk(out, x, (BlockQ8*)w_aos, batch, n, d);
}
void ref_matmul_q8(float* out, float* x, const void* w_aos, int n, int d) {
    matmul(out, x, (BlockQ8*)w_aos, n, d);
}
void ref_matmul_bulk_f32(float* out, float* x, float* w, int batch, int n, int d) {
    matmul_bulk(out, x, w, batch, n, d);
}
void ref_rms_norm(float* out, float* x, float* weight, int size) { rms_norm(out, x, weight, size); }
void ref_softmax(float* x, int size) { softmax(x, size); }

// ---------------------------------------------------------------- forward passes
int ref_forward_prefill(int h, const int* tokens, int T, int start_pos, float* logits_out) {
    Request* r = req_at(h);
    if (!r || !H->has_model || T > H->max_tokens) return -1;
    std::vector<int> t(tokens, tokens + T);
    float* lg = forward_prefill_chunk(t, start_pos, &H->c, &H->w, &H->s, r->seq, *H->mem, *H->cache);
    if (!lg) return -2;
    if (logits_out) memcpy(logits_out, lg, (size_t)H->c.vocab_size * 4);
    return 0;
}

int ref_forward_decode(int B, const int* tokens, const int* positions, const int* handles, float* logits_out) {
    if (!H || !H->has_model || B > H->max_tokens) return -1;
    std::vector<int> t(tokens, tokens + B), p(positions, positions + B);
    std::vector<Request*> rs;
    for (int b = 0; b < B; b++) {
        Request* r = req_at(handles[b]);
        if (!r) return -1;
        rs.push_back(r);
    }
    float* lg = forward_decode_batch(t, p, rs, &H->c, &H->w, &H->s, *H->mem, *H->cache);
    if (!lg) return -2;
    if (logits_out) memcpy(logits_out, lg, (size_t)B * H->c.vocab_size * 4);
    return 0;
}

int ref_forward_paged(int h, int token, int pos, float* logits_out) {
    Request* r = req_at(h);
    if (!r || !H->has_model) return -1;
    float* lg = forward_paged(token, pos, &H->c, &H->w, &H->s, r->seq, *H->mem, *H->cache);
    if (logits_out) memcpy(logits_out, lg, (size_t)H->c.vocab_size * 4);
    return 0;
}

// ingest_prompt (src/model_q8.cpp:695); logits of the last computed token are copied
// out when a prefill ran (returns the logical token count, or <0 on error).
int ref_ingest_prompt(int h, const int* tokens, int n, int enable_cache, float* logits_out, int* computed) {
    Request* r = req_at(h);
    if (!r || !H->has_model) return -1;
    std::vector<int> t(tokens, tokens + n);
    int before = r->seq.logical_token_count;
    // the number of tokens that ingest_prompt will compute is known only afterwards:
    // clear logits so an all-hit call is recognisable
    memset(H->s.logits, 0, (size_t)H->c.vocab_size * 4);
    int cnt = ingest_prompt(t, r->seq, *H->mem, *H->cache, &H->c, &H->w, &H->s, enable_cache != 0);
    (void)before;
    if (logits_out) memcpy(logits_out, H->s.logits, (size_t)H->c.vocab_size * 4);
    if (computed) *computed = -1;
    return cnt;
}

// ---------------------------------------------------------------- scheduler
int ref_sched_reset() {
    if (!H) return -1;
    H->sched.reset(new Continuous_Scheduler());
    H->sched_reqs.clear();
    return 0;
}

int ref_sched_add(int h) {
    Request* r = req_at(h);
    if (!r || !H->sched) return -1;
    H->sched->add_request(r);
    H->sched_reqs.push_back(r);
    return 0;
}

int ref_sched_has_active() { return (H && H->sched) ? (int)H->sched->has_active_requests() : -1; }

// One Continuous_Scheduler::step.  max_new_tokens > 0 overrides the hard-coded 20-token
// finish (src/pagedMemory.hpp:393) by re-deriving is_finished after the step.
// Returns the decode batch size of this step (rows of ref_sched_decode_logits).
int ref_sched_step(int max_new_tokens) {
    if (!H || !H->sched || !H->has_model) return -1;
    // step() first releases finished requests, then decodes every remaining member of
    // the running batch (all of them have is_prefill_done set, :334-341)
    int Bdec = 0;
    for (Request* r : H->sched->running_batch)
        if (!r->is_finished && r->is_prefill_done) Bdec++;
    H->sched->step(&H->c, &H->w, &H->s, *H->mem, *H->cache);
    if (max_new_tokens > 0) {
        for (Request* r : H->sched_reqs)
            r->is_finished = (int)r->generated_tokens.size() >= max_new_tokens;
    }
    H->last_decode_B = Bdec;
    return Bdec;
}

// Logits of the last decode batch of the scheduler (rows in running-batch order).
int ref_sched_decode_logits(float* out, int rows) {
    if (!H || !H->has_model) return -1;
    memcpy(out, H->s.logits, (size_t)rows * H->c.vocab_size * 4);
    return 0;
}

// Request ids of the running batch, in order.
int ref_sched_running(int* out, int cap) {
    if (!H || !H->sched) return -1;
    int i = 0;
    for (Request* r : H->sched->running_batch) {
        if (i < cap) out[i] = r->req_id;
        i++;
    }
    return i;
}

int ref_sched_waiting() {
    if (!H || !H->sched) return -1;
    return (int)H->sched->waiting_queue.size();
}

int ref_req_generated(int h, int* out, int cap) {
    Request* r = req_at(h);
    if (!r) return -1;
    int n = (int)r->generated_tokens.size();
    for (int i = 0; i < n && i < cap; i++) out[i] = r->generated_tokens[i];
    return n;
}

// out: [prefill_idx, is_prefill_done, is_finished, next_token_to_process]
int ref_req_flags(int h, int* out4) {
    Request* r = req_at(h);
    if (!r) return -1;
    out4[0] = r->prefill_idx; out4[1] = r->is_prefill_done; out4[2] = r->is_finished;
    out4[3] = r->next_token_to_process;
    return 0;
}

}  // extern "C"
