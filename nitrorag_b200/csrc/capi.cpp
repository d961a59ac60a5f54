// The C ABI (include/nitro_engine.h) over nitro::Engine.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/nitro_engine.h"
#include "engine.h"

using nitro::Engine;
using nitro::Request;
using nitro::Sequence;

struct nr_engine {
    Engine* impl;
};

namespace {

thread_local std::string g_create_error;

int parse_shape(const void* bytes, size_t size, nitro::ModelShape* s) {
    if (size < 28) {
        g_create_error = "model file shorter than its 28-byte header";
        return NR_ERR_FORMAT;
    }
    int32_t h[7];
    memcpy(h, bytes, 28);
    s->dim = h[0]; s->hidden = h[1]; s->n_layers = h[2]; s->n_heads = h[3];
    s->n_kv_heads = h[4]; s->vocab = h[5]; s->seq_len = h[6];
    for (int i = 0; i < 7; i++)
        if (h[i] <= 0) return NR_ERR_FORMAT;
    if (s->dim % s->n_heads || s->n_heads % s->n_kv_heads || s->head_dim() % 2) return NR_ERR_FORMAT;
    return NR_OK;
}

// Bytes a model file of this shape must hold (header + tensors, src/Server_Inference.cpp:53-68).
size_t expected_file_size(const nitro::ModelShape& s) {
    const size_t D = s.dim, H = s.hidden, L = s.n_layers, V = s.vocab, KV = s.kv_dim(), hd = s.head_dim();
    const size_t q8 = 36;
    size_t n = 28;
    n += V * D * 4 + L * D * 4;
    n += (L * D * D + 2 * L * D * KV + L * D * D) / 32 * q8;
    n += L * D * 4;
    n += 3 * L * H * D / 32 * q8;
    n += D * 4 + 2 * (size_t)s.seq_len * hd / 2 * 4;
    return n;
}

int validate_cfg(const nr_config* c) {
    if (!c) return NR_ERR_INVALID;
    if (c->block_size != nitro::kBlockSize) return NR_ERR_INVALID;
    if (c->total_blocks <= 0 || c->max_tokens_per_batch <= 0 || c->max_new_tokens <= 0) return NR_ERR_INVALID;
    if (c->max_batch <= 0 || c->max_batch > 1024 || c->max_prefill_tokens <= 0) return NR_ERR_INVALID;
    if (c->q8_mode != NR_Q8_FIXED && c->q8_mode != NR_Q8_FAITHFUL) return NR_ERR_INVALID;
    if (c->sched_mode != NR_SCHED_REFERENCE && c->sched_mode != NR_SCHED_PACKED) return NR_ERR_INVALID;
    if (c->kv_dtype != NR_KV_F32 && c->kv_dtype != NR_KV_BF16) return NR_ERR_INVALID;
    return NR_OK;
}

int create_common(const nr_config* cfg, const nitro::ModelShape& shape, const uint8_t* file, size_t size,
                  nr_engine** out) {
    Engine* e = new (std::nothrow) Engine(*cfg, shape);
    if (!e) return NR_ERR_INVALID;
    int rc = e->init_device(file, size);
    if (rc != NR_OK) {
        g_create_error = e->last_error;
        delete e;
        return rc;
    }
    *out = new nr_engine{e};
    return NR_OK;
}

Request* find_req(nr_engine* e, int req_id) {
    auto it = e->impl->requests.find(req_id);
    return it == e->impl->requests.end() ? nullptr : it->second.get();
}

Request* find_seq(nr_engine* e, int handle) {
    auto it = e->impl->seqs.find(handle);
    if (it != e->impl->seqs.end()) return it->second.get();
    return nullptr;
}

int copy_out(const std::vector<int>& v, int32_t* out, int32_t cap, int32_t* n) {
    if (n) *n = (int32_t)v.size();
    if (out)
        for (int32_t i = 0; i < cap && i < (int32_t)v.size(); i++) out[i] = v[i];
    return NR_OK;
}

}  // namespace

extern "C" {

void nr_config_default(nr_config* c) {
    if (!c) return;
    memset(c, 0, sizeof(*c));
    c->total_blocks = 1000;          // src/Server_Inference.cpp:85
    c->max_tokens_per_batch = 256;   // src/pagedMemory.hpp:307
    c->max_new_tokens = 20;          // src/pagedMemory.hpp:393
    c->block_size = nitro::kBlockSize;
    c->sched_mode = NR_SCHED_REFERENCE;
    c->q8_mode = NR_Q8_FIXED;
    c->max_batch = 256;
    c->max_prefill_tokens = 1024;
    c->device = 0;
}

int nr_engine_create_from_memory(const nr_config* cfg, const void* bytes, size_t size, nr_engine** out) {
    if (!out || !bytes) return NR_ERR_INVALID;
    *out = nullptr;
    int rc = validate_cfg(cfg);
    if (rc) return rc;
    nitro::ModelShape shape;
    rc = parse_shape(bytes, size, &shape);
    if (rc) return rc;
    if (shape.dim % 32 || shape.hidden % 32 || shape.kv_dim() % 32) {
        g_create_error = "dim, hidden_dim and kv_dim must be multiples of 32 (Q8_0 blocks)";
        return NR_ERR_FORMAT;
    }
    if (size < expected_file_size(shape)) {
        g_create_error = "model file is " + std::to_string(size) + " bytes, its header implies " +
                         std::to_string(expected_file_size(shape));
        return NR_ERR_FORMAT;
    }
    return create_common(cfg, shape, (const uint8_t*)bytes, size, out);
}

int nr_engine_create(const nr_config* cfg, const char* path, nr_engine** out) {
    if (!out || !path) return NR_ERR_INVALID;
    *out = nullptr;
    int rc = validate_cfg(cfg);
    if (rc) return rc;
    int fd = open(path, O_RDONLY);
    if (fd < 0) {
        g_create_error = std::string("cannot open ") + path;
        return NR_ERR_IO;
    }
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); return NR_ERR_IO; }
    void* data = mmap(nullptr, st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (data == MAP_FAILED) return NR_ERR_IO;
    rc = nr_engine_create_from_memory(cfg, data, (size_t)st.st_size, out);
    munmap(data, st.st_size);
    return rc;
}

int nr_engine_create_host_only(const nr_config* cfg, const int32_t shape7[7], nr_engine** out) {
    if (!out || !shape7) return NR_ERR_INVALID;
    *out = nullptr;
    int rc = validate_cfg(cfg);
    if (rc) return rc;
    nitro::ModelShape shape;
    rc = parse_shape(shape7, 28, &shape);
    if (rc) return rc;
    nr_config c = *cfg;
    c.device = -1;
    return create_common(&c, shape, nullptr, 0, out);
}

int nr_engine_destroy(nr_engine* e) {
    if (!e) return NR_ERR_INVALID;
    delete e->impl;
    delete e;
    return NR_OK;
}

int nr_model_shape(const nr_engine* e, int32_t s[7]) {
    if (!e || !s) return NR_ERR_INVALID;
    const nitro::ModelShape& m = e->impl->shape();
    s[0] = m.dim; s[1] = m.hidden; s[2] = m.n_layers; s[3] = m.n_heads;
    s[4] = m.n_kv_heads; s[5] = m.vocab; s[6] = m.seq_len;
    return NR_OK;
}

void* nr_engine_stream(const nr_engine* e) { return e ? (void*)e->impl->stream() : nullptr; }

const char* nr_last_error(const nr_engine* e) {
    return e ? e->impl->last_error.c_str() : g_create_error.c_str();
}

// ------------------------------------------------------------------ request level
int nr_add_request(nr_engine* e, int32_t req_id, const int32_t* prompt, int32_t n) {
    if (!e || !prompt || n <= 0) return NR_ERR_INVALID;
    Engine& E = *e->impl;
    if (E.requests.count(req_id)) return E.fail(NR_ERR_INVALID, "duplicate request id");
    if (n > E.shape().seq_len) return E.fail(NR_ERR_INVALID, "prompt longer than seq_len");
    for (int i = 0; i < n; i++)
        if (prompt[i] < 0 || prompt[i] >= E.shape().vocab) return E.fail(NR_ERR_INVALID, "token id out of range");
    std::unique_ptr<Request> r(new Request());
    r->req_id = req_id;
    r->prompt_tokens.assign(prompt, prompt + n);
    r->seq.seq_id = req_id;
    E.sched().add_request(r.get());
    E.requests[req_id] = std::move(r);
    return NR_OK;
}

int nr_has_active(nr_engine* e) {
    if (!e) return NR_ERR_INVALID;
    return e->impl->sched().has_active_requests() ? 1 : 0;
}

namespace {
int do_plan(Engine& E, nitro::StepPlan& p) {
    if (E.sched().plan(p, E.mem(), E.cache()) != 0) return E.fail(NR_ERR_NO_BLOCKS, "KV pool exhausted");
    E.stats.steps++;
    E.stats.cache_hit_pages += p.prefill_hits;
    E.stats.evictions = E.cache().evictions();
    return NR_OK;
}
}  // namespace

int nr_step(nr_engine* e, nr_step_out* out) {
    if (!e) return NR_ERR_INVALID;
    Engine& E = *e->impl;
    if (!E.has_device()) return E.fail(NR_ERR_NO_DEVICE, "host-only engine: use nr_step_plan/nr_step_commit");
    nitro::StepPlan p;
    int rc = do_plan(E, p);
    if (rc) return rc;
    const int V = E.shape().vocab;
    std::vector<int> toks;
    std::vector<int> ids;
    const bool want_logits = out && out->emitted_logits;
    const int cap = out ? out->emitted_cap : 0;
    int prefill_tokens = 0;
    if (!p.prefills.empty()) {
        // every chunk of the step in one forward pass; a token for each completed prompt
        const int n = (int)p.prefills.size();
        std::vector<nitro::PrefillSeg> segs(n);
        int n_done = 0;
        for (int i = 0; i < n; i++) {
            const nitro::PrefillPart& part = p.prefills[i];
            segs[i] = {&part.req->seq, part.chunk.data(), (int)part.chunk.size(), part.start, part.done};
            prefill_tokens += segs[i].T;
            n_done += part.done ? 1 : 0;
        }
        std::vector<int> am(std::max(n_done, 1));
        float* lg = nullptr;
        std::vector<float> tmp;
        if (want_logits && n_done > 0) {
            if (n_done <= cap) lg = out->emitted_logits;
            else { tmp.resize((size_t)n_done * V); lg = tmp.data(); }
        }
        rc = E.forward_prefill_batch(segs.data(), n, lg, am.data());
        if (rc) return rc;
        int k = 0;
        for (const nitro::PrefillPart& part : p.prefills)
            if (part.done) {
                toks.push_back(am[k++]);
                ids.push_back(part.req->req_id);
            }
    }
    const int B = (int)p.decode_reqs.size();
    if (B > 0) {
        std::vector<const Sequence*> seqs(B);
        for (int b = 0; b < B; b++) seqs[b] = &p.decode_reqs[b]->seq;
        std::vector<int> am(B);
        float* lg = nullptr;
        std::vector<float> tmp;
        if (want_logits) {
            if ((int)ids.size() + B <= cap) lg = out->emitted_logits + ids.size() * (size_t)V;
            else { tmp.resize((size_t)B * V); lg = tmp.data(); }
        }
        rc = E.forward_decode(B, p.decode_tokens.data(), p.decode_positions.data(), seqs.data(), lg, am.data());
        if (rc) return rc;
        for (int b = 0; b < B; b++) {
            toks.push_back(am[b]);
            ids.push_back(p.decode_reqs[b]->req_id);
        }
    }
    E.sched().commit(p, toks.data(), (int)toks.size());
    if (out) {
        out->n_released = p.n_released;
        out->prefill_req_id = p.prefills.empty() ? -1 : p.prefills[0].req->req_id;
        out->prefill_tokens = prefill_tokens;
        out->prefill_hits = p.prefill_hits;
        out->n_prefill = (int)p.prefills.size();
        out->n_decode = B;
        out->n_emitted = (int)toks.size();
        for (int i = 0; i < (int)toks.size() && i < cap; i++) {
            if (out->emitted_req_ids) out->emitted_req_ids[i] = ids[i];
            if (out->emitted_tokens) out->emitted_tokens[i] = toks[i];
        }
    }
    return NR_OK;
}

// plans in flight for the split API (one at a time per engine)
namespace {
struct PendingPlan {
    nitro::StepPlan plan;
    bool valid = false;
};
std::vector<std::pair<nr_engine*, PendingPlan>> g_pending;
PendingPlan& pending_for(nr_engine* e) {
    for (auto& p : g_pending)
        if (p.first == e) return p.second;
    g_pending.push_back({e, PendingPlan()});
    return g_pending.back().second;
}
}  // namespace

int nr_step_plan(nr_engine* e, nr_plan* plan) {
    if (!e || !plan) return NR_ERR_INVALID;
    Engine& E = *e->impl;
    PendingPlan& pp = pending_for(e);
    int rc = do_plan(E, pp.plan);
    if (rc) return rc;
    pp.valid = true;
    const nitro::StepPlan& p = pp.plan;
    plan->n_released = p.n_released;
    const nitro::PrefillPart* first = p.prefills.empty() ? nullptr : &p.prefills[0];
    plan->prefill_req_id = first ? first->req->req_id : -1;
    plan->prefill_start = first ? first->start : 0;
    plan->prefill_tokens = first ? (int)first->chunk.size() : 0;
    plan->prefill_done = first && first->done ? 1 : 0;
    plan->prefill_hits = p.prefill_hits;
    plan->n_prefill = (int)p.prefills.size();
    for (int i = 0; i < plan->n_prefill && i < plan->prefill_cap; i++) {
        const nitro::PrefillPart& part = p.prefills[i];
        if (plan->prefill_req_ids) plan->prefill_req_ids[i] = part.req->req_id;
        if (plan->prefill_starts) plan->prefill_starts[i] = part.start;
        if (plan->prefill_lens) plan->prefill_lens[i] = (int)part.chunk.size();
        if (plan->prefill_dones) plan->prefill_dones[i] = part.done ? 1 : 0;
    }
    plan->n_decode = (int)p.decode_reqs.size();
    if (plan->decode_req_ids)
        for (int i = 0; i < plan->n_decode && i < plan->decode_cap; i++)
            plan->decode_req_ids[i] = p.decode_reqs[i]->req_id;
    return NR_OK;
}

int nr_step_commit(nr_engine* e, const nr_plan* plan, const int32_t* tokens, int32_t n_tokens) {
    if (!e || !plan || (n_tokens > 0 && !tokens)) return NR_ERR_INVALID;
    PendingPlan& pp = pending_for(e);
    if (!pp.valid) return e->impl->fail(NR_ERR_INVALID, "no plan pending");
    int expect = (int)pp.plan.decode_reqs.size();
    for (const nitro::PrefillPart& part : pp.plan.prefills) expect += part.done ? 1 : 0;
    if (n_tokens != expect) return e->impl->fail(NR_ERR_INVALID, "token count does not match the plan");
    e->impl->sched().commit(pp.plan, tokens, n_tokens);
    pp.valid = false;
    return NR_OK;
}

int nr_request_tokens(nr_engine* e, int32_t req_id, int32_t* out, int32_t cap, int32_t* n) {
    if (!e) return NR_ERR_INVALID;
    Request* r = find_req(e, req_id);
    if (!r) return NR_ERR_UNKNOWN_SEQ;
    return copy_out(r->generated_tokens, out, cap, n);
}

int nr_request_state(nr_engine* e, int32_t req_id, int32_t f[4]) {
    if (!e || !f) return NR_ERR_INVALID;
    Request* r = find_req(e, req_id);
    if (!r) return NR_ERR_UNKNOWN_SEQ;
    f[0] = r->prefill_idx; f[1] = r->is_prefill_done; f[2] = r->is_finished; f[3] = r->next_token_to_process;
    return NR_OK;
}

int nr_request_block_table(nr_engine* e, int32_t req_id, int32_t* out, int32_t cap, int32_t* n) {
    if (!e) return NR_ERR_INVALID;
    Request* r = find_req(e, req_id);
    if (!r) return NR_ERR_UNKNOWN_SEQ;
    return copy_out(r->seq.block_table, out, cap, n);
}

int nr_running_batch(nr_engine* e, int32_t* out, int32_t cap, int32_t* n) {
    if (!e) return NR_ERR_INVALID;
    std::vector<int> ids;
    for (Request* r : e->impl->sched().running()) ids.push_back(r->req_id);
    return copy_out(ids, out, cap, n);
}

// ------------------------------------------------------------------ sequence level
int nr_seq_create(nr_engine* e, int32_t seq_id, int32_t* handle) {
    if (!e || !handle) return NR_ERR_INVALID;
    Engine& E = *e->impl;
    std::unique_ptr<Request> r(new Request());
    r->req_id = seq_id;
    r->seq.seq_id = seq_id;
    int h = E.next_seq_handle++;
    E.seqs[h] = std::move(r);
    *handle = h;
    return NR_OK;
}

int nr_seq_append(nr_engine* e, int32_t handle, int32_t token) {
    if (!e) return NR_ERR_INVALID;
    Request* r = find_seq(e, handle);
    if (!r) return NR_ERR_UNKNOWN_SEQ;
    Engine& E = *e->impl;
    if (r->seq.allocate_next_token(token, E.mem(), E.cache()) != 0) return E.fail(NR_ERR_NO_BLOCKS, "KV pool exhausted");
    return NR_OK;
}

int nr_seq_flush_cache(nr_engine* e, int32_t handle) {
    if (!e) return NR_ERR_INVALID;
    Request* r = find_seq(e, handle);
    if (!r) return NR_ERR_UNKNOWN_SEQ;
    r->seq.flush_cache(e->impl->cache());
    return NR_OK;
}

int nr_seq_release(nr_engine* e, int32_t handle) {
    if (!e) return NR_ERR_INVALID;
    Request* r = find_seq(e, handle);
    if (!r) return NR_ERR_UNKNOWN_SEQ;
    r->seq.release(e->impl->mem(), e->impl->cache());
    return NR_OK;
}

int nr_seq_destroy(nr_engine* e, int32_t handle) {
    if (!e) return NR_ERR_INVALID;
    return e->impl->seqs.erase(handle) ? NR_OK : NR_ERR_UNKNOWN_SEQ;
}

int nr_seq_block_table(nr_engine* e, int32_t handle, int32_t* out, int32_t cap, int32_t* n) {
    if (!e) return NR_ERR_INVALID;
    Request* r = find_seq(e, handle);
    if (!r) return NR_ERR_UNKNOWN_SEQ;
    return copy_out(r->seq.block_table, out, cap, n);
}

int nr_seq_info(nr_engine* e, int32_t handle, int32_t info[3], uint64_t* hash) {
    if (!e || !info) return NR_ERR_INVALID;
    Request* r = find_seq(e, handle);
    if (!r) return NR_ERR_UNKNOWN_SEQ;
    info[0] = r->seq.logical_token_count;
    info[1] = (int32_t)r->seq.token_buffer.size();
    info[2] = (int32_t)r->seq.block_table.size();
    if (hash) *hash = r->seq.current_hash;
    return NR_OK;
}

int nr_forward_prefill(nr_engine* e, int32_t handle, const int32_t* tokens, int32_t T, int32_t start_pos,
                       float* logits_out, int32_t* argmax_out) {
    if (!e || !tokens || T <= 0) return NR_ERR_INVALID;  // the reference returns nullptr for T == 0 (:426)
    Request* r = find_seq(e, handle);
    if (!r) return NR_ERR_UNKNOWN_SEQ;
    Engine& E = *e->impl;
    if (!E.has_device()) return E.fail(NR_ERR_NO_DEVICE, "host-only engine");
    if (start_pos < 0 || start_pos + T > E.shape().seq_len) return E.fail(NR_ERR_INVALID, "positions exceed seq_len");
    for (int t = 0; t < T; t++)
        if (r->seq.allocate_next_token(tokens[t], E.mem(), E.cache()) != 0)
            return E.fail(NR_ERR_NO_BLOCKS, "KV pool exhausted");
    return E.forward_prefill(r->seq, tokens, T, start_pos, logits_out, argmax_out);
}

int nr_forward_decode(nr_engine* e, int32_t B, const int32_t* tokens, const int32_t* positions,
                      const int32_t* handles, float* logits_out, int32_t* argmax_out) {
    if (!e || !tokens || !positions || !handles || B <= 0) return NR_ERR_INVALID;  // (:573)
    Engine& E = *e->impl;
    if (!E.has_device()) return E.fail(NR_ERR_NO_DEVICE, "host-only engine");
    std::vector<Request*> rs(B);
    for (int b = 0; b < B; b++) {
        rs[b] = find_seq(e, handles[b]);
        if (!rs[b]) return NR_ERR_UNKNOWN_SEQ;
    }
    // serial allocation in row order (the reference allocates inside a parallel loop,
    // src/model_q8.cpp:578-582, which matches this order only at one thread)
    for (int b = 0; b < B; b++)
        if (rs[b]->seq.allocate_next_token(tokens[b], E.mem(), E.cache()) != 0)
            return E.fail(NR_ERR_NO_BLOCKS, "KV pool exhausted");
    std::vector<const Sequence*> seqs(B);
    for (int b = 0; b < B; b++) seqs[b] = &rs[b]->seq;
    return E.forward_decode(B, tokens, positions, seqs.data(), logits_out, argmax_out);
}

int nr_forward_paged(nr_engine* e, int32_t handle, int32_t token, int32_t pos, float* logits_out,
                     int32_t* argmax_out) {
    if (!e) return NR_ERR_INVALID;
    Request* r = find_seq(e, handle);
    if (!r) return NR_ERR_UNKNOWN_SEQ;
    Engine& E = *e->impl;
    if (!E.has_device()) return E.fail(NR_ERR_NO_DEVICE, "host-only engine");
    if (r->seq.allocate_next_token(token, E.mem(), E.cache()) != 0) return E.fail(NR_ERR_NO_BLOCKS, "KV pool exhausted");
    const Sequence* s = &r->seq;
    return E.forward_decode(1, &token, &pos, &s, logits_out, argmax_out, /*force_fixed=*/true);
}

int nr_ingest_prompt(nr_engine* e, int32_t handle, const int32_t* prompt, int32_t n, int32_t enable_cache,
                     float* logits_out, int32_t* n_tokens, int32_t* computed) {
    if (!e || (!prompt && n > 0) || n < 0) return NR_ERR_INVALID;
    Request* r = find_seq(e, handle);
    if (!r) return NR_ERR_UNKNOWN_SEQ;
    Engine& E = *e->impl;
    Sequence& s = r->seq;
    int p = 0;
    if (enable_cache) {  // src/model_q8.cpp:698-715
        while (p + nitro::kBlockSize <= n) {
            uint64_t h = nitro::hash_block_state(s.current_hash, prompt + p, nitro::kBlockSize);
            int hit = E.cache().check_cache(h);
            if (hit == -1) break;
            E.mem().inc_ref_count(hit, E.cache());
            s.block_table.push_back(hit);
            s.logical_token_count += nitro::kBlockSize;
            s.current_hash = h;
            p += nitro::kBlockSize;
            E.stats.cache_hit_pages++;
        }
    }
    const int rest = n - p;
    if (computed) *computed = rest;
    if (rest > 0) {
        int rc = nr_forward_prefill(e, handle, prompt + p, rest, s.logical_token_count, logits_out, nullptr);
        if (rc) return rc;
    }
    if (n_tokens) *n_tokens = s.logical_token_count;
    return NR_OK;
}

// ------------------------------------------------------------------ introspection
int nr_pool_free_count(nr_engine* e) { return e ? e->impl->mem().free_count() : NR_ERR_INVALID; }

int nr_pool_free_list(nr_engine* e, int32_t* out, int32_t cap, int32_t* n) {
    if (!e) return NR_ERR_INVALID;
    return copy_out(e->impl->mem().free_list(), out, cap, n);
}

int nr_pool_block_state(nr_engine* e, int32_t block, int32_t st[4]) {
    if (!e || !st) return NR_ERR_INVALID;
    if (block < 0 || block >= e->impl->mem().total_blocks()) return NR_ERR_INVALID;
    const nitro::BlockMeta& b = e->impl->mem().block(block);
    st[0] = b.num_tokens; st[1] = b.ref_count; st[2] = b.parent_id; st[3] = b.child_count;
    return NR_OK;
}

int nr_cache_lookup(nr_engine* e, uint64_t hash, int32_t* block) {
    if (!e || !block) return NR_ERR_INVALID;
    *block = e->impl->cache().check_cache(hash);
    return NR_OK;
}

int nr_cache_size(nr_engine* e) { return e ? e->impl->cache().cache_size() : NR_ERR_INVALID; }

int nr_cache_is_cached(nr_engine* e, int32_t block) {
    if (!e || block < 0 || block >= e->impl->mem().total_blocks()) return NR_ERR_INVALID;
    return e->impl->cache().is_cached(block) ? 1 : 0;
}

int nr_cache_lru(nr_engine* e, int32_t* out, int32_t cap, int32_t* n) {
    if (!e) return NR_ERR_INVALID;
    return copy_out(e->impl->cache().lru_front_to_back(), out, cap, n);
}

int nr_cache_entries(nr_engine* e, uint64_t* hashes, int32_t* blocks, int32_t cap, int32_t* n) {
    if (!e) return NR_ERR_INVALID;
    const auto& m = e->impl->cache().entries();
    if (n) *n = (int32_t)m.size();
    int i = 0;
    for (const auto& kv : m) {
        if (i >= cap) break;
        if (hashes) hashes[i] = kv.first;
        if (blocks) blocks[i] = kv.second;
        i++;
    }
    return NR_OK;
}

int nr_pool_read_page(nr_engine* e, int32_t block, float* k_out, float* v_out) {
    if (!e) return NR_ERR_INVALID;
    return e->impl->read_page(block, k_out, v_out);
}

uint64_t nr_hash_block_state(uint64_t parent, const int32_t* tokens, int32_t n) {
    return nitro::hash_block_state(parent, tokens, n);
}

int32_t nr_argmax(const float* x, int32_t n) {
    int idx = 0;
    float mx = 0.0f;
    for (int i = 0; i < n; i++)
        if (x[i] > mx) { mx = x[i]; idx = i; }
    return idx;
}

int nr_engine_set_profiling(nr_engine* e, int32_t enable) {
    if (!e) return NR_ERR_INVALID;
    return e->impl->set_profiling(enable != 0);
}

int nr_engine_kernel_times(nr_engine* e, double ms[NR_KERNEL_CLASSES], int64_t launches[NR_KERNEL_CLASSES]) {
    if (!e) return NR_ERR_INVALID;
    return e->impl->kernel_times(ms, launches);
}

int nr_replay_decode(nr_engine* e, int32_t n) {
    if (!e || n < 0) return NR_ERR_INVALID;
    return e->impl->replay_decode(n);
}

int nr_replay_decode_attention(nr_engine* e, int32_t n, int32_t with_merge) {
    if (!e || n < 0) return NR_ERR_INVALID;
    return e->impl->replay_decode_attention(n, with_merge != 0);
}

int nr_decode_last_outputs(nr_engine* e, int32_t* argmax_out, float* logits_out, int32_t* B_out) {
    if (!e) return NR_ERR_INVALID;
    return e->impl->last_decode_outputs(argmax_out, logits_out, B_out);
}

int nr_engine_stats(nr_engine* e, nr_stats* out) {
    if (!e || !out) return NR_ERR_INVALID;
    *out = e->impl->stats;
    out->evictions = e->impl->cache().evictions();
    out->kernel_launches = nitro::kernel_launch_count();
    return NR_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ kernel-level entry points
extern "C" {

size_t nr_paged_attention_workspace_size(int32_t B, int32_t n_heads, int32_t head_dim, int32_t max_pages) {
    if (B <= 0 || n_heads <= 0 || (head_dim != 64 && head_dim != 128) || max_pages <= 0) return 0;
    return nitro::decode_attn_workspace_bytes(B, n_heads, head_dim, max_pages);
}

int nr_paged_attention_decode(const float* q, const float* kpool, const float* vpool, const int32_t* block_tables,
                              int32_t max_pages, const int32_t* ctx_lens, int32_t B, int32_t n_heads,
                              int32_t n_kv_heads, int32_t head_dim, int32_t n_layers, int32_t layer, float* out,
                              void* workspace, int32_t* error_flag, void* stream) {
    if (!q || !kpool || !vpool || !block_tables || !ctx_lens || !out || !workspace) return NR_ERR_INVALID;
    if (B <= 0 || B > 1024 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || max_pages <= 0)
        return NR_ERR_INVALID;
    if (head_dim != 64 && head_dim != 128) return NR_ERR_INVALID;
    if (n_layers <= 0 || layer < 0 || layer >= n_layers) return NR_ERR_INVALID;
    nitro::DecodeAttnArgs a;
    a.q = q; a.kpool = kpool; a.vpool = vpool;
    a.geom = nitro::PoolGeom{n_layers, n_kv_heads, head_dim};
    a.layer = layer; a.block_tables = block_tables; a.max_pages = max_pages; a.ctx_lens = ctx_lens;
    a.B = B; a.n_heads = n_heads; a.out = out; a.err = error_flag;
    nitro::decode_attn_bind_workspace(a, workspace, max_pages);
    nitro::launch_decode_attention(a, max_pages * nitro::kBlockSize, (cudaStream_t)stream);
    return cudaGetLastError() == cudaSuccess ? NR_OK : NR_ERR_CUDA;
}

int nr_q8_matmul(const float* x, const int8_t* q, const float* scales, float* out, int32_t M, int32_t N, int32_t K,
                 int32_t q8_mode, void* stream) {
    if (!x || !q || !scales || !out || M <= 0 || N <= 0 || K <= 0) return NR_ERR_INVALID;
    if (K % 32 || N % 2) return NR_ERR_INVALID;
    if (q8_mode != NR_Q8_FIXED && q8_mode != NR_Q8_FAITHFUL) return NR_ERR_INVALID;
    nitro::GemmArgs g;
    g.x = x; g.ldx = K; g.wq = q; g.ws = scales; g.M = M; g.N = N; g.K = K;
    g.kbegin = q8_mode == NR_Q8_FAITHFUL ? K - 32 : 0;
    nitro::Epilogue e;
    e.kind = nitro::kEpiStore; e.out = out; e.ldo = N;
    nitro::launch_gemm(g, e, (cudaStream_t)stream);
    return cudaGetLastError() == cudaSuccess ? NR_OK : NR_ERR_CUDA;
}

size_t nr_q8_quantized_size(int64_t n) { return nitro::q8_quantized_bytes(n); }

int nr_quantize_q8_device(const float* w, int64_t n, uint8_t* out, void* stream) {
    if (n < 0 || (n > 0 && (!w || !out))) return NR_ERR_INVALID;
    if (reinterpret_cast<uintptr_t>(w) % 16 || reinterpret_cast<uintptr_t>(out) % 16) return NR_ERR_INVALID;
    nitro::launch_quantize_q8(w, n, out, (cudaStream_t)stream);
    return cudaGetLastError() == cudaSuccess ? NR_OK : NR_ERR_CUDA;
}

static int select_device(int32_t device) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) return NR_ERR_NO_DEVICE;
    if (device < 0 || device >= count) return NR_ERR_INVALID;
    return cudaSetDevice(device) == cudaSuccess ? NR_OK : NR_ERR_CUDA;
}

int nr_quantize_q8(const float* w, int64_t n, uint8_t* out, int32_t device) {
    if (n < 0 || (n > 0 && (!w || !out))) return NR_ERR_INVALID;
    const int rc = select_device(device);
    return rc != NR_OK ? rc : nitro::quantize_q8_host(w, n, out);
}

int nr_quantize_model_file(const char* in_path, const char* out_path, int32_t device) {
    if (!in_path || !out_path) return NR_ERR_INVALID;
    const int rc = select_device(device);
    return rc != NR_OK ? rc : nitro::quantize_model_file(in_path, out_path);
}

}  // extern "C"
