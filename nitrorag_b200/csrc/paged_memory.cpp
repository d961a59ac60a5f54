// Host-side page metadata; see paged_memory.h for what is reproduced from
// src/pagedMemory.hpp and what changes.
#include "paged_memory.h"

#include <algorithm>

namespace nitro {

uint64_t hash_block_state(uint64_t parent, const int32_t* tokens, int n) {
    uint64_t h = parent;
    for (int i = 0; i < n; i++) {
        uint32_t u = (uint32_t)tokens[i];
        // the 4 bytes of the int in little-endian order, as the reference walks them
        for (int b = 0; b < 4; b++) {
            h ^= (u >> (8 * b)) & 0xffu;
            h *= kFnvPrime;
        }
    }
    return h;
}

// ---------------------------------------------------------------- KVBlockManager
KVBlockManager::KVBlockManager(int total_blocks) : blocks_(total_blocks) {
    free_list_.reserve(total_blocks);
    for (int i = 0; i < total_blocks; i++) free_list_.push_back(i);  // :99-109
}

int KVBlockManager::allocate_block(PrefixCacheManager& cache) {
    if (free_list_.empty()) {
        if (cache.evict_lru_blocks() != 0 || free_list_.empty()) return -1;
    }
    int id = free_list_.back();
    free_list_.pop_back();
    BlockMeta& b = blocks_[id];
    b.ref_count = 1;
    b.num_tokens = 0;
    b.parent_id = -1;
    b.child_count = 0;
    return id;
}

void KVBlockManager::inc_ref_count(int id, PrefixCacheManager& cache) {
    blocks_[id].ref_count++;
    cache.evaluate_evictability(id);
}

void KVBlockManager::free_block(int id, PrefixCacheManager& cache) {
    blocks_[id].ref_count--;
    cache.evaluate_evictability(id);
    if (blocks_[id].ref_count == 0 && !cache.is_cached(id)) {
        blocks_[id].num_tokens = 0;
        free_list_.push_back(id);
    }
}

void KVBlockManager::force_free_block(int id) {
    BlockMeta& b = blocks_[id];
    b.num_tokens = 0;
    b.ref_count = 0;
    b.parent_id = -1;
    b.child_count = 0;
    free_list_.push_back(id);
}

// ---------------------------------------------------------------- PrefixCacheManager
PrefixCacheManager::PrefixCacheManager(KVBlockManager& mm, int total_blocks)
    : mem_(mm),
      cached_(total_blocks, 0),
      cached_hash_(total_blocks, 0),
      lru_prev_(total_blocks, -1),
      lru_next_(total_blocks, -1),
      in_lru_(total_blocks, 0) {
    // :165-166 (the products are doubles truncated to int)
    min_free_blocks_ = std::max(1, (int)(total_blocks * 0.05));
    target_free_blocks_ = std::max(2, (int)(total_blocks * 0.2));
}

void PrefixCacheManager::lru_push_front(int id) {
    lru_prev_[id] = -1;
    lru_next_[id] = lru_head_;
    if (lru_head_ >= 0) lru_prev_[lru_head_] = id;
    lru_head_ = id;
    if (lru_tail_ < 0) lru_tail_ = id;
    in_lru_[id] = 1;
}

void PrefixCacheManager::lru_erase(int id) {
    int p = lru_prev_[id], n = lru_next_[id];
    if (p >= 0) lru_next_[p] = n; else lru_head_ = n;
    if (n >= 0) lru_prev_[n] = p; else lru_tail_ = p;
    lru_prev_[id] = lru_next_[id] = -1;
    in_lru_[id] = 0;
}

std::vector<int> PrefixCacheManager::lru_front_to_back() const {
    std::vector<int> out;
    for (int id = lru_head_; id >= 0; id = lru_next_[id]) out.push_back(id);
    return out;
}

void PrefixCacheManager::evaluate_evictability(int id) {
    if (!is_cached(id)) return;
    const BlockMeta& b = mem_.block(id);
    bool evictable = b.ref_count == 0 && b.child_count == 0;
    bool in_lru = in_lru_[id] != 0;
    if (evictable && !in_lru) lru_push_front(id);
    else if (!evictable && in_lru) lru_erase(id);
}

int PrefixCacheManager::check_cache(uint64_t hash) const {
    auto it = cache_map_.find(hash);
    return it == cache_map_.end() ? -1 : it->second;
}

void PrefixCacheManager::insert_cache(uint64_t hash, int id, int parent_id) {
    // An existing entry for `hash` is overwritten while the page it pointed at keeps its
    // own reverse entry (src/pagedMemory.hpp:194-195); reproduced as is.
    cache_map_[hash] = id;
    cached_[id] = 1;
    cached_hash_[id] = hash;
    BlockMeta& b = mem_.block(id);
    b.parent_id = parent_id;
    b.child_count = 0;
    if (parent_id != -1) {
        mem_.block(parent_id).child_count++;
        evaluate_evictability(parent_id);
    }
    evaluate_evictability(id);
}

int PrefixCacheManager::evict_lru_blocks() {
    if (mem_.free_count() >= min_free_blocks_) return 0;
    while (mem_.free_count() < target_free_blocks_) {
        if (lru_tail_ < 0) {
            if (mem_.free_count() > 0) break;
            return -1;
        }
        int id = lru_tail_;
        lru_erase(id);
        cache_map_.erase(cached_hash_[id]);
        cached_[id] = 0;
        cached_hash_[id] = 0;
        int parent = mem_.block(id).parent_id;
        if (parent != -1) {
            mem_.block(parent).child_count--;
            evaluate_evictability(parent);
        }
        mem_.force_free_block(id);
        evictions_++;
    }
    return 0;
}

int PrefixCacheManager::reclaimable() const {
    int n = 0;
    for (int id = 0; id < (int)cached_.size(); id++)
        if (cached_[id] && mem_.block(id).ref_count == 0) n++;
    return n;
}

// ---------------------------------------------------------------- Sequence
int Sequence::allocate_next_token(int token, KVBlockManager& mm, PrefixCacheManager& cache) {
    if ((int)token_buffer.size() == kBlockSize) {
        // the page that just filled becomes shareable once the next token arrives
        current_hash = hash_block_state(current_hash, token_buffer.data(), kBlockSize);
        int finished = block_table.back();
        int parent = block_table.size() > 1 ? block_table[block_table.size() - 2] : -1;
        cache.insert_cache(current_hash, finished, parent);
        token_buffer.clear();
    }
    if (logical_token_count % kBlockSize == 0) {
        int id = mm.allocate_block(cache);
        if (id < 0) return -1;
        block_table.push_back(id);
    }
    token_buffer.push_back(token);
    mm.block(block_table.back()).num_tokens++;
    logical_token_count++;
    return 0;
}

void Sequence::flush_cache(PrefixCacheManager& cache) {
    if ((int)token_buffer.size() == kBlockSize) {
        current_hash = hash_block_state(current_hash, token_buffer.data(), kBlockSize);
        int parent = block_table.size() > 1 ? block_table[block_table.size() - 2] : -1;
        cache.insert_cache(current_hash, block_table.back(), parent);
    }
}

void Sequence::release(KVBlockManager& mm, PrefixCacheManager& cache) {
    for (int id : block_table) mm.free_block(id, cache);
    block_table.clear();
    token_buffer.clear();
    logical_token_count = 0;
    current_hash = kFnvOffsetBasis;
}

// ---------------------------------------------------------------- ContinuousScheduler
void ContinuousScheduler::add_request(Request* r) {
    r->next_token_to_process = r->prompt_tokens[0];
    waiting_.push_back(r);
}

int ContinuousScheduler::scan_prefix(Request* r, PrefixCacheManager& cache, KVBlockManager& mm, bool mutate,
                                     int* unreferenced) {
    const int n = (int)r->prompt_tokens.size();
    int idx = r->prefill_idx, hits = 0;
    uint64_t h = r->seq.current_hash;
    if (unreferenced) *unreferenced = 0;
    while (idx + kBlockSize <= n && r->seq.token_buffer.empty()) {
        const uint64_t nh = hash_block_state(h, r->prompt_tokens.data() + idx, kBlockSize);
        const int hit = cache.check_cache(nh);
        if (hit == -1) break;
        if (unreferenced && mm.block(hit).ref_count == 0) (*unreferenced)++;
        if (mutate) {
            mm.inc_ref_count(hit, cache);
            r->seq.block_table.push_back(hit);
            r->seq.logical_token_count += kBlockSize;
            r->seq.current_hash = nh;
            r->prefill_idx += kBlockSize;
        }
        h = nh;
        idx += kBlockSize;
        hits++;
    }
    return hits;
}

namespace {
int pages_for(int count) { return (count + kBlockSize - 1) / kBlockSize; }
}  // namespace

int ContinuousScheduler::pages_to_finish(const Request* r, int extra_held) const {
    int64_t final_count = (int64_t)r->prompt_tokens.size() + std::max(max_new_tokens_, 1) - 1;
    if (seq_len_ > 0) final_count = std::min<int64_t>(final_count, seq_len_);
    return std::max(0, pages_for((int)final_count) - (int)r->seq.block_table.size() - extra_held);
}

int ContinuousScheduler::plan(StepPlan& p, KVBlockManager& mm, PrefixCacheManager& cache) {
    p = StepPlan();
    // 1. release finished requests (:318-327)
    for (auto it = running_.begin(); it != running_.end();) {
        if ((*it)->is_finished) {
            (*it)->seq.release(mm, cache);
            it = running_.erase(it);
            p.n_released++;
        } else {
            ++it;
        }
    }
    int budget = max_tokens_per_batch_;
    const bool packed = mode_ == kSchedPacked;
    // 2. decode batch: every running request, one token each (:334-341)
    int reserved = 0;  // packed: pages the running and newly admitted requests can still take
    for (Request* r : running_) {
        if (r->is_prefill_done) {
            p.decode_tokens.push_back(r->next_token_to_process);
            p.decode_positions.push_back(r->seq.logical_token_count);
            p.decode_reqs.push_back(r);
            budget -= 1;
        }
        if (packed) reserved += pages_to_finish(r);
    }
    // 3. admission (:344-375): the FIFO head's prefix-cache scan, then one chunk within the
    // budget; packed mode goes on to the next request while budget and pages last, and
    // admits a request only if every page it can take until it finishes fits beside what
    // the requests already running can still take, so decode never runs the pool dry
    int available = packed ? mm.free_count() + cache.reclaimable() : 0;
    while (!waiting_.empty() && budget > 0) {
        Request* r = waiting_.front();
        const int n = (int)r->prompt_tokens.size();
        if (packed && !(running_.empty() && p.prefills.empty())) {
            int unref = 0;
            const int hits = scan_prefix(r, cache, mm, false, &unref);
            if (available - unref - reserved < pages_to_finish(r, hits)) break;  // wait for pages
        }
        PrefillPart part;
        part.req = r;
        part.hits = scan_prefix(r, cache, mm, true, nullptr);
        p.prefill_hits += part.hits;
        const int remaining = n - r->prefill_idx;
        const int chunk_size = std::min(remaining, budget);
        if (chunk_size > 0) {
            part.chunk.assign(r->prompt_tokens.begin() + r->prefill_idx,
                              r->prompt_tokens.begin() + r->prefill_idx + chunk_size);
            budget -= chunk_size;
        }
        const bool completes = r->prefill_idx + chunk_size == n;
        if (completes) {
            r->is_prefill_done = true;
            running_.push_back(r);
            waiting_.pop_front();
        } else {
            r->prefill_idx += chunk_size;
        }
        part.done = completes;
        if (packed) {
            reserved += pages_to_finish(r);
            available = mm.free_count() + cache.reclaimable();
        }
        // no chunk when the whole prompt was prefix hits (n a multiple of 16): the request
        // then runs without a sampled token, as in the reference
        if (!part.chunk.empty()) p.prefills.push_back(std::move(part));
        if (!packed || !completes) break;
    }
    // 4. the allocations forward_prefill_chunk makes before computing (:428-430), per chunk
    for (PrefillPart& part : p.prefills) {
        Sequence& s = part.req->seq;
        part.start = s.logical_token_count;
        for (int t : part.chunk)
            if (s.allocate_next_token(t, mm, cache) != 0) return -1;
    }
    // 5. the allocations forward_decode_batch makes, in row order (:578-582)
    for (size_t b = 0; b < p.decode_reqs.size(); b++)
        if (p.decode_reqs[b]->seq.allocate_next_token(p.decode_tokens[b], mm, cache) != 0) return -1;
    return 0;
}

void ContinuousScheduler::commit(const StepPlan& p, const int* tokens, int n_tokens) {
    int k = 0;
    // the greedy token of each prefill that completed its prompt (:380-384), in plan order
    for (const PrefillPart& part : p.prefills) {
        if (!part.done || k >= n_tokens) continue;
        Request* r = part.req;
        r->next_token_to_process = tokens[k];
        r->generated_tokens.push_back(tokens[k]);
        k++;
        if ((int)r->generated_tokens.size() >= max_new_tokens_) r->is_finished = true;
    }
    // decode rows (:389-396)
    for (size_t b = 0; b < p.decode_reqs.size() && k < n_tokens; b++, k++) {
        Request* r = p.decode_reqs[b];
        r->next_token_to_process = tokens[k];
        r->generated_tokens.push_back(tokens[k]);
        if ((int)r->generated_tokens.size() >= max_new_tokens_) r->is_finished = true;
    }
}

}  // namespace nitro
