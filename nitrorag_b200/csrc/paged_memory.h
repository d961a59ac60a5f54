// Host-side page metadata of the engine: the 16-token KV block allocator, the FNV-1a
// prefix cache with dependency-aware LRU eviction, per-sequence block tables, requests
// and the reference-mode continuous scheduler.
//
// These reproduce nvivek17/NitroRAG src/pagedMemory.hpp decision for decision (page ids,
// free-list order, hash chain, refcounts, LRU order, eviction thresholds, admission
// order), because block tables and prefix hits must match the reference bit for bit.
// What changes: page *storage* lives in the device pools (the pool here only hands out
// ids), the metadata is single-threaded by design (the reference mutates it from inside
// an OpenMP loop, src/model_q8.cpp:578-582), and exhaustion is a status code instead of
// exit(1) (src/pagedMemory.hpp:117,212).
#pragma once
#include <cstdint>
#include <deque>
#include <memory>
#include <unordered_map>
#include <vector>

namespace nitro {

constexpr int kBlockSize = 16;                              // src/pagedMemory.hpp:9
constexpr uint64_t kFnvOffsetBasis = 14695981039346656037ULL;  // :11
constexpr uint64_t kFnvPrime = 1099511628211ULL;              // :12

// hash_block_state, src/pagedMemory.hpp:14-24.
uint64_t hash_block_state(uint64_t parent, const int32_t* tokens, int n);

// KVBlock metadata, src/pagedMemory.hpp:28-37 (the k/v pointers become device offsets
// derived from the id).
struct BlockMeta {
    int num_tokens = 0;
    int ref_count = 0;
    int parent_id = -1;
    int child_count = 0;
};

class PrefixCacheManager;

// KVBlock_Manager, src/pagedMemory.hpp:42-160.
class KVBlockManager {
public:
    explicit KVBlockManager(int total_blocks);
    // allocate_block (:113-128): evicts when the free list is empty; returns -1 if the pool
    // is still empty afterwards (the reference exits).
    int allocate_block(PrefixCacheManager& cache);
    void inc_ref_count(int id, PrefixCacheManager& cache);  // :129-132
    int free_count() const { return (int)free_list_.size(); }
    void free_block(int id, PrefixCacheManager& cache);     // :137-144
    void force_free_block(int id);                          // :145-151
    BlockMeta& block(int id) { return blocks_[id]; }
    const BlockMeta& block(int id) const { return blocks_[id]; }
    int total_blocks() const { return (int)blocks_.size(); }
    const std::vector<int>& free_list() const { return free_list_; }

private:
    std::vector<BlockMeta> blocks_;
    std::vector<int> free_list_;  // LIFO: back() is handed out next
};

// PrefixCacheManager, src/pagedMemory.hpp:64-229.
class PrefixCacheManager {
public:
    PrefixCacheManager(KVBlockManager& mm, int total_blocks);
    void evaluate_evictability(int id);                        // :171-186
    int check_cache(uint64_t hash) const;                      // :187-192
    void insert_cache(uint64_t hash, int id, int parent_id);   // :193-205
    // evict_lru_block (:206-229).  Returns 0, or -1 when no leaf is evictable and no page
    // is free (the reference exits there).
    int evict_lru_blocks();
    bool is_cached(int id) const { return cached_[id] != 0; }  // :168-170
    int cache_size() const { return (int)cache_map_.size(); }
    // cached pages nobody references: eviction can return each of them to the free list
    int reclaimable() const;
    std::vector<int> lru_front_to_back() const;
    const std::unordered_map<uint64_t, int>& entries() const { return cache_map_; }
    int64_t evictions() const { return evictions_; }

private:
    void lru_push_front(int id);
    void lru_erase(int id);

    KVBlockManager& mem_;
    std::unordered_map<uint64_t, int> cache_map_;  // hash -> page
    std::vector<uint8_t> cached_;                  // reverse_map membership per page
    std::vector<uint64_t> cached_hash_;            // reverse_map value per page
    // evictable leaves: intrusive doubly linked list, front = most recently made evictable
    std::vector<int> lru_prev_, lru_next_;
    std::vector<uint8_t> in_lru_;
    int lru_head_ = -1, lru_tail_ = -1;
    int min_free_blocks_;
    int target_free_blocks_;
    int64_t evictions_ = 0;
};

// Sequence, src/pagedMemory.hpp:233-285.
struct Sequence {
    int seq_id = 0;
    std::vector<int> block_table;
    int logical_token_count = 0;
    uint64_t current_hash = kFnvOffsetBasis;
    std::vector<int> token_buffer;  // tokens of the current page (<= 16)

    // allocate_next_token (:245-264).  Returns 0 or -1 (pool exhausted).
    int allocate_next_token(int token, KVBlockManager& mm, PrefixCacheManager& cache);
    void flush_cache(PrefixCacheManager& cache);                   // :265-273
    void release(KVBlockManager& mm, PrefixCacheManager& cache);   // :274-283
};

// Request, src/pagedMemory.hpp:287-300.
struct Request {
    int req_id = 0;
    std::vector<int> prompt_tokens;
    std::vector<int> generated_tokens;
    int prefill_idx = 0;
    bool is_prefill_done = false;
    bool is_finished = false;
    int next_token_to_process = -1;
    Sequence seq;
};

// One prompt chunk of a step.
struct PrefillPart {
    Request* req = nullptr;
    int start = 0;            // logical position of the first chunk token
    std::vector<int> chunk;
    int hits = 0;             // prefix-cache pages mapped for this request this step
    bool done = false;        // the chunk completes the prompt (a token is sampled)
};

// What one scheduler iteration will compute, after its allocations have been made.
struct StepPlan {
    int n_released = 0;
    std::vector<PrefillPart> prefills;  // reference mode: at most one
    int prefill_hits = 0;               // over all parts
    std::vector<Request*> decode_reqs;
    std::vector<int> decode_tokens;
    std::vector<int> decode_positions;
};

// Scheduling policies (nr_config.sched_mode).
enum SchedMode : int {
    kSchedReference = 0,  // Continuous_Scheduler::step as shipped: one prompt chunk per step
    kSchedPacked = 1,     // prompt chunks of several waiting requests per step, admission by pages
};

// Continuous_Scheduler, src/pagedMemory.hpp:303-398, split into plan (release, batch,
// admission, and every allocation the forward passes make, in the reference's order:
// prefill chunk tokens first, :428-430, then decode rows in batch order, :578-582) and
// commit (record sampled tokens, finish at max_new_tokens instead of the fixed 20, :393).
//
// kSchedPacked keeps the release and decode-batch rules and extends admission: while
// token budget is left after the decode rows, the FIFO head gets its prefix-cache scan
// and a chunk, and a request whose prompt completes makes room for the next one; a new
// request is admitted only if the pages its whole remaining prompt needs fit in the
// free plus reclaimable (cached, unreferenced) pages left after this step's decode rows
// and earlier chunks (always, when nothing else runs).  Prompt chunks are allocated in
// admission order, then the decode rows.
class ContinuousScheduler {
public:
    // seq_len caps a request's final length in the packed mode's page reservation (0: none)
    ContinuousScheduler(int max_tokens_per_batch, int max_new_tokens, int mode = kSchedReference, int seq_len = 0)
        : max_tokens_per_batch_(max_tokens_per_batch), max_new_tokens_(max_new_tokens), mode_(mode),
          seq_len_(seq_len) {}
    void add_request(Request* r);                    // :310-313
    bool has_active_requests() const { return !waiting_.empty() || !running_.empty(); }
    int plan(StepPlan& p, KVBlockManager& mm, PrefixCacheManager& cache);
    void commit(const StepPlan& p, const int* tokens, int n_tokens);
    const std::vector<Request*>& running() const { return running_; }
    size_t waiting() const { return waiting_.size(); }

private:
    // the FIFO head's prefix-cache scan (:344-357): mutate = false only counts the hits
    // and how many of the hit pages are unreferenced (they stop being reclaimable)
    int scan_prefix(Request* r, PrefixCacheManager& cache, KVBlockManager& mm, bool mutate, int* unreferenced);
    // pages request r can still take before it finishes: its whole prompt and
    // max_new_tokens - 1 generated tokens (the last one is never fed back), capped at seq_len
    int pages_to_finish(const Request* r, int extra_held = 0) const;
    std::deque<Request*> waiting_;
    std::vector<Request*> running_;
    int max_tokens_per_batch_;
    int max_new_tokens_;
    int mode_;
    int seq_len_;
};

}  // namespace nitro
