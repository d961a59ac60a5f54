// The engine object behind the C ABI: model shape, device weights, the device KV pools,
// the host page metadata (paged_memory.h) and the forward passes.
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <tuple>
#include <string>
#include <vector>

#include "../../include/nitro_engine.h"
#include "kernels.h"
#include "paged_memory.h"

namespace nitro {

struct ModelShape {
    int dim = 0, hidden = 0, n_layers = 0, n_heads = 0, n_kv_heads = 0, vocab = 0, seq_len = 0;
    int head_dim() const { return dim / n_heads; }
    int kv_dim() const { return n_kv_heads * head_dim(); }
    int max_pages() const { return (seq_len + kBlockSize - 1) / kBlockSize; }
};

// Weights in device memory.  Q8_0 tensors are repacked at load time from the file's
// array of 36-byte blocks (fp32 scale + 32 int8, src/model_q8.cpp:29-32) into two arrays
// with the same values: int8 [rows][K] and fp32 scales [rows][K/32].  Per layer the q, k
// and v projections are stacked into one [dim + 2*kv_dim][dim] matrix and w1/w3 are
// interleaved row by row into one [2*hidden][dim] matrix so that one kernel computes each.
struct DeviceWeights {
    float* emb = nullptr;        // [vocab][dim], also the classifier (src/Server_Inference.cpp:69)
    float* rms_att = nullptr;    // [L][dim]
    float* rms_ffn = nullptr;    // [L][dim]
    float* rms_final = nullptr;  // [dim]
    float* freq_re = nullptr;    // [seq_len][head_dim/2]
    float* freq_im = nullptr;
    int8_t* qkv_q = nullptr; float* qkv_s = nullptr;  // [L][dim+2kv][dim]
    int8_t* wo_q = nullptr;  float* wo_s = nullptr;   // [L][dim][dim]
    int8_t* w13_q = nullptr; float* w13_s = nullptr;  // [L][2*hidden][dim]
    int8_t* w2_q = nullptr;  float* w2_s = nullptr;   // [L][dim][hidden]
    void* base = nullptr;
    size_t bytes = 0;
    // The projection weights once more, pre-split into bf16 hi/lo tiles for the tensor-core
    // kernel (tc_tile_weights; 4 bytes per weight): per layer, then the classifier.  Null
    // when disabled (NITRO_TILED_WEIGHTS=0); the kernel then converts q * scale itself.
    uint8_t* qkv_t = nullptr; uint8_t* wo_t = nullptr; uint8_t* w13_t = nullptr; uint8_t* w2_t = nullptr;
    uint8_t* cls_t = nullptr;
    size_t qkv_t_layer = 0, wo_t_layer = 0, w13_t_layer = 0, w2_t_layer = 0;
    void* tbase = nullptr;
    size_t tbytes = 0;
    // Projections too large for hi/lo tiles get raw Q8 tiles (tc_tile_q8_raw, 1.125 B per
    // weight) that the tensor-core kernel streams through a ring of bulk copies.
    uint8_t* qkv_r = nullptr; uint8_t* wo_r = nullptr; uint8_t* w13_r = nullptr; uint8_t* w2_r = nullptr;
    size_t qkv_r_layer = 0, wo_r_layer = 0, w13_r_layer = 0, w2_r_layer = 0;
    void* rbase = nullptr;
    size_t rbytes = 0;
};

// One prompt chunk of a multi-sequence prefill (Engine::forward_prefill_batch).
struct PrefillSeg {
    const Sequence* seq;
    const int* tokens;
    int T;
    int start_pos;
    bool emit;  // run the classifier on the chunk's last row (the chunk completes the prompt)
};

// Kernel classes timed by the engine's optional per-launch CUDA-event profiling.
enum KernelClass : int { kKEmbed = 0, kKQKV, kKAttn, kKWo, kKW13, kKW2, kKLogits, kKArgmax, kKMerge, kKClasses };

class Engine {
public:
    Engine(const nr_config& cfg, const ModelShape& shape);
    ~Engine();

    // Device set-up; `file` is the whole model image (nullptr for host-only engines).
    int init_device(const uint8_t* file, size_t size);

    const nr_config& cfg() const { return cfg_; }
    const ModelShape& shape() const { return shape_; }
    bool has_device() const { return cfg_.device >= 0; }
    cudaStream_t stream() const { return stream_; }

    // page metadata
    KVBlockManager& mem() { return *mem_; }
    PrefixCacheManager& cache() { return *cache_; }
    ContinuousScheduler& sched() { return *sched_; }

    // requests and bare sequences share one table of Request objects
    std::map<int, std::unique_ptr<Request>> requests;  // scheduler requests by req_id
    std::map<int, std::unique_ptr<Request>> seqs;      // sequence handles
    int next_seq_handle = 1;

    // forward passes over already-allocated tokens (block tables complete)
    int forward_prefill(const Sequence& seq, const int* tokens, int T, int start_pos, float* logits_out,
                        int* argmax_out);
    // Prompt chunks of several sequences in one forward pass: their rows concatenated
    // through every projection, causal attention per chunk; the classifier runs for the
    // chunks with emit set, whose logits rows / token ids are written in chunk order.
    int forward_prefill_batch(const PrefillSeg* segs, int n, float* logits_out, int* argmax_out);
    int forward_decode(int B, const int* tokens, const int* positions, const Sequence* const* seqs,
                       float* logits_out, int* argmax_out, bool force_fixed = false);
    int read_page(int block, float* k_out, float* v_out);
    // Enqueue the kernels of the last decode step again, n times, on the engine stream
    // (its descriptor is still resident); returns without synchronising.
    int replay_decode(int n);
    // Enqueue only the decode attention launches of the last decode step (every layer in
    // order, with or without the merge of split contexts), n times, back to back; the
    // attention output is rewritten with the same values.  For timing the kernel alone.
    int replay_decode_attention(int n, bool with_merge);
    // Outputs of the most recent decode step or replay: B argmax ids, and the B x vocab
    // logits when that step computed them (synchronises the engine stream).
    int last_decode_outputs(int* argmax_out, float* logits_out, int* B_out);

    // profiling: CUDA events around every launch, accumulated per KernelClass
    int set_profiling(bool on);
    int kernel_times(double* ms, int64_t* launches);
    void prof_mark(int cls, bool begin);

    std::string last_error;
    nr_stats stats{};

    int fail(int code, const std::string& msg) {
        last_error = msg;
        return code;
    }

private:
    int upload_weights(const uint8_t* file, size_t size);
    void enqueue_decode(int B, int max_ctx, bool force_fixed, bool want_logits);
    bool use_ss(int M) const;
    int prof_flush();
    int check_cuda(cudaError_t e, const char* what);
    void run_layers(int M, bool prefill, const Sequence* seq, int start_pos, int B_decode, int max_ctx,
                    bool force_fixed);
    DecodeAttnArgs decode_attn_plan(int l, int B, int max_ctx) const;

    nr_config cfg_;
    ModelShape shape_;
    std::unique_ptr<KVBlockManager> mem_;
    std::unique_ptr<PrefixCacheManager> cache_;
    std::unique_ptr<ContinuousScheduler> sched_;

    // device state
    cudaStream_t stream_ = nullptr;
    DeviceWeights w_;
    float* kpool_ = nullptr;
    float* vpool_ = nullptr;
    PoolGeom geom_{};
    int max_rows_ = 0;
    float* d_x_ = nullptr;     // [max_rows][dim] residual stream
    float* d_q_ = nullptr;     // [max_rows][dim]
    float* d_att_ = nullptr;   // [max_rows][dim]
    float* d_h_ = nullptr;     // [max_rows][hidden]
    float* d_logits_ = nullptr;  // [max_batch][vocab]
    unsigned long long* d_keys_ = nullptr;  // [max_rows]
    float* d_ss_ = nullptr;    // [ceil(dim/128)][max_rows] partial sums of squares of x
    int* d_argmax_ = nullptr;  // [max_rows]
    int* d_err_ = nullptr;
    void* d_attn_ws_ = nullptr;
    // large projections have both raw Q8 tiles and hi/lo tiles; batches of at least
    // wide_rows_ rows read the hi/lo tiles: kWideTileRows for the cluster-split kernel,
    // 3 when the stream-K kernel takes batches of 3-64 rows (1-2 rows take the matvec)
    bool wide_tiles_ = false;
    static constexpr int kWideTileRows = 32;
    int wide_rows_ = kWideTileRows;
    // stream-K scratch for raw-tile projections (partial tiles + flags), one slot per SM
    void* d_sk_ = nullptr;
    int sk_capacity_ = 0;
    // activations pre-split into hi/lo tiles for the wide-tile GEMM (rows x K x 4 bytes)
    void* d_xs_ = nullptr;
    int xs_cap_rows_ = 0, xs_cap_k_ = 0;
    // the scratch of the large-matrix and wide-tile projection paths, bound to a GemmArgs
    void attach_streamk(GemmArgs& g) const;
    // set while a multi-sequence prefill runs: its segment and tile tables on the device
    const int* d_seg_ = nullptr;
    const int* d_tiles_ = nullptr;
    int n_tiles_ = 0;
    // step descriptor: tokens, positions, pages, ctx, block tables (device + pinned host)
    int* d_desc_ = nullptr;
    int* h_desc_ = nullptr;
    size_t desc_ints_ = 0;
    int* d_tok_ = nullptr; int* d_pos_ = nullptr; int* d_page_ = nullptr; int* d_ctx_ = nullptr; int* d_bt_ = nullptr;
    int* h_tok_ = nullptr; int* h_pos_ = nullptr; int* h_page_ = nullptr; int* h_ctx_ = nullptr; int* h_bt_ = nullptr;
    int* h_argmax_ = nullptr;
    // last decode step (for replay)
    int last_B_ = 0, last_max_ctx_ = 0;
    bool last_force_fixed_ = false, last_valid_ = false, last_logits_ = false;
    // decode steps captured as CUDA graphs, keyed by (rows, force_fixed, logits); a key is
    // captured the second time it is seen (the first, eager run configures the kernels)
    struct GraphEntry {
        cudaGraphExec_t exec = nullptr;
        int64_t kernels = 0;
        int seen = 0;
    };
    std::map<std::tuple<int, bool, bool>, GraphEntry> graphs_;
    int launch_decode_step(int B, int max_ctx, bool force_fixed, bool want_logits);
    // profiling state
    bool profiling_ = false;
    std::vector<cudaEvent_t> ev_pool_;
    std::vector<std::pair<int, int>> ev_pairs_;  // (first event index, class)
    size_t ev_used_ = 0;
    int open_cls_ = -1;
    double kt_ms_[kKClasses] = {};
    int64_t kt_n_[kKClasses] = {};
};

struct ProfScope {
    Engine* e;
    int cls;
    ProfScope(Engine* eng, int c) : e(eng), cls(c) { e->prof_mark(cls, true); }
    ~ProfScope() { e->prof_mark(cls, false); }
};

}  // namespace nitro
