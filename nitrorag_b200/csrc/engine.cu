// Engine: model load, device pools and the forward passes of the Q8_0 decoder.
//
// forward_prefill follows forward_prefill_chunk (src/model_q8.cpp:424-557) and
// forward_decode follows forward_decode_batch (:571-694), with the per-layer work fused
// into five kernels:
//   1. QKV projection  (RMSNorm prologue, RoPE + K/V page append epilogue)  :443-484 / :586-624
//   2. paged attention                                                      :485-523 / :625-662
//   3. output projection + residual                                         :524-528 / :663-666
//   4. w1|w3 projection (RMSNorm prologue, SwiGLU epilogue)                  :529-545 / :668-681
//   5. w2 projection + residual                                             :546-551 / :682-686
// and the classifier (final RMSNorm prologue, fp32 embedding^T, greedy argmax keys).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>

#include "engine.h"

namespace nitro {

// ------------------------------------------------------------------ small kernels
__global__ void embed_kernel(const float* emb, const int* tokens, int M, int dim, float* x,
                             unsigned long long* keys, float* ss, int ss_ld) {
    const int m = blockIdx.x;
    grid_dependency_wait();  // x, keys and sums of squares may still be read by the previous step
    grid_dependents_launch();
    const float4* src = reinterpret_cast<const float4*>(emb + (int64_t)tokens[m] * dim);
    float4* dst = reinterpret_cast<float4*>(x + (int64_t)m * dim);
    for (int i = threadIdx.x; i < dim / 4; i += blockDim.x) dst[i] = src[i];
    if (threadIdx.x == 0) keys[m] = kArgmaxInitKey;
    if (!ss) return;
    // sums of squares per 128-feature slice (blockDim 128: one element per thread)
    __shared__ float part[4];
    const float* row = emb + (int64_t)tokens[m] * dim;
    for (int p = 0; p * 128 < dim; p++) {
        const int i = p * 128 + threadIdx.x;
        const float v = i < dim ? row[i] : 0.0f;
        const float w = warp_sum(v * v);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = w;
        __syncthreads();
        if (threadIdx.x == 0) ss[(int64_t)p * ss_ld + m] = part[0] + part[1] + part[2] + part[3];
        __syncthreads();
    }
}

__global__ void argmax_finish_kernel(const unsigned long long* keys, int M, int* out) {
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    grid_dependency_wait();
    grid_dependents_launch();
    if (m < M) out[m] = (int)(0xffffffffu - (uint32_t)(keys[m] & 0xffffffffull));
}

void launch_embed(const float* emb, const int* tokens, int M, int dim, float* x, unsigned long long* keys,
                  float* ss, int ss_ld, cudaStream_t s) {
    count_launch();
    launch_ex(embed_kernel, dim3(M), dim3(128), 0, s, 1, emb, tokens, M, dim, x, keys, ss, ss_ld);
}

void launch_argmax_finish(const unsigned long long* keys, int M, int* out, cudaStream_t s) {
    count_launch();
    launch_ex(argmax_finish_kernel, dim3((M + 127) / 128), dim3(128), 0, s, 1, keys, M, out);
}

// ------------------------------------------------------------------ engine
Engine::Engine(const nr_config& cfg, const ModelShape& shape) : cfg_(cfg), shape_(shape) {
    mem_.reset(new KVBlockManager(cfg.total_blocks));
    cache_.reset(new PrefixCacheManager(*mem_, cfg.total_blocks));
    sched_.reset(new ContinuousScheduler(cfg.max_tokens_per_batch, cfg.max_new_tokens, cfg.sched_mode, shape.seq_len));
}

Engine::~Engine() {
    if (!has_device()) return;
    cudaSetDevice(cfg_.device);
    if (stream_) cudaStreamSynchronize(stream_);
    cudaFree(w_.base);
    cudaFree(w_.tbase);
    cudaFree(w_.rbase);
    cudaFree(kpool_);
    cudaFree(vpool_);
    cudaFree(d_x_);
    cudaFree(d_q_);
    cudaFree(d_att_);
    cudaFree(d_h_);
    cudaFree(d_logits_);
    cudaFree(d_keys_);
    cudaFree(d_ss_);
    cudaFree(d_xs_);
    cudaFree(d_sk_);
    cudaFree(d_err_);
    cudaFree(d_attn_ws_);
    cudaFree(d_desc_);
    cudaFreeHost(h_desc_);
    cudaFreeHost(h_argmax_);
    for (auto& ev : ev_pool_) cudaEventDestroy(ev);
    for (auto& kv : graphs_)
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (stream_) cudaStreamDestroy(stream_);
}

int Engine::check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return NR_OK;
    return fail(NR_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define NR_CUDA(call)                                     \
    do {                                                  \
        int _rc = check_cuda((call), #call);              \
        if (_rc != NR_OK) return _rc;                     \
    } while (0)

namespace {

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// Repack `rows` rows of a Q8_0 tensor (array of 36-byte blocks, `K` weights per row) into
// int8 [rows][K] + fp32 scales [rows][K/32], rows written at dst row indices rowmap(r).
template <class RowMap>
void repack_q8(const uint8_t* src, int rows, int K, int8_t* q, float* s, RowMap rowmap) {
    const int nb = K / 32;
    for (int r = 0; r < rows; r++) {
        const int64_t dr = rowmap(r);
        for (int b = 0; b < nb; b++) {
            const uint8_t* blk = src + ((int64_t)r * nb + b) * 36;
            memcpy(s + dr * nb + b, blk, 4);
            memcpy(q + dr * K + (int64_t)b * 32, blk + 4, 32);
        }
    }
}

}  // namespace

int Engine::upload_weights(const uint8_t* file, size_t size) {
    const ModelShape& c = shape_;
    const int D = c.dim, H = c.hidden, L = c.n_layers, KV = c.kv_dim(), hd = c.head_dim();
    const int64_t q8 = 36;
    // byte offsets of each tensor in the file (src/Server_Inference.cpp:53-68)
    int64_t off = 28;
    auto take = [&](int64_t bytes) { int64_t o = off; off += bytes; return o; };
    const int64_t o_emb = take((int64_t)c.vocab * D * 4);
    const int64_t o_rms_att = take((int64_t)L * D * 4);
    const int64_t o_wq = take((int64_t)L * D * D / 32 * q8);
    const int64_t o_wk = take((int64_t)L * D * KV / 32 * q8);
    const int64_t o_wv = take((int64_t)L * D * KV / 32 * q8);
    const int64_t o_wo = take((int64_t)L * D * D / 32 * q8);
    const int64_t o_rms_ffn = take((int64_t)L * D * 4);
    const int64_t o_w1 = take((int64_t)L * H * D / 32 * q8);
    const int64_t o_w2 = take((int64_t)L * D * H / 32 * q8);
    const int64_t o_w3 = take((int64_t)L * H * D / 32 * q8);
    const int64_t o_rms_final = take((int64_t)D * 4);
    const int64_t o_fre = take((int64_t)c.seq_len * hd / 2 * 4);
    const int64_t o_fim = take((int64_t)c.seq_len * hd / 2 * 4);
    if ((size_t)off > size)
        return fail(NR_ERR_FORMAT, "model file is " + std::to_string(size) + " bytes, header implies " +
                                       std::to_string(off));

    // device layout: one allocation, 256-byte aligned pieces
    const int NQKV = D + 2 * KV;
    struct Piece { size_t bytes; void** dst; };
    size_t total = 0;
    std::vector<std::pair<size_t, void**>> pieces = {
        {(size_t)c.vocab * D * 4, (void**)&w_.emb},
        {(size_t)L * D * 4, (void**)&w_.rms_att},
        {(size_t)L * D * 4, (void**)&w_.rms_ffn},
        {(size_t)D * 4, (void**)&w_.rms_final},
        {(size_t)c.seq_len * hd / 2 * 4, (void**)&w_.freq_re},
        {(size_t)c.seq_len * hd / 2 * 4, (void**)&w_.freq_im},
        {(size_t)L * NQKV * D, (void**)&w_.qkv_q},
        {(size_t)L * NQKV * (D / 32) * 4, (void**)&w_.qkv_s},
        {(size_t)L * D * D, (void**)&w_.wo_q},
        {(size_t)L * D * (D / 32) * 4, (void**)&w_.wo_s},
        {(size_t)L * 2 * H * D, (void**)&w_.w13_q},
        {(size_t)L * 2 * H * (D / 32) * 4, (void**)&w_.w13_s},
        {(size_t)L * D * H, (void**)&w_.w2_q},
        {(size_t)L * D * (H / 32) * 4, (void**)&w_.w2_s},
    };
    for (auto& p : pieces) total += align256(p.first);
    NR_CUDA(cudaMalloc(&w_.base, total));
    w_.bytes = total;
    {
        char* p = (char*)w_.base;
        for (auto& pc : pieces) {
            *pc.second = p;
            p += align256(pc.first);
        }
    }
    // host image in the device layout, then one copy
    std::vector<uint8_t> host(total);
    auto hp = [&](void* dptr) { return host.data() + ((char*)dptr - (char*)w_.base); };
    memcpy(hp(w_.emb), file + o_emb, (size_t)c.vocab * D * 4);
    memcpy(hp(w_.rms_att), file + o_rms_att, (size_t)L * D * 4);
    memcpy(hp(w_.rms_ffn), file + o_rms_ffn, (size_t)L * D * 4);
    memcpy(hp(w_.rms_final), file + o_rms_final, (size_t)D * 4);
    memcpy(hp(w_.freq_re), file + o_fre, (size_t)c.seq_len * hd / 2 * 4);
    memcpy(hp(w_.freq_im), file + o_fim, (size_t)c.seq_len * hd / 2 * 4);
    for (int l = 0; l < L; l++) {
        int8_t* q = (int8_t*)hp(w_.qkv_q) + (int64_t)l * NQKV * D;
        float* s = (float*)hp(w_.qkv_s) + (int64_t)l * NQKV * (D / 32);
        repack_q8(file + o_wq + (int64_t)l * D * D / 32 * q8, D, D, q, s, [](int r) { return r; });
        repack_q8(file + o_wk + (int64_t)l * KV * D / 32 * q8, KV, D, q, s, [&](int r) { return D + r; });
        repack_q8(file + o_wv + (int64_t)l * KV * D / 32 * q8, KV, D, q, s, [&](int r) { return D + KV + r; });
        repack_q8(file + o_wo + (int64_t)l * D * D / 32 * q8, D, D, (int8_t*)hp(w_.wo_q) + (int64_t)l * D * D,
                  (float*)hp(w_.wo_s) + (int64_t)l * D * (D / 32), [](int r) { return r; });
        int8_t* q13 = (int8_t*)hp(w_.w13_q) + (int64_t)l * 2 * H * D;
        float* s13 = (float*)hp(w_.w13_s) + (int64_t)l * 2 * H * (D / 32);
        repack_q8(file + o_w1 + (int64_t)l * H * D / 32 * q8, H, D, q13, s13, [](int r) { return 2 * r; });
        repack_q8(file + o_w3 + (int64_t)l * H * D / 32 * q8, H, D, q13, s13, [](int r) { return 2 * r + 1; });
        repack_q8(file + o_w2 + (int64_t)l * D * H / 32 * q8, D, H, (int8_t*)hp(w_.w2_q) + (int64_t)l * D * H,
                  (float*)hp(w_.w2_s) + (int64_t)l * D * (H / 32), [](int r) { return r; });
    }
    NR_CUDA(cudaMemcpy(w_.base, host.data(), total, cudaMemcpyHostToDevice));

    // Tiled hi/lo copies for the tensor-core path (made on the device from the above).
    // They cost 4 B per weight instead of 1.125 B, so a Q8 projection gets them only while
    // its kernel is latency-bound rather than HBM-bound: at most 8 M weights (32 MB of
    // tiles, ~5 us of HBM).  The fp32 classifier always gets them (same 4 B per weight).
    // Larger projections get raw Q8 tiles (below) and, when HBM has room beside the K/V
    // pools, hi/lo tiles as well, which wide batches read instead (run_layers): at 64 rows
    // the on-chip conversion of raw tiles costs more than the extra bytes.
    const char* tiled_env = getenv("NITRO_TILED_WEIGHTS");
    if (!(tiled_env && tiled_env[0] == '0') && D % 64 == 0 && H % 64 == 0) {
        int64_t kTileMax = (int64_t)8 << 20;  // NITRO_TILE_MAX_WEIGHTS overrides (tests use 0)
        if (const char* tm = getenv("NITRO_TILE_MAX_WEIGHTS")) kTileMax = atoll(tm);
        auto small = [&](int64_t n, int64_t k) { return n * k <= kTileMax; };
        size_t wide_bytes = 0;
        for (auto nk : {std::make_pair((int64_t)NQKV, (int64_t)D), std::make_pair((int64_t)D, (int64_t)D),
                        std::make_pair((int64_t)2 * H, (int64_t)D), std::make_pair((int64_t)D, (int64_t)H)})
            if (!small(nk.first, nk.second)) wide_bytes += (size_t)L * align256(tc_tiled_weight_bytes((int)nk.first, (int)nk.second));
        bool wide = false;
        const char* wide_env = getenv("NITRO_WIDE_TILES");
        if (wide_bytes && !(wide_env && wide_env[0] == '0')) {
            size_t free_b = 0, total_b = 0;
            NR_CUDA(cudaMemGetInfo(&free_b, &total_b));
            const size_t pools = (size_t)2 * cfg_.total_blocks * (size_t)c.n_layers * c.n_kv_heads * kBlockSize * hd * 4;
            const size_t raw_b = (size_t)L * ((size_t)NQKV * D + (size_t)D * D + (size_t)2 * H * D + (size_t)D * H) * 9 / 8;
            wide = free_b > wide_bytes + raw_b + pools + ((size_t)4 << 30);  // 4 GB for activations and slack
        }
        wide_tiles_ = wide;
        auto tiled = [&](int64_t n, int64_t k) {
            return small(n, k) || wide ? align256(tc_tiled_weight_bytes((int)n, (int)k)) : 0;
        };
        w_.qkv_t_layer = tiled(NQKV, D);
        w_.wo_t_layer = tiled(D, D);
        w_.w13_t_layer = tiled(2 * H, D);
        w_.w2_t_layer = tiled(D, H);
        const size_t cls = align256(tc_tiled_weight_bytes(c.vocab, D));
        w_.tbytes = (size_t)L * (w_.qkv_t_layer + w_.wo_t_layer + w_.w13_t_layer + w_.w2_t_layer) + cls;
        NR_CUDA(cudaMalloc(&w_.tbase, w_.tbytes));
        uint8_t* p = (uint8_t*)w_.tbase;
        auto carve = [&](size_t per_layer) {
            uint8_t* r = per_layer ? p : nullptr;
            p += (size_t)L * per_layer;
            return r;
        };
        w_.qkv_t = carve(w_.qkv_t_layer);
        w_.wo_t = carve(w_.wo_t_layer);
        w_.w13_t = carve(w_.w13_t_layer);
        w_.w2_t = carve(w_.w2_t_layer);
        w_.cls_t = p;
        for (int l = 0; l < L; l++) {
            if (w_.qkv_t)
                tc_tile_weights(w_.qkv_q + (int64_t)l * NQKV * D, w_.qkv_s + (int64_t)l * NQKV * (D / 32), nullptr, NQKV,
                                D, w_.qkv_t + l * w_.qkv_t_layer, stream_);
            if (w_.wo_t)
                tc_tile_weights(w_.wo_q + (int64_t)l * D * D, w_.wo_s + (int64_t)l * D * (D / 32), nullptr, D, D,
                                w_.wo_t + l * w_.wo_t_layer, stream_);
            if (w_.w13_t)
                tc_tile_weights(w_.w13_q + (int64_t)l * 2 * H * D, w_.w13_s + (int64_t)l * 2 * H * (D / 32), nullptr,
                                2 * H, D, w_.w13_t + l * w_.w13_t_layer, stream_);
            if (w_.w2_t)
                tc_tile_weights(w_.w2_q + (int64_t)l * D * H, w_.w2_s + (int64_t)l * D * (H / 32), nullptr, D, H,
                                w_.w2_t + l * w_.w2_t_layer, stream_);
        }
        tc_tile_weights(nullptr, nullptr, w_.emb, c.vocab, D, w_.cls_t, stream_);
        NR_CUDA(cudaStreamSynchronize(stream_));
        NR_CUDA(cudaGetLastError());

        // the rest (HBM-bound projections) as raw Q8 tiles
        auto raw = [&](int64_t n, int64_t k) { return small(n, k) ? 0 : align256(tc_raw_q8_bytes((int)n, (int)k)); };
        w_.qkv_r_layer = raw(NQKV, D);
        w_.wo_r_layer = raw(D, D);
        w_.w13_r_layer = raw(2 * H, D);
        w_.w2_r_layer = raw(D, H);
        w_.rbytes = (size_t)L * (w_.qkv_r_layer + w_.wo_r_layer + w_.w13_r_layer + w_.w2_r_layer);
        if (w_.rbytes) {
            NR_CUDA(cudaMalloc(&w_.rbase, w_.rbytes));
            uint8_t* r = (uint8_t*)w_.rbase;
            auto carve_r = [&](size_t per_layer) {
                uint8_t* o = per_layer ? r : nullptr;
                r += (size_t)L * per_layer;
                return o;
            };
            w_.qkv_r = carve_r(w_.qkv_r_layer);
            w_.wo_r = carve_r(w_.wo_r_layer);
            w_.w13_r = carve_r(w_.w13_r_layer);
            w_.w2_r = carve_r(w_.w2_r_layer);
            for (int l = 0; l < L; l++) {
                if (w_.qkv_r)
                    tc_tile_q8_raw(w_.qkv_q + (int64_t)l * NQKV * D, w_.qkv_s + (int64_t)l * NQKV * (D / 32), NQKV, D,
                                   w_.qkv_r + l * w_.qkv_r_layer, stream_);
                if (w_.wo_r)
                    tc_tile_q8_raw(w_.wo_q + (int64_t)l * D * D, w_.wo_s + (int64_t)l * D * (D / 32), D, D,
                                   w_.wo_r + l * w_.wo_r_layer, stream_);
                if (w_.w13_r)
                    tc_tile_q8_raw(w_.w13_q + (int64_t)l * 2 * H * D, w_.w13_s + (int64_t)l * 2 * H * (D / 32), 2 * H, D,
                                   w_.w13_r + l * w_.w13_r_layer, stream_);
                if (w_.w2_r)
                    tc_tile_q8_raw(w_.w2_q + (int64_t)l * D * H, w_.w2_s + (int64_t)l * D * (H / 32), D, H,
                                   w_.w2_r + l * w_.w2_r_layer, stream_);
            }
            NR_CUDA(cudaStreamSynchronize(stream_));
            NR_CUDA(cudaGetLastError());
            // batches of 3-64 rows take the stream-K kernel: over the hi/lo tiles where they
            // exist (no conversion on chip), else over the raw tiles
            if (tc_streamk_enabled()) {
                int dev = 0, sms = 0;
                NR_CUDA(cudaGetDevice(&dev));
                NR_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
                sk_capacity_ = std::max(1, sms);
                const size_t sk_bytes = tc_streamk_scratch_bytes(sk_capacity_, std::max(D, H));
                NR_CUDA(cudaMalloc(&d_sk_, sk_bytes));
                NR_CUDA(cudaMemset(d_sk_, 0, sk_bytes));  // the flags start clear
                wide_rows_ = 3;
            }
        }
    }
    return NR_OK;
}

void Engine::attach_streamk(GemmArgs& g) const {
    g.xs_tiles = static_cast<uint8_t*>(d_xs_);
    g.xs_cap_rows = xs_cap_rows_;
    g.xs_cap_k = xs_cap_k_;
    if (!d_sk_) return;
    tc_streamk_bind(g, d_sk_, sk_capacity_, std::max(shape_.dim, shape_.hidden));
}

int Engine::init_device(const uint8_t* file, size_t size) {
    if (!has_device()) return NR_OK;
    const ModelShape& c = shape_;
    if (c.head_dim() != 64 && c.head_dim() != 128)
        return fail(NR_ERR_FORMAT, "head_dim must be 64 or 128, got " + std::to_string(c.head_dim()));
    if (c.dim % 32 || c.hidden % 32 || c.kv_dim() % 32 || c.n_heads % c.n_kv_heads)
        return fail(NR_ERR_FORMAT, "dim, hidden_dim and kv_dim must be multiples of 32");
    NR_CUDA(cudaSetDevice(cfg_.device));
    NR_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    int rc = upload_weights(file, size);
    if (rc != NR_OK) return rc;

    geom_ = PoolGeom{c.n_layers, c.n_kv_heads, c.head_dim(), cfg_.kv_dtype == NR_KV_BF16 ? 1 : 0};
    // layer-major pools (NITRO_KV_PAGE_MAJOR=1 keeps every page's layers together)
    const char* pm_env = getenv("NITRO_KV_PAGE_MAJOR");
    if (!(pm_env && pm_env[0] == '1')) geom_.pages = cfg_.total_blocks;
    const size_t pool_bytes = (size_t)cfg_.total_blocks * geom_.page_floats() * geom_.elem_bytes();
    NR_CUDA(cudaMalloc(&kpool_, pool_bytes));
    NR_CUDA(cudaMalloc(&vpool_, pool_bytes));
    NR_CUDA(cudaMemsetAsync(kpool_, 0, pool_bytes, stream_));
    NR_CUDA(cudaMemsetAsync(vpool_, 0, pool_bytes, stream_));

    max_rows_ = std::max(cfg_.max_batch, cfg_.max_prefill_tokens);
    const int R = max_rows_;
    NR_CUDA(cudaMalloc(&d_x_, (size_t)R * c.dim * 4));
    NR_CUDA(cudaMalloc(&d_q_, (size_t)R * c.dim * 4));
    NR_CUDA(cudaMalloc(&d_att_, (size_t)R * c.dim * 4));
    NR_CUDA(cudaMalloc(&d_h_, (size_t)R * c.hidden * 4));
    NR_CUDA(cudaMalloc(&d_logits_, (size_t)cfg_.max_batch * c.vocab * 4));
    NR_CUDA(cudaMalloc(&d_keys_, (size_t)R * 8));
    NR_CUDA(cudaMalloc(&d_ss_, (size_t)((c.dim + 127) / 128) * R * 4));
    // activations pre-split into bf16 hi/lo tiles for the tensor-core GEMM's wide tiles
    xs_cap_rows_ = (R + 255) / 256 * 256;
    xs_cap_k_ = std::max(c.dim, c.hidden);
    NR_CUDA(cudaMalloc(&d_xs_, (size_t)xs_cap_rows_ * xs_cap_k_ * 4));
    NR_CUDA(cudaMalloc(&d_err_, (size_t)(R + 1) * 4));  // [0] error flag, [1..] argmax ids
    d_argmax_ = d_err_ + 1;
    NR_CUDA(cudaMemsetAsync(d_err_, 0, (size_t)(R + 1) * 4, stream_));
    const size_t ws = decode_attn_workspace_bytes(cfg_.max_batch, c.n_heads, c.head_dim(), c.max_pages());
    NR_CUDA(cudaMalloc(&d_attn_ws_, ws));
    NR_CUDA(cudaMemsetAsync(d_attn_ws_, 0, ws, stream_));
    // decode: tok pos page ctx [max_batch] + block tables; prefill of several chunks:
    // tok pos page [R] + segments [max_batch][4] + query tiles + block tables
    const size_t mb = (size_t)std::max(cfg_.max_batch, 1);
    desc_ints_ = (size_t)3 * R + 4 * mb + 2 * ((size_t)R / 16 + mb) + mb * c.max_pages();
    NR_CUDA(cudaMalloc(&d_desc_, desc_ints_ * 4));
    NR_CUDA(cudaMallocHost(&h_desc_, desc_ints_ * 4));
    NR_CUDA(cudaMallocHost(&h_argmax_, (size_t)(R + 1) * 4));
    NR_CUDA(cudaStreamSynchronize(stream_));
    return NR_OK;
}

// RMSNorm sums of squares travel from the residual epilogues to the next projection when
// every projection of an M-row forward runs on the tensor-core path.
bool Engine::use_ss(int M) const {
    const ModelShape& c = shape_;
    return gemm_uses_tc(M, c.dim, c.dim) && gemm_uses_tc(M, c.dim, c.hidden) &&
           gemm_uses_tc(M, c.dim + 2 * c.kv_dim(), c.dim) && gemm_uses_tc(M, 2 * c.hidden, c.dim);
}

// Decode attention of layer l over the step descriptor's B rows (block tables and context
// lengths in HBM), its split partials in the engine's workspace.
DecodeAttnArgs Engine::decode_attn_plan(int l, int B, int max_ctx) const {
    const ModelShape& c = shape_;
    DecodeAttnArgs a;
    a.q = d_q_; a.kpool = kpool_; a.vpool = vpool_; a.geom = geom_; a.layer = l;
    a.block_tables = d_bt_; a.max_pages = c.max_pages(); a.ctx_lens = d_ctx_;
    a.n_heads = c.n_heads; a.out = d_att_; a.err = d_err_;
    // partial buffers are laid out for max_batch rows so B may vary per call
    a.B = cfg_.max_batch;
    decode_attn_bind_workspace(a, d_attn_ws_, c.max_pages());
    a.B = B;
    return plan_decode_attention(a, max_ctx);
}

void Engine::run_layers(int M, bool prefill, const Sequence* seq, int start_pos, int B_decode, int max_ctx,
                        bool force_fixed) {
    const ModelShape& c = shape_;
    const int D = c.dim, H = c.hidden, KV = c.kv_dim(), NQKV = D + 2 * KV;
    const bool faithful = cfg_.q8_mode == NR_Q8_FAITHFUL && !force_fixed;
    const bool ss = use_ss(M);
    const int ss_parts = (D + 127) / 128;
    for (int l = 0; l < c.n_layers; l++) {
        // 1. q,k,v = Wqkv . rmsnorm(x); RoPE; k,v -> pages
        GemmArgs g;
        g.err = d_err_;
        g.x = d_x_; g.ldx = D; g.norm_gain = w_.rms_att + (int64_t)l * D;
        g.wq = w_.qkv_q + (int64_t)l * NQKV * D; g.ws = w_.qkv_s + (int64_t)l * NQKV * (D / 32);
        g.M = M; g.N = NQKV; g.K = D; g.kbegin = faithful ? D - 32 : 0;
        if (w_.qkv_t && !faithful && (!w_.qkv_r || M >= wide_rows_)) g.wt = w_.qkv_t + l * w_.qkv_t_layer;
        if (w_.qkv_r) g.wr = w_.qkv_r + l * w_.qkv_r_layer;
        attach_streamk(g);
        if (ss) { g.ss_in = d_ss_; g.ss_parts = ss_parts; g.ss_ld = max_rows_; }
        Epilogue e;
        e.kind = kEpiQKV; e.q_out = d_q_; e.kpool = kpool_; e.vpool = vpool_; e.geom = geom_; e.layer = l;
        e.tok_page = d_page_; e.tok_pos = d_pos_; e.freq_re = w_.freq_re; e.freq_im = w_.freq_im;
        e.dim = D; e.kv_dim = KV; e.head_dim = c.head_dim();
        { ProfScope ps(this, kKQKV); launch_gemm(g, e, stream_); }
        // 2. attention
        if (prefill) {
            PrefillAttnArgs a;
            a.q = d_q_; a.kpool = kpool_; a.vpool = vpool_; a.geom = geom_; a.layer = l;
            a.block_table = d_bt_; a.T = M; a.start_pos = start_pos; a.n_heads = c.n_heads;
            a.out = d_att_; a.err = d_err_;
            a.seg = d_seg_; a.tiles = d_tiles_; a.n_tiles = n_tiles_;
            ProfScope ps(this, kKAttn);
            launch_prefill_attention(a, stream_);
        } else {
            const DecodeAttnArgs pa = decode_attn_plan(l, B_decode, max_ctx);
            { ProfScope ps(this, kKAttn); launch_decode_attention_main(pa, stream_); }
            if (decode_attn_splits(pa)) { ProfScope ps(this, kKMerge); launch_decode_merge(pa, stream_); }
        }
        // 3. x += Wo . att
        GemmArgs go;
        go.err = d_err_;
        go.x = d_att_; go.ldx = D; go.wq = w_.wo_q + (int64_t)l * D * D; go.ws = w_.wo_s + (int64_t)l * D * (D / 32);
        go.M = M; go.N = D; go.K = D; go.kbegin = faithful ? D - 32 : 0;
        if (w_.wo_t && !faithful && (!w_.wo_r || M >= wide_rows_)) go.wt = w_.wo_t + l * w_.wo_t_layer;
        if (w_.wo_r) go.wr = w_.wo_r + l * w_.wo_r_layer;
        attach_streamk(go);
        Epilogue eo;
        eo.kind = kEpiResidual; eo.out = d_x_; eo.ldo = D;
        if (ss) { eo.ss_out = d_ss_; eo.ss_ld = max_rows_; }
        { ProfScope ps(this, kKWo); launch_gemm(go, eo, stream_); }
        // 4. h = silu(W1 . rmsnorm(x)) * (W3 . rmsnorm(x))
        GemmArgs g13;
        g13.err = d_err_;
        g13.x = d_x_; g13.ldx = D; g13.norm_gain = w_.rms_ffn + (int64_t)l * D;
        g13.wq = w_.w13_q + (int64_t)l * 2 * H * D; g13.ws = w_.w13_s + (int64_t)l * 2 * H * (D / 32);
        g13.M = M; g13.N = 2 * H; g13.K = D; g13.kbegin = faithful ? D - 32 : 0;
        if (w_.w13_t && !faithful && (!w_.w13_r || M >= wide_rows_)) g13.wt = w_.w13_t + l * w_.w13_t_layer;
        if (w_.w13_r) g13.wr = w_.w13_r + l * w_.w13_r_layer;
        attach_streamk(g13);
        if (ss) { g13.ss_in = d_ss_; g13.ss_parts = ss_parts; g13.ss_ld = max_rows_; }
        Epilogue e13;
        e13.kind = kEpiSwiGLU; e13.out = d_h_; e13.ldo = H;
        { ProfScope ps(this, kKW13); launch_gemm(g13, e13, stream_); }
        // 5. x += W2 . h
        GemmArgs g2;
        g2.err = d_err_;
        g2.x = d_h_; g2.ldx = H; g2.wq = w_.w2_q + (int64_t)l * D * H; g2.ws = w_.w2_s + (int64_t)l * D * (H / 32);
        g2.M = M; g2.N = D; g2.K = H; g2.kbegin = faithful ? H - 32 : 0;
        if (w_.w2_t && !faithful && (!w_.w2_r || M >= wide_rows_)) g2.wt = w_.w2_t + l * w_.w2_t_layer;
        if (w_.w2_r) g2.wr = w_.w2_r + l * w_.w2_r_layer;
        attach_streamk(g2);
        Epilogue e2;
        e2.kind = kEpiResidual; e2.out = d_x_; e2.ldo = D;
        if (ss) { e2.ss_out = d_ss_; e2.ss_ld = max_rows_; }
        { ProfScope ps(this, kKW2); launch_gemm(g2, e2, stream_); }
    }
    (void)seq;
}

int Engine::forward_prefill(const Sequence& seq, const int* tokens, int T, int start_pos, float* logits_out,
                            int* argmax_out) {
    if (!has_device()) return fail(NR_ERR_NO_DEVICE, "host-only engine");
    const ModelShape& c = shape_;
    if (T <= 0) return fail(NR_ERR_INVALID, "empty prefill chunk");
    if (T > cfg_.max_prefill_tokens) return fail(NR_ERR_CAPACITY, "prefill chunk exceeds max_prefill_tokens");
    if (start_pos < 0 || start_pos + T > c.seq_len) return fail(NR_ERR_INVALID, "positions exceed seq_len");
    const int last_page = (start_pos + T - 1) / kBlockSize;
    if (last_page >= (int)seq.block_table.size()) return fail(NR_ERR_INVALID, "block table does not cover the chunk");
    for (int t = 0; t < T; t++)
        if (tokens[t] < 0 || tokens[t] >= c.vocab) return fail(NR_ERR_INVALID, "token id out of range");
    NR_CUDA(cudaSetDevice(cfg_.device));
    // descriptor: tok[T] pos[T] page[T] bt[n_pages]
    const int np = (int)seq.block_table.size();
    int* h = h_desc_;
    h_tok_ = h; h_pos_ = h + T; h_page_ = h + 2 * T; h_bt_ = h + 3 * T;
    for (int t = 0; t < T; t++) {
        const int pos = start_pos + t;
        h_tok_[t] = tokens[t];
        h_pos_[t] = pos;
        h_page_[t] = seq.block_table[pos / kBlockSize];
    }
    for (int p = 0; p < np; p++) h_bt_[p] = seq.block_table[p];
    const size_t n_ints = (size_t)3 * T + np;
    if (n_ints > desc_ints_) return fail(NR_ERR_CAPACITY, "descriptor overflow");
    d_tok_ = d_desc_; d_pos_ = d_desc_ + T; d_page_ = d_desc_ + 2 * T; d_bt_ = d_desc_ + 3 * T;
    NR_CUDA(cudaMemcpyAsync(d_desc_, h_desc_, n_ints * 4, cudaMemcpyHostToDevice, stream_));
    last_valid_ = false;  // the descriptor no longer holds a decode step
    { ProfScope ps(this, kKEmbed); launch_embed(w_.emb, d_tok_, T, c.dim, d_x_, d_keys_, use_ss(T) ? d_ss_ : nullptr, max_rows_, stream_); }
    run_layers(T, true, &seq, start_pos, 0, start_pos + T, false);
    // classifier over the last token (src/model_q8.cpp:553-556)
    GemmArgs gl;
    gl.err = d_err_;
    gl.x = d_x_ + (int64_t)(T - 1) * c.dim; gl.ldx = c.dim; gl.norm_gain = w_.rms_final; gl.wf = w_.emb;
    gl.wt = w_.cls_t;
    gl.M = 1; gl.N = c.vocab; gl.K = c.dim;
    Epilogue el;
    el.kind = kEpiLogits; el.out = logits_out ? d_logits_ : nullptr; el.ldo = c.vocab; el.argmax_keys = d_keys_;
    { ProfScope ps(this, kKLogits); launch_gemm(gl, el, stream_); }
    { ProfScope ps(this, kKArgmax); launch_argmax_finish(d_keys_, 1, d_argmax_, stream_); }
    NR_CUDA(cudaMemcpyAsync(h_argmax_, d_err_, 2 * 4, cudaMemcpyDeviceToHost, stream_));
    if (logits_out)
        NR_CUDA(cudaMemcpyAsync(logits_out, d_logits_, (size_t)c.vocab * 4, cudaMemcpyDeviceToHost, stream_));
    NR_CUDA(cudaStreamSynchronize(stream_));
    NR_CUDA(cudaGetLastError());
    if (h_argmax_[0] != 0) return fail(NR_ERR_TIMEOUT, "device wait timed out");
    if (argmax_out) *argmax_out = h_argmax_[1];
    stats.prefill_tokens += T;
    if (profiling_) return prof_flush();
    return NR_OK;
}

int Engine::forward_prefill_batch(const PrefillSeg* segs, int n, float* logits_out, int* argmax_out) {
    if (!has_device()) return fail(NR_ERR_NO_DEVICE, "host-only engine");
    if (n <= 0) return fail(NR_ERR_INVALID, "no prefill chunk");
    if (n == 1) {
        int tok = 0;
        const int rc = forward_prefill(*segs[0].seq, segs[0].tokens, segs[0].T, segs[0].start_pos,
                                       segs[0].emit ? logits_out : nullptr, &tok);
        if (rc == NR_OK && segs[0].emit && argmax_out) argmax_out[0] = tok;
        return rc;
    }
    if (n > cfg_.max_batch) return fail(NR_ERR_CAPACITY, "more prefill chunks than max_batch");
    const ModelShape& c = shape_;
    const int qt = prefill_attn_query_tile(c.head_dim());
    int T = 0, n_emit = 0, n_tiles = 0;
    size_t bt_ints = 0;
    for (int i = 0; i < n; i++) {
        const PrefillSeg& g = segs[i];
        if (g.T <= 0) return fail(NR_ERR_INVALID, "empty prefill chunk");
        if (g.start_pos < 0 || g.start_pos + g.T > c.seq_len) return fail(NR_ERR_INVALID, "positions exceed seq_len");
        if ((g.start_pos + g.T - 1) / kBlockSize >= (int)g.seq->block_table.size())
            return fail(NR_ERR_INVALID, "block table does not cover the chunk");
        for (int t = 0; t < g.T; t++)
            if (g.tokens[t] < 0 || g.tokens[t] >= c.vocab) return fail(NR_ERR_INVALID, "token id out of range");
        T += g.T;
        n_emit += g.emit ? 1 : 0;
        n_tiles += (g.T + qt - 1) / qt;
        bt_ints += g.seq->block_table.size();
    }
    if (T > cfg_.max_prefill_tokens) return fail(NR_ERR_CAPACITY, "prefill chunks exceed max_prefill_tokens");
    // descriptor: tok[T] pos[T] page[T] seg[n][4] tiles[n_tiles][2] block tables
    const size_t n_ints = (size_t)3 * T + 4 * (size_t)n + 2 * (size_t)n_tiles + bt_ints;
    if (n_ints > desc_ints_) return fail(NR_ERR_CAPACITY, "descriptor overflow");
    NR_CUDA(cudaSetDevice(cfg_.device));
    int* h = h_desc_;
    int* h_seg = h + 3 * T;
    int* h_tiles = h_seg + 4 * n;
    int* h_bts = h_tiles + 2 * n_tiles;
    struct Tile { int seg, qt, last; };
    std::vector<Tile> tiles;
    tiles.reserve(n_tiles);
    int row = 0, bt_off = 0;
    for (int i = 0; i < n; i++) {
        const PrefillSeg& g = segs[i];
        for (int t = 0; t < g.T; t++) {
            const int pos = g.start_pos + t;
            h[row + t] = g.tokens[t];
            h[T + row + t] = pos;
            h[2 * T + row + t] = g.seq->block_table[pos / kBlockSize];
        }
        h_seg[4 * i] = row; h_seg[4 * i + 1] = g.T; h_seg[4 * i + 2] = g.start_pos; h_seg[4 * i + 3] = bt_off;
        for (size_t p = 0; p < g.seq->block_table.size(); p++) h_bts[bt_off + p] = g.seq->block_table[p];
        for (int q = 0; q * qt < g.T; q++) tiles.push_back({i, q, g.start_pos + std::min(g.T, (q + 1) * qt) - 1});
        row += g.T;
        bt_off += (int)g.seq->block_table.size();
    }
    // query tiles by decreasing work (the last position a tile attends), stable
    std::stable_sort(tiles.begin(), tiles.end(), [](const Tile& x, const Tile& y) { return x.last > y.last; });
    for (int j = 0; j < n_tiles; j++) { h_tiles[2 * j] = tiles[j].seg; h_tiles[2 * j + 1] = tiles[j].qt; }
    d_tok_ = d_desc_; d_pos_ = d_desc_ + T; d_page_ = d_desc_ + 2 * T;
    d_seg_ = d_desc_ + 3 * T; d_tiles_ = d_seg_ + 4 * n; d_bt_ = d_desc_ + 3 * T + 4 * n + 2 * n_tiles;
    n_tiles_ = n_tiles;
    NR_CUDA(cudaMemcpyAsync(d_desc_, h_desc_, n_ints * 4, cudaMemcpyHostToDevice, stream_));
    last_valid_ = false;  // the descriptor no longer holds a decode step
    { ProfScope ps(this, kKEmbed); launch_embed(w_.emb, d_tok_, T, c.dim, d_x_, d_keys_, use_ss(T) ? d_ss_ : nullptr, max_rows_, stream_); }
    run_layers(T, true, nullptr, 0, 0, 0, false);
    d_seg_ = nullptr; d_tiles_ = nullptr; n_tiles_ = 0;
    if (n_emit > 0) {
        // the emitting chunks' last rows, gathered, through the classifier (:553-556)
        int k = 0;
        row = 0;
        for (int i = 0; i < n; i++) {
            row += segs[i].T;
            if (!segs[i].emit) continue;
            NR_CUDA(cudaMemcpyAsync(d_att_ + (size_t)k * c.dim, d_x_ + (size_t)(row - 1) * c.dim, (size_t)c.dim * 4,
                                    cudaMemcpyDeviceToDevice, stream_));
            k++;
        }
        GemmArgs gl;
        gl.err = d_err_;
        gl.x = d_att_; gl.ldx = c.dim; gl.norm_gain = w_.rms_final; gl.wf = w_.emb;
        gl.wt = w_.cls_t;
        gl.M = n_emit; gl.N = c.vocab; gl.K = c.dim;
        Epilogue el;
        el.kind = kEpiLogits; el.out = logits_out ? d_logits_ : nullptr; el.ldo = c.vocab; el.argmax_keys = d_keys_;
        { ProfScope ps(this, kKLogits); launch_gemm(gl, el, stream_); }
        { ProfScope ps(this, kKArgmax); launch_argmax_finish(d_keys_, n_emit, d_argmax_, stream_); }
    }
    NR_CUDA(cudaMemcpyAsync(h_argmax_, d_err_, (size_t)(n_emit + 1) * 4, cudaMemcpyDeviceToHost, stream_));
    if (logits_out && n_emit > 0)
        NR_CUDA(cudaMemcpyAsync(logits_out, d_logits_, (size_t)n_emit * c.vocab * 4, cudaMemcpyDeviceToHost, stream_));
    NR_CUDA(cudaStreamSynchronize(stream_));
    NR_CUDA(cudaGetLastError());
    if (h_argmax_[0] != 0) return fail(NR_ERR_TIMEOUT, "device wait timed out");
    if (argmax_out) memcpy(argmax_out, h_argmax_ + 1, (size_t)n_emit * 4);
    stats.prefill_tokens += T;
    if (profiling_) return prof_flush();
    return NR_OK;
}

int Engine::forward_decode(int B, const int* tokens, const int* positions, const Sequence* const* seqs,
                           float* logits_out, int* argmax_out, bool force_fixed) {
    if (!has_device()) return fail(NR_ERR_NO_DEVICE, "host-only engine");
    const ModelShape& c = shape_;
    if (B <= 0) return fail(NR_ERR_INVALID, "empty decode batch");
    if (B > cfg_.max_batch) return fail(NR_ERR_CAPACITY, "decode batch exceeds max_batch");
    const int MP = c.max_pages();
    int max_ctx = 0;
    for (int b = 0; b < B; b++) {
        const int pos = positions[b];
        if (pos < 0 || pos >= c.seq_len) return fail(NR_ERR_INVALID, "position outside [0, seq_len)");
        if (tokens[b] < 0 || tokens[b] >= c.vocab) return fail(NR_ERR_INVALID, "token id out of range");
        if (pos / kBlockSize >= (int)seqs[b]->block_table.size())
            return fail(NR_ERR_INVALID, "block table does not cover the position");
        max_ctx = std::max(max_ctx, pos + 1);
    }
    NR_CUDA(cudaSetDevice(cfg_.device));
    // descriptor: tok[B] pos[B] page[B] ctx[B] bt[B][MP]
    int* h = h_desc_;
    h_tok_ = h; h_pos_ = h + B; h_page_ = h + 2 * B; h_ctx_ = h + 3 * B; h_bt_ = h + 4 * B;
    for (int b = 0; b < B; b++) {
        const int pos = positions[b];
        const std::vector<int>& bt = seqs[b]->block_table;
        h_tok_[b] = tokens[b];
        h_pos_[b] = pos;
        h_page_[b] = bt[pos / kBlockSize];
        h_ctx_[b] = pos + 1;
        const int used = pos / kBlockSize + 1;
        for (int p = 0; p < used; p++) h_bt_[(size_t)b * MP + p] = bt[p];
    }
    const size_t n_ints = (size_t)4 * B + (size_t)B * MP;
    d_tok_ = d_desc_; d_pos_ = d_desc_ + B; d_page_ = d_desc_ + 2 * B; d_ctx_ = d_desc_ + 3 * B;
    d_bt_ = d_desc_ + 4 * B;
    NR_CUDA(cudaMemcpyAsync(d_desc_, h_desc_, n_ints * 4, cudaMemcpyHostToDevice, stream_));
    {
        int rc = launch_decode_step(B, max_ctx, force_fixed, logits_out != nullptr);
        if (rc) return rc;
    }
    last_B_ = B; last_max_ctx_ = max_ctx; last_force_fixed_ = force_fixed; last_valid_ = true;
    last_logits_ = logits_out != nullptr;
    NR_CUDA(cudaMemcpyAsync(h_argmax_, d_err_, (size_t)(B + 1) * 4, cudaMemcpyDeviceToHost, stream_));
    if (logits_out)
        NR_CUDA(cudaMemcpyAsync(logits_out, d_logits_, (size_t)B * c.vocab * 4, cudaMemcpyDeviceToHost, stream_));
    NR_CUDA(cudaStreamSynchronize(stream_));
    NR_CUDA(cudaGetLastError());
    if (h_argmax_[0] != 0) return fail(NR_ERR_TIMEOUT, "device wait timed out");
    if (argmax_out) memcpy(argmax_out, h_argmax_ + 1, (size_t)B * 4);
    stats.decode_tokens += B;
    if (profiling_) return prof_flush();
    return NR_OK;
}

void Engine::enqueue_decode(int B, int max_ctx, bool force_fixed, bool want_logits) {
    const ModelShape& c = shape_;
    d_tok_ = d_desc_; d_pos_ = d_desc_ + B; d_page_ = d_desc_ + 2 * B; d_ctx_ = d_desc_ + 3 * B;
    d_bt_ = d_desc_ + 4 * B;
    { ProfScope ps(this, kKEmbed); launch_embed(w_.emb, d_tok_, B, c.dim, d_x_, d_keys_, use_ss(B) ? d_ss_ : nullptr, max_rows_, stream_); }
    run_layers(B, false, nullptr, 0, B, max_ctx, force_fixed);
    GemmArgs gl;
    gl.err = d_err_;
    gl.x = d_x_; gl.ldx = c.dim; gl.norm_gain = w_.rms_final; gl.wf = w_.emb;
    gl.wt = w_.cls_t;
    gl.M = B; gl.N = c.vocab; gl.K = c.dim;
    if (use_ss(B)) { gl.ss_in = d_ss_; gl.ss_parts = (c.dim + 127) / 128; gl.ss_ld = max_rows_; }
    Epilogue el;
    el.kind = kEpiLogits; el.out = want_logits ? d_logits_ : nullptr; el.ldo = c.vocab; el.argmax_keys = d_keys_;
    { ProfScope ps(this, kKLogits); launch_gemm(gl, el, stream_); }
    { ProfScope ps(this, kKArgmax); launch_argmax_finish(d_keys_, B, d_argmax_, stream_); }
}

static bool graphs_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* env = getenv("NITRO_GRAPHS");
        v = (env && env[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

// Run one decode step's kernels: eagerly, or as a CUDA graph once the step shape has been
// seen before (graph replay removes the per-kernel launch work; the kernels' programmatic
// dependencies are kept as graph edges).
int Engine::launch_decode_step(int B, int max_ctx, bool force_fixed, bool want_logits) {
    if (profiling_ || !graphs_enabled()) {
        enqueue_decode(B, max_ctx, force_fixed, want_logits);
        return NR_OK;
    }
    GraphEntry& g = graphs_[std::make_tuple(B, force_fixed, want_logits)];
    if (!g.exec && g.seen++ == 0) {
        enqueue_decode(B, max_ctx, force_fixed, want_logits);
        return NR_OK;
    }
    if (!g.exec) {
        cudaGraph_t graph = nullptr;
        NR_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
        const int64_t before = kernel_launch_count();
        enqueue_decode(B, max_ctx, force_fixed, want_logits);
        const cudaError_t cap = cudaStreamEndCapture(stream_, &graph);
        if (cap != cudaSuccess) {
            cudaGetLastError();
            return fail(NR_ERR_CUDA, std::string("decode graph capture: ") + cudaGetErrorString(cap));
        }
        g.kernels = kernel_launch_count() - before;
        const cudaError_t inst = cudaGraphInstantiate(&g.exec, graph, 0);
        cudaGraphDestroy(graph);
        if (inst != cudaSuccess) {
            g.exec = nullptr;
            return fail(NR_ERR_CUDA, std::string("decode graph instantiate: ") + cudaGetErrorString(inst));
        }
    }
    NR_CUDA(cudaGraphLaunch(g.exec, stream_));
    for (int64_t i = 0; i < g.kernels; i++) count_launch();
    return NR_OK;
}

int Engine::replay_decode(int n) {
    if (!has_device()) return fail(NR_ERR_NO_DEVICE, "host-only engine");
    if (!last_valid_) return fail(NR_ERR_INVALID, "no decode step to replay");
    NR_CUDA(cudaSetDevice(cfg_.device));
    for (int i = 0; i < n; i++) {
        {
            int rc = launch_decode_step(last_B_, last_max_ctx_, last_force_fixed_, last_logits_);
            if (rc) return rc;
        }
        if (profiling_ && ev_used_ + 512 > ev_pool_.size()) {
            int rc = prof_flush();
            if (rc) return rc;
        }
    }
    NR_CUDA(cudaGetLastError());
    return NR_OK;
}

int Engine::replay_decode_attention(int n, bool with_merge) {
    if (!has_device()) return fail(NR_ERR_NO_DEVICE, "host-only engine");
    if (!last_valid_) return fail(NR_ERR_INVALID, "no decode step to replay");
    NR_CUDA(cudaSetDevice(cfg_.device));
    for (int i = 0; i < n; i++) {
        for (int l = 0; l < shape_.n_layers; l++) {
            const DecodeAttnArgs pa = decode_attn_plan(l, last_B_, last_max_ctx_);
            launch_decode_attention_main(pa, stream_);
            if (with_merge) launch_decode_merge(pa, stream_);
        }
    }
    NR_CUDA(cudaGetLastError());
    return NR_OK;
}

int Engine::last_decode_outputs(int* argmax_out, float* logits_out, int* B_out) {
    if (!has_device()) return fail(NR_ERR_NO_DEVICE, "host-only engine");
    if (!last_valid_) return fail(NR_ERR_INVALID, "no decode step ran");
    if (logits_out && !last_logits_) return fail(NR_ERR_INVALID, "the last decode step computed no logits");
    NR_CUDA(cudaSetDevice(cfg_.device));
    NR_CUDA(cudaMemcpyAsync(h_argmax_, d_err_, (size_t)(last_B_ + 1) * 4, cudaMemcpyDeviceToHost, stream_));
    if (logits_out)
        NR_CUDA(cudaMemcpyAsync(logits_out, d_logits_, (size_t)last_B_ * shape_.vocab * 4, cudaMemcpyDeviceToHost,
                                stream_));
    NR_CUDA(cudaStreamSynchronize(stream_));
    if (h_argmax_[0] != 0) return fail(NR_ERR_TIMEOUT, "device wait timed out");
    if (argmax_out) memcpy(argmax_out, h_argmax_ + 1, (size_t)last_B_ * 4);
    if (B_out) *B_out = last_B_;
    return NR_OK;
}

// ------------------------------------------------------------------ profiling
int Engine::set_profiling(bool on) {
    if (!has_device()) return fail(NR_ERR_NO_DEVICE, "host-only engine");
    NR_CUDA(cudaSetDevice(cfg_.device));
    if (on && ev_pool_.empty()) {
        ev_pool_.resize(8192);
        for (auto& ev : ev_pool_) NR_CUDA(cudaEventCreate(&ev));
    }
    if (on) {
        for (int i = 0; i < kKClasses; i++) { kt_ms_[i] = 0; kt_n_[i] = 0; }
        ev_used_ = 0;
        ev_pairs_.clear();
    } else if (profiling_) {
        int rc = prof_flush();
        if (rc) return rc;
    }
    profiling_ = on;
    return NR_OK;
}

void Engine::prof_mark(int cls, bool begin) {
    if (!profiling_ || ev_used_ + 2 > ev_pool_.size()) return;
    if (begin) {
        open_cls_ = cls;
        ev_pairs_.push_back({(int)ev_used_, cls});
        cudaEventRecord(ev_pool_[ev_used_++], stream_);
    } else {
        cudaEventRecord(ev_pool_[ev_used_++], stream_);
        open_cls_ = -1;
    }
}

int Engine::prof_flush() {
    if (ev_pairs_.empty()) return NR_OK;
    NR_CUDA(cudaStreamSynchronize(stream_));
    for (auto& pr : ev_pairs_) {
        float ms = 0.0f;
        NR_CUDA(cudaEventElapsedTime(&ms, ev_pool_[pr.first], ev_pool_[pr.first + 1]));
        kt_ms_[pr.second] += ms;
        kt_n_[pr.second] += 1;
    }
    ev_pairs_.clear();
    ev_used_ = 0;
    return NR_OK;
}

int Engine::kernel_times(double* ms, int64_t* launches) {
    if (profiling_) {
        int rc = prof_flush();
        if (rc) return rc;
    }
    for (int i = 0; i < kKClasses; i++) {
        if (ms) ms[i] = kt_ms_[i];
        if (launches) launches[i] = kt_n_[i];
    }
    return NR_OK;
}

int Engine::read_page(int block, float* k_out, float* v_out) {
    if (!has_device()) return fail(NR_ERR_NO_DEVICE, "host-only engine");
    if (block < 0 || block >= cfg_.total_blocks) return fail(NR_ERR_INVALID, "block id out of range");
    const ModelShape& c = shape_;
    const int hd = c.head_dim(), KV = c.kv_dim();
    const size_t pf = (size_t)geom_.page_floats(), lf = (size_t)geom_.layer_floats();
    const size_t eb = (size_t)geom_.elem_bytes();
    std::vector<float> tmp(pf);
    std::vector<uint16_t> raw16(geom_.kv_bf16 ? pf : 0);
    NR_CUDA(cudaSetDevice(cfg_.device));
    for (int which = 0; which < 2; which++) {
        float* dst = which == 0 ? k_out : v_out;
        if (!dst) continue;
        const uint8_t* pool = reinterpret_cast<const uint8_t*>(which == 0 ? kpool_ : vpool_);
        uint8_t* host = geom_.kv_bf16 ? reinterpret_cast<uint8_t*>(raw16.data()) : reinterpret_cast<uint8_t*>(tmp.data());
        for (int l = 0; l < c.n_layers; l++)  // the page's tiles of layer l: lf contiguous elements
            NR_CUDA(cudaMemcpyAsync(host + (size_t)l * lf * eb, pool + (size_t)geom_.tile_offset(block, l, 0) * eb,
                                    lf * eb, cudaMemcpyDeviceToHost, stream_));
        NR_CUDA(cudaStreamSynchronize(stream_));
        if (geom_.kv_bf16)  // bf16 is the upper half of an fp32
            for (size_t i = 0; i < pf; i++) {
                const uint32_t u = (uint32_t)raw16[i] << 16;
                memcpy(&tmp[i], &u, 4);
            }
        // [layer][kv_head][16][hd] -> [layer][16][kv_dim]
        for (int l = 0; l < c.n_layers; l++)
            for (int h = 0; h < c.n_kv_heads; h++)
                for (int r = 0; r < kBlockSize; r++)
                    memcpy(dst + ((size_t)l * kBlockSize + r) * KV + (size_t)h * hd,
                           tmp.data() + (((size_t)l * c.n_kv_heads + h) * kBlockSize + r) * hd, (size_t)hd * 4);
    }
    return NR_OK;
}

}  // namespace nitro
