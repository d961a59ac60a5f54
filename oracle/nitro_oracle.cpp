// Test infrastructure only (the checker, never the product).
//
// A plain, scalar CPU restatement of the reference's Q8_0 inference arithmetic
// (nvivek17/NitroRAG, src/model_q8.cpp and scripts/quantize.py), written from the
// reference's behaviour, one function per reference routine, each citing the lines it
// follows.  It is pinned against the reference itself: tests/golden holds outputs of
// the reference code compiled from its own sources (oracle/ref_harness.cpp), and the
// not-gpu tests check every function here against those fixtures.
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this
// library.  The engine never calls it.
//
// Q8 "modes": the reference's batched Q8 matmul (src/model_q8.cpp:382-420) assigns
// instead of accumulating at :416, so it returns the dot product of the LAST 32-wide
// K-block only.  `last_block_only = 1` reproduces that ("faithful"); 0 sums all blocks
// like the single-token matmul at :92-125 ("fixed").
#include <cstdint>
#include <cstring>
#include <cmath>
#include <climits>
#include <vector>
#include <cstdio>
#include <cstdlib>

namespace {

constexpr int QB = 32;        // Q_BLOCK_SIZE, src/model_q8.cpp:28
constexpr int PAGE = 16;      // BLOCK_SIZE, src/pagedMemory.hpp:9

struct Cfg { int dim, hidden, n_layers, n_heads, n_kv_heads, vocab, seq_len; };

// One Q8_0 block as stored in the file: fp32 scale then 32 int8 (src/model_q8.cpp:29-32).
inline float blk_scale(const uint8_t* w, int64_t blk) { float s; memcpy(&s, w + blk * 36, 4); return s; }
inline int8_t blk_q(const uint8_t* w, int64_t blk, int k) { return (int8_t)w[blk * 36 + 4 + k]; }

}  // namespace

extern "C" {

// scripts/quantize.py:7-23: per 32 weights scale = absmax/127 (fp32), 1e-9 for an
// all-zero block; q = round-half-even(w/scale) clamped to [-128,127].  The last block
// of a tensor whose length is not a multiple of 32 is shorter (quantize.py:10-11): its
// scale and its len q bytes follow the full blocks.
void orc_quantize_q8(const float* w, int64_t n, uint8_t* out) {
    for (int64_t b = 0; b * QB < n; b++) {
        const float* blk = w + b * QB;
        const int len = n - b * QB < QB ? (int)(n - b * QB) : QB;
        float amax = 0.0f;
        for (int k = 0; k < len; k++) amax = fmaxf(amax, fabsf(blk[k]));
        float scale = amax != 0.0f ? amax / 127.0f : 1e-9f;
        uint8_t* o = out + b * 36;
        memcpy(o, &scale, 4);
        for (int k = 0; k < len; k++) {
            float r = nearbyintf(blk[k] / scale);   // default rounding mode: half to even
            int q = (int)r;
            q = q < -128 ? -128 : (q > 127 ? 127 : q);
            o[4 + k] = (uint8_t)(int8_t)q;
        }
    }
}

// out[b*d+i] = sum_k x[b*n+k] * (q[i,k]*scale[i,k/32])
// src/model_q8.cpp:92-125 (all blocks) or :382-420 (last block only).
void orc_q8_matmul(float* out, const float* x, const uint8_t* w, int B, int n, int d, int last_block_only) {
    int nb = n / QB;
    for (int b = 0; b < B; b++) {
        for (int i = 0; i < d; i++) {
            float acc = 0.0f;
            int first = last_block_only ? nb - 1 : 0;
            for (int blk = first; blk < nb; blk++) {
                int64_t id = (int64_t)i * nb + blk;
                float s = blk_scale(w, id);
                float part = 0.0f;
                for (int k = 0; k < QB; k++) part += ((float)blk_q(w, id, k) * s) * x[(int64_t)b * n + blk * QB + k];
                acc += part;
            }
            out[(int64_t)b * d + i] = acc;
        }
    }
}

// src/model_q8.cpp:370-381: fp32 out[b*d+i] = sum_j x[b*n+j]*w[i*n+j].
void orc_f32_matmul(float* out, const float* x, const float* w, int B, int n, int d) {
    for (int b = 0; b < B; b++)
        for (int i = 0; i < d; i++) {
            float acc = 0.0f;
            for (int j = 0; j < n; j++) acc += x[(int64_t)b * n + j] * w[(int64_t)i * n + j];
            out[(int64_t)b * d + i] = acc;
        }
}

// src/model_q8.cpp:128-140: out = g * (x / sqrt(mean(x^2) + 1e-5)).
void orc_rms_norm(float* out, const float* x, const float* g, int n) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    ss /= n;
    ss += 1e-5f;
    ss = 1.0f / sqrtf(ss);
    for (int i = 0; i < n; i++) out[i] = g[i] * (ss * x[i]);
}

// src/model_q8.cpp:142-159: max starts at (float)INT32_MIN, exp pass, divide pass.
void orc_softmax(float* x, int n) {
    float mx = (float)INT32_MIN;
    for (int i = 0; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

// src/model_q8.cpp:559-569: first index whose value is strictly greater than the
// running max, which starts at 0.0f with index 0.
int orc_argmax(const float* x, int n) {
    int idx = 0;
    float mx = 0.0f;
    for (int i = 0; i < n; i++) if (x[i] > mx) { mx = x[i]; idx = i; }
    return idx;
}

// src/pagedMemory.hpp:11-24: FNV-1a 64 over each token's 4 little-endian bytes,
// chained from the parent hash.
uint64_t orc_fnv_block_hash(uint64_t parent, const int32_t* tok, int n) {
    uint64_t h = parent;
    for (int t = 0; t < n; t++) {
        uint32_t u = (uint32_t)tok[t];
        for (int k = 0; k < 4; k++) { h ^= (u >> (8 * k)) & 0xffu; h *= 1099511628211ULL; }
    }
    return h;
}

// RoPE on one token's q (dim) and k (kv_dim), src/model_q8.cpp:601-615 (decode) and
// :457-471 (prefill): pairs (j, j+1), angle index (j % head)/2 at row `pos`.
void orc_rope(float* q, float* k, int dim, int kv_dim, int head, int pos, const float* fr, const float* fi) {
    for (int j = 0; j < dim; j += 2) {
        int hd = j % head;
        float c = fr[pos * (head / 2) + hd / 2];
        float s = fi[pos * (head / 2) + hd / 2];
        float q0 = q[j], q1 = q[j + 1];
        q[j] = q0 * c - q1 * s;
        q[j + 1] = q0 * s + q1 * c;
        if (j < kv_dim) {
            float k0 = k[j], k1 = k[j + 1];
            k[j] = k0 * c - k1 * s;
            k[j + 1] = k0 * s + k1 * c;
        }
    }
}

// Decode paged attention for one layer, src/model_q8.cpp:625-662 with softmax :142-159.
// Pool layout as in the reference: page p holds rows [16][kv_dim] for this layer at
// p*page_stride + layer_off.  ctx[b] = pos_b + 1 tokens are read through bt[b*max_pages..].
void orc_paged_decode_attention(float* out, const float* q, const float* kpool, const float* vpool,
                                int64_t page_stride, int64_t layer_off, const int32_t* bt, int max_pages,
                                const int32_t* ctx, int B, int n_heads, int n_kv_heads, int head) {
    int kv_dim = n_kv_heads * head;
    int kv_mul = n_heads / n_kv_heads;
    std::vector<float> att;
    for (int b = 0; b < B; b++) {
        int n = ctx[b];
        att.assign(n, 0.0f);
        for (int h = 0; h < n_heads; h++) {
            const float* qh = q + (int64_t)b * n_heads * head + h * head;
            int kvh = h / kv_mul;
            for (int t = 0; t < n; t++) {
                int pg = bt[(int64_t)b * max_pages + t / PAGE];
                const float* kr = kpool + pg * page_stride + layer_off + (int64_t)(t % PAGE) * kv_dim + kvh * head;
                float sc = 0.0f;
                for (int p = 0; p < head; p++) sc += qh[p] * kr[p];
                att[t] = sc / sqrtf((float)head);
            }
            orc_softmax(att.data(), n);
            float* o = out + (int64_t)b * n_heads * head + h * head;
            for (int p = 0; p < head; p++) o[p] = 0.0f;
            for (int t = 0; t < n; t++) {
                int pg = bt[(int64_t)b * max_pages + t / PAGE];
                const float* vr = vpool + pg * page_stride + layer_off + (int64_t)(t % PAGE) * kv_dim + kvh * head;
                for (int p = 0; p < head; p++) o[p] += att[t] * vr[p];
            }
        }
    }
}

// Causal prefill attention for T query rows at positions start_pos..start_pos+T-1 of one
// sequence, src/model_q8.cpp:485-523: single-pass online softmax with m = -1e9.
void orc_paged_prefill_attention(float* out, const float* q, const float* kpool, const float* vpool,
                                 int64_t page_stride, int64_t layer_off, const int32_t* bt,
                                 int T, int start_pos, int n_heads, int n_kv_heads, int head) {
    int kv_dim = n_kv_heads * head;
    int kv_mul = n_heads / n_kv_heads;
    for (int t = 0; t < T; t++) {
        int pos = start_pos + t;
        for (int h = 0; h < n_heads; h++) {
            const float* qh = q + (int64_t)t * n_heads * head + h * head;
            float* o = out + (int64_t)t * n_heads * head + h * head;
            int kvh = h / kv_mul;
            for (int p = 0; p < head; p++) o[p] = 0.0f;
            float m = -1e9f, dsum = 0.0f;
            for (int u = 0; u <= pos; u++) {
                int pg = bt[u / PAGE];
                int64_t row = pg * page_stride + layer_off + (int64_t)(u % PAGE) * kv_dim + kvh * head;
                float sc = 0.0f;
                for (int p = 0; p < head; p++) sc += qh[p] * kpool[row + p];
                sc /= sqrtf((float)head);
                if (sc > m) {
                    float corr = expf(m - sc);
                    for (int p = 0; p < head; p++) o[p] *= corr;
                    dsum *= corr;
                    m = sc;
                }
                float e = expf(sc - m);
                dsum += e;
                for (int p = 0; p < head; p++) o[p] += e * vpool[row + p];
            }
            for (int p = 0; p < head; p++) o[p] /= dsum;
        }
    }
}

// ------------------------------------------------------------------ whole model
// A model file in the reference format (header of 7 int32 then tensors in the order
// of src/Server_Inference.cpp:53-69) and a KV pool in the reference page layout
// [page][layer][16][kv_dim] (src/pagedMemory.hpp:86-106).  Block tables are supplied by
// the caller: this restatement has no allocator of its own.

struct OrcModel {
    Cfg c;
    std::vector<uint8_t> bytes;
    const float *emb, *rms_att, *rms_ffn, *rms_final, *fr, *fi;
    const uint8_t *wq, *wk, *wv, *wo, *w1, *w2, *w3;
    std::vector<float> kpool, vpool;
    int64_t page_floats;
    int total_pages;
    int kv_bf16 = 0;  // pages hold K/V rounded to bf16 (the engine's NR_KV_BF16 option)
};

// Round to the nearest bf16 (8 significant bits), ties to even, kept as fp32: IEEE
// round-to-nearest-even on the upper 16 bits of the fp32 pattern (finite values).
static float round_bf16(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    u &= 0xFFFF0000u;
    memcpy(&v, &u, 4);
    return v;
}

void* orc_model_open(const char* path, int total_pages) {
    FILE* f = fopen(path, "rb");
    if (!f) return nullptr;
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    OrcModel* m = new OrcModel();
    m->bytes.resize(sz);
    if (fread(m->bytes.data(), 1, sz, f) != (size_t)sz) { fclose(f); delete m; return nullptr; }
    fclose(f);
    const int32_t* h = (const int32_t*)m->bytes.data();
    m->c = Cfg{h[0], h[1], h[2], h[3], h[4], h[5], h[6]};
    const Cfg& c = m->c;
    int head = c.dim / c.n_heads, kv_dim = c.n_kv_heads * head;
    const uint8_t* p = m->bytes.data() + 28;
    auto take = [&](int64_t bytes) { const uint8_t* r = p; p += bytes; return r; };
    auto q8 = [](int64_t n) { return n / QB * 36; };
    m->emb = (const float*)take((int64_t)c.vocab * c.dim * 4);
    m->rms_att = (const float*)take((int64_t)c.n_layers * c.dim * 4);
    m->wq = take(q8((int64_t)c.n_layers * c.dim * c.dim));
    m->wk = take(q8((int64_t)c.n_layers * c.dim * kv_dim));
    m->wv = take(q8((int64_t)c.n_layers * c.dim * kv_dim));
    m->wo = take(q8((int64_t)c.n_layers * c.dim * c.dim));
    m->rms_ffn = (const float*)take((int64_t)c.n_layers * c.dim * 4);
    m->w1 = take(q8((int64_t)c.n_layers * c.hidden * c.dim));
    m->w2 = take(q8((int64_t)c.n_layers * c.dim * c.hidden));
    m->w3 = take(q8((int64_t)c.n_layers * c.hidden * c.dim));
    m->rms_final = (const float*)take((int64_t)c.dim * 4);
    m->fr = (const float*)take((int64_t)c.seq_len * head / 2 * 4);
    m->fi = (const float*)take((int64_t)c.seq_len * head / 2 * 4);
    if (p - m->bytes.data() > sz) { delete m; return nullptr; }
    m->page_floats = (int64_t)c.n_layers * PAGE * kv_dim;
    m->total_pages = total_pages;
    m->kpool.assign((size_t)total_pages * m->page_floats, 0.0f);
    m->vpool.assign((size_t)total_pages * m->page_floats, 0.0f);
    return m;
}

void orc_model_close(void* h) { delete (OrcModel*)h; }

// Pages store K/V rounded to bf16 from now on (no reference counterpart: the reference's
// pages are fp32, src/pagedMemory.hpp:90-94).
void orc_model_set_kv_bf16(void* h, int on) { ((OrcModel*)h)->kv_bf16 = on != 0; }

int orc_model_page(void* h, int page, float* k_out, float* v_out) {
    OrcModel* m = (OrcModel*)h;
    if (page < 0 || page >= m->total_pages) return -1;
    if (k_out) memcpy(k_out, m->kpool.data() + page * m->page_floats, m->page_floats * 4);
    if (v_out) memcpy(v_out, m->vpool.data() + page * m->page_floats, m->page_floats * 4);
    return 0;
}

}  // extern "C"

namespace {

// One transformer block body shared by prefill and decode (src/model_q8.cpp:441-552 and
// :585-687).  Rows r = 0..R-1 each have a position pos[r] and a block table bt_row(r).
template <class BT, class ATT>
void run_layers(OrcModel* m, int R, const int* pos, BT bt_row, ATT attend, std::vector<float>& x, int lbo) {
    const Cfg& c = m->c;
    int head = c.dim / c.n_heads, kv_dim = c.n_kv_heads * head, D = c.dim, Hd = c.hidden;
    std::vector<float> xb((size_t)R * D), q((size_t)R * D), k((size_t)R * kv_dim), v((size_t)R * kv_dim);
    std::vector<float> att((size_t)R * D), tmp((size_t)R * D), h1((size_t)R * Hd), h3((size_t)R * Hd);
    for (int l = 0; l < c.n_layers; l++) {
        for (int r = 0; r < R; r++) orc_rms_norm(&xb[(size_t)r * D], &x[(size_t)r * D], m->rms_att + (int64_t)l * D, D);
        orc_q8_matmul(q.data(), xb.data(), m->wq + (int64_t)l * D * D / QB * 36, R, D, D, lbo);
        orc_q8_matmul(k.data(), xb.data(), m->wk + (int64_t)l * D * kv_dim / QB * 36, R, D, kv_dim, lbo);
        orc_q8_matmul(v.data(), xb.data(), m->wv + (int64_t)l * D * kv_dim / QB * 36, R, D, kv_dim, lbo);
        int64_t layer_off = (int64_t)l * PAGE * kv_dim;
        for (int r = 0; r < R; r++) {
            orc_rope(&q[(size_t)r * D], &k[(size_t)r * kv_dim], D, kv_dim, head, pos[r], m->fr, m->fi);
            // KV append, src/model_q8.cpp:475-484 / :616-623
            const int32_t* bt = bt_row(r);
            int pg = bt[pos[r] / PAGE];
            int64_t off = pg * m->page_floats + layer_off + (int64_t)(pos[r] % PAGE) * kv_dim;
            memcpy(&m->kpool[off], &k[(size_t)r * kv_dim], kv_dim * 4);
            memcpy(&m->vpool[off], &v[(size_t)r * kv_dim], kv_dim * 4);
            if (m->kv_bf16)
                for (int i = 0; i < kv_dim; i++) {
                    m->kpool[off + i] = round_bf16(m->kpool[off + i]);
                    m->vpool[off + i] = round_bf16(m->vpool[off + i]);
                }
        }
        attend(q.data(), att.data(), layer_off);
        orc_q8_matmul(tmp.data(), att.data(), m->wo + (int64_t)l * D * D / QB * 36, R, D, D, lbo);
        for (size_t i = 0; i < (size_t)R * D; i++) x[i] += tmp[i];
        for (int r = 0; r < R; r++) orc_rms_norm(&xb[(size_t)r * D], &x[(size_t)r * D], m->rms_ffn + (int64_t)l * D, D);
        orc_q8_matmul(h1.data(), xb.data(), m->w1 + (int64_t)l * Hd * D / QB * 36, R, D, Hd, lbo);
        orc_q8_matmul(h3.data(), xb.data(), m->w3 + (int64_t)l * Hd * D / QB * 36, R, D, Hd, lbo);
        // SwiGLU, src/model_q8.cpp:535-545 / :672-681
        for (size_t i = 0; i < (size_t)R * Hd; i++) {
            float val = h1[i];
            val *= (1.0f / (1.0f + expf(-val)));
            h1[i] = val * h3[i];
        }
        orc_q8_matmul(tmp.data(), h1.data(), m->w2 + (int64_t)l * D * Hd / QB * 36, R, Hd, D, lbo);
        for (size_t i = 0; i < (size_t)R * D; i++) x[i] += tmp[i];
    }
}

}  // namespace

extern "C" {

// forward_prefill_chunk, src/model_q8.cpp:424-557 (minus the allocator calls at :428-430):
// T tokens at positions start_pos.., K/V written through block table bt, logits of the
// last token.
int orc_forward_prefill(void* h, const int32_t* bt, const int32_t* tokens, int T, int start_pos,
                        float* logits, int last_block_only) {
    OrcModel* m = (OrcModel*)h;
    const Cfg& c = m->c;
    if (T <= 0) return -1;
    int D = c.dim, head = D / c.n_heads;
    std::vector<float> x((size_t)T * D);
    std::vector<int> pos(T);
    for (int t = 0; t < T; t++) {
        memcpy(&x[(size_t)t * D], m->emb + (int64_t)tokens[t] * D, D * 4);
        pos[t] = start_pos + t;
    }
    auto bt_row = [&](int) { return bt; };
    auto attend = [&](const float* q, float* out, int64_t layer_off) {
        orc_paged_prefill_attention(out, q, m->kpool.data(), m->vpool.data(), m->page_floats, layer_off, bt,
                                    T, start_pos, c.n_heads, c.n_kv_heads, head);
    };
    run_layers(m, T, pos.data(), bt_row, attend, x, last_block_only);
    std::vector<float> xn(D);
    orc_rms_norm(xn.data(), &x[(size_t)(T - 1) * D], m->rms_final, D);
    orc_f32_matmul(logits, xn.data(), m->emb, 1, D, c.vocab);
    return 0;
}

// forward_decode_batch, src/model_q8.cpp:571-694 (minus the allocator calls at :578-582):
// one token per row b at position positions[b], block tables bt[b*max_pages..], B x vocab logits.
int orc_forward_decode(void* h, const int32_t* bt, int max_pages, int B, const int32_t* tokens,
                       const int32_t* positions, float* logits, int last_block_only) {
    OrcModel* m = (OrcModel*)h;
    const Cfg& c = m->c;
    if (B <= 0) return -1;
    int D = c.dim, head = D / c.n_heads;
    std::vector<float> x((size_t)B * D);
    std::vector<int> ctx(B);
    for (int b = 0; b < B; b++) {
        memcpy(&x[(size_t)b * D], m->emb + (int64_t)tokens[b] * D, D * 4);
        ctx[b] = positions[b] + 1;
    }
    auto bt_row = [&](int r) { return bt + (int64_t)r * max_pages; };
    auto attend = [&](const float* q, float* out, int64_t layer_off) {
        orc_paged_decode_attention(out, q, m->kpool.data(), m->vpool.data(), m->page_floats, layer_off, bt,
                                   max_pages, ctx.data(), B, c.n_heads, c.n_kv_heads, head);
    };
    run_layers(m, B, positions, bt_row, attend, x, last_block_only);
    std::vector<float> xn((size_t)B * D);
    for (int b = 0; b < B; b++) orc_rms_norm(&xn[(size_t)b * D], &x[(size_t)b * D], m->rms_final, D);
    orc_f32_matmul(logits, xn.data(), m->emb, B, D, c.vocab);
    return 0;
}

}  // extern "C"
