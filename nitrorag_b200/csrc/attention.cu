// Paged attention over the fp32 KV pools, decode and causal prefill.
//
// The pools are laid out [layer][page][kv_head][16][head_dim] in the engine and
// [page][layer][kv_head][16][head_dim] for the standalone entry points (PoolGeom), so one
// (page, layer, kv_head) is a contiguous 16 x head_dim tile (4 KB at head_dim 64).  Every
// tile a CTA needs is fetched with one bulk asynchronous copy (cp.async.bulk, the TMA
// engine's non-tensor form) into shared memory and signalled on an mbarrier, so the SMs
// issue a handful of instructions per 4 KB and keep many tiles in flight.
//
// Scores and the softmax are fp32.  Inside a warp two lanes share one key row (each takes
// half of head_dim; their partial dots are joined with one shuffle), the 16 keys of a page
// are processed at once, and the softmax is the online (running max / running sum) form
// in the exp2 domain.  The reference computes decode scores, then a two-pass softmax
// (src/model_q8.cpp:625-662, :142-159), and prefill with a single-pass online softmax
// (:485-523); both equal softmax(q.k/sqrt(head)) . V up to fp32 rounding.
//
// Decode work is split ("flash-decoding"): a persistent kernel streams (sequence, head,
// chunk of up to chunk_pages pages) items through per-warp bulk-copy rings; an item that
// covers a whole context writes its output, the others write their partial (max, sum,
// unnormalised output) and a small merge kernel, chained behind it with programmatic
// dependent launch, combines them.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace nitro {

namespace {

constexpr int kAttnWarps = 4;


constexpr float kLog2e = 1.4426950408889634f;

// Running softmax state of one query inside a warp.  Lane l owns output dims
// [l*DPL, l*DPL + DPL) with DPL = head_dim / 32.
template <int HD>
struct QState {
    static constexpr int DPL = HD / 32;
    float m;  // running max (log2 domain)
    float l;  // running sum of exp2(s - m)
    float o[DPL];
    __device__ void init() {
        m = -INFINITY;
        l = 0.0f;
#pragma unroll
        for (int i = 0; i < DPL; i++) o[i] = 0.0f;
    }
};

// The lane's half of the query (pre-scaled, in shared memory at qs) as attend_page reads
// it, in registers: float4 j of the lane's half is float4 (j + lane) mod HD/8 of it.
template <int HD>
__device__ __forceinline__ void load_query(float4* qr, const float* qs, int lane) {
    constexpr int HALF4 = HD / 8;
    const float4* qrow = reinterpret_cast<const float4*>(qs + (lane & 1) * (HD / 2));
#pragma unroll
    for (int j = 0; j < HALF4; j++) qr[j] = qrow[(j + lane) & (HALF4 - 1)];
}

// Fold the 16 rows of one K/V page tile (in shared memory) into a query's state.
// qr: the query from load_query (pre-scaled by log2(e)/sqrt(head_dim)); pbuf: 16 floats of
// this warp's shared memory for the page's probabilities (free again once the caller's
// __syncwarp after the page has passed); n_valid: how many leading rows of the page are
// attended (1..16).
template <int HD, typename KT>
__device__ __forceinline__ void attend_page(QState<HD>& st, const float4* qr, float* pbuf, const KT* Kt,
                                            const KT* Vt, int n_valid, int lane) {
    constexpr int HALF4 = HD / 8;  // groups of 4 values per half row
    const int t = lane >> 1, half = lane & 1;
    const KT* krow = Kt + t * HD + half * (HD / 2);
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;  // four short FMA chains
#pragma unroll
    for (int j = 0; j < HALF4; j++) {
        // rotate the float4 index with the lane so the 8 lanes of each shared-memory
        // phase hit 8 different bank groups
        const int jj = (j + lane) & (HALF4 - 1);
        float4 kv = ldkv4(krow + 4 * jj);
        const float4 qv = qr[j];
        s0 = fmaf(qv.x, kv.x, s0);
        s1 = fmaf(qv.y, kv.y, s1);
        s2 = fmaf(qv.z, kv.z, s2);
        s3 = fmaf(qv.w, kv.w, s3);
    }
    float s = (s0 + s1) + (s2 + s3);
    s += __shfl_xor_sync(0xffffffffu, s, 1);  // both lanes of a key row hold its score
    if (t >= n_valid) s = -INFINITY;
    float mp = s;
#pragma unroll
    for (int o = 2; o < 32; o <<= 1) mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, o));
    const float m_new = fmaxf(st.m, mp);
    const float corr = exp2f(st.m - m_new);
    const float p = exp2f(s - m_new);
    if (half == 0) pbuf[t] = p;
    // the 16 lanes of one half hold the 16 keys' probabilities once each
    float ps = p;
#pragma unroll
    for (int o = 2; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    st.l = st.l * corr + ps;
    st.m = m_new;
#pragma unroll
    for (int i = 0; i < QState<HD>::DPL; i++) st.o[i] *= corr;
    __syncwarp();  // pbuf written
    const float4* pb = reinterpret_cast<const float4*>(pbuf);
    const KT* vbase = Vt + lane * QState<HD>::DPL;
#pragma unroll
    for (int t4 = 0; t4 < kPage / 4; t4++) {
        const float4 pp = pb[t4];  // broadcast read
        const float pv[4] = {pp.x, pp.y, pp.z, pp.w};
#pragma unroll
        for (int i4 = 0; i4 < 4; i4++) {
            const int tt = 4 * t4 + i4;
            const float pt = pv[i4];
            if (QState<HD>::DPL == 2) {
                float2 v = ldkv2(vbase + tt * HD);
                st.o[0] = fmaf(pt, v.x, st.o[0]);
                st.o[1] = fmaf(pt, v.y, st.o[1]);
            } else {
                float4 v = ldkv4(vbase + tt * HD);
                st.o[0] = fmaf(pt, v.x, st.o[0]);
                st.o[1] = fmaf(pt, v.y, st.o[1]);
                st.o[2] = fmaf(pt, v.z, st.o[2]);
                st.o[3] = fmaf(pt, v.w, st.o[3]);
            }
        }
    }
}

// ------------------------------------------------------------------ decode
// Persistent kernel, one CTA per SM, every warp an independent worker: it takes work items
// (sequence b, head h, chunk of up to chunk_pages pages) from a global counter and streams
// their K/V page tiles through its own ring of kDecStages shared-memory slots, issuing the
// next item's pages while the current item drains, so the copy engine always has pages
// in flight.  No CTA-wide barrier is taken after set-up.
#ifndef NITRO_DEC_STAGES
#define NITRO_DEC_STAGES 4
#endif
#ifndef NITRO_DEC_WARPS64
#define NITRO_DEC_WARPS64 6
#endif
#ifndef NITRO_DEC_CHUNK64
#define NITRO_DEC_CHUNK64 16
#endif
constexpr int kDecStages = NITRO_DEC_STAGES;

template <int HD, typename KT = float>
struct DecCfg {
    static constexpr int WARPS = HD == 64 ? NITRO_DEC_WARPS64 : NITRO_DEC_WARPS64 / 2;
    static constexpr int TILE = kPage * HD;                              // elements per K or V tile
    static constexpr int TILE_BYTES = TILE * (int)sizeof(KT);
    static constexpr int RING_BYTES = WARPS * kDecStages * 2 * TILE_BYTES;
    static constexpr int SMEM = RING_BYTES + WARPS * (HD + kPage) * 4;   // + a query and a page's p per warp
};

struct DecItem {
    int b, h, split, p0, np, ctx, nsplit;
    bool valid;
    int pid;       // lane i < np: physical page of the item's i-th page
    float q[4];    // lane l: query dims l + 32 j (pre-scaled), j < head_dim / 32
};

// Context length of row b clamped into [0, max_pages * 16] (what the block table can
// address); with `report`, a length outside [1, max_pages * 16] sets kErrBadContext.
__device__ __forceinline__ int checked_ctx(const DecodeAttnArgs& a, int b, bool report) {
    const int ctx = a.ctx_lens[b];
    const int cap = a.max_pages * kPage;
    if (report && (ctx < 1 || ctx > cap) && a.err) atomicCAS(a.err, 0, kErrBadContext);
    return min(max(ctx, 0), cap);
}

// Work items are numbered longest first: every full chunk (chunk_pages pages) of every
// (sequence, head) in sequence order, then the shorter last chunks, longest remainder
// first, so that the items still running when the counter runs dry are the short ones.
struct DecTable {
    int full_prefix[1025];  // full_prefix[b]: first full-chunk item of sequence b
    int tail_seq[1024];     // sequences with a shorter last chunk, longest remainder first
    int ctx[1024];
    int group_off[32][32];  // [32-sequence group][remainder]: count, then offset in bucket
    int bucket[33];         // [remainder]: first slot of the bucket; [0]: number of tails
    int warp_tot[32];
};

// Decode work item `idx` into its sequence / head / chunk, and prefetch everything its
// processing needs (page ids, query) so no dependent global load sits in front of the
// bulk copies later.
template <int HD>
__device__ __forceinline__ DecItem dec_item(int idx, int total, const DecTable& t, const DecodeAttnArgs& a, int lane,
                                            float qscale) {
    DecItem it;
    it.valid = idx < total;
    it.pid = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) it.q[j] = 0.0f;
    if (!it.valid) { it.b = it.h = it.split = it.p0 = it.np = it.ctx = it.nsplit = 0; return it; }
    const int total_full = t.full_prefix[a.B];
    int pages;
    if (idx < total_full) {
        int lo = 0, hi = a.B;  // largest b with full_prefix[b] <= idx
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (t.full_prefix[mid] <= idx) lo = mid; else hi = mid;
        }
        it.b = lo;
        const int rem = idx - t.full_prefix[lo];
        it.split = rem / a.n_heads;
        it.h = rem % a.n_heads;
        it.ctx = t.ctx[lo];
        pages = (it.ctx + kPage - 1) / kPage;
    } else {
        const int j = idx - total_full;
        it.b = t.tail_seq[j / a.n_heads];
        it.h = j % a.n_heads;
        it.ctx = t.ctx[it.b];
        pages = (it.ctx + kPage - 1) / kPage;
        it.split = pages / a.chunk_pages;
    }
    it.nsplit = (pages + a.chunk_pages - 1) / a.chunk_pages;
    it.p0 = it.split * a.chunk_pages;
    it.np = min(a.chunk_pages, pages - it.p0);
    if (lane < it.np) it.pid = a.block_tables[(int64_t)it.b * a.max_pages + it.p0 + lane];
    const float* qrow = a.q + ((int64_t)it.b * a.n_heads + it.h) * HD;
#pragma unroll
    for (int j = 0; j < HD / 32; j++) it.q[j] = qrow[lane + 32 * j] * qscale;
    return it;
}

template <int HD, typename KT>
__global__ void __launch_bounds__(DecCfg<HD>::WARPS * 32, 1) decode_attn_kernel(DecodeAttnArgs a) {
    using C = DecCfg<HD, KT>;
    constexpr int DPL = HD / 32;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const KT* kpool = reinterpret_cast<const KT*>(a.kpool);
    const KT* vpool = reinterpret_cast<const KT*>(a.vpool);
    __shared__ uint64_t bars[C::WARPS][kDecStages];
    __shared__ DecTable tab;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvmul = a.n_heads / a.geom.n_kv_heads;
    const int cp = a.chunk_pages;

    // item table from the step descriptor (written before this step's first kernel, so it
    // is read before waiting on the previous kernel).  Every CTA builds the same table, so
    // it must not depend on timing: the tail order is a stable counting sort.
    for (int i = threadIdx.x; i < 32 * 32; i += blockDim.x) (&tab.group_off[0][0])[i] = 0;
    for (int base = 0; base < a.B; base += blockDim.x) {
        const int b = base + threadIdx.x;
        int cnt = 0;
        if (b < a.B) {
            const int ctx = checked_ctx(a, b, blockIdx.x == 0);
            tab.ctx[b] = ctx;
            const int pages = (ctx + kPage - 1) / kPage;
            cnt = (pages / cp) * a.n_heads;
        }
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane == 31) tab.warp_tot[warp] = incl;
        __syncthreads();
        if (threadIdx.x == 0) {
            int run = base == 0 ? 0 : tab.full_prefix[base];
            for (int w = 0; w < C::WARPS; w++) {
                const int t = tab.warp_tot[w];
                tab.warp_tot[w] = run;
                run += t;
            }
            tab.full_prefix[min(base + (int)blockDim.x, a.B)] = run;
        }
        __syncthreads();
        if (b < a.B) tab.full_prefix[b] = tab.warp_tot[warp] + incl - cnt;
        __syncthreads();
    }
    // last chunks shorter than chunk_pages, bucketed by remainder (longest first), in
    // sequence order inside a bucket: per 32-sequence group, lanes with equal remainders
    // rank themselves by lane; group counts are then turned into offsets per bucket
    const int n_groups = (a.B + 31) / 32;
    auto tail_rem = [&](int b) {
        return b < a.B ? ((tab.ctx[b] + kPage - 1) / kPage) % cp : 0;
    };
    for (int g = warp; g < n_groups; g += C::WARPS) {
        const int r = tail_rem(g * 32 + lane);
        const unsigned same = __match_any_sync(0xffffffffu, r);
        if (r > 0 && lane == __ffs(same) - 1) tab.group_off[g][r] = __popc(same);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int r = threadIdx.x;
        int run = 0;
        for (int g = 0; g < n_groups; g++) {
            const int c = tab.group_off[g][r];
            tab.group_off[g][r] = run;
            run += c;
        }
        tab.bucket[r] = run;  // sequences with remainder r
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int r = cp - 1; r >= 1; r--) {
            const int c = tab.bucket[r];
            tab.bucket[r] = run;
            run += c;
        }
        tab.bucket[0] = run;
    }
    __syncthreads();
    for (int g = warp; g < n_groups; g += C::WARPS) {
        const int b = g * 32 + lane;
        const int r = tail_rem(b);
        const unsigned same = __match_any_sync(0xffffffffu, r);
        if (r > 0) tab.tail_seq[tab.bucket[r] + tab.group_off[g][r] + __popc(same & ((1u << lane) - 1u))] = b;
    }
    __syncthreads();
    const int total = tab.full_prefix[a.B] + tab.bucket[0] * a.n_heads;

    KT* ring = reinterpret_cast<KT*>(smem_raw + warp * kDecStages * 2 * C::TILE_BYTES);
    float* qs = reinterpret_cast<float*>(smem_raw + C::RING_BYTES) + warp * HD;
    float* pbuf = reinterpret_cast<float*>(smem_raw + C::RING_BYTES) + C::WARPS * HD + warp * kPage;
    uint64_t* wb = bars[warp];
    if (lane == 0) {
        for (int s = 0; s < kDecStages; s++) mbar_init(&wb[s], 1);
        fence_barrier_init();
    }
    __syncwarp();
    grid_dependency_wait();  // q, the K/V pages and the work counters come from earlier kernels

    auto fetch = [&]() -> int {
        int v = 0;
        if (lane == 0) v = atomicAdd(a.work, 1);
        return __shfl_sync(0xffffffffu, v, 0);
    };
    const float qscale = kLog2e / sqrtf((float)HD);
    DecItem cur = dec_item<HD>(fetch(), total, tab, a, lane, qscale);
    DecItem nxt = dec_item<HD>(cur.valid ? fetch() : total, total, tab, a, lane, qscale);

    // issue pointer: page `ip` of item `iq` (0 = cur, 1 = nxt); k-th issued page -> slot k % stages
    int iq = 0, ip = 0;
    uint32_t issued = 0, consumed = 0;
    auto issue_some = [&]() {
        while (issued - consumed < (uint32_t)kDecStages) {
            const DecItem& src = iq == 0 ? cur : nxt;
            if (iq > 1 || !src.valid) break;
            if (ip >= src.np) { iq++; ip = 0; continue; }
            const int page = __shfl_sync(0xffffffffu, src.pid, ip);
            if (lane == 0) {
                // the slot's previous page was consumed by every lane before the __syncwarp
                // that ended its processing, so the copy cannot overwrite live data
                const int slot = issued % kDecStages;
                const int64_t off = a.geom.tile_offset(page, a.layer, src.h / kvmul);
                mbar_arrive_expect_tx(&wb[slot], 2u * C::TILE_BYTES);
                bulk_g2s(ring + (2 * slot) * C::TILE, kpool + off, C::TILE_BYTES, &wb[slot]);
                bulk_g2s(ring + (2 * slot + 1) * C::TILE, vpool + off, C::TILE_BYTES, &wb[slot]);
            }
            issued++;
            ip++;
        }
    };

    bool ok = true;
    while (cur.valid) {
        issue_some();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < HD / 32; j++) qs[lane + 32 * j] = cur.q[j];
        __syncwarp();
        float4 qr[HD / 8];
        load_query<HD>(qr, qs, lane);
        QState<HD> st;
        st.init();
        for (int pg = 0; pg < cur.np; pg++) {
            issue_some();
            const int slot = consumed % kDecStages;
            if (ok && !mbar_wait(&wb[slot], (consumed / kDecStages) & 1, a.err)) ok = false;
            if (ok) {
                const int first = (cur.p0 + pg) * kPage;
                attend_page<HD, KT>(st, qr, pbuf, ring + (2 * slot) * C::TILE, ring + (2 * slot + 1) * C::TILE,
                                    min(kPage, cur.ctx - first), lane);
            }
            __syncwarp();  // every lane is done with the slot before it is refilled
            consumed++;
        }
        // retire the item
        const int64_t bh = (int64_t)cur.b * a.n_heads + cur.h;
        float* out = a.out + bh * HD + lane * DPL;
        if (cur.nsplit == 1) {
            const float inv = 1.0f / st.l;
#pragma unroll
            for (int i = 0; i < DPL; i++) out[i] = st.o[i] * inv;
        } else {
            // a split of a longer context: publish (max, sum, unnormalised output); the merge
            // kernel that follows in the stream combines the splits
            float* po = a.part_o + (bh * a.max_splits + cur.split) * HD + lane * DPL;
#pragma unroll
            for (int i = 0; i < DPL; i++) po[i] = st.o[i];
            if (lane == 0) {
                a.part_ml[(bh * a.max_splits + cur.split) * 2] = st.m;
                a.part_ml[(bh * a.max_splits + cur.split) * 2 + 1] = st.l;
            }
        }
        // advance: the issue pointer moves with the item window.  It is at or past the end
        // of the retired item; if it had not crossed into the next one yet, it starts that
        // item from its first page.
        if (iq == 0) { iq = 1; ip = 0; }
        cur = nxt;
        iq -= 1;
        nxt = dec_item<HD>(cur.valid ? fetch() : total, total, tab, a, lane, qscale);
    }
    grid_dependents_launch();
    // every copy this warp issued has been consumed (issued == consumed here); the last warp
    // to finish resets the work counters for the next launch
    if (lane == 0) {
        __threadfence();
        const int done = atomicAdd(a.work + 1, 1);
        if (done == (int)(gridDim.x * C::WARPS) - 1) {
            a.work[0] = 0;
            a.work[1] = 0;
        }
    }
}

// Small batches (B x n_heads up to the SM count): one CTA per (sequence, head), its warps
// taking the sequence's pages round-robin through their own bulk-copy rings and joining
// their softmax states in shared memory (in warp order), so neither split partials in
// global memory nor the merge kernel are needed.
template <int HD, typename KT = float>
struct DecSmall {
    static constexpr int WARPS = HD == 64 ? 8 : 6;
    static constexpr int STAGES = HD == 64 ? 3 : 2;
    static constexpr int TILE = kPage * HD;
    static constexpr int TILE_BYTES = TILE * (int)sizeof(KT);
    static constexpr int RING_BYTES = WARPS * STAGES * 2 * TILE_BYTES;
    static constexpr int SMEM = RING_BYTES + HD * 4 + WARPS * (HD + 2 + kPage) * 4;
};

template <int HD, typename KT>
__global__ void __launch_bounds__(DecSmall<HD>::WARPS * 32, 1) decode_attn_small_kernel(DecodeAttnArgs a) {
    using C = DecSmall<HD, KT>;
    constexpr int DPL = HD / 32;
    constexpr int W = C::WARPS, S = C::STAGES;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    __shared__ uint64_t bars[W][S];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x / a.n_heads, h = blockIdx.x % a.n_heads;
    const int kvh = h / (a.n_heads / a.geom.n_kv_heads);
    const KT* kpool = reinterpret_cast<const KT*>(a.kpool);
    const KT* vpool = reinterpret_cast<const KT*>(a.vpool);
    KT* ring = reinterpret_cast<KT*>(smem_raw + warp * S * 2 * C::TILE_BYTES);
    float* qs = reinterpret_cast<float*>(smem_raw + C::RING_BYTES);
    float* part = qs + HD;  // [W][HD + 2]: o, then m, l
    float* pbuf = part + W * (HD + 2) + warp * kPage;  // this warp's page probabilities

    // page ids of this warp's pages (descriptor data: read before the wait)
    const int ctx = checked_ctx(a, b, h == 0 && threadIdx.x == 0);
    const int pages = (ctx + kPage - 1) / kPage;
    const int mine = pages > warp ? (pages - warp + W - 1) / W : 0;  // pages warp, warp+W, ...
    if (lane < S) mbar_init(&bars[warp][lane], 1);
    fence_barrier_init();
    __syncwarp();
    grid_dependency_wait();  // q and the newest K/V rows come from the previous kernel
    const float qscale = kLog2e / sqrtf((float)HD);
    for (int i = threadIdx.x; i < HD; i += blockDim.x) qs[i] = a.q[((int64_t)b * a.n_heads + h) * HD + i] * qscale;
    auto issue = [&](int j) {  // the warp's j-th page -> slot j % S (lane 0)
        const int p = warp + j * W;
        const int page = a.block_tables[(int64_t)b * a.max_pages + p];
        const int64_t off = a.geom.tile_offset(page, a.layer, kvh);
        uint64_t* bar = &bars[warp][j % S];
        mbar_arrive_expect_tx(bar, 2u * C::TILE_BYTES);
        bulk_g2s(ring + (2 * (j % S)) * C::TILE, kpool + off, C::TILE_BYTES, bar);
        bulk_g2s(ring + (2 * (j % S) + 1) * C::TILE, vpool + off, C::TILE_BYTES, bar);
    };
    if (lane == 0)
        for (int j = 0; j < S && j < mine; j++) issue(j);
    __syncthreads();  // q in shared memory

    float4 qr[HD / 8];
    load_query<HD>(qr, qs, lane);
    QState<HD> st;
    st.init();
    bool ok = true;
    for (int j = 0; j < mine; j++) {
        const int slot = j % S;
        if (ok && !mbar_wait(&bars[warp][slot], (j / S) & 1, a.err)) ok = false;
        if (ok) {
            const int first = (warp + j * W) * kPage;
            attend_page<HD, KT>(st, qr, pbuf, ring + (2 * slot) * C::TILE, ring + (2 * slot + 1) * C::TILE,
                                min(kPage, ctx - first), lane);
        }
        __syncwarp();  // every lane is done with the slot before it is refilled
        if (lane == 0 && ok && j + S < mine) issue(j + S);
    }
    grid_dependents_launch();
    float* pw = part + warp * (HD + 2);
#pragma unroll
    for (int i = 0; i < DPL; i++) pw[lane * DPL + i] = st.o[i];
    if (lane == 0) {
        pw[HD] = mine > 0 && ok ? st.m : -INFINITY;
        pw[HD + 1] = mine > 0 && ok ? st.l : 0.0f;
    }
    __syncthreads();
    if (warp == 0) {
        float gm = -INFINITY;
        for (int w = 0; w < W; w++) gm = fmaxf(gm, part[w * (HD + 2) + HD]);
        float gl = 0.0f, go[DPL];
#pragma unroll
        for (int i = 0; i < DPL; i++) go[i] = 0.0f;
        for (int w = 0; w < W; w++) {
            const float mw = part[w * (HD + 2) + HD];
            const float c = mw == -INFINITY ? 0.0f : exp2f(mw - gm);
            gl += part[w * (HD + 2) + HD + 1] * c;
#pragma unroll
            for (int i = 0; i < DPL; i++) go[i] += part[w * (HD + 2) + lane * DPL + i] * c;
        }
        const float inv = gl > 0.0f ? 1.0f / gl : 0.0f;  // no tokens: zero output
        float* out = a.out + ((int64_t)b * a.n_heads + h) * HD + lane * DPL;
#pragma unroll
        for (int i = 0; i < DPL; i++) out[i] = go[i] * inv;
    }
}

// Combine the splits of every (sequence, head) whose context spans more than one chunk:
// one warp per (sequence, head), weights exp2(m_s - max) broadcast by shuffle.
template <int HD>
__global__ void __launch_bounds__(256) decode_merge_kernel(DecodeAttnArgs a) {
    constexpr int DPL = HD / 32;
    const int lane = threadIdx.x & 31;
    const int64_t bh = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    grid_dependency_wait();
    grid_dependents_launch();
    if (bh >= (int64_t)a.B * a.n_heads) return;
    const int b = (int)(bh / a.n_heads);
    const int pages = (checked_ctx(a, b, false) + kPage - 1) / kPage;
    const int nsplit = (pages + a.chunk_pages - 1) / a.chunk_pages;
    if (nsplit == 0) {  // a row with no tokens (flagged by the attention kernel): zero output
        float* out = a.out + bh * HD + lane * DPL;
#pragma unroll
        for (int i = 0; i < DPL; i++) out[i] = 0.0f;
        return;
    }
    if (nsplit <= 1) return;
    float GM = -INFINITY;
    for (int base = 0; base < nsplit; base += 32)
        if (base + lane < nsplit) GM = fmaxf(GM, a.part_ml[(bh * a.max_splits + base + lane) * 2]);
    GM = warp_max(GM);
    float GL = 0.0f, GO[DPL];
#pragma unroll
    for (int i = 0; i < DPL; i++) GO[i] = 0.0f;
    for (int base = 0; base < nsplit; base += 32) {
        float ms = -INFINITY, ls = 0.0f;
        if (base + lane < nsplit) {
            ms = a.part_ml[(bh * a.max_splits + base + lane) * 2];
            ls = a.part_ml[(bh * a.max_splits + base + lane) * 2 + 1];
        }
        const float cl = (ms == -INFINITY) ? 0.0f : exp2f(ms - GM);
        GL += warp_sum(ls * cl);
        const int cnt = min(32, nsplit - base);
        for (int sp = 0; sp < cnt; sp++) {
            const float c = __shfl_sync(0xffffffffu, cl, sp);
            const float* ps = a.part_o + (bh * a.max_splits + base + sp) * HD + lane * DPL;
#pragma unroll
            for (int i = 0; i < DPL; i++) GO[i] += ps[i] * c;
        }
    }
    const float inv = 1.0f / GL;
    float* out = a.out + bh * HD + lane * DPL;
#pragma unroll
    for (int i = 0; i < DPL; i++) out[i] = GO[i] * inv;
}

// ------------------------------------------------------------------ prefill
// One CTA per (query tile, head); 4 warps of PQW queries each (8 at head_dim 64, 4 at
// 128).  Pages 0..last of the sequence stream through kStages shared-memory stages.
// Inside a warp, lane = (key group kg of 4 keys) x (dim group dg of head_dim / 8 dims):
// each lane holds its queries' dims in registers, forms partial scores for 8 x 4
// (query, key) pairs, joins them over the 8 dim groups with 3 shuffles, and accumulates
// the output for its 4 keys and its dims; the 4 key groups' outputs are joined once at
// the end.  FMA-dense, with independent chains across queries and keys.  Online softmax
// in the exp2 domain as in the decode kernel (the reference's single-pass online softmax,
// src/model_q8.cpp:485-523, up to fp32 rounding).
constexpr int kStages = 4;

template <int HD>
struct PrefillCfg {
    static constexpr int QW = HD == 64 ? 8 : 4;  // queries per warp
    static constexpr int QT = kAttnWarps * QW;   // queries per CTA
    static constexpr int DG = HD / 8;            // dims per lane
};

template <int HD, typename KT>
__global__ void __launch_bounds__(kAttnWarps * 32) prefill_attn_kernel(PrefillAttnArgs a) {
    using P = PrefillCfg<HD>;
    constexpr int TILE = kPage * HD;
    constexpr int TILE_BYTES = TILE * (int)sizeof(KT);
    constexpr int QW = P::QW, DG = P::DG;
    extern __shared__ __align__(128) uint8_t smem_raw[];  // [kStages][2][TILE] page elements
    KT* smem = reinterpret_cast<KT*>(smem_raw);
    const KT* kpool = reinterpret_cast<const KT*>(a.kpool);
    const KT* vpool = reinterpret_cast<const KT*>(a.vpool);
    __shared__ uint64_t full[kStages];

    // blocks in order of decreasing work (later query tiles attend more pages) so the
    // longest start first: block b takes tile n_tiles - 1 - b / n_heads, head b % n_heads;
    // with several sequences the tile table holds that order (written with the descriptor,
    // before the kernel chain of the step)
    int T = a.T, start_pos = a.start_pos, row0 = 0, qt;
    const int* bt = a.block_table;
    const int h = (int)blockIdx.x % a.n_heads;
    if (a.seg) {
        const int j = (int)blockIdx.x / a.n_heads;
        const int sg = a.tiles[2 * j];
        qt = a.tiles[2 * j + 1];
        row0 = a.seg[4 * sg];
        T = a.seg[4 * sg + 1];
        start_pos = a.seg[4 * sg + 2];
        bt = a.block_table + a.seg[4 * sg + 3];
    } else {
        qt = (T + P::QT - 1) / P::QT - 1 - (int)blockIdx.x / a.n_heads;
    }
    const int t0 = qt * P::QT;
    const int nq = min(P::QT, T - t0);
    const int last_pos = start_pos + t0 + nq - 1;
    const int n_pages = last_pos / kPage + 1;
    const int kvh = h / (a.n_heads / a.geom.n_kv_heads);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kg = lane >> 3, dg = lane & 7;  // keys kg*4.., dims dg*DG..
    const int q0 = t0 + warp * QW;            // this warp's first query (token index)

    auto issue = [&](int page_idx) {
        const int s = page_idx % kStages;
        const int64_t off = a.geom.tile_offset(bt[page_idx], a.layer, kvh);
        mbar_arrive_expect_tx(&full[s], 2u * TILE_BYTES);
        bulk_g2s(smem + (2 * s) * TILE, kpool + off, TILE_BYTES, &full[s]);
        bulk_g2s(smem + (2 * s + 1) * TILE, vpool + off, TILE_BYTES, &full[s]);
    };
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    grid_dependency_wait();  // q and this chunk's K/V rows come from the projection kernel
    if (threadIdx.x == 0)
        for (int i = 0; i < kStages && i < n_pages; i++) issue(i);
    __syncthreads();

    // this lane's dims of its warp's queries, pre-scaled for the exp2-domain softmax
    const float qscale = kLog2e / sqrtf((float)HD);
    float q[QW][DG];
#pragma unroll
    for (int i = 0; i < QW; i++) {
        const int t = q0 + i;
        const float4* src =
            reinterpret_cast<const float4*>(a.q + ((int64_t)(row0 + min(t, T - 1)) * a.n_heads + h) * HD + dg * DG);
#pragma unroll
        for (int j = 0; j < DG / 4; j++) {
            const float4 v = src[j];
            q[i][4 * j] = v.x * qscale; q[i][4 * j + 1] = v.y * qscale;
            q[i][4 * j + 2] = v.z * qscale; q[i][4 * j + 3] = v.w * qscale;
        }
    }
    float o[QW][DG], m[QW], l[QW];
#pragma unroll
    for (int i = 0; i < QW; i++) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int d = 0; d < DG; d++) o[i][d] = 0.0f;
    }
    const int warp_last = start_pos + min(q0 + QW, T) - 1;  // position of the warp's last query

    bool ok = true;
    for (int p = 0; p < n_pages; p++) {
        const int s = p % kStages;
        if (ok && !mbar_wait(&full[s], (p / kStages) & 1, a.err)) ok = false;
        if (ok && p * kPage <= warp_last) {
            const KT* Kt = smem + (2 * s) * TILE;
            const KT* Vt = smem + (2 * s + 1) * TILE;
            // scores of (query i, key kg*4 + j) over this lane's dims, then over all dims
            float sc[QW][4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float kr[DG];
                const KT* k4 = Kt + (kg * 4 + j) * HD + dg * DG;
#pragma unroll
                for (int c = 0; c < DG / 4; c++) {
                    const float4 v = ldkv4(k4 + 4 * c);
                    kr[4 * c] = v.x; kr[4 * c + 1] = v.y; kr[4 * c + 2] = v.z; kr[4 * c + 3] = v.w;
                }
#pragma unroll
                for (int i = 0; i < QW; i++) {
                    float acc = 0.0f;
#pragma unroll
                    for (int d = 0; d < DG; d++) acc = fmaf(q[i][d], kr[d], acc);
                    sc[i][j] = acc;
                }
            }
#pragma unroll
            for (int i = 0; i < QW; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float v = sc[i][j];
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    v += __shfl_xor_sync(0xffffffffu, v, 4);
                    sc[i][j] = v;
                }
            // causal mask, running max, probabilities, running sum
#pragma unroll
            for (int i = 0; i < QW; i++) {
                const int qpos = start_pos + q0 + i;
                float mx = -INFINITY;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (p * kPage + kg * 4 + j > qpos) sc[i][j] = -INFINITY;
                    mx = fmaxf(mx, sc[i][j]);
                }
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                const float m_new = fmaxf(m[i], mx);
                const float corr = m_new == -INFINITY ? 1.0f : exp2f(m[i] - m_new);
                float ps = 0.0f;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    sc[i][j] = m_new == -INFINITY ? 0.0f : exp2f(sc[i][j] - m_new);
                    ps += sc[i][j];
                }
                ps += __shfl_xor_sync(0xffffffffu, ps, 8);
                ps += __shfl_xor_sync(0xffffffffu, ps, 16);
                l[i] = l[i] * corr + ps;
                m[i] = m_new;
#pragma unroll
                for (int d = 0; d < DG; d++) o[i][d] *= corr;
            }
            // this lane's 4 keys times their value rows, its dims
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float vr[DG];
                const KT* v4 = Vt + (kg * 4 + j) * HD + dg * DG;
#pragma unroll
                for (int c = 0; c < DG / 4; c++) {
                    const float4 v = ldkv4(v4 + 4 * c);
                    vr[4 * c] = v.x; vr[4 * c + 1] = v.y; vr[4 * c + 2] = v.z; vr[4 * c + 3] = v.w;
                }
#pragma unroll
                for (int i = 0; i < QW; i++)
#pragma unroll
                    for (int d = 0; d < DG; d++) o[i][d] = fmaf(sc[i][j], vr[d], o[i][d]);
            }
        }
        // CTA-uniform: every thread leaves together if any wait gave up
        if (!__syncthreads_and(ok)) { ok = false; break; }
        if (threadIdx.x == 0 && p + kStages < n_pages) issue(p + kStages);
    }
    grid_dependents_launch();
    if (!ok) return;
    // join the 4 key groups' outputs (same running max everywhere), normalise, store
#pragma unroll
    for (int i = 0; i < QW; i++)
#pragma unroll
        for (int d = 0; d < DG; d++) {
            float v = o[i][d];
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            o[i][d] = v;
        }
    if (kg == 0) {
#pragma unroll
        for (int i = 0; i < QW; i++) {
            const int t = q0 + i;
            if (t >= T) continue;
            const float inv = 1.0f / l[i];
            float4* dst = reinterpret_cast<float4*>(a.out + ((int64_t)(row0 + t) * a.n_heads + h) * HD + dg * DG);
#pragma unroll
            for (int c = 0; c < DG / 4; c++)
                dst[c] = make_float4(o[i][4 * c] * inv, o[i][4 * c + 1] * inv, o[i][4 * c + 2] * inv,
                                     o[i][4 * c + 3] * inv);
        }
    }
}

// cudaFuncSetAttribute is per (kernel, device): remember which pairs are configured.
template <class K>
void ensure_smem(K kernel, int bytes) {
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_pair((const void*)kernel, dev);
    if (done.count(key)) return;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    done.insert(key);
}

}  // namespace

int decode_attn_chunk_pages(int head_dim) { return head_dim <= 64 ? NITRO_DEC_CHUNK64 : NITRO_DEC_CHUNK64 / 2; }

// Small batches get shorter chunks (down to this many pages) so that there are enough
// work items for every warp; the partial buffers are laid out for that many splits.
constexpr int kMinChunkPages = 2;

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

size_t decode_attn_workspace_bytes(int B, int n_heads, int head_dim, int max_pages) {
    (void)head_dim;
    const int cp = kMinChunkPages;
    const int ms = (max_pages + cp - 1) / cp;
    size_t o = align_up((size_t)B * n_heads * ms * head_dim * 4, 256);
    size_t ml = align_up((size_t)B * n_heads * ms * 2 * 4, 256);
    size_t cnt = align_up((size_t)B * n_heads * 4 + 2 * 4, 256);
    return o + ml + cnt;
}

void decode_attn_bind_workspace(DecodeAttnArgs& a, void* ws, int max_pages_capacity) {
    const int hd = a.geom.head_dim;
    a.chunk_pages = decode_attn_chunk_pages(hd);
    a.max_splits = (max_pages_capacity + kMinChunkPages - 1) / kMinChunkPages;
    char* p = (char*)ws;
    a.part_o = (float*)p;
    p += align_up((size_t)a.B * a.n_heads * a.max_splits * hd * 4, 256);
    a.part_ml = (float*)p;
    p += align_up((size_t)a.B * a.n_heads * a.max_splits * 2 * 4, 256);
    a.counters = (int*)p;
    a.work = a.counters + (size_t)a.B * a.n_heads;
}

static int sm_count() {
    static std::mutex mu;
    static int counts[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64) return 148;
    if (!counts[dev]) cudaDeviceGetAttribute(&counts[dev], cudaDevAttrMultiProcessorCount, dev);
    return counts[dev] > 0 ? counts[dev] : 148;
}

template <int HD, typename KT>
static void launch_small(const DecodeAttnArgs& a, dim3 g, cudaStream_t s) {
    using C = DecSmall<HD, KT>;
    ensure_smem(decode_attn_small_kernel<HD, KT>, C::SMEM);
    launch_ex(decode_attn_small_kernel<HD, KT>, g, dim3(C::WARPS * 32), C::SMEM, s, 1, a);
}

template <int HD, typename KT>
static void launch_split(const DecodeAttnArgs& a, int grid, cudaStream_t s) {
    using C = DecCfg<HD, KT>;
    ensure_smem(decode_attn_kernel<HD, KT>, C::SMEM);
    launch_ex(decode_attn_kernel<HD, KT>, dim3(grid), dim3(C::WARPS * 32), C::SMEM, s, 1, a);
}

template <int HD, typename KT>
static void launch_prefill(const PrefillAttnArgs& a, cudaStream_t s) {
    dim3 grid((unsigned)((a.seg ? a.n_tiles : (a.T + PrefillCfg<HD>::QT - 1) / PrefillCfg<HD>::QT) * a.n_heads));
    const int smem = kStages * 2 * kPage * HD * (int)sizeof(KT);
    ensure_smem(prefill_attn_kernel<HD, KT>, smem);
    launch_ex(prefill_attn_kernel<HD, KT>, grid, dim3(kAttnWarps * 32), smem, s, 1, a);
}

// Small batches (B x heads up to the SM count) take one CTA per (sequence, head) and
// need no merge; larger ones take the persistent split kernel and the merge kernel.
bool decode_attn_splits(const DecodeAttnArgs& a) { return (int64_t)a.B * a.n_heads > sm_count(); }

DecodeAttnArgs plan_decode_attention(const DecodeAttnArgs& args, int max_ctx) {
    DecodeAttnArgs a = args;
    if (!decode_attn_splits(a)) return a;
    // chunk length: the longest (default) that still gives every warp about two items,
    // estimated from the longest context of the step
    const int warps = sm_count() * (a.geom.head_dim == 64 ? DecCfg<64>::WARPS : DecCfg<128>::WARPS);
    const int64_t pages = (int64_t)a.B * ((max_ctx + kPage - 1) / kPage);
    while (a.chunk_pages > kMinChunkPages && pages / a.chunk_pages * a.n_heads < 2 * warps) a.chunk_pages /= 2;
    if (a.chunk_pages < kMinChunkPages) a.chunk_pages = kMinChunkPages;
    return a;
}

void launch_decode_attention_main(const DecodeAttnArgs& a, cudaStream_t s) {
    count_launch();
    const int grid = sm_count();
    if (!decode_attn_splits(a)) {
        const dim3 g((unsigned)(a.B * a.n_heads));
        if (a.geom.head_dim == 64) {
            if (a.geom.kv_bf16) launch_small<64, __nv_bfloat16>(a, g, s);
            else launch_small<64, float>(a, g, s);
        } else {
            if (a.geom.kv_bf16) launch_small<128, __nv_bfloat16>(a, g, s);
            else launch_small<128, float>(a, g, s);
        }
        return;
    }
    if (a.geom.head_dim == 64) {
        if (a.geom.kv_bf16) launch_split<64, __nv_bfloat16>(a, grid, s);
        else launch_split<64, float>(a, grid, s);
    } else {
        if (a.geom.kv_bf16) launch_split<128, __nv_bfloat16>(a, grid, s);
        else launch_split<128, float>(a, grid, s);
    }
}

void launch_decode_merge(const DecodeAttnArgs& a, cudaStream_t s) {
    if (!decode_attn_splits(a)) return;
    count_launch();
    const dim3 mgrid((unsigned)(((int64_t)a.B * a.n_heads + 7) / 8));
    if (a.geom.head_dim == 64) launch_ex(decode_merge_kernel<64>, mgrid, dim3(256), 0, s, 1, a);
    else launch_ex(decode_merge_kernel<128>, mgrid, dim3(256), 0, s, 1, a);
}

void launch_decode_attention(const DecodeAttnArgs& args, int max_ctx, cudaStream_t s) {
    const DecodeAttnArgs a = plan_decode_attention(args, max_ctx);
    launch_decode_attention_main(a, s);
    launch_decode_merge(a, s);
}

int prefill_attn_query_tile(int head_dim) {
    if (prefill_attn_tc_enabled(head_dim)) return 128;
    return head_dim == 64 ? PrefillCfg<64>::QT : PrefillCfg<128>::QT;
}

void launch_prefill_attention(const PrefillAttnArgs& a, cudaStream_t s) {
    count_launch();
    if (prefill_attn_tc_enabled(a.geom.head_dim)) {
        launch_prefill_attention_tc(a, s);
    } else if (a.geom.head_dim == 64) {
        if (a.geom.kv_bf16) launch_prefill<64, __nv_bfloat16>(a, s);
        else launch_prefill<64, float>(a, s);
    } else {
        if (a.geom.kv_bf16) launch_prefill<128, __nv_bfloat16>(a, s);
        else launch_prefill<128, float>(a, s);
    }
}

}  // namespace nitro

// ---------------------------------------------------------------------------------------
// Decode attention with library-owned scratch (nr_paged_attention_decode_static).
//
// Some callers may not allocate device memory at all while they step: a server that handed
// all of HBM to its own KV page pool at start-up has nothing left for a cudaMalloc, and
// cudaMalloc/cudaFree synchronise the device, which a step loop that keeps several
// streams busy cannot afford.  This entry point runs the same two kernels as
// nr_paged_attention_decode with their split partials and work counters in one fixed
// array that is part of the library's device image, so the call itself allocates nothing.
//
// The array is shared by every call on a device and keeps whatever the last call left in
// it: the work counters are cleared on the stream before each launch, the partials are
// always written before they are read.  Two calls whose kernels overlap (different
// streams, or different host threads on one stream without ordering) race on it.
// Every call resolves the array's address with cudaGetSymbolAddress (the first call on a
// device may load the module there); the first call on each device also sets the kernels'
// shared-memory limits, so make it outside any stream capture.  Those limits are recorded
// once per device for the life of the process, like every other kernel of this library:
// do not use the library across a cudaDeviceReset.
namespace nitro {

static constexpr size_t kStaticScratchBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

// The array's device address on the current device.  Resolved on every call (cheap once
// the module is loaded) rather than cached, so a context torn down and created again
// never gets an address from the old one.
static int static_scratch(void** out) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || !p) return -1;
    *out = p;
    return 0;
}

}  // namespace nitro

#include "../../include/nitro_engine.h"

static_assert(nitro::kStaticScratchBytes == NR_ATTN_STATIC_SCRATCH_BYTES, "scratch size and header disagree");

extern "C" int nr_paged_attention_decode_static(const float* q, const float* kpool, const float* vpool,
                                                const int32_t* block_tables, int32_t max_pages,
                                                const int32_t* ctx_lens, int32_t B, int32_t n_heads,
                                                int32_t n_kv_heads, int32_t head_dim, int32_t n_layers,
                                                int32_t layer, float* out, int32_t* error_flag, void* stream) {
    if (!q || !kpool || !vpool || !block_tables || !ctx_lens || !out) return NR_ERR_INVALID;
    if (B <= 0 || B > 1024 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || max_pages <= 0)
        return NR_ERR_INVALID;
    if (head_dim != 64 && head_dim != 128) return NR_ERR_INVALID;
    if (n_layers <= 0 || layer < 0 || layer >= n_layers) return NR_ERR_INVALID;
    if (nitro::decode_attn_workspace_bytes(B, n_heads, head_dim, max_pages) > nitro::kStaticScratchBytes)
        return NR_ERR_CAPACITY;
    void* ws = nullptr;
    if (nitro::static_scratch(&ws) != 0) return NR_ERR_CUDA;
    nitro::DecodeAttnArgs a;
    a.q = q; a.kpool = kpool; a.vpool = vpool;
    a.geom = nitro::PoolGeom{n_layers, n_kv_heads, head_dim};
    a.layer = layer; a.block_tables = block_tables; a.max_pages = max_pages; a.ctx_lens = ctx_lens;
    a.B = B; a.n_heads = n_heads; a.out = out; a.err = error_flag;
    nitro::decode_attn_bind_workspace(a, ws, max_pages);
    cudaStream_t s = (cudaStream_t)stream;
    const size_t counter_bytes = ((size_t)B * n_heads + 2) * sizeof(int);
    if (cudaMemsetAsync(a.counters, 0, counter_bytes, s) != cudaSuccess) return NR_ERR_CUDA;
    nitro::launch_decode_attention(a, max_pages * nitro::kPage, s);
    return cudaGetLastError() == cudaSuccess ? NR_OK : NR_ERR_CUDA;
}
