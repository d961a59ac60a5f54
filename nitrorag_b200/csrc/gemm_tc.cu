// Q8_0 (and fp32) projections on the 5th-generation tensor cores (tcgen05), for token
// batches wide enough to make the product a real dense contraction (decode batches and
// prefill chunks of more than 8 tokens).
//
// Orientation: D[n][m] = sum_k W[n][k] * X[m][k], weight rows n on the MMA's M side (128
// rows per CTA), tokens m on its N side (NT = 64, 128 or 256 per CTA), fp32 accumulators
// in tensor memory (TMEM), one column per token.
//
// Precision: the reference multiplies in fp32 (w = q * scale, then w * x, fp32 sums).
// Each operand is split into two bf16 halves, v = hi + lo with hi = bf16(v) and
// lo = bf16(v - hi) (17 significant bits together), and the product is accumulated as
// hi*hi + hi*lo + lo*hi by three MMAs into the same fp32 accumulator; the dropped lo*lo
// term and the split residues are ~2^-17 relative, far inside the 1e-3 / 1e-4 logits bar.
//
// Pipeline per CTA (256 threads, two warpgroups): every thread dequantises half a weight
// row of each 64-wide K chunk (one Q8_0 block, w = q * scale) and a quarter-chunk slice of
// one token's activations (the RMSNorm of the row applied on the fly) into the UMMA
// canonical K-major layout in shared memory; thread 0 issues 4 x 3 MMAs per chunk.  When a
// CTA's chunks all fit in shared memory (the decode shapes), its weights are staged before
// the grid-dependency wait, i.e. while the previous kernel still runs, and only the
// activations wait; otherwise chunks go through a 2-stage ring with the next chunk's loads
// issued one ahead.  When the weight tiles are too few to fill the GPU, the K range of a
// tile is split over the CTAs of a thread-block cluster; token slice r of the tile is
// summed by CTA r from partials its peers push into its shared memory (deterministic rank
// order), then the epilogue runs.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <set>
#include <tuple>
#include <utility>

#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace nitro {

namespace {

constexpr int TC_M = 128;     // weight rows per CTA = UMMA M
constexpr int TC_KC = 64;     // K elements per pipeline stage
constexpr int TC_STAGES = 2;      // pipeline stages of the 128/256-token tiles
constexpr int TC_MAX_STAGES = 4;  // 64-token tiles stage up to 4 chunks
constexpr int TC_WORKERS = 256;              // staging and epilogue threads: two warpgroups
constexpr int TC_THREADS = TC_WORKERS + 32;  // + one warp that issues the MMAs
constexpr int kIssuerWarp = TC_WORKERS / 32;
constexpr uint32_t TC_TILE_BYTES = 2u * TC_M * TC_KC * 2u;  // hi + lo halves of one 128 x 64 weight tile
// raw Q8 tile: int8 [half][16-byte piece][128 rows][16 B] (8 KB) then fp32 scales
// [half][128 rows] (1 KB); a warp's 32 rows read 512 contiguous bytes per piece
constexpr uint32_t TC_RAW_BYTES = TC_M * TC_KC + TC_M * 2 * 4;
constexpr int TC_RAW_MAX = 12;  // ring slots of raw tiles
#ifndef NITRO_TC_MAX_KSPLIT
#define NITRO_TC_MAX_KSPLIT 8  // largest K split (CTAs per cluster)
#endif

// Named CTA barriers between the staging warps (arrive) and the MMA-issuing warp (sync).
__device__ __forceinline__ void named_arrive(int id, int count) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Split cluster barrier: arrive (publishing this thread's earlier memory operations) and,
// later, wait for every thread of the cluster to have arrived.
__device__ __forceinline__ void cluster_arrive_release() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait_acquire() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Distributed shared memory: this CTA's shared address `saddr` mapped into CTA `rank` of
// the cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}

// 16-byte asynchronous store into a cluster peer's shared memory that completes as 16
// transaction bytes on the peer's mbarrier `bar` (both addresses from map_rank).
__device__ __forceinline__ void st_async4(uint32_t addr, float a, float b, float c, float d, uint32_t bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
                 "f"(a), "f"(b), "f"(c), "f"(d), "r"(bar)
                 : "memory");
}

// Bounded wait on a local mbarrier whose transaction bytes come from other CTAs of the
// cluster (acquire at cluster scope makes their data visible to this thread).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(1000u)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; i++) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((i & 15) == 0 && global_ns() - t0 > kWaitLimitNs) break;
    }
    if (err) atomicCAS(err, 0, kErrWaitTimeout);
    return false;
}

// ------------------------------------------------------------------ operand staging
template <int NT>
struct TcSmem {
    static constexpr int A_BYTES = TC_M * TC_KC * 2;   // one bf16 half of the weight tile
    static constexpr int B_BYTES = NT * TC_KC * 2;     // one bf16 half of the token tile
    static constexpr int STAGE = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int MAX_STAGES = NT == 64 ? TC_MAX_STAGES : TC_STAGES;
};

struct SplitArgs {
    int ksplit;  // K-range splits per tile = CTAs per thread-block cluster (grid.x)
    int stages;  // shared-memory stages (one per chunk when a CTA's chunks all fit)
    int recv_off;  // byte offset of the split-K receive buffer in dynamic shared memory
    int recv_pad;  // floats of padding per receive-buffer row (4, or 0 when short of space)
    int gain_off;  // byte offset of the staged RMSNorm gain slice in dynamic shared memory
    int raw_off;   // raw Q8 tiles: byte offset and number of ring slots
    int raw_slots;
};

// Thread roles.  Thread t owns weight row (t & 127) of the tile, which is also its TMEM
// lane, and K half (t >> 7) of every chunk (32 values = one Q8_0 block).  Activation units
// are (token, 16-wide K quarter) pairs.  In the epilogue warpgroup g (= t >> 7) takes the
// g-th half of the columns this CTA finishes.

// Raw global loads of this thread's share of one chunk's weights (issued ahead of the
// conversion so their latency overlaps other work).
template <bool F32W>
struct WRegs {
    int4 q[F32W ? 1 : 2];
    float4 f[F32W ? 8 : 1];
    float s;
};

template <bool F32W>
__device__ __forceinline__ void load_w(WRegs<F32W>& r, const GemmArgs& a, int n, int k) {
    if (n < a.N) {
        if (F32W) {
            const float4* src = reinterpret_cast<const float4*>(a.wf + (int64_t)n * a.K + k);
#pragma unroll
            for (int i = 0; i < 8; i++) r.f[i] = __ldg(src + i);
        } else {
            const int4* src = reinterpret_cast<const int4*>(a.wq + (int64_t)n * a.K + k);
            r.q[0] = __ldg(src);
            r.q[1] = __ldg(src + 1);
            r.s = __ldg(a.ws + (int64_t)n * (a.K >> 5) + (k >> 5));
        }
    }
}

// This thread's 32 weights of one chunk (registers -> bf16 hi/lo core rows).
template <bool F32W>
__device__ __forceinline__ void stage_w(const WRegs<F32W>& r, const GemmArgs& a, int n, int k, uint8_t* a_hi,
                                        uint8_t* a_lo, int row, int half) {
    float w[32];
    if (n < a.N) {
        if (F32W) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                w[4 * i] = r.f[i].x; w[4 * i + 1] = r.f[i].y; w[4 * i + 2] = r.f[i].z; w[4 * i + 3] = r.f[i].w;
            }
        } else {
            const int8_t* q = reinterpret_cast<const int8_t*>(r.q);
#pragma unroll
            for (int j = 0; j < 32; j++) w[j] = (float)q[j] * r.s;
        }
        if (k < a.kbegin) {  // faithful mode: only k >= kbegin contributes
#pragma unroll
            for (int j = 0; j < 32; j++)
                if (k + j < a.kbegin) w[j] = 0.0f;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; j++) w[j] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 4; j++) split_store8(w + 8 * j, a_hi + core_off(row, half * 4 + j), a_lo + core_off(row, half * 4 + j));
}

// This thread's 32 weights of one chunk from a raw Q8 tile in shared memory (-> bf16 hi/lo).
__device__ __forceinline__ void stage_w_raw(const uint8_t* raw, const GemmArgs& a, int n, int k, uint8_t* a_hi,
                                            uint8_t* a_lo, int row, int half) {
    float w[32];
    if (n < a.N) {
        const int4 p0 = *reinterpret_cast<const int4*>(raw + ((half * 2 + 0) * TC_M + row) * 16);
        const int4 p1 = *reinterpret_cast<const int4*>(raw + ((half * 2 + 1) * TC_M + row) * 16);
        const float sc = reinterpret_cast<const float*>(raw + TC_M * TC_KC)[half * TC_M + row];
        const int8_t* q0 = reinterpret_cast<const int8_t*>(&p0);
        const int8_t* q1 = reinterpret_cast<const int8_t*>(&p1);
#pragma unroll
        for (int j = 0; j < 16; j++) {
            w[j] = (float)q0[j] * sc;
            w[16 + j] = (float)q1[j] * sc;
        }
        if (k < a.kbegin) {  // faithful mode: only k >= kbegin contributes
#pragma unroll
            for (int j = 0; j < 32; j++)
                if (k + j < a.kbegin) w[j] = 0.0f;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; j++) w[j] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 4; j++) split_store8(w + 8 * j, a_hi + core_off(row, half * 4 + j), a_lo + core_off(row, half * 4 + j));
}

// 16 activations of token row r (K quarter kq of a chunk), times the RMSNorm gain when
// there is one -> bf16 hi/lo.  The row's 1/rms is applied to the accumulators instead.
__device__ __forceinline__ void stage_x16(const float4* x4, const float* g, bool valid, uint8_t* b_hi, uint8_t* b_lo,
                                          int r, int kq) {
    float xv[16];
    if (valid) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            xv[4 * i] = x4[i].x; xv[4 * i + 1] = x4[i].y; xv[4 * i + 2] = x4[i].z; xv[4 * i + 3] = x4[i].w;
        }
        if (g) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float4 g4 = reinterpret_cast<const float4*>(g)[i];
                xv[4 * i] *= g4.x;
                xv[4 * i + 1] *= g4.y;
                xv[4 * i + 2] *= g4.z;
                xv[4 * i + 3] *= g4.w;
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; i++) xv[i] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 2; j++) split_store8(xv + 8 * j, b_hi + core_off(r, kq * 2 + j), b_lo + core_off(r, kq * 2 + j));
}

// The activation tile of one chunk (all NT token rows), loaded and staged by unit.
template <int NT>
__device__ __forceinline__ void stage_chunk_x(const GemmArgs& a, const float* g, int m_base, int k0, uint8_t* b_hi,
                                              uint8_t* b_lo, int tid) {
    for (int u = tid; u < NT * 4; u += TC_WORKERS) {
        const int r = u >> 2, kq = u & 3, m = m_base + r;
        float4 x4[4];
        if (m < a.M) {
            const float4* src = reinterpret_cast<const float4*>(a.x + (int64_t)m * a.ldx + k0 + kq * 16);
#pragma unroll
            for (int i = 0; i < 4; i++) x4[i] = src[i];
        }
        stage_x16(x4, g ? g + kq * 16 : nullptr, m < a.M, b_hi, b_lo, r, kq);
    }
}

__device__ __forceinline__ void issue_chunk_mmas(uint32_t tmem, uint32_t idesc, const uint8_t* a_hi, const uint8_t* a_lo,
                                                 const uint8_t* b_hi, const uint8_t* b_lo, bool first) {
    const uint32_t ah = smem_addr(a_hi), al = smem_addr(a_lo), bh = smem_addr(b_hi), bl = smem_addr(b_lo);
#pragma unroll
    for (int kk = 0; kk < TC_KC / 16; kk++) {
        const uint32_t o = kk * 256;  // 16 K-elements = two core matrices along K
        umma_bf16(tmem, umma_desc(ah + o), umma_desc(bh + o), idesc, (!first || kk > 0) ? 1u : 0u);
        umma_bf16(tmem, umma_desc(ah + o), umma_desc(bl + o), idesc, 1u);
        umma_bf16(tmem, umma_desc(al + o), umma_desc(bh + o), idesc, 1u);
    }
}

template <int NT, bool F32W, int EPI>
__global__ void __launch_bounds__(TC_THREADS, EPI == kEpiLogits ? 2 : 1) tc_gemm_kernel(GemmArgs a, Epilogue e, SplitArgs sp) {
    using S = TcSmem<NT>;
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint64_t mma_bar[TC_MAX_STAGES];
    __shared__ uint64_t w_bar[TC_MAX_STAGES];  // tiled weights: the stage's bulk copy has landed
    __shared__ uint64_t raw_bar[TC_RAW_MAX];   // raw Q8 tiles: the slot's bulk copy has landed
    __shared__ uint64_t done_bar;
    __shared__ uint64_t recv_bar;  // split K: the partials of this CTA's slice have all arrived
    __shared__ uint32_t tmem_slot;
    __shared__ float inv_rms[NT];
    // per-warp-quarter column reductions of the epilogue (argmax keys, sums of squares) in
    // stage memory, which is free once every MMA has completed
    unsigned long long* red_key = reinterpret_cast<unsigned long long*>(smem);  // [4][NT]
    float* red_ss = reinterpret_cast<float*>(smem + 4 * NT * 8);                 // [4][NT]
    const int epi = EPI >= 0 ? EPI : e.kind;  // EPI < 0: the epilogue kind is read at run time

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool worker = warp < kIssuerWarp;  // else: the warp whose lane 0 issues the MMAs
    const int row = tid & (TC_M - 1), wg = (tid >> 7) & 1;  // weight row / TMEM lane, warpgroup = K half
    // grid (ksplit, n_tiles, m_tiles); the ksplit CTAs of one tile form one cluster
    const int split = blockIdx.x, n_tile = blockIdx.y, m_tile = blockIdx.z;
    const int n_base = n_tile * TC_M, m_base = m_tile * NT;
    const int nchunk_total = a.K / TC_KC;
    const int c_begin = (int)((int64_t)split * nchunk_total / sp.ksplit);
    const int c_end = (int)((int64_t)(split + 1) * nchunk_total / sp.ksplit);
    // the reference's batched arithmetic keeps only the last 32-wide block (kbegin = K-32)
    const int c_first = max(c_begin, a.kbegin / TC_KC);
    const int nch = max(0, c_end - c_first);
    const int stages = sp.stages;
    const int ks = sp.ksplit;
    // raw Q8 tiles streamed through a ring of sp.raw_slots bulk copies (large matrices)
    const bool use_raw = !F32W && a.wr != nullptr && a.wt == nullptr && sp.raw_slots >= 2;
    const int RS = sp.raw_slots;
    // every chunk of this CTA has its own stage: all weights are staged before waiting for
    // the previous kernel (weights are read-only; activations are not)
    const bool staged = nch <= stages && !use_raw;
    // 128/256-token tiles in a ring over hi/lo weight tiles: the activations come pre-split
    // (tc_split_x_kernel, a.xs_tiles) and are bulk-copied with each weight tile instead of
    // being converted by every CTA of the launch
    const bool xs = NT >= 128 && !F32W && a.xs_tiles != nullptr && a.wt != nullptr && !staged && !use_raw;
    const int n = n_base + row;  // this thread's weight row
    auto stage_ptr = [&](int st, int part) { return smem + st * S::STAGE + (part < 2 ? part * S::A_BYTES : 2 * S::A_BYTES + (part - 2) * S::B_BYTES); };
    float* gain_s = reinterpret_cast<float*>(smem + sp.gain_off);  // [nch][64] when staged

    // Columns (tokens) this CTA finishes: its slice of the tile when K is split, else all;
    // warpgroup wg takes half of them.
    const int slice = NT / ks;  // multiple of 8
    int rank = 0;
    if (ks > 1) rank = (int)cg::this_cluster().block_rank();
    const int fin_begin = ks > 1 ? rank * slice : 0;
    const int fin_cols = ks > 1 ? slice : NT;
    const int my_cols = fin_cols / 2;  // multiple of 4
    const int my_begin = fin_begin + wg * my_cols;
    constexpr int PRE = 8;  // epilogue columns whose inputs are fetched early

    if (warp == 0) {
        tmem_alloc(&tmem_slot, NT);
        tmem_relinquish();
    }
    if (tid == 0) {
        for (int st = 0; st < TC_MAX_STAGES; st++) {
            mbar_init(&mma_bar[st], 1);
            mbar_init(&w_bar[st], xs ? 2 : 1);  // xs: the weight and the activation copies arrive
        }
        for (int r = 0; r < TC_RAW_MAX; r++) mbar_init(&raw_bar[r], 1);
        mbar_init(&done_bar, 1);
        mbar_init(&recv_bar, 1);
        if (ks > 1) mbar_arrive_expect_tx(&recv_bar, (uint32_t)(TC_M * NT * 4));  // ks partials of slice x 128 rows
        fence_barrier_init();
    }
    // the peers may push into this CTA's receive buffer once its barrier exists: arrive
    // here, wait right before the first push
    if (ks > 1) cluster_arrive_release();
    // ---- before the grid dependency: everything that does not depend on the previous kernel
    WRegs<F32W> cur;
    // tiled weights: one bulk copy per chunk (all of them when staged, the first for a ring)
    auto fetch_tile = [&](int i, int st) {
        mbar_arrive_expect_tx(&w_bar[st], TC_TILE_BYTES);
        bulk_g2s(stage_ptr(st, 0), a.wt + ((size_t)n_tile * nchunk_total + c_first + i) * TC_TILE_BYTES, TC_TILE_BYTES,
                 &w_bar[st]);
    };
    auto fetch_xtile = [&](int i, int st) {  // xs: chunk c_first + i's activation rows m_base.. (hi, lo)
        const uint8_t* src = a.xs_tiles + (size_t)(c_first + i) * 2 * a.xs_rows * 128 + (size_t)(m_base / 8) * 1024;
        mbar_arrive_expect_tx(&w_bar[st], 2u * NT * 128u);
        bulk_g2s(stage_ptr(st, 2), src, NT * 128, &w_bar[st]);
        bulk_g2s(stage_ptr(st, 3), src + (size_t)a.xs_rows * 128, NT * 128, &w_bar[st]);
    };
    uint8_t* raw_ring = smem + sp.raw_off;
    auto fetch_raw = [&](int i) {  // chunk i -> slot i % RS
        uint64_t* bar = &raw_bar[i % RS];
        mbar_arrive_expect_tx(bar, TC_RAW_BYTES);
        bulk_g2s(raw_ring + (size_t)(i % RS) * TC_RAW_BYTES,
                 a.wr + ((size_t)n_tile * nchunk_total + c_first + i) * TC_RAW_BYTES, TC_RAW_BYTES, bar);
    };
    if (use_raw) {
        if (tid == 0)
            for (int i = 0; i < min(nch, RS); i++) fetch_raw(i);
    } else if (a.wt) {
        if (tid == 0)
            for (int i = 0; i < min(nch, stages); i++) fetch_tile(i, i);
        if (staged && a.norm_gain)
            for (int t = tid; t < nch * (TC_KC / 4); t += TC_THREADS)
                reinterpret_cast<float4*>(gain_s)[t] =
                    __ldg(reinterpret_cast<const float4*>(a.norm_gain + c_first * TC_KC) + t);
    } else if (staged && worker) {
        if (a.norm_gain)
            for (int t = tid; t < nch * (TC_KC / 4); t += TC_THREADS)
                reinterpret_cast<float4*>(gain_s)[t] =
                    __ldg(reinterpret_cast<const float4*>(a.norm_gain + c_first * TC_KC) + t);
        if (nch >= 2) {
            WRegs<F32W> r1;
            load_w<F32W>(cur, a, n, c_first * TC_KC + wg * 32);
            load_w<F32W>(r1, a, n, (c_first + 1) * TC_KC + wg * 32);
            stage_w<F32W>(cur, a, n, c_first * TC_KC + wg * 32, stage_ptr(0, 0), stage_ptr(0, 1), row, wg);
            stage_w<F32W>(r1, a, n, (c_first + 1) * TC_KC + wg * 32, stage_ptr(1, 0), stage_ptr(1, 1), row, wg);
            for (int i = 2; i < nch; i++) {
                load_w<F32W>(cur, a, n, (c_first + i) * TC_KC + wg * 32);
                stage_w<F32W>(cur, a, n, (c_first + i) * TC_KC + wg * 32, stage_ptr(i, 0), stage_ptr(i, 1), row, wg);
            }
        } else if (nch == 1) {
            load_w<F32W>(cur, a, n, c_first * TC_KC + wg * 32);
            stage_w<F32W>(cur, a, n, c_first * TC_KC + wg * 32, stage_ptr(0, 0), stage_ptr(0, 1), row, wg);
        }
    } else if (nch > 0 && worker && !use_raw) {
        load_w<F32W>(cur, a, n, c_first * TC_KC + wg * 32);
    }
    // QKV: where this thread's row goes (q row, or a K/V pool column) and the token
    // positions, pages and rotary factors of its first PRE epilogue columns (the decode
    // descriptors are written before the step's first kernel)
    int pos_pre[EPI == kEpiQKV || EPI < 0 ? PRE : 1], page_pre[EPI == kEpiQKV || EPI < 0 ? PRE : 1];
    float fcr_pre[EPI == kEpiQKV || EPI < 0 ? PRE : 1], fci_pre[EPI == kEpiQKV || EPI < 0 ? PRE : 1];
    const int np = n & ~1;
    int qkv_kind = 3, fbase = 0;  // 0 q, 1 k, 2 v, 3 none; rotary pair index of the row
    int64_t row_off = 0;          // q: column in q_out; k/v: offset inside page 0's tile row
    float* pool = nullptr;
    if (epi == kEpiQKV) {
        const int D = e.dim, KV = e.kv_dim, hd = e.head_dim;
        if (n < a.N) {
            if (np < D) {
                qkv_kind = 0;
                row_off = n;
                fbase = (np % hd) >> 1;
            } else {
                const int cidx = np < D + KV ? n - D : n - D - KV;
                qkv_kind = np < D + KV ? 1 : 2;
                pool = qkv_kind == 1 ? e.kpool : e.vpool;
                row_off = e.geom.tile_offset(0, e.layer, cidx / hd) + cidx % hd;
                fbase = ((cidx & ~1) % hd) >> 1;
            }
        }
        const bool rope = qkv_kind < 2;
#pragma unroll
        for (int j = 0; j < PRE; j++) {
            const int m = min(m_base + my_begin + j, a.M - 1);
            pos_pre[j] = e.tok_pos[m];
            page_pre[j] = e.tok_page[m];
        }
#pragma unroll
        for (int j = 0; j < PRE; j++) {
            fcr_pre[j] = 1.0f;
            fci_pre[j] = 0.0f;
            if (rope && j < my_cols) {
                const int fi = pos_pre[j] * (hd >> 1) + fbase;
                fcr_pre[j] = e.freq_re[fi];
                fci_pre[j] = e.freq_im[fi];
            }
        }
    }

    grid_dependency_wait();
    // ---- after it: activations, RMS sums, residual inputs
    // 64-token tiles with every chunk staged: the activation units of all chunks are
    // requested before the RMS partial sums so the round trips overlap
    float4 xr[S::MAX_STAGES][NT == 64 ? 4 : 1];
    const int ur = tid >> 2, ukq = tid & 3;  // NT == 64: this thread's activation unit
    if (NT == 64 && staged && worker) {
#pragma unroll
        for (int i = 0; i < S::MAX_STAGES; i++) {
            if (i < nch && m_base + ur < a.M) {
                const float4* src = reinterpret_cast<const float4*>(a.x + (int64_t)(m_base + ur) * a.ldx +
                                                                    (c_first + i) * TC_KC + ukq * 16);
#pragma unroll
                for (int j = 0; j < 4; j++) xr[i][j] = src[j];
            }
        }
    }
    float xo_pre[EPI == kEpiResidual || EPI < 0 ? PRE : 1];
    if (epi == kEpiResidual) {
#pragma unroll
        for (int j = 0; j < PRE; j++) {
            const int m = m_base + my_begin + j;
            xo_pre[j] = (j < my_cols && m < a.M && n < a.N) ? e.out[(int64_t)m * e.ldo + n] : 0.0f;
        }
    }
    // RMSNorm: a token's 1/rms scales its accumulators in the epilogue (the sum over k is
    // linear), so the sums of squares are needed only after the MMAs.  64-token tiles
    // request them after staging (they would hold up the staging barrier), four threads
    // per token, and add them up while the MMAs run.
    constexpr int SSP = 8;
    float ssv[SSP];
    const bool ss_pre = NT == 64 && a.norm_gain && a.ss_in && a.ss_parts <= 4 * SSP;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const uint32_t idesc = umma_idesc_bf16(TC_M, NT);

    // Workers convert each chunk's activations (and, without tiled weights in a ring, its
    // weights) into the chunk's stage and arrive on named barrier 1 + stage; the issuer
    // warp syncs on it and its lane 0 issues the chunk's MMAs, so MMAs run while the next
    // chunk is converted.  Every wait is bounded; a thread whose wait gave up still takes
    // every barrier (skipping its work), so no party is left waiting.
    bool ok = true;
    if (worker) {
        if (staged) {
            for (int i = 0; i < nch; i++) {
                const float* g = a.norm_gain ? gain_s + i * TC_KC : nullptr;
                if (NT == 64) {
                    const int m = m_base + ur;
                    float4 x4[4];
#pragma unroll
                    for (int j = 0; j < 4; j++) x4[j] = xr[0][j];
#pragma unroll
                    for (int s2 = 1; s2 < S::MAX_STAGES; s2++)
                        if (i == s2)
#pragma unroll
                            for (int j = 0; j < 4; j++) x4[j] = xr[s2][j];
                    stage_x16(x4, g ? g + ukq * 16 : nullptr, m < a.M, stage_ptr(i, 2), stage_ptr(i, 3), ur, ukq);
                } else {
                    stage_chunk_x<NT>(a, g, m_base, (c_first + i) * TC_KC, stage_ptr(i, 2), stage_ptr(i, 3), tid);
                }
                fence_async_smem();
                named_arrive(1 + i, TC_THREADS);
            }
        } else {
            // 64-token tiles of the Q8 kernel: this thread's activation unit and gain slice of
            // the next chunk are requested one chunk ahead (the fp32-weight classifier kernel,
            // limited to 96 registers for two CTAs per SM, loads them per chunk)
            constexpr bool XPF = NT <= 128 && !F32W;
            constexpr int XU = NT <= 128 ? NT / 64 : 1;  // activation units per thread
            float4 xn[XU][4], gn[4];
            auto fetch_x = [&](int it) {
                const int k = (c_first + it) * TC_KC + ukq * 16;
#pragma unroll
                for (int u = 0; u < XU; u++)
                    if (m_base + ur + 64 * u < a.M) {
                        const float4* src =
                            reinterpret_cast<const float4*>(a.x + (int64_t)(m_base + ur + 64 * u) * a.ldx + k);
#pragma unroll
                        for (int j = 0; j < 4; j++) xn[u][j] = src[j];
                    }
                if (a.norm_gain) {
                    const float4* g4 = reinterpret_cast<const float4*>(a.norm_gain + k);
#pragma unroll
                    for (int j = 0; j < 4; j++) gn[j] = __ldg(g4 + j);
                }
            };
            if (XPF && !xs && nch > 0) fetch_x(0);
            for (int it = 0; it < nch; it++) {
                const int st = it % stages, use = it / stages;
                const int k0 = (c_first + it) * TC_KC;
                WRegs<F32W> nxt;
                if (!a.wt && !use_raw && it + 1 < nch) load_w<F32W>(nxt, a, n, k0 + TC_KC + wg * 32);
                // the stage was last read by the MMAs of chunk it - stages
                if (ok && use > 0 && !mbar_wait(&mma_bar[st], (use - 1) & 1, a.err)) ok = false;
                if (ok && use_raw && !mbar_wait(&raw_bar[it % RS], (it / RS) & 1, a.err)) ok = false;
                if (ok) {
                    if (use_raw)
                        stage_w_raw(raw_ring + (size_t)(it % RS) * TC_RAW_BYTES, a, n, k0 + wg * 32, stage_ptr(st, 0),
                                    stage_ptr(st, 1), row, wg);
                    else if (!a.wt)
                        stage_w<F32W>(cur, a, n, k0 + wg * 32, stage_ptr(st, 0), stage_ptr(st, 1), row, wg);
                    if (xs) {
                        // the issuer's bulk copy brings this chunk's activations
                    } else if (XPF) {
#pragma unroll
                        for (int u = 0; u < XU; u++)
                            stage_x16(xn[u], a.norm_gain ? reinterpret_cast<const float*>(gn) : nullptr,
                                      m_base + ur + 64 * u < a.M, stage_ptr(st, 2), stage_ptr(st, 3), ur + 64 * u, ukq);
                    } else {
                        stage_chunk_x<NT>(a, a.norm_gain ? a.norm_gain + k0 : nullptr, m_base, k0, stage_ptr(st, 2),
                                          stage_ptr(st, 3), tid);
                    }
                }
                // the next chunk's activations (and gain) load while this one goes through
                // the barrier and the MMAs
                if (XPF && !xs && it + 1 < nch) fetch_x(it + 1);
                fence_async_smem();
                named_arrive(1 + st, TC_THREADS);
                if (!a.wt && !use_raw && it + 1 < nch) cur = nxt;
            }
        }
    } else {
        // issuer warp; with tiled weights in a ring, lane 0 also refills each stage with the
        // tile of chunk it - 1 + stages once the MMAs of chunk it - 1 are done with it (xs:
        // and its activations; the first stages' activations once they exist)
        if (xs && lane == 0)
            for (int i = 0; i < min(nch, stages); i++) fetch_xtile(i, i);
        for (int it = 0; it < nch; it++) {
            const int st = staged ? it : it % stages, use = staged ? 0 : it / stages;
            if (!staged && a.wt && lane == 0 && ok && it >= 1 && it - 1 + stages < nch) {
                const int sp_ = (it - 1) % stages;
                if (mbar_wait(&mma_bar[sp_], ((it - 1) / stages) & 1, a.err)) {
                    fetch_tile(it - 1 + stages, sp_);
                    if (xs) fetch_xtile(it - 1 + stages, sp_);
                } else {
                    ok = false;
                }
            }
            // raw ring: the workers converted chunk it - 1 before the barrier this warp passed
            // last iteration, so its slot takes chunk it - 1 + RS
            if (use_raw && lane == 0 && it >= 1 && it - 1 + RS < nch) fetch_raw(it - 1 + RS);
            __syncwarp();
            named_sync(1 + st, TC_THREADS);
            if (lane == 0) {
                if (a.wt && ok && !mbar_wait(&w_bar[st], use & 1, a.err)) ok = false;
                tc_fence_after();
                if (ok)
                    issue_chunk_mmas(tmem, idesc, stage_ptr(st, 0), stage_ptr(st, 1), stage_ptr(st, 2), stage_ptr(st, 3), it == 0);
                if (!staged) umma_commit(&mma_bar[st]);  // always, so the stage's phases stay in step
            }
            __syncwarp();
        }
        if (lane == 0 && nch > 0) umma_commit(&done_bar);  // completes after every MMA above
    }
    // the sums of squares are needed only after the MMAs: requested once staging is done
    if (ss_pre && worker) {
        const int m = m_base + ur;
#pragma unroll
        for (int i = 0; i < SSP; i++) {
            const int p = ukq + 4 * i;
            ssv[i] = (m < a.M && p < a.ss_parts) ? __ldcg(a.ss_in + (int64_t)p * a.ss_ld + m) : 0.0f;
        }
    }
    // 1/rms per token while the MMAs run
    if (a.norm_gain && worker) {
        if (ss_pre) {
            float ss = 0.0f;
#pragma unroll
            for (int i = 0; i < SSP; i++) ss += ssv[i];
            ss += __shfl_xor_sync(0xffffffffu, ss, 1);
            ss += __shfl_xor_sync(0xffffffffu, ss, 2);
            if (ukq == 0) inv_rms[ur] = 1.0f / sqrtf(ss / (float)a.K + 1e-5f);
        } else if (a.ss_in) {
            // sums of squares published by the producer of x, one per 128-feature slice;
            // four threads per token, joined by two shuffles
            for (int u = tid; u < NT * 4; u += TC_WORKERS) {
                const int r = u >> 2, p0 = u & 3, m = m_base + r;
                float ss = 0.0f;
                if (m < a.M)
                    for (int p = p0; p < a.ss_parts; p += 4) ss += __ldcg(a.ss_in + (int64_t)p * a.ss_ld + m);
                ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                if (p0 == 0) inv_rms[r] = 1.0f / sqrtf(ss / (float)a.K + 1e-5f);
            }
        } else {
            const int nw = TC_WORKERS / 32;
            for (int r = warp; r < NT; r += nw) {
                const int m = m_base + r;
                float ss = 0.0f;
                if (m < a.M) {
                    const float* xrow = a.x + (int64_t)m * a.ldx;
                    for (int k = lane * 4; k < a.K; k += 128) {
                        float4 v = *reinterpret_cast<const float4*>(xrow + k);
                        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                    }
                }
                ss = warp_sum(ss);
                if (lane == 0) inv_rms[r] = 1.0f / sqrtf(ss / (float)a.K + 1e-5f);
            }
        }
    }
    bool bail = false;
    {   // every MMA done (and inv_rms published)
        const bool got = nch > 0 ? mbar_wait(&done_bar, 0, a.err) : true;
        if (!__syncthreads_and(got && ok)) bail = true;
    }
    tc_fence_after();
    grid_dependents_launch();

    // Accumulators.  With K split over a cluster, token slice r of the tile belongs to the
    // cluster's CTA r: every CTA sends its partial of slice r straight into CTA r's receive
    // buffer ([ks][128][slice + 4] fp32, row-major per thread) with asynchronous 16-byte
    // distributed-shared-memory stores that count down CTA r's receive barrier, and CTA r
    // sums its slice locally in rank order (deterministic) once all ks x 128 x slice values
    // are in.  A CTA whose wait gave up sends zeros so its peers still complete.  Without a
    // split the epilogue reads TMEM directly.
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const int rst = slice + sp.recv_pad;  // padded: the 8 rows of a 16-byte phase hit 8 bank groups
    float* recv = reinterpret_cast<float*>(smem + sp.recv_off);
    if (ks > 1 && !worker) cluster_wait_acquire();
    if (ks > 1 && worker) {
        const int half = NT / 2;
        const uint32_t my_recv = smem_addr(recv + ((size_t)rank * TC_M + row) * rst);
        const uint32_t my_bar = smem_addr(&recv_bar);
        for (int c32 = wg * half; c32 < (wg + 1) * half; c32 += 32) {
            float v[32];
            if (nch > 0 && !bail) {
                tmem_ld32(tl + c32, v);
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] = 0.0f;
            }
            if (c32 == wg * half) cluster_wait_acquire();  // every peer's receive barrier is initialised
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int c0 = c32 + 8 * u;
                const int q = c0 / slice;
                const uint32_t dst = map_rank(my_recv + (uint32_t)(c0 - q * slice) * 4u, (uint32_t)q);
                const uint32_t bar = map_rank(my_bar, (uint32_t)q);
                st_async4(dst, v[8 * u], v[8 * u + 1], v[8 * u + 2], v[8 * u + 3], bar);
                st_async4(dst + 16u, v[8 * u + 4], v[8 * u + 5], v[8 * u + 6], v[8 * u + 7], bar);
            }
        }
    }
    if (ks > 1 && !__syncthreads_and(mbar_wait_cluster(&recv_bar, 0, a.err))) bail = true;
    if (bail) {  // a wait gave up (error flag set): release TMEM and leave
        tc_fence_before();
        __syncthreads();
        if (warp == 0) tmem_dealloc(tmem, NT);
        return;
    }
    const bool even = (n & 1) == 0;
    for (int c0 = my_begin; worker && c0 < my_begin + my_cols; c0 += 4) {
        const int jb = c0 - my_begin;  // index of the group's first column among this thread's
        float v[4];
        if (ks > 1) {
            const float* src = recv + (size_t)row * rst + (c0 - fin_begin);
            float4 s4 = reinterpret_cast<const float4*>(src)[0];
            for (int q = 1; q < ks; q++) {
                const float4 t4 = reinterpret_cast<const float4*>(src + (size_t)q * TC_M * rst)[0];
                s4.x += t4.x; s4.y += t4.y; s4.z += t4.z; s4.w += t4.w;
            }
            v[0] = s4.x; v[1] = s4.y; v[2] = s4.z; v[3] = s4.w;
        } else if (nch > 0) {
            tmem_ld4(tl + c0, v);
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++) v[j] = 0.0f;
        }
        if (a.norm_gain) {
#pragma unroll
            for (int j = 0; j < 4; j++) v[j] *= inv_rms[c0 + j];
        }
        // Epilogue of the group; every global load of the group comes before its stores.
        if (epi == kEpiLogits) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int c = c0 + j, m = m_base + c;
                const bool ok = m < a.M && n < a.N;
                if (ok && e.out) e.out[(int64_t)m * e.ldo + n] = v[j];
                unsigned long long key = (ok && v[j] > 0.0f) ? argmax_key(v[j], n) : 0ull;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
                    key = k2 > key ? k2 : key;
                }
                if (lane == 0) red_key[(warp & 3) * NT + c] = key;
            }
        } else if (epi == kEpiResidual) {
            float xo[4];
            if (jb == 0 || jb == 4) {  // fetched right after the grid dependency wait
#pragma unroll
                for (int j = 0; j < 4; j++) xo[j] = jb == 0 ? xo_pre[j] : xo_pre[4 + j];
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int m = m_base + c0 + j;
                    xo[j] = (m < a.M && n < a.N) ? e.out[(int64_t)m * e.ldo + n] : 0.0f;
                }
            }
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int c = c0 + j, m = m_base + c;
                const bool ok = m < a.M && n < a.N;
                const float xn = ok ? xo[j] + v[j] : 0.0f;
                if (ok) e.out[(int64_t)m * e.ldo + n] = xn;
                if (e.ss_out) {  // this tile's share of the next RMSNorm's sum of squares
                    const float sq = warp_sum(xn * xn);
                    if (lane == 0) red_ss[(warp & 3) * NT + c] = sq;
                }
            }
        } else if (epi == kEpiStore) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int m = m_base + c0 + j;
                if (m < a.M && n < a.N) e.out[(int64_t)m * e.ldo + n] = v[j];
            }
        } else {
            float other[4];
#pragma unroll
            for (int j = 0; j < 4; j++) other[j] = __shfl_xor_sync(0xffffffffu, v[j], 1);  // pair partner's row
            if (epi == kEpiSwiGLU) {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int m = m_base + c0 + j;
                    if (even && m < a.M && n < a.N) {
                        const float g = v[j];
                        const float hgate = g * (1.0f / (1.0f + expf(-g)));
                        e.out[(int64_t)m * e.ldo + (n >> 1)] = hgate * other[j];
                    }
                }
            } else if (epi == kEpiQKV) {
                const int D = e.dim, hd = e.head_dim;
                const bool rope = qkv_kind < 2;
                int pos[4], page[4];
                float fcr[4], fci[4];
                if (jb == 0 || jb == 4) {  // fetched before the grid dependency wait
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        pos[j] = jb == 0 ? pos_pre[j] : pos_pre[4 + j];
                        page[j] = jb == 0 ? page_pre[j] : page_pre[4 + j];
                        fcr[j] = jb == 0 ? fcr_pre[j] : fcr_pre[4 + j];
                        fci[j] = jb == 0 ? fci_pre[j] : fci_pre[4 + j];
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int m = min(m_base + c0 + j, a.M - 1);
                        pos[j] = e.tok_pos[m];
                        page[j] = e.tok_page[m];
                    }
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        fcr[j] = 1.0f; fci[j] = 0.0f;
                        if (rope) {
                            const int fi = pos[j] * (hd >> 1) + fbase;
                            fcr[j] = e.freq_re[fi];
                            fci[j] = e.freq_im[fi];
                        }
                    }
                }
                const int64_t pf = e.geom.page_stride();
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int m = m_base + c0 + j;
                    if (m >= a.M || qkv_kind == 3) continue;
                    const float v0 = even ? v[j] : other[j];  // value of row n & ~1
                    const float v1 = even ? other[j] : v[j];  // value of row n | 1
                    const float r = rope ? (even ? (v0 * fcr[j] - v1 * fci[j]) : (v0 * fci[j] + v1 * fcr[j])) : v[j];
                    if (qkv_kind == 0)
                        e.q_out[(int64_t)m * D + row_off] = r;
                    else
                        store_kv(pool, e.geom, (int64_t)page[j] * pf + (int64_t)(pos[j] & (kPage - 1)) * hd + row_off, r);
                }
            }
        }
    }
    if (epi == kEpiLogits || (epi == kEpiResidual && e.ss_out)) {
        __syncthreads();
        for (int cix = fin_begin + tid; cix < fin_begin + fin_cols; cix += TC_THREADS) {
            const int m = m_base + cix;
            if (m >= a.M) continue;
            if (epi == kEpiLogits) {
                unsigned long long best = red_key[cix];
#pragma unroll
                for (int w = 1; w < 4; w++) best = red_key[w * NT + cix] > best ? red_key[w * NT + cix] : best;
                if (best != 0ull) {
                    unsigned long long* slot = e.argmax_keys + m;
                    if (best > *(volatile unsigned long long*)slot) atomicMax(slot, best);
                }
            } else {
                e.ss_out[(int64_t)n_tile * e.ss_ld + m] = red_ss[cix] + red_ss[NT + cix] + red_ss[2 * NT + cix] + red_ss[3 * NT + cix];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, NT);
}

// ------------------------------------------------------------------ stream-K, batches of up to 64 rows
// Large Q8 projections at decode batches (3-64 token rows) are HBM-bound, but their
// 128-row tiles are too few to fill 148 SMs evenly (96 tiles for the 7B shape's q,k,v,
// 172 for w1/w3), and a cluster K split cannot keep every cluster resident.  So one CTA
// per SM takes an equal contiguous share of the (tile, 64-wide K chunk) units in
// tile-major order (the weight tiles' order in memory) and accumulates each tile's run of
// chunks in TMEM.  Operands arrive by bulk copy, issued by one thread several units ahead
// of the MMAs: the weights as pre-split hi/lo tiles straight into an A slot, or as raw Q8
// tiles into a ring that 16 worker warps convert into A slots; the activations as bf16
// hi/lo tiles that tc_split_x_kernel writes once per launch into scratch (the RMSNorm
// gain applied), so no unit waits on a global-load round trip.
// A share starts inside a tile at most once: the partial sums of that first run go to
// global scratch and a release flag is set.  The CTA whose share holds the tile's chunk 0
// (where that run ends its share) waits for the flags of the CTAs after it that cover the
// rest of the tile, adds their partials in CTA order (a fixed order: the result does not
// depend on timing), clears the flags for the next launch and runs the epilogue.  A partial
// is written at the start of its CTA's share and read at the end of an earlier CTA's, so
// the waits are short; every wait is bounded.
struct StreamKArgs {
    int units;      // n_tiles x chunks
    int chunks;     // K / 64
    int raw_slots;  // raw-tile ring slots (raw tiles only)
    int raw_off;    // byte offset of the raw ring in dynamic shared memory
    int xrows;      // activation rows copied per unit: the batch rounded up to 8
};

constexpr int SK_NT = 64;        // token columns per tile (the batch, zero-padded)
constexpr int SK_SB = 4;         // activation slots
constexpr uint32_t SK_XTILE = 2u * SK_NT * TC_KC * 2u;  // hi + lo halves of one 64 x 64 activation tile
constexpr int kSkWorkerBar = 8;  // named barrier of the worker warps (the stages use 1 and 2)

__host__ __device__ inline int sk_first_unit(int cta, int grid, int units) { return (int)((int64_t)cta * units / grid); }

// The CTA whose share holds unit u.
__device__ __forceinline__ int sk_cta_of(int u, int grid, int units) {
    int c = (int)(((int64_t)u * grid) / units);
    while (c + 1 < grid && sk_first_unit(c + 1, grid, units) <= u) c++;
    while (c > 0 && sk_first_unit(c, grid, units) > u) c--;
    return c;
}

// Bounded wait for another CTA's release flag.
__device__ __forceinline__ bool sk_wait_flag(const int* f, int* err) {
    if (ld_acquire_gpu(f)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; i++) {
        if (ld_acquire_gpu(f)) return true;
        if ((i & 15) == 0 && global_ns() - t0 > kWaitLimitNs) break;
    }
    if (err) atomicCAS(err, 0, kErrWaitTimeout);
    return false;
}

constexpr int SK_WORKERS = 512;               // conversion / epilogue threads: 16 warps
// + a producer warp (bulk copies) and two warps that issue the MMAs, alternating units
constexpr int SK_THREADS = SK_WORKERS + 3 * 32;
constexpr int kSkProducerWarp = SK_WORKERS / 32;
constexpr int kSkBarThreads = SK_WORKERS + 32;  // a stage barrier: the workers and one issuer warp
constexpr int SK_COLS = SK_NT / (SK_WORKERS / TC_M);  // epilogue columns per thread (16)

// Eight fp32 values -> bf16 hi/lo (hi = bf16(v), lo = bf16(v - hi)), one 16-byte core-matrix
// row each, in packed f32x2 arithmetic; w[i] holds values 2i, 2i+1.
__device__ __forceinline__ void split8_store(const unsigned long long w[4], uint8_t* hi_dst, uint8_t* lo_dst) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint32_t w0, w1;
        unpack2(w[i], w0, w1);
        __nv_bfloat162 hb = __floats2bfloat162_rn(__uint_as_float(w0), __uint_as_float(w1));
        h[i] = *reinterpret_cast<uint32_t*>(&hb);
        uint32_t r0, r1;
        unpack2(sub2(w[i], pack2(h[i] << 16, h[i] & 0xFFFF0000u)), r0, r1);
        __nv_bfloat162 lb = __floats2bfloat162_rn(__uint_as_float(r0), __uint_as_float(r1));
        l[i] = *reinterpret_cast<uint32_t*>(&lb);
    }
    *reinterpret_cast<uint4*>(hi_dst) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo_dst) = make_uint4(l[0], l[1], l[2], l[3]);
}

// This thread's 16 weights of one chunk (16-byte piece kq of row `row` in a raw tile):
// w = q * scale rounded once, as stage_w_raw, the int8 -> float step by byte permutes
// (exact), then bf16 hi/lo into K groups 2 kq and 2 kq + 1 of the row.
__device__ __forceinline__ void stage_w16_raw(const uint8_t* raw, uint8_t* a_hi, uint8_t* a_lo, int row, int kq) {
    const uint4 p = *reinterpret_cast<const uint4*>(raw + (kq * TC_M + row) * 16);
    const float sc = reinterpret_cast<const float*>(raw + TC_M * TC_KC)[(kq >> 1) * TC_M + row];
    const unsigned long long sc2 = pack2(__float_as_uint(sc), __float_as_uint(sc)), unb = q8_unbias2();
    const uint32_t words[4] = {p.x ^ 0x80808080u, p.y ^ 0x80808080u, p.z ^ 0x80808080u, p.w ^ 0x80808080u};
#pragma unroll
    for (int g = 0; g < 2; g++) {
        unsigned long long w[4];
#pragma unroll
        for (int i = 0; i < 4; i++) w[i] = mul2(add2(q8_pair_biased(words[2 * g + (i >> 1)], (i & 1) * 2), unb), sc2);
        split8_store(w, a_hi + core_off(row, 2 * kq + g), a_lo + core_off(row, 2 * kq + g));
    }
}

// The RESIDUAL epilogue's inputs (the residual rows) of one thread's columns, loaded early.
__device__ __forceinline__ void sk_residual_in(const GemmArgs& a, const Epilogue& e, float* xo, int n, int c_base) {
#pragma unroll
    for (int j = 0; j < SK_COLS; j++) {
        const int m = c_base + j;
        xo[j] = (e.kind == kEpiResidual && n < a.N && m < a.M) ? e.out[(int64_t)m * e.ldo + n] : 0.0f;
    }
}

// Epilogue of one thread's SK_COLS token columns c_base.. of weight row n (xo: the residual
// inputs from sk_residual_in); the RESIDUAL kind leaves each column's sum of squares over
// the warp's 32 rows in red_ss.
__device__ __forceinline__ void sk_epilogue(const GemmArgs& a, const Epilogue& e, float* v, const float* xo, int n,
                                            int c_base, const float* inv_rms, float* red_ss, int warp, int lane,
                                            bool ok) {
    const int epi = e.kind;
    if (a.norm_gain) {
#pragma unroll
        for (int j = 0; j < SK_COLS; j++) v[j] *= inv_rms[c_base + j];
    }
    const bool nrow = ok && n < a.N;
    if (epi == kEpiStore) {
#pragma unroll
        for (int j = 0; j < SK_COLS; j++) {
            const int m = c_base + j;
            if (nrow && m < a.M) e.out[(int64_t)m * e.ldo + n] = v[j];
        }
    } else if (epi == kEpiResidual) {
#pragma unroll
        for (int j = 0; j < SK_COLS; j++) {
            const int m = c_base + j;
            const bool w = nrow && m < a.M;
            const float xn = w ? xo[j] + v[j] : 0.0f;
            if (w) e.out[(int64_t)m * e.ldo + n] = xn;
            if (e.ss_out) {
                const float sq = warp_sum(xn * xn);
                if (lane == 0) red_ss[(warp & 3) * SK_NT + m] = sq;
            }
        }
    } else if (epi == kEpiSwiGLU) {
        const bool even = (n & 1) == 0;
#pragma unroll
        for (int j = 0; j < SK_COLS; j++) {
            const int m = c_base + j;
            const float other = __shfl_xor_sync(0xffffffffu, v[j], 1);  // w3 row next to this w1 row
            if (even && nrow && m < a.M) {
                const float g = v[j];
                e.out[(int64_t)m * e.ldo + (n >> 1)] = g * (1.0f / (1.0f + expf(-g))) * other;
            }
        }
    } else if (epi == kEpiQKV) {
        const int D = e.dim, KV = e.kv_dim, hd = e.head_dim;
        const int np = n & ~1;
        const bool even = (n & 1) == 0;
        int kind = 3, fbase = 0;  // 0 q, 1 k, 2 v, 3 none
        int64_t row_off = 0;
        float* pool = nullptr;
        if (nrow) {
            if (np < D) {
                kind = 0;
                row_off = n;
                fbase = (np % hd) >> 1;
            } else {
                const int cidx = np < D + KV ? n - D : n - D - KV;
                kind = np < D + KV ? 1 : 2;
                pool = kind == 1 ? e.kpool : e.vpool;
                row_off = e.geom.tile_offset(0, e.layer, cidx / hd) + cidx % hd;
                fbase = ((cidx & ~1) % hd) >> 1;
            }
        }
        const bool rope = kind < 2;
        const int64_t pf = e.geom.page_stride();
#pragma unroll
        for (int j = 0; j < SK_COLS; j++) {
            const int m = c_base + j;
            const float other = __shfl_xor_sync(0xffffffffu, v[j], 1);  // the rotary pair's other row
            if (m >= a.M || kind == 3) continue;
            const int pos = e.tok_pos[m];
            float r = v[j];
            if (rope) {
                const int fi = pos * (hd >> 1) + fbase;
                const float fcr = e.freq_re[fi], fci = e.freq_im[fi];
                const float v0 = even ? v[j] : other, v1 = even ? other : v[j];
                r = even ? (v0 * fcr - v1 * fci) : (v0 * fci + v1 * fcr);
            }
            if (kind == 0)
                e.q_out[(int64_t)m * D + row_off] = r;
            else
                store_kv(pool, e.geom, (int64_t)e.tok_page[m] * pf + (int64_t)(pos & (kPage - 1)) * hd + row_off, r);
        }
    }
}

// The activations of one launch as bf16 hi/lo tiles in the UMMA layout, per 64-wide K
// chunk [hi: rows_pad x 128 B][lo: rows_pad x 128 B] (8-row core-matrix groups of 1 KB),
// x times the RMSNorm gain; rows from the batch up to xrows are zero.  One thread per
// (chunk, row < xrows, 8-wide K group).  The stream-K kernel uses rows_pad = 64 (16 KB
// per chunk); the cluster kernel's 128/256-token tiles copy rows m_base.. of it.
__global__ void __launch_bounds__(256) tc_split_x_kernel(GemmArgs a, int xrows, int rows_pad, uint8_t* out) {
    grid_dependency_wait();  // x comes from the previous kernel
    grid_dependents_launch();
    const int chunks = a.K / TC_KC;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (int64_t)chunks * xrows * 8) return;
    const int c = (int)(t / (xrows * 8)), rem = (int)(t % (xrows * 8));
    const int r = rem >> 3, g = rem & 7;
    const int k = c * TC_KC + g * 8;
    unsigned long long w[4] = {0ull, 0ull, 0ull, 0ull};
    if (r < a.M) {
        const float4* src = reinterpret_cast<const float4*>(a.x + (int64_t)r * a.ldx + k);
        float4 x0 = src[0], x1 = src[1];
        if (a.norm_gain) {
            const float4 g0 = __ldg(reinterpret_cast<const float4*>(a.norm_gain + k));
            const float4 g1 = __ldg(reinterpret_cast<const float4*>(a.norm_gain + k) + 1);
            x0.x *= g0.x; x0.y *= g0.y; x0.z *= g0.z; x0.w *= g0.w;
            x1.x *= g1.x; x1.y *= g1.y; x1.z *= g1.z; x1.w *= g1.w;
        }
        w[0] = pack2(__float_as_uint(x0.x), __float_as_uint(x0.y));
        w[1] = pack2(__float_as_uint(x0.z), __float_as_uint(x0.w));
        w[2] = pack2(__float_as_uint(x1.x), __float_as_uint(x1.y));
        w[3] = pack2(__float_as_uint(x1.z), __float_as_uint(x1.w));
    }
    uint8_t* tile = out + (size_t)c * 2 * rows_pad * 128;
    split8_store(w, tile + core_off(r, g), tile + (size_t)rows_pad * 128 + core_off(r, g));
}

// The 12 MMAs of one 64-wide K chunk (hi*hi + hi*lo + lo*hi per 16-wide K step) from
// descriptors made once per slot (a K step is 256 B further: +16 in the address field).
__device__ __forceinline__ void issue_unit_mmas(uint32_t d, uint32_t idesc, uint64_t dah, uint64_t dal, uint64_t dbh,
                                                uint64_t dbl, bool first) {
#pragma unroll
    for (int kk = 0; kk < TC_KC / 16; kk++) {
        const uint64_t o = (uint64_t)kk * 16;
        umma_bf16(d, dah + o, dbh + o, idesc, (!first || kk > 0) ? 1u : 0u);
        umma_bf16(d, dah + o, dbl + o, idesc, 1u);
        umma_bf16(d, dal + o, dbh + o, idesc, 1u);
    }
}

// WT: the weights come as pre-split hi/lo tiles (tc_tile_weights), bulk-copied straight
// into an A slot (no conversion, 4 slots); otherwise as raw Q8 tiles that the workers
// convert into 2 A slots.  Warps: 0-15 workers (raw conversion, epilogues), 16 producer
// (every bulk copy), 17-18 MMA issuers: unit it goes to issuer it % 2, which accumulates
// it into its own TMEM accumulator of the run (4 x 64 columns: 2 runs in flight x 2
// issuers); the epilogue adds the run's two accumulators in issuer order.
template <bool WT>
__global__ void __launch_bounds__(SK_THREADS, 1) tc_streamk_kernel(GemmArgs a, Epilogue e, StreamKArgs sk) {
    constexpr int NT = SK_NT;
    constexpr int SA = WT ? 4 : 2;  // weight (A) slots
    constexpr int SB = SK_SB;       // activation (B) slots
    constexpr uint32_t A_BYTES = TC_M * TC_KC * 2;  // one bf16 half of a weight tile
    constexpr uint32_t B_BYTES = NT * TC_KC * 2;    // one bf16 half of an activation tile
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint64_t full_bar[SB];          // unit in B slot s: its tiles have landed (WT: A and B)
    __shared__ uint64_t mma_bar[SB];           // unit in B slot s: its MMAs are done
    __shared__ uint64_t raw_bar[TC_RAW_MAX];   // raw: the ring slot's tile has landed
    __shared__ uint64_t raw_free[TC_RAW_MAX];  // raw: every worker warp has converted the slot
    // two runs in flight: full = both issuers' MMAs of the run are done, free = every
    // worker warp has loaded the run's accumulators
    __shared__ uint64_t acc_full[2], acc_free[2];
    __shared__ uint32_t tmem_slot;
    __shared__ int partners_ok;
    __shared__ float inv_rms[NT];
    __shared__ float red_ss[4 * NT];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool worker = warp < kSkProducerWarp;
    // worker roles: weight row / TMEM lane `row` and 16-wide K piece `kq` of every chunk;
    // epilogue columns cg * SK_COLS ..
    const int row = tid & (TC_M - 1), kq = (tid >> 7) & 3;
    const int cg = (warp >> 2) & 3;
    const int G = gridDim.x, cta = blockIdx.x, C = sk.chunks;
    const int u0 = sk_first_unit(cta, G, sk.units);
    const int nu = sk_first_unit(cta + 1, G, sk.units) - u0;
    const int RS = sk.raw_slots;
    uint8_t* a_slots = smem;                     // [SA][hi | lo]
    uint8_t* b_slots = smem + SA * 2 * A_BYTES;  // [SB][hi | lo]
    uint8_t* raw_ring = smem + sk.raw_off;
    auto a_ptr = [&](int s) { return a_slots + (size_t)s * 2 * A_BYTES; };
    auto b_ptr = [&](int s) { return b_slots + (size_t)s * 2 * B_BYTES; };

    if (warp == 0) {
        tmem_alloc(&tmem_slot, 4 * NT);
        tmem_relinquish();
    }
    auto fetch_w = [&](int i) {  // unit u0 + i's weights: A slot i % SA, or (raw) ring slot i % RS
        if (WT) {
            uint64_t* bar = &full_bar[i % SB];
            mbar_arrive_expect_tx(bar, TC_TILE_BYTES);
            bulk_g2s(a_ptr(i % SA), a.wt + (size_t)(u0 + i) * TC_TILE_BYTES, TC_TILE_BYTES, bar);
        } else {
            mbar_arrive_expect_tx(&raw_bar[i % RS], TC_RAW_BYTES);
            bulk_g2s(raw_ring + (size_t)(i % RS) * TC_RAW_BYTES, a.wr + (size_t)(u0 + i) * TC_RAW_BYTES, TC_RAW_BYTES,
                     &raw_bar[i % RS]);
        }
    };
    const uint32_t xbytes = (uint32_t)sk.xrows * 128;  // rows x 64 bf16 of one half
    auto fetch_x = [&](int i) {  // unit u0 + i's activation tile (chunk (u0 + i) % C): B slot i % SB
        const uint8_t* src = a.sk_xs + (size_t)((u0 + i) % C) * SK_XTILE;
        uint64_t* bar = &full_bar[i % SB];
        mbar_arrive_expect_tx(bar, 2 * xbytes);
        if (xbytes == B_BYTES) {
            bulk_g2s(b_ptr(i % SB), src, 2 * B_BYTES, bar);
        } else {
            bulk_g2s(b_ptr(i % SB), src, xbytes, bar);
            bulk_g2s(b_ptr(i % SB) + B_BYTES, src + B_BYTES, xbytes, bar);
        }
    };
    if (tid == 0) {
        for (int s = 0; s < SB; s++) {
            mbar_init(&full_bar[s], WT ? 2 : 1);  // WT: the weight and the activation copies arrive
            mbar_init(&mma_bar[s], 1);
        }
        for (int r = 0; r < TC_RAW_MAX; r++) {
            mbar_init(&raw_bar[r], 1);
            mbar_init(&raw_free[r], SK_WORKERS / 32);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(&acc_full[s], 2);
            mbar_init(&acc_free[s], SK_WORKERS / 32);
        }
        fence_barrier_init();
        // weights are read-only: the first tiles are requested before the dependency wait
        for (int i = 0; i < min(nu, WT ? SA : RS); i++) fetch_w(i);
    }
    // activation rows past the copied ones stay zero in every B slot
    if (worker)
        for (int i = tid; i < SB * 2 * (NT - sk.xrows) * 8; i += SK_WORKERS) {
            const int s = i / (2 * (NT - sk.xrows) * 8), rem = i % (2 * (NT - sk.xrows) * 8);
            const int half = rem / ((NT - sk.xrows) * 8), r = sk.xrows + (rem % ((NT - sk.xrows) * 8)) / 8, g = rem % 8;
            *reinterpret_cast<uint4*>(b_ptr(s) + half * B_BYTES + core_off(r, g)) = make_uint4(0u, 0u, 0u, 0u);
        }
    grid_dependency_wait();
    // 1/rms of every token row; the RMSNorm gain is in the activation tiles and the 1/rms
    // scales the sums (linear in x) in the epilogue
    if (a.norm_gain && worker) {
        if (a.ss_in) {
            if (tid < NT * 4) {
                const int r = tid >> 2, p0 = tid & 3;
                float ss = 0.0f;
                if (r < a.M)
                    for (int p = p0; p < a.ss_parts; p += 4) ss += __ldcg(a.ss_in + (int64_t)p * a.ss_ld + r);
                ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                if (p0 == 0) inv_rms[r] = 1.0f / sqrtf(ss / (float)a.K + 1e-5f);
            }
        } else {
            for (int r = warp; r < NT; r += SK_WORKERS / 32) {
                float ss = 0.0f;
                if (r < a.M)
                    for (int k = lane * 4; k < a.K; k += 128) {
                        const float4 x4 = *reinterpret_cast<const float4*>(a.x + (int64_t)r * a.ldx + k);
                        ss += x4.x * x4.x + x4.y * x4.y + x4.z * x4.z + x4.w * x4.w;
                    }
                ss = warp_sum(ss);
                if (lane == 0) inv_rms[r] = 1.0f / sqrtf(ss / (float)a.K + 1e-5f);
            }
        }
    }
    fence_async_smem();  // the zeroed B rows, for the MMAs
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const uint32_t idesc = umma_idesc_bf16(TC_M, NT);
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);

    if (worker) {
        bool ok = true;
        int t = u0 / C, c = u0 % C;  // tile and chunk of the current unit
        int runs = 0, run_c0 = c, run_first = 0;
        for (int it = 0; it < nu; it++) {
            if (!WT) {
                // the A slot was last read by the MMAs of unit it - SA
                const int prev = it - SA;
                if (ok && prev >= 0 && !mbar_wait(&mma_bar[prev % SB], (prev / SB) & 1, a.err)) ok = false;
                if (ok && !mbar_wait(&raw_bar[it % RS], (it / RS) & 1, a.err)) ok = false;
                if (ok)
                    stage_w16_raw(raw_ring + (size_t)(it % RS) * TC_RAW_BYTES, a_ptr(it % SA), a_ptr(it % SA) + A_BYTES,
                                  row, kq);
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_free[it % RS]);  // the producer may refill the slot
                named_arrive(1 + it % 2, kSkBarThreads);         // the unit's issuer may start
            }
            const bool run_end = it == nu - 1 || c == C - 1;
            const int t_cur = t, c_cur = c;
            if (++c == C) { c = 0; t++; }
            if (!run_end) continue;

            // end of a run: load its accumulators (the first unit's issuer, then the other's
            // when the run has two or more units), hand them back to the issuers, then a
            // partial or the tile's epilogue
            const int reg = runs & 1, i0 = run_first & 1;
            if (ok && !mbar_wait(&acc_full[reg], (runs >> 1) & 1, a.err)) ok = false;
            runs++;
            tc_fence_after();
            float v[SK_COLS], w2[SK_COLS];
            tmem_ld16(tl + (reg * 2 + 0) * NT + cg * SK_COLS, v);
            tmem_ld16(tl + (reg * 2 + 1) * NT + cg * SK_COLS, w2);
            if (it > run_first) {  // issuer 1-i0 has units in the run too: add in issuer order
#pragma unroll
                for (int j = 0; j < SK_COLS; j++) v[j] += w2[j];
            } else if (i0 == 1) {
#pragma unroll
                for (int j = 0; j < SK_COLS; j++) v[j] = w2[j];
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_free[reg]);
            run_first = it + 1;
            if (it == nu - 1) grid_dependents_launch();
            if (run_c0 > 0) {
                // the tile belongs to an earlier CTA: [cta][column][row] partial, then the flag
                float* dst = a.sk_partial + ((size_t)cta * NT + cg * SK_COLS) * TC_M + row;
#pragma unroll
                for (int j = 0; j < SK_COLS; j++) __stcg(dst + (size_t)j * TC_M, ok ? v[j] : 0.0f);
                __threadfence();
                named_sync(kSkWorkerBar, SK_WORKERS);
                if (tid == 0) st_release_gpu(a.sk_flags + cta, 1);
            } else {
                const int last = c_cur == C - 1 ? cta : sk_cta_of(t_cur * C + C - 1, G, sk.units);
                float xo[SK_COLS];  // requested before the partners' partials arrive
                sk_residual_in(a, e, xo, t_cur * TC_M + row, cg * SK_COLS);
                if (last > cta) {  // the rest of the tile is in the shares of CTAs cta+1..last
                    // one thread per partner polls its flag (the polls overlap)
                    if (tid == 0) partners_ok = 1;
                    named_sync(kSkWorkerBar, SK_WORKERS);
                    if (tid < last - cta && !sk_wait_flag(a.sk_flags + cta + 1 + tid, a.err)) partners_ok = 0;
                    named_sync(kSkWorkerBar, SK_WORKERS);
                    if (partners_ok) {
                        // partials added in CTA order, two partners' loads in flight at a time
                        for (int p = cta + 1; p <= last; p += 2) {
                            const bool two = p + 1 <= last;
                            const float* s0 = a.sk_partial + ((size_t)p * NT + cg * SK_COLS) * TC_M + row;
                            const float* s1 = s0 + (size_t)NT * TC_M;
                            float pa[SK_COLS], pb[SK_COLS];
#pragma unroll
                            for (int j = 0; j < SK_COLS; j++) pa[j] = __ldcg(s0 + (size_t)j * TC_M);
#pragma unroll
                            for (int j = 0; j < SK_COLS; j++) pb[j] = two ? __ldcg(s1 + (size_t)j * TC_M) : 0.0f;
#pragma unroll
                            for (int j = 0; j < SK_COLS; j++) v[j] += pa[j];
                            if (two) {
#pragma unroll
                                for (int j = 0; j < SK_COLS; j++) v[j] += pb[j];
                            }
                        }
                        if (tid < last - cta) atomicExch(a.sk_flags + cta + 1 + tid, 0);
                    } else {
                        ok = false;
                    }
                }
                sk_epilogue(a, e, v, xo, t_cur * TC_M + row, cg * SK_COLS, inv_rms, red_ss, warp, lane, ok);
                if (e.kind == kEpiResidual && e.ss_out) {  // this tile's share of the next RMSNorm
                    named_sync(kSkWorkerBar, SK_WORKERS);
                    if (tid < NT && tid < a.M)
                        e.ss_out[(int64_t)t_cur * e.ss_ld + tid] =
                            red_ss[tid] + red_ss[NT + tid] + red_ss[2 * NT + tid] + red_ss[3 * NT + tid];
                }
            }
            run_c0 = 0;  // every later run starts at a tile's chunk 0
        }
    } else if (warp == kSkProducerWarp) {
        // producer: activation tiles (and WT weight tiles) SB units ahead, a slot refilled
        // once the MMAs of the unit that last read it are done; (raw) the raw ring RS units
        // ahead, a slot refilled once every worker warp has converted it
        if (lane == 0) {
            bool ok = true;
            for (int i = 0; i < min(nu, SB); i++) fetch_x(i);
            int next_raw = RS;
            for (int j = SB; j < nu; j++) {
                if (!WT)
                    for (; next_raw < nu && next_raw < j + RS; next_raw++) {  // keep the raw ring full meanwhile
                        const int done = next_raw - RS;
                        if (!mbar_try_wait(&raw_free[done % RS], (done / RS) & 1)) break;
                        fetch_w(next_raw);
                    }
                if (ok && !mbar_wait(&mma_bar[(j - SB) % SB], ((j - SB) / SB) & 1, a.err)) ok = false;
                if (WT) fetch_w(j);
                fetch_x(j);
            }
            if (!WT)
                for (; next_raw < nu; next_raw++) {
                    const int done = next_raw - RS;
                    if (ok && !mbar_wait(&raw_free[done % RS], (done / RS) & 1, a.err)) ok = false;
                    fetch_w(next_raw);
                }
        }
        grid_dependents_launch();
    } else {
        // MMA issuer m (warps 17, 18): units it with it % 2 == m; lane 0 works, the warp
        // takes the stage barriers
        const int m = warp - kSkProducerWarp - 1;
        bool ok = true;
        int c = u0 % C, run = 0;
        bool mine = false;  // this issuer has MMAs in the current run
        // slot descriptors: the address field (bytes >> 4, below 2^14) advances by the
        // slot stride without carrying into the next field
        const uint64_t da0 = umma_desc(smem_addr(a_slots)), db0 = umma_desc(smem_addr(b_slots));
        for (int it = 0; it < nu; it++) {
            const bool first = it == 0 || c == 0;
            if (first) {
                if (it > 0) run++;
                mine = false;
                // the run's accumulators are free once the workers loaded run - 2's
                if (lane == 0 && run >= 2 && ok && !mbar_wait(&acc_free[run & 1], ((run - 2) >> 1) & 1, a.err)) ok = false;
            }
            const bool run_end = it == nu - 1 || c == C - 1;
            if (++c == C) c = 0;
            if ((it & 1) == m) {
                const int sa = it % SA, sb = it % SB;
                __syncwarp();
                if (!WT) named_sync(1 + m, kSkBarThreads);  // the workers converted this unit's weights
                if (lane == 0) {
                    if (ok && !mbar_wait(&full_bar[sb], (it / SB) & 1, a.err)) ok = false;
                    tc_fence_after();
                    const uint64_t dah = da0 + (uint64_t)sa * (2 * A_BYTES >> 4);
                    const uint64_t dbh = db0 + (uint64_t)sb * (2 * B_BYTES >> 4);
                    issue_unit_mmas(tmem + (uint32_t)(((run & 1) * 2 + m) * NT), idesc, dah, dah + (A_BYTES >> 4), dbh,
                                    dbh + (B_BYTES >> 4), !mine);
                    umma_commit(&mma_bar[sb]);
                }
                mine = true;
            }
            if (run_end && lane == 0) {
                // this issuer's share of the run is complete (or it had none)
                if (mine) umma_commit(&acc_full[run & 1]);
                else mbar_arrive(&acc_full[run & 1]);
            }
        }
        grid_dependents_launch();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 4 * NT);
}

// ------------------------------------------------------------------ int8 digit-plane matvec, 1-10 rows
// Small batches over large Q8 matrices (decode at batch 1-10 on the 7B shape).  The int8
// weights go to the tensor core as they are: the raw tiles' layout ([16-byte K piece][128
// rows][16 B]) is a K-major UMMA layout (K core matrices 2048 B apart, 8-row groups 128 B
// apart), so a kind::i8 MMA of K = 32 covers one Q8_0 block with no conversion on chip.
// The activations are written once per launch (tc_i8_digits_kernel) as three int8 digit
// planes per token and 32-wide block: with xs = max|x g| / 127 over the block and
// t = x g / xs, d0 = rint(t), d1 = rint((t - d0) 254), d2 = rint(((t - d0) 254 - d1) 254),
// so x g = xs (d0 + d1 / 254 + d2 / 254^2) to ~1e-7 of the block's largest value.  One
// MMA (M = 128 weight rows, N = 16 or 32 columns = 3 digit planes x up to 10 tokens) gives
// every block's integer dot products exactly (int32); reader warps take them from TMEM and
// add s[n][block] xs[block][m] (I0 + I1 / 254 + I2 / 254^2) into fp32 sums per row and
// token: the Q8 products of src/model_q8.cpp:107-111 with the block scale applied once
// per block.  Units, shares, partials and epilogues are the stream-K kernel's.
constexpr int I8_RS = 16;         // at most this many ring slots
constexpr int I8_THREADS = 192;   // 4 reader warps (a row each lane), producer, MMA issuer
constexpr int kI8ReaderBar = 9;   // named barrier of the 128 reader threads
constexpr float kI8D1 = 1.0f / 254.0f, kI8D2 = 1.0f / 64516.0f;

__host__ __device__ constexpr int i8_block_tile(int ncol) { return ncol * 32; }  // bytes of one block's digits

__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version for sm_100; no swizzle
    return d;
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(0u)
        : "memory");
}

// Instruction descriptor of kind::i8: D s32, A and B signed 8-bit, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// The activations' digit planes: thread per (block kb, column c = 3 m + plane); block
// kb's tile is [16-wide K group][8-column group][8 columns][16 B]; xs[kb][m] after the
// tiles.  Columns past 3 M are zero.
template <int NCOL>
__global__ void __launch_bounds__(256) tc_i8_digits_kernel(GemmArgs a) {
    grid_dependency_wait();  // x comes from the previous kernel
    grid_dependents_launch();
    const int blocks = a.K / 32;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= blocks * NCOL) return;
    const int kb = t / NCOL, c = t % NCOL, m = c / 3, plane = c % 3;
    __align__(16) int8_t d[32];
    float xs = 0.0f;
    if (m < a.M) {
        float v[32], amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            float4 x4 = *reinterpret_cast<const float4*>(a.x + (int64_t)m * a.ldx + kb * 32 + 4 * j);
            if (a.norm_gain) {
                const float4 g4 = __ldg(reinterpret_cast<const float4*>(a.norm_gain + kb * 32) + j);
                x4.x *= g4.x; x4.y *= g4.y; x4.z *= g4.z; x4.w *= g4.w;
            }
            v[4 * j] = x4.x; v[4 * j + 1] = x4.y; v[4 * j + 2] = x4.z; v[4 * j + 3] = x4.w;
        }
#pragma unroll
        for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(v[j]));
        xs = amax / 127.0f;
        const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const float tt = v[j] * inv;
            const float d0 = rintf(tt), r1 = (tt - d0) * 254.0f;
            const float d1 = rintf(r1), d2 = rintf((r1 - d1) * 254.0f);
            const float dv = plane == 0 ? d0 : (plane == 1 ? d1 : d2);
            d[j] = (int8_t)fmaxf(-127.0f, fminf(127.0f, dv));
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; j++) d[j] = 0;
    }
    uint8_t* tile = a.sk_xs + (size_t)kb * i8_block_tile(NCOL);
#pragma unroll
    for (int g = 0; g < 2; g++)
        *reinterpret_cast<uint4*>(tile + g * (NCOL / 8) * 128 + (c / 8) * 128 + (c % 8) * 16) =
            *reinterpret_cast<const uint4*>(d + 16 * g);
    if (plane == 0 && m < 16) {
        float* xst = reinterpret_cast<float*>(a.sk_xs + (size_t)blocks * i8_block_tile(NCOL));
        xst[kb * 16 + m] = xs;
    }
}

// UCH consecutive 64-wide chunks of one tile form a unit (their raw tiles are adjacent in
// memory: one bulk copy), so every wait and copy covers UCH x 9 KB of weights.
template <int NCOL, int UCH>
__global__ void __launch_bounds__(I8_THREADS, 1) tc_i8_kernel(GemmArgs a, Epilogue e, StreamKArgs sk) {
    constexpr int BT = i8_block_tile(NCOL);            // digit bytes of one block
    constexpr int NB = 2 * UCH;                        // Q8_0 blocks per unit
    constexpr int UB = UCH * TC_RAW_BYTES + NB * BT;   // one ring slot: raw tiles, then the unit's digit tiles
    constexpr int R = 512 / (NB * NCOL) < 8 ? 512 / (NB * NCOL) : 8;  // TMEM result regions in flight
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint64_t full_bar[I8_RS];      // raw tiles and digits of the slot's unit have landed (2 arrivals)
    __shared__ uint64_t slot_free[I8_RS];     // the reader warps are done with the slot
    __shared__ uint64_t mma_done[8];
    __shared__ uint64_t region_free[8];
    __shared__ uint32_t tmem_slot;
    __shared__ int partners_ok;
    __shared__ float inv_rms[16];
    __shared__ float red_ss[4 * SK_NT];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x, C = sk.chunks / UCH;  // units per tile
    const int RS = sk.raw_slots;
    const int u0 = sk_first_unit(cta, G, sk.units);
    const int nu = sk_first_unit(cta + 1, G, sk.units) - u0;
    const int blocks = a.K / 32;
    float* xst = reinterpret_cast<float*>(smem + (size_t)RS * UB);  // [blocks][16] block scales of x
    auto slot_ptr = [&](int s) { return smem + (size_t)s * UB; };

    if (warp == 0) {
        tmem_alloc(&tmem_slot, R * NB * NCOL);
        tmem_relinquish();
    }
    auto fetch_w = [&](int i) {
        uint64_t* bar = &full_bar[i % RS];
        mbar_arrive_expect_tx(bar, UCH * TC_RAW_BYTES);
        bulk_g2s(slot_ptr(i % RS), a.wr + (size_t)(u0 + i) * UCH * TC_RAW_BYTES, UCH * TC_RAW_BYTES, bar);
    };
    auto fetch_d = [&](int i) {  // the unit's blocks NB * ((u0 + i) % C) ..
        uint64_t* bar = &full_bar[i % RS];
        mbar_arrive_expect_tx(bar, NB * BT);
        bulk_g2s(slot_ptr(i % RS) + UCH * TC_RAW_BYTES, a.sk_xs + (size_t)((u0 + i) % C) * NB * BT, NB * BT, bar);
    };
    if (tid == 0) {
        for (int s = 0; s < RS; s++) {
            mbar_init(&full_bar[s], 2);
            mbar_init(&slot_free[s], 4);
        }
        for (int r = 0; r < R; r++) {
            mbar_init(&mma_done[r], 1);
            mbar_init(&region_free[r], 4);
        }
        fence_barrier_init();
        // weights are read-only: the first tiles are requested before the dependency wait
        for (int i = 0; i < min(nu, RS); i++) fetch_w(i);
    }
    grid_dependency_wait();
    // x block scales into shared memory; 1/rms of each token row
    const float* xs_g = reinterpret_cast<const float*>(a.sk_xs + (size_t)blocks * BT);
    for (int i = tid; i < blocks * 16; i += I8_THREADS) xst[i] = xs_g[i];
    if (a.norm_gain && warp < 4) {
        for (int r = warp; r < 16; r += 4) {
            float ss = 0.0f;
            if (r < a.M)
                for (int k = lane * 4; k < a.K; k += 128) {
                    const float4 x4 = *reinterpret_cast<const float4*>(a.x + (int64_t)r * a.ldx + k);
                    ss += x4.x * x4.x + x4.y * x4.y + x4.z * x4.z + x4.w * x4.w;
                }
            ss = warp_sum(ss);
            if (lane == 0) inv_rms[r] = 1.0f / sqrtf(ss / (float)a.K + 1e-5f);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp < 4) {
        // readers: thread = weight row `tid` of the tile (TMEM lane)
        bool ok = true;
        const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
        float acc[16];
#pragma unroll
        for (int m = 0; m < 16; m++) acc[m] = 0.0f;
        int t = u0 / C, c = u0 % C, run_c0 = c;
        for (int it = 0; it < nu; it++) {
            const int s = it % RS, r = it % R;
            if (ok && !mbar_wait(&mma_done[r], (it / R) & 1, a.err)) ok = false;
            tc_fence_after();
            // the unit's blocks 64 TMEM columns at a time (2 loads in flight, one wait)
            constexpr int BPL = 32 / NCOL;  // blocks per 32-column load
#pragma unroll
            for (int j0 = 0; j0 < NB; j0 += 2 * BPL) {
                uint32_t iv[2][32];
#pragma unroll
                for (int h = 0; h < 2; h++)
                    if (j0 + h * BPL < NB) tmem_ld32_async(tl + (uint32_t)((r * NB + j0 + h * BPL) * NCOL), iv[h]);
                tmem_wait_ld();
                tmem_regs_ready(iv[0]);
                if (j0 + BPL < NB) tmem_regs_ready(iv[1]);
#pragma unroll
                for (int jj = 0; jj < 2 * BPL; jj++) {
                    const int j = j0 + jj;
                    if (j >= NB) break;
                    const uint32_t* col = iv[jj / BPL] + (jj % BPL) * NCOL;
                    // block j: half j % 2 of raw tile j / 2 ([half][128 rows] scales after its int8)
                    const float ws = reinterpret_cast<const float*>(slot_ptr(s) + (j >> 1) * TC_RAW_BYTES +
                                                                    TC_M * TC_KC)[(j & 1) * TC_M + tid];
                    const float* xsb = xst + (c * NB + j) * 16;
#pragma unroll
                    for (int m = 0; m < NCOL / 3; m++) {
                        const float p = (float)(int)col[3 * m] + (float)(int)col[3 * m + 1] * kI8D1 +
                                        (float)(int)col[3 * m + 2] * kI8D2;
                        acc[m] = fmaf(ws, xsb[m] * p, acc[m]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&region_free[r]);
                mbar_arrive(&slot_free[s]);
            }
            const bool run_end = it == nu - 1 || c == C - 1;
            const int t_cur = t, c_cur = c;
            if (++c == C) { c = 0; t++; }
            if (!run_end) continue;

            float v[SK_COLS];
#pragma unroll
            for (int m = 0; m < SK_COLS; m++) v[m] = acc[m];
#pragma unroll
            for (int m = 0; m < 16; m++) acc[m] = 0.0f;
            if (it == nu - 1) grid_dependents_launch();
            if (run_c0 > 0) {
                // the tile belongs to an earlier CTA: [cta][token][row] partial, then the flag
                float* dst = a.sk_partial + (size_t)cta * SK_NT * TC_M + tid;
#pragma unroll
                for (int m = 0; m < SK_COLS; m++) __stcg(dst + (size_t)m * TC_M, ok ? v[m] : 0.0f);
                __threadfence();
                named_sync(kI8ReaderBar, 128);
                if (tid == 0) st_release_gpu(a.sk_flags + cta, 1);
            } else {
                const int last = c_cur == C - 1 ? cta : sk_cta_of(t_cur * C + C - 1, G, sk.units);
                float xo[SK_COLS];
                sk_residual_in(a, e, xo, t_cur * TC_M + tid, 0);
                if (last > cta) {
                    if (tid == 0) partners_ok = 1;
                    named_sync(kI8ReaderBar, 128);
                    if (tid < last - cta && !sk_wait_flag(a.sk_flags + cta + 1 + tid, a.err)) partners_ok = 0;
                    named_sync(kI8ReaderBar, 128);
                    if (partners_ok) {
                        for (int p = cta + 1; p <= last; p++) {
                            const float* src = a.sk_partial + (size_t)p * SK_NT * TC_M + tid;
                            float pa[SK_COLS];
#pragma unroll
                            for (int m = 0; m < SK_COLS; m++) pa[m] = __ldcg(src + (size_t)m * TC_M);
#pragma unroll
                            for (int m = 0; m < SK_COLS; m++) v[m] += pa[m];
                        }
                        if (tid < last - cta) atomicExch(a.sk_flags + cta + 1 + tid, 0);
                    } else {
                        ok = false;
                    }
                }
                sk_epilogue(a, e, v, xo, t_cur * TC_M + tid, 0, inv_rms, red_ss, warp, lane, ok);
                if (e.kind == kEpiResidual && e.ss_out) {
                    named_sync(kI8ReaderBar, 128);
                    if (tid < a.M)
                        e.ss_out[(int64_t)t_cur * e.ss_ld + tid] =
                            red_ss[tid] + red_ss[SK_NT + tid] + red_ss[2 * SK_NT + tid] + red_ss[3 * SK_NT + tid];
                    named_sync(kI8ReaderBar, 128);
                }
            }
            run_c0 = 0;
        }
    } else if (warp == 4) {
        // producer: digits of the first slots, then every slot refilled (raw tiles and
        // digits) once the readers are done with its previous unit
        if (lane == 0) {
            bool ok = true;
            for (int i = 0; i < min(nu, RS); i++) fetch_d(i);
            for (int j = RS; j < nu; j++) {
                const int done = j - RS;
                if (ok && !mbar_wait(&slot_free[done % RS], (done / RS) & 1, a.err)) ok = false;
                fetch_w(j);
                fetch_d(j);
            }
        }
        grid_dependents_launch();
    } else {
        // MMA issuer: one K = 32 MMA per Q8_0 block of the unit into the unit's region
        if (lane == 0) {
            bool ok = true;
            const uint32_t idesc = umma_idesc_i8(TC_M, NCOL);
            for (int it = 0; it < nu; it++) {
                const int s = it % RS, r = it % R;
                if (ok && !mbar_wait(&full_bar[s], (it / RS) & 1, a.err)) ok = false;
                const int prev = it - R;
                if (ok && prev >= 0 && !mbar_wait(&region_free[r], (prev / R) & 1, a.err)) ok = false;
                tc_fence_after();
                const uint32_t base = smem_addr(slot_ptr(s));
#pragma unroll
                for (int j = 0; j < NB; j++) {
                    const uint64_t da = desc_kmajor(base + (j >> 1) * TC_RAW_BYTES + (j & 1) * 2 * 2048, 2048, 128);
                    const uint64_t db = desc_kmajor(base + UCH * TC_RAW_BYTES + j * BT, (NCOL / 8) * 128, 128);
                    umma_i8(tmem + (uint32_t)((r * NB + j) * NCOL), da, db, idesc);
                }
                umma_commit(&mma_done[r]);
            }
        }
        grid_dependents_launch();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, R * NB * NCOL);
}

// Allow the kernel the largest dynamic shared memory the device offers next to its static
// shared memory (per kernel and device, once).
template <class K>
int tc_ensure_smem(K kernel) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_pair((const void*)kernel, dev);
    auto it = done.find(key);
    if (it != done.end()) return it->second;
    cudaFuncAttributes fa;
    int optin = 0;
    cudaFuncGetAttributes(&fa, kernel);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    const int budget = optin - (int)fa.sharedSizeBytes;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, budget);
    done[key] = budget;
    return budget;
}

using TcKernel = void (*)(GemmArgs, Epilogue, SplitArgs);

// Clusters of `ks` CTAs with `smem` bytes each that fit on the device at once (cached per
// device; a failed query reports "no limit").
int tc_max_clusters(TcKernel kernel, int ks, int smem, int n_tiles, int m_tiles) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, int, int>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    const auto key = std::make_tuple((const void*)kernel, ks, smem, dev);
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ks, n_tiles, m_tiles);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = ks;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = 1 << 30;
    }
    cache[key] = n;
    return n;
}

// SMs of the current device (the runtime caches the attribute).
int device_sms() {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms > 0 ? sms : 148;
}

template <int NT>
void tc_launch(const GemmArgs& a, const Epilogue& e, cudaStream_t s) {
    const int n_tiles = (a.N + TC_M - 1) / TC_M;
    const int m_tiles = (a.M + NT - 1) / NT;
    const int chunks = a.K / TC_KC;
    TcKernel kernel;
    if (a.wf) {
        kernel = tc_gemm_kernel<NT, true, kEpiLogits>;
    } else {
        // one kernel for every Q8 projection kind: the four projections of a layer then
        // share their instruction-cache footprint (measured ~1.5 % faster per step than a
        // kernel per kind)
        kernel = tc_gemm_kernel<NT, false, -1>;
    }
    const int budget = tc_ensure_smem(kernel);
    const bool raw = !a.wf && a.wr && !a.wt;
    // Stages and shared memory for a split: a stage per chunk when all of a CTA's chunks
    // fit (the receive buffer of a split, padded if there is room, and the RMSNorm gain
    // slice next to them), else a 2-stage ring: its loads run one chunk ahead in registers,
    // and the small footprint lets two CTAs share an SM.
    auto plan = [&](int ks, SplitArgs* sp) {
        const int per_cta = (chunks + ks - 1) / ks;
        sp->ksplit = ks;
        auto layout = [&](int stages, int pad) {
            sp->stages = stages;
            sp->recv_pad = pad;
            sp->recv_off = stages * TcSmem<NT>::STAGE;
            sp->gain_off = sp->recv_off + (ks > 1 ? (NT + pad * ks) * TC_M * 4 : 0);
            sp->raw_off = sp->gain_off + (a.norm_gain ? stages * TC_KC * 4 : 0);
            sp->raw_slots = 0;
            return sp->raw_off;
        };
        if (raw) {  // a 2-stage ring fed by as many raw-tile slots as fit
            const int base = layout(TC_STAGES, 4);
            sp->raw_slots = std::min(TC_RAW_MAX, (budget - base) / (int)TC_RAW_BYTES);
            return base + sp->raw_slots * (int)TC_RAW_BYTES;
        }
        if (per_cta <= TcSmem<NT>::MAX_STAGES) {
            const int st = std::max(TC_STAGES, per_cta);
            for (int pad = 4; pad >= 0; pad -= 4) {
                const int bytes = layout(st, pad);
                if (bytes <= budget) return bytes;
            }
        }
        return layout(TC_STAGES, 4);
    };
    // Fill the GPU: when the tiles alone are fewer than the SMs, split K across the CTAs
    // of a cluster (power of two up to 8, at most one split per chunk, NT/ksplit >= 8), but
    // only as far as every cluster of the launch can be resident at once.  The faithful
    // path reads one chunk per row and never splits.
    int ksplit = 1;
    const int tiles = n_tiles * m_tiles;
    if (a.kbegin == 0 && NT <= 128)
        while (ksplit < NITRO_TC_MAX_KSPLIT && tiles * ksplit < device_sms() && ksplit * 2 <= chunks &&
               NT / (ksplit * 2) >= 8)
            ksplit *= 2;
    SplitArgs sp;
    int smem = plan(ksplit, &sp);
    while (ksplit > 1 && tc_max_clusters(kernel, ksplit, smem, n_tiles, m_tiles) < tiles) {
        ksplit /= 2;
        smem = plan(ksplit, &sp);
    }
    // 128/256-token tiles streaming hi/lo weight tiles: the activations split once for the
    // launch (the kernel's ring path copies them with each weight tile)
    GemmArgs ax = a;
    ax.xs_tiles = nullptr;
    const int rows_pad = m_tiles * NT;
    if (NT >= 128 && a.xs_tiles && a.wt && !a.wf && !raw && a.kbegin == 0 &&
        (chunks + ksplit - 1) / ksplit > TcSmem<NT>::MAX_STAGES && rows_pad <= a.xs_cap_rows && a.K <= a.xs_cap_k) {
        ax.xs_tiles = a.xs_tiles;
        ax.xs_rows = rows_pad;
        const int64_t threads = (int64_t)chunks * rows_pad * 8;
        count_launch();
        launch_ex(tc_split_x_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, s, 1, ax, rows_pad, rows_pad,
                  a.xs_tiles);
    }
    launch_ex(kernel, dim3(ksplit, n_tiles, m_tiles), dim3(TC_THREADS), smem, s, ksplit, ax, e, sp);
}

// Pre-split weights: one thread per (row, 8-wide K group) writes the bf16 hi/lo halves of
// w = q * scale (or w) at the place the kernel's staging would put them; tile (t, c) of
// the output is [hi 16 KB][lo 16 KB] for rows 128t.. and K chunk c.
__global__ void tile_weights_kernel(const int8_t* q, const float* scales, const float* wf, int N, int K, uint8_t* out) {
    const int groups = K / 8;
    const int64_t rows = (int64_t)((N + TC_M - 1) / TC_M) * TC_M;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= rows * groups) return;
    const int n = (int)(t / groups), g = (int)(t % groups);
    float w[8];
    if (n < N) {
        if (wf) {
#pragma unroll
            for (int j = 0; j < 8; j++) w[j] = wf[(int64_t)n * K + g * 8 + j];
        } else {
            const float sc = scales[(int64_t)n * (K / 32) + g / 4];
#pragma unroll
            for (int j = 0; j < 8; j++) w[j] = (float)q[(int64_t)n * K + g * 8 + j] * sc;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) w[j] = 0.0f;
    }
    uint8_t* tile = out + ((int64_t)(n / TC_M) * (K / TC_KC) + g / 8) * TC_TILE_BYTES;
    const uint32_t o = core_off(n % TC_M, g % 8);
    split_store8(w, tile + o, tile + TC_TILE_BYTES / 2 + o);
}

// Raw Q8 tiles: one thread per (row, 16-byte group of a 64-column chunk).
__global__ void tile_q8_raw_kernel(const int8_t* q, const float* scales, int N, int K, uint8_t* out) {
    const int groups = K / 16;
    const int64_t rows = (int64_t)((N + TC_M - 1) / TC_M) * TC_M;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= rows * groups) return;
    const int n = (int)(t / groups), g = (int)(t % groups);
    const int chunk = g / 4, piece = g % 4;  // piece = half * 2 + (16-byte part)
    uint8_t* tile = out + ((int64_t)(n / TC_M) * (K / TC_KC) + chunk) * TC_RAW_BYTES;
    const int r = n % TC_M;
    int4 v = make_int4(0, 0, 0, 0);
    if (n < N) v = *reinterpret_cast<const int4*>(q + (int64_t)n * K + g * 16);
    *reinterpret_cast<int4*>(tile + (piece * TC_M + r) * 16) = v;
    if ((piece & 1) == 0) {
        const int half = piece >> 1;
        reinterpret_cast<float*>(tile + TC_M * TC_KC)[half * TC_M + r] =
            n < N ? scales[(int64_t)n * (K / 32) + chunk * 2 + half] : 0.0f;
    }
}

}  // namespace

size_t tc_raw_q8_bytes(int N, int K) {
    return (size_t)((N + TC_M - 1) / TC_M) * (size_t)(K / TC_KC) * TC_RAW_BYTES;
}

void tc_tile_q8_raw(const int8_t* q, const float* scales, int N, int K, uint8_t* out, cudaStream_t s) {
    const int64_t n = (int64_t)((N + TC_M - 1) / TC_M) * TC_M * (K / 16);
    tile_q8_raw_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(q, scales, N, K, out);
}

size_t tc_tiled_weight_bytes(int N, int K) {
    return (size_t)((N + TC_M - 1) / TC_M) * (size_t)(K / TC_KC) * TC_TILE_BYTES;
}

void tc_tile_weights(const int8_t* q, const float* scales, const float* wf, int N, int K, uint8_t* out, cudaStream_t s) {
    const int64_t n = (int64_t)((N + TC_M - 1) / TC_M) * TC_M * (K / 8);
    tile_weights_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(q, scales, wf, N, K, out);
}

bool tc_streamk_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* env = getenv("NITRO_STREAMK");
        v = (env && env[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

// Scratch layout: partial tiles [ctas][64][128] fp32, activation tiles [max_k / 64][16 KB],
// flags [ctas].
size_t tc_streamk_scratch_bytes(int ctas, int max_k) {
    return (size_t)ctas * SK_NT * TC_M * sizeof(float) + (size_t)(max_k / TC_KC) * SK_XTILE + (size_t)ctas * sizeof(int);
}

void tc_streamk_bind(GemmArgs& g, void* scratch, int ctas, int max_k) {
    uint8_t* p = static_cast<uint8_t*>(scratch);
    g.sk_partial = reinterpret_cast<float*>(p);
    p += (size_t)ctas * SK_NT * TC_M * sizeof(float);
    g.sk_xs = p;
    p += (size_t)(max_k / TC_KC) * SK_XTILE;
    g.sk_flags = reinterpret_cast<int*>(p);
    g.sk_capacity = ctas;
    g.sk_max_k = max_k;
}

namespace {

// Smallest batch the stream-K kernel takes (NITRO_STREAMK_MIN_ROWS; 1-2 rows otherwise go
// to the streamed matvec).
int streamk_min_rows() {
    static int v = -1;
    if (v < 0) {
        const char* env = getenv("NITRO_STREAMK_MIN_ROWS");
        v = env ? std::max(1, atoi(env)) : 3;
    }
    return v;
}

bool tc_i8_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* env = getenv("NITRO_I8_MATVEC");
        v = (env && env[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

// Chunks per unit of the digit-plane kernel (4 when the chunk count allows), its ring
// slots within ~196 KB of shared memory, and the shared memory they take with the x block
// scales.
int i8_uch(int K) { return (K / TC_KC) % 4 == 0 ? 4 : ((K / TC_KC) % 2 == 0 ? 2 : 1); }
int i8_slots(int ncol, int uch) {
    return std::min(I8_RS, (196 * 1024) / (uch * (int)TC_RAW_BYTES + 2 * uch * i8_block_tile(ncol)));
}
int i8_smem(int ncol, int K) {
    const int uch = i8_uch(K);
    return i8_slots(ncol, uch) * (uch * (int)TC_RAW_BYTES + 2 * uch * i8_block_tile(ncol)) + (K / 32) * 16 * 4;
}

bool i8_takes(const GemmArgs& a) {
    return tc_i8_enabled() && a.sk_partial && a.sk_flags && a.sk_xs && a.sk_capacity > 0 && a.K <= a.sk_max_k &&
           a.wr && !a.wf && a.kbegin == 0 && a.M >= 1 && a.M <= 10 && a.K % TC_KC == 0 && a.N % 2 == 0 &&
           i8_smem(32, a.K) <= 224 * 1024 && i8_slots(32, i8_uch(a.K)) >= 3;
}

template <int NCOL, int UCH>
void tc_launch_i8_u(const GemmArgs& a, const Epilogue& e, StreamKArgs sk, int grid, cudaStream_t s) {
    sk.units = ((a.N + TC_M - 1) / TC_M) * (sk.chunks / UCH);
    sk.raw_slots = i8_slots(NCOL, UCH);
    grid = std::max(1, std::min(grid, sk.units));
    tc_ensure_smem(tc_i8_kernel<NCOL, UCH>);
    launch_ex(tc_i8_kernel<NCOL, UCH>, dim3(grid), dim3(I8_THREADS), i8_smem(NCOL, a.K), s, 1, a, e, sk);
}

template <int NCOL>
void tc_launch_i8(const GemmArgs& a, const Epilogue& e, cudaStream_t s) {
    StreamKArgs sk;
    sk.chunks = a.K / TC_KC;
    sk.xrows = 0;
    sk.raw_off = 0;
    const int sms = device_sms();
    const int dthreads = (a.K / 32) * NCOL;
    count_launch();
    launch_ex(tc_i8_digits_kernel<NCOL>, dim3((unsigned)((dthreads + 255) / 256)), dim3(256), 0, s, 1, a);
    const int grid = std::min(sms, a.sk_capacity);
    const int uch = i8_uch(a.K);
    if (uch == 4) tc_launch_i8_u<NCOL, 4>(a, e, sk, grid, s);
    else if (uch == 2) tc_launch_i8_u<NCOL, 2>(a, e, sk, grid, s);
    else tc_launch_i8_u<NCOL, 1>(a, e, sk, grid, s);
}

bool streamk_takes(const GemmArgs& a) {
    return tc_streamk_enabled() && a.sk_partial && a.sk_flags && a.sk_xs && a.sk_capacity > 0 && a.K <= a.sk_max_k &&
           (a.wr || a.wt) && !a.wf && a.kbegin == 0 && a.M >= streamk_min_rows() && a.M <= SK_NT && a.K % TC_KC == 0 &&
           a.N % 2 == 0;
}

void tc_launch_streamk(const GemmArgs& a, const Epilogue& e, cudaStream_t s) {
    StreamKArgs sk;
    sk.chunks = a.K / TC_KC;
    sk.units = ((a.N + TC_M - 1) / TC_M) * sk.chunks;
    sk.xrows = (a.M + 7) / 8 * 8;
    const int sms = device_sms();
    // the activations as hi/lo tiles, once for the launch
    const int64_t xthreads = (int64_t)sk.chunks * sk.xrows * 8;
    count_launch();
    launch_ex(tc_split_x_kernel, dim3((unsigned)((xthreads + 255) / 256)), dim3(256), 0, s, 1, a, sk.xrows, SK_NT,
              a.sk_xs);
    const int grid = std::max(1, std::min(std::min(sms, sk.units), a.sk_capacity));
    constexpr int A_SLOT = 2 * TC_M * TC_KC * 2, B_SLOT = (int)SK_XTILE;
    if (a.wt) {  // hi/lo tiles: no conversion, 4 A slots
        sk.raw_off = 4 * A_SLOT + SK_SB * B_SLOT;
        sk.raw_slots = 0;
        tc_ensure_smem(tc_streamk_kernel<true>);
        launch_ex(tc_streamk_kernel<true>, dim3(grid), dim3(SK_THREADS), sk.raw_off, s, 1, a, e, sk);
        return;
    }
    const int budget = tc_ensure_smem(tc_streamk_kernel<false>);
    sk.raw_off = 2 * A_SLOT + SK_SB * B_SLOT;
    sk.raw_slots = std::min(TC_RAW_MAX, (budget - sk.raw_off) / (int)TC_RAW_BYTES);
    launch_ex(tc_streamk_kernel<false>, dim3(grid), dim3(SK_THREADS), sk.raw_off + sk.raw_slots * (int)TC_RAW_BYTES, s,
              1, a, e, sk);
}

}  // namespace

// Raw Q8 tiles send batches of 3-8 tokens here too: for large matrices the tensor-core
// kernels stream them far better than the matvec (1-2 tokens take the streamed matvec).
bool tc_gemm_supported(const GemmArgs& a) {
    return a.K % TC_KC == 0 && a.N % 2 == 0 &&
           (a.M > 8 || (a.wr != nullptr && !a.wf && a.M > 2) || streamk_takes(a) || i8_takes(a));
}

void launch_tc_gemm(const GemmArgs& a, const Epilogue& e, cudaStream_t s) {
    count_launch();
    if (i8_takes(a)) {
        if (a.M <= 5) tc_launch_i8<16>(a, e, s);
        else tc_launch_i8<32>(a, e, s);
        return;
    }
    if (streamk_takes(a)) {
        tc_launch_streamk(a, e, s);
        return;
    }
    // 256-token tiles only when they alone fill the GPU (they never split K)
    const int n_tiles = (a.N + TC_M - 1) / TC_M;
    if (a.M <= 64) tc_launch<64>(a, e, s);
    else if (a.M <= 128 || n_tiles * ((a.M + 255) / 256) < device_sms()) tc_launch<128>(a, e, s);
    else tc_launch<256>(a, e, s);
}


}  // namespace nitro
