// Causal prefill attention on the 5th-generation tensor cores (tcgen05), head_dim 64.
//
// One CTA per (128-query tile, head): 256 threads, two per query row (TMEM lane r is read
// by warp r/32 of both warpgroups, each taking half of the row's keys and output dims).
// Keys are taken 64 at a time (4 pages):
//
//   1. the block's K and V page tiles (fp32, bulk copies issued one block ahead) are
//      split into bf16 hi/lo halves in the UMMA K-major layout: K as the B operand of
//      S = Q K^T (rows = keys, K = dims), V transposed as the B operand of O = P V
//      (rows = dims, K = keys); pages past the context are zero;
//   2. one thread issues S = Qhi Khi + Qhi Klo + Qlo Khi (4 x 3 MMAs, M=128, N=64, K=64)
//      into TMEM columns 0-63;
//   3. every thread loads its half row of S, applies the causal mask, joins the row maximum
//      with its partner through shared memory and applies the online softmax (running max
//      and sum in the exp2 domain, the scores already scaled by log2(e)/sqrt(64) through
//      Q), then writes its half row of P as bf16 hi/lo;
//   4. one thread issues O_blk = P V the same way into TMEM columns 64-127; every thread
//      adds its half row of O_blk into its running output (rescaled by the max correction).
//
// The hi/lo split keeps ~17 significant bits per operand and the dropped lo*lo term is
// ~2^-17 relative, so scores and outputs agree with fp32 to ~1e-5 relative, the same
// arithmetic as the projections.  The reference's single-pass online softmax
// (src/model_q8.cpp:485-523) computes the same function up to fp32 rounding.
//
// Every mbarrier wait is bounded; a CTA whose wait gave up sets the error flag, releases
// its tensor memory and writes nothing.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <set>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace nitro {

namespace {

constexpr int FA_M = 128;                     // queries per CTA = UMMA M = TMEM lanes
constexpr int FA_THREADS = 2 * FA_M;          // two warpgroups: each row's keys and dims split in halves
constexpr int FA_N = 64;                      // keys per block = UMMA N of S
constexpr int FA_HD = 64;                     // head_dim = K of S = N of O
constexpr int FA_PAGES = FA_N / kPage;        // pages per key block
constexpr int FA_PAGE_BYTES = kPage * FA_HD * 4;  // one fp32 K (or V) page tile (bf16 pages: half)
constexpr int FA_RAW = 2 * FA_PAGES * FA_PAGE_BYTES;  // K and V tiles of one block (32 KB)
// dynamic shared memory, bytes: bf16 halves of Q [128][64], K [64][64], P [128][64],
// V^T [64][64], then two stages of raw page tiles (laid out for fp32 pages)
constexpr int OFF_QH = 0, OFF_QL = 16384, OFF_KH = 32768, OFF_KL = 40960, OFF_PH = 49152, OFF_PL = 65536,
              OFF_VH = 81920, OFF_VL = 90112, OFF_RAW = 98304;
constexpr int FA_SMEM = OFF_RAW + 2 * FA_RAW;
constexpr uint32_t FA_TMEM_COLS = 128;  // S in columns 0-63, O_blk in 64-127

template <typename KT>
__global__ void __launch_bounds__(FA_THREADS, 1) prefill_attn_tc_kernel(PrefillAttnArgs a) {
    constexpr int PAGE_BYTES = kPage * FA_HD * (int)sizeof(KT);  // one K (or V) page tile
    const KT* kpool = reinterpret_cast<const KT*>(a.kpool);
    const KT* vpool = reinterpret_cast<const KT*>(a.vpool);
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint64_t raw_bar[2], s_bar, o_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ float red[2][FA_M];  // per-row partial maxima (and, at the end, sums) of the two halves
    const int tid = threadIdx.x, warp = tid >> 5;
    const int r = tid & (FA_M - 1);  // query row = TMEM lane
    const int c = tid >> 7;          // warpgroup: keys / output dims c*32..c*32+31

    // (segment, query tile) of this CTA: longest tiles first (see prefill_attn_kernel)
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
        qt = (T + FA_M - 1) / FA_M - 1 - (int)blockIdx.x / a.n_heads;
    }
    const int t0 = qt * FA_M;
    const int nq = min(FA_M, T - t0);
    const int n_pages = (start_pos + t0 + nq - 1) / kPage + 1;
    const int n_blocks = (n_pages + FA_PAGES - 1) / FA_PAGES;
    const int kvh = h / (a.n_heads / a.geom.n_kv_heads);

    if (tid == 0) {
        mbar_init(&raw_bar[0], 1);
        mbar_init(&raw_bar[1], 1);
        mbar_init(&s_bar, 1);
        mbar_init(&o_bar, 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(&tmem_slot, FA_TMEM_COLS);
        tmem_relinquish();
    }
    // K and V tiles of key block b into raw stage b & 1 (thread 0)
    auto issue = [&](int b) {
        uint8_t* raw = smem + OFF_RAW + (b & 1) * FA_RAW;
        const int p0 = b * FA_PAGES, np = min(FA_PAGES, n_pages - p0);
        uint64_t* bar = &raw_bar[b & 1];
        mbar_arrive_expect_tx(bar, (uint32_t)(2 * np * PAGE_BYTES));
        for (int p = 0; p < np; p++) {
            const int64_t off = a.geom.tile_offset(bt[p0 + p], a.layer, kvh);
            bulk_g2s(raw + p * PAGE_BYTES, kpool + off, PAGE_BYTES, bar);
            bulk_g2s(raw + (FA_PAGES + p) * PAGE_BYTES, vpool + off, PAGE_BYTES, bar);
        }
    };
    grid_dependency_wait();  // q and this chunk's K/V rows come from the projection kernel
    if (tid == 0) issue(0);

    // half of this row's query (dims c*32..+31), pre-scaled for the exp2-domain softmax,
    // as bf16 hi/lo
    {
        const float qscale = 1.4426950408889634f / 8.0f;  // log2(e) / sqrt(64)
        const float4* src = reinterpret_cast<const float4*>(
            a.q + ((int64_t)(row0 + t0 + min(r, nq - 1)) * a.n_heads + h) * FA_HD + c * 32);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float4 x0 = src[2 * j], x1 = src[2 * j + 1];
            const float v[8] = {x0.x * qscale, x0.y * qscale, x0.z * qscale, x0.w * qscale,
                                x1.x * qscale, x1.y * qscale, x1.z * qscale, x1.w * qscale};
            split_store8(v, smem + OFF_QH + core_off(r, c * 4 + j), smem + OFF_QL + core_off(r, c * 4 + j));
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t idesc = umma_idesc_bf16(FA_M, FA_N);
    const int qpos = r < nq ? start_pos + t0 + r : -1;  // rows past the chunk attend nothing

    float o[32];  // output dims c*32..c*32+31 of row r
#pragma unroll
    for (int i = 0; i < 32; i++) o[i] = 0.0f;
    float m = -INFINITY, l = 0.0f;  // running max (shared by both halves) and this half's sum
    bool ok = true;
    for (int b = 0; b < n_blocks; b++) {
        const int st = b & 1;
        // stage b+1 was last read by block b-1's conversion, which every thread finished
        if (tid == 0 && b + 1 < n_blocks) issue(b + 1);
        if (ok && !mbar_wait(&raw_bar[st], (uint32_t)(b >> 1) & 1, a.err)) ok = false;
        const uint8_t* raw = smem + OFF_RAW + st * FA_RAW;
        const int valid_keys = min(FA_N, (n_pages - b * FA_PAGES) * kPage);
        // K: thread t converts a quarter key row (key t/4, dims (t&3)*16..+15)
        {
            const int key = tid >> 2, qd = tid & 3;
            const KT* krow = reinterpret_cast<const KT*>(raw) + key * FA_HD + qd * 16;
#pragma unroll
            for (int g = 0; g < 2; g++) {
                float v[8];
                if (key < valid_keys) {
                    const float4 x0 = ldkv4(krow + 8 * g), x1 = ldkv4(krow + 8 * g + 4);
                    v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
                    v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 8; i++) v[i] = 0.0f;
                }
                split_store8(v, smem + OFF_KH + core_off(key, qd * 2 + g), smem + OFF_KL + core_off(key, qd * 2 + g));
            }
        }
        // V transposed: thread t converts dim t/4 of keys (t&3)*16..+15
        {
            const int dim = tid >> 2, qk = tid & 3;
            const KT* vbase = reinterpret_cast<const KT*>(raw + FA_PAGES * PAGE_BYTES);
#pragma unroll
            for (int g = 0; g < 2; g++) {
                float v[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int key = qk * 16 + g * 8 + i;  // page tiles are contiguous: key * 64 + dim
                    v[i] = key < valid_keys ? ldkv1(vbase + key * FA_HD + dim) : 0.0f;
                }
                split_store8(v, smem + OFF_VH + core_off(dim, qk * 2 + g), smem + OFF_VL + core_off(dim, qk * 2 + g));
            }
        }
        fence_async_smem();  // the operands are read by the tensor cores (async proxy)
        tc_fence_before();
        ok = __syncthreads_and(ok);
        tc_fence_after();
        if (!ok) break;
        if (tid == 0) {
            const uint32_t qh = smem_addr(smem + OFF_QH), ql = smem_addr(smem + OFF_QL);
            const uint32_t kh = smem_addr(smem + OFF_KH), kl = smem_addr(smem + OFF_KL);
#pragma unroll
            for (int kk = 0; kk < FA_HD / 16; kk++) {
                const uint32_t off = kk * 256;  // 16 K elements = two core matrices
                umma_bf16(tmem, umma_desc(qh + off), umma_desc(kh + off), idesc, kk > 0 ? 1u : 0u);
                umma_bf16(tmem, umma_desc(qh + off), umma_desc(kl + off), idesc, 1u);
                umma_bf16(tmem, umma_desc(ql + off), umma_desc(kh + off), idesc, 1u);
            }
            umma_commit(&s_bar);
        }
        if (ok && !mbar_wait(&s_bar, (uint32_t)b & 1, a.err)) ok = false;
        tc_fence_after();
        // this half's 32 scores of row r; the row maximum joins both halves in shared memory
        float sc[32];
        tmem_ld32(tmem + lane_base + c * 32, sc);
        const int kpos0 = b * FA_N + c * 32;
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            if (kpos0 + j > qpos) sc[j] = -INFINITY;  // causal (and rows past the chunk)
            mx = fmaxf(mx, sc[j]);
        }
        red[c][r] = mx;
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        const float m_new = fmaxf(m, fmaxf(mx, red[c ^ 1][r]));
        const float corr = m_new == -INFINITY ? 1.0f : exp2f(m - m_new);
        float ps = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            sc[j] = m_new == -INFINITY ? 0.0f : exp2f(sc[j] - m_new);
            ps += sc[j];
        }
        l = l * corr + ps;
        m = m_new;
#pragma unroll
        for (int j = 0; j < 4; j++)
            split_store8(sc + 8 * j, smem + OFF_PH + core_off(r, c * 4 + j), smem + OFF_PL + core_off(r, c * 4 + j));
        fence_async_smem();
        tc_fence_before();
        ok = __syncthreads_and(ok);
        tc_fence_after();
        if (!ok) break;
        if (tid == 0) {
            const uint32_t ph = smem_addr(smem + OFF_PH), pl = smem_addr(smem + OFF_PL);
            const uint32_t vh = smem_addr(smem + OFF_VH), vl = smem_addr(smem + OFF_VL);
#pragma unroll
            for (int kk = 0; kk < FA_N / 16; kk++) {
                const uint32_t off = kk * 256;
                umma_bf16(tmem + 64, umma_desc(ph + off), umma_desc(vh + off), idesc, kk > 0 ? 1u : 0u);
                umma_bf16(tmem + 64, umma_desc(ph + off), umma_desc(vl + off), idesc, 1u);
                umma_bf16(tmem + 64, umma_desc(pl + off), umma_desc(vh + off), idesc, 1u);
            }
            umma_commit(&o_bar);
        }
        if (ok && !mbar_wait(&o_bar, (uint32_t)b & 1, a.err)) ok = false;
        tc_fence_after();
        {
            float ob[32];
            tmem_ld32(tmem + lane_base + 64 + c * 32, ob);
#pragma unroll
            for (int i = 0; i < 32; i++) o[i] = fmaf(o[i], corr, ob[i]);
        }
        // the next block's operands overwrite K, V^T, P and red, and its MMAs overwrite S
        // and O_blk: every thread's reads above are complete at the next block's barrier
        tc_fence_before();
    }
    grid_dependents_launch();
    // the row's sum over both halves
    red[c][r] = l;
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, FA_TMEM_COLS);
    if (!ok || r >= nq) return;
    const float inv = 1.0f / (l + red[c ^ 1][r]);
    float4* dst = reinterpret_cast<float4*>(a.out + ((int64_t)(row0 + t0 + r) * a.n_heads + h) * FA_HD + c * 32);
#pragma unroll
    for (int i = 0; i < 8; i++)
        dst[i] = make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
}

}  // namespace

bool prefill_attn_tc_enabled(int head_dim) {
    static int v = -1;
    if (v < 0) {
        const char* env = getenv("NITRO_DISABLE_TC_ATTN");
        v = (env && env[0] == '1') ? 0 : 1;
    }
    return v == 1 && head_dim == FA_HD;
}

void launch_prefill_attention_tc(const PrefillAttnArgs& a, cudaStream_t s) {
    static std::mutex mu;
    static std::set<int> configured;  // devices whose kernels have their shared-memory limit set
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!configured.count(dev)) {
            cudaFuncSetAttribute(prefill_attn_tc_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM);
            cudaFuncSetAttribute(prefill_attn_tc_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 FA_SMEM);
            configured.insert(dev);
        }
    }
    const int tiles = a.seg ? a.n_tiles : (a.T + FA_M - 1) / FA_M;
    const dim3 grid((unsigned)(tiles * a.n_heads));
    if (a.geom.kv_bf16) launch_ex(prefill_attn_tc_kernel<__nv_bfloat16>, grid, dim3(FA_THREADS), FA_SMEM, s, 1, a);
    else launch_ex(prefill_attn_tc_kernel<float>, grid, dim3(FA_THREADS), FA_SMEM, s, 1, a);
}

}  // namespace nitro
