// Q8_0 / fp32 projections on CUDA cores with fused prologue and epilogues.
//
// Three shapes:
//   * gemv_kernel, M <= 8 token rows (decode at small batch, the last prefill token):
//     HBM-bound matvec.  One warp owns an adjacent pair of output rows and streams their
//     int8 weights with 16-byte loads (16 weights per lane per step, one fp32 scale per
//     32-wide block), dequantises in registers (w = q * scale, as src/model_q8.cpp:107-111)
//     and accumulates every token row against them.
//   * gemv_ring_kernel, M <= 2 over large Q8 matrices: whole-row units streamed through a
//     shared-memory ring by a producer warp, activations held in registers.
//   * gemm_tiled_kernel, M > 8: 64x64 output tiles staged through shared memory in
//     32-wide K chunks (one Q8 block), register double-buffered, 8x4 micro-tile per thread.
//
// All apply, when asked, the RMSNorm of the input rows (src/model_q8.cpp:128-140) while
// loading them, and one of the epilogues of kernels.h.  Accumulation is fp32 throughout.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace nitro {

namespace {

std::atomic<int64_t> g_launches{0};

__device__ __forceinline__ float silu_mul(float a, float b) {
    // src/model_q8.cpp:541-542: val *= 1/(1+expf(-val)); val *= h3
    float v = a * (1.0f / (1.0f + expf(-a)));
    return v * b;
}

__device__ __forceinline__ void argmax_offer(unsigned long long* key_slot, unsigned long long key) {
    // a plain read first: most offers lose to the current maximum and skip the atomic
    if (key > *(volatile unsigned long long*)key_slot) atomicMax(key_slot, key);
}

// Epilogue for one token row m and the adjacent output rows (n, n+1), n even.
__device__ __forceinline__ void epi_pair(const Epilogue& e, int m, int n, float v0, float v1) {
    switch (e.kind) {
    case kEpiStore:
        e.out[(int64_t)m * e.ldo + n] = v0;
        e.out[(int64_t)m * e.ldo + n + 1] = v1;
        break;
    case kEpiResidual:
        e.out[(int64_t)m * e.ldo + n] += v0;
        e.out[(int64_t)m * e.ldo + n + 1] += v1;
        break;
    case kEpiSwiGLU:
        e.out[(int64_t)m * e.ldo + (n >> 1)] = silu_mul(v0, v1);
        break;
    case kEpiQKV: {
        const int D = e.dim, KV = e.kv_dim, hd = e.head_dim;
        const int pos = e.tok_pos[m];
        if (n < D + KV) {
            // RoPE pair (j, j+1), angle index (j % head)/2 (src/model_q8.cpp:601-615)
            int c = n < D ? n : n - D;
            int fi = pos * (hd >> 1) + ((c % hd) >> 1);
            float fcr = e.freq_re[fi], fci = e.freq_im[fi];
            float r0 = v0 * fcr - v1 * fci;
            float r1 = v0 * fci + v1 * fcr;
            if (n < D) {
                e.q_out[(int64_t)m * D + n] = r0;
                e.q_out[(int64_t)m * D + n + 1] = r1;
            } else {
                const int64_t at = e.geom.tile_offset(e.tok_page[m], e.layer, c / hd) +
                                   (int64_t)(pos & (kPage - 1)) * hd + (c % hd);
                store_kv(e.kpool, e.geom, at, r0);
                store_kv(e.kpool, e.geom, at + 1, r1);
            }
        } else {
            int c = n - D - KV;
            const int64_t at = e.geom.tile_offset(e.tok_page[m], e.layer, c / hd) +
                               (int64_t)(pos & (kPage - 1)) * hd + (c % hd);
            store_kv(e.vpool, e.geom, at, v0);
            store_kv(e.vpool, e.geom, at + 1, v1);
        }
        break;
    }
    default:
        break;
    }
}

__device__ __forceinline__ void load16_f32(const float* p, float* r) {
    const float4* p4 = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float4 v = __ldg(p4 + i);
        r[4 * i] = v.x; r[4 * i + 1] = v.y; r[4 * i + 2] = v.z; r[4 * i + 3] = v.w;
    }
}

// 16 consecutive Q8 weights of row n starting at k (k % 16 == 0), dequantised.
__device__ __forceinline__ void load16_q8(const int8_t* wq, const float* ws, int64_t n, int K, int k, float* r) {
    int4 raw = __ldg(reinterpret_cast<const int4*>(wq + n * K + k));
    float s = __ldg(ws + n * (K >> 5) + (k >> 5));
    const int8_t* q = reinterpret_cast<const int8_t*>(&raw);
#pragma unroll
    for (int i = 0; i < 16; i++) r[i] = (float)q[i] * s;
}

// Per-row inverse RMS of x rows [m0, m0+count) into inv[] (one warp per row).
__device__ __forceinline__ void rms_rows(const float* x, int ldx, int K, int m0, int count, int M, float* inv) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int r = warp; r < count; r += nw) {
        int m = m0 + r;
        float ss = 0.0f;
        if (m < M) {
            const float* row = x + (int64_t)m * ldx;
            for (int k = lane * 4; k < K; k += 128) {
                float4 v = *reinterpret_cast<const float4*>(row + k);
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
        }
        ss = warp_sum(ss);
        if (lane == 0) inv[r] = 1.0f / sqrtf(ss / (float)K + 1e-5f);
    }
}

// ------------------------------------------------------------------ matvec, M <= 8
// One warp per adjacent pair of output rows; lane l covers K positions l*16 + 512 i.
// The weights of the first GV_PF steps (all of K up to 2048 for Q8, 1024 for fp32) are
// requested before the grid-dependency wait, i.e. while the previous kernel still runs,
// and each step's slot is refilled GV_PF steps ahead; only the activations wait.  The
// RMSNorm is folded into the dot product: every warp sees each whole input row anyway,
// so it sums x^2 alongside w . (g * x) and scales by 1/rms at the end (the faithful
// mode, which reads only the last block, computes the row sums separately).
constexpr int GV_PF = 4;  // Q8 steps prefetched (2 for fp32 weights)

template <bool F32W>
struct GvW {  // one step's weights of the warp's two rows for this lane
    int4 q[F32W ? 1 : 2];
    float s[F32W ? 1 : 2];
    float4 f[F32W ? 8 : 1];
};

template <bool F32W>
__device__ __forceinline__ void gv_load(GvW<F32W>& w, const GemmArgs& a, int n, int k) {
    if (F32W) {
        const float4* r0 = reinterpret_cast<const float4*>(a.wf + (int64_t)n * a.K + k);
        const float4* r1 = reinterpret_cast<const float4*>(a.wf + (int64_t)(n + 1) * a.K + k);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            w.f[i] = __ldg(r0 + i);
            w.f[4 + i] = __ldg(r1 + i);
        }
    } else {
        w.q[0] = __ldg(reinterpret_cast<const int4*>(a.wq + (int64_t)n * a.K + k));
        w.q[1] = __ldg(reinterpret_cast<const int4*>(a.wq + (int64_t)(n + 1) * a.K + k));
        w.s[0] = __ldg(a.ws + (int64_t)n * (a.K >> 5) + (k >> 5));
        w.s[1] = __ldg(a.ws + (int64_t)(n + 1) * (a.K >> 5) + (k >> 5));
    }
}

// Four int8 (one 32-bit word) -> exact floats: with the sign bit flipped each byte is
// q + 128; placed in the low mantissa byte of 2^23 it reads 2^23 + q + 128.
__device__ __forceinline__ void q8x4_to_f32(uint32_t w, float* f) {
    const uint32_t u = w ^ 0x80808080u;
    f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - 8388736.0f;
    f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - 8388736.0f;
    f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - 8388736.0f;
    f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - 8388736.0f;
}

// Long rows (K beyond 2048 / 4096) are split over 2 / 4 warps of the CTA, which then
// join their partial sums through shared memory.
__host__ __device__ inline int gv_ksplit(int k_len) { return k_len > 4096 ? 4 : (k_len > 2048 ? 2 : 1); }

template <int MT, bool F32W>
__global__ void __launch_bounds__(128) gemv_kernel(GemmArgs a, Epilogue e) {
    constexpr int WARPS = 4;
    constexpr int PF = F32W ? 2 : GV_PF;
    __shared__ float inv_rms[MT];
    __shared__ float part[WARPS][MT][3];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool norm = a.norm_gain != nullptr;
    const bool fold = norm && a.kbegin == 0;  // 1/rms from the warps' own pass over x
    const int KW = gv_ksplit(a.K - a.kbegin);
    const int kw = warp % KW;                  // this warp's share of the row pair's K range
    const int n = (blockIdx.x * (WARPS / KW) + warp / KW) * 2;
    const bool active = n < a.N;
    const int k0 = a.kbegin + kw * 512 + lane * 16;
    const int kstep = 512 * KW;

    // ---- before the wait: weights (read-only)
    GvW<F32W> wp[PF];
#pragma unroll
    for (int i = 0; i < PF; i++)
        if (active && k0 + kstep * i < a.K) gv_load<F32W>(wp[i], a, n, k0 + kstep * i);
    grid_dependency_wait();
    if (norm && !fold) {
        rms_rows(a.x, a.ldx, a.K, 0, MT, a.M, inv_rms);
        __syncthreads();
    }
    float acc0[MT], acc1[MT], ss[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) acc0[m] = acc1[m] = ss[m] = 0.0f;

    // slot j of the register ring holds step i0 + j; after it is used it is refilled with
    // step i0 + j + PF, so PF steps of weights stay in flight
#pragma unroll 1
    for (int i0 = 0; active && k0 + kstep * i0 < a.K; i0 += PF)
#pragma unroll
    for (int j = 0; j < PF; j++) {
        const int i = i0 + j;
        const int k = k0 + kstep * i;
        if (k >= a.K) break;
        const GvW<F32W> wcur = wp[j];
        if (k + kstep * PF < a.K) gv_load<F32W>(wp[j], a, n, k + kstep * PF);
        float g[16];
        if (norm) load16_f32(a.norm_gain + k, g);  // with the activations: no extra round trip
#pragma unroll
        for (int m = 0; m < MT; m++) {
            if (m < a.M) {
                float xv[16];
                load16_f32(a.x + (int64_t)m * a.ldx + k, xv);
                if (norm) {
                    const float sc = fold ? 1.0f : inv_rms[m];
                    float q = 0.0f;
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        q = fmaf(xv[j], xv[j], q);
                        xv[j] = g[j] * (sc * xv[j]);
                    }
                    ss[m] += q;
                }
                float s0 = 0.0f, s1 = 0.0f;
                if (F32W) {
#pragma unroll
                    for (int q4 = 0; q4 < 4; q4++) {
                        const float4 a4 = wcur.f[q4], b4 = wcur.f[4 + q4];
                        s0 = fmaf(a4.x, xv[4 * q4], s0); s0 = fmaf(a4.y, xv[4 * q4 + 1], s0);
                        s0 = fmaf(a4.z, xv[4 * q4 + 2], s0); s0 = fmaf(a4.w, xv[4 * q4 + 3], s0);
                        s1 = fmaf(b4.x, xv[4 * q4], s1); s1 = fmaf(b4.y, xv[4 * q4 + 1], s1);
                        s1 = fmaf(b4.z, xv[4 * q4 + 2], s1); s1 = fmaf(b4.w, xv[4 * q4 + 3], s1);
                    }
                } else {
                    // sum_k q_k x_k over this lane's 16 weights (one Q8 block), times the
                    // block's scale; q -> float through the exponent trick (full-rate ALU
                    // ops instead of the quarter-rate integer conversion)
                    const uint32_t* w0 = reinterpret_cast<const uint32_t*>(&wcur.q[0]);
                    const uint32_t* w1 = reinterpret_cast<const uint32_t*>(&wcur.q[1]);
#pragma unroll
                    for (int wi = 0; wi < 4; wi++) {
                        float f0[4], f1[4];
                        q8x4_to_f32(w0[wi], f0);
                        q8x4_to_f32(w1[wi], f1);
#pragma unroll
                        for (int b = 0; b < 4; b++) {
                            s0 = fmaf(f0[b], xv[4 * wi + b], s0);
                            s1 = fmaf(f1[b], xv[4 * wi + b], s1);
                        }
                    }
                    s0 *= wcur.s[0];
                    s1 *= wcur.s[1];
                }
                acc0[m] += s0;
                acc1[m] += s1;
            }
        }
    }
    grid_dependents_launch();
#pragma unroll
    for (int m = 0; m < MT; m++) {
        acc0[m] = warp_sum(acc0[m]);
        acc1[m] = warp_sum(acc1[m]);
        if (fold) ss[m] = warp_sum(ss[m]);
    }
    if (KW > 1) {  // join the K shares of each row pair (uniform branch: every warp takes it)
        if (lane == 0)
#pragma unroll
            for (int m = 0; m < MT; m++) {
                part[warp][m][0] = acc0[m];
                part[warp][m][1] = acc1[m];
                part[warp][m][2] = ss[m];
            }
        __syncthreads();
#pragma unroll
        for (int m = 0; m < MT; m++) {
            acc0[m] = acc1[m] = ss[m] = 0.0f;
            for (int t = warp - kw; t < warp - kw + KW; t++) {  // in warp order: deterministic
                acc0[m] += part[t][m][0];
                acc1[m] += part[t][m][1];
                ss[m] += part[t][m][2];
            }
        }
    }
    if (fold) {
#pragma unroll
        for (int m = 0; m < MT; m++) {
            const float inv = 1.0f / sqrtf(ss[m] / (float)a.K + 1e-5f);
            acc0[m] *= inv;
            acc1[m] *= inv;
        }
    }
    if (!active || kw != 0) return;
#pragma unroll
    for (int m = 0; m < MT; m++) {
        if (m < a.M && lane == m) {
            if (e.kind == kEpiLogits) {
                if (e.out) {
                    e.out[(int64_t)m * e.ldo + n] = acc0[m];
                    e.out[(int64_t)m * e.ldo + n + 1] = acc1[m];
                }
                // n before n+1: the smaller index wins a tie
                float best = acc0[m];
                int bi = n;
                if (acc1[m] > best) { best = acc1[m]; bi = n + 1; }
                if (best > 0.0f) argmax_offer(e.argmax_keys + m, argmax_key(best, bi));
            } else {
                epi_pair(e, m, n, acc0[m], acc1[m]);
            }
        }
    }
}

// ------------------------------------------------------------------ ring matvec, M <= 2
// Large Q8 matrices at one or two token rows (decode at batch 1-2; the 7B shape's
// projections).  One CTA per SM takes a contiguous range of units of G whole rows: their
// int8 rows and scales are contiguous in the row-major arrays, so one producer thread
// streams each unit with two bulk copies into a ring of shared-memory slots, requested
// before the grid-dependency wait for the first slots.  16 consumer warps read every
// unit, warp w taking row w % G and K segment w / G of 16 / G; a lane's share of its
// segment sits at the same K positions in every unit, so the lane keeps those activations
// (times the RMSNorm gain, as packed pairs) in registers for the whole launch, and the
// inner loop is one 16-byte shared load per 16 weights, one byte permute per weight
// (int8 -> exact float, as q8_pair_biased) and packed f32x2 adds and FMAs; the block scale
// multiplies each 16-weight partial (the products of src/model_q8.cpp:107-111, summed in
// another order).  Segment partials meet in shared memory: after one named barrier of the
// consumer warps per unit, warp w < G / 2 adds row pair (2w, 2w + 1)'s partials in segment
// order and runs the epilogue.  Each warp releases the slot to the producer as soon as its
// lanes have read their weights, before the reduction.
constexpr int GR_CONSUMERS = 16;
constexpr int GR_THREADS = (GR_CONSUMERS + 1) * 32;
constexpr int GR_SLOTS_MAX = 8;
constexpr int GR_XPAIRS = 32;  // activation pairs a lane may hold: MT x CPL x 8

struct RingPlan {
    int G;           // rows per unit: 2, 4 or 8
    int slot_bytes;  // G x (K + K / 8)
    int slots;
    int units;       // N / G
};

// Named barrier 1 over the consumer warps of the ring matvec (the producer warp is not in it).
__device__ __forceinline__ void gr_consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(GR_CONSUMERS * 32) : "memory");
}

template <int MT, int CPL>
__global__ void __launch_bounds__(GR_THREADS, 1) gemv_ring_kernel(GemmArgs a, Epilogue e, RingPlan rp) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[GR_SLOTS_MAX], empty[GR_SLOTS_MAX];
    __shared__ float part[GR_SLOTS_MAX][8][8][MT];  // [slot][row of unit][segment][token]
    __shared__ float red[GR_CONSUMERS + 1][MT];
    __shared__ float inv_rms[MT];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = a.K, G = rp.G, S = GR_CONSUMERS / G, L = K / S;
    const int u0 = (int)((int64_t)blockIdx.x * rp.units / gridDim.x);
    const int nu = (int)((int64_t)(blockIdx.x + 1) * rp.units / gridDim.x) - u0;
    const bool producer = warp == GR_CONSUMERS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < rp.slots; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GR_CONSUMERS);
        }
        fence_barrier_init();
    }
    __syncthreads();
    auto fetch = [&](int i) {  // unit u0 + i -> slot i % slots
        const int s = i % rp.slots;
        uint8_t* dst = smem + (size_t)s * rp.slot_bytes;
        const int64_t n = (int64_t)(u0 + i) * G;
        mbar_arrive_expect_tx(&full[s], (uint32_t)(G * (K + K / 8)));
        bulk_g2s(dst, a.wq + n * K, (uint32_t)(G * K), &full[s]);
        bulk_g2s(dst + G * K, a.ws + n * (K / 32), (uint32_t)(G * K / 8), &full[s]);
    };
    // weights are read-only: the first units are requested before the dependency wait
    if (producer && lane == 0)
        for (int i = 0; i < min(nu, rp.slots); i++) fetch(i);
    grid_dependency_wait();

    // consumer geometry: row r of every unit, K segment sg; the lane's chunks of 16
    const int r = warp % G, sg = warp / G;
    const int kseg = sg * L;
    // the lane's activations (times the gain) as packed pairs, and the RMSNorm sums
    unsigned long long xp[MT][CPL * 8];
    float ss[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) ss[m] = 0.0f;
    if (!producer) {
#pragma unroll
        for (int c = 0; c < CPL; c++) {
            const int k = kseg + (lane + 32 * c) * 16;
            const bool valid = (lane + 32 * c) * 16 < L;
#pragma unroll
            for (int m = 0; m < MT; m++) {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (valid && m < a.M) v = *reinterpret_cast<const float4*>(a.x + (int64_t)m * a.ldx + k + 4 * j);
                    ss[m] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                    if (valid && a.norm_gain) {
                        const float4 g = __ldg(reinterpret_cast<const float4*>(a.norm_gain + k + 4 * j));
                        v.x *= g.x; v.y *= g.y; v.z *= g.z; v.w *= g.w;
                    }
                    xp[m][c * 8 + 2 * j] = pack2(__float_as_uint(v.x), __float_as_uint(v.y));
                    xp[m][c * 8 + 2 * j + 1] = pack2(__float_as_uint(v.z), __float_as_uint(v.w));
                }
            }
        }
    }
    // 1/rms of each token row: the warps of row 0 of the unit hold every K position once
    if (a.norm_gain) {
#pragma unroll
        for (int m = 0; m < MT; m++) {
            const float t = warp_sum(ss[m]);
            if (lane == 0) red[warp][m] = (!producer && r == 0) ? t : 0.0f;
        }
    }
    __syncthreads();
    if (a.norm_gain && threadIdx.x < MT) {
        float t = 0.0f;
        for (int w = 0; w < GR_CONSUMERS; w++) t += red[w][threadIdx.x];
        inv_rms[threadIdx.x] = 1.0f / sqrtf(t / (float)K + 1e-5f);
    }
    __syncthreads();

    if (producer) {
        // refill each slot once all consumer warps have released it
        if (lane == 0) {
            bool ok = true;
            for (int i = rp.slots; i < nu && ok; i++) {
                const int s = i % rp.slots;
                if (!mbar_wait(&empty[s], ((i / rp.slots) - 1) & 1, a.err)) ok = false;
                else fetch(i);
            }
        }
        grid_dependents_launch();
        return;
    }
    const unsigned long long unb = q8_unbias2();
    bool ok = true;
    int s = 0;         // slot of unit i
    uint32_t ph = 0;   // its fill parity
    const uint8_t* slot_base = smem;
    for (int i = 0; i < nu; i++) {
        if (ok && !mbar_wait(&full[s], ph, a.err)) ok = false;
        const uint8_t* q = slot_base + (size_t)r * K + kseg;
        const float* sc = reinterpret_cast<const float*>(slot_base + (size_t)G * K) + (size_t)r * (K / 32) + (kseg >> 5);
        float acc[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) acc[m] = 0.0f;
        if (ok) {
#pragma unroll
            for (int c = 0; c < CPL; c++) {
                const int kl = (lane + 32 * c) * 16;
                if (kl < L) {
                    const uint4 w4 = *reinterpret_cast<const uint4*>(q + kl);
                    const float bs = sc[kl >> 5];
                    const uint32_t u[4] = {w4.x ^ 0x80808080u, w4.y ^ 0x80808080u, w4.z ^ 0x80808080u,
                                           w4.w ^ 0x80808080u};
                    unsigned long long d[MT];
#pragma unroll
                    for (int m = 0; m < MT; m++) d[m] = 0ull;
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const unsigned long long qv = add2(q8_pair_biased(u[j >> 1], (j & 1) * 2), unb);
#pragma unroll
                        for (int m = 0; m < MT; m++) d[m] = fma2(qv, xp[m][c * 8 + j], d[m]);
                    }
#pragma unroll
                    for (int m = 0; m < MT; m++) {
                        uint32_t lo, hi;
                        unpack2(d[m], lo, hi);
                        acc[m] = fmaf(__uint_as_float(lo) + __uint_as_float(hi), bs, acc[m]);
                    }
                }
            }
        }
        __syncwarp();  // every lane has read its weights and scales from the slot
        if (lane == 0) mbar_arrive(&empty[s]);  // the refill may start during the reduction
#pragma unroll
        for (int m = 0; m < MT; m++) acc[m] = warp_sum(acc[m]);
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < MT; m++) part[s][r][sg][m] = acc[m];
        }
        // every consumer warp passes this barrier once per unit, so the counts match; the
        // unit's partials are then complete, and part[s] is next written `slots` units later,
        // after the readers below have passed the following units' barriers
        gr_consumer_sync();
        if (warp < G / 2 && lane < MT && lane < a.M && ok) {  // row pair (2 warp, 2 warp + 1)
            const int r0 = 2 * warp;
            float v0 = 0.0f, v1 = 0.0f;
            for (int t = 0; t < S; t++) {
                v0 += part[s][r0][t][lane];
                v1 += part[s][r0 + 1][t][lane];
            }
            if (a.norm_gain) {
                v0 *= inv_rms[lane];
                v1 *= inv_rms[lane];
            }
            epi_pair(e, lane, (u0 + i) * G + r0, v0, v1);
        }
        if (++s == rp.slots) {
            s = 0;
            ph ^= 1u;
            slot_base = smem;
        } else {
            slot_base += rp.slot_bytes;
        }
    }
    grid_dependents_launch();
}

// Whether the ring matvec takes this launch, and its shape: whole-row units of at most
// 48 KB, the lane's activations in at most GR_XPAIRS packed pairs, at least 3 ring slots.
bool ring_plan(const GemmArgs& a, RingPlan* rp, int* cpl) {
    if (a.wf || !a.wq || a.M > 2 || a.kbegin != 0 || a.K % 32 != 0 || a.N % 2 != 0) return false;
    if (reinterpret_cast<uintptr_t>(a.wq) % 16 || reinterpret_cast<uintptr_t>(a.ws) % 16) return false;
    if ((int64_t)a.N * a.K < ((int64_t)4 << 20)) return false;  // small matrices: launch latency rules
    for (int G = 8; G >= 2; G /= 2) {
        const int S = GR_CONSUMERS / G;
        if (a.N % G || a.K % (16 * S)) continue;
        const int slot = G * (a.K + a.K / 8);
        // every unit's two copies start and end on 16-byte boundaries
        if (slot > 48 * 1024 || (G * a.K) % 16 || (G * a.K / 8) % 16) continue;
        const int c = (a.K / S / 16 + 31) / 32;
        if (c < 1 || a.M * c * 8 > GR_XPAIRS) continue;
        rp->G = G;
        rp->slot_bytes = slot;
        rp->slots = std::min(GR_SLOTS_MAX, (200 * 1024) / slot);
        rp->units = a.N / G;
        *cpl = c;
        return rp->slots >= 3;
    }
    return false;
}

// ------------------------------------------------------------------ tiled, M > 8
constexpr int TN = 64, TM = 64, KC = 32;

template <bool F32W>
__global__ void __launch_bounds__(128) gemm_tiled_kernel(GemmArgs a, Epilogue e) {
    __shared__ __align__(16) float Ws[2][KC][TN];
    __shared__ __align__(16) float Xs[2][KC][TM];
    __shared__ float inv_rms[TM];
    const int tid = threadIdx.x;
    const int n_base = blockIdx.x * TN, m_base = blockIdx.y * TM;
    const bool norm = a.norm_gain != nullptr;
    grid_dependency_wait();
    if (norm) {
        rms_rows(a.x, a.ldx, a.K, m_base, TM, a.M, inv_rms);
        __syncthreads();
    }
    const int tn = tid & 15, tm = tid >> 4;      // compute: 4 n x 8 m per thread
    const int lr = tid >> 1, lh = (tid & 1) * 16;  // loader: row/token lr, k half lh
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;

    float wreg[16], xreg[16];
    auto load_chunk = [&](int kc) {
        const int n = n_base + lr;
        if (n < a.N) {
            if (F32W) load16_f32(a.wf + (int64_t)n * a.K + kc + lh, wreg);
            else load16_q8(a.wq, a.ws, n, a.K, kc + lh, wreg);
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++) wreg[i] = 0.0f;
        }
        const int m = m_base + lr;
        if (m < a.M) {
            load16_f32(a.x + (int64_t)m * a.ldx + kc + lh, xreg);
            if (norm) {
                float g[16];
                load16_f32(a.norm_gain + kc + lh, g);
                float inv = inv_rms[lr];
#pragma unroll
                for (int i = 0; i < 16; i++) xreg[i] = g[i] * (inv * xreg[i]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++) xreg[i] = 0.0f;
        }
    };
    auto store_chunk = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
            Ws[buf][lh + i][lr] = wreg[i];
            Xs[buf][lh + i][lr] = xreg[i];
        }
    };

    const int nk = (a.K - a.kbegin) / KC;
    load_chunk(a.kbegin);
    store_chunk(0);
    __syncthreads();
    for (int c = 0; c < nk; c++) {
        const int buf = c & 1;
        if (c + 1 < nk) load_chunk(a.kbegin + (c + 1) * KC);
#pragma unroll
        for (int k = 0; k < KC; k++) {
            float4 w = *reinterpret_cast<const float4*>(&Ws[buf][k][tn * 4]);
            float4 x0 = *reinterpret_cast<const float4*>(&Xs[buf][k][tm * 8]);
            float4 x1 = *reinterpret_cast<const float4*>(&Xs[buf][k][tm * 8 + 4]);
            float wv[4] = {w.x, w.y, w.z, w.w};
            float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = fmaf(wv[i], xv[j], acc[i][j]);
        }
        if (c + 1 < nk) store_chunk(buf ^ 1);
        __syncthreads();
    }

    grid_dependents_launch();
    const int n0 = n_base + tn * 4;
    if (e.kind == kEpiLogits) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int m = m_base + tm * 8 + j;
            unsigned long long best = 0ull;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int n = n0 + i;
                if (n < a.N && m < a.M) {
                    if (e.out) e.out[(int64_t)m * e.ldo + n] = acc[i][j];
                    if (acc[i][j] > 0.0f) {
                        unsigned long long k = argmax_key(acc[i][j], n);
                        best = k > best ? k : best;
                    }
                }
            }
            // the 16 lanes sharing tm hold the tile's 64 columns of row m
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) {
                unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
                best = other > best ? other : best;
            }
            if (tn == 0 && best != 0ull && m < a.M) argmax_offer(e.argmax_keys + m, best);
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int m = m_base + tm * 8 + j;
        if (m >= a.M) continue;
#pragma unroll
        for (int i = 0; i < 4; i += 2) {
            const int n = n0 + i;
            if (n < a.N) epi_pair(e, m, n, acc[i][j], acc[i + 1][j]);
        }
    }
}

template <int MT>
void gemv_dispatch(const GemmArgs& a, const Epilogue& e, cudaStream_t s) {
    const int pairs_per_cta = 4 / gv_ksplit(a.K - a.kbegin);
    dim3 grid((a.N / 2 + pairs_per_cta - 1) / pairs_per_cta);
    if (a.wf) launch_ex(gemv_kernel<MT, true>, grid, dim3(128), 0, s, 1, a, e);
    else launch_ex(gemv_kernel<MT, false>, grid, dim3(128), 0, s, 1, a, e);
}

}  // namespace

static bool stream_disabled() {
    static int v = -1;
    if (v < 0) {
        const char* env = getenv("NITRO_STREAM_GEMV");
        v = (env && env[0] == '0') ? 1 : 0;
    }
    return v == 1;
}

static bool tc_disabled() {
    static int v = -1;
    if (v < 0) {
        const char* env = getenv("NITRO_DISABLE_TC");
        v = (env && env[0] == '1') ? 1 : 0;
    }
    return v == 1;
}

bool gemm_uses_tc(int M, int N, int K) {
    GemmArgs g;
    g.M = M; g.N = N; g.K = K;
    return M > 8 && !tc_disabled() && tc_gemm_supported(g);
}

template <int MT, int CPL>
void launch_ring(const GemmArgs& a, const Epilogue& e, const RingPlan& rp, cudaStream_t s) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);  // cached by the runtime
    if (sms <= 0) sms = 148;
    const int smem = rp.slots * rp.slot_bytes;
    cudaFuncSetAttribute(gemv_ring_kernel<MT, CPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    const int grid = std::max(1, std::min(sms, rp.units));
    launch_ex(gemv_ring_kernel<MT, CPL>, dim3(grid), dim3(GR_THREADS), smem, s, 1, a, e, rp);
}

template <int MT>
void dispatch_ring(const GemmArgs& a, const Epilogue& e, const RingPlan& rp, int cpl, cudaStream_t s) {
    if (cpl <= 1) launch_ring<MT, 1>(a, e, rp, s);
    else if (cpl <= 2) launch_ring<MT, 2>(a, e, rp, s);
    else if (MT == 1 && cpl <= 3) launch_ring<MT, (MT == 1 ? 3 : 2)>(a, e, rp, s);
    else launch_ring<MT, (MT == 1 ? 4 : 2)>(a, e, rp, s);
}

void launch_gemm(const GemmArgs& a, const Epilogue& e, cudaStream_t s) {
    if (!tc_disabled() && tc_gemm_supported(a)) {
        launch_tc_gemm(a, e, s);
        return;
    }
    g_launches++;
    RingPlan rp;
    int cpl = 0;
    if (!stream_disabled() && ring_plan(a, &rp, &cpl)) {
        if (a.M <= 1) dispatch_ring<1>(a, e, rp, cpl, s);
        else dispatch_ring<2>(a, e, rp, cpl, s);
        return;
    }
    if (a.M <= 1) gemv_dispatch<1>(a, e, s);
    else if (a.M <= 2) gemv_dispatch<2>(a, e, s);
    else if (a.M <= 4) gemv_dispatch<4>(a, e, s);
    else if (a.M <= 8) gemv_dispatch<8>(a, e, s);
    else {
        dim3 grid((a.N + TN - 1) / TN, (a.M + TM - 1) / TM);
        if (a.wf) launch_ex(gemm_tiled_kernel<true>, grid, dim3(128), 0, s, 1, a, e);
        else launch_ex(gemm_tiled_kernel<false>, grid, dim3(128), 0, s, 1, a, e);
    }
}

int64_t kernel_launch_count() { return g_launches.load(); }
void count_launch() { g_launches++; }

}  // namespace nitro
