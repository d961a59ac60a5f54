// Device helpers shared by the engine's sm_100a kernels: bulk (TMA, non-tensor) copies
// global -> shared completed on an mbarrier, bounded mbarrier waits, warp reductions and
// the KV page addressing.
#pragma once
#include <cstdint>
#include <cstdlib>
#include <utility>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace nitro {

constexpr int kPage = 16;  // tokens per KV page (src/pagedMemory.hpp:9)

// Error codes a kernel records in its error flag (first writer wins).
constexpr int kErrWaitTimeout = 1;
// A decode context length outside [1, max_pages * 16]: the kernel clamps it into
// [0, max_pages * 16] (a row with no tokens left gets a zero output) and goes on.
constexpr int kErrBadContext = 2;

// Time limit of every mbarrier wait (nanoseconds of %globaltimer).  A wait that gives up
// sets the kernel's error flag; the kernel then skips the work that needed the data.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

// Page layout of the device K and V pools, in elements (fp32, or bf16 with kv_bf16 = 1).
// Page-major (pages == 0): [page][layer][kv_head][16][head_dim], a page's layers together.
// Layer-major (pages = the pool's page count): [layer][page][kv_head][16][head_dim], so the
// tiles one layer's attention reads lie in one region of 1/n_layers of the pool.  Either way
// the 16 rows of one (page, layer, kv_head) form one contiguous tile of 16*head_dim elements.
// Offsets below count elements.
struct PoolGeom {
    int n_layers;
    int n_kv_heads;
    int head_dim;
    int kv_bf16 = 0;
    int64_t pages = 0;
    __host__ __device__ int elem_bytes() const { return kv_bf16 ? 2 : 4; }
    // elements of one page over all layers
    __host__ __device__ int64_t page_floats() const { return (int64_t)n_layers * n_kv_heads * kPage * head_dim; }
    // elements of one (page, layer): all kv heads' tiles, contiguous in both layouts
    __host__ __device__ int64_t layer_floats() const { return (int64_t)n_kv_heads * kPage * head_dim; }
    // distance between the same (layer, kv_head) tile of consecutive pages
    __host__ __device__ int64_t page_stride() const { return pages ? layer_floats() : page_floats(); }
    __host__ __device__ int64_t tile_offset(int64_t page, int layer, int kvh) const {
        const int64_t slab = pages ? (int64_t)layer * pages + page : page * n_layers + layer;
        return slab * layer_floats() + (int64_t)kvh * kPage * head_dim;
    }
};

#if defined(__CUDACC__)
// K/V page elements (from shared memory) as fp32: fp32 pages load as they are; bf16 pages
// hold the upper 16 bits of an fp32, so a shift widens them exactly.
__device__ __forceinline__ float4 ldkv4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ldkv4(const __nv_bfloat16* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xffff0000u));
}
__device__ __forceinline__ float2 ldkv2(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ float2 ldkv2(const __nv_bfloat16* p) {
    const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
__device__ __forceinline__ float ldkv1(const float* p) { return *p; }
__device__ __forceinline__ float ldkv1(const __nv_bfloat16* p) {
    return __uint_as_float((uint32_t)*reinterpret_cast<const uint16_t*>(p) << 16);
}

// Store one K or V value at element index idx of a pool of geometry g (the K/V append).
__device__ __forceinline__ void store_kv(float* pool, const PoolGeom& g, int64_t idx, float v) {
    if (g.kv_bf16) reinterpret_cast<__nv_bfloat16*>(pool)[idx] = __float2bfloat16_rn(v);
    else pool[idx] = v;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async proxy (the bulk-copy engine).
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// One bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from global
// to this CTA's shared memory; completion is signalled on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(1000u)  // suspend at most ~1 us per poll
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wait for phase `parity` of `bar` to complete, for at most kWaitLimitNs.  On timeout
// the error flag is set and false returned; the caller skips the work that needed the
// data and returns.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15) == 0 && global_ns() - t0 > kWaitLimitNs) break;
    }
    if (err) atomicCAS(err, 0, kErrWaitTimeout);
    return false;
}

// Programmatic dependent launch: wait until the previous kernel in the stream has
// completed and its writes are visible (a no-op when launched without the attribute), and
// allow the next kernel to start its independent prologue early.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Two fp32 values in one 64-bit register for sm_100's packed f32x2 arithmetic (one
// instruction for both lanes, each rounded as the scalar operation would be).
__device__ __forceinline__ unsigned long long pack2(uint32_t lo, uint32_t hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ void unpack2(unsigned long long v, uint32_t& lo, uint32_t& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long sub2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
// int8 weights to exact floats without a conversion instruction: with u = q + 128 (the
// byte xor 0x80) in the low byte of 0x4B000000 the float is 2^23 + u, and adding
// -(2^23 + 128) (bits 0xCB000080) leaves q exactly.  Bytes b and b + 1 (b even) of a word
// that is already xor 0x80808080:
__device__ __forceinline__ unsigned long long q8_pair_biased(uint32_t u, int b) {
    return pack2(__byte_perm(u, 0x4B000000u, 0x7540 + b), __byte_perm(u, 0x4B000000u, 0x7541 + b));
}
__device__ __forceinline__ unsigned long long q8_unbias2() { return pack2(0xCB000080u, 0xCB000080u); }

// Release / acquire flags between CTAs of one grid (GPU scope).
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Greedy-sampling key: larger key = larger logit, ties broken towards the smaller index,
// so an atomicMax over keys reproduces argmax's "first strictly greater" rule
// (src/model_q8.cpp:559-569).  Only logits > 0 produce candidates; the initial key
// encodes (0.0f, index 0), the reference's starting point.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}
#endif  // __CUDACC__

constexpr unsigned long long kArgmaxInitKey = (0x80000000ull << 32) | 0xffffffffull;

// Programmatic dependent launch for every engine kernel (NITRO_PDL=0 turns it off): each
// kernel waits (griddepcontrol.wait) before touching what earlier kernels produce, so the
// launch of kernel N+1 and its independent prologue overlap kernel N's tail.
inline bool pdl_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* env = getenv("NITRO_PDL");
        v = (env && env[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

template <typename Kern, typename... Args>
inline cudaError_t launch_ex(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, unsigned cluster_x,
                             Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    unsigned n = 0;
    if (pdl_enabled()) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        n++;
    }
    if (cluster_x > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = cluster_x;
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = 1;
        n++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace nitro
