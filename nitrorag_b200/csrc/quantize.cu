// Q8_0 quantizer on the GPU: scripts/quantize.py (nvivek17/NitroRAG) byte for byte.
//
// quantize.py:7-23, per 32 consecutive weights of a tensor (the last block may be
// shorter): absmax = max |w|; scale = absmax / 127 in fp32 (1e-9 when absmax is 0);
// q = round(w / scale) with round-half-to-even (Python's round of a float32), clamped to
// [-128, 127]; the block is written as the fp32 scale (4 bytes, little endian) followed by
// its q bytes.  NumPy evaluates both divisions in float32 (a Python float operand is
// weakly typed), so IEEE fp32 division with round-to-nearest (`__fdiv_rn`) and
// `__float2int_rn` reproduce them exactly; denormals are kept (no flush-to-zero).
//
// The work is pure streaming (4 bytes in, 1.125 bytes out per weight), so the kernel is
// written for HBM: a group is four blocks (128 weights, 512 bytes), one 16-byte load per
// lane; a warp loads eight consecutive groups (4 KB; 4 and 16 measured 0.78 and 0.68 of
// HBM against 0.80) before it reduces each block's absmax over
// the 8 lanes that hold it and writes each group's 144 output bytes with 4-byte stores
// (144 = 4 x 36, so every store is aligned).  The tensor's last partial group takes a
// scalar path.  (Assembling a warp step's 576 output bytes in shared memory for 16-byte
// stores measured slower: 4.93 against 5.12 TB/s.)
//
// quantize_model_file is the script's driver (quantize.py:27-60): the header and the fp32
// tensors are copied, the seven projection tensors quantized, each as one flat array.
// Files are streamed through two pinned slots so reading, the GPU pass and writing
// overlap.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/nitro_engine.h"
#include "common.cuh"
#include "kernels.h"

namespace nitro {

namespace {

constexpr int kQBlock = 32;
constexpr int kGroup = 4 * kQBlock;          // weights per warp step
constexpr int kGroupOut = 4 * (4 + kQBlock);  // output bytes per group

__device__ __forceinline__ float q8_scale(float absmax) { return absmax != 0.0f ? __fdiv_rn(absmax, 127.0f) : 1e-9f; }

__device__ __forceinline__ uint32_t q8_byte(float w, float scale) {
    int q = __float2int_rn(__fdiv_rn(w, scale));
    q = max(-128, min(127, q));
    return (uint32_t)(q & 0xff);
}

// One full group: the lane's 4 weights -> its 4 bytes (and, for the first lane of each
// block, the block's scale), written at group_out (shared or global memory).
__device__ __forceinline__ void q8_group(float4 v, uint8_t* group_out, int lane) {
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    const float s = q8_scale(m);
    const uint32_t packed =
        q8_byte(v.x, s) | (q8_byte(v.y, s) << 8) | (q8_byte(v.z, s) << 16) | (q8_byte(v.w, s) << 24);
    uint8_t* blk = group_out + (lane >> 3) * (4 + kQBlock);
    const int sub = lane & 7;  // this lane's float4 inside its block
    if (sub == 0) *reinterpret_cast<float*>(blk) = s;
    *reinterpret_cast<uint32_t*>(blk + 4 + 4 * sub) = packed;
}

#ifndef NITRO_Q8_UNROLL
#define NITRO_Q8_UNROLL 8
#endif
constexpr int kUnroll = NITRO_Q8_UNROLL;  // groups per warp step: 4 KB of loads in flight

__global__ void __launch_bounds__(256) q8_quantize_kernel(const float* __restrict__ w, int64_t n,
                                                          uint8_t* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t full = n / kGroup;
    const int64_t steps = full / kUnroll;
    // kUnroll consecutive groups per warp step, all loads issued before any arithmetic
    for (int64_t t = gw; t < steps; t += warps) {
        const int64_t g0 = t * kUnroll;
        float4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; u++) v[u] = __ldcs(reinterpret_cast<const float4*>(w + (g0 + u) * kGroup) + lane);
#pragma unroll
        for (int u = 0; u < kUnroll; u++) q8_group(v[u], out + (g0 + u) * kGroupOut, lane);
    }
    // the remaining full groups, one per warp
    for (int64_t g = steps * kUnroll + gw; g < full; g += warps)
        q8_group(__ldcs(reinterpret_cast<const float4*>(w + g * kGroup) + lane), out + g * kGroupOut, lane);
    // the tensor's last, partial group (one warp): lane by lane, blocks of up to 32 weights
    if (full * kGroup < n && gw == warps - 1) {
        for (int64_t b0 = full * kGroup; b0 < n; b0 += kQBlock) {
            const int len = n - b0 < kQBlock ? (int)(n - b0) : kQBlock;
            const float x = lane < len ? w[b0 + lane] : 0.0f;
            float m = fabsf(x);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float s = q8_scale(m);
            uint8_t* blk = out + (b0 / kQBlock) * (4 + kQBlock);
            if (lane < 4) blk[lane] = (uint8_t)(__float_as_uint(s) >> (8 * lane));
            if (lane < len) blk[4 + lane] = (uint8_t)q8_byte(x, s);
        }
    }
}

}  // namespace

size_t q8_quantized_bytes(int64_t n) {
    if (n <= 0) return 0;
    const int64_t full = n / kQBlock, rem = n % kQBlock;
    return (size_t)full * (4 + kQBlock) + (rem ? (size_t)(4 + rem) : 0);
}

void launch_quantize_q8(const float* w, int64_t n, uint8_t* out, cudaStream_t s) {
    if (n <= 0) return;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    static int per_sm = 0;  // resident CTAs per SM (same on every B200)
    if (per_sm == 0 && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, q8_quantize_kernel, 256, 0) != cudaSuccess)
        per_sm = 4;
    const int64_t steps = (n + kGroup * kUnroll - 1) / (kGroup * kUnroll);
    // one wave of resident CTAs (8 warps each, 2 KB of loads in flight per warp) striding
    // over the tensor; smaller tensors get one warp step each
    const int64_t ctas = std::max<int64_t>(1, std::min<int64_t>((steps + 7) / 8, (int64_t)sms * std::max(per_sm, 1)));
    count_launch();
    q8_quantize_kernel<<<(unsigned)ctas, 256, 0, s>>>(w, n, out);
}

namespace {

// Two pinned host slots and two device slots of `piece` weights, one stream each.
struct QuantPipe {
    static constexpr int64_t kPiece = (int64_t)16 << 20;  // weights per slot (64 MB in)
    float* h_in[2] = {nullptr, nullptr};
    uint8_t* h_out[2] = {nullptr, nullptr};
    float* d_in[2] = {nullptr, nullptr};
    uint8_t* d_out[2] = {nullptr, nullptr};
    cudaStream_t st[2] = {nullptr, nullptr};
    cudaError_t err = cudaSuccess;

    int64_t piece = kPiece;
    std::mutex mu;  // one user at a time
    // slots for pieces of kPiece weights
    cudaError_t init() {
        piece = kPiece;
        const size_t in_b = (size_t)piece * 4, out_b = q8_quantized_bytes(piece);
        for (int i = 0; i < 2; i++) {
            if ((err = cudaMallocHost(&h_in[i], in_b)) != cudaSuccess) return err;
            if ((err = cudaMallocHost(&h_out[i], out_b)) != cudaSuccess) return err;
            if ((err = cudaMalloc(&d_in[i], in_b)) != cudaSuccess) return err;
            if ((err = cudaMalloc(&d_out[i], out_b)) != cudaSuccess) return err;
            if ((err = cudaStreamCreateWithFlags(&st[i], cudaStreamNonBlocking)) != cudaSuccess) return err;
        }
        return cudaSuccess;
    }
    ~QuantPipe() {
        for (int i = 0; i < 2; i++) {
            if (st[i]) cudaStreamSynchronize(st[i]);
            cudaFreeHost(h_in[i]);
            cudaFreeHost(h_out[i]);
            cudaFree(d_in[i]);
            cudaFree(d_out[i]);
            if (st[i]) cudaStreamDestroy(st[i]);
        }
    }
    // Enqueue slot i: h_in[i] (n weights, already filled) -> h_out[i].  Pieces are whole
    // blocks except a tensor's last one, so a piece's output is q8_quantized_bytes(n).
    cudaError_t enqueue(int i, int64_t n) {
        if ((err = cudaMemcpyAsync(d_in[i], h_in[i], (size_t)n * 4, cudaMemcpyHostToDevice, st[i])) != cudaSuccess)
            return err;
        launch_quantize_q8(d_in[i], n, d_out[i], st[i]);
        if ((err = cudaGetLastError()) != cudaSuccess) return err;
        return err = cudaMemcpyAsync(h_out[i], d_out[i], q8_quantized_bytes(n), cudaMemcpyDeviceToHost, st[i]);
    }
};

// Quantize n weights read by `fill(dst, offset, count)` (false: the input ended early)
// and hand each piece's bytes to `drain(src, bytes)` (false: write error), in order.
template <class Fill, class Drain>
int quantize_stream(QuantPipe& p, int64_t n, Fill fill, Drain drain) {
    const int64_t P = p.piece;  // a multiple of 128: pieces are whole blocks but the last
    const int64_t pieces = (n + P - 1) / P;
    int64_t pending_n = -1;  // weights of the piece in flight in the other slot
    for (int64_t k = 0; k <= pieces; k++) {
        const int slot = (int)(k & 1);
        if (k < pieces) {
            const int64_t off = k * P, cnt = std::min<int64_t>(P, n - off);
            if (!fill(p.h_in[slot], off, cnt)) return NR_ERR_FORMAT;  // input shorter than declared
            if (p.enqueue(slot, cnt) != cudaSuccess) return NR_ERR_CUDA;
            if (k == 0) {
                pending_n = cnt;
                continue;
            }
        }
        // drain the previous piece while this one runs
        const int prev = slot ^ 1;
        if (cudaStreamSynchronize(p.st[prev]) != cudaSuccess) return NR_ERR_CUDA;
        if (!drain(p.h_out[prev], q8_quantized_bytes(pending_n))) return NR_ERR_IO;
        if (k < pieces) pending_n = std::min<int64_t>(P, n - k * P);
    }
    return NR_OK;
}

// The current device's pipeline, made on its first use and kept for the process (two
// pinned and two device slots, ~164 MB each side), so repeated calls pay no allocation.
QuantPipe* device_pipe() {
    static std::mutex mu;
    static QuantPipe* pipes[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!pipes[dev]) {
        QuantPipe* p = new QuantPipe();
        if (p->init() != cudaSuccess) {
            delete p;
            cudaGetLastError();
            return nullptr;
        }
        pipes[dev] = p;
    }
    return pipes[dev];
}

}  // namespace

int quantize_q8_host(const float* w, int64_t n, uint8_t* out) {
    if (n <= 0) return NR_OK;
    QuantPipe* pp = device_pipe();
    if (!pp) return NR_ERR_CUDA;
    std::lock_guard<std::mutex> lock(pp->mu);
    QuantPipe& p = *pp;
    uint8_t* dst = out;
    return quantize_stream(
        p, n,
        [&](float* buf, int64_t off, int64_t cnt) {
            memcpy(buf, w + off, (size_t)cnt * 4);
            return true;
        },
        [&](const uint8_t* src, size_t bytes) {
            memcpy(dst, src, bytes);
            dst += bytes;
            return true;
        });
}

int quantize_model_file(const char* in_path, const char* out_path) {
    FILE* fi = fopen(in_path, "rb");
    if (!fi) return NR_ERR_IO;
    FILE* fo = fopen(out_path, "wb");
    if (!fo) {
        fclose(fi);
        return NR_ERR_IO;
    }
    int rc = NR_OK;
    int32_t h[7] = {0, 0, 0, 0, 0, 0, 0};
    if (fread(h, 4, 7, fi) != 7) rc = NR_ERR_FORMAT;
    // dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len (quantize.py:31-35)
    for (int i = 0; rc == NR_OK && i < 7; i++)
        if (h[i] <= 0) rc = NR_ERR_FORMAT;
    if (rc == NR_OK && h[0] % h[3] != 0) rc = NR_ERR_FORMAT;
    const int64_t dim = h[0], hidden = h[1], L = h[2], heads = h[3], kv_heads = h[4], vocab = h[5], seq = h[6];
    const int64_t head_size = rc == NR_OK ? dim / heads : 0, kv_dim = kv_heads * head_size;
    QuantPipe* pp = rc == NR_OK ? device_pipe() : nullptr;
    if (rc == NR_OK && !pp) rc = NR_ERR_CUDA;
    if (rc == NR_OK && fwrite(h, 4, 7, fo) != 7) rc = NR_ERR_IO;
    if (rc == NR_OK) {
        std::lock_guard<std::mutex> lock(pp->mu);
        QuantPipe& p = *pp;
        std::vector<char> buf((size_t)1 << 24);
        auto copy_fp32 = [&](int64_t count) {  // quantize.py:39-40
            int64_t left = count * 4;
            while (left > 0) {
                const size_t c = (size_t)std::min<int64_t>(left, (int64_t)buf.size());
                if (fread(buf.data(), 1, c, fi) != c) return NR_ERR_FORMAT;
                if (fwrite(buf.data(), 1, c, fo) != c) return NR_ERR_IO;
                left -= (int64_t)c;
            }
            return NR_OK;
        };
        auto convert_to_q8 = [&](int64_t count) {  // quantize.py:42-44
            return quantize_stream(
                p, count,
                [&](float* dst, int64_t, int64_t cnt) { return fread(dst, 4, (size_t)cnt, fi) == (size_t)cnt; },
                [&](const uint8_t* src, size_t bytes) { return fwrite(src, 1, bytes, fo) == bytes; });
        };
        // quantize.py:47-60, in file order
        const int64_t steps[][2] = {
            {0, vocab * dim},         {0, L * dim},          {1, L * dim * dim},    {1, L * dim * kv_dim},
            {1, L * dim * kv_dim},    {1, L * dim * dim},    {0, L * dim},          {1, L * dim * hidden},
            {1, L * hidden * dim},    {1, L * dim * hidden}, {0, dim},              {0, seq * head_size / 2},
            {0, seq * head_size / 2},
        };
        for (const auto& st : steps) {
            rc = st[0] ? convert_to_q8(st[1]) : copy_fp32(st[1]);
            if (rc) break;
        }
    }
    fclose(fi);
    if (fclose(fo) != 0 && rc == NR_OK) rc = NR_ERR_IO;
    return rc;
}

}  // namespace nitro
