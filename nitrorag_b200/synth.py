"""Seeded synthetic models and workloads in the reference's formats.

* ``quantize_q8`` restates scripts/quantize.py:7-23 (nvivek17/NitroRAG) vectorised:
  per 32 weights ``scale = absmax/127`` in fp32 (``1e-9`` for an all-zero block), weights
  ``round-half-even(w/scale)`` clamped to [-128, 127], stored as 36-byte blocks.
* ``write_model`` writes the Q8_0 model file the reference loads
  (src/Server_Inference.cpp:41-69): a 7 x int32 header, then fp32 embedding, fp32 RMS
  gains, Q8_0 wq wk wv wo, fp32 RMS gains, Q8_0 w1 w2 w3, fp32 final gain and the fp32
  RoPE tables ``freq_cis_real/imag[pos][i] = cos/sin(pos * theta**(-2i/head_dim))``.
  Weights are N(0, std) fp32 from numpy's PCG64 stream of ``seed``; RMS gains are 1.
* Workload generators for the shapes the benchmarks use (uniform-random token ids).
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass

import numpy as np

Q_BLOCK = 32


@dataclass(frozen=True)
class ModelShape:
    dim: int
    hidden_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    vocab_size: int
    seq_len: int

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def header(self) -> bytes:
        return struct.pack("7i", self.dim, self.hidden_dim, self.n_layers, self.n_heads, self.n_kv_heads,
                           self.vocab_size, self.seq_len)

    def q8_weights(self) -> int:
        D, H, L, KV = self.dim, self.hidden_dim, self.n_layers, self.kv_dim
        return L * (2 * D * D + 2 * D * KV + 3 * D * H)

    def q8_bytes(self) -> int:
        return self.q8_weights() // Q_BLOCK * 36

    def kv_bytes_per_token(self) -> int:
        return 2 * self.n_layers * self.kv_dim * 4

    def decode_weight_bytes(self) -> int:
        """Bytes of weights one decode step must read: Q8 blocks, fp32 classifier, RMS gains."""
        return self.q8_bytes() + self.vocab_size * self.dim * 4 + (2 * self.n_layers + 1) * self.dim * 4


# 110M (configs 1-4) and the 7B shape (config 5).  seq_len 1024 for the
# 110M decoder; config 4 needs positions up to 1039, so it uses seq_len 2048.
SHAPE_110M = ModelShape(768, 2048, 12, 12, 12, 32000, 1024)
SHAPE_110M_LONG = ModelShape(768, 2048, 12, 12, 12, 32000, 2048)
SHAPE_7B = ModelShape(4096, 11008, 32, 32, 32, 32000, 4096)
SHAPE_TINY = ModelShape(128, 256, 2, 2, 2, 512, 512)


def quantize_q8(w: np.ndarray) -> bytes:
    """scripts/quantize.py:7-23 on a flat float32 array (length a multiple of 32)."""
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1, Q_BLOCK)
    amax = np.max(np.abs(w), axis=1)
    scale = np.where(amax != 0, amax / np.float32(127.0), np.float32(1e-9)).astype(np.float32)
    q = np.rint(w / scale[:, None])
    q = np.clip(q, -128, 127).astype(np.int8)
    out = np.empty((w.shape[0], 36), np.uint8)
    out[:, :4] = scale.view(np.uint8).reshape(-1, 4)
    out[:, 4:] = q.view(np.uint8)
    return out.tobytes()


def rope_tables(seq_len: int, head_dim: int, theta: float = 10000.0):
    i = np.arange(head_dim // 2, dtype=np.float64)
    freqs = theta ** (-2.0 * i / head_dim)
    ang = np.arange(seq_len, dtype=np.float64)[:, None] * freqs[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def _normal(rng: np.random.Generator, n: int, std: float) -> np.ndarray:
    return (rng.standard_normal(n, dtype=np.float32) * np.float32(std)).astype(np.float32)


def write_model(path: str, shape: ModelShape, seed: int = 1234, std: float = 0.02,
                fp32_path: str | None = None) -> str:
    """Write a seeded synthetic Q8_0 model.  With ``fp32_path`` also write the unquantised
    llama2.c-format fp32 file that scripts/quantize.py converts into the same Q8_0 file."""
    rng = np.random.Generator(np.random.PCG64(seed))
    D, H, L, KV = shape.dim, shape.hidden_dim, shape.n_layers, shape.kv_dim
    ones_ld = np.ones(L * D, np.float32).tobytes()
    fr, fi = rope_tables(shape.seq_len, shape.head_dim)
    f32 = open(fp32_path, "wb") if fp32_path else None
    with open(path, "wb") as f:
        def both(b: bytes):
            f.write(b)
            if f32:
                f32.write(b)

        def q8_tensor(rows: int, cols: int):
            # generated layer by layer so the 7B shape never holds a whole tensor
            for _ in range(L):
                w = _normal(rng, rows * cols, std)
                f.write(quantize_q8(w))
                if f32:
                    f32.write(w.tobytes())

        both(shape.header())
        both(_normal(rng, shape.vocab_size * D, std).tobytes())  # token embedding (= classifier)
        both(ones_ld)                                           # rms_att
        q8_tensor(D, D)    # wq
        q8_tensor(KV, D)   # wk
        q8_tensor(KV, D)   # wv
        q8_tensor(D, D)    # wo
        both(ones_ld)      # rms_ffn
        q8_tensor(H, D)    # w1
        q8_tensor(D, H)    # w2
        q8_tensor(H, D)    # w3
        both(np.ones(D, np.float32).tobytes())  # rms_final
        both(fr.tobytes())
        both(fi.tobytes())
    if f32:
        f32.close()
    return path


def write_model_on_device(path: str, shape: ModelShape, seed: int = 1234, std: float = 0.02) -> str:
    """The same file layout and Q8_0 quantisation as write_model, with the N(0, std) values
    drawn by torch's CUDA generator (seeded) instead of PCG64: seconds instead of tens of
    minutes for the 7B shape.  The values differ from write_model's, so this is for
    throughput runs, not for parity against files written by write_model."""
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    D, H, L, KV = shape.dim, shape.hidden_dim, shape.n_layers, shape.kv_dim

    def normal(n: int) -> "torch.Tensor":
        return torch.randn(n, device="cuda", generator=g, dtype=torch.float32) * std

    def q8(w: "torch.Tensor") -> bytes:
        w = w.reshape(-1, Q_BLOCK)
        amax = w.abs().amax(dim=1)
        scale = torch.where(amax != 0, amax / 127.0, torch.full_like(amax, 1e-9))
        q = torch.clamp(torch.round(w / scale[:, None]), -128, 127).to(torch.int8)
        blk = torch.empty((w.shape[0], 36), dtype=torch.uint8, device="cuda")
        blk[:, :4] = scale.contiguous().view(torch.uint8).reshape(-1, 4)
        blk[:, 4:] = q.view(torch.uint8)
        return blk.cpu().numpy().tobytes()

    ones_ld = np.ones(L * D, np.float32).tobytes()
    fr, fi = rope_tables(shape.seq_len, shape.head_dim)
    with open(path, "wb") as f:
        def q8_tensor(rows: int, cols: int):
            for _ in range(L):
                f.write(q8(normal(rows * cols)))

        f.write(shape.header())
        f.write(normal(shape.vocab_size * D).cpu().numpy().tobytes())
        f.write(ones_ld)
        q8_tensor(D, D)
        q8_tensor(KV, D)
        q8_tensor(KV, D)
        q8_tensor(D, D)
        f.write(ones_ld)
        q8_tensor(H, D)
        q8_tensor(D, H)
        q8_tensor(H, D)
        f.write(np.ones(D, np.float32).tobytes())
        f.write(fr.tobytes())
        f.write(fi.tobytes())
    return path


def model_cache_dir() -> str:
    """NITRO_MODEL_CACHE if set, else ``.model_cache`` at the top of the source tree
    (git-ignored; generated model files are never committed)."""
    return os.environ.get("NITRO_MODEL_CACHE") or os.path.join(
        os.path.dirname(os.path.dirname(os.path.abspath(__file__))), ".model_cache")


def cached_model_on_device(shape: ModelShape, seed: int = 1234, cache_dir: str | None = None) -> str:
    """cached_model for write_model_on_device files (separate names)."""
    cache_dir = cache_dir or model_cache_dir()
    os.makedirs(cache_dir, exist_ok=True)
    name = "q8dev_{}x{}x{}x{}x{}x{}x{}_s{}.bin".format(shape.dim, shape.hidden_dim, shape.n_layers, shape.n_heads,
                                                       shape.n_kv_heads, shape.vocab_size, shape.seq_len, seed)
    path = os.path.join(cache_dir, name)
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write_model_on_device(tmp, shape, seed)
        os.replace(tmp, path)
    return path


def cached_model(shape: ModelShape, seed: int = 1234, cache_dir: str | None = None) -> str:
    """Path of the synthetic model for (shape, seed), written on first use."""
    cache_dir = cache_dir or model_cache_dir()
    os.makedirs(cache_dir, exist_ok=True)
    name = "q8_{}x{}x{}x{}x{}x{}x{}_s{}.bin".format(shape.dim, shape.hidden_dim, shape.n_layers, shape.n_heads,
                                                    shape.n_kv_heads, shape.vocab_size, shape.seq_len, seed)
    path = os.path.join(cache_dir, name)
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write_model(tmp, shape, seed)
        os.replace(tmp, path)
    return path


def random_prompt(rng: np.random.Generator, n: int, vocab: int) -> np.ndarray:
    return rng.integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)


def decode_workload(n_reqs: int, lo: int, hi: int, vocab: int, seed: int = 7):
    """n_reqs uniform-random prompts with lengths uniform in [lo, hi]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    lens = rng.integers(lo, hi + 1, size=n_reqs)
    return [random_prompt(rng, int(n), vocab) for n in lens]


def paged_attention_case(seed: int = 2, B: int = 64, n_heads: int = 12, head_dim: int = 64,
                         pool_pages: int = 8192, ctx_lo: int = 128, ctx_hi: int = 1024):
    """The paged-attention microbenchmark: context lengths uniform in [ctx_lo, ctx_hi] (query
    position included), pages of each sequence consecutive slices of one seeded permutation
    of the pool (disjoint), q/K/V N(0,1).  Returns (ctx, block_tables[B][max_pages], q)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    ctx = rng.integers(ctx_lo, ctx_hi + 1, size=B).astype(np.int32)
    max_pages = (ctx_hi + 15) // 16
    perm = rng.permutation(pool_pages).astype(np.int32)
    bt = np.zeros((B, max_pages), np.int32)
    at = 0
    for b in range(B):
        n = (int(ctx[b]) + 15) // 16
        bt[b, :n] = perm[at:at + n]
        at += n
    q = rng.standard_normal((B, n_heads * head_dim), dtype=np.float32)
    return ctx, bt, q


def poisson_prefix_workload(n: int = 50, rate: float = 20.0, shared_len: int = 384, shared_frac: float = 0.6,
                            lo: int = 64, hi: int = 512, vocab: int = 32000, seed: int = 33):
    """Config 3: n requests arriving by a Poisson process of `rate` per second (arrival
    times, seconds); a fraction `shared_frac` of them (a seeded Bernoulli draw) are one
    shared `shared_len`-token prefix plus a random suffix, total length U[shared_len + 1,
    hi]; the others U[lo, hi] random tokens.  Returns (arrivals, prompts)."""
    rng = np.random.default_rng(seed)
    arrive = np.cumsum(rng.exponential(1 / rate, n))
    shared = rng.integers(0, vocab, shared_len).astype(np.int32)
    prompts = []
    for _ in range(n):
        if rng.random() < shared_frac:
            m = int(rng.integers(shared_len + 1, hi + 1))
            prompts.append(np.concatenate([shared, rng.integers(0, vocab, m - shared_len).astype(np.int32)]))
        else:
            prompts.append(rng.integers(0, vocab, int(rng.integers(lo, hi + 1))).astype(np.int32))
    return arrive, prompts


def virtual_clock_admissions(arrive, step_s: float = 0.010):
    """Admission schedule of a request stream under a virtual clock: step k admits every
    request with arrival time <= k * step_s.  Yields, per scheduler iteration k, the
    indices admitted before it; the caller stops when nothing is left to run."""
    nxt, k = 0, 0
    while True:
        batch = []
        while nxt < len(arrive) and arrive[nxt] <= k * step_s:
            batch.append(nxt)
            nxt += 1
        yield batch
        k += 1
