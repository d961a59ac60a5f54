"""Kernel-level parity on the GPU: Q8_0 matmul and paged decode attention, called through
the C ABI (nr_q8_matmul, nr_paged_attention_decode) and compared with the CPU
restatement of the reference (oracle/nitro_oracle.cpp)."""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_close
from nitrorag_b200 import synth
from nitrorag_b200._lib import NR_Q8_FAITHFUL, NR_Q8_FIXED, lib

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for gpu tests")
    return torch


def _aos_to_soa(w_aos: bytes, rows: int, K: int):
    blk = np.frombuffer(w_aos, np.uint8).reshape(rows, K // 32, 36)
    scales = blk[:, :, :4].copy().view(np.float32).reshape(rows, K // 32)
    q = blk[:, :, 4:].copy().view(np.int8).reshape(rows, K)
    return q, scales


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 9, 17, 64, 65, 130, 300])
@pytest.mark.parametrize("mode", [NR_Q8_FIXED, NR_Q8_FAITHFUL])
@pytest.mark.parametrize("NK", [(768, 768), (256, 2048), (2304, 768), (4096, 768), (32000 // 250 * 2, 128),
                                (128, 4608), (64, 11008), (4096, 4096), (8192, 2048)])
def test_q8_matmul(torch_cuda, restatement, M, mode, NK):
    """CUDA-core matvec (M <= 8) and tcgen05 GEMM (M > 8); the narrow shapes split K over a
    thread-block cluster (1 to 8 CTAs) and reduce through distributed shared memory."""
    torch = torch_cuda
    N, K = NK
    rng = np.random.default_rng(M * 7 + N)
    w = (rng.standard_normal(N * K) * 0.02).astype(np.float32)
    w_aos = synth.quantize_q8(w)
    x = rng.standard_normal((M, K)).astype(np.float32)
    want = restatement.q8_matmul(x, w_aos, K, N, last_block_only=(mode == NR_Q8_FAITHFUL))
    q, s = _aos_to_soa(w_aos, N, K)
    dq, ds, dx = (torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(x).cuda())
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    for _ in range(2):
        rc = lib().nr_q8_matmul(dx.data_ptr(), dq.data_ptr(), ds.data_ptr(), out.data_ptr(), M, N, K, mode,
                                C.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        if M <= 8:  # fp32 CUDA-core path
            assert_close(got, want, rtol=1e-4, atol=1e-5, what=f"q8 M={M} mode={mode}")
        else:
            # bf16 hi/lo split on the tensor cores: ~2^-16 of each product's magnitude, so the
            # absolute bound scales with the output's RMS (cancelling outputs can be tiny)
            scale = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
            assert_close(got, want, rtol=1e-3, atol=1e-4 * scale, what=f"q8 M={M} mode={mode}")


_LARGE = {}


def _large_q8(N, K):
    """Seeded Q8_0 weights of one large shape, made once per session."""
    if (N, K) not in _LARGE:
        rng = np.random.default_rng(N + K)
        w_aos = synth.quantize_q8((rng.standard_normal(N * K) * 0.02).astype(np.float32))
        _LARGE.clear()
        _LARGE[(N, K)] = (w_aos, *_aos_to_soa(w_aos, N, K))
    return _LARGE[(N, K)]


@pytest.mark.parametrize("NK", [(12288, 4096), (4096, 11008), (22016, 4096), (12290, 4096), (4098, 2048)])
@pytest.mark.parametrize("M", [1, 2])
def test_q8_matvec_large(torch_cuda, restatement, M, NK):
    """One and two token rows over the 7B shape's projection matrices, a row count that is
    not a multiple of 4 and one that is only even: the ring matvec (units of 2-8 whole
    rows streamed through shared memory, activations in registers, row-pair partials
    joined in shared memory) against the restatement, to the fp32 bar of the matvec."""
    torch = torch_cuda
    N, K = NK
    w_aos, q, s = _large_q8(N, K)
    x = np.random.default_rng(M + N).standard_normal((M, K)).astype(np.float32)
    want = restatement.q8_matmul(x, w_aos, K, N)
    dq, ds, dx = (torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(x).cuda())
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    got = []
    for _ in range(2):
        rc = lib().nr_q8_matmul(dx.data_ptr(), dq.data_ptr(), ds.data_ptr(), out.data_ptr(), M, N, K, NR_Q8_FIXED,
                                C.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0
        torch.cuda.synchronize()
        got.append(out.cpu().numpy())
    assert np.array_equal(got[0], got[1])  # a fixed summation order
    assert_close(got[0], want, rtol=1e-4, atol=1e-5, what=f"q8 matvec M={M} {N}x{K}")


def _engine_pools(kref, vref, n_layers, n_kv, hd):
    """[page][layer][16][kv_dim] (reference) -> [page][layer][kv_head][16][hd] (engine)."""
    P = kref.shape[0]
    k = kref.reshape(P, n_layers, 16, n_kv, hd).transpose(0, 1, 3, 2, 4).copy()
    v = vref.reshape(P, n_layers, 16, n_kv, hd).transpose(0, 1, 3, 2, 4).copy()
    return k, v


def _run_decode_attention(torch, q, k_eng, v_eng, bt, ctx, n_heads, n_kv, hd, n_layers, layer, repeat=1):
    B = len(ctx)
    max_pages = bt.shape[1]
    dq = torch.from_numpy(q).cuda()
    dk = torch.from_numpy(k_eng).cuda()
    dv = torch.from_numpy(v_eng).cuda()
    dbt = torch.from_numpy(bt).cuda()
    dctx = torch.from_numpy(ctx).cuda()
    out = torch.zeros((B, n_heads * hd), dtype=torch.float32, device="cuda")
    ws_bytes = lib().nr_paged_attention_workspace_size(B, n_heads, hd, max_pages)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(repeat):
        rc = lib().nr_paged_attention_decode(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dbt.data_ptr(), max_pages,
                                             dctx.data_ptr(), B, n_heads, n_kv, hd, n_layers, layer, out.data_ptr(),
                                             ws.data_ptr(), err.data_ptr(), stream)
        assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out.cpu().numpy()


@pytest.mark.parametrize("hd,n_heads,n_kv", [(64, 12, 12), (128, 4, 4), (64, 8, 2)])
def test_paged_attention_small(torch_cuda, restatement, hd, n_heads, n_kv):
    """Ragged contexts incl. 1 token, exact page multiples, multi-chunk splits; 2 layers."""
    torch = torch_cuda
    rng = np.random.default_rng(hd + n_kv)
    ctx = np.array([1, 15, 16, 17, 128, 129, 300, 513], np.int32)
    B, n_layers, layer, P = len(ctx), 2, 1, 96
    kv_dim = n_kv * hd
    max_pages = 40
    perm = rng.permutation(P).astype(np.int32)
    bt = np.zeros((B, max_pages), np.int32)
    at = 0
    for b in range(B):
        n = (ctx[b] + 15) // 16
        bt[b, :n] = perm[at:at + n]
        at += n
    kref = rng.standard_normal((P, n_layers, 16, kv_dim)).astype(np.float32)
    vref = rng.standard_normal((P, n_layers, 16, kv_dim)).astype(np.float32)
    q = rng.standard_normal((B, n_heads * hd)).astype(np.float32)
    want = restatement.paged_decode_attention(q, kref, vref, n_layers * 16 * kv_dim, layer * 16 * kv_dim, bt, ctx,
                                              n_heads, n_kv, hd)
    k_eng, v_eng = _engine_pools(kref, vref, n_layers, n_kv, hd)
    got = _run_decode_attention(torch, q, k_eng, v_eng, bt, ctx, n_heads, n_kv, hd, n_layers, layer, repeat=2)
    assert_close(got, want, rtol=1e-4, atol=1e-5, what="paged attention")


def test_paged_attention_microbench_config(torch_cuda, restatement):
    """The benchmark's configuration at full size: 64 sequences, ctx U[128,1024], 12x64,
    8192-page single-layer pool, pages from a seeded permutation, N(0,1) values."""
    torch = torch_cuda
    ctx, bt, q = synth.paged_attention_case(seed=2)
    P, hd, H = 8192, 64, 12
    rng = np.random.default_rng(5)
    kref = rng.standard_normal((P, 1, 16, H * hd), dtype=np.float32)
    vref = rng.standard_normal((P, 1, 16, H * hd), dtype=np.float32)
    want = restatement.paged_decode_attention(q, kref, vref, 16 * H * hd, 0, bt, ctx, H, H, hd)
    k_eng, v_eng = _engine_pools(kref, vref, 1, H, hd)
    got = _run_decode_attention(torch, q, k_eng, v_eng, bt, ctx, H, H, hd, 1, 0, repeat=3)
    assert_close(got, want, rtol=1e-4, atol=1e-5, what="paged attention config 2")


@pytest.mark.parametrize("B,n_heads", [(8, 4), (64, 12)])
def test_paged_attention_context_out_of_range(torch_cuda, restatement, B, n_heads):
    """A context length beyond what the block-table row can address (max_pages * 16) and a
    zero length: the call sets the error flag to 2, the too-long row attends to its
    max_pages * 16 tokens, the empty row gets a zero output, every other row is unchanged.
    The block table has one spare row of valid page ids and the workspace is oversized, so
    every read and write of the call stays inside its buffers."""
    torch = torch_cuda
    hd, n_kv, n_layers, max_pages = 64, n_heads, 1, 8
    cap = max_pages * 16
    rng = np.random.default_rng(B + n_heads)
    ctx = rng.integers(1, cap + 1, B).astype(np.int32)
    ctx[1], ctx[2] = cap + 20, 0
    P = (B + 1) * max_pages
    bt = rng.permutation(P).astype(np.int32).reshape(B + 1, max_pages)
    kv_dim = n_kv * hd
    kref = rng.standard_normal((P, n_layers, 16, kv_dim)).astype(np.float32)
    vref = rng.standard_normal((P, n_layers, 16, kv_dim)).astype(np.float32)
    q = rng.standard_normal((B, n_heads * hd)).astype(np.float32)
    clamped = np.clip(ctx, 0, cap).astype(np.int32)
    clamped[2] = 1  # the oracle needs a non-empty row; its output is replaced below
    want = restatement.paged_decode_attention(q, kref, vref, n_layers * 16 * kv_dim, 0, bt[:B], clamped, n_heads,
                                              n_kv, hd)
    want[2] = 0.0
    k_eng, v_eng = _engine_pools(kref, vref, n_layers, n_kv, hd)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k_eng, v_eng))
    dbt, dctx = torch.from_numpy(bt).cuda(), torch.from_numpy(ctx).cuda()
    out = torch.full((B, n_heads * hd), float("nan"), dtype=torch.float32, device="cuda")
    ws_bytes = 2 * lib().nr_paged_attention_workspace_size(B, n_heads, hd, 2 * max_pages)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib().nr_paged_attention_decode(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dbt.data_ptr(), max_pages,
                                         dctx.data_ptr(), B, n_heads, n_kv, hd, n_layers, 0, out.data_ptr(),
                                         ws.data_ptr(), err.data_ptr(),
                                         C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 2
    assert_close(out.cpu().numpy(), want, rtol=1e-4, atol=1e-5, what="paged attention, clamped contexts")
