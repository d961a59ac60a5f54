"""nr_paged_attention_decode_static: decode attention whose scratch is a fixed array in the
library's device image (no workspace argument, no device allocation by the call).  Checked
against nr_paged_attention_decode, which takes a caller-allocated workspace, on the same
inputs; the file sorts last so that it also runs after every other GPU test."""
import ctypes as C

import numpy as np
import pytest

from conftest import assert_close
from nitrorag_b200 import synth
from nitrorag_b200._lib import lib

pytestmark = pytest.mark.gpu

NR_ERR_CAPACITY = -8
STATIC_SCRATCH_BYTES = 8 << 20


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for gpu tests")
    return torch


def _case(rng, ctx, n_layers, n_heads, n_kv, hd, max_pages, P):
    B = len(ctx)
    perm = rng.permutation(P).astype(np.int32)
    bt = np.zeros((B, max_pages), np.int32)
    at = 0
    for b in range(B):
        n = (int(ctx[b]) + 15) // 16
        bt[b, :n] = perm[at:at + n]
        at += n
    k = rng.standard_normal((P, n_layers, n_kv, 16, hd), dtype=np.float32)
    v = rng.standard_normal((P, n_layers, n_kv, 16, hd), dtype=np.float32)
    q = rng.standard_normal((B, n_heads * hd), dtype=np.float32)
    return q, k, v, bt


def _with_workspace(torch, d, B, n_heads, n_kv, hd, n_layers, layer, max_pages):
    ws_bytes = lib().nr_paged_attention_workspace_size(B, n_heads, hd, max_pages)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.zeros((B, n_heads * hd), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib().nr_paged_attention_decode(d["q"].data_ptr(), d["k"].data_ptr(), d["v"].data_ptr(), d["bt"].data_ptr(),
                                         max_pages, d["ctx"].data_ptr(), B, n_heads, n_kv, hd, n_layers, layer,
                                         out.data_ptr(), ws.data_ptr(), err.data_ptr(),
                                         C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out.cpu().numpy()


def _static(torch, d, out, err, B, n_heads, n_kv, hd, n_layers, layer, max_pages):
    return lib().nr_paged_attention_decode_static(d["q"].data_ptr(), d["k"].data_ptr(), d["v"].data_ptr(),
                                                  d["bt"].data_ptr(), max_pages, d["ctx"].data_ptr(), B, n_heads,
                                                  n_kv, hd, n_layers, layer, out.data_ptr(), err.data_ptr(),
                                                  C.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("hd,n_heads,n_kv,ctx_kind", [(64, 12, 12, "config2"), (64, 8, 2, "ragged"),
                                                      (128, 4, 4, "ragged"), (128, 8, 2, "wide"),
                                                      (64, 16, 4, "wide")])
def test_static_scratch_matches_workspace_entry(torch_cuda, hd, n_heads, n_kv, ctx_kind):
    """Two calls in a row on different layers and queries (the second reuses the scratch the
    first left behind), each equal to the workspace entry point; a third call shows the
    calls take no device memory."""
    torch = torch_cuda
    rng = np.random.default_rng(hd * 31 + n_kv)
    if ctx_kind == "config2":
        ctx, _, _ = synth.paged_attention_case(seed=3)
        ctx = ctx.astype(np.int32)
        max_pages, P, n_layers = 64, 4608, 2
    elif ctx_kind == "wide":
        # more (sequence, head) pairs than SMs: the split kernel and the merge kernel, whose
        # partials live in the static array (head_dim 128 doubles their rows)
        B = 24 if hd == 128 else 48
        ctx = rng.integers(1, 1025, B).astype(np.int32)
        ctx[:3] = [1, 16, 1024]
        max_pages, n_layers = 64, 2
        P = int(sum((c + 15) // 16 for c in ctx)) + 8
    else:
        ctx = np.array([1, 15, 16, 17, 128, 129, 300, 513], np.int32)
        max_pages, P, n_layers = 40, 96, 3
    B = len(ctx)
    assert lib().nr_paged_attention_workspace_size(B, n_heads, hd, max_pages) <= STATIC_SCRATCH_BYTES
    q, k, v, bt = _case(rng, ctx, n_layers, n_heads, n_kv, hd, max_pages, P)
    q2 = rng.standard_normal(q.shape, dtype=np.float32)
    d = {"q": torch.from_numpy(q).cuda(), "k": torch.from_numpy(k).cuda(), "v": torch.from_numpy(v).cuda(),
         "bt": torch.from_numpy(bt).cuda(), "ctx": torch.from_numpy(ctx).cuda()}
    d2 = dict(d, q=torch.from_numpy(q2).cuda())
    want1 = _with_workspace(torch, d, B, n_heads, n_kv, hd, n_layers, 0, max_pages)
    want2 = _with_workspace(torch, d2, B, n_heads, n_kv, hd, n_layers, n_layers - 1, max_pages)

    out1 = torch.full((B, n_heads * hd), float("nan"), dtype=torch.float32, device="cuda")
    out2 = torch.full((B, n_heads * hd), float("nan"), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _static(torch, d, out1, err, B, n_heads, n_kv, hd, n_layers, 0, max_pages) == 0
    assert _static(torch, d2, out2, err, B, n_heads, n_kv, hd, n_layers, n_layers - 1, max_pages) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert_close(out1.cpu().numpy(), want1, rtol=1e-4, atol=1e-5, what="static scratch, call 1")
    assert_close(out2.cpu().numpy(), want2, rtol=1e-4, atol=1e-5, what="static scratch, call 2")

    free_before = torch.cuda.mem_get_info()[0]
    assert _static(torch, d, out1, err, B, n_heads, n_kv, hd, n_layers, 0, max_pages) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    assert int(err.item()) == 0
    assert_close(out1.cpu().numpy(), want1, rtol=1e-4, atol=1e-5, what="static scratch, call 3")


def test_static_scratch_rejects_oversize(torch_cuda):
    """A batch whose scratch exceeds the fixed array is refused before anything is launched."""
    torch = torch_cuda
    B, H, hd, max_pages = 1024, 32, 128, 256
    assert lib().nr_paged_attention_workspace_size(B, H, hd, max_pages) > STATIC_SCRATCH_BYTES
    dummy = torch.zeros(16, dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    p = dummy.data_ptr()
    rc = lib().nr_paged_attention_decode_static(p, p, p, p, max_pages, p, B, H, H, hd, 1, 0, p, err.data_ptr(),
                                                C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == NR_ERR_CAPACITY
