"""The allocation-free GEMV entry point (g4b_gemv_i4_noalloc) through the C ABI.

Some callers cannot allocate device memory when they run the GEMV -- for
example a host that records its decode step into a CUDA graph, or one whose
allocator refuses allocations after start-up -- so they cannot provide the
split-K workspace g4b_gemv_i4 asks for.  g4b_gemv_i4_noalloc uses a fixed
scratch array inside the library instead.  This file checks, on two calls in a
row (the second one reusing whatever the first left in the shared scratch),
that it returns bit for bit what g4b_gemv_i4 returns and agrees with the CPU
oracle of vk/gemv.comp + vk/reduce.comp; that requests larger than the
built-in scratch are refused; and that a rejected call queues nothing on the
stream.  It is collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
from g4b import _lib as L
from g4b import ops, pack
from util import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ptr(t):
    return int(t.data_ptr())


def _case(N, K, M, fp8, xdt, seed):
    W = (np.random.default_rng(seed).standard_normal((N, K)) * 0.02).astype(np.float32)
    pw = pack.quant(W, fp8=fp8, prefill_i8=False)
    X = torch.from_numpy(np.random.default_rng(seed + 1).standard_normal((M, K)).astype(np.float32)).to(DEV).to(xdt)
    return pw, ops.to_device(pw, DEV), X


def _noalloc(lib, X, dw, out, stream):
    return lib.g4b_gemv_i4_noalloc(_ptr(X), 0 if X.dtype == torch.float32 else 1, X.shape[0], _ptr(dw.wp),
                                   _ptr(dw.scales), dw.scale_fmt, dw.inv, _ptr(out), 0, dw.N, dw.K, 0, stream)


def _oracle(pw, X):
    xs = X.float().cpu().numpy()
    sc = pw.scales.view(np.uint16) if pw.scale_fmt == L.SCALE_F16 else pw.scales
    return np.stack([O.gemv(xs[m], pw.wp, sc, pw.scale_fmt, pw.inv, pw.N, pw.K, pw.split) for m in range(xs.shape[0])])


@pytest.mark.parametrize("N,K,M,fp8,xdt", [
    (15360, 3840, 1, False, torch.float16),   # configs[0]: the decode GEMV (split-K scratch in use)
    (262144, 3840, 1, True, torch.float16),   # lm_head with e4m3 scales
    (3840, 15360, 1, False, torch.float32),   # down_proj shape, f32 activations
    (4096, 3840, 4, False, torch.float16),    # small batch (streaming kernel)
])
def test_noalloc_matches_workspace_entry_point_twice(N, K, M, fp8, xdt):
    lib = L.load()
    pw, dw, X = _case(N, K, M, fp8, xdt, seed=N + K + M)
    assert ops.gemv_workspace_bytes(M, N, K, 0) <= 4 << 20
    ref = ops.gemv_i4(X, dw, out_dtype=torch.float32).reshape(M, N)
    torch.cuda.synchronize()
    want = _oracle(pw, X)
    stream = int(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        out = torch.full((M, N), float("nan"), device=DEV)
        st = _noalloc(lib, X, dw, out, stream)
        assert st == L.G4B_OK, L.last_error()
        torch.cuda.synchronize()
        # the same kernel and plan as g4b_gemv_i4, only the scratch differs: the same bits
        assert torch.equal(out, ref), f"noalloc call {call + 1} differs from g4b_gemv_i4 (N={N} K={K} M={M})"
        assert_close(out.cpu().numpy(), want, f"noalloc call {call + 1} vs oracle, N={N} K={K} M={M}")
    assert L.query(L.Q_KERNEL_STATUS) == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = L.load()
    N, K, M = 15360, 3840, 8
    assert ops.gemv_workspace_bytes(M, N, K, 0) > 4 << 20
    _, dw, X = _case(N, K, M, False, torch.float16, seed=5)
    out = torch.zeros((M, N), device=DEV)
    st = _noalloc(lib, X, dw, out, int(torch.cuda.current_stream().cuda_stream))
    assert st == L.G4B_E_WORKSPACE
    assert "scratch" in L.last_error()


def test_noalloc_rejected_call_queues_nothing():
    """A call rejected for a NULL x or a misaligned weight pointer returns its
    error and leaves the stream untouched: recorded under stream capture, the
    captured graph has no node (no counter memset), and no kernel was counted."""
    lib = L.load()
    rt = C.CDLL("libcudart.so.12")
    N, K = 15360, 3840
    _, dw, X = _case(N, K, 1, False, torch.float16, seed=9)
    out = torch.zeros((1, N), device=DEV)
    s = torch.cuda.Stream()
    sh = C.c_void_p(int(s.cuda_stream))
    torch.cuda.synchronize()
    launches = L.query(L.Q_LAUNCHES)
    for bad in ("null_x", "misaligned_wp"):
        graph = C.c_void_p()
        assert rt.cudaStreamBeginCapture(sh, 2) == 0          # cudaStreamCaptureModeRelaxed
        if bad == "null_x":
            st = lib.g4b_gemv_i4_noalloc(None, 1, 1, _ptr(dw.wp), _ptr(dw.scales), dw.scale_fmt, dw.inv,
                                         _ptr(out), 0, N, K, 0, sh)
        else:
            st = lib.g4b_gemv_i4_noalloc(_ptr(X), 1, 1, _ptr(dw.wp) + 4, _ptr(dw.scales), dw.scale_fmt, dw.inv,
                                         _ptr(out), 0, N, K, 0, sh)
        assert rt.cudaStreamEndCapture(sh, C.byref(graph)) == 0
        nodes = C.c_size_t(0)
        assert rt.cudaGraphGetNodes(graph, None, C.byref(nodes)) == 0
        rt.cudaGraphDestroy(graph)
        assert st == (L.G4B_E_ARG if bad == "null_x" else L.G4B_E_ALIGN), (bad, st, L.last_error())
        assert nodes.value == 0, f"{bad}: the rejected call queued {nodes.value} operation(s)"
    assert L.query(L.Q_LAUNCHES) == launches
    # and the entry point still works afterwards
    ref = ops.gemv_i4(X, dw, out_dtype=torch.float32).reshape(1, N)
    st = _noalloc(lib, X, dw, out, int(torch.cuda.current_stream().cuda_stream))
    assert st == L.G4B_OK, L.last_error()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
