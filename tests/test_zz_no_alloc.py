"""The allocation-free GEMV entry point (g4b_gemv_i4_noalloc) through the C ABI.

Some callers cannot allocate device memory when they run the GEMV -- for
example a host that records its decode step into a CUDA graph, or one whose
allocator refuses allocations after start-up -- so they cannot provide the
split-K workspace g4b_gemv_i4 asks for.  g4b_gemv_i4_noalloc uses a fixed
scratch array inside the library instead.  This file checks, on two calls in a
row (the second one reusing whatever the first left in the shared scratch),
that it returns what g4b_gemv_i4 returns, and that requests larger than the
built-in scratch are refused.  It is collected last on purpose.
"""
import numpy as np
import pytest
import torch

from g4b import _lib as L
from g4b import ops, pack
from util import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ptr(t):
    return int(t.data_ptr())


def _case(N, K, M, fp8, xdt, seed):
    W = (np.random.default_rng(seed).standard_normal((N, K)) * 0.02).astype(np.float32)
    dw = ops.to_device(pack.quant(W, fp8=fp8, prefill_i8=False), DEV)
    X = torch.from_numpy(np.random.default_rng(seed + 1).standard_normal((M, K)).astype(np.float32)).to(DEV).to(xdt)
    return dw, X


def _noalloc(lib, X, dw, out, stream):
    return lib.g4b_gemv_i4_noalloc(_ptr(X), 0 if X.dtype == torch.float32 else 1, X.shape[0], _ptr(dw.wp),
                                   _ptr(dw.scales), dw.scale_fmt, dw.inv, _ptr(out), 0, dw.N, dw.K, 0, stream)


@pytest.mark.parametrize("N,K,M,fp8,xdt", [
    (15360, 3840, 1, False, torch.float16),   # configs[0]: the decode GEMV (split-K scratch in use)
    (262144, 3840, 1, True, torch.float16),   # lm_head with e4m3 scales
    (3840, 15360, 1, False, torch.float32),   # down_proj shape, f32 activations
    (4096, 3840, 4, False, torch.float16),    # small batch (streaming kernel)
])
def test_noalloc_matches_workspace_entry_point_twice(N, K, M, fp8, xdt):
    lib = L.load()
    dw, X = _case(N, K, M, fp8, xdt, seed=N + K + M)
    assert ops.gemv_workspace_bytes(M, N, K, 0) <= 4 << 20
    ref = ops.gemv_i4(X, dw, out_dtype=torch.float32)
    torch.cuda.synchronize()
    stream = int(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        out = torch.full((M, N), float("nan"), device=DEV)
        st = _noalloc(lib, X, dw, out, stream)
        assert st == L.G4B_OK, L.last_error()
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), ref.cpu().numpy().reshape(M, N), f"noalloc call {call + 1} N={N} K={K} M={M}")
    assert L.query(L.Q_KERNEL_STATUS) == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = L.load()
    N, K, M = 15360, 3840, 8
    assert ops.gemv_workspace_bytes(M, N, K, 0) > 4 << 20
    dw, X = _case(N, K, M, False, torch.float16, seed=5)
    out = torch.zeros((M, N), device=DEV)
    st = _noalloc(lib, X, dw, out, int(torch.cuda.current_stream().cuda_stream))
    assert st == L.G4B_E_WORKSPACE
    assert "scratch" in L.last_error()
