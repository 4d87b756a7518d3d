"""The prefill layer's row-wise norm and activation dispatches (g4b_rows_rmsnorm,
g4b_rows_normadd, g4b_gelumul: vk/pre_norm.comp, vk/pre_na.comp, vk/gelumul.comp)
against the CPU oracle's rmsnorm / normadd / gelumul applied row by row.  The sums
of squares are formed in another order, so the bar is tests/util.py's (max relative
error 1e-2 with a 1e-3 x rms floor, cosine >= 0.9999); f16 inputs are given to the
oracle as the f16 values the device reads, and f16 outputs are compared after the
oracle's result is rounded to f16 the same way."""
import numpy as np
import pytest
import torch

import oracle as O
from g4b import _lib as L
from g4b import ops
from util import assert_close

pytestmark = pytest.mark.gpu


def _f16(a):
    return a.astype(np.float16).astype(np.float32)


@pytest.mark.parametrize("M,D,xdt,ydt", [(1, 3840, torch.float32, torch.float32), (37, 3840, torch.float32,
                                                                                   torch.float16),
                                         (64, 4096, torch.float16, torch.float32), (5, 256, torch.float16,
                                                                                    torch.float16)])
def test_rows_rmsnorm_matches_oracle(M, D, xdt, ydt):
    rng = np.random.default_rng(M + D)
    x = (rng.standard_normal((M, D)) * rng.uniform(0.1, 10, (M, 1))).astype(np.float32)
    if xdt == torch.float16:
        x = _f16(x)
    w = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    y = ops.rows_rmsnorm(torch.from_numpy(x).cuda().to(xdt), torch.from_numpy(w).cuda(), out_dtype=ydt)
    torch.cuda.synchronize()
    ref = np.stack([O.rmsnorm(x[m], w) for m in range(M)])
    if ydt == torch.float16:
        ref = _f16(ref)
    assert_close(y.float().cpu().numpy(), ref, f"rows_rmsnorm M={M} D={D}")
    assert L.query(L.Q_KERNEL_STATUS) == 0


@pytest.mark.parametrize("M,D,xdt,scl", [(1, 3840, torch.float32, 1.0), (33, 3840, torch.float16, 0.75),
                                         (8, 512, torch.float32, 1.25)])
def test_rows_normadd_matches_oracle(M, D, xdt, scl):
    rng = np.random.default_rng(7 * M + D)
    x = rng.standard_normal((M, D)).astype(np.float32)
    if xdt == torch.float16:
        x = _f16(x)
    w = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    h = rng.standard_normal((M, D)).astype(np.float32)
    hd = torch.from_numpy(h).cuda()
    ops.rows_normadd(torch.from_numpy(x).cuda().to(xdt), torch.from_numpy(w).cuda(), hd, scl)
    torch.cuda.synchronize()
    ref = np.stack([O.normadd(x[m], w, h[m], scl) for m in range(M)])
    assert_close(hd.cpu().numpy(), ref, f"rows_normadd M={M} D={D} scl={scl}")


@pytest.mark.parametrize("n,dt,odt", [(15360, torch.float32, torch.float32), (2048 * 15360, torch.float16,
                                                                              torch.float16), (4, torch.float16,
                                                                                               torch.float32)])
def test_gelumul_matches_oracle(n, dt, odt):
    rng = np.random.default_rng(n % 1000)
    g = (rng.standard_normal(n) * 3).astype(np.float32)
    u = rng.standard_normal(n).astype(np.float32)
    if dt == torch.float16:
        g, u = _f16(g), _f16(u)
    out = ops.gelumul(torch.from_numpy(g).cuda().to(dt), torch.from_numpy(u).cuda().to(dt), out_dtype=odt)
    torch.cuda.synchronize()
    ref = O.gelumul(g, u)
    if odt == torch.float16:
        ref = _f16(ref)
    assert_close(out.float().cpu().numpy(), ref, f"gelumul n={n}")


def test_rows_reject_bad_shapes():
    lib = L.load()
    z = torch.zeros(64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.g4b_rows_rmsnorm(z.data_ptr(), L.DT_F32, z.data_ptr(), z.data_ptr(), L.DT_F32, 2, 30, s) == L.G4B_E_SHAPE
    assert lib.g4b_rows_normadd(z.data_ptr(), 9, z.data_ptr(), z.data_ptr(), 2, 32, 1.0, s) == L.G4B_E_ARG
    assert lib.g4b_gelumul(z.data_ptr(), z.data_ptr(), L.DT_F32, z.data_ptr() + 4, L.DT_F32, 32, s) == L.G4B_E_ALIGN
