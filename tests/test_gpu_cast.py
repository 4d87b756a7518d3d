"""GPU parity of the activation casts through the C ABI, all bit-exact:
f32 <-> f16 (vk/cast_dn.comp, vk/cast_up.comp) against numpy's RNE cast, and
the per-token int8 quantiser (vk/cast_i8.comp) against the oracle."""
import numpy as np
import pytest
import torch

import oracle as O
from g4b import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("n", [1, 7, 8, 4096, 1_000_003])
def test_cast_f32_f16_roundtrip_bit_exact(n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 10.0 ** rng.integers(-6, 5, n)).astype(np.float32)
    x[: min(n, 4)] = np.array([0.0, -0.0, 65519.0, 1e-8], np.float32)[: min(n, 4)]
    xt = torch.from_numpy(x).to(DEV)
    h = ops.cast(xt, torch.float16)
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16)
    assert np.array_equal(h.cpu().numpy().view(np.uint16), ref.view(np.uint16))
    back = ops.cast(h, torch.float32)
    assert np.array_equal(back.cpu().numpy(), ref.astype(np.float32))


def _edge_rows(K):
    rng = np.random.default_rng(2)
    X = rng.standard_normal((6, K)).astype(np.float32)
    X[0] = 0.0                                  # all-zero row: s = 1e-12, q = 0
    X[1, :] = 0.0
    X[1, 0] = 127.0                             # s = 1, exact halves below round half-even
    X[1, 1:9] = [0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5, -126.5]
    X[2] *= 1e-30                               # tiny magnitudes
    X[3] *= 1e30                                # huge magnitudes
    X[4, 5] = -1e4                              # one outlier
    return X


@pytest.mark.parametrize("M,K", [(6, 64), (64, 3840), (33, 15360), (4096, 15360)])
@pytest.mark.parametrize("xdt", [torch.float32, torch.float16])
def test_cast_i8_bit_exact(M, K, xdt):
    X = np.random.default_rng(M + K).standard_normal((M, K)).astype(np.float32)
    if M == 6:
        X = _edge_rows(K)
    if xdt == torch.float16:
        with np.errstate(over="ignore"):
            X = np.clip(X, -60000, 60000).astype(np.float16).astype(np.float32)
    Xt = torch.from_numpy(X).to(DEV).to(xdt)
    A8, sa = ops.cast_i8(Xt)
    torch.cuda.synchronize()
    rA, rs = O.cast_i8(X)
    assert np.array_equal(sa.cpu().numpy().view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(A8.cpu().numpy(), rA)
