"""GPU parity of the int8 prefill GEMMs (g4b_gemm_w8a8, g4b_gemm_w4a8) through the C ABI.

Oracle: oracle/g4b_oracle.c orc_gemm_w8a8 (vk/coopgemm_w8a8.comp:18-37) and
orc_gemm_w4a8 / orc_w4a8_requant (vk/coopgemm_w4a8.comp:21-50).  Everything
here is integer or a fixed sequence of correctly rounded f32 products, so the
bar is bit-exact: the int32 accumulators (C_debug) and the f16 outputs
f16((float(C) * sa[m]) * f32(sw[n])) must equal the oracle's bits.

At config 4's full size (M=4096, N=3840, K=15360) the CPU oracle is too slow
for a test, so the int32 accumulators are checked against torch._int_mm
(cuBLAS int8 GEMM, exact integer arithmetic) on the same operands, and the
f16 outputs against the oracle's epilogue applied to those accumulators.
"""
import numpy as np
import pytest
import torch

import oracle as O
from g4b import _lib as L
from g4b import ops, pack
from util import weights, activations

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _prep(M, N, K, seed):
    pw = pack.quant(weights(N, K, seed), fp8=False, prefill_i8=True)
    dw = ops.to_device(pw, DEV, w4a8=True)
    X = activations(M, K, seed=seed + 1)
    A8, sa = O.cast_i8(X)
    return pw, dw, A8, sa


def _epilogue(Cm, sa, sw16):
    """The shaders' epilogue on int32 accumulators, in f32 with the shader's order."""
    v = (Cm.astype(np.float32) * sa[:, None].astype(np.float32)) * sw16.astype(np.float32)[None, :]
    return v.astype(np.float32)


SHAPES = [(256, 128, 128), (1, 128, 32), (17, 48, 96), (300, 384, 160), (512, 640, 1024), (129, 272, 544)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("ydt", [torch.float16, torch.float32])
def test_w8a8_matches_oracle(M, N, K, ydt):
    pw, dw, A8, sa = _prep(M, N, K, seed=M + N + K)
    Cref, Yref = O.gemm_w8a8(A8, pw.w8, sa, pw.sw8.view(np.uint16))
    acc = torch.empty((M, N), dtype=torch.int32, device=DEV)
    Y = ops.gemm_w8a8(torch.from_numpy(A8).to(DEV), torch.from_numpy(sa).to(DEV), dw, out_dtype=ydt, acc=acc)
    torch.cuda.synchronize()
    assert L.query(L.Q_KERNEL_STATUS) == 0
    assert np.array_equal(acc.cpu().numpy(), Cref), f"int32 accumulators differ M={M} N={N} K={K}"
    if ydt == torch.float16:
        assert np.array_equal(Y.cpu().numpy().view(np.uint16), Yref), "f16 outputs differ"
    else:
        assert np.array_equal(Y.cpu().numpy(), _epilogue(Cref, sa, pw.sw8)), "f32 outputs differ"


@pytest.mark.parametrize("M,N,K", [(300, 384, 160), (2048, 1280, 256)])
def test_w8a8_quarter_units_give_the_whole_tiles_bits(M, N, K, monkeypatch):
    """When the last wave of tiles fills at most a quarter of the SMs, each of
    its tiles runs as four 64-token units; G4B_S8_QUARTER_TAIL=0 keeps whole
    tiles.  Both give the oracle's bits.  (300, 384, 160): every tile split,
    the second token tile ragged; (2048, 1280, 256): 80 tiles, a last wave too
    full to split on a 148-SM part."""
    pw, dw, A8, sa = _prep(M, N, K, seed=7)
    Cref, Yref = O.gemm_w8a8(A8, pw.w8, sa, pw.sw8.view(np.uint16))
    for q in ("1", "0"):
        monkeypatch.setenv("G4B_S8_QUARTER_TAIL", q)
        acc = torch.empty((M, N), dtype=torch.int32, device=DEV)
        Y = ops.gemm_w8a8(torch.from_numpy(A8).to(DEV), torch.from_numpy(sa).to(DEV), dw, acc=acc)
        torch.cuda.synchronize()
        assert L.query(L.Q_KERNEL_STATUS) == 0
        assert np.array_equal(acc.cpu().numpy(), Cref), f"int32 accumulators differ (quarter units {q})"
        assert np.array_equal(Y.cpu().numpy().view(np.uint16), Yref), f"f16 outputs differ (quarter units {q})"


@pytest.mark.parametrize("M,N,K", [s for s in SHAPES if s[1] % 32 == 0])
def test_w4a8_matches_oracle(M, N, K):
    pw, dw, A8, sa = _prep(M, N, K, seed=2 * M + N + K)
    ratio16 = dw.ratio16.cpu().numpy().view(np.uint16)
    Cref, Yref = O.gemm_w4a8(A8, pw.wp, ratio16, sa, pw.sw8.view(np.uint16), N)
    acc = torch.empty((M, N), dtype=torch.int32, device=DEV)
    Y = ops.gemm_w4a8(torch.from_numpy(A8).to(DEV), torch.from_numpy(sa).to(DEV), dw, acc=acc)
    torch.cuda.synchronize()
    assert L.query(L.Q_KERNEL_STATUS) == 0
    assert np.array_equal(acc.cpu().numpy(), Cref), f"int32 accumulators differ M={M} N={N} K={K}"
    assert np.array_equal(Y.cpu().numpy().view(np.uint16), Yref), "f16 outputs differ"


def test_w4a8_requant_clamps_and_ties():
    """Ratios large enough that (q - 8) * r leaves [-127, 127] (the clamp path),
    exact .5 products (round-half-to-even) and subnormal ratios."""
    M, N, K = 256, 256, 256
    pw, dw, A8, sa = _prep(M, N, K, seed=7)
    rng = np.random.default_rng(11)
    r = rng.uniform(0.0, 24.0, size=(K // 32, N)).astype(np.float16)
    r[:, :32] = np.float16(2.5)                      # (q - 8) * 2.5: every odd q - 8 is a tie
    r[:, 32:64] = np.float16(31.75)                  # |(q - 8) * r| up to 254: clamped
    r[:, 64:96] = np.float16(6e-8)                   # f16 subnormals
    r[0, 96:128] = np.float16(15.9375)               # largest ratio the unclamped path takes
    dw.ratio16 = torch.from_numpy(r).to(DEV)
    w8 = O.w4a8_requant(pw.wp, r.view(np.uint16), N, K)
    assert w8.min() == -127 and w8.max() == 127
    Cref, Yref = O.gemm_w4a8(A8, pw.wp, r.view(np.uint16), sa, pw.sw8.view(np.uint16), N)
    acc = torch.empty((M, N), dtype=torch.int32, device=DEV)
    Y = ops.gemm_w4a8(torch.from_numpy(A8).to(DEV), torch.from_numpy(sa).to(DEV), dw, acc=acc)
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy(), Cref)
    assert np.array_equal(Y.cpu().numpy().view(np.uint16), Yref)


def test_w8a8_extreme_int8_values():
    """All-(-127) and all-(+127) operands: the largest int32 sums the path can make."""
    M, N, K = 256, 128, 15360
    A8 = np.full((M, K), -127, np.int8)
    A8[1::2] = 127
    W8 = np.full((K, N), 127, np.int8)
    W8[:, 1::2] = -127
    sa = np.full((M,), 1e-3, np.float32)
    sw = np.full((N,), 1e-3, np.float16)
    dw = ops.DeviceWeight(N=N, K=K, nblk=K // 32, split=1, scale_fmt=0, inv=1.0,
                          wp=torch.zeros((K, N // 8), dtype=torch.int32, device=DEV),
                          scales=torch.zeros((K // 32, N), dtype=torch.float16, device=DEV),
                          scales16=torch.zeros((K // 32, N), dtype=torch.float16, device=DEV),
                          w8=torch.from_numpy(W8).to(DEV), sw8=torch.from_numpy(sw).to(DEV))
    acc = torch.empty((M, N), dtype=torch.int32, device=DEV)
    Y = ops.gemm_w8a8(torch.from_numpy(A8).to(DEV), torch.from_numpy(sa).to(DEV), dw, acc=acc)
    Cref, Yref = O.gemm_w8a8(A8, W8, sa, sw.view(np.uint16))
    torch.cuda.synchronize()
    assert abs(int(Cref[0, 0])) == 127 * 127 * K
    assert np.array_equal(acc.cpu().numpy(), Cref)
    assert np.array_equal(Y.cpu().numpy().view(np.uint16), Yref)


@pytest.mark.parametrize("w4", [False, True])
def test_config4_full_size_exact(w4):
    """Config 4 (M=4096, N=3840, K=15360) end to end on the GPU: cast_i8 of
    f16 activations, then the GEMM; int32 accumulators bit-exact against
    torch._int_mm on the same int8 operands, f16 outputs bit-exact against
    the shader epilogue of those accumulators."""
    M, N, K = 4096, 3840, 15360
    pw = pack.quant(weights(N, K, 0), fp8=False, prefill_i8=True)
    dw = ops.to_device(pw, DEV, w4a8=w4)
    X16 = torch.from_numpy(activations(M, K, seed=1).astype(np.float16)).to(DEV)
    A8, sa = ops.cast_i8(X16)
    acc = torch.empty((M, N), dtype=torch.int32, device=DEV)
    if w4:
        Y = ops.gemm_w4a8(A8, sa, dw, acc=acc)
        W8 = torch.from_numpy(O.w4a8_requant(pw.wp, dw.ratio16.cpu().numpy().view(np.uint16), N, K)).to(DEV)
    else:
        Y = ops.gemm_w8a8(A8, sa, dw, acc=acc)
        W8 = dw.w8
    try:
        ref = torch._int_mm(A8, W8)
    except RuntimeError:                 # some cuBLASLt builds want a column-major mat2
        ref = torch._int_mm(A8, W8.t().contiguous().t())
    torch.cuda.synchronize()
    assert L.query(L.Q_KERNEL_STATUS) == 0
    assert torch.equal(acc, ref)
    Yref = _epilogue(ref.cpu().numpy(), sa.cpu().numpy(), pw.sw8).astype(np.float16)
    assert np.array_equal(Y.cpu().numpy().view(np.uint16), Yref.view(np.uint16))


def test_s8_rejects_bad_shapes():
    lib = L.load()
    sh = torch.cuda.current_stream().cuda_stream
    A8 = torch.zeros((4, 64), dtype=torch.int8, device=DEV)
    W8 = torch.zeros((64, 136), dtype=torch.int8, device=DEV)
    sa = torch.zeros((4,), dtype=torch.float32, device=DEV)
    sw = torch.zeros((136,), dtype=torch.float16, device=DEV)
    Y = torch.zeros((4, 136), dtype=torch.float16, device=DEV)
    before = L.launches()
    assert lib.g4b_gemm_w8a8(A8.data_ptr(), W8.data_ptr(), sa.data_ptr(), sw.data_ptr(), Y.data_ptr(), 1, None,
                             4, 136, 64, sh) == L.G4B_E_SHAPE                    # N % 16
    assert lib.g4b_gemm_w8a8(A8.data_ptr(), W8.data_ptr(), sa.data_ptr(), sw.data_ptr(), Y.data_ptr(), 1, None,
                             4, 128, 48, sh) == L.G4B_E_SHAPE                    # K % 32
    assert lib.g4b_gemm_w8a8(A8.data_ptr() + 1, W8.data_ptr(), sa.data_ptr(), sw.data_ptr(), Y.data_ptr(), 1,
                             None, 4, 128, 64, sh) == L.G4B_E_ALIGN
    assert lib.g4b_gemm_w4a8(A8.data_ptr(), W8.data_ptr(), sw.data_ptr(), sa.data_ptr(), sw.data_ptr(),
                             Y.data_ptr(), 1, None, 4, 112, 64, sh) == L.G4B_E_SHAPE  # N % 32
    assert lib.g4b_gemm_w4a8(A8.data_ptr(), W8.data_ptr(), None, sa.data_ptr(), sw.data_ptr(),
                             Y.data_ptr(), 1, None, 4, 128, 64, sh) == L.G4B_E_ARG
    assert L.launches() == before
