"""GPU parity of the decode path through the C ABI: int4 GEMV (f16 and e4m3
scales, f32/f16 activations and outputs, reference and library splits, M <= 8
and looped M), the split-K reduce, the dequantiser, and determinism.

Oracle: oracle/g4b_oracle.c (orc_gemv restates vk/gemv.comp / vk/gemv_fp8.comp
+ vk/reduce.comp).  Floating-point bar (tests/util.py): max relative error
<= 1e-2 with denominator max(|ref|, 1e-3 * rms(ref)), cosine >= 0.9999.
Integer/byte/index outputs (dequantised f16 weights, reduce order) bit-exact.
"""
import numpy as np
import pytest
import torch

import oracle as O
from g4b import _lib as L
from g4b import ops, pack
from util import assert_close, cosine, rel_err, weights, activations

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _packed(N, K, seed=0, fp8=False, std=0.02):
    W = weights(N, K, seed, std)
    pw = pack.quant(W, fp8=fp8, prefill_i8=False)
    return W, pw, ops.to_device(pw, DEV)


def _oracle_y(pw, x32, split=None):
    split = pw.split if split is None else split
    return O.gemv(x32, pw.wp, pw.scales.view(np.uint16) if pw.scale_fmt == 0 else pw.scales,
                  pw.scale_fmt, pw.inv, pw.N, pw.K, split)


@pytest.mark.parametrize("N,K", [(15360, 3840), (4096, 3840), (2048, 3840), (3840, 4096), (3840, 15360),
                                 (256, 32), (272, 64), (48, 96), (1040, 1024),
                                 (800, 576), (2080, 64), (32, 3840)])
@pytest.mark.parametrize("fp8", [False, True])
def test_gemv_matches_oracle(N, K, fp8):
    W, pw, dw = _packed(N, K, seed=N + K, fp8=fp8)
    x = activations(1, K, seed=7)[0]
    ref = _oracle_y(pw, x)
    for xdt in (torch.float32, torch.float16):
        xt = torch.from_numpy(x).to(DEV).to(xdt)
        x_used = xt.float().cpu().numpy()
        ref_x = ref if xdt == torch.float32 else _oracle_y(pw, x_used)
        for split in (0, pw.split):
            y = ops.gemv_i4(xt, dw, split=split, out_dtype=torch.float32)
            torch.cuda.synchronize()
            assert_close(y.cpu().numpy(), ref_x, f"N={N} K={K} fp8={fp8} x={xdt} split={split}")


def test_gemv_f16_output_config1():
    """Config 1: W[15360, 3840] N(0, 0.02), x f16 N(0, 1), y f16, f32 accumulate."""
    N, K = 15360, 3840
    W, pw, dw = _packed(N, K, seed=0)
    x16 = activations(1, K, seed=1)[0].astype(np.float16)
    ref = _oracle_y(pw, x16.astype(np.float32))
    y = ops.gemv_i4(torch.from_numpy(x16).to(DEV), dw, out_dtype=torch.float16)
    torch.cuda.synchronize()
    out = y.float().cpu().numpy()
    assert_close(out, ref, "config1 f16 out")
    # The f16 output is the f32 result rounded once.  Against the exact product
    # (f64, from the bit-exact f32 dequantisation) rounded to f16 it may differ by
    # one f16 ulp plus f32 summation noise: at the 1e-3 x rms guard a 2e-6
    # absolute f32 error (the oracle's own, summing 3840 products in order) is
    # already 1.5e-3 of the denominator, so the bound is 3e-3.
    Wd = ops.dequant_i4(dw, out_dtype=torch.float32).double()          # [K, N], exact (q - 8) * s
    exact = (torch.from_numpy(x16).to(DEV).double() @ Wd).cpu().numpy()
    assert rel_err(out, exact.astype(np.float16).astype(np.float32)) < 3e-3
    assert rel_err(ref, exact) < 3e-3                                   # the oracle meets the same bound


@pytest.mark.parametrize("M", [2, 3, 4, 5, 8, 13])
@pytest.mark.parametrize("xdt", [torch.float32, torch.float16])
def test_gemv_small_batch(M, xdt):
    N, K = 4096, 3840
    W, pw, dw = _packed(N, K, seed=3)
    X = activations(M, K, seed=11)
    Xt = torch.from_numpy(X).to(DEV).to(xdt)
    ref = _oracle_y(pw, Xt.float().cpu().numpy())
    Y = ops.gemv_i4(Xt, dw, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert Y.shape == (M, N)
    for m in range(M):
        assert_close(Y[m].cpu().numpy(), ref[m], f"M={M} token {m}")


def test_gemv_vk_gemv_fixture():
    """benchmarks/vk_gemv.py:56-65,143 through the CUDA kernel: cos > 0.98 vs f32 W@x."""
    K, N, SPLIT = 3840, 4096, 8
    rng = np.random.default_rng(0)
    xa = (rng.standard_normal(K) * 0.5).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.1).astype(np.float32)
    pw = pack.quant(W, fp8=False, prefill_i8=False)
    dw = ops.to_device(pw, DEV)
    y = ops.gemv_i4(torch.from_numpy(xa).to(DEV), dw, split=SPLIT)
    torch.cuda.synchronize()
    assert cosine(y.cpu().numpy(), W @ xa) > 0.98
    assert_close(y.cpu().numpy(), _oracle_y(pw, xa, SPLIT), "vk_gemv fixture vs oracle")


def test_gemv_deterministic_and_workspace_reusable():
    N, K = 3840, 15360
    W, pw, dw = _packed(N, K, seed=5)
    x = torch.from_numpy(activations(1, K, seed=2)[0]).to(DEV)
    outs = [ops.gemv_i4(x, dw).cpu() for _ in range(4)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    # different shapes through the same workspace in a row
    W2, pw2, dw2 = _packed(15360, 3840, seed=6)
    x2 = torch.from_numpy(activations(1, 3840, seed=3)[0]).to(DEV)
    a = ops.gemv_i4(x2, dw2).cpu()
    b = ops.gemv_i4(x, dw).cpu()
    c = ops.gemv_i4(x2, dw2).cpu()
    assert torch.equal(a, c) and torch.equal(b, outs[0])


def test_gemv_workspace_errors():
    N, K = 3840, 15360
    W, pw, dw = _packed(N, K, seed=5)
    x = torch.zeros(K, device=DEV)
    need = ops.gemv_workspace_bytes(1, N, K, 0)
    assert need > 0
    small = torch.zeros(need - 256, dtype=torch.uint8, device=DEV)
    with pytest.raises(L.G4BError) as ei:
        ops.gemv_i4(x, dw, workspace=small)
    assert ei.value.code == L.G4B_E_WORKSPACE
    with pytest.raises(L.G4BError) as ei:
        ops.gemv_i4(x, dw, split=7)
    assert ei.value.code == L.G4B_E_SHAPE


def test_reduce_partials_bit_exact():
    rng = np.random.default_rng(8)
    for N, split in [(4096, 40), (15360, 12), (3840, 48), (16, 1)]:
        part = rng.standard_normal((split, N)).astype(np.float32)
        ref = O.reduce(part, N, split)
        y = ops.reduce_partials(torch.from_numpy(part).to(DEV), split)
        torch.cuda.synchronize()
        assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("fp8", [False, True])
def test_dequant_bit_exact(fp8):
    N, K = 1024, 512
    W, pw, dw = _packed(N, K, seed=21, fp8=fp8, std=0.05)
    if fp8:
        ref32 = O.dequant(pw.wp, pw.scales, 1, pw.inv, N, K)            # (q - 8) * e4m3(scale) * inv
        out32 = ops.dequant_i4(dw, torch.float32).cpu().numpy()
        assert np.array_equal(out32.view(np.uint32), ref32.view(np.uint32))
    else:
        ref16 = O.dequant(pw.wp, pw.scales.view(np.uint16), 0, 1.0, N, K)  # f16((q - 8) * scale), i4h tile
        out16 = ops.dequant_i4(dw, torch.float16).cpu().numpy()
        assert np.array_equal(out16.view(np.uint16), ref16)
        q = ((pw.wp[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 15).reshape(K, N).astype(np.float32)
        s = np.repeat(pw.scales.astype(np.float32), 32, axis=0)
        out32 = ops.dequant_i4(dw, torch.float32).cpu().numpy()
        assert np.array_equal(out32, (q - 8) * s)                         # exact in f32


def test_query_device():
    assert L.query(L.Q_DEVICE_OK) == 1
    assert L.query(L.Q_SM_COUNT) >= 100
    before = L.launches()
    W, pw, dw = _packed(256, 64)
    ops.gemv_i4(torch.zeros(64, device=DEV), dw)
    assert L.launches() == before + 1


def test_gemv_shared_workspace_across_shapes_matches_oracle():
    """One workspace tensor reused by shapes with different partial sizes, in an
    order where a larger call's partials cover a smaller call's former layout."""
    cases = [(15360, 3840, 12), (2048, 3840, 0), (3840, 15360, 0), (4096, 3840, 40), (15360, 3840, 0)]
    need = max(ops.gemv_workspace_bytes(1, N, K, s) for N, K, s in cases)
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    for rep in range(2):
        for N, K, s in cases:
            W, pw, dw = _packed(N, K, seed=N + 3 * K)
            x = activations(1, K, seed=N)[0]
            y = ops.gemv_i4(torch.from_numpy(x).to(DEV), dw, split=s, workspace=ws)
            torch.cuda.synchronize()
            assert_close(y.cpu().numpy(), _oracle_y(pw, x), f"rep {rep} N={N} K={K} split={s}")


@pytest.mark.parametrize("fp8", [False, True])
def test_gemv_lm_head_shape(fp8):
    """lm_head [262144, 3840]: the widest GEMV of the decode stream (1024 column tiles)."""
    from g4b.quant_gpu import quant_device
    N, K = 262144, 3840
    gen = torch.Generator(device=DEV)
    gen.manual_seed(4)
    W = torch.randn((N, K), generator=gen, device=DEV).mul_(0.02)
    dw = quant_device(W, pf=False, fp8=fp8, prefill_i8=False)
    del W
    x = activations(1, K, seed=9)[0].astype(np.float16)
    for rep in range(2):
        y = ops.gemv_i4(torch.from_numpy(x).to(DEV), dw, out_dtype=torch.float32)
        torch.cuda.synchronize()
    wp = dw.wp.cpu().numpy().view(np.uint32)
    sc = dw.scales.cpu().numpy()
    ref = O.gemv(x.astype(np.float32), wp, sc.view(np.uint16) if not fp8 else sc, dw.scale_fmt, dw.inv, N, K, 1)
    assert_close(y.cpu().numpy(), ref, f"lm_head fp8={fp8}")
    assert L.query(L.Q_KERNEL_STATUS) == 0


@pytest.mark.parametrize("fp8", [False, True])
def test_gemv_pdl_chain_keeps_dependencies(fp8):
    """GEMVs launched with programmatic dependent launch, each consuming the
    previous one's output through one shared workspace, eager and in a graph."""
    K = 3840
    layers = [_packed(K, K, seed=40 + i, fp8=fp8) for i in range(4)]
    x0 = activations(1, K, seed=3)[0]
    ref = x0
    for _, pw, _ in layers:
        ref = _oracle_y(pw, ref.astype(np.float32)).astype(np.float32)
    ws = torch.zeros(ops.gemv_workspace_bytes(1, K, K, 0) + 256, dtype=torch.uint8, device=DEV)
    bufs = [torch.empty(K, device=DEV) for _ in range(len(layers) + 1)]
    stream = torch.cuda.Stream()

    def chain():
        for i, (_, _, dw) in enumerate(layers):
            ops.gemv_i4(bufs[i], dw, out=bufs[i + 1], stream=stream, workspace=ws, pdl=True)

    bufs[0].copy_(torch.from_numpy(x0))
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        chain()
    stream.synchronize()
    assert_close(bufs[-1].cpu().numpy(), ref, f"pdl chain eager fp8={fp8}")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        chain()
    for b in bufs[1:]:
        b.zero_()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
    stream.synchronize()
    assert_close(bufs[-1].cpu().numpy(), ref, f"pdl chain graph fp8={fp8}")
    assert L.query(L.Q_KERNEL_STATUS) == 0
    del g


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("xdt", [torch.float16, torch.float32])
def test_gemv_fused_segments_match_oracle(fp8, xdt):
    """g4b_gemv_i4_fused: q/k/v (three widths) and gate/up on one x, each
    segment against the oracle; the e4m3 segments carry different inverse
    scales (one weight is 16x larger, so its shift differs)."""
    K = 3840
    x = activations(1, K, seed=21)[0]
    xt = torch.from_numpy(x).to(DEV).to(xdt)
    x_used = xt.float().cpu().numpy()
    for Ns in ([4096, 2048, 2048], [15360, 15360], [800]):
        packed = []
        for i, N in enumerate(Ns):
            std = 0.32 if i == 1 else 0.02
            packed.append(_packed(N, K, seed=50 + 7 * i + N, fp8=fp8, std=std))
        if fp8 and len(Ns) > 1:
            assert packed[0][1].inv != packed[1][1].inv
        outs = ops.gemv_i4_fused(xt, [p[2] for p in packed], out_dtype=torch.float32)
        torch.cuda.synchronize()
        for (W, pw, dw), y in zip(packed, outs):
            assert_close(y.cpu().numpy(), _oracle_y(pw, x_used), f"fused N={pw.N} of {Ns} fp8={fp8} x={xdt}")
    assert L.query(L.Q_KERNEL_STATUS) == 0


def test_gemv_fused_rejects_bad_arguments():
    lib = L.load()
    K = 256
    _, _, a = _packed(256, K, seed=1)
    _, _, b = _packed(272, K, seed=2)                                   # N % 32 != 0
    x = torch.zeros(K, dtype=torch.float16, device=DEV)
    y = torch.zeros(512, dtype=torch.float32, device=DEV)
    sh = torch.cuda.current_stream().cuda_stream
    mk = lambda ws: (L.GemvSegment * len(ws))(*[L.GemvSegment(w.wp.data_ptr(), w.scales.data_ptr(), 1.0,  # noqa
                                                                y.data_ptr(), w.N) for w in ws])
    import ctypes
    before = L.launches()
    segs = mk([a, b])
    assert lib.g4b_gemv_i4_fused(x.data_ptr(), 1, 2, ctypes.cast(segs, ctypes.c_void_p), 0, 0, K, None, 0, 0,
                                 sh) == L.G4B_E_SHAPE
    segs = mk([a, a, a, a])
    assert lib.g4b_gemv_i4_fused(x.data_ptr(), 1, 4, ctypes.cast(segs, ctypes.c_void_p), 0, 0, K, None, 0, 0,
                                 sh) == L.G4B_E_ARG
    segs = mk([a])
    assert lib.g4b_gemv_i4_fused(x.data_ptr(), 1, 1, ctypes.cast(segs, ctypes.c_void_p), 0, 0, 96, None, 0, 0,
                                 sh) == L.G4B_E_SHAPE                    # K % 64
    assert L.launches() == before
