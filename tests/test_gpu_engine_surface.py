"""The engine-shaped surface (g4b.engine_surface): gemv_ds/gemv and gemm_ds/gmm
used the way src/vk_engine.py uses them, checked against the CPU oracle.

- gemv into one packed q/k/v buffer at byte offsets (src/vk_engine.py:270-273),
  f32 activation buffers, within the floating-point bar of tests/util.py;
- gmm's f16 path (cast_dn -> W4A16 GEMM -> cast_up), within that bar;
- gmm's PREFILL_I8 path (cast_i8 -> W8A8 -> cast_up): bit-exact, since every
  step is integer or a fixed sequence of correctly rounded operations;
- fence_wait's timeout message.
"""
import numpy as np
import pytest
import torch

import oracle as O
from g4b import engine_surface as E
from util import assert_close, weights, activations

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("fp8", [False, True])
def test_gemv_qkv_into_one_buffer(fp8):
    H, nq, nk = 3840, 4096, 2048
    Ws = {"q": weights(nq, H, 1), "k": weights(nk, H, 2), "v": weights(nk, H, 3)}
    qw = {k: (E.quant(W, pf=False, fp8=fp8, prefill_i8=False), W.shape) for k, W in Ws.items()}
    x = activations(1, H, seed=4)[0]
    inbuf = torch.from_numpy(x).to(DEV)
    qkv = torch.full((nq + 2 * nk,), np.nan, dtype=torch.float32, device=DEV)
    ds = [E.gemv_ds(qw["q"], inbuf, qkv, 0), E.gemv_ds(qw["k"], inbuf, qkv, nq * 4),
          E.gemv_ds(qw["v"], inbuf, qkv, (nq + nk) * 4)]
    for g in ds:
        E.gemv(g)
    E.fence_wait("qkv")
    out = qkv.cpu().numpy()
    off = 0
    for k in ("q", "k", "v"):
        (bw, bs, split, nblk, inv, _b16, _w8, _s8), (N, K) = qw[k]
        sc = bs.cpu().numpy()
        ref = O.gemv(x, bw.cpu().numpy().view(np.uint32), sc.view(np.uint16) if not fp8 else sc,
                     1 if fp8 else 0, inv, N, K, split)
        assert_close(out[off:off + N], ref, f"{k} fp8={fp8}")
        off += N


def test_gemv_reference_split_matches():
    N, K = 15360, 3840
    W = weights(N, K, 0)
    qw = (E.quant(W, pf=False, fp8=False, prefill_i8=False), (N, K))
    inbuf = torch.from_numpy(activations(1, K, seed=1)[0]).to(DEV)
    a = torch.empty(N, dtype=torch.float32, device=DEV)
    b = torch.empty(N, dtype=torch.float32, device=DEV)
    E.gemv(E.gemv_ds(qw, inbuf, a))
    E.gemv(E.gemv_ds(qw, inbuf, b), reference_split=True)
    E.fence_wait()
    assert_close(a.cpu().numpy(), b.cpu().numpy(), "library split vs reference split")


def test_gemv_ds_rejects_bad_buffers():
    N, K = 256, 256
    qw = (E.quant(weights(N, K, 0), pf=False, fp8=False, prefill_i8=False), (N, K))
    x = torch.zeros(K, dtype=torch.float32, device=DEV)
    with pytest.raises(ValueError):
        E.gemv_ds(qw, x, torch.zeros(N, dtype=torch.float32, device=DEV), out_off=4)
    with pytest.raises(TypeError):
        E.gemv_ds(qw, x.half(), torch.zeros(N, dtype=torch.float32, device=DEV))


def test_gmm_f16_path():
    N, K, mc = 3840, 3840, E.MC
    W = weights(N, K, 5)
    qw = (E.quant(W, pf=True, fp8=False, prefill_i8=False), (N, K))
    X = activations(mc, K, seed=6)
    inbuf = torch.from_numpy(X).to(DEV)
    outbuf = torch.empty(mc * N, dtype=torch.float32, device=DEV)
    t = E.gemm_ds(qw, inbuf, outbuf, prefill_i8=False)
    E.gmm(t)
    E.fence_wait("gmm")
    (bw, _bs, _s, _n, _i, bs16, _w8, _sw8), _ = qw
    ref = O.gemm_i4(X.astype(np.float16).view(np.uint16), bw.cpu().numpy().view(np.uint32),
                    bs16.cpu().numpy().view(np.uint16), mc, N, K)
    assert_close(outbuf.view(mc, N).cpu().numpy(), ref, "gmm f16 path")


def test_gmm_prefill_i8_path_bit_exact():
    N, K, mc = 3840, 15360, E.MC
    W = weights(N, K, 7)
    qw = (E.quant(W, pf=True, fp8=False, prefill_i8=True), (N, K))
    X = activations(mc, K, seed=8)
    inbuf = torch.from_numpy(X).to(DEV)
    outbuf = torch.empty(mc * N, dtype=torch.float32, device=DEV)
    t = E.gemm_ds(qw, inbuf, outbuf, prefill_i8=True)
    E.gmm(t)
    E.fence_wait("gmm i8")
    (_bw, _bs, _s, _n, _i, _b16, w8, sw8), _ = qw
    A8, sa = O.cast_i8(X)
    _C, Y16 = O.gemm_w8a8(A8, w8.cpu().numpy(), sa, sw8.cpu().numpy().view(np.uint16))
    ref = Y16.view(np.float16).astype(np.float32)
    assert np.array_equal(outbuf.view(mc, N).cpu().numpy(), ref)


def test_fence_wait_timeout_message():
    """A stream held by a sleeping kernel: fence_wait with a 1 ms bound raises
    the engine's timeout error, then a second wait without a bound succeeds."""
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        torch.cuda._sleep(200_000_000)              # ~0.1 s of GPU time on this stream
    with pytest.raises(RuntimeError, match=r"GPU fence TIMEOUT after 1ms at \[sleep\]"):
        E.fence_wait("sleep", stream=s, timeout_ms=1)
    E.fence_wait("sleep", stream=s, timeout_ms=0)
