"""The reference benchmarks' own seeded correctness checks, re-run through the
CPU oracle.  These are the only checks the reference holds for the shader
math (cosine thresholds, no golden outputs): passing them pins the oracle's
shader restatements to what the reference validated on its hardware.

  benchmarks/vk_gemv.py:56-65,142-143        gemv+reduce vs f32 W@x, cos > 0.98
  benchmarks/coopgemm_i4.py:42-52,66-67      int4 GEMM vs X16 @ Wdq.T (0.9999-1.0 published)
  benchmarks/coopgemm_w4a8.py:74-110,126-137 W8A8 / W4A8 vs the f16 path (W8A8 0.99993 published)
  benchmarks/coopgemm_i8.py:41-44,77-80      s8 x s8 -> s32 exactness
"""
import numpy as np

import oracle as O
from util import cosine


def _pack_like_benchmark(W):
    r = O.pack_reference(W, prefill_i8=True)
    return r


def test_vk_gemv_fixture():
    K, N, SPLIT = 3840, 4096, 8
    rng = np.random.default_rng(0)
    xa = (rng.standard_normal(K) * 0.5).astype(np.float32)          # drawn first
    W = (rng.standard_normal((N, K)) * 0.1).astype(np.float32)
    r = _pack_like_benchmark(W)
    y = O.gemv(xa, r["wp"], r["scales16"], 0, 1.0, N, K, SPLIT)
    ref = (W @ xa).astype(np.float32)
    assert cosine(y, ref) > 0.98


def _i4_fixture(M, N, K):
    rng = np.random.default_rng(0)
    Xf = (rng.standard_normal((M, K)) * 0.1).astype(np.float32)
    X16 = Xf.astype(np.float16)
    Wf = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    r = _pack_like_benchmark(Wf)
    nblk = K // 32
    q = r["q"].astype(np.float32)
    Wdq = ((q - 8).reshape(N, nblk, 32) * r["sc_f32"][:, :, None]).reshape(N, K)
    ref = X16.astype(np.float32) @ Wdq.T
    Y = O.gemm_i4(X16.view(np.uint16), r["wp"], r["scales16"], M, N, K)
    return Y, ref


def test_coopgemm_i4_fixture_down():
    Y, ref = _i4_fixture(128, 3840, 15360)
    assert cosine(Y, ref) >= 0.9999


def test_coopgemm_i4_fixture_gate():
    Y, ref = _i4_fixture(128, 15360, 3840)
    assert cosine(Y, ref) >= 0.9999


def test_coopgemm_w4a8_fixture():
    M, K, N = 128, 3840, 15360
    rng = np.random.default_rng(0)
    W = (rng.standard_normal((N, K)) * 0.08).astype(np.float32)
    r = _pack_like_benchmark(W)
    nblk = K // 32
    deqW = (r["q"].astype(np.float32) - 8.0) * np.repeat(r["sc_f32"], 32, axis=1)
    X = (rng.standard_normal((M, K)) * 0.3).astype(np.float32)
    s_a = np.maximum(np.abs(X).max(1) / 127.0, 1e-12).astype(np.float32)
    A_i8 = np.clip(np.round(X / s_a[:, None]), -127, 127).astype(np.int8)
    Y_f16path = X @ deqW.T
    # W8A8 with the precomputed int8 weights
    _, Y8 = O.gemm_w8a8(A_i8, r["w8"], s_a, r["sw8"])
    c8 = cosine(Y8.view(np.float16).astype(np.float32), Y_f16path)
    assert c8 >= 0.9999, c8                                       # published 0.99993
    # W4A8 with the on-the-fly requant
    ratio = O.w4a8_ratio(r["sc_f32"], r["sw_f32"])
    _, Y4 = O.gemm_w4a8(A_i8, r["wp"], ratio, s_a, r["sw8"], N)
    c4 = cosine(Y4.view(np.float16).astype(np.float32), Y_f16path)
    assert c4 >= 0.999, c4
    # the oracle's cast_i8 reproduces the benchmark's numpy activation quantiser
    A_o, sa_o = O.cast_i8(X)
    assert np.array_equal(sa_o, s_a)
    assert np.count_nonzero(A_o != A_i8) == 0


def test_coopgemm_i8_exactness_fixture():
    M = N = 1024
    K = 2048
    rng = np.random.default_rng(0)
    A = rng.integers(-8, 8, size=(M, K), dtype=np.int8)
    B = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    ref = A.astype(np.int32) @ B.astype(np.int32)
    C, _ = O.gemm_w8a8(A, B, np.ones(M, np.float32), np.full(N, 0x3C00, np.uint16))
    assert np.array_equal(C, ref)
