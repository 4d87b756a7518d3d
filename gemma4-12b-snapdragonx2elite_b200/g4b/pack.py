"""Host-side int4 weight packing: the engine's ``quant()`` (src/vk_engine.py:125-159).

The packed layout is the reference's, byte for byte, so the CUDA kernels read
exactly the buffers the Vulkan shaders read:

* ``wp``      [K, N/8] uint32: nibble j of word (k, g) is column 8g+j, holding
  ``clip(round_half_even(W / scale) + 8, 0, 15)`` (src/vk_engine.py:128-130)
* ``scales``  [K/32, N]: f16 block scales ``max(absmax/7, 1e-8)`` (:127, 131), or
  with ``GEMV_FP8=1`` e4m3 bytes of the scales lifted by a per-tensor power of
  two into e4m3's normal range, with ``inv = 2^-shift`` (:133-137)
* ``scales16`` [K/32, N] f16: always kept, the prefill GEMM reads it (:150)
* ``split``   the reference's split-K heuristic (:143-148)
* ``w8``/``sw8`` with ``PREFILL_I8=1`` (and ``pf``): the W8A8 prefill weights, the
  int4-dequantised rows re-quantised to int8 [K, N] against a per-row f16
  scale (:152-157)

``GEMV_FP8`` and ``PREFILL_I8`` are read from the environment at import, as the
reference engine reads them (src/vk_engine.py:8-9); ``quant`` also takes them as
keyword overrides.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional

import numpy as np

BLK = 32
FP8 = os.environ.get("GEMV_FP8") == "1"
PREFILL_I8 = os.environ.get("PREFILL_I8") == "1"


@dataclass
class PackedWeight:
    """Host (numpy) form of one packed linear layer, weight W[N, K]."""
    N: int
    K: int
    wp: np.ndarray                  # [K, N/8] uint32
    scales: np.ndarray              # [nblk, N] float16 or uint8 (e4m3)
    scale_fmt: int                  # 0 = f16, 1 = e4m3
    inv: float                      # e4m3 2^-shift (1.0 for f16 scales)
    split: int                      # the reference's split-K choice
    nblk: int
    scales16: np.ndarray            # [nblk, N] float16 (prefill)
    w8: Optional[np.ndarray] = None     # [K, N] int8 (W8A8 prefill)
    sw8: Optional[np.ndarray] = None    # [N] float16
    sw_f32: Optional[np.ndarray] = None  # [N] float32 (s_w before f16 storage; W4A8 ratio input)
    sc_f32: Optional[np.ndarray] = None  # [N, nblk] float32 block scales (W4A8 ratio input)

    def as_reference_tuple(self):
        """The 8-tuple ``quant()`` returns: (bw, bs, split, nblk, inv, bs16, w8, sw8)."""
        return (self.wp, self.scales, self.split, self.nblk, self.inv, self.scales16, self.w8, self.sw8)


def split_for(N: int, nblk: int) -> int:
    """src/vk_engine.py:143-148: ~384 workgroups in total on the Adreno."""
    rows = (N // 8 + 63) // 64
    want = max(1, -(-384 // max(rows, 1)))
    best = 1
    for s in range(1, nblk + 1):
        if nblk % s == 0 and (abs(s - want), s) < (abs(best - want), best):
            best = s
    return best


def block_scales(W: np.ndarray) -> np.ndarray:
    """[N, K] f32 -> [N, nblk] f32 block scales max(absmax / 7, 1e-8)."""
    N, K = W.shape
    a = np.abs(W.reshape(N, K // BLK, BLK)).max(axis=2)
    return np.maximum(a / np.float32(7.0), np.float32(1e-8)).astype(np.float32)


def nibbles(W: np.ndarray, sc: np.ndarray) -> np.ndarray:
    """[N, K] uint8 in [0, 15]: round-half-even(W / scale) + 8, clipped."""
    N, K = W.shape
    r = np.rint(W.reshape(N, K // BLK, BLK) / sc[:, :, None]) + np.float32(8.0)
    return np.clip(r, 0, 15).astype(np.uint8).reshape(N, K)


def pack_nibbles(q: np.ndarray) -> np.ndarray:
    """[N, K] nibbles -> [K, N/8] uint32 words, column 8g+j at bits 4j."""
    N, K = q.shape
    qt = np.ascontiguousarray(q.T).reshape(K, N // 8, 8).astype(np.uint32)
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, None, :]
    return np.bitwise_or.reduce(qt << shifts, axis=2).astype(np.uint32)


def e4m3_scales(sc: np.ndarray):
    """[N, nblk] f32 scales -> ([nblk, N] e4m3 bytes, inv): src/vk_engine.py:133-137."""
    import torch

    mx = float(sc.max())
    shift = int(np.floor(np.log2(256.0 / mx))) if mx > 0 else 0
    lifted = np.clip(sc * np.float32(2.0 ** shift), 0.0, 448.0).astype(np.float32)
    e8 = torch.from_numpy(np.ascontiguousarray(lifted.T)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return e8, float(2.0 ** -shift)


def w8a8_weights(q: np.ndarray, sc: np.ndarray):
    """src/vk_engine.py:152-157 -> (w8 [K, N] int8, sw16 [N] f16, s_w [N] f32)."""
    N, K = q.shape
    deq = (q.astype(np.float32) - np.float32(8.0)) * np.repeat(sc, BLK, axis=1)
    s_w = np.maximum(np.abs(deq).max(axis=1) / np.float32(127.0), np.float32(1e-12)).astype(np.float32)
    w8 = np.clip(np.rint(deq / s_w[:, None]), -127, 127).astype(np.int8)
    return np.ascontiguousarray(w8.T), s_w.astype(np.float16), s_w


def w4a8_ratio(sc: np.ndarray, s_w: np.ndarray) -> np.ndarray:
    """[nblk, N] f16 ratio = block scale / s_w (benchmarks/coopgemm_w4a8.py:84)."""
    return np.ascontiguousarray((sc / s_w[:, None]).T).astype(np.float16)


def quant(W, pf: bool = True, *, fp8: Optional[bool] = None, prefill_i8: Optional[bool] = None) -> PackedWeight:
    """Pack a [N, K] weight exactly as the engine's quant(W, pf) does."""
    fp8 = FP8 if fp8 is None else fp8
    prefill_i8 = PREFILL_I8 if prefill_i8 is None else prefill_i8
    W = np.ascontiguousarray(W, dtype=np.float32)
    N, K = W.shape
    if K % BLK or N % 8:
        raise ValueError(f"quant: K={K} must be a multiple of {BLK} and N={N} of 8")
    nblk = K // BLK
    sc = block_scales(W)
    q = nibbles(W, sc)
    wp = pack_nibbles(q)
    sc16 = np.ascontiguousarray(sc.T).astype(np.float16)
    if fp8:
        scales, inv, fmt = *e4m3_scales(sc), 1
    else:
        scales, inv, fmt = sc16, 1.0, 0
    pw = PackedWeight(N=N, K=K, wp=wp, scales=scales, scale_fmt=fmt, inv=inv,
                      split=split_for(N, nblk), nblk=nblk, scales16=sc16, sc_f32=sc)
    if prefill_i8 and pf:
        pw.w8, pw.sw8, pw.sw_f32 = w8a8_weights(q, sc)
    return pw
