"""The reference engine's per-op dispatch surface, on the g4b CUDA library.

gemma4-adreno's engine (src/vk_engine.py) drives its quantized matmuls through
four helpers, and a caller that swaps its Vulkan dispatches for g4b keeps the
same four calls with the same argument meaning:

    quant(W, pf=True)                      src/vk_engine.py:125-159
        -> (bw, bs, split, nblk, inv, bs16, w8, sw8), the buffers now CUDA tensors
    gemv_ds(qw, inbuf, outbuf, out_off=0)  src/vk_engine.py:214-226
        -> a recorded GEMV (the descriptor sets: GEMV + optional reduce)
    gemv(g)                                src/vk_engine.py:270-272
        -> runs it: g4b_gemv_i4 (split-K reduce fused in)
    gemm_ds(qw, inbuf, outbuf)             src/vk_engine.py:351-365
        -> a recorded prefill GEMM of MC rows
    gmm(t)                                 src/vk_engine.py:391-400
        -> runs it: cast_dn, g4b_gemm_i4, cast_up; or, under PREFILL_I8,
           g4b_cast_i8, g4b_gemm_w8a8, cast_up

`qw` is the engine's pair `(quant(W), (N, K))`.  As in the engine the
activations are f32 buffers: `inbuf` is an f32 tensor of at least K (GEMV) or
MC*K (GEMM) elements, `outbuf` an f32 tensor, and `out_off` is a BYTE offset
into it (the engine packs q, k and v into one buffer at byte offsets 0,
nq*4 and (nq+nk)*4, src/vk_engine.py:270-273).  The env switches keep their
meaning: GEMV_FP8=1 packs e4m3 GEMV scales, PREFILL_I8=1 packs the int8
prefill weights and routes gmm() through the W8A8 GEMM.  All work is queued
on the current CUDA stream; `fence_wait()` is the engine's bounded fence wait
(GEMMA4_FENCE_TIMEOUT_MS, src/vk_engine.py:294-302).
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np
import torch

from . import _lib as L
from . import ops
from . import pack

FP8 = pack.FP8
PREFILL_I8 = pack.PREFILL_I8
BLK = 32
MC = 128                       # the engine's prefill chunk (src/vk_engine.py:339)

_FENCE_MS = int(os.environ.get("GEMMA4_FENCE_TIMEOUT_MS", "0"))


def quant(W, pf: bool = True, device="cuda", fp8: Optional[bool] = None,
          prefill_i8: Optional[bool] = None) -> Tuple:
    """quant(W, pf) with the packed buffers resident on `device`.

    Returns the engine's 8-tuple (bw, bs, split, nblk, inv, bs16, w8, sw8):
    bw [K, N/8] int32 words, bs the GEMV scales (f16, or e4m3 bytes under
    GEMV_FP8), bs16 the f16 prefill scales, w8/sw8 the W8A8 weights or None."""
    pw = pack.quant(np.asarray(W, np.float32), pf, fp8=fp8, prefill_i8=prefill_i8)
    dw = ops.to_device(pw, device)
    return (dw.wp, dw.scales, dw.split, dw.nblk, dw.inv, dw.scales16, dw.w8, dw.sw8)


def _device_weight(qw) -> ops.DeviceWeight:
    (bw, bs, split, nblk, inv, bs16, w8, sw8), (N, K) = qw
    fmt = L.SCALE_E4M3 if bs.dtype == torch.uint8 else L.SCALE_F16
    return ops.DeviceWeight(N=N, K=K, nblk=nblk, split=split, scale_fmt=fmt, inv=inv, wp=bw, scales=bs,
                            scales16=bs16, w8=w8, sw8=sw8)


@dataclass
class GemvDispatch:
    """A recorded GEMV: what gemv_ds() binds (src/vk_engine.py:214-226)."""
    w: ops.DeviceWeight
    x: torch.Tensor              # [K] f32 view of inbuf
    y: torch.Tensor              # [N] f32 view of outbuf at out_off
    split: int
    N: int


def gemv_ds(qw, inbuf: torch.Tensor, outbuf: torch.Tensor, out_off: int = 0) -> GemvDispatch:
    """Bind a GEMV y = W x: x = inbuf[:K], y = outbuf at byte offset out_off.

    Shape rules as the engine's: N % 16 == 0, K % 32 == 0, and the reference's
    `split` (from quant) must divide K/32."""
    w = _device_weight(qw)
    if inbuf.dtype != torch.float32 or outbuf.dtype != torch.float32:
        raise TypeError("gemv_ds: the engine's activation buffers are f32")
    if out_off % 4:
        raise ValueError(f"gemv_ds: out_off={out_off} is not a multiple of 4 bytes")
    o = out_off // 4
    if inbuf.numel() < w.K or outbuf.numel() < o + w.N:
        raise ValueError(f"gemv_ds: buffers too small for N={w.N}, K={w.K}, out_off={out_off}")
    return GemvDispatch(w=w, x=inbuf.view(-1)[:w.K], y=outbuf.view(-1)[o:o + w.N], split=w.split, N=w.N)


def gemv(g: GemvDispatch, stream: Optional[torch.cuda.Stream] = None, pdl: bool = False,
         reference_split: bool = False) -> None:
    """Run a recorded GEMV (the GEMV dispatch and, for split > 1, its reduce).

    The K-split is the library's choice for the B200's SMs unless
    reference_split=True asks for quant()'s Adreno-tuned `split`; the result
    is the same up to f32 summation order."""
    ops.gemv_i4(g.x, g.w, split=g.split if reference_split else 0, out=g.y.view(1, -1), stream=stream, pdl=pdl)


@dataclass
class GemmDispatch:
    """A recorded prefill GEMM: what gemm_ds() binds (src/vk_engine.py:351-365)."""
    w: ops.DeviceWeight
    X: torch.Tensor              # [MC, K] f32 view of inbuf
    Y: torch.Tensor              # [MC, N] f32 view of outbuf
    Y16: torch.Tensor            # [MC, N] f16 staging (the engine's Yf16)
    i8: bool
    N: int
    K: int


def gemm_ds(qw, inbuf: torch.Tensor, outbuf: torch.Tensor, mc: int = MC,
            prefill_i8: Optional[bool] = None) -> GemmDispatch:
    """Bind a prefill GEMM of `mc` rows: Y[mc, N] = X[mc, K] @ W."""
    w = _device_weight(qw)
    i8 = PREFILL_I8 if prefill_i8 is None else prefill_i8
    if i8 and (w.w8 is None or w.sw8 is None):
        raise ValueError("gemm_ds: PREFILL_I8 needs quant(W, pf=True) with the int8 weights")
    if inbuf.dtype != torch.float32 or outbuf.dtype != torch.float32:
        raise TypeError("gemm_ds: the engine's activation buffers are f32")
    if inbuf.numel() < mc * w.K or outbuf.numel() < mc * w.N:
        raise ValueError(f"gemm_ds: buffers too small for MC={mc}, N={w.N}, K={w.K}")
    X = inbuf.view(-1)[:mc * w.K].view(mc, w.K)
    Y = outbuf.view(-1)[:mc * w.N].view(mc, w.N)
    Y16 = torch.empty((mc, w.N), dtype=torch.float16, device=Y.device)
    return GemmDispatch(w=w, X=X, Y=Y, Y16=Y16, i8=i8, N=w.N, K=w.K)


def gmm(t: GemmDispatch, stream: Optional[torch.cuda.Stream] = None) -> None:
    """Run a recorded prefill GEMM exactly as the engine's gmm() sequences it:
    f16 path: cast_dn (f32 -> f16) -> W4A16 GEMM -> Yf16 -> cast_up (f16 -> f32);
    PREFILL_I8: cast_i8 (f32 -> int8 + per-row scale) -> W8A8 GEMM -> Yf16 -> cast_up.
    The f16 staging keeps the engine's rounding of every output to f16."""
    if t.i8:
        A8, sa = ops.cast_i8(t.X, stream=stream)
        ops.gemm_w8a8(A8, sa, t.w, out=t.Y16, stream=stream)
    else:
        ops.gemm_i4(t.X, t.w, out=t.Y16, stream=stream)
    ops.cast(t.Y16, torch.float32, out=t.Y, stream=stream)


def fence_wait(label: str = "", stream: Optional[torch.cuda.Stream] = None,
               timeout_ms: Optional[int] = None) -> None:
    """Wait for the queued work, bounded by GEMMA4_FENCE_TIMEOUT_MS (0 = no
    limit) as the engine's _wait_fence() is; on timeout raise the engine's
    RuntimeError("GPU fence TIMEOUT after <ms>ms at [<label>]")."""
    ms = _FENCE_MS if timeout_ms is None else int(timeout_ms)
    dev = torch.device("cuda", torch.cuda.current_device())
    st = L.load().g4b_stream_wait(ops._stream_handle(stream, dev), ms)
    if st == L.G4B_E_TIMEOUT:
        raise RuntimeError(f"GPU fence TIMEOUT after {ms}ms at [{label}]")
    L.check("g4b_stream_wait", st)
