"""quant() on the GPU: the engine's weight packing (src/vk_engine.py:125-159)
run by the CUDA library, bit-exact to the host packer in ``g4b.pack``.

The reference re-quantises the whole model on the host at every start-up
(about four minutes, service/README.md:7-9); here a [N, K] f32 weight already
in HBM is packed at memory speed.  The only host step is the e4m3 shift,
computed from the device-side max scale with the reference's own formula.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import _lib as L
from .ops import DeviceWeight, _ptr
from .pack import BLK, FP8, PREFILL_I8, split_for


def quant_device(W: torch.Tensor, pf: bool = True, *, fp8: Optional[bool] = None,
                 prefill_i8: Optional[bool] = None, w4a8: bool = False,
                 stream: Optional[torch.cuda.Stream] = None) -> DeviceWeight:
    fp8 = FP8 if fp8 is None else fp8
    prefill_i8 = PREFILL_I8 if prefill_i8 is None else prefill_i8
    if not (W.is_cuda and W.dtype == torch.float32 and W.dim() == 2):
        raise ValueError("quant_device: W must be a 2-D float32 CUDA tensor")
    W = W.contiguous()
    N, K = W.shape
    if K % BLK or N % 8:
        raise ValueError(f"quant_device: K={K} must be a multiple of {BLK} and N={N} of 8")
    nblk = K // BLK
    dev = W.device
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    sh = int(s.cuda_stream)
    lib = L.load()
    wp = torch.empty((K, N // 8), dtype=torch.int32, device=dev)
    sc16 = torch.empty((nblk, N), dtype=torch.float16, device=dev)
    sc32 = torch.empty((N, nblk), dtype=torch.float32, device=dev)
    amax = torch.zeros((1,), dtype=torch.int32, device=dev)
    L.check("g4b_quant_i4", lib.g4b_quant_i4(_ptr(W), N, K, _ptr(wp), _ptr(sc16), _ptr(sc32), _ptr(amax), sh))
    scales, fmt, inv = sc16, L.SCALE_F16, 1.0
    if fp8:
        s.synchronize()
        mx = float(np.array([amax.item()], np.int32).view(np.float32)[0])
        shift = int(np.floor(np.log2(256.0 / mx))) if mx > 0 else 0   # src/vk_engine.py:134
        e8 = torch.empty((nblk, N), dtype=torch.uint8, device=dev)
        L.check("g4b_quant_e4m3", lib.g4b_quant_e4m3(_ptr(sc32), N, K, shift, _ptr(e8), sh))
        scales, fmt, inv = e8, L.SCALE_E4M3, float(2.0 ** -shift)
    dw = DeviceWeight(N=N, K=K, nblk=nblk, split=split_for(N, nblk), scale_fmt=fmt, inv=inv,
                      wp=wp, scales=scales, scales16=sc16)
    if prefill_i8 and pf:
        dw.w8 = torch.empty((K, N), dtype=torch.int8, device=dev)
        dw.sw8 = torch.empty((N,), dtype=torch.float16, device=dev)
        ratio = torch.empty((nblk, N), dtype=torch.float16, device=dev) if w4a8 else None
        L.check("g4b_quant_w8a8", lib.g4b_quant_w8a8(_ptr(wp), _ptr(sc32), N, K, _ptr(dw.w8), _ptr(dw.sw8),
                                                     None, _ptr(ratio), sh))
        dw.ratio16 = ratio
    return dw
