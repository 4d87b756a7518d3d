"""torch-tensor front end of the g4b CUDA library.

PyTorch provides device memory, streams and the tensors' pointers; every
computation runs in the CUDA library through its C ABI (``include/g4b.h``).
If the library cannot be loaded these functions raise -- there is no CPU or
PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import threading
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _lib as L
from .pack import PackedWeight, w4a8_ratio

_DT = {torch.float32: L.DT_F32, torch.float16: L.DT_F16}


def _stream_handle(stream: Optional[torch.cuda.Stream], device: torch.device) -> int:
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return int(s.cuda_stream)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else int(t.data_ptr())


def _need(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


@dataclass
class DeviceWeight:
    """One packed linear layer resident in HBM (the reference's Buf set for a layer)."""
    N: int
    K: int
    nblk: int
    split: int
    scale_fmt: int
    inv: float
    wp: torch.Tensor                      # [K, N/8] int32 (bit pattern of the uint32 words)
    scales: torch.Tensor                  # [nblk, N] float16 or uint8
    scales16: torch.Tensor                # [nblk, N] float16
    w8: Optional[torch.Tensor] = None     # [K, N] int8
    sw8: Optional[torch.Tensor] = None    # [N] float16
    ratio16: Optional[torch.Tensor] = None  # [nblk, N] float16 (W4A8)

    @property
    def weight_bytes(self) -> int:
        return self.wp.numel() * 4 + self.scales.numel() * self.scales.element_size()


def to_device(pw: PackedWeight, device="cuda", w4a8: bool = False) -> DeviceWeight:
    dev = torch.device(device)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    dw = DeviceWeight(N=pw.N, K=pw.K, nblk=pw.nblk, split=pw.split, scale_fmt=pw.scale_fmt, inv=pw.inv,
                      wp=t(pw.wp.view(np.int32)), scales=t(pw.scales), scales16=t(pw.scales16))
    if pw.w8 is not None:
        dw.w8 = t(pw.w8)
        dw.sw8 = t(pw.sw8)
        if w4a8 and pw.sw_f32 is not None and pw.sc_f32 is not None:
            dw.ratio16 = t(w4a8_ratio(pw.sc_f32, pw.sw_f32))
    return dw


# ------------------------------------------------------------------ workspace
class _Workspaces:
    """Zero-filled scratch per (device, stream, use), grown on demand (never on
    a hot path once warmed up: the same size is reused).

    Each use has its own buffer: the GEMV workspace begins with arrival
    counters that every GEMV leaves at zero for the next one, so no other
    kernel may write it (the W4A16 GEMM's f32 -> f16 staging has its own)."""

    def __init__(self):
        self._lock = threading.Lock()
        self._bufs: dict = {}

    def get(self, device: torch.device, stream: int, nbytes: int, use: str = "gemv") -> torch.Tensor:
        key = (device.index, stream, use)
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
                self._bufs[key] = buf
            return buf


WORKSPACES = _Workspaces()


# ----------------------------------------------------------------------- ops
def gemv_workspace_bytes(M: int, N: int, K: int, split: int = 0) -> int:
    return int(L.load().g4b_gemv_workspace_bytes(M, N, K, split))


def gemv_i4(x: torch.Tensor, w: DeviceWeight, split: int = 0, out: Optional[torch.Tensor] = None,
            out_dtype: torch.dtype = torch.float32, stream: Optional[torch.cuda.Stream] = None,
            workspace: Optional[torch.Tensor] = None, pdl: bool = False) -> torch.Tensor:
    """y = x @ dequant(W).T for x [K] or [M, K] (M <= 8 per kernel; larger M loops).

    pdl=True launches with programmatic dependent launch (g4b_gemv_i4_ex,
    G4B_GEMV_PDL): only valid when the previous kernel on the stream does not
    write this layer's packed weights or scales."""
    _need(x, "x")
    squeeze = x.dim() == 1
    x2 = x.view(1, -1) if squeeze else x
    M, K = x2.shape
    if K != w.K:
        raise ValueError(f"gemv_i4: x has K={K}, weight has K={w.K}")
    if out is None:
        out = torch.empty((M, w.N), dtype=out_dtype, device=x.device)
    _need(out, "out")
    sh = _stream_handle(stream, x.device)
    lib = L.load()
    need = lib.g4b_gemv_workspace_bytes(M, w.N, w.K, split)
    ws = workspace
    if need and ws is None:
        ws = WORKSPACES.get(x.device, sh, need)
    L.check("g4b_gemv_i4", lib.g4b_gemv_i4_ex(
        _ptr(x2), _DT[x2.dtype], M, _ptr(w.wp), _ptr(w.scales), w.scale_fmt, w.inv,
        _ptr(out), _DT[out.dtype], w.N, w.K, split, _ptr(ws), ws.numel() if ws is not None else 0,
        L.GEMV_PDL if pdl else 0, sh))
    return out.view(-1) if squeeze else out


def gemv_fused_workspace_bytes(Ns, K: int) -> int:
    arr = (ctypes.c_int * len(Ns))(*Ns)
    return int(L.load().g4b_gemv_fused_workspace_bytes(len(Ns), arr, K))


def gemv_i4_fused(x: torch.Tensor, ws_: list, outs: Optional[list] = None, out_dtype: torch.dtype = torch.float32,
                  stream: Optional[torch.cuda.Stream] = None, workspace: Optional[torch.Tensor] = None,
                  pdl: bool = False) -> list:
    """Up to three GEMVs on one x [K] in one launch (q/k/v, gate/up):
    returns [W_i x for each weight].  All weights share K and the scale format."""
    _need(x, "x")
    if not 1 <= len(ws_) <= 3:
        raise ValueError("gemv_i4_fused: 1 to 3 weights")
    K = x.numel()
    fmt = ws_[0].scale_fmt
    if any(w.K != K or w.scale_fmt != fmt for w in ws_):
        raise ValueError("gemv_i4_fused: weights must share K and the scale format")
    if outs is None:
        outs = [torch.empty((w.N,), dtype=out_dtype, device=x.device) for w in ws_]
    for o in outs:
        _need(o, "out")
    if any(o.dtype != outs[0].dtype for o in outs):
        raise ValueError("gemv_i4_fused: all outputs must share one dtype")
    sh = _stream_handle(stream, x.device)
    lib = L.load()
    need = gemv_fused_workspace_bytes([w.N for w in ws_], K)
    ws = workspace
    if need and ws is None:
        ws = WORKSPACES.get(x.device, sh, need)
    segs = (L.GemvSegment * len(ws_))(*[L.GemvSegment(_ptr(w.wp), _ptr(w.scales), w.inv, _ptr(o), w.N)
                                         for w, o in zip(ws_, outs)])
    L.check("g4b_gemv_i4_fused", lib.g4b_gemv_i4_fused(
        _ptr(x), _DT[x.dtype], len(ws_), ctypes.cast(segs, ctypes.c_void_p), fmt, _DT[outs[0].dtype], K,
        _ptr(ws), ws.numel() if ws is not None else 0, L.GEMV_PDL if pdl else 0, sh))
    return outs


class GemvChain:
    """A recorded chain of M = 1 GEMV steps run as one persistent launch
    (g4b_gemv_chain_*): the engine's per-token command buffer of gemv()
    dispatches with a barrier after each.  Each step is (x, [weights], [outs])
    or (x, [weights], [outs], flags): 1 to 3 GEMVs that read x; a step may read
    any earlier step's output.  Tensor parallel: with `exchange` (a
    g4b.comm.PeerBuffers of exchange_bytes(steps, world) bytes), a step flagged
    L.CHAIN_ALLREDUCE (one weight) has its output summed over the ranks inside
    the launch, and the next step (x = None) reads that sum as its x.
    The tensors named in the steps must stay alive while the chain is used;
    `run` reads their current contents on every call.

    `xforms` (one rank only): one entry per step, None or a dict with "kind"
    ("rmsnorm", "normadd" or "gelu_mul") and the tensors "a", "b", "w",
    "w_post", "h_out" and floats "scale", "eps" that kind uses
    (g4b_chain_xform): the element-wise work between the GEMVs, fused into the
    step's activation load; such a step's x may be None."""

    @staticmethod
    def exchange_bytes(steps: list, world: int) -> int:
        return sum(8 * world * st[1][0].N for st in steps if len(st) > 3 and st[3] & L.CHAIN_ALLREDUCE)

    _XF_KINDS = {"rmsnorm": L.XF_RMSNORM, "normadd": L.XF_NORMADD, "gelu_mul": L.XF_GELU_MUL}

    def __init__(self, steps: list, device: Optional[torch.device] = None, exchange=None,
                 xforms: Optional[list] = None, x_dtype: Optional[torch.dtype] = None):
        if not steps:
            raise ValueError("GemvChain: no steps")
        if xforms is not None and (len(xforms) != len(steps) or exchange is not None):
            raise ValueError("GemvChain: one xform (or None) per step, and none with an exchange")
        self.lib = L.load()
        x0, w0, o0 = steps[0][:3]
        fused = [xforms is not None and xforms[j] is not None for j in range(len(steps))]
        if x0 is None and not fused[0]:
            raise ValueError("GemvChain: the first step needs its x")
        xdt = x_dtype if x_dtype is not None else (x0.dtype if x0 is not None else None)
        if xdt is None:
            raise ValueError("GemvChain: give x_dtype when the first step's x is fused")
        self.device = (x0.device if x0 is not None else o0[0].device) if device is None else device
        self._keep = []
        arr = (L.GemvChainStep * len(steps))()
        fmt = w0[0].scale_fmt
        prev_flags = 0
        for j, st in enumerate(steps):
            x, ws_, outs = st[:3]
            flags = st[3] if len(st) > 3 else 0
            if not 1 <= len(ws_) <= 3 or len(outs) != len(ws_):
                raise ValueError(f"GemvChain: step {j} needs 1 to 3 weights and one output per weight")
            if x is None:
                if not (prev_flags & L.CHAIN_ALLREDUCE or fused[j]):
                    raise ValueError(f"GemvChain: step {j} has no x and does not follow an all-reduced step")
                K = ws_[0].K
            else:
                _need(x, "x")
                if x.dtype != xdt:
                    raise ValueError("GemvChain: all steps share the x dtype")
                K = x.numel()
            if any(o.dtype != o0[0].dtype for o in outs):
                raise ValueError("GemvChain: all steps share the output dtype")
            if any(w.K != K or w.scale_fmt != fmt for w in ws_):
                raise ValueError(f"GemvChain: step {j} weights must have K = x.numel() and one scale format")
            for o in outs:
                _need(o, "out")
            arr[j].x = _ptr(x) if x is not None else None
            arr[j].K = K
            arr[j].nseg = len(ws_)
            arr[j].flags = flags
            for i, (w, o) in enumerate(zip(ws_, outs)):
                arr[j].seg[i] = L.GemvSegment(_ptr(w.wp), _ptr(w.scales), w.inv, _ptr(o), w.N)
            self._keep.append((x, ws_, outs))
            prev_flags = flags
        h = ctypes.c_void_p()
        if xforms is not None:
            xa = (L.ChainXform * len(steps))()
            for j, f in enumerate(xforms):
                if f is None:
                    continue
                xa[j].kind = self._XF_KINDS[f["kind"]]
                for key in ("a", "b", "w", "w_post", "h_out"):
                    t = f.get(key)
                    if t is not None:
                        _need(t, key)
                        setattr(xa[j], key, _ptr(t))
                xa[j].scale = float(f.get("scale", 1.0))
                xa[j].eps = float(f.get("eps", 1e-6))
            self._keep.append(xforms)
            L.check("g4b_gemv_chain_create_fused", self.lib.g4b_gemv_chain_create_fused(
                ctypes.cast(arr, ctypes.c_void_p), ctypes.cast(xa, ctypes.c_void_p), len(steps), _DT[xdt], fmt,
                _DT[o0[0].dtype], ctypes.byref(h)))
        elif exchange is None:
            L.check("g4b_gemv_chain_create", self.lib.g4b_gemv_chain_create(
                ctypes.cast(arr, ctypes.c_void_p), len(steps), _DT[xdt], fmt, _DT[o0[0].dtype],
                ctypes.byref(h)))
        else:
            self._keep.append(exchange)
            L.check("g4b_gemv_chain_create_tp", self.lib.g4b_gemv_chain_create_tp(
                ctypes.cast(arr, ctypes.c_void_p), len(steps), _DT[xdt], fmt, _DT[o0[0].dtype],
                exchange.ptrs.data_ptr(), exchange.rank, exchange.world, exchange.nbytes, ctypes.byref(h)))
        self.handle = h.value
        self.nsteps = len(steps)
        self.workspace_bytes = int(self.lib.g4b_gemv_chain_workspace_bytes(self.handle))
        self.workspace = torch.zeros(self.workspace_bytes + 256, dtype=torch.uint8, device=self.device)

    def run(self, stream: Optional[torch.cuda.Stream] = None, pdl: bool = False) -> None:
        """pdl: launch as a programmatic dependent of the previous kernel on the stream
        (G4B_CHAIN_RUN_PDL): the weights stream while that kernel finishes."""
        if self.handle is None:
            raise RuntimeError("GemvChain: closed")
        sh = _stream_handle(stream, self.device)
        L.check("g4b_gemv_chain_run", self.lib.g4b_gemv_chain_run_ex(
            self.handle, _ptr(self.workspace), self.workspace.numel(), L.CHAIN_RUN_PDL if pdl else 0, sh))

    def close(self) -> None:
        if getattr(self, "handle", None) is not None:
            self.lib.g4b_gemv_chain_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gemm_i4_workspace_bytes(M: int, N: int, K: int, x_dtype: torch.dtype = torch.float16) -> int:
    """Workspace g4b_gemm_i4 can use: the f16 copy of an f32 X, plus the split-K
    partials of a small-M GEMM (batched decode)."""
    return int(L.load().g4b_gemm_i4_workspace_bytes(M, N, K, _DT[x_dtype]))


def gemm_i4(X: torch.Tensor, w: DeviceWeight, out: Optional[torch.Tensor] = None,
            out_dtype: torch.dtype = torch.float16, stream: Optional[torch.cuda.Stream] = None,
            workspace: Optional[torch.Tensor] = None, pdl: bool = False) -> torch.Tensor:
    """W4A16 prefill GEMM: Y[M, N] = X[M, K] @ dequant(W) with f16 block scales
    (gmm()'s f16 path: cast_dn -> coopgemm_i4h -> cast_up).  pdl: launch as a
    programmatic dependent of the previous kernel (G4B_GEMM_PDL)."""
    _need(X, "X")
    M, K = X.shape
    if K != w.K:
        raise ValueError(f"gemm_i4: X has K={K}, weight has K={w.K}")
    if out is None:
        out = torch.empty((M, w.N), dtype=out_dtype, device=X.device)
    _need(out, "out")
    sh = _stream_handle(stream, X.device)
    lib = L.load()
    need = lib.g4b_gemm_i4_workspace_bytes(M, w.N, w.K, _DT[X.dtype])
    ws = workspace
    if need and ws is None:
        ws = WORKSPACES.get(X.device, sh, need, use="gemm_i4")
    L.check("g4b_gemm_i4", lib.g4b_gemm_i4_ex(
        _ptr(X), _DT[X.dtype], _ptr(w.wp), _ptr(w.scales16), _ptr(out), _DT[out.dtype], M, w.N, w.K,
        _ptr(ws), ws.numel() if ws is not None else 0, L.GEMM_PDL if pdl else 0, sh))
    return out


def gemm_i4_fused(X: torch.Tensor, ws_: list, outs: Optional[list] = None, out_dtype: torch.dtype = torch.float16,
                  stream: Optional[torch.cuda.Stream] = None, workspace: Optional[torch.Tensor] = None,
                  pdl: bool = False) -> list:
    """2-3 W4A16 GEMMs on one X [M <= 64, K] as one launch (a decode batch's q|k|v or gate|up):
    returns [X @ dequant(W_g)] for the weights in ws_."""
    _need(X, "X")
    M, K = X.shape
    if not 1 <= len(ws_) <= 3 or any(w.K != K for w in ws_):
        raise ValueError("gemm_i4_fused: 1 to 3 weights with X's K")
    if outs is None:
        outs = [torch.empty((M, w.N), dtype=out_dtype, device=X.device) for w in ws_]
    for o in outs:
        _need(o, "out")
    segs = (L.GemmSeg * len(ws_))()
    for g, (w, o) in enumerate(zip(ws_, outs)):
        segs[g].wp, segs[g].scales_f16, segs[g].y, segs[g].N = _ptr(w.wp), _ptr(w.scales16), _ptr(o), w.N
    sh = _stream_handle(stream, X.device)
    lib = L.load()
    need = lib.g4b_gemm_i4_workspace_bytes(M, sum(w.N for w in ws_), K, _DT[X.dtype])
    ws = workspace
    if need and ws is None:
        ws = WORKSPACES.get(X.device, sh, need, use="gemm_i4")
    L.check("g4b_gemm_i4_fused", lib.g4b_gemm_i4_fused(
        _ptr(X), _DT[X.dtype], M, K, ctypes.cast(segs, ctypes.c_void_p), len(ws_), _DT[outs[0].dtype], _ptr(ws),
        ws.numel() if ws is not None else 0, L.GEMM_PDL if pdl else 0, sh))
    return outs


def gemm_w8a8(A8: torch.Tensor, sa: torch.Tensor, w: DeviceWeight, out: Optional[torch.Tensor] = None,
              out_dtype: torch.dtype = torch.float16, acc: Optional[torch.Tensor] = None,
              stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """W8A8 prefill GEMM (PREFILL_I8): Y = f16((A8 @ W8) * sa[m] * sw[n]).

    A8 [M, K] int8 and sa [M] f32 come from cast_i8; the weight's int8 W8
    [K, N] and f16 sw8 [N] come from quant(..., prefill_i8=True).  acc, if
    given ([M, N] int32), receives the exact int32 accumulators."""
    _need(A8, "A8")
    _need(sa, "sa")
    if w.w8 is None or w.sw8 is None:
        raise ValueError("gemm_w8a8: weight was packed without prefill_i8 (no int8 weights)")
    M, K = A8.shape
    if K != w.K or A8.dtype != torch.int8:
        raise ValueError(f"gemm_w8a8: A8 must be int8 [M, {w.K}], got {tuple(A8.shape)} {A8.dtype}")
    if out is None:
        out = torch.empty((M, w.N), dtype=out_dtype, device=A8.device)
    _need(out, "out")
    if acc is not None:
        _need(acc, "acc")
    L.check("g4b_gemm_w8a8", L.load().g4b_gemm_w8a8(
        _ptr(A8), _ptr(w.w8), _ptr(sa), _ptr(w.sw8), _ptr(out), _DT[out.dtype], _ptr(acc), M, w.N, w.K,
        _stream_handle(stream, A8.device)))
    return out


def gemm_w4a8(A8: torch.Tensor, sa: torch.Tensor, w: DeviceWeight, out: Optional[torch.Tensor] = None,
              out_dtype: torch.dtype = torch.float16, acc: Optional[torch.Tensor] = None,
              stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """W4A8 prefill GEMM: the int4 weights requantised in the kernel to int8
    against the per-column scale (ratio16 = f16(scale / s_w)), then as gemm_w8a8."""
    _need(A8, "A8")
    _need(sa, "sa")
    if w.ratio16 is None or w.sw8 is None:
        raise ValueError("gemm_w4a8: weight has no W4A8 ratio (to_device(..., w4a8=True))")
    M, K = A8.shape
    if K != w.K or A8.dtype != torch.int8:
        raise ValueError(f"gemm_w4a8: A8 must be int8 [M, {w.K}], got {tuple(A8.shape)} {A8.dtype}")
    if out is None:
        out = torch.empty((M, w.N), dtype=out_dtype, device=A8.device)
    _need(out, "out")
    if acc is not None:
        _need(acc, "acc")
    L.check("g4b_gemm_w4a8", L.load().g4b_gemm_w4a8(
        _ptr(A8), _ptr(w.wp), _ptr(w.ratio16), _ptr(sa), _ptr(w.sw8), _ptr(out), _DT[out.dtype], _ptr(acc),
        M, w.N, w.K, _stream_handle(stream, A8.device)))
    return out


def reduce_partials(partial: torch.Tensor, split: int, out: Optional[torch.Tensor] = None,
                    stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    _need(partial, "partial")
    N = partial.numel() // split
    if out is None:
        out = torch.empty((N,), dtype=torch.float32, device=partial.device)
    L.check("g4b_reduce_partials", L.load().g4b_reduce_partials(
        _ptr(partial), _ptr(out), N, split, _stream_handle(stream, partial.device)))
    return out


def dequant_i4(w: DeviceWeight, out_dtype: torch.dtype = torch.float16,
               stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    out = torch.empty((w.K, w.N), dtype=out_dtype, device=w.wp.device)
    L.check("g4b_dequant_i4", L.load().g4b_dequant_i4(
        _ptr(w.wp), _ptr(w.scales), w.scale_fmt, w.inv, _ptr(out), _DT[out_dtype], w.N, w.K,
        _stream_handle(stream, out.device)))
    return out


def cast(x: torch.Tensor, dtype: torch.dtype, out: Optional[torch.Tensor] = None,
         stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    _need(x, "x")
    if out is None:
        out = torch.empty(x.shape, dtype=dtype, device=x.device)
    L.check("g4b_cast", L.load().g4b_cast(_ptr(x), _DT[x.dtype], _ptr(out), _DT[out.dtype], x.numel(),
                                          _stream_handle(stream, x.device)))
    return out


def cast_i8(X: torch.Tensor, stream: Optional[torch.cuda.Stream] = None):
    """Per-token int8 quantisation -> (A8 [M, K] int8, sa [M] f32)."""
    _need(X, "X")
    M, K = X.shape
    A8 = torch.empty((M, K), dtype=torch.int8, device=X.device)
    sa = torch.empty((M,), dtype=torch.float32, device=X.device)
    L.check("g4b_cast_i8", L.load().g4b_cast_i8(_ptr(X), _DT[X.dtype], _ptr(A8), _ptr(sa), M, K,
                                                _stream_handle(stream, X.device)))
    return A8, sa


def stream_wait(stream: Optional[torch.cuda.Stream] = None, timeout_ms: int = 0) -> None:
    """Bounded wait for a stream (the engine's fence wait with a timeout)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    L.check("g4b_stream_wait", L.load().g4b_stream_wait(_stream_handle(stream, dev), int(timeout_ms)))


# ----------------------------------------------------------------- decode attention
def attn_workspace_bytes(nH: int, nkv: int, hd: int, max_T: int) -> int:
    return int(L.load().g4b_attn_workspace_bytes(nH, nkv, hd, max_T))


def attn_prepkv(qkv: torch.Tensor, knw: torch.Tensor, cos_t: torch.Tensor, sin_t: torch.Tensor, kc: torch.Tensor,
                vc: torch.Tensor, pos: torch.Tensor, nkv: int, hd: int, koff: int, voff: int, keqv: bool = False,
                window: int = 0, stream: Optional[torch.cuda.Stream] = None) -> None:
    """vk/prepkv.comp: this token's normed, rotated k and normed v into the f16 caches
    kc / vc [nkv, stride, hd] at slot pos (pos % window for a sliding ring).
    pos is a one-element int32 device tensor."""
    for t, n in ((qkv, "qkv"), (knw, "knw"), (cos_t, "cos"), (sin_t, "sin"), (kc, "kc"), (vc, "vc"), (pos, "pos")):
        _need(t, n)
    stride = kc.shape[1]
    sh = _stream_handle(stream, qkv.device)
    L.check("g4b_attn_prepkv", L.load().g4b_attn_prepkv(
        _ptr(qkv), _DT[qkv.dtype], _ptr(knw), _ptr(cos_t), _ptr(sin_t), _ptr(kc), _ptr(vc), nkv, hd, koff, voff,
        1 if keqv else 0, stride, window, _ptr(pos), sh))


def attn_decode(qkv: torch.Tensor, qnw: torch.Tensor, cos_t: torch.Tensor, sin_t: torch.Tensor, kc: torch.Tensor,
                vc: torch.Tensor, pos: torch.Tensor, nH: int, nkv: int, hd: int, qoff: int = 0, window: int = 0,
                out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float32,
                stream: Optional[torch.cuda.Stream] = None, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """vk/attn.comp: one token's attention over the cached keys (flash decoding)."""
    for t, n in ((qkv, "qkv"), (qnw, "qnw"), (cos_t, "cos"), (sin_t, "sin"), (kc, "kc"), (vc, "vc"), (pos, "pos")):
        _need(t, n)
    stride = kc.shape[1]
    if out is None:
        out = torch.empty((nH * hd,), dtype=out_dtype, device=qkv.device)
    sh = _stream_handle(stream, qkv.device)
    need = attn_workspace_bytes(nH, nkv, hd, window if window > 0 else stride)
    ws = workspace
    if need and ws is None:
        ws = WORKSPACES.get(qkv.device, sh, need, use="attn")
    L.check("g4b_attn_decode", L.load().g4b_attn_decode(
        _ptr(qkv), _DT[qkv.dtype], _ptr(qnw), _ptr(cos_t), _ptr(sin_t), _ptr(kc), _ptr(vc), _ptr(out),
        _DT[out.dtype], nH, nkv, hd, qoff, stride, window, _ptr(pos), _ptr(ws), ws.numel() if ws is not None else 0,
        sh))
    return out


def attn_decode_prepkv(qkv: torch.Tensor, qnw: torch.Tensor, knw: torch.Tensor, cos_t: torch.Tensor,
                       sin_t: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor, pos: torch.Tensor, nH: int, nkv: int,
                       hd: int, koff: int, voff: int, keqv: bool = False, qoff: int = 0, window: int = 0,
                       out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float32,
                       stream: Optional[torch.cuda.Stream] = None,
                       workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """vk/prepkv.comp then vk/attn.comp in one launch: this token's k / v into the caches, then its
    attention over them."""
    for t, n in ((qkv, "qkv"), (qnw, "qnw"), (knw, "knw"), (cos_t, "cos"), (sin_t, "sin"), (kc, "kc"), (vc, "vc"),
                 (pos, "pos")):
        _need(t, n)
    stride = kc.shape[1]
    if out is None:
        out = torch.empty((nH * hd,), dtype=out_dtype, device=qkv.device)
    sh = _stream_handle(stream, qkv.device)
    need = attn_workspace_bytes(nH, nkv, hd, window if window > 0 else stride)
    ws = workspace
    if need and ws is None:
        ws = WORKSPACES.get(qkv.device, sh, need, use="attn")
    L.check("g4b_attn_decode_prepkv", L.load().g4b_attn_decode_prepkv(
        _ptr(qkv), _DT[qkv.dtype], _ptr(qnw), _ptr(knw), _ptr(cos_t), _ptr(sin_t), _ptr(kc), _ptr(vc), _ptr(out),
        _DT[out.dtype], nH, nkv, hd, qoff, koff, voff, 1 if keqv else 0, stride, window, _ptr(pos), _ptr(ws),
        ws.numel() if ws is not None else 0, sh))
    return out


def attn_prefill_prepkv(k: torch.Tensor, v: torch.Tensor, knw: torch.Tensor, cosM: torch.Tensor, sinM: torch.Tensor,
                        kc: torch.Tensor, vc: torch.Tensor, p0: torch.Tensor, nkv: int, hd: int, window: int = 0,
                        stream: Optional[torch.cuda.Stream] = None) -> None:
    """vk/pre_prepkv.comp: a chunk's k / v rows ([M, row] views, head h at h * hd; v may be k) into the
    f16 caches at slots p0 .. p0 + M - 1 (% window); cosM / sinM [M, hd] are the tokens' rotations.
    p0 is a one-element int32 device tensor."""
    for t, n in ((knw, "knw"), (cosM, "cosM"), (sinM, "sinM"), (kc, "kc"), (vc, "vc"), (p0, "p0")):
        _need(t, n)
    if k.dim() != 2 or k.shape != v.shape or k.stride(1) != 1 or v.stride(0) != k.stride(0) or k.dtype != v.dtype:
        raise ValueError("attn_prefill_prepkv: k and v must be [M, row] views with the same row stride and dtype")
    sh = _stream_handle(stream, k.device)
    L.check("g4b_attn_prefill_prepkv", L.load().g4b_attn_prefill_prepkv(
        _ptr(k), _ptr(v), _DT[k.dtype], k.stride(0), k.shape[0], _ptr(knw), _ptr(cosM), _ptr(sinM), _ptr(kc),
        _ptr(vc), nkv, hd, kc.shape[1], window, _ptr(p0), sh))


def attn_prefill(q: torch.Tensor, qnw: torch.Tensor, cosM: torch.Tensor, sinM: torch.Tensor, kc: torch.Tensor,
                 vc: torch.Tensor, p0: torch.Tensor, nH: int, nkv: int, hd: int, window: int = 0,
                 out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float32,
                 stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """vk/pre_attn.comp: causal attention of a chunk's queries q [M, row] (head h at h * hd) over the
    cache; returns out [M, nH * hd] (or writes the given [M, row] view)."""
    for t, n in ((qnw, "qnw"), (cosM, "cosM"), (sinM, "sinM"), (kc, "kc"), (vc, "vc"), (p0, "p0")):
        _need(t, n)
    if q.dim() != 2 or q.stride(1) != 1:
        raise ValueError("attn_prefill: q must be an [M, row] view")
    M = q.shape[0]
    if out is None:
        out = torch.empty((M, nH * hd), dtype=out_dtype, device=q.device)
    if out.dim() != 2 or out.stride(1) != 1 or out.shape[0] != M:
        raise ValueError("attn_prefill: out must be an [M, row] view")
    sh = _stream_handle(stream, q.device)
    L.check("g4b_attn_prefill", L.load().g4b_attn_prefill(
        _ptr(q), _DT[q.dtype], q.stride(0), M, _ptr(qnw), _ptr(cosM), _ptr(sinM), _ptr(kc), _ptr(vc), _ptr(out),
        _DT[out.dtype], out.stride(0), nH, nkv, hd, kc.shape[1], window, _ptr(p0), sh))
    return out


# ----------------------------------------------------------------- prefill element-wise rows
def rows_rmsnorm(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
                 out_dtype: Optional[torch.dtype] = None, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """vk/pre_norm.comp over the rows of x [M, D]: x * rsqrt(mean(x^2) + 1e-6) * w."""
    _need(x, "x")
    _need(w, "w")
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    M, D = x.shape
    L.check("g4b_rows_rmsnorm", L.load().g4b_rows_rmsnorm(
        _ptr(x), _DT[x.dtype], _ptr(w), _ptr(out), _DT[out.dtype], M, D, _stream_handle(stream, x.device)))
    return out


def rows_normadd(x: torch.Tensor, w: torch.Tensor, h: torch.Tensor, scl: float = 1.0,
                 stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """vk/pre_na.comp over the rows of x [M, D]: h = (h + rmsnorm(x) * w) * scl, in place (h f32)."""
    for t, n in ((x, "x"), (w, "w"), (h, "h")):
        _need(t, n)
    M, D = x.shape
    L.check("g4b_rows_normadd", L.load().g4b_rows_normadd(
        _ptr(x), _DT[x.dtype], _ptr(w), _ptr(h), M, D, float(scl), _stream_handle(stream, x.device)))
    return h


def gelumul(gate: torch.Tensor, up: torch.Tensor, out: Optional[torch.Tensor] = None,
            out_dtype: Optional[torch.dtype] = None, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """vk/gelumul.comp: gelu_tanh(gate) * up, element-wise."""
    _need(gate, "gate")
    _need(up, "up")
    if gate.dtype != up.dtype or gate.numel() != up.numel():
        raise ValueError("gelumul: gate and up must match in dtype and size")
    if out is None:
        out = torch.empty(gate.shape, dtype=out_dtype or gate.dtype, device=gate.device)
    L.check("g4b_gelumul", L.load().g4b_gelumul(
        _ptr(gate), _ptr(up), _DT[gate.dtype], _ptr(out), _DT[out.dtype], gate.numel(),
        _stream_handle(stream, gate.device)))
    return out
