"""numpy front end of the C oracle (``g4b_oracle.c``). Test infrastructure only."""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(HERE, "libg4b_oracle.so")
_lib = None

BLK = 32

__all__ = [
    "lib", "build", "f16_to_f32", "f32_to_f16", "e4m3_decode", "e4m3_encode",
    "quant_i4", "fp8_scales", "split_for", "w8a8_weights", "w4a8_ratio", "gemv", "reduce",
    "dequant", "gemm_i4", "cast_i8", "gemm_w8a8", "w4a8_requant", "gemm_w4a8",
    "num_threads", "set_num_threads", "pack_reference", "rmsnorm", "normadd", "gelumul", "decode_token",
    "attn_prepkv", "attn_decode", "attn_prefill_prepkv", "attn_prefill",
]


def build(force: bool = False) -> str:
    """Compile the oracle shared object with its Makefile (gcc + OpenMP)."""
    if force or not os.path.exists(_LIB_PATH) or \
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(HERE, "g4b_oracle.c")):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        P = C.c_void_p
        i = C.c_int
        f = C.c_float
        L.orc_f16_to_f32.restype = f; L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_f32_to_f16.restype = C.c_uint16; L.orc_f32_to_f16.argtypes = [f]
        L.orc_e4m3_decode.restype = f; L.orc_e4m3_decode.argtypes = [C.c_uint8]
        L.orc_e4m3_encode.restype = C.c_uint8; L.orc_e4m3_encode.argtypes = [f]
        L.orc_quant_i4.argtypes = [P, i, i, P, P, P, P]
        L.orc_fp8_scales.restype = C.c_double; L.orc_fp8_scales.argtypes = [P, i, i, P]
        L.orc_split.restype = i; L.orc_split.argtypes = [i, i]
        L.orc_w8a8_weights.argtypes = [P, P, i, i, P, P, P]
        L.orc_w4a8_ratio.argtypes = [P, P, i, i, P]
        L.orc_gemv.argtypes = [P, i, P, P, i, f, i, i, i, P, P]
        L.orc_reduce.argtypes = [P, P, i, i]
        L.orc_dequant.argtypes = [P, P, i, f, i, i, P]
        L.orc_gemm_i4.argtypes = [P, P, P, i, i, i, P]
        L.orc_cast_i8.argtypes = [P, i, i, P, P]
        L.orc_gemm_w8a8.argtypes = [P, P, P, P, i, i, i, P, P]
        L.orc_w4a8_requant.argtypes = [P, P, i, i, P]
        L.orc_gemm_w4a8.argtypes = [P, P, P, P, P, i, i, i, P, P]
        L.orc_rmsnorm.argtypes = [P, P, P, i, f]
        L.orc_normadd.argtypes = [P, P, P, i, f, f]
        L.orc_gelumul.argtypes = [P, P, P, i]
        L.orc_attn_prepkv.argtypes = [P, P, P, P, P, P, i, i, i, i, i, i, i, i]
        L.orc_attn_decode.argtypes = [P, P, P, P, P, P, P, i, i, i, i, i, i, i]
        L.orc_attn_prefill_prepkv.argtypes = [P, P, P, P, P, P, P, i, i, i, i, i, i, i]
        L.orc_attn_prefill.argtypes = [P, P, P, P, P, P, P, i, i, i, i, i, i, i, i]
        L.orc_num_threads.restype = i
        L.orc_set_num_threads.argtypes = [i]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


def f16_to_f32(h) -> np.ndarray:
    h = _c(h, np.uint16)
    f = np.vectorize(lambda v: lib().orc_f16_to_f32(int(v)), otypes=[np.float32])
    return f(h) if h.size else h.astype(np.float32)


def f32_to_f16(x) -> np.ndarray:
    x = _c(x, np.float32)
    f = np.vectorize(lambda v: lib().orc_f32_to_f16(float(v)), otypes=[np.uint16])
    return f(x) if x.size else x.astype(np.uint16)


def e4m3_decode(b) -> np.ndarray:
    b = _c(b, np.uint8)
    return np.vectorize(lambda v: lib().orc_e4m3_decode(int(v)), otypes=[np.float32])(b)


def e4m3_encode(x) -> np.ndarray:
    x = _c(x, np.float32)
    return np.vectorize(lambda v: lib().orc_e4m3_encode(float(v)), otypes=[np.uint8])(x)


def quant_i4(W):
    """src/vk_engine.py:126-131 -> (wp [K, N/8] u32, sc [N, nblk] f32, q [N, K] u8, sc16 [nblk, N] u16)."""
    W = _c(W, np.float32)
    N, K = W.shape
    nblk = K // BLK
    sc = np.empty((N, nblk), np.float32)
    q = np.empty((N, K), np.uint8)
    wp = np.empty((K, N // 8), np.uint32)
    sc16 = np.empty((nblk, N), np.uint16)
    lib().orc_quant_i4(_p(W), N, K, _p(sc), _p(q), _p(wp), _p(sc16))
    return wp, sc, q, sc16


def fp8_scales(sc):
    """src/vk_engine.py:133-137 -> (e8 [nblk, N] u8, inv)."""
    sc = _c(sc, np.float32)
    N, nblk = sc.shape
    e8 = np.empty((nblk, N), np.uint8)
    inv = lib().orc_fp8_scales(_p(sc), N, nblk, _p(e8))
    return e8, float(inv)


def split_for(N: int, nblk: int) -> int:
    return lib().orc_split(int(N), int(nblk))


def w8a8_weights(q, sc):
    """src/vk_engine.py:152-157 -> (w8t [K, N] i8, sw16 [N] u16, sw_f32 [N])."""
    q = _c(q, np.uint8)
    sc = _c(sc, np.float32)
    N, K = q.shape
    w8t = np.empty((K, N), np.int8)
    sw16 = np.empty((N,), np.uint16)
    swf = np.empty((N,), np.float32)
    lib().orc_w8a8_weights(_p(q), _p(sc), N, K, _p(w8t), _p(sw16), _p(swf))
    return w8t, sw16, swf


def w4a8_ratio(sc, sw_f32):
    sc = _c(sc, np.float32)
    swf = _c(sw_f32, np.float32)
    N, nblk = sc.shape
    r = np.empty((nblk, N), np.uint16)
    lib().orc_w4a8_ratio(_p(sc), _p(swf), N, nblk, _p(r))
    return r


def gemv(x, wp, scales, fmt: int, inv: float, N: int, K: int, split: int, want_partial=False):
    """vk/gemv.comp + reduce.comp.  x: [K] or [M, K] f32. Returns y ([N] or [M, N] f32)."""
    x = _c(x, np.float32)
    squeeze = x.ndim == 1
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    wp = _c(wp, np.uint32)
    scales = _c(scales, np.uint16 if fmt == 0 else np.uint8)
    y = np.empty((M, N), np.float32)
    part = np.empty((split, M, N), np.float32) if want_partial else None
    lib().orc_gemv(_p(x2), M, _p(wp), _p(scales), int(fmt), float(inv), N, K, int(split), _p(part), _p(y))
    y = y[0] if squeeze else y
    return (y, part) if want_partial else y


def reduce(partial, N: int, split: int):
    partial = _c(partial, np.float32)
    y = np.empty((N,), np.float32)
    lib().orc_reduce(_p(partial), _p(y), N, split)
    return y


def dequant(wp, scales, fmt: int, inv: float, N: int, K: int):
    """fmt 0 -> [K, N] f16 bits (u16); fmt 1 -> [K, N] f32."""
    wp = _c(wp, np.uint32)
    scales = _c(scales, np.uint16 if fmt == 0 else np.uint8)
    out = np.empty((K, N), np.uint16 if fmt == 0 else np.float32)
    lib().orc_dequant(_p(wp), _p(scales), int(fmt), float(inv), N, K, _p(out))
    return out


def gemm_i4(X16, wp, sc16, M: int, N: int, K: int):
    X16 = _c(X16, np.uint16)
    Y = np.empty((M, N), np.float32)
    lib().orc_gemm_i4(_p(X16), _p(_c(wp, np.uint32)), _p(_c(sc16, np.uint16)), M, N, K, _p(Y))
    return Y


def cast_i8(X):
    X = _c(X, np.float32)
    M, K = X.shape
    A8 = np.empty((M, K), np.int8)
    sa = np.empty((M,), np.float32)
    lib().orc_cast_i8(_p(X), M, K, _p(A8), _p(sa))
    return A8, sa


def gemm_w8a8(A8, W8, sa, sw16):
    A8 = _c(A8, np.int8)
    W8 = _c(W8, np.int8)
    M, K = A8.shape
    N = W8.shape[1]
    Cm = np.empty((M, N), np.int32)
    Y16 = np.empty((M, N), np.uint16)
    lib().orc_gemm_w8a8(_p(A8), _p(W8), _p(_c(sa, np.float32)), _p(_c(sw16, np.uint16)), M, N, K,
                        _p(Cm), _p(Y16))
    return Cm, Y16


def w4a8_requant(wp, ratio16, N: int, K: int):
    w8 = np.empty((K, N), np.int8)
    lib().orc_w4a8_requant(_p(_c(wp, np.uint32)), _p(_c(ratio16, np.uint16)), N, K, _p(w8))
    return w8


def gemm_w4a8(A8, wp, ratio16, sa, sw16, N: int):
    A8 = _c(A8, np.int8)
    M, K = A8.shape
    Cm = np.empty((M, N), np.int32)
    Y16 = np.empty((M, N), np.uint16)
    lib().orc_gemm_w4a8(_p(A8), _p(_c(wp, np.uint32)), _p(_c(ratio16, np.uint16)),
                        _p(_c(sa, np.float32)), _p(_c(sw16, np.uint16)), M, N, K, _p(Cm), _p(Y16))
    return Cm, Y16


def pack_reference(W, fp8: bool = False, prefill_i8: bool = False):
    """The whole of quant() (src/vk_engine.py:125-159) through the C restatement.

    Returns a dict with the same fields the reference returns: wp, scales (raw
    bytes as the shader reads them), scales16, split, nblk, inv, w8, sw8."""
    W = _c(W, np.float32)
    N, K = W.shape
    nblk = K // BLK
    wp, sc, q, sc16 = quant_i4(W)
    out = {"wp": wp, "scales16": sc16, "split": split_for(N, nblk), "nblk": nblk, "inv": 1.0,
           "sc_f32": sc, "q": q}
    if fp8:
        e8, inv = fp8_scales(sc)
        out["scales"] = e8
        out["inv"] = inv
    else:
        out["scales"] = sc16
    if prefill_i8:
        w8t, sw16, swf = w8a8_weights(q, sc)
        out["w8"] = w8t
        out["sw8"] = sw16
        out["sw_f32"] = swf
    return out


# ---------------------------------------------------------------- decode-layer element-wise ops
def rmsnorm(x, w, eps: float = 1e-6):
    """vk/rmsnorm.comp:8-12 (f32)."""
    x = _c(x, np.float32)
    w = _c(w, np.float32)
    y = np.empty_like(x)
    lib().orc_rmsnorm(_p(x), _p(w), _p(y), x.size, float(eps))
    return y


def normadd(x, w, h, sc: float = 1.0, eps: float = 1e-6):
    """vk/normadd.comp:8-12: returns (h + rmsnorm(x) * w) * sc (f32); h is not modified."""
    x = _c(x, np.float32)
    w = _c(w, np.float32)
    out = np.array(h, dtype=np.float32, copy=True)
    lib().orc_normadd(_p(x), _p(w), _p(out), x.size, float(sc), float(eps))
    return out


def gelumul(gate, up):
    """vk/gelumul.comp:7-8 (f32)."""
    g = _c(gate, np.float32)
    u = _c(up, np.float32)
    out = np.empty_like(g)
    lib().orc_gelumul(_p(g), _p(u), _p(out), g.size)
    return out


def decode_token(h0, layers, lm_head, final_w, gemv_fn, round_x=None, round_y=None, eps: float = 1e-6):
    """One decode token's weight path in the engine's dispatch order
    (src/vk_engine.py:277-287) with attention left out: per layer rmsnorm ->
    q|k|v -> o (on q, standing in for the attention output) -> normadd ->
    rmsnorm -> gate|up -> gelumul -> down -> normadd; then rmsnorm -> lm_head.

    layers: dicts with the packed weights "q", "k", "v", "o", "gate", "up",
    "down" (anything gemv_fn takes) and the f32 norm weights "inw", "paw",
    "pfw", "ofw" and layer scalar "scl".  gemv_fn(x, w) -> f32 y.  round_x /
    round_y round a GEMV's input / output to the dtype the device chain keeps
    them in (None: f32).  Returns (logits, final residual h, per-layer outputs)."""
    rx = round_x or (lambda v: np.asarray(v, np.float32))
    ry = round_y or (lambda v: np.asarray(v, np.float32))
    h = np.asarray(h0, np.float32).copy()
    outs = []
    for L in layers:
        x = rx(rmsnorm(h, L["inw"], eps))
        q, k, v = (ry(gemv_fn(x, L[n])) for n in ("q", "k", "v"))
        o = ry(gemv_fn(rx(q), L["o"]))
        h = normadd(o, L["paw"], h, 1.0, eps)
        x2 = rx(rmsnorm(h, L["pfw"], eps))
        gate, up = ry(gemv_fn(x2, L["gate"])), ry(gemv_fn(x2, L["up"]))
        act = rx(gelumul(gate, up))
        down = ry(gemv_fn(act, L["down"]))
        h = normadd(down, L["ofw"], h, L.get("scl", 1.0), eps)
        outs.append({"q": q, "k": k, "v": v, "o": o, "gate": gate, "up": up, "down": down})
    logits = ry(gemv_fn(rx(rmsnorm(h, final_w, eps)), lm_head))
    return logits, h, outs


# ---------------------------------------------------------------- decode attention
def attn_prepkv(qkv, knw, cos_t, sin_t, kc, vc, nkv: int, hd: int, koff: int, voff: int, keqv: bool,
                window: int, pos: int):
    """vk/prepkv.comp:14-31 on host arrays: writes slot pos (pos % window) of kc / vc
    ([nkv, stride, hd] uint16 f16 bits) in place."""
    qkv = _c(qkv, np.float32)
    assert kc.dtype == np.uint16 and vc.dtype == np.uint16 and kc.flags.c_contiguous and vc.flags.c_contiguous
    lib().orc_attn_prepkv(_p(qkv), _p(_c(knw, np.float32)), _p(_c(cos_t, np.float32)), _p(_c(sin_t, np.float32)),
                          _p(kc), _p(vc), nkv, hd, koff, voff, 1 if keqv else 0, kc.shape[1], window, pos)


def attn_decode(qkv, qnw, cos_t, sin_t, kc, vc, nH: int, nkv: int, hd: int, qoff: int, window: int, pos: int):
    """vk/attn.comp:15-55 on host arrays: the [nH * hd] f32 attention output."""
    out = np.empty((nH * hd,), np.float32)
    lib().orc_attn_decode(_p(_c(qkv, np.float32)), _p(_c(qnw, np.float32)), _p(_c(cos_t, np.float32)),
                          _p(_c(sin_t, np.float32)), _p(_c(kc, np.uint16)), _p(_c(vc, np.uint16)), _p(out), nH, nkv,
                          hd, qoff, kc.shape[1], window, pos)
    return out


def attn_prefill_prepkv(k, v, knw, cosM, sinM, kc, vc, nkv: int, hd: int, window: int, p0: int):
    """vk/pre_prepkv.comp:15-30 on host arrays: k, v [M, row] f32 (v may be k), cosM / sinM [M, hd];
    writes slots p0 .. p0 + M - 1 (% window) of kc / vc ([nkv, stride, hd] uint16 f16 bits) in place."""
    k = _c(k, np.float32)
    v = _c(v, np.float32)
    assert k.shape == v.shape and k.ndim == 2
    assert kc.dtype == np.uint16 and vc.dtype == np.uint16 and kc.flags.c_contiguous and vc.flags.c_contiguous
    lib().orc_attn_prefill_prepkv(_p(k), _p(v), _p(_c(knw, np.float32)), _p(_c(cosM, np.float32)),
                                  _p(_c(sinM, np.float32)), _p(kc), _p(vc), k.shape[0], nkv, hd, k.shape[1],
                                  kc.shape[1], window, p0)


def attn_prefill(q, qnw, cosM, sinM, kc, vc, nH: int, nkv: int, hd: int, window: int, p0: int):
    """vk/pre_attn.comp:16-53 on host arrays: q [M, row] f32 -> the [M, row] f32 attention output
    (columns beyond nH * hd are zero)."""
    q = _c(q, np.float32)
    assert q.ndim == 2 and q.shape[1] >= nH * hd
    out = np.zeros_like(q)
    lib().orc_attn_prefill(_p(q), _p(_c(qnw, np.float32)), _p(_c(cosM, np.float32)), _p(_c(sinM, np.float32)),
                           _p(_c(kc, np.uint16)), _p(_c(vc, np.uint16)), _p(out), q.shape[0], nH, nkv, hd, q.shape[1],
                           kc.shape[1], window, p0)
    return out
