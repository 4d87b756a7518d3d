"""Decode attention (g4b_attn_prepkv, g4b_attn_decode) against the CPU oracle of
vk/prepkv.comp and vk/attn.comp, through the C ABI.

Every case fills the f16 caches with earlier tokens' keys and values, writes
this token's k and v with prepkv (and checks that slot against the oracle's
and that no other slot moved), then runs attention and compares it with the
oracle run on the very cache contents the device holds.  Floating-point bar:
tests/util.py (max relative error 1e-2, cosine >= 0.9999), with the attention
outputs' denominator floor util.ATTN_GUARD (1e-2 x rms: a score's last-bit
rounding moves an output that cancels to near zero by ~1e-5 x rms) and the
k / v slots' the default 1e-3 x rms (their rsqrt differs in the last bits,
which can move an f16 rounding)."""
import numpy as np
import pytest
import torch

import oracle as O
from g4b import _lib as L
from g4b import ops
from util import ATTN_GUARD, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rope(hd, pos, theta=10000.0):
    inv = 1.0 / theta ** (np.arange(0, hd, 2, dtype=np.float64) / hd)
    ang = np.concatenate([pos * inv, pos * inv])
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def _case(nH, nkv, hd, stride, window, pos, keqv, dtype, seed):
    rng = np.random.default_rng(seed)
    nq, nk = nH * hd, nkv * hd
    qkv = rng.standard_normal(nq + 2 * nk).astype(np.float32)
    if dtype == torch.float16:
        qkv = qkv.astype(np.float16).astype(np.float32)          # the values the device sees
    knw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    qnw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kc = rng.standard_normal((nkv, stride, hd)).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((nkv, stride, hd)).astype(np.float16).view(np.uint16)
    cos_t, sin_t = _rope(hd, pos)
    t = lambda a, dt=None: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    dev = dict(qkv=t(qkv).to(dtype), knw=t(knw), qnw=t(qnw), kc=t(kc.view(np.int16)), vc=t(vc.view(np.int16)),
               cos=t(cos_t), sin=t(sin_t), pos=torch.tensor([pos], dtype=torch.int32, device=DEV))
    host = dict(qkv=qkv, knw=knw, qnw=qnw, kc=kc.copy(), vc=vc.copy(), cos=cos_t, sin=sin_t)
    return dev, host


@pytest.mark.parametrize("nH,nkv,hd,stride,window,pos,keqv,dtype", [
    (16, 8, 256, 4096, 0, 0, False, torch.float32),        # first token: one key
    (16, 8, 256, 4096, 0, 17, False, torch.float32),
    (16, 8, 256, 4096, 0, 4095, False, torch.float16),     # full cache, f16 q|k|v
    (16, 8, 256, 1024, 1024, 3000, False, torch.float32),  # sliding ring: slot = pos % window, T = window
    (16, 8, 256, 1024, 1024, 300, True, torch.float32),    # k = v (attention_k_eq_v)
    (4, 2, 512, 2048, 0, 1500, False, torch.float32),      # head_dim 512, 2 query heads per KV head
    (8, 1, 128, 512, 0, 200, False, torch.float16),        # 8 query heads per KV head
])
def test_attention_matches_oracle(nH, nkv, hd, stride, window, pos, keqv, dtype):
    dev, host = _case(nH, nkv, hd, stride, window, pos, keqv, dtype, seed=pos + hd + nH)
    nq, nk = nH * hd, nkv * hd
    koff, voff = nq, nq + nk
    kc_before = dev["kc"].clone()
    ops.attn_prepkv(dev["qkv"], dev["knw"], dev["cos"], dev["sin"], dev["kc"], dev["vc"], dev["pos"], nkv, hd, koff,
                    voff, keqv=keqv, window=window)
    O.attn_prepkv(host["qkv"], host["knw"], host["cos"], host["sin"], host["kc"], host["vc"], nkv, hd, koff, voff,
                  keqv, window, pos)
    torch.cuda.synchronize()
    slot = pos % window if window else pos
    kd = dev["kc"].cpu().numpy().view(np.uint16)
    vd = dev["vc"].cpu().numpy().view(np.uint16)
    f = lambda u: u.view(np.float16).astype(np.float32)  # noqa: E731
    assert_close(f(kd[:, slot]), f(host["kc"][:, slot]), "prepkv k slot")
    assert_close(f(vd[:, slot]), f(host["vc"][:, slot]), "prepkv v slot")
    others = np.ones(stride, bool)
    others[slot] = False
    assert np.array_equal(kd[:, others], kc_before.cpu().numpy().view(np.uint16)[:, others])
    # attention on exactly the cache the device holds
    for out_dtype in (torch.float32, torch.float16):
        out = ops.attn_decode(dev["qkv"], dev["qnw"], dev["cos"], dev["sin"], dev["kc"], dev["vc"], dev["pos"], nH,
                              nkv, hd, qoff=0, window=window, out_dtype=out_dtype)
        torch.cuda.synchronize()
        ref = O.attn_decode(host["qkv"], host["qnw"], host["cos"], host["sin"], kd, vd, nH, nkv, hd, 0, window, pos)
        assert_close(out.float().cpu().numpy(), ref, f"attn nH={nH} nkv={nkv} hd={hd} pos={pos} window={window}",
                     guard=ATTN_GUARD)
    assert L.query(L.Q_KERNEL_STATUS) == 0


@pytest.mark.parametrize("nH,nkv,hd,stride,window,pos,keqv,dtype", [
    (16, 8, 256, 4096, 0, 0, False, torch.float32),
    (16, 8, 256, 4096, 0, 3000, False, torch.float16),
    (16, 8, 256, 1024, 1024, 3000, True, torch.float32),   # ring, k = v
    (4, 2, 512, 2048, 0, 1500, False, torch.float32),
    (8, 1, 128, 512, 0, 200, False, torch.float16),
])
def test_fused_prepkv_attention_matches_oracle(nH, nkv, hd, stride, window, pos, keqv, dtype):
    """g4b_attn_decode_prepkv: the cache write and the attention in one launch give what the oracle's
    prepkv then attention give."""
    dev, host = _case(nH, nkv, hd, stride, window, pos, keqv, dtype, seed=pos + 7 * hd + nH)
    nq, nk = nH * hd, nkv * hd
    kc_before = dev["kc"].clone()
    out = ops.attn_decode_prepkv(dev["qkv"], dev["qnw"], dev["knw"], dev["cos"], dev["sin"], dev["kc"], dev["vc"],
                                 dev["pos"], nH, nkv, hd, nq, nq + nk, keqv=keqv, window=window)
    O.attn_prepkv(host["qkv"], host["knw"], host["cos"], host["sin"], host["kc"], host["vc"], nkv, hd, nq, nq + nk,
                  keqv, window, pos)
    torch.cuda.synchronize()
    slot = pos % window if window else pos
    kd = dev["kc"].cpu().numpy().view(np.uint16)
    vd = dev["vc"].cpu().numpy().view(np.uint16)
    f = lambda u: u.view(np.float16).astype(np.float32)  # noqa: E731
    assert_close(f(kd[:, slot]), f(host["kc"][:, slot]), "fused prepkv k slot")
    assert_close(f(vd[:, slot]), f(host["vc"][:, slot]), "fused prepkv v slot")
    others = np.ones(stride, bool)
    others[slot] = False
    assert np.array_equal(kd[:, others], kc_before.cpu().numpy().view(np.uint16)[:, others])
    ref = O.attn_decode(host["qkv"], host["qnw"], host["cos"], host["sin"], kd, vd, nH, nkv, hd, 0, window, pos)
    assert_close(out.cpu().numpy(), ref, f"fused attn nH={nH} hd={hd} pos={pos} window={window}", guard=ATTN_GUARD)
    assert L.query(L.Q_KERNEL_STATUS) == 0


def test_attention_graph_follows_the_device_position():
    """One captured graph serves every token: the position is read from device
    memory at run time, so replays after updating it attend over more keys."""
    nH, nkv, hd, stride = 16, 8, 256, 2048
    dev, host = _case(nH, nkv, hd, stride, 0, 100, False, torch.float32, seed=7)
    nq, nk = nH * hd, nkv * hd
    s = torch.cuda.Stream()
    out = torch.empty(nH * hd, device=DEV)
    ws = torch.zeros(ops.attn_workspace_bytes(nH, nkv, hd, stride) + 256, dtype=torch.uint8, device=DEV)

    def token():
        ops.attn_prepkv(dev["qkv"], dev["knw"], dev["cos"], dev["sin"], dev["kc"], dev["vc"], dev["pos"], nkv, hd, nq,
                        nq + nk, stream=s)
        ops.attn_decode(dev["qkv"], dev["qnw"], dev["cos"], dev["sin"], dev["kc"], dev["vc"], dev["pos"], nH, nkv, hd,
                        out=out, stream=s, workspace=ws)

    with torch.cuda.stream(s):
        token()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            token()
    for pos in (100, 101, 1500):
        dev["pos"].fill_(pos)
        with torch.cuda.stream(s):
            g.replay()
        s.synchronize()
        kd = dev["kc"].cpu().numpy().view(np.uint16)
        vd = dev["vc"].cpu().numpy().view(np.uint16)
        ref = O.attn_decode(host["qkv"], host["qnw"], host["cos"], host["sin"], kd, vd, nH, nkv, hd, 0, 0, pos)
        assert_close(out.cpu().numpy(), ref, f"graph replay at pos {pos}", guard=ATTN_GUARD)
    del g
    assert L.query(L.Q_KERNEL_STATUS) == 0


def test_attention_rejects_unsupported_shapes():
    lib = L.load()
    z = torch.zeros(4096, device=DEV)
    p = torch.zeros(1, dtype=torch.int32, device=DEV)
    # 8 query heads per KV head at head_dim 512 is beyond the kernel's registers
    st = lib.g4b_attn_decode(z.data_ptr(), L.DT_F32, z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(),
                             z.data_ptr(), z.data_ptr(), L.DT_F32, 8, 1, 512, 0, 4, 0, p.data_ptr(), None, 0,
                             torch.cuda.current_stream().cuda_stream)
    assert st == L.G4B_E_SHAPE and "query heads" in L.last_error()


# ---------------------------------------------------------------- prefill (vk/pre_prepkv.comp, vk/pre_attn.comp)
def _rope_rows(hd, p0, M):
    rows = [_rope(hd, p0 + m) for m in range(M)]
    return np.stack([r[0] for r in rows]), np.stack([r[1] for r in rows])


@pytest.mark.parametrize("nH,nkv,hd,stride,window,p0,M,keqv,dtype", [
    (16, 8, 256, 4096, 0, 0, 300, False, torch.float32),      # a prompt's first chunk
    (16, 8, 256, 2048, 0, 1000, 128, False, torch.float16),   # a chunk after a cached prefix
    (16, 8, 256, 512, 512, 700, 200, False, torch.float32),   # sliding ring: wraps, future slots masked
    (4, 2, 128, 64, 64, 30, 100, True, torch.float32),        # chunk longer than the ring; k = v
    (4, 2, 512, 1024, 0, 100, 70, False, torch.float32),      # head_dim 512
    (8, 1, 128, 512, 0, 5, 77, False, torch.float16),         # 8 query heads per KV head
    (2, 2, 256, 256, 0, 40, 1, False, torch.float32),         # one token
])
def test_prefill_attention_matches_oracle(nH, nkv, hd, stride, window, p0, M, keqv, dtype):
    rng = np.random.default_rng(M + hd + p0)
    nq, nk = nH * hd, nkv * hd
    q = rng.standard_normal((M, nq)).astype(np.float32)
    k = rng.standard_normal((M, nk)).astype(np.float32)
    v = k if keqv else rng.standard_normal((M, nk)).astype(np.float32)
    if dtype == torch.float16:
        q, k, v = (a.astype(np.float16).astype(np.float32) for a in (q, k, v))
    knw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    qnw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kc = rng.standard_normal((nkv, stride, hd)).astype(np.float16).view(np.uint16)   # the cached prefix
    vc = rng.standard_normal((nkv, stride, hd)).astype(np.float16).view(np.uint16)
    cosM, sinM = _rope_rows(hd, p0, M)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    qd, kd_in, vd_in = t(q).to(dtype), t(k).to(dtype), t(v).to(dtype)
    if keqv:
        vd_in = kd_in
    kcd, vcd = t(kc.view(np.int16)), t(vc.view(np.int16))
    p0d = torch.tensor([p0], dtype=torch.int32, device=DEV)
    ops.attn_prefill_prepkv(kd_in, vd_in, t(knw), t(cosM), t(sinM), kcd, vcd, p0d, nkv, hd, window=window)
    O.attn_prefill_prepkv(k, v, knw, cosM, sinM, kc, vc, nkv, hd, window, p0)
    torch.cuda.synchronize()
    kd = kcd.cpu().numpy().view(np.uint16)
    vd = vcd.cpu().numpy().view(np.uint16)
    f = lambda u: u.view(np.float16).astype(np.float32)  # noqa: E731
    assert_close(f(kd), f(kc), "prefill prepkv k")
    assert_close(f(vd), f(vc), "prefill prepkv v")
    ref = O.attn_prefill(q, qnw, cosM, sinM, kd, vd, nH, nkv, hd, window, p0)
    for out_dtype in (torch.float32, torch.float16):
        out = ops.attn_prefill(qd, t(qnw), t(cosM), t(sinM), kcd, vcd, p0d, nH, nkv, hd, window=window,
                               out_dtype=out_dtype)
        torch.cuda.synchronize()
        assert_close(out.float().cpu().numpy(), ref, f"prefill attn nH={nH} hd={hd} p0={p0} M={M} window={window}",
                     guard=ATTN_GUARD)
    assert L.query(L.Q_KERNEL_STATUS) == 0


def test_prefill_attention_writes_into_row_views():
    """q and out as column slices of wider rows (the engine's q|k|v and attention buffers)."""
    nH, nkv, hd, stride, M, p0 = 4, 2, 256, 512, 50, 60
    rng = np.random.default_rng(3)
    row = nH * hd + 2 * nkv * hd
    qkv = torch.from_numpy(rng.standard_normal((M, row)).astype(np.float32)).to(DEV)
    kc = torch.from_numpy(rng.standard_normal((nkv, stride, hd)).astype(np.float16).view(np.int16)).to(DEV)
    vc = kc.clone()
    qnw = torch.ones(hd, device=DEV)
    cosM, sinM = (torch.from_numpy(a).to(DEV) for a in _rope_rows(hd, p0, M))
    p0d = torch.tensor([p0], dtype=torch.int32, device=DEV)
    wide = torch.full((M, nH * hd + 64), 7.0, device=DEV)
    ops.attn_prefill(qkv[:, :nH * hd], qnw, cosM, sinM, kc, vc, p0d, nH, nkv, hd, out=wide[:, :nH * hd])
    ref = ops.attn_prefill(qkv[:, :nH * hd].contiguous(), qnw, cosM, sinM, kc, vc, p0d, nH, nkv, hd)
    torch.cuda.synchronize()
    assert torch.equal(wide[:, :nH * hd], ref)
    assert bool((wide[:, nH * hd:] == 7.0).all())
