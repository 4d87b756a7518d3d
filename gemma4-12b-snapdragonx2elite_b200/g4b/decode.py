"""One decode token's weight path as one fused GEMV-chain launch (one GPU).

The engine records, per layer (src/vk_engine.py:277-287):

    rmsnorm -> q, k, v GEMVs -> attention -> o GEMV -> normadd ->
    rmsnorm -> gate, up GEMVs -> gelumul -> down GEMV -> normadd,

then rmsnorm -> lm_head, each a dispatch with a barrier after it.  Here the
whole token, attention excepted, is ONE g4b_gemv_chain launch
(g4b_gemv_chain_create_fused): every element-wise dispatch is fused into the
activation load of the GEMV step after it --

    q|k|v  x = rmsnorm(h, input_layernorm)              (layer 0: of the input h)
           or x = rmsnorm(h' = normadd(down, post_feedforward_layernorm, h), input_layernorm)
    o      x = q                       (attention is outside this path: o reads q in its place)
    gate|up x = rmsnorm(h' = normadd(o, post_attention_layernorm, h), pre_feedforward_layernorm)
    down   x = gelu_tanh(gate) * up
    lm_head x = rmsnorm(h' = normadd(down, post_feedforward_layernorm, h), final norm)

-- so a token is 4 steps per layer plus lm_head, 193 for the 48-layer model,
and the residual h is carried in two f32 buffers that alternate.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

from . import ops

EPS = 1e-6  # vk/rmsnorm.comp:11, vk/normadd.comp:11


@dataclass
class LayerNorms:
    """A layer's f32 norm weights [hidden] and layer scalar (src/vk_engine.py:196-205)."""
    inw: torch.Tensor     # input_layernorm            (before q|k|v)
    paw: torch.Tensor     # post_attention_layernorm   (normadd after o)
    pfw: torch.Tensor     # pre_feedforward_layernorm  (before gate|up)
    ofw: torch.Tensor     # post_feedforward_layernorm (normadd after down)
    scl: float = 1.0      # layer_scalar (vk/normadd.comp's d.y)


def token_plan(layers, norms: List[LayerNorms], lm_head, final_w, bufs: dict, eps: float = EPS):
    """The chain steps and their element-wise work for one token.

    layers: objects with the packed weights q, k, v, o, gate, up, down;
    bufs: "h0" (the input hidden state, f32), "hA", "hB" (f32 residuals) and
    the outputs "q", "k", "v", "o", "gate", "up", "down", "logits" in the
    chain's dtype.  Returns (steps, xforms, final residual buffer name)."""
    steps, xf = [], []
    cur = "h0"                       # the residual entering the next normadd

    def nxt(name):
        return "hB" if name == "hA" else "hA"

    prev_ofw, prev_scl = None, 1.0
    for li, (Ly, nm) in enumerate(zip(layers, norms)):
        if li == 0:
            f = {"kind": "rmsnorm", "a": bufs["h0"], "w": nm.inw, "eps": eps}
        else:
            out = nxt(cur)
            f = {"kind": "normadd", "a": bufs["down"], "b": bufs[cur], "w_post": prev_ofw, "w": nm.inw,
                 "h_out": bufs[out], "scale": prev_scl, "eps": eps}
            cur = out
        steps.append((None, [Ly.q, Ly.k, Ly.v], [bufs["q"], bufs["k"], bufs["v"]]))
        xf.append(f)
        steps.append((bufs["q"], [Ly.o], [bufs["o"]]))
        xf.append(None)
        out = nxt(cur)
        steps.append((None, [Ly.gate, Ly.up], [bufs["gate"], bufs["up"]]))
        xf.append({"kind": "normadd", "a": bufs["o"], "b": bufs[cur], "w_post": nm.paw, "w": nm.pfw,
                   "h_out": bufs[out], "scale": 1.0, "eps": eps})
        cur = out
        steps.append((None, [Ly.down], [bufs["down"]]))
        xf.append({"kind": "gelu_mul", "a": bufs["gate"], "b": bufs["up"]})
        prev_ofw, prev_scl = nm.ofw, nm.scl
    out = nxt(cur)
    steps.append((None, [lm_head], [bufs["logits"]]))
    xf.append({"kind": "normadd", "a": bufs["down"], "b": bufs[cur], "w_post": prev_ofw, "w": final_w,
               "h_out": bufs[out], "scale": prev_scl, "eps": eps})
    return steps, xf, out


class FusedDecodeToken:
    """A token's GEMVs and element-wise work as one launch on one GPU.

    dtype is the activations' and outputs' dtype (f16 or f32); the residual
    and the norm weights are f32, as in the engine.  Write the token's hidden
    state into `h0`, call run(), read `logits` (and `h`, the final residual)."""

    def __init__(self, layers, norms: List[LayerNorms], lm_head, final_w: torch.Tensor,
                 dtype: torch.dtype = torch.float16, eps: float = EPS, device: Optional[torch.device] = None):
        dev = device or lm_head.wp.device
        H = layers[0].q.K
        L0 = layers[0]
        z = lambda n, dt: torch.zeros(n, dtype=dt, device=dev)  # noqa: E731
        self.bufs = {"h0": z(H, torch.float32), "hA": z(H, torch.float32), "hB": z(H, torch.float32),
                     "q": z(L0.q.N, dtype), "k": z(L0.k.N, dtype), "v": z(L0.v.N, dtype), "o": z(L0.o.N, dtype),
                     "gate": z(L0.gate.N, dtype), "up": z(L0.up.N, dtype), "down": z(L0.down.N, dtype),
                     "logits": z(lm_head.N, dtype)}
        steps, xf, self._hname = token_plan(layers, norms, lm_head, final_w, self.bufs, eps)
        self._keep = (layers, norms, lm_head, final_w)
        self.chain = ops.GemvChain(steps, xforms=xf, x_dtype=dtype, device=dev)
        self.nsteps = len(steps)

    @property
    def h0(self) -> torch.Tensor:
        return self.bufs["h0"]

    @property
    def logits(self) -> torch.Tensor:
        return self.bufs["logits"]

    @property
    def h(self) -> torch.Tensor:
        return self.bufs[self._hname]

    def run(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        self.chain.run(stream)

    def close(self) -> None:
        self.chain.close()


def layer_segments(layers, norms: List[LayerNorms], lm_head, final_w, bufs: dict, eps: float = EPS):
    """The same token split at every layer's attention, for an engine that runs
    attention itself: segment 0 is layer 0's q|k|v; segment l + 1 starts with
    layer l's o on bufs["attn"] (the attention output, written between the
    segments) and runs gate|up, down and then layer l + 1's q|k|v -- or, after
    the last layer, lm_head.  Returns ([(steps, xforms)], final residual name)."""
    segs = []
    cur = "h0"

    def nxt(name):
        return "hB" if name == "hA" else "hA"

    L0, n0 = layers[0], norms[0]
    segs.append(([(None, [L0.q, L0.k, L0.v], [bufs["q"], bufs["k"], bufs["v"]])],
                 [{"kind": "rmsnorm", "a": bufs["h0"], "w": n0.inw, "eps": eps}]))
    for li, (Ly, nm) in enumerate(zip(layers, norms)):
        steps, xf = [(bufs["attn"], [Ly.o], [bufs["o"]])], [None]
        out = nxt(cur)
        steps.append((None, [Ly.gate, Ly.up], [bufs["gate"], bufs["up"]]))
        xf.append({"kind": "normadd", "a": bufs["o"], "b": bufs[cur], "w_post": nm.paw, "w": nm.pfw,
                   "h_out": bufs[out], "scale": 1.0, "eps": eps})
        cur = out
        steps.append((None, [Ly.down], [bufs["down"]]))
        xf.append({"kind": "gelu_mul", "a": bufs["gate"], "b": bufs["up"]})
        out = nxt(cur)
        if li + 1 < len(layers):
            Ln, nn = layers[li + 1], norms[li + 1]
            steps.append((None, [Ln.q, Ln.k, Ln.v], [bufs["q"], bufs["k"], bufs["v"]]))
            xf.append({"kind": "normadd", "a": bufs["down"], "b": bufs[cur], "w_post": nm.ofw, "w": nn.inw,
                       "h_out": bufs[out], "scale": nm.scl, "eps": eps})
        else:
            steps.append((None, [lm_head], [bufs["logits"]]))
            xf.append({"kind": "normadd", "a": bufs["down"], "b": bufs[cur], "w_post": nm.ofw, "w": final_w,
                       "h_out": bufs[out], "scale": nm.scl, "eps": eps})
        cur = out
        segs.append((steps, xf))
    return segs, cur


class SegmentedDecodeToken:
    """A token as one fused chain launch per layer, split at attention.

    run(stream, attention) launches segment 0, then for every layer calls
    attention(layer, stream) -- which must read bufs "qkv" (q, k and v one
    after another) and write bufs["attn"] ([q width], the chain's dtype) on
    that stream, e.g. g4b.ops.attn_prepkv + attn_decode -- and launches the
    next segment.  Buffers as FusedDecodeToken's, plus "qkv" and "attn"."""

    def __init__(self, layers, norms: List[LayerNorms], lm_head, final_w: torch.Tensor,
                 dtype: torch.dtype = torch.float16, eps: float = EPS, device: Optional[torch.device] = None):
        dev = device or lm_head.wp.device
        H = layers[0].q.K
        L0 = layers[0]
        z = lambda n, dt: torch.zeros(n, dtype=dt, device=dev)  # noqa: E731
        # q, k and v are views of one q|k|v buffer, as the engine's B["qkv"] (src/vk_engine.py:180): the
        # KV-cache write and the attention read k and v at offsets into it
        qkv = z(L0.q.N + L0.k.N + L0.v.N, dtype)
        self.bufs = {"h0": z(H, torch.float32), "hA": z(H, torch.float32), "hB": z(H, torch.float32),
                     "qkv": qkv, "q": qkv[:L0.q.N], "k": qkv[L0.q.N:L0.q.N + L0.k.N], "v": qkv[L0.q.N + L0.k.N:],
                     "attn": z(L0.o.K, dtype), "o": z(L0.o.N, dtype), "gate": z(L0.gate.N, dtype),
                     "up": z(L0.up.N, dtype), "down": z(L0.down.N, dtype), "logits": z(lm_head.N, dtype)}
        segs, self._hname = layer_segments(layers, norms, lm_head, final_w, self.bufs, eps)
        self._keep = (layers, norms, lm_head, final_w)
        self.chains = [ops.GemvChain(st, xforms=xf, x_dtype=dtype, device=dev) for st, xf in segs]

    @property
    def h0(self) -> torch.Tensor:
        return self.bufs["h0"]

    @property
    def logits(self) -> torch.Tensor:
        return self.bufs["logits"]

    def run(self, stream: Optional[torch.cuda.Stream], attention, pdl: bool = True) -> None:
        """pdl: each segment after the first is a programmatic dependent of the attention before it, so
        its weights start streaming while attention runs (G4B_CHAIN_RUN_PDL); the results are the same."""
        self.chains[0].run(stream)
        for li, ch in enumerate(self.chains[1:]):
            attention(li, stream)
            ch.run(stream, pdl=pdl)

    def close(self) -> None:
        for ch in self.chains:
            ch.close()
