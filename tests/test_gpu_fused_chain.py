"""A decode token's GEMVs with the engine's element-wise dispatches fused into
one chain launch (g4b.decode.FusedDecodeToken, g4b_gemv_chain_create_fused),
against the CPU oracle run dispatch by dispatch in the engine's order
(oracle.decode_token: vk/rmsnorm.comp, vk/gemv.comp + vk/reduce.comp,
vk/normadd.comp, vk/gelumul.comp restated).  The device keeps activations in
the chain's dtype, so the oracle rounds each GEMV's input and output to it
too.  The sums of squares are formed in another order, so the result is not
bitwise.  Bar: cosine >= 0.9999 and max relative error <= 1e-2 (tests/util.py);
with f32 activations the denominator is max(|ref|, 1e-3 x rms), as for a single
GEMV.  With f16 activations every GEMV's input and output is rounded to f16 on
both sides, and a value that lands near a rounding midpoint may round the other
way: over two layers that moves an output by a couple of f16 ulps, so the
denominator is max(|ref|, rms) (an error bound relative to the vector's rms)."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from g4b import _lib as L
from g4b import decode, ops, pack
from util import assert_close

pytestmark = pytest.mark.gpu
H, NQ, NKV, FFN, VOCAB, LAYERS = 512, 512, 256, 1024, 2048, 2


def _model(fp8, seed=0):
    rng = np.random.default_rng(seed)
    host, dev, norms, dnorms = [], [], [], []
    shapes = {"q": (NQ, H), "k": (NKV, H), "v": (NKV, H), "o": (H, NQ), "gate": (FFN, H), "up": (FFN, H),
              "down": (H, FFN)}
    for li in range(LAYERS):
        hl = {n: pack.quant((rng.standard_normal(s) * 0.02).astype(np.float32), pf=False, fp8=fp8,
                            prefill_i8=False) for n, s in shapes.items()}
        nw = {k: (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32) for k in ("inw", "paw", "pfw", "ofw")}
        nw["scl"] = float(0.75 + 0.1 * li)
        host.append({**hl, **nw})
        dev.append(type("Layer", (), {n: ops.to_device(w, "cuda") for n, w in hl.items()})())
        dnorms.append(decode.LayerNorms(**{k: torch.from_numpy(nw[k]).cuda() for k in ("inw", "paw", "pfw", "ofw")},
                                        scl=nw["scl"]))
    lm = pack.quant((rng.standard_normal((VOCAB, H)) * 0.02).astype(np.float32), pf=False, fp8=fp8,
                    prefill_i8=False)
    finw = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    h0 = rng.standard_normal(H).astype(np.float32)
    return host, dev, dnorms, lm, finw, h0


def _oracle_gemv(x, pw):
    sc = pw.scales.view(np.uint16) if pw.scale_fmt == 0 else pw.scales
    return O.gemv(np.asarray(x, np.float32), pw.wp, sc, pw.scale_fmt, pw.inv, pw.N, pw.K, pw.split)


@pytest.mark.parametrize("dtype,fp8", [(torch.float16, False), (torch.float32, False), (torch.float16, True)])
def test_fused_token_matches_oracle(dtype, fp8):
    host, dev, dnorms, lm, finw, h0 = _model(fp8)
    tok = decode.FusedDecodeToken(dev, dnorms, ops.to_device(lm, "cuda"), torch.from_numpy(finw).cuda(),
                                  dtype=dtype)
    tok.h0.copy_(torch.from_numpy(h0))
    tok.run()
    torch.cuda.synchronize()
    assert L.query(L.Q_KERNEL_STATUS) == 0
    rnd = (lambda v: np.asarray(v, np.float32).astype(np.float16).astype(np.float32)) \
        if dtype == torch.float16 else None
    logits, h, outs = O.decode_token(h0, host, lm, finw, _oracle_gemv, round_x=rnd, round_y=rnd)
    what = f"fused token {dtype} {'e4m3' if fp8 else 'f16'} scales"
    guard = 1.0 if dtype == torch.float16 else 1e-3
    assert_close(tok.logits.float().cpu().numpy(), logits, f"{what}: logits", guard=guard)
    assert_close(tok.h.cpu().numpy(), h, f"{what}: final residual", guard=guard)
    # the last layer's intermediate outputs too
    for n in ("q", "o", "gate", "up", "down"):
        assert_close(tok.bufs[n].float().cpu().numpy(), outs[-1][n], f"{what}: {n}", guard=guard)
    tok.close()


def test_fused_token_repeat_and_graph_replay_are_identical():
    host, dev, dnorms, lm, finw, h0 = _model(False, seed=3)
    tok = decode.FusedDecodeToken(dev, dnorms, ops.to_device(lm, "cuda"), torch.from_numpy(finw).cuda(),
                                  dtype=torch.float16)
    tok.h0.copy_(torch.from_numpy(h0))
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        tok.run(s)
        first = tok.logits.clone()
        for _ in range(3):
            tok.run(s)
        again = tok.logits.clone()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            tok.run(s)
        g.replay()
        g.replay()
    s.synchronize()
    assert torch.equal(first, again) and torch.equal(first, tok.logits)
    assert L.query(L.Q_KERNEL_STATUS) == 0
    del g
    tok.close()


def test_fused_chain_rejects_a_norm_on_a_vector_the_step_before_did_not_write():
    """NORMADD's branch output must be the previous step's first output (its
    tile sums feed the norm); anything else is refused before any launch."""
    host, dev, dnorms, lm, finw, h0 = _model(False, seed=5)
    bufs = {k: torch.zeros(n, dtype=torch.float16, device="cuda") for k, n in
            (("q", NQ), ("k", NKV), ("v", NKV), ("o", H), ("gate", FFN), ("up", FFN), ("down", H),
             ("logits", VOCAB))}
    bufs.update({k: torch.zeros(H, device="cuda") for k in ("h0", "hA", "hB")})
    steps, xf, _ = decode.token_plan(dev, dnorms, ops.to_device(lm, "cuda"), torch.from_numpy(finw).cuda(), bufs)
    xf[2] = dict(xf[2], a=bufs["down"])          # gate|up normadd on a vector step 1 did not write
    before = L.query(L.Q_LAUNCHES)
    with pytest.raises(L.G4BError) as e:
        ops.GemvChain(steps, xforms=xf, x_dtype=torch.float16)
    assert e.value.code == L.G4B_E_ARG and "NORMADD" in str(e.value)
    assert L.query(L.Q_LAUNCHES) == before


@pytest.mark.parametrize("pdl", [False, True])
def test_segmented_token_equals_the_fused_token(pdl):
    """The token split at attention (one chain launch per layer, g4b.decode.SegmentedDecodeToken) with
    an attention stand-in that hands q on (what the fused token's o step reads) gives the fused token's
    bits: each step's partition and arithmetic are the same.  pdl: the segments are programmatic
    dependents of the kernel before them (G4B_CHAIN_RUN_PDL), eager and in a graph."""
    host, dev, dnorms, lm, finw, h0 = _model(False, seed=5)
    lmd = ops.to_device(lm, "cuda")
    fw = torch.from_numpy(finw).cuda()
    fused = decode.FusedDecodeToken(dev, dnorms, lmd, fw, dtype=torch.float16)
    seg = decode.SegmentedDecodeToken(dev, dnorms, lmd, fw, dtype=torch.float16)
    fused.h0.copy_(torch.from_numpy(h0))
    seg.h0.copy_(torch.from_numpy(h0))
    s = torch.cuda.Stream()

    def attention(li, stream):
        with torch.cuda.stream(stream):
            seg.bufs["attn"].copy_(seg.bufs["q"])

    with torch.cuda.stream(s):
        fused.run(s)
        seg.run(s, attention, pdl=pdl)
        eager = seg.logits.clone()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            seg.run(s, attention, pdl=pdl)
        seg.logits.zero_()
        g.replay()
    s.synchronize()
    assert L.query(L.Q_KERNEL_STATUS) == 0
    assert torch.equal(eager, fused.logits), (eager.float() - fused.logits.float()).abs().max()
    assert torch.equal(seg.logits, fused.logits)
    del g
    fused.close()
    seg.close()
