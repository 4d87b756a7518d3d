"""g4b.decode.token_plan on CPU: the fused decode token's step layout (which
GEMVs each step runs, what element-wise work its activation load does, and
how the residual buffers alternate), without a GPU."""
from g4b import decode


class W:
    def __init__(self, name, N, K):
        self.name, self.N, self.K = name, N, K


def _layer(i):
    return type("L", (), {n: W(f"{n}{i}", 8, 8) for n in ("q", "k", "v", "o", "gate", "up", "down")})()


def test_token_plan_layout():
    layers = [_layer(i) for i in range(3)]
    norms = [decode.LayerNorms(inw=f"inw{i}", paw=f"paw{i}", pfw=f"pfw{i}", ofw=f"ofw{i}", scl=0.5 + i)
             for i in range(3)]
    bufs = {k: k for k in ("h0", "hA", "hB", "q", "k", "v", "o", "gate", "up", "down", "logits")}
    steps, xf, final = decode.token_plan(layers, norms, W("lm", 8, 8), "finw", bufs)
    assert len(steps) == len(xf) == 4 * 3 + 1
    kinds = [None if f is None else f["kind"] for f in xf]
    assert kinds == ["rmsnorm", None, "normadd", "gelu_mul"] + ["normadd", None, "normadd", "gelu_mul"] * 2 + \
        ["normadd"]
    # the first norm reads the input hidden state; o reads q; down reads gelu(gate) * up
    assert xf[0]["a"] == "h0" and xf[0]["w"] == "inw0"
    for li in range(3):
        b = 4 * li
        assert [w.name for w in steps[b][1]] == [f"q{li}", f"k{li}", f"v{li}"]
        assert steps[b + 1][0] == "q" and steps[b + 1][1][0].name == f"o{li}"
        g = xf[b + 2]
        assert (g["a"], g["w_post"], g["w"], g["scale"]) == ("o", f"paw{li}", f"pfw{li}", 1.0)
        assert (xf[b + 3]["a"], xf[b + 3]["b"]) == ("gate", "up")
        if li:
            q = xf[b]
            assert (q["a"], q["w_post"], q["w"], q["scale"]) == ("down", f"ofw{li - 1}", f"inw{li}", 0.5 + li - 1)
    last = xf[-1]
    assert (last["a"], last["w_post"], last["w"], last["scale"]) == ("down", "ofw2", "finw", 2.5)
    # every normadd reads the residual the one before wrote, writes the other buffer, never the input
    adds = [f for f in xf if f is not None and f["kind"] == "normadd"]
    assert adds[0]["b"] == "h0"
    for p, n in zip(adds, adds[1:]):
        assert n["b"] == p["h_out"] and n["h_out"] != n["b"]
    assert all(f["h_out"] in ("hA", "hB") for f in adds) and final == adds[-1]["h_out"]


def test_layer_segments_split_at_attention():
    """layer_segments: segment 0 = layer 0's q|k|v; segment l+1 = o on the
    attention buffer, gate|up, down, then the next layer's q|k|v (lm_head after
    the last layer); the element-wise work matches token_plan's."""
    layers = [_layer(i) for i in range(3)]
    norms = [decode.LayerNorms(inw=f"inw{i}", paw=f"paw{i}", pfw=f"pfw{i}", ofw=f"ofw{i}", scl=0.5 + i)
             for i in range(3)]
    bufs = {k: k for k in ("h0", "hA", "hB", "q", "k", "v", "attn", "o", "gate", "up", "down", "logits")}
    segs, final = decode.layer_segments(layers, norms, W("lm", 8, 8), "finw", bufs)
    assert len(segs) == 4
    assert [w.name for w in segs[0][0][0][1]] == ["q0", "k0", "v0"] and segs[0][1][0]["a"] == "h0"
    for li in range(3):
        steps, xf = segs[li + 1]
        assert steps[0][0] == "attn" and steps[0][1][0].name == f"o{li}" and xf[0] is None
        assert [st[1][0].name for st in steps[1:]] == [f"gate{li}", f"down{li}", f"q{li + 1}" if li < 2 else "lm"]
        assert [f["kind"] for f in xf[1:]] == ["normadd", "gelu_mul", "normadd"]
    # the flat plan and the split plan do the same element-wise work in the same order
    tsteps, txf, tfinal = decode.token_plan(layers, norms, W("lm", 8, 8), "finw", bufs)
    flat = [f for _, xf in segs for f in xf]
    assert [None if f is None else (f["kind"], f.get("w"), f.get("w_post"), f.get("b"), f.get("h_out")) for f in flat] == \
        [None if f is None else (f["kind"], f.get("w"), f.get("w_post"), f.get("b"), f.get("h_out")) for f in txf]
    assert final == tfinal
