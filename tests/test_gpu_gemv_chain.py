"""GPU parity of the GEMV chain (g4b_gemv_chain_*): a recorded list of M = 1
GEMV steps run by one persistent launch, each step free to read what the steps
before it wrote (the engine's per-token command buffer of gemv() dispatches
with a barrier after each, src/vk_engine.py:254-290).

Bar: each step is within the GEMV tolerance of oracle/g4b_oracle.c on the x
the chain actually fed it; it matches the same step launched on its own
(g4b_gemv_i4 / g4b_gemv_i4_fused) up to f32 summation order (the chain may
split a step's k-chunks over its CTAs differently); and repeated runs of one
chain give identical bits.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from g4b import _lib as L
from g4b import ops, pack
from g4b import quant_gpu as qz
from util import activations, assert_close, weights

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _packed(N, K, seed, fp8=False, std=0.02):
    W = weights(N, K, seed, std)
    pw = pack.quant(W, fp8=fp8, prefill_i8=False)
    return pw, ops.to_device(pw, DEV)


def _oracle(pw, x32):
    sc = pw.scales.view(np.uint16) if pw.scale_fmt == 0 else pw.scales
    return O.gemv(x32, pw.wp, sc, pw.scale_fmt, pw.inv, pw.N, pw.K, pw.split)


def _layer_chain(layers, dt, H, Q, F, V, fp8, seed):
    """A decode-shaped chain with true dependencies: q|k|v on h, o on q,
    gate|up on o's output, down on gate, the next layer on down's output,
    lm_head last.  Returns (steps, packed weights per step, the input)."""
    packed, steps = [], []
    h = torch.from_numpy(activations(1, H, seed=seed)[0]).to(DEV).to(dt)
    x = h
    shapes = [[Q, Q // 2, Q // 2], [H], [F, F], [H]]
    for li in range(layers):
        for si, Ns in enumerate(shapes):
            K = x.numel()
            # std K^-1/2 keeps the activations near unit scale along the chain (f16 stays normal)
            ws = [_packed(N, K, seed=1000 * li + 10 * si + i, fp8=fp8, std=K ** -0.5) for i, N in enumerate(Ns)]
            outs = [torch.empty(N, dtype=dt, device=DEV) for N in Ns]
            steps.append((x, [w[1] for w in ws], outs))
            packed.append([w[0] for w in ws])
            x = outs[0]
    ws = [_packed(V, x.numel(), seed=77, fp8=fp8, std=x.numel() ** -0.5)]
    outs = [torch.empty(V, dtype=dt, device=DEV)]
    steps.append((x, [ws[0][1]], outs))
    packed.append([ws[0][0]])
    return steps, packed, h


def _assert_same_up_to_order(o, r, what):
    """Equal up to the order of the f32 split-K sums: f32 within 1e-5 relative
    (plus 1e-6 rms), f16 within one f16 rounding step."""
    o = o.float()
    r = r.float()
    rms = r.pow(2).mean().sqrt().item()
    rtol, atol = (2e-3, 1e-3 * rms) if what.endswith("f16") else (1e-5, 1e-6 * rms)
    assert torch.allclose(o, r, rtol=rtol, atol=atol), f"{what}: max diff {(o - r).abs().max().item()}"


def _run_separately(steps, dt):
    """The same steps launched one GEMV launch at a time, on copies of the
    chain's own inputs: the bit-exact reference for every step."""
    got = []
    for x, ws, outs in steps:
        if len(ws) == 1:
            got.append([ops.gemv_i4(x, ws[0], out_dtype=dt)])
        else:
            got.append(ops.gemv_i4_fused(x, ws, out_dtype=dt))
    torch.cuda.synchronize()
    return got


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("dt", [torch.float32, torch.float16])
def test_chain_small_layers_match_separate_launches_and_oracle(fp8, dt):
    steps, packed, _ = _layer_chain(3, dt, H=256, Q=512, F=1024, V=4096, fp8=fp8, seed=5)
    chain = ops.GemvChain(steps)
    chain.run()
    torch.cuda.synchronize()
    sep = _run_separately(steps, dt)           # reads the x buffers the chain just wrote
    for j, ((x, ws, outs), ref) in enumerate(zip(steps, sep)):
        for i, (o, r) in enumerate(zip(outs, ref)):
            _assert_same_up_to_order(o, r, f"step {j} segment {i} {'f16' if dt == torch.float16 else 'f32'}")
        x32 = x.float().cpu().numpy()
        for i, (o, pw) in enumerate(zip(outs, packed[j])):
            assert_close(o.float().cpu().numpy(), _oracle(pw, x32).astype(np.float32),
                         f"step {j} segment {i} fp8={fp8} dt={dt}")
    assert L.query(L.Q_KERNEL_STATUS) == 0
    chain.close()


def test_chain_repeat_and_graph_replay_are_identical():
    """The chain's counters reset themselves: eager runs and graph replays give
    the same bits every time."""
    steps, _, h = _layer_chain(2, torch.float32, H=512, Q=1024, F=2048, V=8192, fp8=False, seed=9)
    chain = ops.GemvChain(steps)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        chain.run(stream)
    stream.synchronize()
    first = [o.clone() for _, _, outs in steps for o in outs]
    for _ in range(3):
        for _, _, outs in steps:
            for o in outs:
                o.zero_()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            chain.run(stream)
        stream.synchronize()
        assert all(torch.equal(a, b) for a, b in zip(first, [o for _, _, outs in steps for o in outs]))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        chain.run(stream)
    for _, _, outs in steps:
        for o in outs:
            o.zero_()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(4):
            g.replay()
    stream.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(first, [o for _, _, outs in steps for o in outs]))
    # a new hidden state flows through the whole chain
    h.copy_(torch.from_numpy(activations(1, h.numel(), seed=99)[0]).to(DEV))
    with torch.cuda.stream(stream):
        g.replay()
    stream.synchronize()
    sep = _run_separately(steps, torch.float32)
    _assert_same_up_to_order(steps[-1][2][0], sep[-1][0], "lm_head after a new hidden state f32")
    assert not torch.equal(steps[-1][2][0], first[-1])
    assert L.query(L.Q_KERNEL_STATUS) == 0
    del g
    chain.close()


@pytest.mark.parametrize("dt", [torch.float32, torch.float16])
def test_forwarded_x_gives_the_bits_of_the_whole_step_wait(dt, monkeypatch):
    """A step whose x is the step before's first output reads that output as
    epoch-tagged words, each 256-row slice as soon as its own words are stored
    (forwarded x); with G4B_CHAIN_FORWARD=0 at creation every step instead
    waits for the whole step before it and loads x from memory.  Both give the
    same bits, run after run.  Two extra steps: one reading an output from two
    steps back after a run of forwarded steps (its wait then covers every step
    before it), and one forwarded from that."""
    steps, packed, _ = _layer_chain(2, dt, H=512, Q=1024, F=2048, V=4096, fp8=False, seed=13)
    down = steps[-2][2][0]
    e_w = _packed(768, down.numel(), seed=901, std=down.numel() ** -0.5)
    e_out = torch.empty(768, dtype=dt, device=DEV)
    f_w = _packed(512, 768, seed=902, std=768 ** -0.5)
    f_out = torch.empty(512, dtype=dt, device=DEV)
    steps = steps + [(down, [e_w[1]], [e_out]), (e_out, [f_w[1]], [f_out])]
    outs = [o for _, _, oo in steps for o in oo]
    runs = []
    for fwd in ("1", "0"):
        monkeypatch.setenv("G4B_CHAIN_FORWARD", fwd)
        chain = ops.GemvChain(steps)
        got = []
        for _ in range(2):
            for o in outs:
                o.fill_(float("nan"))
            chain.run()
            torch.cuda.synchronize()
            got.append([o.clone() for o in outs])
        assert all(torch.equal(a, b) for a, b in zip(*got)), f"forward={fwd}: runs differ"
        assert L.query(L.Q_KERNEL_STATUS) == 0
        chain.close()
        runs.append(got[0])
    for k, (a, b) in enumerate(zip(*runs)):
        assert torch.equal(a, b), f"output {k}: forwarded x differs from the whole-step wait"
    sep = _run_separately(steps[-2:], dt)
    tag = "f16" if dt == torch.float16 else "f32"
    _assert_same_up_to_order(e_out, sep[0][0], f"two steps back {tag}")
    _assert_same_up_to_order(f_out, sep[1][0], f"forwarded from it {tag}")
    x32 = down.float().cpu().numpy()
    assert_close(e_out.float().cpu().numpy(), _oracle(e_w[0], x32).astype(np.float32), f"two steps back {tag}")


def test_step_overwriting_the_input_of_the_step_before():
    """Step 1 reads step 0's first output and writes its result over step 0's
    own input h, which step 0's second segment may still be reading: the chain
    keeps the whole-step wait there instead of forwarding x.  Step 2 reads the
    new h (forwarded).  Every output is what the steps give one at a time."""
    K = 512
    h0 = torch.from_numpy(activations(1, K, seed=61)[0]).to(DEV)
    h = h0.clone()
    a = [_packed(512, K, seed=62, std=K ** -0.5), _packed(768, K, seed=63, std=K ** -0.5)]
    b = _packed(K, 512, seed=64, std=512 ** -0.5)
    c = _packed(256, K, seed=65, std=K ** -0.5)
    ya, yb, yc = (torch.empty(n, dtype=torch.float32, device=DEV) for n in (512, 768, 256))
    steps = [(h, [a[0][1], a[1][1]], [ya, yb]), (ya, [b[1]], [h]), (h, [c[1]], [yc])]
    chain = ops.GemvChain(steps)
    for _ in range(2):
        h.copy_(h0)
        chain.run()
        torch.cuda.synchronize()
        ra = ops.gemv_i4_fused(h0, [a[0][1], a[1][1]], out_dtype=torch.float32)
        rb = ops.gemv_i4(ra[0], b[1], out_dtype=torch.float32)
        rc = ops.gemv_i4(rb, c[1], out_dtype=torch.float32)
        torch.cuda.synchronize()
        _assert_same_up_to_order(ya, ra[0], "step 0 segment 0 f32")
        _assert_same_up_to_order(yb, ra[1], "step 0 segment 1 f32")
        _assert_same_up_to_order(h, rb, "step 1 (over h) f32")
        _assert_same_up_to_order(yc, rc, "step 2 f32")
    assert L.query(L.Q_KERNEL_STATUS) == 0
    chain.close()


@pytest.mark.parametrize("fp8", [False, True])
def test_chain_config2_shapes(fp8):
    """Two full-size layers of the configs[1] stack and the full lm_head, f16
    activations (the bench's dtype), against separate launches; a second run
    gives the same bits."""
    H, Q, KV, F, V = 3840, 4096, 2048, 15360, 262144
    gen = torch.Generator(device=DEV)
    gen.manual_seed(3)

    def dq(N, K):
        W = torch.randn((N, K), generator=gen, device=DEV).mul_(0.02)
        return qz.quant_device(W, pf=False, fp8=fp8, prefill_i8=False)

    h = torch.randn(H, generator=gen, device=DEV).to(torch.float16)
    steps = []
    x = h
    for _ in range(2):
        outs = [torch.empty(n, dtype=torch.float16, device=DEV) for n in (Q, KV, KV)]
        steps.append((x, [dq(Q, H), dq(KV, H), dq(KV, H)], outs))
        o = [torch.empty(H, dtype=torch.float16, device=DEV)]
        steps.append((outs[0], [dq(H, Q)], o))
        gu = [torch.empty(F, dtype=torch.float16, device=DEV) for _ in range(2)]
        steps.append((o[0], [dq(F, H), dq(F, H)], gu))
        d = [torch.empty(H, dtype=torch.float16, device=DEV)]
        steps.append((gu[0], [dq(H, F)], d))
        x = d[0]
    steps.append((x, [dq(V, H)], [torch.empty(V, dtype=torch.float16, device=DEV)]))
    chain = ops.GemvChain(steps)
    chain.run()
    torch.cuda.synchronize()
    sep = _run_separately(steps, torch.float16)
    for j, ((_, _, outs), ref) in enumerate(zip(steps, sep)):
        for i, (o, r) in enumerate(zip(outs, ref)):
            _assert_same_up_to_order(o, r, f"step {j} segment {i} fp8={fp8} f16")
    assert torch.isfinite(steps[-1][2][0].float()).all()
    first = [o.clone() for _, _, outs in steps for o in outs]
    chain.run()
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(first, [o for _, _, outs in steps for o in outs]))
    assert L.query(L.Q_KERNEL_STATUS) == 0
    chain.close()


@pytest.mark.parametrize("fp8", [False, True])
def test_chain_ragged_steps(fp8):
    """Steps whose item counts are far below the SM count (a single item; a
    fused step of three narrow segments), ragged N, and a step with more tiles
    than SMs, each on its own input, against the oracle."""
    specs = [(1024, [800]), (256, [96]), (512, [32, 64, 288]), (256, [40000]), (2048, [3840])]
    steps, packed = [], []
    for si, (K, Ns) in enumerate(specs):
        x = torch.from_numpy(activations(1, K, seed=300 + si)[0]).to(DEV)
        ws = [_packed(N, K, seed=400 + 10 * si + i, fp8=fp8) for i, N in enumerate(Ns)]
        outs = [torch.empty(N, dtype=torch.float32, device=DEV) for N in Ns]
        steps.append((x, [w[1] for w in ws], outs))
        packed.append([w[0] for w in ws])
    chain = ops.GemvChain(steps)
    chain.run()
    torch.cuda.synchronize()
    sep = _run_separately(steps, torch.float32)
    for j, ((x, _, outs), ref) in enumerate(zip(steps, sep)):
        x32 = x.cpu().numpy()
        for i, (o, r, pw) in enumerate(zip(outs, ref, packed[j])):
            assert_close(o.cpu().numpy(), _oracle(pw, x32).astype(np.float32), f"step {j} segment {i} fp8={fp8}")
            _assert_same_up_to_order(o, r, f"step {j} segment {i} f32")
    assert L.query(L.Q_KERNEL_STATUS) == 0
    chain.close()


def test_chain_rejects_bad_arguments():
    lib = L.load()
    pw, dw = _packed(256, 256, seed=1)
    _, dw96 = _packed(256, 96, seed=2)
    x = torch.zeros(256, dtype=torch.float32, device=DEV)
    y = torch.zeros(256, dtype=torch.float32, device=DEV)

    def step(w, xx=x, nseg=1):
        st = L.GemvChainStep()
        st.x = xx.data_ptr()
        st.K = w.K
        st.nseg = nseg
        for i in range(3):
            st.seg[i] = L.GemvSegment(w.wp.data_ptr(), w.scales.data_ptr(), 1.0, y.data_ptr(), w.N)
        return st

    h = ctypes.c_void_p()
    before = L.launches()
    arr = (L.GemvChainStep * 1)(step(dw96))
    assert lib.g4b_gemv_chain_create(ctypes.cast(arr, ctypes.c_void_p), 1, 0, 0, 0, ctypes.byref(h)) == L.G4B_E_SHAPE
    arr = (L.GemvChainStep * 1)(step(dw, nseg=0))
    assert lib.g4b_gemv_chain_create(ctypes.cast(arr, ctypes.c_void_p), 1, 0, 0, 0, ctypes.byref(h)) == L.G4B_E_ARG
    arr = (L.GemvChainStep * 1)(step(dw))
    assert lib.g4b_gemv_chain_create(ctypes.cast(arr, ctypes.c_void_p), 0, 0, 0, 0, ctypes.byref(h)) == L.G4B_E_ARG
    assert lib.g4b_gemv_chain_create(ctypes.cast(arr, ctypes.c_void_p), 1, 5, 0, 0, ctypes.byref(h)) == L.G4B_E_ARG
    assert lib.g4b_gemv_chain_create(ctypes.cast(arr, ctypes.c_void_p), 1, 0, 0, 0, ctypes.byref(h)) == L.G4B_OK
    need = lib.g4b_gemv_chain_workspace_bytes(h)
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    sh = torch.cuda.current_stream().cuda_stream
    assert lib.g4b_gemv_chain_run(h, ws.data_ptr(), need - 1, sh) == L.G4B_E_WORKSPACE
    assert lib.g4b_gemv_chain_run(h, ws.data_ptr() + 4, need, sh) == L.G4B_E_ALIGN
    assert lib.g4b_gemv_chain_run(None, ws.data_ptr(), need, sh) == L.G4B_E_ARG
    assert L.launches() == before
    assert lib.g4b_gemv_chain_run(h, ws.data_ptr(), need, sh) == L.G4B_OK
    torch.cuda.synchronize()
    assert_close(y.cpu().numpy(), _oracle(pw, np.zeros(256, np.float32)).astype(np.float32), "chain zero x")
    lib.g4b_gemv_chain_destroy(h)
    assert L.query(L.Q_KERNEL_STATUS) == 0
