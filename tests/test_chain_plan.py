"""Where each GEMV-chain step's x comes from (g4b_gemv_chain_plan: the decisions
g4b_gemv_chain_create* makes, computed on the host, so no GPU is needed).

The chain records the engine's per-token command buffer of gemv() dispatches
with a barrier after each (src/vk_engine.py:254-290, bar() at :261).  A step
whose x is the step before's first output may read it slice by slice as
forwarded words instead of waiting for the whole step; an x that no step writes
may be loaded before the step's wait.  These tests pin those decisions on the
layouts the engine and the bench use, and on the hazards that must keep the
whole-step wait: a step writing over what the step before still reads or
writes, mixed dtypes, all-reduced inputs and element-wise steps.  Pointers are
plain addresses here; nothing is dereferenced.
"""
import ctypes

import pytest

from g4b import _lib as L

F16, F32 = 1, 0
BASE = 1 << 32


class Arena:
    """Distinct fake device addresses, 256-byte aligned."""

    def __init__(self):
        self.next = BASE

    def buf(self, nbytes):
        a = self.next
        self.next += (nbytes + 255) // 256 * 256 + 4096
        return a


def _step(x, K, outs, flags=0):
    st = L.GemvChainStep()
    st.x = x
    st.K = K
    st.nseg = len(outs)
    for i, (y, N) in enumerate(outs):
        st.seg[i] = L.GemvSegment(0x1000, 0x2000, 1.0, y, N)
    st.flags = flags
    return st


def _plan(steps, x_dtype, y_dtype, xforms=None):
    lib = L.load()
    arr = (L.GemvChainStep * len(steps))(*steps)
    out = (L.ChainStepPlan * len(steps))()
    xa = None
    if xforms is not None:
        xa = (L.ChainXform * len(steps))()
        for j, f in enumerate(xforms):
            if f is not None:
                xa[j].kind = f["kind"]
                for k in ("a", "b", "w", "w_post", "h_out"):
                    setattr(xa[j], k, f.get(k))
    rc = lib.g4b_gemv_chain_plan(ctypes.cast(arr, ctypes.c_void_p),
                                 ctypes.cast(xa, ctypes.c_void_p) if xa is not None else None,
                                 len(steps), x_dtype, y_dtype, ctypes.cast(out, ctypes.c_void_p))
    assert rc == 0, rc
    return [(p.x_forwarded, p.wait_from, p.x_early) for p in out]


def _token(ar, layers, dt_bytes, reuse=True, allreduce=0):
    """tp.chain_steps' layout: q|k|v on h, o on q, gate|up on o's output (part),
    down on gate, the next layer on down's output, lm_head last."""
    H, Q, KV, F, V = 3840, 4096, 2048, 15360, 262144
    bufs = {n: ar.buf(N * dt_bytes) for n, N in (("q", Q), ("k", KV), ("v", KV), ("part", H), ("gate", F),
                                                  ("up", F), ("logits", V))}
    h = ar.buf(H * dt_bytes)
    steps, x = [], h
    for _ in range(layers):
        b = bufs if reuse else {n: ar.buf(N * dt_bytes) for n, N in (("q", Q), ("k", KV), ("v", KV),
                                                                      ("part", H), ("gate", F), ("up", F))}
        steps.append(_step(x if not allreduce or not steps else None, H, [(b["q"], Q), (b["k"], KV), (b["v"], KV)]))
        steps.append(_step(b["q"], Q, [(b["part"], H)], allreduce))
        steps.append(_step(None if allreduce else b["part"], H, [(b["gate"], F), (b["up"], F)]))
        steps.append(_step(b["gate"], F, [(b["part"], H)], allreduce))
        x = None if allreduce else b["part"]
    steps.append(_step(x, H, [(bufs["logits"], V)]))
    return steps


@pytest.mark.parametrize("dt", [F32, F16])
def test_dependent_token_forwards_every_step(dt):
    """The one-GPU dependent token (buffers reused layer after layer): every
    step after the first takes its x as forwarded words and waits on no count."""
    steps = _token(Arena(), 3, 4 if dt == F32 else 2)
    plan = _plan(steps, dt, dt)
    assert plan[0] == (0, 0, 0)
    assert all(p[0] == 1 for p in plan[1:]), plan
    assert all(p[2] == 0 for p in plan)


def test_mixed_dtypes_keep_the_whole_step_wait():
    """f16 x with f32 outputs: an output is not the next step's x dtype, so
    nothing is forwarded and every step waits for the one before."""
    steps = _token(Arena(), 2, 4)
    plan = _plan(steps, F16, F32)
    assert all(p[0] == 0 for p in plan)
    assert [p[1] for p in plan[1:]] == list(range(len(plan) - 1))


def test_independent_stream_loads_x_early_and_waits_for_the_step_before():
    """The configs[1] stream: every step has its own x, which no step writes.
    No step is forwarded; each waits for the step before (the command buffer's
    barrier) and loads its first x slice before that wait."""
    ar = Arena()
    steps = [_step(ar.buf(3840 * 2), 3840, [(ar.buf(4096 * 2), 4096)]) for _ in range(6)]
    plan = _plan(steps, F16, F16)
    assert [p[0] for p in plan] == [0] * 6
    assert [p[1] for p in plan[1:]] == [0, 1, 2, 3, 4]
    assert [p[2] for p in plan] == [0, 1, 1, 1, 1, 1]


def test_x_written_later_in_the_chain_is_not_loaded_early():
    """Step 1's x is overwritten by step 3: it is not loaded before step 1's
    wait (the chain's order says step 1 reads it first, and a later writer
    must not race an early load)."""
    ar = Arena()
    x1 = ar.buf(1024 * 2)
    steps = [_step(ar.buf(1024 * 2), 1024, [(ar.buf(512 * 2), 512)]),
             _step(x1, 1024, [(ar.buf(512 * 2), 512)]),
             _step(ar.buf(1024 * 2), 1024, [(ar.buf(512 * 2), 512)]),
             _step(ar.buf(1024 * 2), 1024, [(x1, 1024)])]
    plan = _plan(steps, F16, F16)
    assert plan[1][2] == 0 and plan[2][2] == 1 and plan[3][2] == 1


def test_step_writing_what_the_step_before_reads_keeps_the_wait():
    """Step 1 reads step 0's first output and writes over step 0's own input;
    step 0's second segment may still be reading it, so step 1 waits for step
    0.  Step 2 reads step 1's output (forwarded).  Step 3 reads step 0's output
    two steps back: it waits, and its wait reaches back over the forwarded
    step 2 to step 1."""
    ar = Arena()
    h, ya, yb, yc, yd = (ar.buf(n * 4) for n in (512, 512, 768, 256, 128))
    steps = [_step(h, 512, [(ya, 512), (yb, 768)]),
             _step(ya, 512, [(h, 512)]),
             _step(h, 512, [(yc, 256)]),
             _step(ya, 512, [(yd, 128)])]
    plan = _plan(steps, F32, F32)
    assert [p[0] for p in plan] == [0, 0, 1, 0]
    assert plan[1][1] == 0 and plan[3][1] == 1


def test_step_writing_what_the_step_before_writes_keeps_the_wait():
    """Step 1's output lands on step 0's second output (still being written
    when step 1 could start): no forwarding there."""
    ar = Arena()
    h, ya, yb = ar.buf(512 * 4), ar.buf(512 * 4), ar.buf(768 * 4)
    steps = [_step(h, 512, [(ya, 512), (yb, 768)]), _step(ya, 512, [(yb, 256)])]
    assert _plan(steps, F32, F32)[1][0] == 0


def test_all_reduced_inputs_are_not_forwarded_and_o_and_down_are():
    """The tensor-parallel token: the steps after an all-reduced step read the
    all-reduce's words (no count, no forwarding); o reads q and down reads gate
    as forwarded words."""
    steps = _token(Arena(), 2, 4, allreduce=L.CHAIN_ALLREDUCE)
    plan = _plan(steps, F32, F32)
    kinds = ["qkv", "o", "gateup", "down"] * 2 + ["lm"]
    for k, p in zip(kinds, plan):
        if k in ("o", "down"):
            assert p[0] == 1, (k, plan)
        else:
            assert p[0] == 0 and p[2] == 0, (k, plan)


def test_forwarding_off_by_environment(monkeypatch):
    monkeypatch.setenv("G4B_CHAIN_FORWARD", "0")
    steps = _token(Arena(), 2, 2)
    plan = _plan(steps, F16, F16)
    assert all(p[0] == 0 and p[2] == 0 for p in plan)
    assert [p[1] for p in plan[1:]] == list(range(len(plan) - 1))


def test_fused_token_forwards_o_only():
    """A token with the element-wise work fused (g4b.decode.token_plan's
    layout): o reads q as forwarded words; the rmsnorm / normadd / gelu*up steps
    wait for the step before, reaching back over the forwarded o."""
    ar = Arena()
    H, Q, KV, F = 512, 512, 256, 1024
    b = {n: ar.buf(N * 2) for n, N in (("q", Q), ("k", KV), ("v", KV), ("o", H), ("gate", F), ("up", F),
                                        ("down", H), ("logits", 2048))}
    h0, hA, hB = ar.buf(H * 4), ar.buf(H * 4), ar.buf(H * 4)
    w = ar.buf(H * 4)
    steps = [_step(None, H, [(b["q"], Q), (b["k"], KV), (b["v"], KV)]), _step(b["q"], Q, [(b["o"], H)]),
             _step(None, H, [(b["gate"], F), (b["up"], F)]), _step(None, F, [(b["down"], H)]),
             _step(None, H, [(b["logits"], 2048)])]
    xf = [{"kind": L.XF_RMSNORM, "a": h0, "w": w},
          None,
          {"kind": L.XF_NORMADD, "a": b["o"], "b": h0, "w": w, "w_post": w, "h_out": hA},
          {"kind": L.XF_GELU_MUL, "a": b["gate"], "b": b["up"]},
          {"kind": L.XF_NORMADD, "a": b["down"], "b": hA, "w": w, "w_post": w, "h_out": hB}]
    plan = _plan(steps, F16, F16, xf)
    assert [p[0] for p in plan] == [0, 1, 0, 0, 0]
    assert plan[2][1] == 0 and plan[3][1] == 2 and plan[4][1] == 3
    assert all(p[2] == 0 for p in plan)


def test_plan_rejects_bad_arguments():
    lib = L.load()
    out = (L.ChainStepPlan * 1)()
    st = (L.GemvChainStep * 1)(_step(BASE, 256, [(BASE + 8192, 256)]))
    assert lib.g4b_gemv_chain_plan(None, None, 1, F16, F16, ctypes.cast(out, ctypes.c_void_p)) < 0
    assert lib.g4b_gemv_chain_plan(ctypes.cast(st, ctypes.c_void_p), None, 0, F16, F16,
                                   ctypes.cast(out, ctypes.c_void_p)) < 0
    assert lib.g4b_gemv_chain_plan(ctypes.cast(st, ctypes.c_void_p), None, 1, 7, F16,
                                   ctypes.cast(out, ctypes.c_void_p)) < 0
