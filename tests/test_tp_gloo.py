"""Tensor-parallel decode logic (g4b.tp) on CPU: world size 2 over gloo.

Each rank packs the layers, takes its column / row shards, and runs the
decode chain with the CPU oracle's GEMV (oracle/g4b_oracle.c orc_gemv, the
restatement of vk/gemv.comp + vk/reduce.comp) and gloo collectives; rank 0
compares the gathered logits with the same chain on unsharded weights.  The
sharded result differs only in f32 summation order: the bar is tests/util.py's
(max rel err 1e-2 with a 1e-3 x rms guard, cosine >= 0.9999).  Also checks
that packing a shard gives the same bytes as slicing the packed weight.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "gemma4-12b-snapdragonx2elite_b200"))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from g4b import pack, tp  # noqa: E402
from util import assert_close, weights  # noqa: E402

H, NQ, NKV, FFN, VOCAB, LAYERS = 512, 1024, 512, 2048, 2048, 2


def _shapes():
    return {"q": (NQ, H), "k": (NKV, H), "v": (NKV, H), "o": (H, NQ), "gate": (FFN, H), "up": (FFN, H),
            "down": (H, FFN)}


def _full_model():
    layers = []
    seed = 0
    for _ in range(LAYERS):
        d = {}
        for name, (N, K) in _shapes().items():
            d[name] = pack.quant(weights(N, K, seed), fp8=False, prefill_i8=False)
            seed += 1
        layers.append(tp.TPLayer(**d))
    lm = pack.quant(weights(VOCAB, H, 99), fp8=False, prefill_i8=False)
    return layers, lm


def _oracle_gemv(x, pw):
    import oracle as O
    return O.gemv(np.asarray(x, np.float32), pw.wp, pw.scales.view(np.uint16), 0, 1.0, pw.N, pw.K, 1)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layers, lm = _full_model()
        kinds = dict(tp.LAYER_KINDS)
        mine = [tp.TPLayer(**{n: (tp.shard_columns if kinds[n] == "col" else tp.shard_rows)(getattr(L, n), world, rank)
                              for n in kinds}) for L in layers]
        lm_mine = tp.shard_columns(lm, world, rank)

        def gemv(x, w, out):
            out.copy_(torch.from_numpy(_oracle_gemv(x.numpy(), w)))

        def gemv_fused(x, ws, outs):
            for w, o in zip(ws, outs):
                gemv(x, w, o)

        dec = tp.TPDecoder(layers=mine, lm_head=lm_mine, gemv=gemv, all_reduce=lambda t: dist.all_reduce(t),
                           all_gather=lambda out, t: dist.all_gather_into_tensor(out, t),
                           new_buffer=lambda n: torch.zeros(n, dtype=torch.float32), hidden=H, vocab=VOCAB,
                           world=world, gemv_fused=gemv_fused)
        x = torch.from_numpy(np.random.default_rng(5).standard_normal(H).astype(np.float32))
        logits = dec.step(x).numpy().copy()
        if rank == 0:
            ref = tp.decode_reference(layers, lm, x.numpy(), _oracle_gemv)
            q.put(("ok", logits, ref))
        dist.barrier()
    except Exception as e:  # report, never hang the parent
        q.put(("error", repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_tp_decode_world2_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    status, logits, ref = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert status == "ok", logits
    assert all(p.exitcode == 0 for p in procs)
    assert_close(logits, ref, "TP world 2 vs unsharded")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_of_packed_equals_packed_shard(world):
    N, K = 2048, 2048
    W = weights(N, K, 3)
    full = pack.quant(W, fp8=False, prefill_i8=True)
    for r in range(world):
        n0, n1 = tp.split_range(N, world, r, tp.COL_ALIGN)
        c = tp.shard_columns(full, world, r)
        p = pack.quant(W[n0:n1], fp8=False, prefill_i8=True)
        assert np.array_equal(c.wp, p.wp) and np.array_equal(c.scales16, p.scales16)
        k0, k1 = tp.split_range(K, world, r, tp.ROW_ALIGN)
        rr = tp.shard_rows(full, world, r)
        p = pack.quant(W[:, k0:k1], fp8=False, prefill_i8=False)
        assert np.array_equal(rr.wp, p.wp) and np.array_equal(rr.scales16, p.scales16)


def test_split_covers_and_rejects():
    for n, world in ((4096, 8), (2048, 8), (15360, 8), (262144, 8), (3840, 2)):
        spans = [tp.split_range(n, world, r, 256) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert all((b - a) % 256 == 0 for a, b in spans)
    with pytest.raises(ValueError):
        tp.split_range(96, 2, 0, 64)
    with pytest.raises(ValueError):
        tp.split_range(256, 2, 0, 256)   # one unit cannot go to two ranks
    assert tp.validate_world(3840, 4096, 2048, 15360, 262144, 8) is None


@pytest.mark.parametrize("world", [3, 5, 6, 7])
def test_world_with_unequal_logits_shards_is_refused(world):
    """Worlds whose lm_head column shards would differ in size (262144 columns =
    1024 units of 256 do not split evenly over 3, 5, 6 or 7 ranks) are refused
    by validate_world, before any rank reaches the equal-count all-gather."""
    spans = [tp.split_range(262144, world, r, tp.COL_ALIGN) for r in range(world)]
    assert len({b - a for a, b in spans}) > 1
    why = tp.validate_world(3840, 4096, 2048, 15360, 262144, world)
    assert why is not None and "all-gather" in why


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_power_of_two_worlds_are_accepted(world):
    assert tp.validate_world(3840, 4096, 2048, 15360, 262144, world) is None


def test_chain_steps_layout():
    """tp.chain_steps: per layer q|k|v, o (all-reduced), gate|up on the sum
    (no x), down (all-reduced), then lm_head on the final sum."""
    class W:
        def __init__(self, N, K):
            self.N, self.K = N, K
    L = tp.TPLayer(q=W(512, 256), k=W(256, 256), v=W(256, 256), o=W(256, 512), gate=W(1024, 256),
                   up=W(1024, 256), down=W(256, 1024))
    bufs = {k: k for k in ("q", "k", "v", "part", "gate", "up", "logits_local")}
    steps = tp.chain_steps([L, L], W(4096, 256), "h", bufs, 1)
    assert len(steps) == 9
    assert steps[0][0] == "h" and steps[4][0] is None and steps[8][0] is None
    assert [len(st) > 3 and st[3] == 1 for st in steps] == [False, True, False, True] * 2 + [False]
    assert steps[1][0] == "q" and steps[3][0] == "gate"
    for j, st in enumerate(steps):
        if len(st) > 3 and st[3]:
            assert len(st[1]) == 1 and steps[j + 1][1][0].K == st[1][0].N
