"""Worker for tests/test_gpu_tp.py: one rank of a tensor-parallel decode over
NCCL (launched by torch.distributed.run).  Rank 0 also runs the same chain
with the unsharded weights on its own GPU, and again on the host through the
CPU oracle (oracle.gemv: vk/gemv.comp + vk/reduce.comp restated, on host
copies of the unsharded packed weights), and compares the gathered logits
with both (tests/util.py bar).  Exit code 0 = match."""
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "gemma4-12b-snapdragonx2elite_b200"))
sys.path.insert(0, HERE)

from g4b import _lib as L  # noqa: E402
from g4b import comm, ops, tp  # noqa: E402
from g4b import quant_gpu as qz  # noqa: E402
from util import assert_close  # noqa: E402

sys.path.insert(0, ROOT)
import oracle as O  # noqa: E402


def _oracle_gemv(h, w):
    """The unsharded GEMV on the host: the oracle over w's packed words and scales."""
    sc = w.scales.cpu().numpy()
    sc = sc.view(np.uint16) if w.scale_fmt == L.SCALE_F16 else sc
    return O.gemv(np.asarray(h, np.float32), w.wp.cpu().numpy().view(np.uint32), sc, w.scale_fmt, w.inv,
                  w.N, w.K, w.split)

# every column / row shard splits in 256-wide units over up to 8 ranks
H, NQ, NKV, FFN, VOCAB, LAYERS = 1024, 2048, 2048, 4096, 8192, 2


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    L.load()
    fp8 = os.environ.get("TP_FP8") == "1"
    use_chain = os.environ.get("TP_ALLREDUCE", "nccl") == "chain"
    use_peer = os.environ.get("TP_ALLREDUCE", "nccl") == "peer"
    peer = comm.PeerAllReduce(H, dev) if use_peer else None
    if peer is not None:
        # the peer all-reduce alone: identical bits on every rank, equal to NCCL's two-rank sum
        a = torch.randn((H,), generator=torch.Generator(device=dev).manual_seed(100 + rank), device=dev)
        ref = a.clone()
        dist.all_reduce(ref)
        got = peer(a.clone())
        for _ in range(3):                       # repeated calls alternate the buffer halves
            got2 = peer(a.clone())
        torch.cuda.synchronize()
        allg = [torch.empty_like(got) for _ in range(world)]
        dist.all_gather(allg, got)
        ok_ar = all(torch.equal(allg[0], g_) for g_ in allg) and torch.equal(got, got2)
        if world == 2:
            ok_ar = ok_ar and torch.equal(got, ref)
        if not ok_ar:
            print("peer all-reduce mismatch", flush=True)
            sys.exit(1)
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    shapes = {"q": (NQ, H), "k": (NKV, H), "v": (NKV, H), "o": (H, NQ), "gate": (FFN, H), "up": (FFN, H),
              "down": (H, FFN)}
    kinds = dict(tp.LAYER_KINDS)
    full, mine = [], []
    for _ in range(LAYERS):
        f, m = {}, {}
        for name, (N, K) in shapes.items():
            W = torch.randn((N, K), generator=gen, device=dev).mul_(0.02)
            if rank == 0:
                f[name] = qz.quant_device(W, pf=False, fp8=fp8, prefill_i8=False)
            if kinds[name] == "col":
                n0, n1 = tp.split_range(N, world, rank, tp.COL_ALIGN)
                m[name] = qz.quant_device(W[n0:n1].contiguous(), pf=False, fp8=fp8, prefill_i8=False)
            else:
                k0, k1 = tp.split_range(K, world, rank, tp.ROW_ALIGN)
                m[name] = qz.quant_device(W[:, k0:k1].contiguous(), pf=False, fp8=fp8, prefill_i8=False)
        full.append(tp.TPLayer(**f) if rank == 0 else None)
        mine.append(tp.TPLayer(**m))
    Wl = torch.randn((VOCAB, H), generator=gen, device=dev).mul_(0.02)
    n0, n1 = tp.split_range(VOCAB, world, rank, tp.COL_ALIGN)
    lm = qz.quant_device(Wl[n0:n1].contiguous(), pf=False, fp8=fp8, prefill_i8=False)
    lm_full = qz.quant_device(Wl, pf=False, fp8=fp8, prefill_i8=False) if rank == 0 else None
    stream = torch.cuda.Stream(dev)

    def gemv(x, w, out):
        ops.gemv_i4(x, w, out=out, stream=stream, pdl=True)

    def gemv_fused(x, ws, outs):
        ops.gemv_i4_fused(x, ws, outs=outs, stream=stream, pdl=True)

    all_reduce = (lambda t: peer(t, stream=stream, pdl=True)) if peer is not None else (lambda t: dist.all_reduce(t))
    dec = tp.TPDecoder(layers=mine, lm_head=lm, gemv=gemv, all_reduce=all_reduce,
                       all_gather=lambda out, t: dist.all_gather_into_tensor(out, t),
                       new_buffer=lambda n: torch.zeros(n, dtype=torch.float32, device=dev),
                       hidden=H, vocab=VOCAB, world=world, gemv_fused=gemv_fused)
    x = torch.randn((H,), generator=gen, device=dev)
    xchg = None
    if use_chain:
        # the whole token as one persistent launch per rank, all-reduces inside it
        b = dec.bufs
        b["part"] = torch.zeros(H, dtype=torch.float32, device=dev)
        steps = tp.chain_steps(mine, lm, x, b, L.CHAIN_ALLREDUCE)
        xchg = comm.PeerBuffers(ops.GemvChain.exchange_bytes(steps, world), dev)
        chain = ops.GemvChain(steps, exchange=xchg)

        def step(_x):
            chain.run(stream)
            dist.all_gather_into_tensor(b["logits"], b["logits_local"])
            return b["logits"]
    else:
        step = dec.step
    with torch.cuda.stream(stream):
        logits = step(x).clone()
        # the same step captured in a CUDA graph (collectives included) and replayed
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step(x)
        for _ in range(3):
            g.replay()
    stream.synchronize()
    replay = dec.bufs["logits"].clone()
    ok = torch.tensor([1], device=dev)
    if rank == 0:
        ref = tp.decode_reference(full, lm_full, x, lambda h, w: ops.gemv_i4(h, w, out_dtype=torch.float32))
        torch.cuda.synchronize()
        host = tp.decode_reference(full, lm_full, x.cpu().numpy(), _oracle_gemv)
        try:
            assert_close(logits.cpu().numpy(), ref.cpu().numpy(), f"TP world {world} vs unsharded")
            assert_close(logits.cpu().numpy(), host, f"TP world {world} vs the CPU oracle")
            assert torch.equal(logits, replay), "graph replay differs from the eager step"
            assert L.query(L.Q_KERNEL_STATUS) == 0
        except AssertionError as e:
            print(e, flush=True)
            ok.zero_()
    dist.broadcast(ok, 0)
    del g
    if peer is not None:
        peer.close()
    if xchg is not None:
        chain.close()
        xchg.close()
    dist.destroy_process_group()
    sys.exit(0 if ok.item() == 1 else 1)


if __name__ == "__main__":
    main()
