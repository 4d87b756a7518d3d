"""Tensor-parallel decode and M-split prefill over the GPUs of one node.

The packed int4 layout shards without repacking, because both splits fall on
whole words and whole scale blocks (src/vk_engine.py:126-131):

- column-parallel (q, k, v, gate, up, lm_head): rank r owns output columns
  [n0, n1) -- the words wp[:, n0/8 : n1/8] and the scales [:, n0 : n1].  Its
  GEMV writes y[n0:n1].
- row-parallel (o, down): rank r owns input rows [k0, k1) -- wp[k0:k1, :] and
  scales[k0/32 : k1/32, :].  Its GEMV is one split-K slice of the full GEMV
  (vk/gemv.comp:15-16), and an all-reduce(sum) over the ranks is the
  cross-GPU reduce.comp (vk/reduce.comp:8-12).

A decode layer runs q/k/v column-parallel, o row-parallel, then an
all-reduce; gate/up column-parallel, down row-parallel, then an all-reduce.
So there are two collectives per layer and no gather inside the layer.  The
column split of q (and of gate) is the row split of o (and of down), so each
rank feeds its own slice forward.  The lm_head is column-parallel, followed
by an all-gather of the logits.  Attention and the gated GELU sit between
those GEMVs in the engine (src/vk_engine.py:277-287) and are outside this
path.  The decode stream here hands q's slice to o and gate's slice to down
in their place, which keeps the data dependencies of a real decode step.

Packing a shard of W gives the same bytes as slicing the packed W
(`shard_columns` / `shard_rows` on the host arrays); tests check that.

Prefill splits the M rows over the ranks with the weights replicated; no
collective is needed.

Collectives go through torch.distributed: NCCL over NVLink on GPUs, gloo in
the CPU tests.  The compute is a caller-supplied GEMV, g4b.ops.gemv_i4 on the
GPU.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, List, Optional

import numpy as np

from .pack import BLK, PackedWeight

# Shard granularity: 256 keeps column shards on whole words and row shards on
# whole 32-row scale blocks, keeps every shard on the GEMV's fastest path
# (N % 32, K % 256), and makes q's (gate's) column split the same ranges as
# o's (down's) row split, so each rank feeds its own slice forward.  Shards
# are balanced in units of 256 (e.g. down's K = 15360 over 8 ranks: 1792 or 2048).
COL_ALIGN = 256
ROW_ALIGN = 256


def split_range(n: int, world: int, rank: int, align: int) -> tuple[int, int]:
    """[lo, hi) of rank's share of n items in units of `align` (balanced)."""
    if n % align:
        raise ValueError(f"tp: size {n} is not a multiple of {align}")
    units = n // align
    if units < world:
        raise ValueError(f"tp: {n} cannot be split over {world} ranks in units of {align}")
    lo = units * rank // world
    hi = units * (rank + 1) // world
    return lo * align, hi * align


def shard_columns(pw: PackedWeight, world: int, rank: int) -> PackedWeight:
    """Rank's output-column shard of a packed weight (host arrays)."""
    n0, n1 = split_range(pw.N, world, rank, COL_ALIGN)
    sl = lambda a: None if a is None else np.ascontiguousarray(a[..., n0:n1])  # noqa: E731
    return PackedWeight(
        N=n1 - n0, K=pw.K, wp=np.ascontiguousarray(pw.wp[:, n0 // 8:n1 // 8]), scales=sl(pw.scales),
        scale_fmt=pw.scale_fmt, inv=pw.inv, split=pw.split, nblk=pw.nblk, scales16=sl(pw.scales16),
        w8=sl(pw.w8), sw8=None if pw.sw8 is None else np.ascontiguousarray(pw.sw8[n0:n1]),
        sw_f32=None if pw.sw_f32 is None else np.ascontiguousarray(pw.sw_f32[n0:n1]),
        sc_f32=None if pw.sc_f32 is None else np.ascontiguousarray(pw.sc_f32[n0:n1]))


def shard_rows(pw: PackedWeight, world: int, rank: int) -> PackedWeight:
    """Rank's input-row (K) shard of a packed weight (host arrays).  The int8
    W8A8 weights are not row-sharded: their per-column scale spans all of K."""
    k0, k1 = split_range(pw.K, world, rank, ROW_ALIGN)
    b0, b1 = k0 // BLK, k1 // BLK
    return PackedWeight(
        N=pw.N, K=k1 - k0, wp=np.ascontiguousarray(pw.wp[k0:k1]), scales=np.ascontiguousarray(pw.scales[b0:b1]),
        scale_fmt=pw.scale_fmt, inv=pw.inv, split=1, nblk=b1 - b0,
        scales16=np.ascontiguousarray(pw.scales16[b0:b1]),
        sc_f32=None if pw.sc_f32 is None else np.ascontiguousarray(pw.sc_f32[:, b0:b1]))


# ------------------------------------------------------------ decode stack
LAYER_KINDS = (("q", "col"), ("k", "col"), ("v", "col"), ("o", "row"),
               ("gate", "col"), ("up", "col"), ("down", "row"))


@dataclass
class TPLayer:
    """One decode layer's shards on this rank (any weight object the GEMV takes)."""
    q: object
    k: object
    v: object
    o: object
    gate: object
    up: object
    down: object


@dataclass
class TPDecoder:
    """The tensor-parallel decode weight stream of one rank.

    gemv(x, w, out) computes out = W x for this rank's shard `w`;
    gemv_fused(x, [w...], [out...]), if given, runs the GEMVs that read the
    same x (q|k|v, gate|up) as one launch; all_reduce(t) / all_gather(out, t)
    are the collectives (in place / into `out`).  Buffers are preallocated
    once; `step` allocates nothing."""
    layers: List[TPLayer]
    lm_head: object
    gemv: Callable
    all_reduce: Callable
    all_gather: Callable
    new_buffer: Callable          # new_buffer(n) -> f32 vector
    hidden: int
    vocab: int
    world: int
    gemv_fused: Optional[Callable] = None
    bufs: dict = field(default_factory=dict)

    def __post_init__(self):
        L0 = self.layers[0]
        n = lambda w: w.N  # noqa: E731
        self.bufs = {
            "h": self.new_buffer(self.hidden),
            "q": self.new_buffer(n(L0.q)), "k": self.new_buffer(n(L0.k)), "v": self.new_buffer(n(L0.v)),
            "gate": self.new_buffer(n(L0.gate)), "up": self.new_buffer(n(L0.up)),
            "logits_local": self.new_buffer(n(self.lm_head)),
            "logits": self.new_buffer(n(self.lm_head) * self.world),
        }

    def step(self, x):
        """One token through every layer; returns the gathered logits buffer.
        x: the replicated hidden state (f32, `hidden` long)."""
        b = self.bufs
        h = x
        for L in self.layers:
            if self.gemv_fused is not None:
                self.gemv_fused(h, [L.q, L.k, L.v], [b["q"], b["k"], b["v"]])
            else:
                self.gemv(h, L.q, b["q"])
                self.gemv(h, L.k, b["k"])
                self.gemv(h, L.v, b["v"])
            # attention would combine q, k, v here; o consumes this rank's heads
            self.gemv(b["q"], L.o, b["h"])
            self.all_reduce(b["h"])
            h = b["h"]
            if self.gemv_fused is not None:
                self.gemv_fused(h, [L.gate, L.up], [b["gate"], b["up"]])
            else:
                self.gemv(h, L.gate, b["gate"])
                self.gemv(h, L.up, b["up"])
            # the gated GELU would combine gate and up here; down consumes this rank's slice
            self.gemv(b["gate"], L.down, b["h"])
            self.all_reduce(b["h"])
            h = b["h"]
        self.gemv(h, self.lm_head, b["logits_local"])
        self.all_gather(b["logits"], b["logits_local"])
        return b["logits"]


def chain_steps(layers: List[TPLayer], lm_head, h, bufs: dict, allreduce_flag: int) -> list:
    """One token of the tensor-parallel decode as GEMV chain steps
    (g4b.ops.GemvChain): per layer q|k|v on the replicated hidden state, o on
    this rank's q shard with its output all-reduced inside the chain, gate|up
    on that sum, down on this rank's gate shard, all-reduced again; lm_head
    last on the final sum.  `h` is the first layer's input (f32, hidden long);
    `bufs` holds the per-rank outputs ("q", "k", "v", "part", "gate", "up",
    "logits_local").  The logits all-gather follows the chain.

    allreduce_flag 0 (one rank, or the collectives left out): the o and down
    outputs are not all-reduced, and the steps after them read "part" itself."""
    steps = []
    x = h
    after = None if allreduce_flag else bufs["part"]
    for L in layers:
        steps.append((x, [L.q, L.k, L.v], [bufs["q"], bufs["k"], bufs["v"]]))
        steps.append((bufs["q"], [L.o], [bufs["part"]], allreduce_flag))
        steps.append((after, [L.gate, L.up], [bufs["gate"], bufs["up"]]))
        steps.append((bufs["gate"], [L.down], [bufs["part"]], allreduce_flag))
        x = after
    steps.append((after, [lm_head], [bufs["logits_local"]]))
    return steps


def decode_reference(layers_full, lm_full, x, gemv_full):
    """The same chain on one device with unsharded weights (the check for TPDecoder)."""
    h = x
    for L in layers_full:
        q = gemv_full(h, L.q)
        gemv_full(h, L.k)
        gemv_full(h, L.v)
        h = gemv_full(q, L.o)
        gate = gemv_full(h, L.gate)
        gemv_full(h, L.up)
        h = gemv_full(gate, L.down)
    return gemv_full(h, lm_full)


# ------------------------------------------------------------ prefill
def prefill_rows(M: int, world: int, rank: int) -> tuple[int, int]:
    """The prefill rows [m0, m1) of this rank (M split, weights replicated)."""
    lo = M * rank // world
    hi = M * (rank + 1) // world
    return lo, hi


def shard_layer_shapes(shapes, world: int):
    """Per-rank (N, K) of each (name, N, K, kind) for a TP world size."""
    out = []
    for name, N, K, kind in shapes:
        if kind == "col":
            n0, n1 = split_range(N, world, 0, COL_ALIGN)
            out.append((name, n1 - n0, K, kind))
        else:
            k0, k1 = split_range(K, world, 0, ROW_ALIGN)
            out.append((name, N, k1 - k0, kind))
    return out


def validate_world(hidden: int, nq: int, nkv: int, ffn: int, vocab: int, world: int) -> Optional[str]:
    """None if the decode stack shards over `world` ranks, else why not.

    Every sharded size must split in units of 256.  The logits are gathered
    with an equal-count all-gather, so the lm_head's column shards must also
    be the same size on every rank (vocab a multiple of 256 * world); a world
    that fails this is refused here, before any collective runs."""
    if world < 1:
        return f"tp: world size {world} must be at least 1"
    try:
        for n in (nq, nkv, ffn, vocab):
            split_range(n, world, 0, COL_ALIGN)
        for k in (nq, ffn):
            split_range(k, world, 0, ROW_ALIGN)
    except ValueError as e:
        return str(e)
    if vocab % (COL_ALIGN * world):
        return (f"tp: the logits all-gather needs equal shards, but vocab {vocab} does not split into {world} "
                f"shards of whole {COL_ALIGN}-column units")
    return None
