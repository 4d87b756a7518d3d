"""Generate golden packing vectors by running the reference's own ``quant()``.

The reference engine (``src/vk_engine.py``) initialises Vulkan and loads the
model at import time, so it cannot be imported here.  This script instead
parses that file, pulls out the ``quant`` function definition
(src/vk_engine.py:125-159) with :mod:`ast`, and executes that unmodified
function in a namespace that supplies the module globals it reads:

* ``np`` / ``torch``                      -- the same libraries the engine imports
* ``BLK = 32``                            -- src/vk_engine.py:12
* ``FP8`` / ``PREFILL_I8``                -- the env switches, src/vk_engine.py:8-9
* ``Buf``                                 -- a stand-in for the host-visible Vulkan
  buffer class (src/vk_engine.py:56-69) that simply keeps the bytes written.

Every array the reference would have uploaded to the GPU is recorded
byte-for-byte and saved to ``tests/golden/quant_golden.npz`` together with the
seeded input weights, so the product packer and the oracle can be checked
against the reference itself without the reference on the machine.

Run from the repository root, in a container that has a checkout of the
reference project, giving its root directory::

    python tests/golden/make_golden.py --ref <path to the reference checkout>

The outputs are small (a few hundred KB) and are committed.
"""
from __future__ import annotations

import argparse
import ast
import json
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


class _RecordingBuf:
    """Stand-in for the engine's ``Buf``: keeps the bytes ``write`` received."""

    def __init__(self, nbytes):
        self.size = nbytes
        self.data = None

    def write(self, arr):
        a = np.ascontiguousarray(arr)
        self.data = a.tobytes()


def load_reference_quant(ref_root: str, fp8: bool, prefill_i8: bool):
    path = os.path.join(ref_root, "src", "vk_engine.py")
    with open(path, "r", encoding="utf-8") as f:
        src = f.read()
    tree = ast.parse(src, filename=path)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "quant")
    mod = ast.Module(body=[fn], type_ignores=[])
    code = compile(mod, path, "exec")
    ns = {"np": np, "torch": torch, "BLK": 32, "FP8": fp8, "PREFILL_I8": prefill_i8,
          "Buf": _RecordingBuf}
    exec(code, ns)
    return ns["quant"], fn.lineno


def run_quant(quant, W, pf=True):
    bw, bs, split, nblk, inv, bs16, w8, sw8 = quant(W, pf)
    out = {
        "wp": np.frombuffer(bw.data, np.uint32).copy(),
        "scales": np.frombuffer(bs.data, np.uint8).copy(),       # raw bytes (f16 pairs or e4m3 quads)
        "scales16": np.frombuffer(bs16.data, np.uint16).copy(),  # the f16 prefill copy
        "split": np.int64(split), "nblk": np.int64(nblk), "inv": np.float64(inv),
    }
    if w8 is not None:
        out["w8"] = np.frombuffer(w8.data, np.int8).copy()
        out["sw8"] = np.frombuffer(sw8.data, np.uint16).copy()
    return out


def edge_weights():
    """Hand-built [N=32, K=128] weights hitting the packing's edge cases."""
    N, K = 32, 128
    W = np.zeros((N, K), np.float32)
    rng = np.random.default_rng(7)
    W[:] = rng.standard_normal((N, K)).astype(np.float32) * 0.02
    # row 0: block 0 all zero (scale floor 1e-8), block 1 exact half-way ratios (round-half-even)
    W[0, 0:32] = 0.0
    W[0, 32:64] = np.float32(0.0)
    W[0, 32] = 7.0                      # absmax 7 -> scale 1.0
    W[0, 33:40] = [0.5, 1.5, 2.5, 3.5, -0.5, -1.5, -2.5]
    W[0, 40:47] = [4.5, 5.5, 6.5, -3.5, -4.5, -5.5, -6.5]
    W[0, 47] = -7.0
    # row 1: a single huge outlier per block (others collapse to nibble 8)
    W[1, 64] = 100.0
    W[1, 96] = -0.001
    # row 2: denormal-range values (scale floor dominates)
    W[2, :] = np.float32(1e-12)
    # row 3: block with negative absmax (-7 -> q=1 after +8) and max positive (7 -> 15)
    W[3, 0:32] = np.linspace(-7.0, 7.0, 32, dtype=np.float32)
    return W


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root directory of a checkout of the reference project")
    ap.add_argument("--out", default=os.path.join(HERE, "quant_golden.npz"))
    ap.add_argument("--skip-split-table", action="store_true")
    args = ap.parse_args()

    q_f16, lineno = load_reference_quant(args.ref, fp8=False, prefill_i8=True)
    q_fp8, _ = load_reference_quant(args.ref, fp8=True, prefill_i8=True)

    arrays = {}
    cases = {
        "rand_64x128": (np.random.default_rng(0).standard_normal((64, 128)) * 0.02).astype(np.float32),
        "rand_128x256": (np.random.default_rng(1).standard_normal((128, 256)) * 0.02).astype(np.float32),
        "rand_48x96_wide": (np.random.default_rng(2).standard_normal((48, 96)) * 3.0).astype(np.float32),
        "edge_32x128": edge_weights(),
    }
    for name, W in cases.items():
        arrays[f"{name}/W"] = W
        for tag, qf in (("f16", q_f16), ("fp8", q_fp8)):
            out = run_quant(qf, W, pf=True)
            for k, v in out.items():
                arrays[f"{name}/{tag}/{k}"] = np.asarray(v)
    # lm_head packing (pf=False) skips the int8 weights
    out = run_quant(q_f16, cases["rand_64x128"], pf=False)
    arrays["rand_64x128/f16_nopf/has_w8"] = np.int64(0 if "w8" not in out else 1)

    split_table = []
    if not args.skip_split_table:
        q_nosplit, _ = load_reference_quant(args.ref, fp8=False, prefill_i8=False)
        shapes = [(4096, 3840), (2048, 3840), (3840, 4096), (15360, 3840), (3840, 15360),
                  (262144, 3840), (4096, 4096), (64, 128), (256, 512), (16, 32)]
        for (N, K) in shapes:
            W = np.zeros((N, K), np.float32)
            out = run_quant(q_nosplit, W, pf=False)
            split_table.append([N, K, int(out["split"])])
            del W, out
    arrays["split_table"] = np.array(split_table, np.int64).reshape(-1, 3)

    meta = {"reference_file": "src/vk_engine.py", "quant_def_line": lineno,
            "torch": torch.__version__, "numpy": np.__version__,
            "cases": list(cases.keys())}
    arrays["meta_json"] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
    np.savez_compressed(args.out, **arrays)
    print(f"wrote {args.out}: {len(arrays)} arrays; split table {split_table}")


if __name__ == "__main__":
    main()
