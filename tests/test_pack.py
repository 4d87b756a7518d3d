"""The product's host packer (g4b.pack) against the reference's own quant()
output (golden vectors) and against the oracle restatement."""
import json
import os

import numpy as np
import pytest

import oracle as O
from g4b import pack

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quant_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("tag,fp8", [("f16", False), ("fp8", True)])
def test_pack_matches_reference_quant(golden, tag, fp8):
    for name in json.loads(bytes(golden["meta_json"]).decode())["cases"]:
        p = pack.quant(golden[f"{name}/W"], True, fp8=fp8, prefill_i8=True)
        pre = f"{name}/{tag}"
        wp, bs, split, nblk, inv, bs16, w8, sw8 = p.as_reference_tuple()
        assert np.array_equal(wp.reshape(-1), golden[f"{pre}/wp"])
        assert np.array_equal(np.ascontiguousarray(bs).view(np.uint8).reshape(-1), golden[f"{pre}/scales"])
        assert np.array_equal(bs16.view(np.uint16).reshape(-1), golden[f"{pre}/scales16"])
        assert (split, nblk, inv) == (int(golden[f"{pre}/split"]), int(golden[f"{pre}/nblk"]), float(golden[f"{pre}/inv"]))
        assert np.array_equal(w8.reshape(-1), golden[f"{pre}/w8"])
        assert np.array_equal(sw8.view(np.uint16).reshape(-1), golden[f"{pre}/sw8"])


def test_pack_lm_head_has_no_int8(golden):
    p = pack.quant(golden["rand_64x128/W"], pf=False, prefill_i8=True)
    assert p.w8 is None and p.sw8 is None


def test_pack_split_table(golden):
    for N, K, s in golden["split_table"]:
        assert pack.split_for(int(N), int(K) // 32) == int(s)


@pytest.mark.parametrize("N,K,seed", [(512, 1024, 11), (1024, 3840, 12)])
def test_pack_matches_oracle_larger(N, K, seed):
    W = (np.random.default_rng(seed).standard_normal((N, K)) * 0.02).astype(np.float32)
    for fp8 in (False, True):
        p = pack.quant(W, fp8=fp8, prefill_i8=True)
        r = O.pack_reference(W, fp8=fp8, prefill_i8=True)
        assert np.array_equal(p.wp, r["wp"])
        assert np.array_equal(np.ascontiguousarray(p.scales).view(np.uint8), np.ascontiguousarray(r["scales"]).view(np.uint8))
        assert np.array_equal(p.w8, r["w8"]) and np.array_equal(p.sw8.view(np.uint16), r["sw8"])
        assert p.inv == r["inv"] and p.split == r["split"]


def test_pack_rejects_bad_shapes():
    with pytest.raises(ValueError):
        pack.quant(np.zeros((16, 48), np.float32))
    with pytest.raises(ValueError):
        pack.quant(np.zeros((12, 64), np.float32))


def test_w4a8_ratio_matches_oracle():
    W = (np.random.default_rng(9).standard_normal((64, 256)) * 0.08).astype(np.float32)
    p = pack.quant(W, prefill_i8=True)
    r = O.pack_reference(W, prefill_i8=True)
    ratio = pack.w4a8_ratio(p.sc_f32, p.sw_f32)
    assert np.array_equal(ratio.view(np.uint16), O.w4a8_ratio(r["sc_f32"], r["sw_f32"]))
