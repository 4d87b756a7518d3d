"""The CPU oracle pinned to the reference: golden packing vectors produced by
running the reference's own quant() (tests/golden/make_golden.py), plus the
numeric conversions the oracle relies on, checked exhaustively against numpy
and torch."""
import json
import os

import numpy as np
import pytest
import torch

import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quant_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def _cases(g):
    return json.loads(bytes(g["meta_json"]).decode())["cases"]


@pytest.mark.parametrize("tag,fp8", [("f16", False), ("fp8", True)])
def test_oracle_packing_matches_reference_quant(golden, tag, fp8):
    for name in _cases(golden):
        W = golden[f"{name}/W"]
        r = O.pack_reference(W, fp8=fp8, prefill_i8=True)
        pre = f"{name}/{tag}"
        assert np.array_equal(r["wp"].reshape(-1), golden[f"{pre}/wp"]), name
        assert np.array_equal(np.ascontiguousarray(r["scales"]).view(np.uint8).reshape(-1), golden[f"{pre}/scales"]), name
        assert np.array_equal(r["scales16"].reshape(-1), golden[f"{pre}/scales16"]), name
        assert r["split"] == int(golden[f"{pre}/split"]), name
        assert r["nblk"] == int(golden[f"{pre}/nblk"]), name
        assert r["inv"] == float(golden[f"{pre}/inv"]), name
        assert np.array_equal(r["w8"].reshape(-1), golden[f"{pre}/w8"]), name
        assert np.array_equal(r["sw8"].reshape(-1), golden[f"{pre}/sw8"]), name


def test_oracle_split_table_matches_reference(golden):
    table = golden["split_table"]
    assert len(table) >= 6
    for N, K, split in table:
        assert O.split_for(int(N), int(K) // 32) == int(split), (N, K)


def test_lm_head_packing_skips_int8(golden):
    assert int(golden["rand_64x128/f16_nopf/has_w8"]) == 0


def test_f16_decode_all_patterns():
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([O.lib().orc_f16_to_f32(int(v)) for v in h], np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_f16_encode_rne():
    rng = np.random.default_rng(3)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 5, 20000).astype(np.float32),
        np.array([0.0, -0.0, 65504.0, 65520.0, 65519.99, 1e-8, 2.0 ** -25, 2.0 ** -24, 3 * 2.0 ** -26,
                  6.1e-5, 2.0 ** -14, 1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11], np.float32),
    ]).astype(np.float32)
    ref = x.astype(np.float16).view(np.uint16)
    got = np.array([O.lib().orc_f32_to_f16(float(v)) for v in x], np.uint16)
    assert np.array_equal(got, ref)


def test_e4m3_decode_matches_torch_except_nan_codes():
    codes = np.arange(256, dtype=np.uint8)
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    got = O.e4m3_decode(codes)
    finite = ~np.isnan(ref)
    assert np.array_equal(got[finite], ref[finite])
    # the shader decodes the two NaN codes as +-480 (vk/gemv_fp8.comp:14-18)
    assert got[0x7F] == 480.0 and got[0xFF] == -480.0


def test_e4m3_encode_matches_torch():
    rng = np.random.default_rng(4)
    grid = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    grid = grid[np.isfinite(grid) & (np.abs(grid) <= 448)]
    mids = []
    srt = np.unique(np.abs(grid))
    mids = (srt[1:] + srt[:-1]) / 2                       # exact ties -> round-half-even
    x = np.concatenate([rng.uniform(0, 448, 20000), rng.uniform(0, 2 ** -5, 5000), mids, -mids, srt,
                        np.nextafter(mids.astype(np.float32), np.float32(0)),
                        np.nextafter(mids.astype(np.float32), np.float32(1000))]).astype(np.float32)
    x = x[np.abs(x) <= 448]
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    got = O.e4m3_encode(x)
    assert np.array_equal(got, ref)


def test_oracle_gemv_partials_reduce_consistently():
    rng = np.random.default_rng(5)
    N, K, split = 64, 256, 4
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    r = O.pack_reference(W)
    x = rng.standard_normal(K).astype(np.float32)
    y, part = O.gemv(x, r["wp"], r["scales"], 0, 1.0, N, K, split, want_partial=True)
    assert np.array_equal(O.reduce(part.reshape(split, N), N, split), y)
