"""Packed-weight files (g4b.packfile) on CPU: quant()'s buffers written to a
safetensors file and read back byte for byte, checked against the golden
vectors the reference's own quant() produced (tests/golden/quant_golden.npz),
plus the error paths."""
import json
import os

import numpy as np
import pytest

from g4b import pack, packfile

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "quant_golden.npz")


def _golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("tag", ["f16", "fp8"])
def test_round_trip_is_byte_identical_to_the_reference_quant(tmp_path, tag):
    g = _golden()
    cases = ["rand_64x128", "rand_128x256", "rand_48x96_wide", "edge_32x128"]
    ws = {c: pack.quant(g[f"{c}/W"], pf=True, fp8=tag == "fp8", prefill_i8=True) for c in cases}
    path = str(tmp_path / "w.safetensors")
    packfile.save(path, ws)
    back = packfile.load(path)
    assert list(back) == cases
    for c in cases:
        b = back[c]
        # the bytes the reference's own quant() uploaded for the same W (bw, bs, bs16, w8, sw8) and its
        # split, nblk and inv
        assert b.wp.tobytes() == g[f"{c}/{tag}/wp"].tobytes()
        assert b.scales.tobytes() == g[f"{c}/{tag}/scales"].tobytes()
        assert b.scales16.tobytes() == g[f"{c}/{tag}/scales16"].tobytes()
        assert b.w8.tobytes() == g[f"{c}/{tag}/w8"].tobytes()
        assert b.sw8.tobytes() == g[f"{c}/{tag}/sw8"].tobytes()
        assert b.split == int(g[f"{c}/{tag}/split"]) and b.nblk == int(g[f"{c}/{tag}/nblk"])
        assert b.inv == float(g[f"{c}/{tag}/inv"])
        # and every field equals the packer's
        a = ws[c]
        for f in ("wp", "scales", "scales16", "w8", "sw8"):
            assert getattr(a, f).tobytes() == getattr(b, f).tobytes(), (c, f)
        assert (a.N, a.K, a.nblk, a.split, a.scale_fmt, a.inv) == (b.N, b.K, b.nblk, b.split, b.scale_fmt, b.inv)


def test_selected_names_and_lm_head_without_int8(tmp_path):
    rng = np.random.default_rng(3)
    ws = {"layers.0.q": pack.quant((rng.standard_normal((256, 512)) * 0.02).astype(np.float32), pf=True,
                                   fp8=False, prefill_i8=True),
          "lm_head": pack.quant((rng.standard_normal((512, 256)) * 0.02).astype(np.float32), pf=False,
                                fp8=False, prefill_i8=True)}
    path = str(tmp_path / "m.safetensors")
    packfile.save(path, ws)
    h = packfile.read_header(path)
    assert h["format"] == packfile.FORMAT and set(h["weights"]) == set(ws)
    only = packfile.load(path, names=["lm_head"])
    assert list(only) == ["lm_head"] and only["lm_head"].w8 is None
    assert only["lm_head"].as_reference_tuple()[0].tobytes() == ws["lm_head"].wp.tobytes()
    with pytest.raises(KeyError):
        packfile.load(path, names=["missing"])


def test_foreign_and_inconsistent_files_are_refused(tmp_path):
    from safetensors.numpy import save_file

    p1 = str(tmp_path / "plain.safetensors")
    save_file({"x": np.zeros(4, np.float32)}, p1)
    with pytest.raises(ValueError, match="not a g4b packed-weight file"):
        packfile.load(p1)
    pw = pack.quant((np.random.default_rng(0).standard_normal((64, 128)) * 0.02).astype(np.float32), fp8=False,
                    prefill_i8=False)
    # a header that claims another K than the stored words have
    meta = {"format": packfile.FORMAT, "version": 1, "block": 32,
            "weights": {"w": {"N": 64, "K": 256, "nblk": 8, "split": 1, "scale_fmt": 0, "inv": 1.0}}}
    p2 = str(tmp_path / "bad.safetensors")
    save_file({"w.wp": pw.wp, "w.scales": pw.scales}, p2, metadata={packfile.META_KEY: json.dumps(meta)})
    with pytest.raises(ValueError, match="w.wp"):
        packfile.load(p2)
    meta["version"] = 99
    save_file({"w.wp": pw.wp, "w.scales": pw.scales}, p2, metadata={packfile.META_KEY: json.dumps(meta)})
    with pytest.raises(ValueError, match="version"):
        packfile.load(p2)
