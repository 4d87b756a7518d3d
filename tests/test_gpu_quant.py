"""GPU packing (g4b_quant_i4 / g4b_quant_e4m3 / g4b_quant_w8a8) bit-exact to the
reference's own quant() output (golden vectors) and to the host packer."""
import json
import os

import numpy as np
import pytest
import torch

from g4b import pack
from g4b.quant_gpu import quant_device

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quant_golden.npz")


def _np(t):
    return t.cpu().numpy()


@pytest.mark.parametrize("tag,fp8", [("f16", False), ("fp8", True)])
def test_quant_device_matches_reference_quant(tag, fp8):
    g = np.load(GOLDEN)
    for name in json.loads(bytes(g["meta_json"]).decode())["cases"]:
        W = torch.from_numpy(g[f"{name}/W"]).cuda()
        d = quant_device(W, True, fp8=fp8, prefill_i8=True)
        pre = f"{name}/{tag}"
        assert np.array_equal(_np(d.wp).view(np.uint32).reshape(-1), g[f"{pre}/wp"]), name
        assert np.array_equal(np.ascontiguousarray(_np(d.scales)).view(np.uint8).reshape(-1), g[f"{pre}/scales"]), name
        assert np.array_equal(_np(d.scales16).view(np.uint16).reshape(-1), g[f"{pre}/scales16"]), name
        assert d.inv == float(g[f"{pre}/inv"]) and d.split == int(g[f"{pre}/split"]), name
        assert np.array_equal(_np(d.w8).reshape(-1), g[f"{pre}/w8"]), name
        assert np.array_equal(_np(d.sw8).view(np.uint16).reshape(-1), g[f"{pre}/sw8"]), name


@pytest.mark.parametrize("N,K", [(4096, 3840), (3840, 15360), (1024, 64)])
def test_quant_device_matches_host_packer(N, K):
    W = (np.random.default_rng(N + K).standard_normal((N, K)) * 0.02).astype(np.float32)
    for fp8 in (False, True):
        p = pack.quant(W, fp8=fp8, prefill_i8=True)
        d = quant_device(torch.from_numpy(W).cuda(), fp8=fp8, prefill_i8=True, w4a8=True)
        assert np.array_equal(_np(d.wp).view(np.uint32), p.wp)
        assert np.array_equal(np.ascontiguousarray(_np(d.scales)).view(np.uint8),
                              np.ascontiguousarray(p.scales).view(np.uint8))
        assert d.inv == p.inv
        assert np.array_equal(_np(d.w8), p.w8)
        assert np.array_equal(_np(d.sw8).view(np.uint16), p.sw8.view(np.uint16))
        ratio = pack.w4a8_ratio(p.sc_f32, p.sw_f32)
        assert np.array_equal(_np(d.ratio16).view(np.uint16), ratio.view(np.uint16))
