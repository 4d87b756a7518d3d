"""Packed-weight files on the GPU: weights packed by the GPU packer, saved and
loaded straight into device memory are the same bytes, and the decode GEMV on
them gives the same bits as on freshly packed weights (and matches the oracle)."""
import numpy as np
import pytest
import torch

import oracle as O
from g4b import ops, pack, packfile
from g4b import quant_gpu as qz
from util import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fp8", [False, True])
def test_device_pack_save_load_round_trip(tmp_path, fp8):
    gen = torch.Generator(device="cuda").manual_seed(0)
    W = torch.randn((4096, 3840), generator=gen, device="cuda").mul_(0.02)
    dw = qz.quant_device(W, pf=True, fp8=fp8, prefill_i8=True)
    path = str(tmp_path / "w.safetensors")
    packfile.save(path, {"q": dw})
    back = packfile.load_device(path, "cuda")["q"]
    for f in ("wp", "scales", "scales16", "w8", "sw8"):
        assert torch.equal(getattr(back, f).view(torch.uint8), getattr(dw, f).view(torch.uint8)), f
    assert (back.N, back.K, back.split, back.nblk, back.scale_fmt, back.inv) == \
        (dw.N, dw.K, dw.split, dw.nblk, dw.scale_fmt, dw.inv)
    # and the host packer agrees with the GPU packer byte for byte
    host = pack.quant(W.cpu().numpy(), pf=True, fp8=fp8, prefill_i8=True)
    assert back.wp.cpu().numpy().view(np.uint32).tobytes() == host.wp.tobytes()
    assert back.scales.cpu().numpy().tobytes() == host.scales.tobytes()


def test_gemv_on_loaded_weights(tmp_path):
    rng = np.random.default_rng(1)
    Wn = (rng.standard_normal((15360, 3840)) * 0.02).astype(np.float32)
    pw = pack.quant(Wn, pf=False, fp8=False, prefill_i8=False)
    path = str(tmp_path / "gate.safetensors")
    packfile.save(path, {"gate": pw})
    dw = packfile.load_device(path, "cuda")["gate"]
    x = torch.from_numpy(rng.standard_normal(3840).astype(np.float16)).cuda()
    y = ops.gemv_i4(x, dw, out_dtype=torch.float32)
    y_ref = ops.gemv_i4(x, ops.to_device(pw, "cuda"), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    want = O.gemv(x.float().cpu().numpy(), pw.wp, pw.scales.view(np.uint16), 0, 1.0, pw.N, pw.K, pw.split)
    assert_close(y.cpu().numpy(), want, "gemv on loaded weights vs oracle")
