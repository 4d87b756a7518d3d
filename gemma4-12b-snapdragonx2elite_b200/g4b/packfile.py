"""Packed-weight files: quant()'s output saved once and loaded straight back.

The reference re-quantises every weight at each start-up: its engine calls
quant() per linear layer while it builds the Vulkan buffers
(src/vk_engine.py:186, 198-199, 209), which takes about four minutes for the
12B model (service/README.md:7-9).  A packed file holds exactly the buffers
quant() uploads, so loading is a read and a host-to-device copy.

Format: a safetensors file (a JSON header followed by raw little-endian
tensors), with, for every weight <name>:

  <name>.wp        uint32  [K, N/8]   packed nibbles, quant()'s ``bw``
  <name>.scales    float16 [nblk, N]  (f16 scales) or uint8 [nblk, N] (e4m3
                                      bytes, GEMV_FP8), quant()'s ``bs``
  <name>.scales16  float16 [nblk, N]  the prefill GEMM's f16 scales, ``bs16``
                                      (stored only with e4m3 scales; with f16
                                      scales it is ``bs`` itself)
  <name>.w8        int8    [K, N]     W8A8 prefill weights (PREFILL_I8)
  <name>.sw8       float16 [N]        their per-row scale s_w
  <name>.ratio16   float16 [nblk, N]  W4A8 requant ratio f16(scale / s_w)
                                      (optional, benchmarks/coopgemm_w4a8.py:84)

and the metadata entry "g4b.packed", a JSON object
``{"format": "g4b-packed-int4", "version": 1, "block": 32, "weights":
{<name>: {"N", "K", "nblk", "split", "scale_fmt", "inv"}}}`` carrying the rest
of quant()'s tuple (split, nblk, inv) and the scale format.  Every array is
written byte for byte as quant() (or the GPU packer, which is bit-exact to
it) produced it, so a loaded weight is the packed weight.
"""
from __future__ import annotations

import json
from typing import Dict, Iterable, Optional, Union

import numpy as np

from .pack import BLK, PackedWeight

FORMAT = "g4b-packed-int4"
VERSION = 1
META_KEY = "g4b.packed"


def _host(a):
    """numpy view of a numpy array or a (device) torch tensor, on the host."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return np.ascontiguousarray(a)
    t = a.detach()
    if t.is_cuda:
        t = t.cpu()
    return np.ascontiguousarray(t.numpy())


def _fields(w):
    """The arrays and metadata of a PackedWeight (host) or a g4b.ops.DeviceWeight."""
    wp = _host(w.wp)
    if wp.dtype != np.uint32:
        wp = wp.view(np.uint32)
    scales = _host(w.scales)
    scales16 = _host(w.scales16)
    arrays = {"wp": wp, "scales": scales}
    if int(w.scale_fmt) != 0:
        arrays["scales16"] = scales16
    w8 = _host(getattr(w, "w8", None))
    if w8 is not None:
        arrays["w8"] = w8
        arrays["sw8"] = _host(w.sw8)
    ratio = _host(getattr(w, "ratio16", None))
    if ratio is not None:
        arrays["ratio16"] = ratio
    meta = {"N": int(w.N), "K": int(w.K), "nblk": int(w.nblk), "split": int(w.split),
            "scale_fmt": int(w.scale_fmt), "inv": float(w.inv)}
    return arrays, meta


def _check(name: str, m: dict, arrays: dict) -> None:
    """Shapes and dtypes of one weight's arrays against its metadata."""
    N, K, nblk, fmt = m["N"], m["K"], m["nblk"], m["scale_fmt"]
    if K % BLK or N % 8 or nblk != K // BLK or fmt not in (0, 1):
        raise ValueError(f"packfile: weight {name!r} has inconsistent sizes N={N} K={K} nblk={nblk} fmt={fmt}")
    want = {"wp": ((K, N // 8), np.uint32),
            "scales": ((nblk, N), np.float16 if fmt == 0 else np.uint8),
            "scales16": ((nblk, N), np.float16),
            "w8": ((K, N), np.int8), "sw8": ((N,), np.float16), "ratio16": ((nblk, N), np.float16)}
    for key, a in arrays.items():
        shape, dt = want[key]
        if tuple(a.shape) != shape or a.dtype != dt:
            raise ValueError(f"packfile: {name}.{key} is {a.dtype}{tuple(a.shape)}, expected "
                             f"{np.dtype(dt)}{shape}")
    for key in ("wp", "scales"):
        if key not in arrays:
            raise ValueError(f"packfile: weight {name!r} has no {key!r} tensor")
    if fmt == 1 and "scales16" not in arrays:
        raise ValueError(f"packfile: weight {name!r} has e4m3 scales but no scales16 tensor")
    if ("w8" in arrays) != ("sw8" in arrays):
        raise ValueError(f"packfile: weight {name!r} has only one of w8 / sw8")


def save(path: str, weights: Dict[str, object]) -> None:
    """Write packed weights (g4b.pack.PackedWeight or g4b.ops.DeviceWeight,
    e.g. from g4b.quant_gpu.quant_device) to one safetensors file."""
    from safetensors.numpy import save_file

    tensors, meta = {}, {}
    for name, w in weights.items():
        if "." in name.split("/")[-1] and name.rsplit(".", 1)[-1] in ("wp", "scales", "scales16", "w8", "sw8",
                                                                     "ratio16"):
            raise ValueError(f"packfile: weight name {name!r} ends in a reserved tensor suffix")
        arrays, m = _fields(w)
        _check(name, m, arrays)
        meta[name] = m
        for key, a in arrays.items():
            tensors[f"{name}.{key}"] = a
    header = {"format": FORMAT, "version": VERSION, "block": BLK, "weights": meta}
    save_file(tensors, path, metadata={META_KEY: json.dumps(header)})


def read_header(path: str) -> dict:
    """The file's "g4b.packed" metadata, checked for format and version."""
    from safetensors import safe_open

    with safe_open(path, framework="numpy") as f:
        md = f.metadata() or {}
    if META_KEY not in md:
        raise ValueError(f"packfile: {path} has no {META_KEY!r} metadata: not a g4b packed-weight file")
    h = json.loads(md[META_KEY])
    if h.get("format") != FORMAT or h.get("version") != VERSION or h.get("block") != BLK:
        raise ValueError(f"packfile: {path} is {h.get('format')!r} version {h.get('version')!r} block "
                         f"{h.get('block')!r}; this reader takes {FORMAT!r} version {VERSION} block {BLK}")
    return h


def _names(h: dict, names: Optional[Iterable[str]]):
    allw = h["weights"]
    if names is None:
        return list(allw)
    names = list(names)
    missing = [n for n in names if n not in allw]
    if missing:
        raise KeyError(f"packfile: no weight(s) {missing} in the file")
    return names


def load(path: str, names: Optional[Iterable[str]] = None) -> Dict[str, PackedWeight]:
    """Read packed weights into host PackedWeight objects (quant()'s return,
    ``PackedWeight.as_reference_tuple()``), byte for byte as saved."""
    from safetensors import safe_open

    h = read_header(path)
    out = {}
    with safe_open(path, framework="numpy") as f:
        keys = set(f.keys())
        for name in _names(h, names):
            m = h["weights"][name]
            arrays = {k: f.get_tensor(f"{name}.{k}") for k in ("wp", "scales", "scales16", "w8", "sw8", "ratio16")
                      if f"{name}.{k}" in keys}
            _check(name, m, arrays)
            out[name] = PackedWeight(
                N=m["N"], K=m["K"], wp=arrays["wp"], scales=arrays["scales"], scale_fmt=m["scale_fmt"],
                inv=float(m["inv"]), split=m["split"], nblk=m["nblk"],
                scales16=arrays.get("scales16", arrays["scales"] if m["scale_fmt"] == 0 else None),
                w8=arrays.get("w8"), sw8=arrays.get("sw8"))
            if "ratio16" in arrays:
                out[name].ratio16 = arrays["ratio16"]
    return out


def load_device(path: str, device: Union[str, "torch.device"] = "cuda",  # noqa: F821
                names: Optional[Iterable[str]] = None) -> dict:
    """Read packed weights straight into device memory as g4b.ops.DeviceWeight
    objects: each tensor is read from the file and copied to the device once;
    nothing is quantised."""
    import torch
    from safetensors import safe_open

    from .ops import DeviceWeight

    dev = torch.device(device)
    h = read_header(path)
    out = {}
    with safe_open(path, framework="pt", device="cpu") as f:
        keys = set(f.keys())
        for name in _names(h, names):
            m = h["weights"][name]
            t = {k: f.get_tensor(f"{name}.{k}") for k in ("wp", "scales", "scales16", "w8", "sw8", "ratio16")
                 if f"{name}.{k}" in keys}
            _check(name, m, {k: v.numpy() for k, v in t.items()})
            d = {k: v.to(dev, non_blocking=False) for k, v in t.items()}
            out[name] = DeviceWeight(
                N=m["N"], K=m["K"], nblk=m["nblk"], split=m["split"], scale_fmt=m["scale_fmt"], inv=float(m["inv"]),
                wp=d["wp"].view(torch.int32), scales=d["scales"],
                scales16=d.get("scales16", d["scales"] if m["scale_fmt"] == 0 else None),
                w8=d.get("w8"), sw8=d.get("sw8"), ratio16=d.get("ratio16"))
    return out
