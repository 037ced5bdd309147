"""Offline weight-pack files: the K-major operand packs of every routed linear, written
once and loaded without re-quantising.

The reference quantises every nn.Linear at load time (``quantize_weights_int8`` and a
transpose, EE/python/dispatch.py:43-48, :115-124) and keeps the int8 [K, N] buffer and its
scales.  The tensor-core kernels here read three K-major packs per weight -- int8, e4m3
and fp16 [N, K] -- plus the fp32 per-channel scale (``WeightPack``); a pack file stores
exactly those, so a model loads by copying bytes.

File layout (little endian):
  bytes 0..7    magic b"EEPACK01"
  bytes 8..15   header length h (uint64)
  bytes 16..    header: UTF-8 JSON {"packs": {name: {"K": K, "N": N,
                "w_i8": [offset, nbytes], "w_e4m3": [...], "w_f16": [...], "scale": [...]}}}
  then the arrays, each starting at a multiple of 256 bytes from the file start:
  int8 [N, K], uint8 e4m3 codes [N, K], fp16 [N, K], fp32 [N].
"""
from __future__ import annotations

import json
import os
import struct
from typing import Dict

import numpy as np
import torch

MAGIC = b"EEPACK01"
_FIELDS = (("w_i8", np.int8, torch.int8), ("w_e4m3", np.uint8, torch.uint8), ("w_f16", np.float16, torch.float16),
           ("scale", np.float32, torch.float32))


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


def save_packs(path: str, packs: Dict[str, object]) -> None:
    """Write named packs (objects with K, N, w_i8, w_e4m3, w_f16, scale) to ``path``."""
    arrays, header = [], {"packs": {}}
    for name, p in packs.items():
        K, N = int(p.K), int(p.N)
        entry = {"K": K, "N": N}
        for field, np_t, _ in _FIELDS:
            a = getattr(p, field).detach().contiguous().cpu().numpy().astype(np_t, copy=False)
            want = (N,) if field == "scale" else (N, K)
            if a.shape != want:
                raise RuntimeError(f"{name}.{field} has shape {a.shape}, expected {want}")
            arrays.append((name, field, a))
            entry[field] = [0, int(a.nbytes)]
        header["packs"][name] = entry
    # offsets depend on the header's length; fix the point with the widest offsets first
    for _ in range(3):
        blob = json.dumps(header, sort_keys=True).encode()
        off = _align(16 + len(blob) + 64)  # room for the offsets to grow by a few digits
        for name, field, a in arrays:
            header["packs"][name][field][0] = off
            off = _align(off + a.nbytes)
    blob = json.dumps(header, sort_keys=True).encode()
    first = min((e[f][0] for e in header["packs"].values() for f, _, _ in _FIELDS), default=16 + len(blob))
    if 16 + len(blob) > first:
        raise RuntimeError("pack-file header layout failed")
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<Q", len(blob)))
        f.write(blob)
        for name, field, a in arrays:
            f.seek(header["packs"][name][field][0])
            f.write(a.tobytes())
    os.replace(tmp, path)


class LoadedPack:
    """The four arrays of one pack, as torch tensors on ``device`` (same fields as
    WeightPack, which ``to_weight_pack`` builds without recomputing anything)."""

    def __init__(self, K: int, N: int, tensors: dict):
        self.K, self.N = K, N
        for k, v in tensors.items():
            setattr(self, k, v)

    def to_weight_pack(self):
        from .kernels import WeightPack

        return WeightPack.from_arrays(self.w_i8, self.w_e4m3, self.w_f16, self.scale)


def load_packs(path: str, device="cpu") -> Dict[str, LoadedPack]:
    """Read every pack of a file written by ``save_packs``; the arrays are placed on
    ``device`` (a CUDA device: staged through pinned host memory)."""
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        if f.read(8) != MAGIC:
            raise RuntimeError(f"{path} is not a weight-pack file (bad magic)")
        (hlen,) = struct.unpack("<Q", f.read(8))
        if 16 + hlen > size:
            raise RuntimeError(f"{path}: truncated header")
        header = json.loads(f.read(hlen).decode())
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    device = torch.device(device)
    out = {}
    for name, e in header["packs"].items():
        K, N = int(e["K"]), int(e["N"])
        tensors = {}
        for field, np_t, t_t in _FIELDS:
            off, nbytes = e[field]
            count = N if field == "scale" else N * K
            if nbytes != count * np.dtype(np_t).itemsize or off % 256 or off + nbytes > size:
                raise RuntimeError(f"{path}: {name}.{field} is malformed or truncated")
            a = np.frombuffer(mm, dtype=np_t, count=count, offset=off).reshape((N,) if field == "scale" else (N, K))
            t = torch.from_numpy(a.copy())
            if device.type == "cuda":
                t = t.pin_memory().to(device, non_blocking=True)
            tensors[field] = t
        out[name] = LoadedPack(K, N, tensors)
    if device.type == "cuda":
        torch.cuda.synchronize(device)
    return out


def save_dispatched_llama(blocks, path: str) -> None:
    """Write the packs of every routed linear of ``build_dispatched_llama``'s blocks
    (names ``layers.<i>.<gate_proj|up_proj|down_proj|qkv_proj|o_proj>``)."""
    packs = {}
    for i, blk in enumerate(blocks):
        for name in ("gate_proj", "up_proj", "down_proj", "qkv_proj", "o_proj"):
            lin = getattr(blk, name, None)
            if lin is not None:
                packs[f"layers.{i}.{name}"] = lin._pack()
    save_packs(path, packs)
