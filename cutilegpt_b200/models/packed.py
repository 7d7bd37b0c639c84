"""Packed on-disk weight format for fast replica start-up.

One file per model: an 8-byte magic, a little-endian uint64 header length, a
UTF-8 JSON header (config, dtype, tensor table), then every tensor's raw
bytes at 4 KiB-aligned offsets, already in the layout the kernels read
(Linear weights [out, in], K-major, in the compute dtype). Loading maps the
file and copies each tensor straight to the device: no transposes, no dtype
conversion, no pickle. A tied lm_head is stored once (``"lm_head.weight":
"wte"`` in the header).

This is the "packed bf16 on-disk format" of the weight-ingestion path; the
reference's own loaders (cutile_gpt/models/gpt.py:231-343) read HF / minGPT
state dicts and transpose on every load.
"""
from __future__ import annotations

import json
import os
import struct
from typing import Dict, Tuple

import numpy as np
import torch

from .config import GPTConfig

MAGIC = b"CGPTB200"
VERSION = 1
ALIGN = 4096
_DTYPES = {torch.bfloat16: "bf16", torch.float32: "f32"}
_TORCH = {v: k for k, v in _DTYPES.items()}


def save(path: str, config: GPTConfig, weights: Dict[str, torch.Tensor], tied: bool) -> None:
    """Writes `weights` (one dtype, the model's) and `config` to `path`."""
    dtypes = {t.dtype for t in weights.values()}
    if len(dtypes) != 1 or next(iter(dtypes)) not in _DTYPES:
        raise ValueError(f"packed format needs one dtype of {list(_DTYPES)}, got {dtypes}")
    dt = next(iter(dtypes))
    table, blobs, off = {}, [], 0
    for name in sorted(weights):
        if tied and name == "lm_head.weight":
            continue
        t = weights[name].detach().contiguous().cpu()
        nbytes = t.numel() * t.element_size()
        table[name] = {"shape": list(t.shape), "offset": off, "nbytes": nbytes}
        blobs.append((off, t))
        off += (nbytes + ALIGN - 1) // ALIGN * ALIGN
    header = {"version": VERSION, "dtype": _DTYPES[dt],
              "config": {k: getattr(config, k) for k in ("vocab_size", "block_size", "n_layer", "n_head", "n_embd")},
              "tensors": table, "tied": {"lm_head.weight": "wte"} if tied else {}}
    hb = json.dumps(header, sort_keys=True).encode()
    data0 = (len(MAGIC) + 8 + len(hb) + ALIGN - 1) // ALIGN * ALIGN
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for o, t in blobs:
            f.seek(data0 + o)
            f.write(t.view(torch.uint8).numpy().tobytes() if t.dtype == torch.bfloat16 else t.numpy().tobytes())
        f.truncate(data0 + off)
    os.replace(tmp, path)


def read_header(path: str) -> Tuple[dict, int]:
    """(header, byte offset of the tensor data); raises ValueError on a foreign or damaged file."""
    with open(path, "rb") as f:
        magic = f.read(len(MAGIC))
        if magic != MAGIC:
            raise ValueError(f"{path}: not a packed cutilegpt_b200 weight file")
        (hl,) = struct.unpack("<Q", f.read(8))
        if hl > 64 << 20:
            raise ValueError(f"{path}: header length {hl} is not plausible")
        header = json.loads(f.read(hl).decode())
    if header.get("version") != VERSION:
        raise ValueError(f"{path}: unsupported packed format version {header.get('version')}")
    data0 = (len(MAGIC) + 8 + hl + ALIGN - 1) // ALIGN * ALIGN
    return header, data0


def load(path: str, device: torch.device) -> Tuple[GPTConfig, torch.dtype, Dict[str, torch.Tensor]]:
    """(config, dtype, weight dict on `device`) from a packed file (memory-mapped, one copy per tensor)."""
    header, data0 = read_header(path)
    dt = _TORCH[header["dtype"]]
    cfg = GPTConfig(**header["config"])
    size = os.path.getsize(path)
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out: Dict[str, torch.Tensor] = {}
    esize = torch.tensor([], dtype=dt).element_size()
    for name, e in header["tensors"].items():
        o, n = data0 + int(e["offset"]), int(e["nbytes"])
        shape = tuple(int(x) for x in e["shape"])
        if o + n > size or n != int(np.prod(shape, dtype=np.int64)) * esize:
            raise ValueError(f"{path}: tensor {name} is out of bounds or mis-sized")
        raw = torch.from_numpy(np.array(mm[o:o + n]))          # host copy of the slice
        out[name] = raw.view(dt).view(shape).to(device, non_blocking=False)
    for alias, src in header.get("tied", {}).items():
        out[alias] = out[src]
    del mm
    return cfg, dt, out
