"""Packed on-disk weight format (cutilegpt_b200/models/packed.py): CPU round trip, tying, rejection."""
import os
import struct

import pytest
import torch

from cutilegpt_b200.models import packed
from cutilegpt_b200.models.config import GPTConfig
from cutilegpt_b200.models.init import init_state


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("tied", [True, False])
def test_round_trip(tmp_path, dtype, tied):
    cfg = GPTConfig(n_layer=2, n_head=2, n_embd=32, vocab_size=101, block_size=16)
    w = {k: v.to(dtype) for k, v in init_state(cfg, 3).items()}
    w["lm_head.weight"] = w["wte"] if tied else torch.randn_like(w["wte"])
    path = str(tmp_path / "m.cgpt")
    packed.save(path, cfg, w, tied)
    header, data0 = packed.read_header(path)
    assert data0 % packed.ALIGN == 0 and all(e["offset"] % packed.ALIGN == 0 for e in header["tensors"].values())
    assert ("lm_head.weight" in header["tensors"]) == (not tied)
    cfg2, dt2, w2 = packed.load(path, torch.device("cpu"))
    assert cfg2 == cfg and dt2 == dtype and set(w2) == set(w)
    for k in w:
        assert torch.equal(w2[k], w[k]), k
    assert (w2["lm_head.weight"] is w2["wte"]) == tied


def test_rejects_foreign_and_truncated_files(tmp_path):
    cfg = GPTConfig(n_layer=1, n_head=2, n_embd=16, vocab_size=50, block_size=8)
    w = init_state(cfg, 4)
    path = str(tmp_path / "m.cgpt")
    packed.save(path, cfg, w, True)
    bad = tmp_path / "bad.cgpt"
    bad.write_bytes(b"NOTAMODEL" + b"\0" * 100)
    with pytest.raises(ValueError):
        packed.load(str(bad), torch.device("cpu"))
    raw = open(path, "rb").read()
    short = tmp_path / "short.cgpt"
    short.write_bytes(raw[: len(raw) // 2])
    with pytest.raises(ValueError):
        packed.load(str(short), torch.device("cpu"))
    huge = tmp_path / "huge.cgpt"
    huge.write_bytes(packed.MAGIC + struct.pack("<Q", 1 << 40))
    with pytest.raises(ValueError):
        packed.read_header(str(huge))
    with pytest.raises(ValueError):
        packed.save(str(tmp_path / "mixed.cgpt"), cfg, {**w, "wte": w["wte"].bfloat16()}, True)
    assert not os.path.exists(str(tmp_path / "mixed.cgpt"))
