"""ShardedGPT with a real CutileGPT on the GPU, over an NCCL process group.

One GPU is enough here: a world-size-1 NCCL group runs the real collective
(all_gather of CUDA tensors through NCCL) and ShardedGPT drives the real
model. The two-rank sharding logic itself is covered with gloo ranks on the
CPU in test_distributed.py.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist

from cutilegpt_b200 import CutileGPT, GPTConfig
from cutilegpt_b200.distributed import ShardedGPT, gather_batch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture
def nccl_group():
    assert not dist.is_initialized()
    store = dist.TCPStore("127.0.0.1", _free_port(), 1, True, timeout=datetime.timedelta(seconds=30))
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", store=store, rank=0, world_size=1, timeout=datetime.timedelta(seconds=30),
                            device_id=torch.device("cuda", 0))
    yield
    dist.destroy_process_group()


def test_sharded_real_model_matches_unsharded(nccl_group):
    cfg = GPTConfig(n_layer=2, n_head=12, n_embd=768, vocab_size=50257, block_size=1024)
    m = CutileGPT(cfg, dtype=torch.bfloat16, device="cuda", seed=3)
    idx = torch.randint(0, cfg.vocab_size, (4, 32), generator=torch.Generator().manual_seed(5)).cuda()
    sg = ShardedGPT(m)
    sg.time_gather = True
    ref_seq = m.generate(idx, 8, top_k=1)
    assert torch.equal(sg.generate(idx, 8, top_k=1), ref_seq)
    logits, last = sg.forward_gather_last(idx)
    ref_logits, _ = m(idx)
    assert torch.equal(logits, ref_logits)
    assert torch.equal(last, ref_logits[:, -1, :])
    # the collective itself, through NCCL on device tensors: rows in, the same rows out
    got = gather_batch(ref_logits[:, -1, :].contiguous(), idx.shape[0])
    assert got.is_cuda and torch.equal(got, ref_logits[:, -1, :])
    got_tok = gather_batch(ref_seq, idx.shape[0])
    assert torch.equal(got_tok, ref_seq)
