"""Vocab-sharded LM-head argmax (BatchedDecoder(vocab_shard=...), MQBatchArgs
vocab_shards / keys_out): each of G ranks decoding the same sequences scores a
contiguous 1/G of the vocabulary and one int64 max all-reduce of packed keys
(order(logit) << 32 | ~row, sign bit flipped) gives the global argmax with the
lowest row on ties, like torch.argmax.

CPU: the reduction on two gloo ranks, from keys packed on the host by the same
rule.  GPU: the kernel's shard keys (two shards run one after the other on one
GPU, combined by max) give the same tokens as the unsharded step.
"""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "megaqwen-a10_b200"))

from megaqwen_b200.batch import keys_to_tokens, pack_keys, reduce_shard_keys  # noqa: E402


def _logits():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(5, 1000, generator=g)
    x[1, 700] = x[1, 200] = x[1].max() + 1.0   # tie across the two shards: the lower row wins
    x[2, 10] = x[2, 11] = x[2].max() + 1.0     # tie inside one shard
    x[3] = -x[3].abs() - 1.0                   # all negative
    return x


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    x = _logits()
    n = x.shape[1] // world
    keys = pack_keys(x[:, rank * n:(rank + 1) * n], row0=rank * n)
    reduce_shard_keys(keys, dist)
    out[rank] = keys_to_tokens(keys).tolist()
    dist.destroy_process_group()


def test_shard_reduction_gloo_matches_argmax():
    world, port = 2, _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_rank, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    want = torch.argmax(_logits(), dim=1).tolist()
    assert res[0] == res[1] == want


def test_pack_keys_single_shard():
    x = _logits()
    assert keys_to_tokens(pack_keys(x)).tolist() == torch.argmax(x, dim=1).tolist()


@pytest.mark.gpu
def test_kernel_shard_keys_match_unsharded():
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import megaqwen_b200 as mq
    from test_gpu_parity import build_int8
    L, B, S = 2, 8, 512
    dec = build_int8(mq.make_synthetic_state(seed=9, num_layers=L), L, S)
    pos = [3, 17, 100, 250, 400, 31, 0, 77]
    toks = [5, 77, 1234, 99999, 42, 7, 151935, 1]
    bds = [mq.BatchedDecoder(dec, B, S)] + [mq.BatchedDecoder(dec, B, S, vocab_shard=(r, 2, None, None)) for r in range(2)]
    g = torch.Generator(device="cuda").manual_seed(1)
    kc = torch.randn(bds[0].k_cache.shape, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(bds[0].v_cache.shape, generator=g, device="cuda").to(torch.bfloat16)
    for bd in bds:
        bd.k_cache.copy_(kc)
        bd.v_cache.copy_(vc)
        bd.set_state(toks, pos)
    want = bds[0].step(1).tolist()
    keys = []
    for bd in bds[1:]:
        bd.step(1)
        bd.check_device()
        keys.append(bd.keys.clone())
    assert keys_to_tokens(torch.maximum(keys[0], keys[1])).tolist() == want
