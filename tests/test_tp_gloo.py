"""Megatron tensor parallelism of the decode path, checked on CPU ranks.

Two gloo ranks each build their shard of the seeded model with exactly the
offsets b2_model_init_random uses (q/k/v rows by head, o-proj columns,
gate/up rows, down columns, lm_head rows by vocabulary shard), run the
forward with the two sum all-reduces per layer (after o-proj and after down)
and an all-gather of the vocabulary shards, and must reproduce the unsharded
oracle forward.  The same decomposition is what the device path runs with
NCCL; this test covers its index arithmetic without a GPU.
"""
import os
import socket

import numpy as np
import pytest

import oracle as O

CFG = O.Config(vocab=96, hidden=64, inter=128, layers=2, nq=4, nkv=2, head_dim=16, theta=10000.0, eps=1e-5)
SEED = 31


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _shard_forward(rank, world, ids, all_reduce, all_gather):
    c = CFG
    H, D, I, V = c.hidden, c.head_dim, c.inter, c.vocab
    nq, nkv, Il, Vl = c.nq // world, c.nkv // world, c.inter // world, c.vocab // world
    f = lambda a: a.astype(np.float64)  # noqa: E731
    tid = O.layer_tensor_id
    emb = f(O.init_tensor(SEED, O.T_EMBED, V, H, 0.02))
    lm = f(O.init_tensor(SEED, O.T_LM_HEAD, Vl, H, 0.02, row_offset=rank * Vl))
    S = len(ids)
    cos, sin = O.rope_table(0, S, D, c.theta)

    def rms(x):
        return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + c.eps)

    def rope(x):  # [S, heads, D]
        h = D // 2
        x1, x2 = x[..., :h], x[..., h:]
        cs, sn = cos[:, None, :], sin[:, None, :]
        return np.concatenate([x1 * cs - x2 * sn, x2 * cs + x1 * sn], axis=-1)

    x = emb[ids]
    for l in range(c.layers):
        wq = f(O.init_tensor(SEED, tid(l, "wq"), nq * D, H, 0.02, row_offset=rank * nq * D))
        wk = f(O.init_tensor(SEED, tid(l, "wk"), nkv * D, H, 0.02, row_offset=rank * nkv * D))
        wv = f(O.init_tensor(SEED, tid(l, "wv"), nkv * D, H, 0.02, row_offset=rank * nkv * D))
        wo = f(O.init_tensor(SEED, tid(l, "wo"), H, nq * D, 0.02, col_offset=rank * nq * D, ld_global=c.nq * D))
        wg = f(O.init_tensor(SEED, tid(l, "wg"), Il, H, 0.02, row_offset=rank * Il))
        wu = f(O.init_tensor(SEED, tid(l, "wu"), Il, H, 0.02, row_offset=rank * Il))
        wd = f(O.init_tensor(SEED, tid(l, "wd"), H, Il, 0.02, col_offset=rank * Il, ld_global=I))
        xn = rms(x)
        q = rope((xn @ wq.T).reshape(S, nq, D))
        k = rope((xn @ wk.T).reshape(S, nkv, D))
        v = (xn @ wv.T).reshape(S, nkv, D)
        att = np.zeros((S, nq, D))
        for h in range(nq):
            kv = h // (nq // nkv)
            sc = q[:, h] @ k[:, kv].T / np.sqrt(D)
            sc = np.where(np.tril(np.ones((S, S), bool)), sc, -np.inf)
            p = np.exp(sc - sc.max(axis=1, keepdims=True))
            att[:, h] = (p / p.sum(axis=1, keepdims=True)) @ v[:, kv]
        x = x + all_reduce(att.reshape(S, nq * D) @ wo.T)
        xn = rms(x)
        g, u = xn @ wg.T, xn @ wu.T
        x = x + all_reduce((g / (1 + np.exp(-g)) * u) @ wd.T)
    return all_gather(rms(x) @ lm.T)


def _worker(rank, world, port, ids, expected):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)

    def all_reduce(a):
        t = torch.from_numpy(np.ascontiguousarray(a))
        dist.all_reduce(t)
        return t.numpy()

    def all_gather(a):
        t = torch.from_numpy(np.ascontiguousarray(a))
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        return np.concatenate([p.numpy() for p in parts], axis=-1)

    try:
        got = _shard_forward(rank, world, ids, all_reduce, all_gather)
        assert np.max(np.abs(got - expected)) < 1e-4, np.max(np.abs(got - expected))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tp_decomposition_matches_unsharded_oracle(world):
    import torch.multiprocessing as mp
    ids = np.array([5, 17, 3, 88, 41, 9, 60], np.int64)
    W = O.seeded_weights(CFG, SEED)
    expected = O.forward(CFG, W, ids).astype(np.float64)
    mp.spawn(_worker, args=(world, _free_port(), ids, expected), nprocs=world, join=True)
