"""Paged KV cache and the model runner over it.

The pool follows the reference's runner contract (docs/runner_interface.md):
per layer, K and V pools [num_blocks][block_size][kv_heads][head_dim],
per-sequence block tables of physical block ids owned by the scheduler,
block size 16.  Checked here:
  * K/V rows written through block tables equal, bit for bit, the rows the
    contiguous cache holds for the same sequence;
  * decode over scattered blocks at mixed lengths (crossing 128-position
    tiles) gives the contiguous model's logits, and the oracle's (max-abs
    2e-2, cosine 0.9999, greedy ids under the near-tie rule);
  * PagedRunner (prefill / decode_step / step) with sequences joining and
    leaving between steps, and the prefix "share" mode (shared blocks are
    not rewritten);
  * batches above the GEMV step's limit (the tensor-core step) on the pool.
"""
import numpy as np
import pytest

import b2engine as b2
import oracle as O
from test_gpu_model import TIE_MARGIN, check_logits

pytestmark = pytest.mark.gpu

CFG = O.Config(vocab=400, hidden=512, inter=768, layers=2, nq=4, nkv=2, head_dim=128, theta=5e5)
BS = 16
SEED = 606


def make(paged_blocks=0, max_batch=4, max_seq=512):
    c = CFG
    m = b2.Model(c.vocab, c.hidden, c.inter, c.layers, c.nq, c.nkv, c.head_dim, eps=c.eps, theta=c.theta,
                 max_batch=max_batch, max_seq=max_seq, kv_blocks=paged_blocks, block_size=BS)
    m.init_random(SEED, 0.02)
    return m


class BlockTable:
    def __init__(self, ids, n):
        self.physical_block_ids = list(ids)
        self.num_tokens = n


class Seq:
    def __init__(self, prompt, blocks):
        self.prompt_ids = np.asarray(prompt, np.int64)
        self.block_table = BlockTable(blocks, len(prompt))
        self.last_token_id = None
        self.generated = []


class Batch:
    def __init__(self, kind, seqs):
        self.batch_type = kind
        self.sequences = seqs


def blocks_for(n):
    return (n + BS - 1) // BS


def test_paged_kv_rows_equal_contiguous_and_logits_match(cuda):
    rng = np.random.default_rng(1)
    lens = [37, 70, 130]
    prompts = [rng.integers(0, CFG.vocab, n) for n in lens]
    conts = rng.integers(0, CFG.vocab, (3, 6))
    nblocks = 64
    perm = rng.permutation(nblocks)
    tables, nxt = [], 0
    for n in lens:  # blocks for prompt + 6 decode steps, scattered
        k = blocks_for(n + 6)
        tables.append(list(perm[nxt:nxt + k]))
        nxt += k
    pm = make(paged_blocks=nblocks, max_batch=4)
    cms = [make(0, max_batch=1) for _ in lens]
    ref_logits = [[] for _ in lens]
    for i, (p, cm) in enumerate(zip(prompts, cms)):
        _, lg = pm.prefill_paged(p, tables[i], want_logits=True)
        ref_logits[i].append(cm.prefill(p[None, :])[0])
        check_logits(lg, ref_logits[i][0], f"prefill {i}")
    # K/V rows of every prefilled position: pool block rows == contiguous cache rows
    nkv, D, L = CFG.nkv, CFG.head_dim, CFG.layers
    pool = pm.read("kv", np.float16, L * 2 * nblocks * BS * nkv * D).reshape(L, 2, nblocks, BS, nkv, D)
    for i, (n, cm) in enumerate(zip(lens, cms)):
        sl, sb, skv, sh, sp = cm.kv_layout()
        cache = cm.read("kv", np.float16, sl * L).reshape(L, 1, 2, nkv, 512, D)
        for pos in range(n):
            blk, slot = tables[i][pos // BS], pos % BS
            got = pool[:, :, blk, slot, :, :]
            want = cache[:, 0, :, :, pos, :]
            assert np.array_equal(got.view(np.uint16), want.view(np.uint16)), (i, pos)
    # decode the three sequences together over the pool, each alone on its contiguous model
    W = O.seeded_weights(CFG, SEED)
    orefs = [O.forward(CFG, W, np.concatenate([prompts[i], conts[i]]), logit_row0=lens[i] - 1) for i in range(3)]
    width = max(len(t) for t in tables)
    bt = np.zeros((3, width), np.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = t
    for s in range(conts.shape[1]):
        seq_lens = [lens[i] + s + 1 for i in range(3)]
        nx, lg = pm.decode_step_paged(conts[:, s], seq_lens, bt, want_logits=True)
        for i in range(3):
            want, _ = cms[i].decode_step([conts[i, s]], [lens[i] + s])
            assert float(np.max(np.abs(lg[i] - want[0]))) <= 2e-3, (s, i)
            check_logits(lg[i], orefs[i][s + 1], f"decode {s} seq {i}")
            row = orefs[i][s + 1]
            if int(nx[i]) != int(np.argmax(row)):
                srt = np.sort(row)[::-1]
                assert srt[0] - srt[1] < TIE_MARGIN, (s, i)
    pm.close()
    for cm in cms:
        cm.close()


def test_runner_continuous_batching(cuda):
    """Sequences join (prefill) and leave between decode steps; every token
    the runner emits is the oracle's argmax given the sequence so far."""
    rng = np.random.default_rng(2)
    nblocks = 96
    free = list(rng.permutation(nblocks))
    m = make(paged_blocks=nblocks, max_batch=4)
    runner = b2.PagedRunner(m)
    W = O.seeded_weights(CFG, SEED)

    def admit(n):
        prompt = rng.integers(0, CFG.vocab, n)
        blocks = [free.pop() for _ in range(blocks_for(n + 12))]  # room for its decode steps
        s = Seq(prompt, blocks)
        s.last_token_id = runner.step(Batch(runner.PREFILL, [s]))[0]
        s.generated.append(s.last_token_id)
        return s

    live = [admit(20), admit(45)]
    finished = []
    for step in range(10):
        if step == 3:
            live.append(admit(129))
        if step == 6:
            finished.append(live.pop(0))
        nxt = runner.step(Batch(runner.DECODE, live))
        for s, t in zip(live, nxt):
            assert s.block_table.num_tokens == len(s.prompt_ids) + len(s.generated)
            s.last_token_id = t
            s.generated.append(t)
            assert abs(s.last_logit_margin) >= 0.0
    for s in finished + live:
        seq = np.concatenate([s.prompt_ids, np.asarray(s.generated[:-1], np.int64)])
        ref = O.forward(CFG, W, seq, logit_row0=len(s.prompt_ids) - 1)
        for i, t in enumerate(s.generated):
            row = ref[i]
            if t != int(np.argmax(row)):
                srt = np.sort(row)[::-1]
                assert srt[0] - srt[1] < TIE_MARGIN, (len(s.prompt_ids), i)
    m.close()


def test_prefix_share_mode_keeps_shared_blocks(cuda):
    """Two sequences share their first two blocks (32 prompt tokens); the
    second prefill recomputes the whole prompt but leaves the shared blocks'
    bytes alone (skip_blocks), and both then decode correctly."""
    rng = np.random.default_rng(3)
    nblocks = 32
    m = make(paged_blocks=nblocks, max_batch=2)
    prefix = rng.integers(0, CFG.vocab, 32)
    a = np.concatenate([prefix, rng.integers(0, CFG.vocab, 10)])
    b = np.concatenate([prefix, rng.integers(0, CFG.vocab, 25)])
    ta = [5, 9, 2, 30]
    tb = [5, 9, 17, 11, 23]
    ta_first, _ = m.prefill_paged(a, ta)
    nkv, D, L = CFG.nkv, CFG.head_dim, CFG.layers
    total = L * 2 * nblocks * BS * nkv * D
    before = m.read("kv", np.float16, total).reshape(L, 2, nblocks, BS * nkv * D).copy()
    m.reset()
    tb_first, _ = m.prefill_paged(b, tb, skip_blocks=2)
    after = m.read("kv", np.float16, total).reshape(L, 2, nblocks, BS * nkv * D)
    for blk in (5, 9, 2, 30):
        assert np.array_equal(before[:, :, blk].view(np.uint16), after[:, :, blk].view(np.uint16)), blk
    W = O.seeded_weights(CFG, SEED)
    ra = O.forward(CFG, W, np.concatenate([a, [ta_first]]), logit_row0=len(a))
    rb = O.forward(CFG, W, np.concatenate([b, [tb_first]]), logit_row0=len(b))
    width = 5
    bt = np.zeros((2, width), np.int32)
    bt[0, :4], bt[1, :5] = ta, tb
    _, lg = m.decode_step_paged([ta_first, tb_first], [len(a) + 1, len(b) + 1], bt, want_logits=True)
    check_logits(lg[0], ra[0], "a")
    check_logits(lg[1], rb[0], "b")
    m.close()


def test_paged_tensor_core_step(cuda):
    """12 sequences (the batched tensor-core step) at mixed lengths over the
    pool against the oracle."""
    rng = np.random.default_rng(4)
    B, nblocks = 12, 160
    m = make(paged_blocks=nblocks, max_batch=B, max_seq=256)
    perm = list(rng.permutation(nblocks))
    lens = [int(x) for x in rng.integers(5, 140, B)]
    prompts = [rng.integers(0, CFG.vocab, n) for n in lens]
    tables, firsts = [], []
    for p in prompts:
        t = [perm.pop() for _ in range(blocks_for(len(p) + 3))]
        tables.append(t)
        firsts.append(m.prefill_paged(p, t)[0])
    width = max(len(t) for t in tables)
    bt = np.zeros((B, width), np.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = t
    W = O.seeded_weights(CFG, SEED)
    toks = np.array(firsts, np.int64)
    hist = [[int(t)] for t in toks]
    for s in range(3):
        nx, lg = m.decode_step_paged(toks, [lens[i] + s + 1 for i in range(B)], bt, want_logits=True)
        for i in range(B):
            seq = np.concatenate([prompts[i], np.asarray(hist[i], np.int64)])
            ref = O.forward(CFG, W, seq, logit_row0=len(seq) - 1)[0]
            check_logits(lg[i], ref, f"step {s} seq {i}")
        toks = nx
        for i in range(B):
            hist[i].append(int(nx[i]))
    m.close()


def test_paged_model_rejects_contiguous_calls(cuda):
    m = make(paged_blocks=8, max_batch=1)
    assert b2.lib().b2_model_decode_step(m.h, None, None, 1, None, None) == -1  # null arguments first
    ids = np.zeros(4, np.int64)
    pos = np.zeros(1, np.int32)
    assert b2.lib().b2_model_decode_step(m.h, ids.ctypes.data, pos.ctypes.data, 1, None, None) == -5
    assert b2.lib().b2_model_prefill(m.h, ids.ctypes.data, 1, 4, None) == -5
    m.close()
