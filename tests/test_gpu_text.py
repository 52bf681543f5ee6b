"""Text in, text out on the CUDA path: Model.generate_text with the host
tokenizer (the reference's generate flow, apps/generate.cpp:858-940, for a
Llama-3 vocabulary and a Qwen2 one).

The chat messages go through the vocabulary's template, the ids through the
tcgen05 prefill and the device-resident greedy decode loop; every generated
id must be the oracle's argmax at its position (teacher forced on the
generated sequence), except on a near tie (top-1 / top-2 margin below 0.05),
and the text must be the tokenizer's decode of those ids.  A stop id ends
generation at its first occurrence, whatever the step chunk.
"""
import os

import numpy as np
import pytest

import b2engine as b2
import oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _check_greedy(cfg, w, prompt_ids, new):
    seq = np.array(prompt_ids + new[:-1], np.int64)
    ref = O.forward(cfg, w, seq, logit_row0=len(prompt_ids) - 1)
    for i, t in enumerate(new):
        top = int(np.argmax(ref[i]))
        if t != top:
            srt = np.sort(ref[i])[::-1]
            assert srt[0] - srt[1] < 0.05, f"step {i}: {t} vs oracle {top}"


@pytest.mark.parametrize("kind", ["llama3", "qwen2"])
def test_generate_text_matches_oracle(cuda, kind):
    tok = b2.Tokenizer(os.path.join(GOLDEN, f"tokenizer_{kind}.json"))
    cfg = O.Config(vocab=2624, hidden=512, inter=1024, layers=2, nq=4, nkv=2, head_dim=128, theta=500000.0)
    m = b2.Model(cfg.vocab, cfg.hidden, cfg.inter, cfg.layers, cfg.nq, cfg.nkv, cfg.head_dim, theta=cfg.theta,
                 max_batch=1, max_seq=256)
    m.init_random(11, 0.02)
    w = O.seeded_weights(cfg, 11)
    msgs = [{"role": "system", "content": "Answer briefly."}, {"role": "user", "content": "Wie spät ist es? 12:30"}]
    text, prompt_ids, new = m.generate_text(tok, messages=msgs, max_new_tokens=24, chunk=16)
    assert prompt_ids == tok.encode(tok.apply_chat_template(msgs))
    assert len(new) == 24 or new[-1] in tok.stop_ids
    assert text == tok.decode(new, skip_special=True)
    _check_greedy(cfg, w, prompt_ids, new)

    # a stop id cuts generation at its first occurrence, across chunk edges
    stop = new[9]
    first = new.index(stop)
    tok.stop_ids = [stop]
    m.reset()
    text2, _, new2 = m.generate_text(tok, messages=msgs, max_new_tokens=24, chunk=4)
    assert new2 == new[: first + 1]
    assert text2 == tok.decode(new2, skip_special=True)

    # a plain prompt takes the file's post-processor (Llama-3: BOS first)
    m.reset()
    _, pids, _ = m.generate_text(tok, prompt="Bandwidth-bound decode, 3 steps", max_new_tokens=3)
    assert pids == tok.encode("Bandwidth-bound decode, 3 steps", add_special=True)
    if kind == "llama3":
        assert pids[0] == tok.info.bos_id
    m.close()
