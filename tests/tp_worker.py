"""One rank of the tensor-parallel parity check (launched by test_gpu_tp.py
under torch.distributed.run; not collected by pytest).

Every rank builds its Megatron shard of the seeded model on its own GPU (NCCL
communicator from a unique id rank 0 shares over the gloo process group),
runs the batched prefill, teacher-forced decode steps and device greedy
generation; rank 0 compares the gathered logits and the greedy ids with the
unsharded oracle (same criteria as test_gpu_model.py) and writes a JSON verdict.
"""
import datetime as dt
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (os.path.join(ROOT, "serving-engine_b200"), os.path.join(ROOT, "oracle"), HERE):
    sys.path.insert(0, p)


def main():
    import torch
    import torch.distributed as dist

    import b2engine as b2
    import oracle as O

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("gloo", timeout=dt.timedelta(seconds=120))
    out_path = sys.argv[1]
    verdict = {"ok": True, "cases": []}
    cases = [
        ("small", O.Config(vocab=1000, hidden=256, inter=704, layers=2, nq=8, nkv=4, head_dim=32, theta=1e4), 12, 8),
        ("llama8b-width", O.Config(vocab=128256, hidden=4096, inter=14336, layers=2, nq=32, nkv=8, head_dim=128,
                                   theta=5e5), 16, 6),
        # Llama-3-70B widths at reduced depth (full depth needs 278 GB of fp32 weights on the host)
        ("llama70b-width", O.Config(vocab=128256, hidden=8192, inter=28672, layers=1, nq=64, nkv=8, head_dim=128,
                                    theta=5e5), 12, 4),
    ]
    cases = [(n, c, s0, nd, x, "fp16") for (n, c, s0, nd) in cases for x in ("nccl", "p2p")
             if c.nkv % world == 0 and c.inter % world == 0 and c.vocab % world == 0]
    # 4-bit weights for the decode GEMVs, sharded (every exchange form of the
    # 4-bit GEMV: consumers of the peer sums, producers that push them)
    c4 = O.Config(vocab=4096, hidden=4096, inter=14336, layers=2, nq=32, nkv=8, head_dim=128, theta=5e5)
    if c4.nkv % world == 0 and (c4.inter // world) % 128 == 0:
        cases += [("llama8b-width-int4", c4, 10, 6, x, "int4") for x in ("nccl", "p2p")]
    only = [t for t in os.environ.get("B2_TP_CASES", "").split(",") if t]  # optional name filter
    if only:
        cases = [c for c in cases if any(t in c[0] for t in only)]
    for name, cfg, S0, n_dec, xch, wfmt in cases:
        obj = [b2.nccl_unique_id() if rank == 0 else None]  # one id per communicator
        dist.broadcast_object_list(obj, src=0)
        m = b2.Model(cfg.vocab, cfg.hidden, cfg.inter, cfg.layers, cfg.nq, cfg.nkv, cfg.head_dim, eps=cfg.eps,
                     theta=cfg.theta, max_batch=1, max_seq=128, tp_rank=rank, tp_size=world, nccl_id=obj[0])
        m.init_random(77, 0.02)
        if wfmt != "fp16":
            m.quantize_weights(wfmt)
        if xch == "p2p":  # partial sums over NVLink peer memory instead of NCCL
            handles = [None] * world
            dist.all_gather_object(handles, m.p2p_handle())
            m.p2p_open(handles)
        rng = np.random.default_rng(5)
        prompt = rng.integers(0, cfg.vocab, S0)
        if wfmt == "fp16":
            lg0 = m.prefill(prompt[None, :])
            gen = m.generate_greedy(n_dec)[:, 0]
            m.reset()
            m.prefill(prompt[None, :], want_logits=False)
            dec = []
            for i in range(3):
                lg, _ = m.decode_step([gen[i]], [S0 + i])
                dec.append(lg[0])
        else:
            # prefill keeps the fp16 weights: every position goes through the
            # quantised decode GEMVs instead (greedy after the prompt)
            m.reset()
            ids = [int(t) for t in prompt]
            rows_q = []
            for pos in range(S0 + n_dec - 1):
                lg, nx = m.decode_step([ids[pos]], [pos], want_logits=True, want_next=True)
                if pos >= S0 - 1:
                    rows_q.append(lg[0])
                    ids.append(int(nx[0]))
            gen = np.array(ids[S0:], np.int64)
            lg0, dec = rows_q[:1], rows_q[1:4]
            lg0 = np.asarray(lg0)
        status = b2.device_status()
        m.close()
        verdict["ok"] &= status == 0
        if rank == 0:
            W = O.seeded_weights(cfg, 77)
            if wfmt == "int4":
                W = O.int4_weights(W)
            ref = O.forward(cfg, W, np.concatenate([prompt, gen[:-1]]).astype(np.int64), logit_row0=S0 - 1)
            rows = [lg0[0]] + dec
            worst_d, worst_cos = 0.0, 1.0
            for i, g in enumerate(rows):
                g = g.astype(np.float64)
                r = ref[i].astype(np.float64)
                worst_d = max(worst_d, float(np.max(np.abs(g - r))))
                worst_cos = min(worst_cos, float(g @ r / (np.linalg.norm(g) * np.linalg.norm(r))))
            greedy_ok = True
            for i, t in enumerate(gen):
                top = int(np.argmax(ref[i]))
                if t != top:
                    s = np.sort(ref[i])[::-1]
                    greedy_ok &= bool(s[0] - s[1] < 0.05)
            ok = worst_d <= 2e-2 and worst_cos >= 0.9999 and greedy_ok
            verdict["ok"] &= ok
            verdict["cases"].append({"name": name, "exchange": xch, "weights": wfmt, "max_abs": worst_d, "cos": worst_cos,
                                     "greedy_ok": greedy_ok, "device_status": status})
    dist.barrier()
    if rank == 0:
        with open(out_path, "w") as f:
            json.dump(verdict, f)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
