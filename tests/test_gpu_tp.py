"""Tensor parallelism on 2 GPUs: the Megatron-sharded decode path (NCCL sum
after o and down, vocabulary-sharded lm_head with a max-reduced argmax) must
match the unsharded oracle -- fp16 weights at small, Llama-3-8B and 70B
widths, and 4-bit weights at Llama-3-8B widths, each with both exchanges.
Skipped where fewer than 2 GPUs are visible.  (tp_worker.py takes an
optional B2_TP_CASES filter on the case names for a shorter run.)"""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_tp2_matches_oracle(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "tp.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(HERE, "tp_worker.py"), str(out)]
    env = dict(os.environ)
    env.setdefault("NCCL_SOCKET_IFNAME", "lo")  # one node: bootstrap over loopback
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    verdict = json.loads(out.read_text())
    assert verdict["ok"], verdict
