"""Expert parallelism on 2 GPUs through the C ABI (mr_moe_layer_forward_ep):
each rank's outputs equal the one-GPU layer over all ranks' tokens — bit
for bit on the fused paths (down GEMV storing routed partials into the home
rank over NVLink, after an NCCL all-gather of the tokens or a peer
all-to-all dispatch of them), within fp32 summation order on the NCCL path —
and the expert ids are the same. Runs tests/ep_worker.py as two torchrun ranks; skipped with fewer than
two GPUs."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
REL_L2 = 2e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_parallel_two_ranks_match_one_gpu():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), os.path.join(HERE, "ep_worker.py")]
    p = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=400)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    lines = [l for l in p.stdout.splitlines() if l.startswith("EPRESULT ")]
    assert len(lines) == 2, p.stdout[-3000:]
    for line in lines:
        res = json.loads(line[len("EPRESULT "):])
        for name, r in res["results"].items():
            assert r["finite"], (res["rank"], name)
            assert r["ids_equal"], (res["rank"], name)
            assert r["rel_l2"] < r.get("bound", REL_L2), (res["rank"], name, r["rel_l2"])
            if r["fused"]:
                assert r["bit_equal"], (res["rank"], name, r["rel_l2"])
