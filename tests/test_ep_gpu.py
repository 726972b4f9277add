"""GPU, >= 2 devices: the expert-parallel stack (experts split over ranks,
partials combined through NVLink mailboxes) against the single-GPU stack."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world,T,mix,port", [(2, 1, 0, 29529), (2, 4, 0, 29531), (2, 24, 0, 29533), (2, 1, 24, 29535),
                                              (2, 24, 1, 29537)])
def test_ep_stack_matches_single_gpu(world, T, mix, port):
    """T=1 and T=4: the flagged-word decode kernel on every rank, partials
    exchanged as tagged words over NVLink; T=24: tiled router, shared ring
    arena and grid-distributed top-k, arrival counters, with every rank
    routing all tokens.  mix: a step of that many tokens between the replays
    on the same stack (decode steps exchange tagged words, batched steps count
    arrivals: each must leave the other's state intact)."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", EP_T=str(T), EP_MIX=str(mix))
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(HERE, "_ep_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("{")][-1]
    res = json.loads(line)
    assert res["device_error"] == 0
    assert res["ranks_bitwise_equal"] and res["replays_equal"]
    # same routing as one GPU (a different expert set would differ by O(1));
    # only the fp32 summation order of the partials differs
    assert res["rel_vs_single_gpu"] < 1e-4
