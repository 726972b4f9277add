"""Worker for tests/test_ep_gpu.py: one rank of an expert-parallel stack.
Launched by torch.distributed.run; prints one JSON line on rank 0."""
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import breadv2_b200 as bb  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    import datetime

    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    T = int(os.environ.get("EP_T", "4"))
    cfg = dict(n_layers=int(os.environ.get("EP_LAYERS", "3")), hidden=1024, inter=512, n_experts=32, top_k=4,
               max_tokens=max(8, T, int(os.environ.get("EP_MIX", "0"))), shared_expert=True, norm_eps=1e-6, seed=21)
    st = bb.ExpertStack(**cfg, rank=rank, world=world)
    st.connect_peers(dist)
    h0 = bb.synth_normal(T * 1024, 1.0, 21, 7, device="cuda").view(T, 1024)
    outs = []
    mix = int(os.environ.get("EP_MIX", "0"))  # a step of MIX tokens between the replays
    for _ in range(3):  # replays reuse the mailbox slots
        h = h0.clone()
        st.step(h)
        torch.cuda.synchronize()
        outs.append(h.cpu())
        if mix:
            hm = bb.synth_normal(mix * 1024, 1.0, 21, 8, device="cuda").view(mix, 1024)
            st.step(hm)
            torch.cuda.synchronize()
    err = bb.device_error()
    same_replay = all(torch.equal(outs[0], o) for o in outs[1:])
    gathered = [None] * world
    dist.all_gather_object(gathered, outs[0].numpy().tobytes())
    ranks_equal = all(g == gathered[0] for g in gathered)
    dist.barrier()
    st.close()
    if rank == 0:
        ref = bb.ExpertStack(**cfg, rank=0, world=1)
        h = h0.clone()
        ref.step(h)
        torch.cuda.synchronize()
        rel = float((outs[0] - h.cpu()).norm() / h.cpu().norm())
        ref.close()
        print(json.dumps({"rel_vs_single_gpu": rel, "ranks_bitwise_equal": ranks_equal, "replays_equal": same_replay,
                          "device_error": err}), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
