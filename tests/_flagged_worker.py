"""Worker for tests/test_flagged_gpu.py: runs a fixed sequence of stack steps
and MoE block calls on cuda:0 and saves every output to the .npz named by
argv[1].  The parent runs it twice, once with BREAD_NO_FLAGGED=1 (grid-barrier
path) and once without (flagged-word exchange for up to 8 tokens)."""
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import breadv2_b200 as bb  # noqa: E402


def main(path):
    dev = "cuda:0"
    out = {}
    # stack: small shapes (16 experts, fewer router rows than CTAs: presence
    # words) and full layer shapes (257 router rows: one in every CTA), with
    # launches of other sizes in between (a stale word must never be taken)
    st = bb.ExpertStack(n_layers=3, hidden=512, inter=256, n_experts=16, top_k=4, max_tokens=16, seed=11)
    for n, T in enumerate([1, 3, 8, 16, 1, 3]):
        h = bb.synth_normal(T * 512, 1.0, 11, 500 + T, device=dev).view(T, 512)
        st.step(h)
        out[f"small_{n}_T{T}"] = h.cpu().numpy()
    st.close()
    st = bb.ExpertStack(n_layers=4, max_tokens=64, seed=3)
    for n, T in enumerate([1, 4, 64, 1, 8]):
        h = bb.synth_normal(T * 2048, 1.0, 3, 700 + T, device=dev).view(T, 2048)
        st.step(h)
        out[f"cfg_{n}_T{T}"] = h.cpu().numpy()
    st.close()
    # one MoE block through the caller-workspace entry, back to back
    H, I, E, K = 2048, 512, 256, 8
    nb_g, nb_d = I * H // 256, H * I // 256
    gate = [bb.synth_blocks(nb_g, 12, 9, 10 + e, device=dev) for e in range(E)]
    up = [bb.synth_blocks(nb_g, 12, 9, 1000 + e, device=dev) for e in range(E)]
    down = [bb.synth_blocks(nb_d, 14, 9, 2000 + e, device=dev) for e in range(E)]
    shared = (bb.synth_blocks(nb_g, 12, 9, 3000, device=dev), bb.synth_blocks(nb_g, 12, 9, 3001, device=dev),
              bb.synth_blocks(nb_d, 14, 9, 3002, device=dev))
    W_r = bb.synth_normal(E * H, 0.02, 9, 3003, device=dev).view(E, H)
    w_sg = bb.synth_normal(H, 0.02, 9, 3004, half=True, device=dev)
    tabs = [bb.pointer_table(t, dev) for t in (gate, up, down)]
    for n, T in enumerate([1, 2, 8, 1]):
        x = bb.synth_normal(T * H, 1.0, 9, 4000 + T, device=dev).view(T, H)
        y = torch.zeros_like(x)
        idx, _, _ = bb.moe_ffn(*tabs, W_r, w_sg, shared, x, y, I, K, want_routing=True)
        out[f"ffn_{n}_T{T}"] = y.cpu().numpy()
        out[f"ffn_idx_{n}_T{T}"] = idx.cpu().numpy()
    torch.cuda.synchronize()
    out["device_error"] = np.array([bb.device_error()])
    np.savez(path, **out)


if __name__ == "__main__":
    main(sys.argv[1])
