"""GPU: failure detection without a GPU fault.

The reference exits the process on any CUDA error (bread_utils.h:14-21) and
skips an expert whose weights are not cached (one_layer.cu:1949-1958).  Here
every device-side wait is bounded and bad expert pointers are refused before
any copy is issued; these tests make both happen on purpose:

* a peer that never arrives: an expert-parallel stack of world 2 on ONE GPU
  whose "peer" mailbox is a local buffer nobody writes into, with a short
  peer timeout -- the step must return, set the device error word
  (DEVERR_TIMEOUT) and leave the context usable;
* an expert pointer that is NULL or not 16-byte aligned reaching the kernel
  (the router picks that expert): DEVERR_ROUTE, no copy from it, no fault.
"""
import ctypes

import numpy as np
import pytest
import torch

import breadv2_b200 as bb

pytestmark = pytest.mark.gpu
DEVERR_TIMEOUT, DEVERR_ROUTE = 1, 2


@pytest.mark.parametrize("T", [1, 24])
def test_peer_never_arrives_times_out(cuda, T):
    """T = 1 runs the flagged-word decode kernel (partials polled as tagged
    words), T = 24 the grid-barrier kernel (arrival counters)."""
    assert bb.device_error(clear=True) == 0
    st = bb.ExpertStack(n_layers=3, hidden=1024, inter=256, n_experts=32, top_k=4, max_tokens=24, seed=3, rank=0,
                        world=2)
    own, nbytes = st.mailbox()
    fake_peer = torch.zeros(nbytes // 8 + 32, dtype=torch.int64, device=cuda)  # never written by anyone
    arr = (ctypes.c_void_p * 2)(own, fake_peer.data_ptr())
    bb.check(bb.lib().bread_stack_set_peers(st.handle, arr, 2), "set_peers")
    bb.check(bb.lib().bread_stack_set_peer_timeout(st.handle, ctypes.c_double(0.05)), "set_peer_timeout")
    h = bb.synth_normal(T * 1024, 1.0, 3, 9, device=cuda).view(T, 1024)
    st.step(h)
    torch.cuda.synchronize()  # the launch finishes: every later wait gives up once one has run out
    assert bb.device_error(clear=True) & DEVERR_TIMEOUT
    st.close()
    # the context is still usable: a one-GPU stack steps and is correct afterwards
    one = bb.ExpertStack(n_layers=2, hidden=1024, inter=256, n_experts=32, top_k=4, max_tokens=2, seed=3)
    a = bb.synth_normal(1024, 1.0, 3, 10, device=cuda).view(1, 1024)
    b = a.clone()
    one.step(a)
    one.step(b)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.isfinite(a).all()
    assert bb.device_error(clear=True) == 0
    one.close()


@pytest.mark.parametrize("bad", ["null", "misaligned"])
def test_bad_expert_pointer_sets_route_error(cuda, bad):
    """bread_moe_ffn with expert 3's gate pointer NULL (an expert the caller
    never loaded) or 2 bytes off (not 16-byte aligned), and a router that
    always picks expert 3: the kernel refuses the copy, sets DEVERR_ROUTE and
    returns; a correct call right after gives the right answer."""
    assert bb.device_error(clear=True) == 0
    H, I, E, K, T = 1024, 256, 16, 4, 2
    nb_g, nb_d = I * H // 256, H * I // 256
    gate = [bb.synth_blocks(nb_g, 12, 5, 10 + e, device=cuda) for e in range(E)]
    up = [bb.synth_blocks(nb_g, 12, 5, 100 + e, device=cuda) for e in range(E)]
    down = [bb.synth_blocks(nb_d, 14, 5, 200 + e, device=cuda) for e in range(E)]
    W_r = bb.synth_normal(E * H, 0.02, 5, 300, device=cuda).view(E, H)
    x = bb.synth_normal(T * H, 1.0, 5, 301, device=cuda).view(T, H)
    W_r[3] = x.mean(0) * 10.0  # expert 3 wins every token's routing
    shift = torch.zeros(nb_g * 144 + 16, dtype=torch.uint8, device=cuda)
    ptrs = [t.data_ptr() for t in gate]
    ptrs[3] = 0 if bad == "null" else shift.data_ptr() + 2
    tabs = [bb.pointer_table(ptrs, cuda), bb.pointer_table(up, cuda), bb.pointer_table(down, cuda)]
    out = torch.zeros(T, H, device=cuda)
    idx, _, _ = bb.moe_ffn(*tabs, W_r, None, None, x, out, I, K, want_routing=True)
    torch.cuda.synchronize()
    assert (idx.cpu().numpy() == 3).any(axis=1).all()
    assert bb.device_error(clear=True) & DEVERR_ROUTE
    good = [bb.pointer_table(t, cuda) for t in (gate, up, down)]
    o1 = torch.zeros(T, H, device=cuda)
    o2 = torch.zeros(T, H, device=cuda)
    bb.moe_ffn(*good, W_r, None, None, x, o1, I, K)
    bb.moe_ffn(*good, W_r, None, None, x, o2, I, K)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.isfinite(o1).all()
    assert bb.device_error(clear=True) == 0
