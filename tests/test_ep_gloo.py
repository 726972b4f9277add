"""CPU, gloo, world size 2: the expert-parallel algorithm of the stack.

* partition: rank r owns routed experts [r*E/W, (r+1)*E/W) and the shared
  expert of layers with l % W == r; the router is replicated, so every rank
  routes identically;
* combine: every rank sums the ranks' partials in rank order.
Each rank computes its partial with the oracle; the combined result must match
the single-process oracle.  Also checks the IPC handle exchange of
ExpertStack.connect_peers with the CUDA calls replaced by fakes."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _layer(rng, H, I, E):
    from oracle import blocks as B

    gate = [B.matrix(12, rng, I, H) for _ in range(E)]
    up = [B.matrix(12, rng, I, H) for _ in range(E)]
    down = [B.matrix(14, rng, H, I) for _ in range(E)]
    sh = (B.matrix(12, rng, I, H), B.matrix(12, rng, I, H), B.matrix(14, rng, H, I))
    W = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    sg = (rng.standard_normal(H) * 0.02).astype(np.float16).view(np.uint16)
    return gate, up, down, sh, W, sg


def _partial(orc, lay, x, rank, world, layer_idx, H, I, E, K):
    gate, up, down, sh, W, sg = lay
    idx, w, sgw, _ = orc.route(x, W, sg, K)  # replicated router
    lo, hi = rank * E // world, (rank + 1) * E // world
    wl = np.where((idx >= lo) & (idx < hi), w, 0.0).astype(np.float32)  # remote experts contribute 0
    own_shared = layer_idx % world == rank
    es = orc.ExpertSet(gate, up, down, *(sh if own_shared else (None, None, None)))
    return orc.moe_f64(es, x, idx, wl, sgw, H, I)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys

    sys.path.insert(0, ROOT)
    import oracle as orc

    dist.init_process_group("gloo", rank=rank, world_size=world)
    H, I, E, K, T, L = 256, 256, 8, 2, 3, 2
    rng = np.random.default_rng(5)
    layers = [_layer(rng, H, I, E) for _ in range(L)]
    h = rng.standard_normal((T, H))
    for l in range(L):
        x = (h / np.sqrt((h * h).mean(axis=1, keepdims=True) + 1e-6)).astype(np.float32)
        part = _partial(orc, layers[l], x, rank, world, l, H, I, E, K)
        parts = [None] * world
        dist.all_gather_object(parts, part)
        h = h + sum(parts[r] for r in range(world))  # rank order
    if rank == 0:
        href = rng  # noqa: F841
        h1 = np.random.default_rng(5)
        layers1 = [_layer(h1, H, I, E) for _ in range(L)]
        hs = h1.standard_normal((T, H))
        for l in range(L):
            x = (hs / np.sqrt((hs * hs).mean(axis=1, keepdims=True) + 1e-6)).astype(np.float32)
            gate, up, down, sh, W, sg = layers1[l]
            idx, w, sgw, _ = orc.route(x, W, sg, K)
            hs = hs + orc.moe_f64(orc.ExpertSet(gate, up, down, *sh), x, idx, w, sgw, H, I)
        q.put(float(np.linalg.norm(h - hs) / np.linalg.norm(hs)))
    dist.barrier()
    dist.destroy_process_group()


def test_ep_partition_and_combine_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rel = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert rel < 1e-12


def _exchange_worker(rank, world, port, q):
    """connect_peers with fake IPC: each rank must pass set_peers the pointers
    ordered by rank, its own mailbox at its own index."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import ctypes
    import sys

    sys.path.insert(0, ROOT)
    import breadv2_b200 as bb

    dist.init_process_group("gloo", rank=rank, world_size=world)
    own = 0x100000 * (rank + 1)

    class FakeLib:
        def bread_ipc_get_handle(self, ptr, buf):
            ctypes.memmove(buf, (b"R%d" % (ptr.value // 0x100000 - 1)).ljust(64, b"\0"), 64)
            return 0

        def bread_ipc_open_handle(self, buf, out):
            r = int(bytes(buf.raw[1:3]).rstrip(b"\0"))
            out._obj.value = 0x900000 + r
            return 0

        def bread_stack_set_peers(self, handle, arr, n):
            q.put((rank, [arr[i] for i in range(n)]))
            return 0

        def bread_ipc_close_handle(self, p):
            return 0

    st = bb.ExpertStack.__new__(bb.ExpertStack)
    st.cfg = bb.StackConfig(1, 256, 256, 8, 2, 1, 1, 1e-6, 1, rank, world)
    st.handle = ctypes.c_void_p(1)
    st._opened = []
    st.mailbox = lambda: (own, 4096)
    real = bb.lib
    bb.lib = lambda: FakeLib()
    try:
        st.connect_peers(dist)
    finally:
        bb.lib = real
        st.handle = None
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_connect_peers_exchange_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        exp = [0x100000 * (r + 1) if j == r else 0x900000 + j for j in range(world)]
        assert got[r] == exp
