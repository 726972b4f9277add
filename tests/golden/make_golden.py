"""Generates tests/golden/*.npz from the reference's OWN CPU code.

    python tests/golden/make_golden.py

Runs arahe-dev/breadv2's CPU functions compiled from its sources
(oracle/_ref/libbread_ref.so, built by oracle/Makefile where the reference
checkout exists) on seeded inputs and stores inputs + outputs.  The fixtures
pin the oracle restatement (oracle/oracle.c) and the CUDA kernels on machines
without the reference checkout.

Fixtures:
  dequant.npz  Q4_K / Q6_K blocks (baseline, subnormal, zero, large, mixed,
               and the reference's known-answer blocks) with the outputs of
               layer_ops.cu:44/77 (exact fp16 decode) and
               dequant_q4k_cpu.c:90/141 (flush-to-zero decode)
  matvec.npz   cpu_matvec_q4k / cpu_matvec_q6k (layer_ops.cu:133-167)
  route.npz    route_layer arithmetic (one_layer.cu:937-992 loop order with the
               reference's cpu_softmax / cpu_topk / cpu_sigmoid)
  swiglu.npz   cpu_swiglu (layer_ops.cu:214-220)
  moe.npz      the expert block of expert_bench.cu:158-179 plus a shared expert
               (H = I = 256, 4 experts, top-2, 2 tokens)
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from oracle import blocks as B  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def main() -> int:
    oracle.build()
    if not oracle.ref_available():
        print("reference library missing: build it where the reference checkout exists", file=sys.stderr)
        return 1
    rng = np.random.default_rng(20261201)

    # --- dequant
    d = {}
    for qt, gen, name in ((12, B.q4k_blocks, "q4k"), (14, B.q6k_blocks, "q6k")):
        parts = [gen(rng, 24, m) for m in ("baseline", "subnormal", "zero_scale", "large", "mixed")]
        parts.append((B.kat_q4k_block() if qt == 12 else B.kat_q6k_block())[None, :])
        blk = np.concatenate(parts).astype(np.uint8)
        n = blk.shape[0]
        d[f"{name}_blocks"] = blk
        d[f"{name}_exact"] = oracle.ref_dequant(blk.reshape(-1), qt, n, ftz=False)
        d[f"{name}_ftz"] = oracle.ref_dequant(blk.reshape(-1), qt, n, ftz=True)
    np.savez_compressed(os.path.join(OUT, "dequant.npz"), **d)

    # --- matvec
    m = {}
    w4 = B.matrix(12, rng, 64, 2048)
    x4 = rng.standard_normal(2048).astype(np.float32)
    m["q4k_w"], m["q4k_x"], m["q4k_y"] = w4, x4, oracle.ref_matvec(w4, 12, x4, 64, 2048)
    w6 = B.matrix(14, rng, 128, 512)
    x6 = rng.standard_normal(512).astype(np.float32)
    m["q6k_w"], m["q6k_x"], m["q6k_y"] = w6, x6, oracle.ref_matvec(w6, 14, x6, 128, 512)
    np.savez_compressed(os.path.join(OUT, "matvec.npz"), **m)

    # --- routing: T=4, H=512, E=64, top-8, shared gate present
    T, H, E, K = 4, 512, 64, 8
    x = rng.standard_normal((T, H)).astype(np.float32)
    W = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    sg = (rng.standard_normal(H) * 0.02).astype(np.float16).view(np.uint16)
    idx, wt, sgw = oracle.ref_route(x, W, sg, K)
    np.savez_compressed(os.path.join(OUT, "route.npz"), x=x, W_r=W, w_sg=sg, idx=idx, w=wt, sg_weight=sgw, top_k=K)

    # --- swiglu
    g = (rng.standard_normal(512) * 8).astype(np.float32)
    u = (rng.standard_normal(512) * 8).astype(np.float32)
    np.savez_compressed(os.path.join(OUT, "swiglu.npz"), g=g, u=u, out=oracle.ref_swiglu(g, u))

    # --- MoE block: H=256, I=256, E=4, top-2, T=2, shared expert
    T, H, I, E, K = 2, 256, 256, 4, 2
    gate = [B.matrix(12, rng, I, H) for _ in range(E)]
    up = [B.matrix(12, rng, I, H) for _ in range(E)]
    down = [B.matrix(14, rng, H, I) for _ in range(E)]
    sh = (B.matrix(12, rng, I, H), B.matrix(12, rng, I, H), B.matrix(14, rng, H, I))
    x = rng.standard_normal((T, H)).astype(np.float32)
    W = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    sgv = (rng.standard_normal(H) * 0.02).astype(np.float16).view(np.uint16)
    idx, wt, sgw = oracle.ref_route(x, W, sgv, K)
    es = oracle.ExpertSet(gate, up, down, *sh)
    out = oracle.ref_moe_block(es, x, idx, wt, sgw, H, I, n_threads=2)
    np.savez_compressed(os.path.join(OUT, "moe.npz"), gate=np.stack(gate), up=np.stack(up), down=np.stack(down),
                        sh_gate=sh[0], sh_up=sh[1], sh_down=sh[2], x=x, W_r=W, w_sg=sgv, idx=idx, w=wt,
                        sg_weight=sgw, out=out, dims=np.array([T, H, I, E, K]))
    for f in sorted(os.listdir(OUT)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(OUT, f)))
    return 0


if __name__ == "__main__":
    sys.exit(main())
